"""Bayesian-model-averaging ensemble of PC networks.

Reference: PredicitiveCoding/Networks/Ensemble/EnsembleNetwork.cs:40-357.  Every member learns
each sample; prediction averages per-member Boltzmann class probabilities softmax(-beta F_c)
(ProbabilityAveraging) or the raw class energies (EnergyAveraging).
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass, field, replace
from typing import List, Optional, Sequence

import torch

from ..network import Network, NetworkConfig


@dataclass
class EnsembleConfig:
    member_configs: Sequence[NetworkConfig] = field(default_factory=lambda: [NetworkConfig(), NetworkConfig()])
    base_path: Optional[str] = None
    prediction_mode: str = "probability_averaging"   # or "energy_averaging"
    softmax_temperature: float = 1.0

    def validate(self) -> None:
        if len(self.member_configs) < 2:
            raise ValueError("An ensemble needs at least 2 members.")
        tops = {c.layer_sizes[-1] for c in self.member_configs}
        ins = {c.layer_sizes[0] for c in self.member_configs}
        if len(tops) != 1 or len(ins) != 1:
            raise ValueError("All members must share input and output sizes.")
        if self.prediction_mode not in ("probability_averaging", "energy_averaging"):
            raise ValueError("unknown prediction mode")
        if self.softmax_temperature <= 0:
            raise ValueError("SoftmaxTemperature must be > 0.")


@dataclass
class EnsemblePrediction:
    predicted_class: int
    member_predictions: List[int]
    member_energies: List[List[float]]
    aggregated_probabilities: Optional[List[float]]
    aggregated_energies: Optional[List[float]]


class EnsembleNetwork:
    def __init__(self, config: EnsembleConfig, seed: int = 0):
        config.validate()
        self.config = config
        self.members = [Network(replace(c, path=None if config.base_path is None else
                                        os.path.join(config.base_path, f"member_{i}")), seed=seed * 7919 + i)
                        for i, c in enumerate(config.member_configs)]

    def learn(self, x, label, steps: int) -> None:
        for m in self.members:
            m.learn(x, label, steps)

    @staticmethod
    def _avg_probs(energies: List[List[float]], beta: float) -> List[float]:
        c = len(energies[0])
        avg = [0.0] * c
        for en in energies:
            v = [-beta * e for e in en]
            mx = max(v)
            p = [math.exp(x - mx) for x in v]
            s = sum(p)
            for k in range(c):
                avg[k] += p[k] / s
        return [a / len(energies) for a in avg]

    def predict_detailed(self, x, steps: int) -> EnsemblePrediction:
        en = [m.class_energies(x, steps) for m in self.members]
        preds = [min(range(len(e)), key=lambda k: e[k]) for e in en]
        if self.config.prediction_mode == "probability_averaging":
            probs = self._avg_probs(en, self.config.softmax_temperature)
            return EnsemblePrediction(max(range(len(probs)), key=lambda k: probs[k]), preds, en, probs, None)
        avg = [sum(e[k] for e in en) / len(en) for k in range(len(en[0]))]
        return EnsemblePrediction(min(range(len(avg)), key=lambda k: avg[k]), preds, en, None, avg)

    def predict(self, x, steps: int) -> int:
        return self.predict_detailed(x, steps).predicted_class

    def average_weight_norm(self) -> float:
        return sum(m.average_weight_norm() for m in self.members) / len(self.members)
