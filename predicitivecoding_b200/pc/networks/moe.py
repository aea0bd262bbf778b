"""Mixtures of PC experts gated by free energy: flat, hierarchical (two-level) and temporal.

Reference: PredicitiveCoding/Networks/MoE/MixtureOfExperts.cs:28-225 (gates g = softmax(-beta F_i)
with an optional floor, experts learn with lr scaled by their gate, prediction = the class of the
lowest-energy expert), HierarchicalMixtureOfExperts.cs:27-160, TemporalMixtureOfExperts.cs:36-200.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass, field, replace
from typing import List, Optional, Sequence

import torch

from ..network import Network, NetworkConfig


def compute_gates(energies: Sequence[float], temperature: float, min_gate: float = 0.0) -> List[float]:
    """g_i = softmax(-temperature * F_i); with min_gate > 0 the gates are floored and renormalised."""
    v = [-temperature * e for e in energies]
    mx = max(v)
    g = [math.exp(x - mx) for x in v]
    s = sum(g)
    g = [x / s for x in g]
    if min_gate > 0:
        g = [max(min_gate, x) for x in g]
        s = sum(g)
        g = [x / s for x in g]
    return g


def _sub(base: Optional[NetworkConfig], path: Optional[str], name: str) -> NetworkConfig:
    cfg = base or NetworkConfig()
    return replace(cfg, path=None if path is None else os.path.join(path, name))


@dataclass
class MixtureOfExpertsConfig:
    base_path: Optional[str] = None
    expert_count: int = 3
    expert_config: NetworkConfig = field(default_factory=NetworkConfig)
    gating_temperature: float = 1.0
    min_gate_weight: float = 0.0

    def validate(self) -> None:
        if self.expert_count < 2:
            raise ValueError("ExpertCount must be >= 2.")
        if self.gating_temperature <= 0:
            raise ValueError("GatingTemperature must be > 0.")
        if self.min_gate_weight < 0:
            raise ValueError("MinGateWeight must be >= 0.")
        if self.min_gate_weight >= 1.0 / self.expert_count:
            raise ValueError("MinGateWeight must be < 1/ExpertCount.")


@dataclass
class MoEPrediction:
    predicted_class: int
    winning_expert: int
    expert_classes: List[int]
    expert_energies: List[float]


class MixtureOfExperts:
    def __init__(self, config: MixtureOfExpertsConfig, seed: int = 0):
        config.validate()
        self.config = config
        gen = torch.Generator().manual_seed(seed)
        self.experts = [Network(_sub(config.expert_config, config.base_path, f"expert_{i}"),
                                seed=int(torch.randint(0, 2 ** 31 - 1, (1,), generator=gen)))
                        for i in range(config.expert_count)]
        self.last_gates = [0.0] * config.expert_count
        self.last_energies = [0.0] * config.expert_count

    @property
    def expert_count(self) -> int:
        return len(self.experts)

    def learn(self, x, label, steps: int) -> None:
        self.last_energies = [e.infer_energy(x, label, steps) for e in self.experts]
        self.last_gates = compute_gates(self.last_energies, self.config.gating_temperature, self.config.min_gate_weight)
        for e, g in zip(self.experts, self.last_gates):
            e.learn_gated(x, label, steps, g)

    def predict_detailed(self, x, steps: int) -> MoEPrediction:
        res = [e.predict_with_energy(x, steps) for e in self.experts]
        win = min(range(len(res)), key=lambda i: res[i][1])
        return MoEPrediction(res[win][0], win, [r[0] for r in res], [r[1] for r in res])

    def predict(self, x, steps: int) -> int:
        return self.predict_detailed(x, steps).predicted_class

    def average_weight_norm(self) -> float:
        return sum(e.average_weight_norm() for e in self.experts) / len(self.experts)

    def expert_weight_norms(self) -> List[float]:
        return [e.average_weight_norm() for e in self.experts]

    def flush_all(self) -> None:
        for e in self.experts:
            e.flush_store()


@dataclass
class HierarchicalMoEConfig:
    base_path: Optional[str] = None
    group_count: int = 2
    experts_per_group: int = 2
    expert_config: NetworkConfig = field(default_factory=NetworkConfig)
    group_gating_temperature: float = 1.0
    expert_gating_temperature: float = 1.0
    min_gate_weight: float = 0.0

    def validate(self) -> None:
        if self.group_count < 2 or self.experts_per_group < 2:
            raise ValueError("GroupCount and ExpertsPerGroup must be >= 2.")
        if self.group_gating_temperature <= 0 or self.expert_gating_temperature <= 0:
            raise ValueError("Gating temperatures must be > 0.")
        if not (0 <= self.min_gate_weight < 1.0 / self.experts_per_group):
            raise ValueError("MinGateWeight must be in [0, 1/ExpertsPerGroup).")


class HierarchicalMixtureOfExperts:
    """Group gate x within-group gate; expert responsibility = product (HierarchicalMixtureOfExperts.cs)."""

    def __init__(self, config: HierarchicalMoEConfig, seed: int = 0):
        config.validate()
        self.config = config
        gen = torch.Generator().manual_seed(seed)
        self.groups = [[Network(_sub(config.expert_config, config.base_path, os.path.join(f"group_{g}", f"expert_{e}")),
                                seed=int(torch.randint(0, 2 ** 31 - 1, (1,), generator=gen)))
                        for e in range(config.experts_per_group)] for g in range(config.group_count)]
        self.last_group_gates = [0.0] * config.group_count
        self.last_responsibilities = [[0.0] * config.experts_per_group for _ in range(config.group_count)]

    def learn(self, x, label, steps: int) -> None:
        c = self.config
        energies = [[e.infer_energy(x, label, steps) for e in grp] for grp in self.groups]
        group_energy = []
        for g, en in enumerate(energies):
            r = compute_gates(en, c.expert_gating_temperature, c.min_gate_weight)
            self.last_responsibilities[g] = r
            group_energy.append(sum(ri * ei for ri, ei in zip(r, en)))
        self.last_group_gates = compute_gates(group_energy, c.group_gating_temperature, 0.0)
        for g, grp in enumerate(self.groups):
            for e, net in enumerate(grp):
                r = self.last_group_gates[g] * self.last_responsibilities[g][e]
                self.last_responsibilities[g][e] = r
                net.learn_gated(x, label, steps, r)

    def predict(self, x, steps: int) -> int:
        best_e, best_c = float("inf"), 0
        for grp in self.groups:
            for net in grp:
                c, e = net.predict_with_energy(x, steps)
                if e < best_e:
                    best_e, best_c = e, c
        return best_c


@dataclass
class TemporalMoEConfig:
    base_path: Optional[str] = None
    expert_count: int = 3
    expert_config: NetworkConfig = field(default_factory=NetworkConfig)
    gating_temperature: float = 1.0
    min_gate_weight: float = 0.0
    expert_temporal_precisions: Optional[Sequence[float]] = None
    default_temporal_precision: float = 1.0

    def precision_for(self, i: int) -> float:
        return (self.expert_temporal_precisions[i] if self.expert_temporal_precisions is not None
                else self.default_temporal_precision)

    def validate(self) -> None:
        MixtureOfExpertsConfig(None, self.expert_count, self.expert_config, self.gating_temperature,
                               self.min_gate_weight).validate()
        if self.expert_temporal_precisions is not None:
            if len(self.expert_temporal_precisions) != self.expert_count:
                raise ValueError("ExpertTemporalPrecisions length must equal ExpertCount.")
            if any(p < 0 for p in self.expert_temporal_precisions):
                raise ValueError("All ExpertTemporalPrecisions must be >= 0.")


class TemporalMixtureOfExperts:
    """Temporal experts with their own continuity precisions (TemporalMixtureOfExperts.cs)."""

    def __init__(self, config: TemporalMoEConfig, seed: int = 0):
        config.validate()
        self.config = config
        gen = torch.Generator().manual_seed(seed)
        self.experts = [Network(_sub(config.expert_config, config.base_path, f"expert_{i}"),
                                seed=int(torch.randint(0, 2 ** 31 - 1, (1,), generator=gen)))
                        for i in range(config.expert_count)]
        self.precisions = [config.precision_for(i) for i in range(config.expert_count)]
        self.priors = [None] * config.expert_count
        self.last_gates = [0.0] * config.expert_count
        self.last_energies = [0.0] * config.expert_count

    def step(self, x, label, steps: int) -> None:
        self.last_energies = [e.infer_energy_temporal(x, label, steps, self.priors[i], self.precisions[i])
                              for i, e in enumerate(self.experts)]
        self.last_gates = compute_gates(self.last_energies, self.config.gating_temperature, self.config.min_gate_weight)
        for i, e in enumerate(self.experts):
            self.priors[i], _ = e.learn_temporal_gated(x, label, steps, self.priors[i], self.precisions[i],
                                                       self.last_gates[i])

    def predict_detailed(self, x, steps: int) -> MoEPrediction:
        res = [e.predict_with_energy_temporal(x, steps, self.priors[i], self.precisions[i])
               for i, e in enumerate(self.experts)]
        win = min(range(len(res)), key=lambda i: res[i][1])
        return MoEPrediction(res[win][0], win, [r[0] for r in res], [r[1] for r in res])

    def predict(self, x, steps: int) -> int:
        return self.predict_detailed(x, steps).predicted_class

    def advance(self, x, label, steps: int) -> int:
        for i, e in enumerate(self.experts):
            self.priors[i] = e.infer_temporal(x, steps, self.priors[i], self.precisions[i], True, label)
        return self.predict(x, steps)

    def reset(self) -> None:
        self.priors = [None] * len(self.experts)

    def expert_has_prior(self, i: int) -> bool:
        return self.priors[i] is not None
