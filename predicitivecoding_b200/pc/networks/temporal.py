"""TemporalNetwork: the previous step's hidden states act as temporal priors (Friston 2008).

Reference: PredicitiveCoding/Networks/Temporal/TemporalNetwork.cs:31-112.
"""
from __future__ import annotations

from ..network import Network


class TemporalNetwork:
    def __init__(self, net: Network, temporal_precision: float = 1.0):
        if temporal_precision < 0:
            raise ValueError("temporal_precision must be >= 0.")
        if net.layer_count < 3:
            raise ValueError("TemporalNetwork requires at least 3 layers (input, >=1 hidden, output).")
        self.base = net
        self.temporal_precision = temporal_precision
        self._priors = None

    @property
    def has_prior(self) -> bool:
        return self._priors is not None

    def step(self, x, label, steps: int) -> None:
        self._priors = self.base.learn_temporal(x, label, steps, self._priors, self.temporal_precision)

    def predict(self, x, steps: int) -> int:
        return self.base.predict_temporal(x, steps, self._priors, self.temporal_precision)

    def advance(self, x, label, steps: int) -> int:
        self._priors = self.base.infer_temporal(x, steps, self._priors, self.temporal_precision, True, label)
        return self.base.predict_temporal(x, steps, self._priors, self.temporal_precision)

    def reset(self) -> None:
        self._priors = None
