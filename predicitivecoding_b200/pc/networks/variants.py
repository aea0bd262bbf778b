"""PC architectures that change the relaxation itself: attention-gated errors and 2-hop skips.

Reference: PredicitiveCoding/Networks/Attentive/AttentiveNetwork.cs:48-290 (a learnable
per-unit gate a = sigmoid(s) scales each error before it drives the layer above;
s += eta (|eps| a (1 - a) - lambda s) after learning) and Residual/ResidualNetwork.cs:45-300
(a skip predictor W_skip from layer l+2 adds SkipPrecision * f(W_skip mu + b) to the prediction
of layer l, drives mu_{l+2} with eta * SkipPrecision * W_skip^T (g' * eps_l), and learns with
the same Hebbian rule).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import torch

from ..layer import Layer, activate, derivative, init_weights
from ..network import Network, NetworkConfig


@dataclass
class AttentiveNetworkConfig:
    base_config: NetworkConfig = field(default_factory=NetworkConfig)
    attention_learning_rate: float = 0.01
    attention_regularization: float = 0.1


class AttentiveNetwork(Network):
    def __init__(self, config: AttentiveNetworkConfig, seed: int = 0):
        super().__init__(config.base_config, seed)
        self.att_config = config
        sizes = config.base_config.layer_sizes
        self.att_logits = [torch.zeros(sizes[l]) for l in range(len(sizes) - 1)]

    def _lower_error(self, layers: List[Layer], l: int) -> torch.Tensor:
        return torch.sigmoid(self.att_logits[l - 1]) * layers[l - 1].eps

    def _after_learn(self, layers: List[Layer], lr_scale: float) -> None:
        eta, lam = self.att_config.attention_learning_rate, self.att_config.attention_regularization
        for l, s in enumerate(self.att_logits):
            a = torch.sigmoid(s)
            s += eta * (layers[l].eps.abs() * a * (1 - a) - lam * s)

    def attention_weights(self, layer_index: int) -> torch.Tensor:
        return torch.sigmoid(self.att_logits[layer_index]).clone()

    def mean_attention(self, layer_index: int) -> float:
        return float(self.attention_weights(layer_index).mean())

    def attention_entropy(self, layer_index: int) -> float:
        a = self.attention_weights(layer_index)
        return float(-(a * a.clamp(min=1e-7).log() + (1 - a) * (1 - a).clamp(min=1e-7).log()).sum())


@dataclass
class ResidualNetworkConfig:
    base_config: NetworkConfig = field(default_factory=NetworkConfig)
    skip_precision: float = 0.5
    skip_weight_learning_rate: Optional[float] = None
    skip_activation: Optional[str] = None

    @property
    def effective_skip_lr(self) -> float:
        return self.skip_weight_learning_rate if self.skip_weight_learning_rate is not None else self.base_config.weight_lr

    @property
    def effective_skip_activation(self) -> str:
        return self.skip_activation or self.base_config.activation


class ResidualNetwork(Network):
    def __init__(self, config: ResidualNetworkConfig, seed: int = 0):
        super().__init__(config.base_config, seed)
        self.res_config = config
        sizes = list(config.base_config.layer_sizes)
        gen = torch.Generator().manual_seed(seed + 104729)
        self.skip_w = [init_weights(sizes[t + 2], sizes[t], config.effective_skip_activation, gen)
                       for t in range(len(sizes) - 2)]
        self.skip_b = [torch.zeros(sizes[t]) for t in range(len(sizes) - 2)]
        self._skip_pre: List[torch.Tensor] = []
        self._skip_pred: List[torch.Tensor] = []

    def _after_predictions(self, layers: List[Layer]) -> None:
        act = self.res_config.effective_skip_activation
        self._skip_pre, self._skip_pred = [], []
        for t, (W, b) in enumerate(zip(self.skip_w, self.skip_b)):
            pre = W @ layers[t + 2].mu + b
            pred = activate(pre, act)
            self._skip_pre.append(pre)
            self._skip_pred.append(pred)
            layers[t + 1].pred = layers[t + 1].pred + self.res_config.skip_precision * pred

    def _after_state_updates(self, layers: List[Layer]) -> None:
        act = self.res_config.effective_skip_activation
        eta = self.config.state_lr * self.res_config.skip_precision
        for t, W in enumerate(self.skip_w):
            src = t + 2
            if layers[src].is_clamped:
                continue
            delta = derivative(self._skip_pre[t], self._skip_pred[t], act) * layers[t].eps
            layers[src].mu = layers[src].mu + eta * (W.T @ delta)

    def _after_learn(self, layers: List[Layer], lr_scale: float) -> None:
        act = self.res_config.effective_skip_activation
        eta = self.res_config.effective_skip_lr * lr_scale * self.res_config.skip_precision
        for t in range(len(self.skip_w)):
            src = t + 2
            pre = self.skip_w[t] @ layers[src].mu + self.skip_b[t]
            pred = activate(pre, act)
            delta = derivative(pre, pred, act) * layers[t].eps
            self.skip_w[t] = self.skip_w[t] + eta * torch.outer(delta, layers[src].mu)
            self.skip_b[t] = self.skip_b[t] + eta * delta
