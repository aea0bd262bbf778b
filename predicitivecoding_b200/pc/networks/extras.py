"""Spiking, episodic-memory, multimodal and routed PC networks.

Reference (PredicitiveCoding/Networks/): Spiking/SpikingNetwork.cs:28-170 (leaky
integrate-and-fire units whose input current is the PC drive W^T delta_{l} - eps_l;
firing rates r = rho r + (1 - rho) spike stand in for the value nodes), Memory/MemoryNetwork.cs +
MemoryBank.cs (ring buffer of latent codes, cosine top-k retrieval, softmax(T * sim) weighted
prior on the top layer), MultiModal/MultiModalNetwork.cs:25-190 (one encoder per modality +
associative network on the concatenated latents; cross-modal generation), Routed/RoutedNetwork.cs:30-200
(a PC router network learns to predict the energy-derived gates; top-k experts learn, gated).
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field, replace
from typing import Dict, List, Optional, Sequence

import torch

from ..layer import activate, derivative, init_weights
from ..network import Network, NetworkConfig
from .moe import compute_gates


def _vec(x) -> torch.Tensor:
    return torch.as_tensor(x, dtype=torch.float32).reshape(-1)


def _child(cfg: NetworkConfig, base: Optional[str], name: str) -> NetworkConfig:
    return replace(cfg, path=os.path.join(base, name) if base else None)


# ---------------------------------------------------------------- spiking
@dataclass
class SpikingNetworkConfig:
    layer_sizes: Sequence[int] = (20, 32, 4)
    activation: str = "tanh"
    ticks: int = 32
    dt: float = 1.0
    leak: float = 0.1
    drive_rate: float = 0.2
    threshold: float = 1.0
    rate_decay: float = 0.5
    weight_learning_rate: float = 0.01

    def validate(self) -> None:
        if len(self.layer_sizes) < 2:
            raise ValueError("layer_sizes must have at least 2 elements.")
        if self.ticks < 1 or self.threshold <= 0 or not 0 <= self.rate_decay < 1:
            raise ValueError("invalid spiking dynamics parameters")


class SpikingNetwork:
    def __init__(self, config: SpikingNetworkConfig, seed: int = 0):
        config.validate()
        self.config = config
        self.L = len(config.layer_sizes)
        gen = torch.Generator().manual_seed(seed)
        s = config.layer_sizes
        self.w = [None] + [init_weights(s[l], s[l - 1], config.activation, gen) for l in range(1, self.L)]
        self.b = [None] + [torch.zeros(s[l - 1]) for l in range(1, self.L)]

    @property
    def input_dim(self) -> int:
        return self.config.layer_sizes[0]

    @property
    def output_dim(self) -> int:
        return self.config.layer_sizes[-1]

    def _err(self, r, l):
        pre = self.w[l] @ r[l] + self.b[l]
        pred = activate(pre, self.config.activation)
        err = r[l - 1] - pred
        return err * derivative(pre, pred, self.config.activation), err

    def _settle(self, x, label=None):
        c = self.config
        x = _vec(x)
        if x.numel() != self.input_dim:
            raise ValueError("input has the wrong size")
        V = [torch.zeros(n) for n in c.layer_sizes]
        r = [torch.zeros(n) for n in c.layer_sizes]
        clamp = label is not None
        for _ in range(c.ticks):
            r[0] = x.clone()
            if clamp:
                r[-1] = label.clone()
            deltas, errs = [None] * self.L, [torch.zeros(n) for n in c.layer_sizes]
            for l in range(1, self.L):
                deltas[l], errs[l - 1] = self._err(r, l)
            for l in range(1, self.L):
                if clamp and l == self.L - 1:
                    continue
                drive = self.w[l].T @ deltas[l] - errs[l]
                V[l] = V[l] + c.dt * (-c.leak * V[l] + c.drive_rate * drive)
                spike = (V[l] >= c.threshold).float()
                V[l] = V[l] - spike * c.threshold
                r[l] = c.rate_decay * r[l] + (1 - c.rate_decay) * spike
        r[0] = x.clone()
        if clamp:
            r[-1] = label.clone()
        return r

    def _energy(self, r) -> float:
        return sum(0.5 * float((self._err(r, l)[1] ** 2).sum()) for l in range(1, self.L))

    def infer(self, x) -> torch.Tensor:
        return self._settle(x)[-1]

    def infer_energy(self, x) -> float:
        return self._energy(self._settle(x))

    def learn(self, x, label) -> None:
        label = _vec(label)
        if label.numel() != self.output_dim:
            raise ValueError("label has the wrong size")
        r = self._settle(x, label)
        eta = self.config.weight_learning_rate
        for l in range(1, self.L):
            delta, _ = self._err(r, l)
            self.w[l] = self.w[l] + eta * torch.outer(delta, r[l])
            self.b[l] = self.b[l] + eta * delta

    def predict(self, x) -> int:
        best, arg = float("inf"), 0
        for c in range(self.output_dim):
            oh = torch.zeros(self.output_dim)
            oh[c] = 1.0
            f = self._energy(self._settle(x, oh))
            if f < best:
                best, arg = f, c
        return arg


# ---------------------------------------------------------------- memory
class MemoryBank:
    """Fixed-capacity ring buffer of (key, value) latent codes with cosine top-k lookup."""

    def __init__(self, capacity: int, key_dim: int, value_dim: int):
        if capacity < 1:
            raise ValueError("capacity must be >= 1")
        self.capacity, self.key_dim, self.value_dim = capacity, key_dim, value_dim
        self.keys = torch.zeros(capacity, key_dim)
        self.values = torch.zeros(capacity, value_dim)
        self.head = 0
        self.count = 0

    def write(self, key, value) -> None:
        key, value = _vec(key), _vec(value)
        if key.numel() != self.key_dim or value.numel() != self.value_dim:
            raise ValueError("key/value has the wrong size")
        self.keys[self.head] = key
        self.values[self.head] = value
        self.head = (self.head + 1) % self.capacity
        self.count = min(self.count + 1, self.capacity)

    def query_top_k(self, query, k: int):
        q = _vec(query)
        if q.numel() != self.key_dim:
            raise ValueError("query has the wrong size")
        n = self.count
        if n == 0:
            return []
        K = self.keys[:n]
        den = K.norm(dim=1) * q.norm()
        sim = torch.where(den < 1e-9, torch.zeros_like(den), (K @ q) / den.clamp(min=1e-30))
        order = sorted(range(n), key=lambda i: -float(sim[i]))[: min(k, n)]
        return [(self.values[i].clone(), float(sim[i])) for i in order]


@dataclass
class MemoryNetworkConfig:
    network_config: NetworkConfig = field(default_factory=NetworkConfig)
    memory_capacity: int = 1024
    retrieval_top_k: int = 4
    memory_precision: float = 0.5
    attention_temperature: float = 10.0
    base_path: Optional[str] = None


class MemoryNetwork:
    def __init__(self, config: MemoryNetworkConfig, seed: int = 0):
        self.config = config
        cfg = replace(config.network_config, path=config.base_path)
        self.net = Network(cfg, seed=seed)
        d = cfg.layer_sizes[-1]
        self.memory = MemoryBank(config.memory_capacity, d, d)

    @property
    def memory_count(self) -> int:
        return self.memory.count

    def attend_memory(self, query) -> Optional[torch.Tensor]:
        entries = self.memory.query_top_k(query, self.config.retrieval_top_k)
        if not entries:
            return None
        sims = torch.tensor([s for _, s in entries])
        w = torch.softmax(self.config.attention_temperature * (sims - sims.max()), 0)
        return sum(wi * v for wi, (v, _) in zip(w, entries))

    def _with_prior(self, prior, fn):
        if prior is not None:
            self.net.set_top_layer_prior(prior, self.config.memory_precision)
        try:
            return fn()
        finally:
            self.net.set_top_layer_prior(None, 1.0)

    def _prior(self, x, steps):
        if self.memory.count == 0:
            return None
        return self.attend_memory(self.net.infer_get_top(x, steps))

    def predict(self, x, steps: int) -> int:
        return self._with_prior(self._prior(x, steps), lambda: self.net.predict(x, steps))

    def predict_with_energy(self, x, steps: int):
        return self._with_prior(self._prior(x, steps), lambda: self.net.predict_with_energy(x, steps))

    def learn(self, x, label, steps: int) -> None:
        z = self.net.infer_get_top(x, steps)
        self._with_prior(self.attend_memory(z), lambda: self.net.learn(x, label, steps))
        self.memory.write(z, z)

    def compute_energy(self) -> float:
        return self.net.compute_energy()


# ---------------------------------------------------------------- multimodal
@dataclass
class ModalityConfig:
    name: str = "modality"
    network_config: NetworkConfig = field(default_factory=NetworkConfig)


@dataclass
class MultiModalNetworkConfig:
    modalities: Sequence[ModalityConfig] = ()
    associative_config: NetworkConfig = field(default_factory=NetworkConfig)
    train_associative_generatively: bool = False
    base_path: Optional[str] = None

    def validate(self) -> None:
        if len(self.modalities) < 2:
            raise ValueError("MultiModalNetwork requires at least 2 modalities.")
        total = sum(m.network_config.layer_sizes[-1] for m in self.modalities)
        if self.associative_config.layer_sizes[0] != total:
            raise ValueError("associative input size must equal the sum of modality latent sizes")


class MultiModalNetwork:
    def __init__(self, config: MultiModalNetworkConfig, seed: int = 0):
        config.validate()
        self.config = config
        self.modalities = [Network(_child(m.network_config, config.base_path, f"modality_{m.name}"),
                                   seed=seed * 13 + i) for i, m in enumerate(config.modalities)]
        self.associative = Network(_child(config.associative_config, config.base_path, "associative"),
                                   seed=seed * 13 + 997)
        self.latent_dims = [m.network_config.layer_sizes[-1] for m in config.modalities]
        self.offsets = [sum(self.latent_dims[:i]) for i in range(len(self.latent_dims))]

    @property
    def modality_count(self) -> int:
        return len(self.modalities)

    def modality_name(self, i: int) -> str:
        return self.config.modalities[i].name

    def encode_all(self, inputs: Dict[int, object], steps: int) -> torch.Tensor:
        return torch.cat([self.modalities[i].infer_get_top(inputs[i], steps) if i in inputs
                          else torch.zeros(d) for i, d in enumerate(self.latent_dims)])

    def learn(self, inputs: Dict[int, object], label, steps: int) -> None:
        for i, x in inputs.items():
            self.modalities[i].learn_unsupervised(x, steps)
        z = self.encode_all(inputs, steps)
        self.associative.learn(z, label, steps)
        if self.config.train_associative_generatively:
            self.associative.learn_unsupervised(z, steps)

    def predict(self, inputs: Dict[int, object], steps: int) -> int:
        return self.associative.predict(self.encode_all(inputs, steps), steps)

    def predict_with_energy(self, inputs: Dict[int, object], steps: int):
        return self.associative.predict_with_energy(self.encode_all(inputs, steps), steps)

    def cross_modal_generate(self, src: int, x, dst: int, steps: int) -> torch.Tensor:
        if not self.config.train_associative_generatively:
            raise RuntimeError("cross_modal_generate requires train_associative_generatively = True.")
        z = self.encode_all({src: x}, steps)
        full = self.associative.generate(self.associative.infer_get_top(z, steps), steps)
        o, d = self.offsets[dst], self.latent_dims[dst]
        return self.modalities[dst].generate(full[o:o + d], steps)


# ---------------------------------------------------------------- routed
@dataclass
class RoutedNetworkConfig:
    expert_config: NetworkConfig = field(default_factory=NetworkConfig)
    router_config: NetworkConfig = field(default_factory=NetworkConfig)
    expert_count: int = 4
    top_k: int = 2
    gating_temperature: float = 1.0
    pe_mix_alpha: float = 0.5
    min_gate_weight: float = 0.01
    base_path: Optional[str] = None

    def validate(self) -> None:
        if self.expert_count < 2:
            raise ValueError("expert_count must be >= 2.")
        if not 1 <= self.top_k <= self.expert_count:
            raise ValueError("top_k must be in [1, expert_count].")
        if self.router_config.layer_sizes[-1] != self.expert_count:
            raise ValueError("router top layer must have expert_count units")
        if self.router_config.layer_sizes[0] != self.expert_config.layer_sizes[0]:
            raise ValueError("router and experts must share the input size")


@dataclass
class RoutedPrediction:
    predicted_class: int
    winning_expert: int
    active_experts: List[int]
    expert_classes: List[int]
    expert_energies: List[float]
    router_gates: List[float]


def _top_k(g: Sequence[float], k: int) -> List[int]:
    return sorted(range(len(g)), key=lambda i: (-g[i], i))[:k]


class RoutedNetwork:
    def __init__(self, config: RoutedNetworkConfig, seed: int = 0):
        config.validate()
        self.config = config
        self.experts = [Network(_child(config.expert_config, config.base_path, f"expert_{i}"), seed=seed * 7 + i)
                        for i in range(config.expert_count)]
        self.router = Network(_child(config.router_config, config.base_path, "router"), seed=seed * 7 + 1001)
        n = config.expert_count
        self.last_gate_weights = [0.0] * n
        self.last_expert_energies = [0.0] * n
        self.last_router_weights = [0.0] * n

    def _router_gates(self, x, steps):
        return torch.softmax(self.router.infer_get_top(x, steps) / self.config.gating_temperature, 0).tolist()

    def learn(self, x, label, steps: int) -> None:
        c = self.config
        self.last_expert_energies = [e.infer_energy(x, label, steps) for e in self.experts]
        pe = compute_gates(self.last_expert_energies, c.gating_temperature, c.min_gate_weight)
        self.last_router_weights = self._router_gates(x, steps)
        a = c.pe_mix_alpha
        self.last_gate_weights = [(1 - a) * r + a * g for r, g in zip(self.last_router_weights, pe)]
        self.router.learn(x, torch.tensor(self.last_gate_weights), steps)
        active = set(_top_k(self.last_gate_weights, c.top_k))
        for i, e in enumerate(self.experts):
            e.learn_gated(x, label, steps, self.last_gate_weights[i] if i in active else 0.0)

    def predict_detailed(self, x, steps: int) -> RoutedPrediction:
        gates = self._router_gates(x, steps)
        active = _top_k(gates, self.config.top_k)
        n = len(self.experts)
        cls, en = [0] * n, [0.0] * n
        best, bc, win = float("inf"), 0, active[0]
        for i in active:
            cls[i], en[i] = self.experts[i].predict_with_energy(x, steps)
            if en[i] < best:
                best, bc, win = en[i], cls[i], i
        return RoutedPrediction(bc, win, active, cls, en, gates)

    def predict(self, x, steps: int) -> int:
        return self.predict_detailed(x, steps).predicted_class

    def average_weight_norm(self) -> float:
        return sum(e.average_weight_norm() for e in self.experts) / len(self.experts)
