"""PC architectures composed from whole networks.

Reference (PredicitiveCoding/Networks/): Hierarchical/HierarchicalNetwork.cs:30-208 (stacked
generative PCNs trained greedily, encode bottom-up / decode top-down), Active/ActiveNetwork.cs:28-245
(world model on [observation | one-hot action] -> next observation; action = argmin of the
expected free energy G = GoalPrecision * 1/2||pred - goal||^2 - ExplorationWeight * 1/2||pred - obs||^2),
DeepRecurrent/DeepRecurrentNetwork.cs:29-209 (cascade of temporal stages), Gated/GatedStateNetwork.cs:27-214
(working memory m updated by an LSTM-like gate g = sigmoid(slope (|z - m| - bias)), used as the top
prior), Hopfield/HopfieldNetwork.cs + HopfieldMemory.cs (modern Hopfield retrieval
xi <- softmax(beta X xi) X in the latent space), Graph/GraphPredictiveNetwork.cs:24-224 (one shared
edge predictor, message passing by blending neighbour predictions), Generative/GenerativeNetwork.cs:25-168
(encode/decode/sample with a Gaussian top prior).
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field, replace
from typing import Callable, List, Optional, Sequence

import torch

from ..network import Network, NetworkConfig


def _child(cfg: NetworkConfig, base: Optional[str], name: Optional[str]) -> NetworkConfig:
    if base is None:
        return replace(cfg, path=None)
    return replace(cfg, path=os.path.join(base, name) if name else base)


# ---------------------------------------------------------------- hierarchical
@dataclass
class HierarchicalNetworkConfig:
    modules: Sequence[NetworkConfig] = ()
    base_path: Optional[str] = None

    def validate(self) -> None:
        if len(self.modules) < 1:
            raise ValueError("At least one module is required.")
        for a, b in zip(self.modules, self.modules[1:]):
            if a.layer_sizes[-1] != b.layer_sizes[0]:
                raise ValueError("Each module's top size must equal the next module's input size.")


class HierarchicalNetwork:
    def __init__(self, config: HierarchicalNetworkConfig, seed: int = 0):
        config.validate()
        self.config = config
        self.modules = [Network(_child(c, config.base_path, f"module_{k}"), seed=seed * 31 + k)
                        for k, c in enumerate(config.modules)]

    def encode(self, x, steps: int) -> torch.Tensor:
        for m in self.modules:
            x = m.infer_get_top(x, steps)
        return x

    def encode_all(self, x, steps: int) -> List[torch.Tensor]:
        out = []
        for m in self.modules:
            x = m.infer_get_top(x, steps)
            out.append(x)
        return out

    def decode(self, z, steps: int) -> torch.Tensor:
        for m in reversed(self.modules):
            z = m.generate(z, steps)
        return z

    def reconstruct(self, x, steps: int) -> torch.Tensor:
        return self.decode(self.encode(x, steps), steps)

    def reconstruction_error(self, x, steps: int) -> float:
        x = torch.as_tensor(x, dtype=torch.float32).reshape(-1)
        return 0.5 * float(((x - self.reconstruct(x, steps)) ** 2).sum())

    def learn(self, x, steps: int) -> None:
        for m in self.modules:
            m.learn_unsupervised(x, steps)
            x = m.infer_get_top(x, steps)

    def module_energy(self, k: int) -> float:
        return self.modules[k].compute_energy()


# ---------------------------------------------------------------- active inference
@dataclass
class ActiveNetworkConfig:
    observation_dim: int = 4
    action_count: int = 2
    world_model_config: Optional[NetworkConfig] = None
    goal_precision: float = 1.0
    exploration_weight: float = 0.0
    base_path: Optional[str] = None

    def validate(self) -> None:
        if self.observation_dim < 1 or self.action_count < 1:
            raise ValueError("observation_dim and action_count must be >= 1.")
        wm = self.world_model_config
        if wm is not None and (wm.layer_sizes[0] != self.observation_dim + self.action_count
                               or wm.layer_sizes[-1] != self.observation_dim):
            raise ValueError("World model must map [obs | one-hot action] -> next obs.")


class ActiveNetwork:
    def __init__(self, config: ActiveNetworkConfig, seed: int = 0):
        config.validate()
        self.config = config
        wm = config.world_model_config or NetworkConfig(
            layer_sizes=(config.observation_dim + config.action_count, 32, config.observation_dim))
        self.world = Network(_child(wm, config.base_path, None), seed=seed)

    def _input(self, obs, action: int) -> torch.Tensor:
        obs = torch.as_tensor(obs, dtype=torch.float32).reshape(-1)
        if obs.numel() != self.config.observation_dim:
            raise ValueError("observation has the wrong size")
        if not 0 <= action < self.config.action_count:
            raise ValueError("action out of range")
        a = torch.zeros(self.config.action_count)
        a[action] = 1.0
        return torch.cat([obs, a])

    def predict_next(self, obs, action: int, steps: int) -> torch.Tensor:
        return self.world.infer_get_top(self._input(obs, action), steps)

    def select_action(self, obs, goal, steps: int):
        goal = torch.as_tensor(goal, dtype=torch.float32).reshape(-1)
        obs = torch.as_tensor(obs, dtype=torch.float32).reshape(-1)
        scores = []
        for a in range(self.config.action_count):
            p = self.predict_next(obs, a, steps)
            prag = 0.5 * float(((p - goal) ** 2).sum())
            epi = 0.5 * float(((p - obs) ** 2).sum()) if self.config.exploration_weight > 0 else 0.0
            scores.append(self.config.goal_precision * prag - self.config.exploration_weight * epi)
        return min(range(len(scores)), key=lambda i: scores[i]), scores

    def act(self, obs, goal, steps: int) -> int:
        return self.select_action(obs, goal, steps)[0]

    def observe(self, obs, action: int, next_obs, steps: int) -> None:
        self.world.learn(self._input(obs, action), next_obs, steps)

    def step(self, obs, goal, environment: Callable, steps: int):
        a = self.act(obs, goal, steps)
        nxt = environment(obs, a)
        self.observe(obs, a, nxt, steps)
        return a, nxt


# ---------------------------------------------------------------- deep recurrent
@dataclass
class DeepRecurrentNetworkConfig:
    stages: Sequence[NetworkConfig] = ()
    temporal_precision: Sequence[float] = (1.0,)
    base_path: Optional[str] = None

    def precision_for(self, k: int) -> float:
        return self.temporal_precision[k] if k < len(self.temporal_precision) else self.temporal_precision[-1]

    def validate(self) -> None:
        if not self.stages:
            raise ValueError("At least one stage is required.")
        for s in self.stages:
            if len(s.layer_sizes) < 3:
                raise ValueError("Each stage needs >= 3 layers (temporal priors live on hidden layers).")


class DeepRecurrentNetwork:
    def __init__(self, config: DeepRecurrentNetworkConfig, seed: int = 0):
        config.validate()
        self.config = config
        self.stages = [Network(_child(c, config.base_path, f"stage_{k}"), seed=seed * 17 + k)
                       for k, c in enumerate(config.stages)]
        self.priors = [None] * len(self.stages)

    @property
    def has_context(self) -> bool:
        return self.priors[0] is not None

    def step(self, x, steps: int) -> torch.Tensor:
        for k, s in enumerate(self.stages):
            x, self.priors[k] = s.learn_unsupervised_temporal(x, steps, self.priors[k], self.config.precision_for(k))
        return x

    def encode(self, x, steps: int) -> torch.Tensor:
        for k, s in enumerate(self.stages):
            x, self.priors[k] = s.infer_get_top_temporal(x, steps, self.priors[k], self.config.precision_for(k))
        return x

    def reset(self) -> None:
        self.priors = [None] * len(self.stages)


# ---------------------------------------------------------------- gated working memory
@dataclass
class GatedStateNetworkConfig:
    network_config: NetworkConfig = field(default_factory=NetworkConfig)
    gate_slope: float = 4.0
    gate_bias: float = 0.5
    working_memory_precision: float = 1.0
    base_path: Optional[str] = None

    def validate(self) -> None:
        if self.gate_slope <= 0 or self.working_memory_precision <= 0:
            raise ValueError("gate_slope and working_memory_precision must be > 0.")


class GatedStateNetwork:
    def __init__(self, config: GatedStateNetworkConfig, seed: int = 0):
        config.validate()
        self.config = config
        self.net = Network(_child(config.network_config, config.base_path, None), seed=seed)
        self.memory: Optional[torch.Tensor] = None

    def _update(self, z: torch.Tensor) -> None:
        if self.memory is None:
            self.memory = z.clone()
            return
        g = torch.sigmoid(self.config.gate_slope * ((z - self.memory).abs() - self.config.gate_bias))
        self.memory = (1 - g) * self.memory + g * z

    def _apply(self) -> None:
        if self.memory is not None:
            self.net.set_top_layer_prior(self.memory, self.config.working_memory_precision)

    def step(self, x, steps: int) -> torch.Tensor:
        self._update(self.net.infer_get_top(x, steps))
        self._apply()
        return self.memory.clone()

    def predict(self, x, steps: int) -> int:
        self._apply()
        return self.net.predict(x, steps)

    def learn(self, x, label, steps: int) -> None:
        self._update(self.net.infer_get_top(x, steps))
        self._apply()
        self.net.learn(x, label, steps)

    def reset(self) -> None:
        self.memory = None
        self.net.set_top_layer_prior(None, 1.0)


# ---------------------------------------------------------------- Hopfield
class HopfieldMemory:
    def __init__(self, dim: int):
        if dim < 1:
            raise ValueError("dim must be >= 1.")
        self.dim = dim
        self.patterns: List[torch.Tensor] = []

    @property
    def count(self) -> int:
        return len(self.patterns)

    def store(self, p) -> None:
        p = torch.as_tensor(p, dtype=torch.float32).reshape(-1)
        if p.numel() != self.dim:
            raise ValueError("pattern has the wrong size")
        self.patterns.append(p.clone())

    def clear(self) -> None:
        self.patterns.clear()

    def retrieve(self, q, beta: float, iterations: int) -> torch.Tensor:
        xi = torch.as_tensor(q, dtype=torch.float32).reshape(-1).clone()
        if not self.patterns:
            return xi
        X = torch.stack(self.patterns)
        for _ in range(iterations):
            xi = torch.softmax(beta * (X @ xi), 0) @ X
        return xi


@dataclass
class HopfieldNetworkConfig:
    network_config: NetworkConfig = field(default_factory=NetworkConfig)
    retrieval_beta: float = 8.0
    retrieval_iterations: int = 3
    base_path: Optional[str] = None


class HopfieldNetwork:
    def __init__(self, config: HopfieldNetworkConfig, seed: int = 0):
        self.config = config
        self.net = Network(_child(config.network_config, config.base_path, None), seed=seed)
        self.memory = HopfieldMemory(self.net.config.layer_sizes[-1])

    def learn(self, x, steps: int) -> None:
        self.net.learn_unsupervised(x, steps)

    def store(self, x, steps: int) -> torch.Tensor:
        z = self.net.infer_get_top(x, steps)
        self.memory.store(z)
        return z

    def recall_latent(self, x, steps: int) -> torch.Tensor:
        return self.memory.retrieve(self.net.infer_get_top(x, steps), self.config.retrieval_beta,
                                    self.config.retrieval_iterations)

    def recall(self, x, steps: int) -> torch.Tensor:
        return self.net.generate(self.recall_latent(x, steps), steps)


# ---------------------------------------------------------------- graph
@dataclass
class GraphPredictiveNetworkConfig:
    edge_predictor_config: NetworkConfig = field(default_factory=lambda: NetworkConfig(layer_sizes=(8, 16, 8)))
    blend_rate: float = 0.5
    base_path: Optional[str] = None

    def validate(self) -> None:
        if self.edge_predictor_config.layer_sizes[0] != self.edge_predictor_config.layer_sizes[-1]:
            raise ValueError("The edge predictor maps node features to node features (same size).")
        if not 0 <= self.blend_rate <= 1:
            raise ValueError("blend_rate must be in [0, 1].")


class GraphPredictiveNetwork:
    def __init__(self, config: GraphPredictiveNetworkConfig, seed: int = 0):
        config.validate()
        self.config = config
        self.edge = Network(_child(config.edge_predictor_config, config.base_path, None), seed=seed)

    @property
    def feature_dim(self) -> int:
        return self.edge.config.layer_sizes[0]

    @staticmethod
    def _check(feats, nbrs):
        if len(feats) != len(nbrs):
            raise ValueError("one neighbour list per node is required")
        for ns in nbrs:
            for j in ns:
                if not 0 <= j < len(feats):
                    raise ValueError("neighbour index out of range")

    def learn(self, feats, nbrs, steps: int) -> None:
        self._check(feats, nbrs)
        for i, ns in enumerate(nbrs):
            for j in ns:
                self.edge.learn(feats[i], feats[j], steps)

    def complete(self, feats, nbrs, observed, steps: int, rounds: int) -> List[torch.Tensor]:
        self._check(feats, nbrs)
        if rounds < 1:
            raise ValueError("rounds must be >= 1.")
        cur = [torch.as_tensor(f, dtype=torch.float32).reshape(-1).clone() for f in feats]
        a = self.config.blend_rate
        for _ in range(rounds):
            nxt = []
            for i, ns in enumerate(nbrs):
                if observed[i] or not ns:
                    nxt.append(cur[i])
                    continue
                cons = sum(self.edge.infer_get_top(cur[j], steps) for j in ns) / len(ns)
                nxt.append((1 - a) * cur[i] + a * cons)
            cur = nxt
        return cur

    def graph_energy(self, feats, nbrs, steps: int) -> float:
        self._check(feats, nbrs)
        return sum(self.edge.infer_energy(feats[i], feats[j], steps) for i, ns in enumerate(nbrs) for j in ns)


# ---------------------------------------------------------------- generative
@dataclass
class GenerativeNetworkConfig:
    network_config: NetworkConfig = field(default_factory=NetworkConfig)
    prior_strength: float = 0.1
    base_path: Optional[str] = None


class GenerativeNetwork:
    def __init__(self, config: GenerativeNetworkConfig, seed: int = 0):
        self.config = config
        self.net = Network(_child(config.network_config, config.base_path, None), seed=seed)
        self.input_dim = self.net.config.layer_sizes[0]
        self.latent_dim = self.net.config.layer_sizes[-1]
        if config.prior_strength > 0:
            self.net.set_top_layer_prior(torch.zeros(self.latent_dim), config.prior_strength)

    def encode(self, x, steps: int) -> torch.Tensor:
        return self.net.infer_get_top(x, steps)

    def decode(self, z, steps: int) -> torch.Tensor:
        return self.net.generate(z, steps)

    def reconstruct(self, x, steps: int) -> torch.Tensor:
        return self.decode(self.encode(x, steps), steps)

    def reconstruction_error(self, x, steps: int) -> float:
        x = torch.as_tensor(x, dtype=torch.float32).reshape(-1)
        return 0.5 * float(((x - self.reconstruct(x, steps)) ** 2).sum())

    def learn(self, x, steps: int) -> None:
        self.net.learn_unsupervised(x, steps)

    def sample(self, steps: int, gen: Optional[torch.Generator] = None) -> torch.Tensor:
        return self.decode(torch.randn(self.latent_dim, generator=gen), steps)
