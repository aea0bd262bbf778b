"""Cortical area models composed from the predictive-coding networks: the retinotopic visual
hierarchy (V1 columns shared across patches -> V2/V4/IT) and the sensory, memory, limbic,
executive, control, language and neuromodulatory areas.

Reference: PredictiveCoding.Cortex/VisualCortex.cs:1-225, RetinotopicMap.cs:1-152,
VisualCortexConfig.cs, and the 45 area files under Sensory/, Memory/, Limbic/, Executive/,
Control/, Language/, Neuromodulation/.  Each class keeps the reference's role and public
operations; the network-backed areas share ``_NetArea`` (encode = settle and read the top layer,
learn = unsupervised or supervised PC learning), and the scalar areas implement their dynamics
directly (energy-softmax gating for basal ganglia / thalamus / cingulate conflict, surprise
adaptation for locus coeruleus / nucleus basalis, TD and baseline errors for the dopamine system,
difference-of-Gaussians for retina/LGN, and so on).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field, replace
from typing import Dict, List, Optional, Sequence, Set, Tuple

import numpy as np
import torch

from ..pc.network import Network, NetworkConfig
from ..pc.networks import (DeepRecurrentNetwork, DeepRecurrentNetworkConfig, GatedStateNetwork,
                           GatedStateNetworkConfig, HierarchicalMixtureOfExperts, HierarchicalMoEConfig,
                           HierarchicalNetwork, HierarchicalNetworkConfig, HopfieldNetwork, HopfieldNetworkConfig,
                           TemporalNetwork, compute_gates)


def _t(x) -> torch.Tensor:
    return torch.as_tensor(x, dtype=torch.float32).reshape(-1)


def _softmax_gates(energies: Sequence[float], temperature: float) -> List[float]:
    return compute_gates(list(energies), temperature, 0.0)


# ---------------------------------------------------------------- retinotopy and visual cortex
class RetinotopicMap:
    def __init__(self, channels: int, height: int, width: int, patch: int, stride: int):
        if not 1 <= patch <= min(height, width) or stride < 1:
            raise ValueError("patch must be in [1, min(height, width)] and stride >= 1")
        self.c, self.h, self.w, self.p, self.s = channels, height, width, patch, stride
        self.gh, self.gw = self.grid(height, patch, stride), self.grid(width, patch, stride)

    @staticmethod
    def grid(dim: int, patch: int, stride: int) -> int:
        return (dim - patch) // stride + 1

    @property
    def patch_count(self) -> int:
        return self.gh * self.gw

    @property
    def patch_dim(self) -> int:
        return self.c * self.p * self.p

    def extract(self, image) -> List[torch.Tensor]:
        im = _t(image)
        if im.numel() != self.c * self.h * self.w:
            raise ValueError("image has the wrong size (C*H*W)")
        im = im.view(self.c, self.h, self.w)
        return [im[:, gy * self.s:gy * self.s + self.p, gx * self.s:gx * self.s + self.p].reshape(-1).clone()
                for gy in range(self.gh) for gx in range(self.gw)]

    def assemble(self, patches: Sequence[torch.Tensor]) -> torch.Tensor:
        """Overlap-averaged image from per-patch reconstructions."""
        acc = torch.zeros(self.c, self.h, self.w)
        cnt = torch.zeros(1, self.h, self.w)
        k = 0
        for gy in range(self.gh):
            for gx in range(self.gw):
                y, x = gy * self.s, gx * self.s
                acc[:, y:y + self.p, x:x + self.p] += _t(patches[k]).view(self.c, self.p, self.p)
                cnt[:, y:y + self.p, x:x + self.p] += 1
                k += 1
        return (acc / cnt.clamp(min=1)).reshape(-1)


@dataclass(frozen=True)
class VisualCortexConfig:
    image_channels: int = 3
    image_height: int = 32
    image_width: int = 32
    patch_size: int = 8
    patch_stride: int = 4
    v1_column: NetworkConfig = field(default_factory=lambda: NetworkConfig(layer_sizes=(192, 32, 8)))
    higher_areas: Optional[HierarchicalNetworkConfig] = None
    classifier: Optional[NetworkConfig] = None

    @property
    def grid_h(self) -> int:
        return RetinotopicMap.grid(self.image_height, self.patch_size, self.patch_stride)

    @property
    def grid_w(self) -> int:
        return RetinotopicMap.grid(self.image_width, self.patch_size, self.patch_stride)

    @property
    def feature_map_dim(self) -> int:
        return self.grid_h * self.grid_w * self.v1_column.layer_sizes[-1]

    def validate(self) -> None:
        if self.v1_column.layer_sizes[0] != self.image_channels * self.patch_size ** 2:
            raise ValueError("v1_column input must equal C*P*P")
        if self.higher_areas is not None and self.higher_areas.modules[0].layer_sizes[0] != self.feature_map_dim:
            raise ValueError("first higher area must take the flattened V1 feature map")
        it = self.higher_areas.modules[-1].layer_sizes[-1] if self.higher_areas else self.feature_map_dim
        if self.classifier is not None and self.classifier.layer_sizes[0] != it:
            raise ValueError("classifier input must equal the IT latent size")


class VisualCortex:
    def __init__(self, cfg: VisualCortexConfig, seed: int = 0):
        cfg.validate()
        self.cfg = cfg
        self.map = RetinotopicMap(cfg.image_channels, cfg.image_height, cfg.image_width, cfg.patch_size,
                                  cfg.patch_stride)
        self.v1 = Network(cfg.v1_column, seed=seed)
        self.higher = HierarchicalNetwork(cfg.higher_areas, seed=seed + 1) if cfg.higher_areas else None
        self.classifier = Network(cfg.classifier, seed=seed + 2) if cfg.classifier else None

    def encode_v1(self, image, steps: int) -> torch.Tensor:
        return torch.cat([self.v1.infer_get_top(p, steps) for p in self.map.extract(image)])

    def encode(self, image, steps: int) -> torch.Tensor:
        v1 = self.encode_v1(image, steps)
        return self.higher.encode(v1, steps) if self.higher else v1

    def encode_areas(self, image, steps: int) -> List[torch.Tensor]:
        v1 = self.encode_v1(image, steps)
        return [v1] + (self.higher.encode_all(v1, steps) if self.higher else [])

    def learn(self, image, steps: int) -> None:
        for p in self.map.extract(image):
            self.v1.learn_unsupervised(p, steps)
        if self.higher:
            self.higher.learn(self.encode_v1(image, steps), steps)

    def learn_supervised(self, image, label, steps: int) -> None:
        if self.classifier is None:
            raise RuntimeError("learn_supervised needs a classifier")
        self.learn(image, steps)
        self.classifier.learn(self.encode(image, steps), label, steps)

    def predict(self, image, steps: int) -> int:
        if self.classifier is None:
            raise RuntimeError("predict needs a classifier")
        return self.classifier.predict(self.encode(image, steps), steps)

    def predict_with_energy(self, image, steps: int):
        return self.classifier.predict_with_energy(self.encode(image, steps), steps)

    def reconstruct(self, image, steps: int) -> torch.Tensor:
        fm = self.encode_v1(image, steps)
        if self.higher:
            fm = self.higher.decode(self.higher.encode(fm, steps), steps)
        k = self.cfg.v1_column.layer_sizes[-1]
        return self.map.assemble([self.v1.generate(fm[i * k:(i + 1) * k], steps) for i in range(self.map.patch_count)])

    def reconstruction_error(self, image, steps: int) -> float:
        return 0.5 * float(((_t(image) - self.reconstruct(image, steps)) ** 2).sum())

    def v1_energy(self) -> float:
        return self.v1.compute_energy()


# ---------------------------------------------------------------- shared building blocks
class _NetArea:
    """An area whose computation is one PC network: encode = settle + top layer."""

    def __init__(self, cfg: NetworkConfig, seed: int = 0):
        self.net = Network(cfg, seed=seed)

    def encode(self, x, steps: int) -> torch.Tensor:
        return self.net.infer_get_top(x, steps)

    def learn(self, x, steps: int) -> None:
        self.net.learn_unsupervised(x, steps)

    def learn_supervised(self, x, label, steps: int) -> None:
        self.net.learn(x, label, steps)

    def recognize(self, x, steps: int) -> int:
        return self.net.predict(x, steps)

    def reconstruct(self, x, steps: int) -> torch.Tensor:
        return self.net.generate(self.encode(x, steps), steps)

    def energy(self) -> float:
        return self.net.compute_energy()


class _PatternMemory:
    """Labelled pattern store with cosine recognition and a familiarity score."""

    def __init__(self, threshold: float = 0.8):
        self.items: List[Tuple[torch.Tensor, object]] = []
        self.threshold = threshold

    def memorize(self, pattern, label) -> None:
        self.items.append((_t(pattern), label))

    def _scores(self, q):
        q = _t(q)
        return [(float(torch.dot(q, p) / (q.norm() * p.norm() + 1e-12)), lab) for p, lab in self.items]

    def recognize(self, pattern):
        s = self._scores(pattern)
        return max(s, key=lambda v: v[0])[1] if s else None

    def familiarity(self, pattern) -> float:
        s = self._scores(pattern)
        return max(v[0] for v in s) if s else 0.0

    def is_novel(self, pattern) -> bool:
        return self.familiarity(pattern) < self.threshold

    def clear_memory(self) -> None:
        self.items.clear()


# ---------------------------------------------------------------- sensory
class RetinaLgn:
    """Centre-surround (difference of Gaussians) responses per channel, edge-clamped separable blurs."""

    def __init__(self, channels: int, height: int, width: int, center_sigma: float = 0.6, surround_sigma: float = 1.5):
        if surround_sigma <= center_sigma:
            raise ValueError("surround_sigma must exceed center_sigma")
        self.c, self.h, self.w, self.cs, self.ss = channels, height, width, center_sigma, surround_sigma

    def _blur(self, im: torch.Tensor, sigma: float) -> torch.Tensor:
        r = max(1, math.ceil(3 * sigma))
        k = torch.exp(-torch.arange(-r, r + 1, dtype=torch.float32) ** 2 / (2 * sigma * sigma))
        k = k / k.sum()
        idx_x = (torch.arange(self.w)[:, None] + torch.arange(-r, r + 1)[None]).clamp(0, self.w - 1)
        idx_y = (torch.arange(self.h)[:, None] + torch.arange(-r, r + 1)[None]).clamp(0, self.h - 1)
        t = (im[:, :, idx_x] * k).sum(-1)                               # [C, H, W] after the x pass
        return (t[:, idx_y, :] * k[None, None, :, None]).sum(2)        # [C, H, 2r+1, W] -> y pass

    def process(self, image) -> torch.Tensor:
        im = _t(image)
        if im.numel() != self.c * self.h * self.w:
            raise ValueError("image has the wrong size")
        im = im.view(self.c, self.h, self.w)
        return (self._blur(im, self.cs) - self._blur(im, self.ss)).reshape(-1)


class SuperiorColliculus:
    def __init__(self, cells: int, visual_weight: float = 1.0, auditory_weight: float = 1.0, enhancement: float = 0.0):
        self.n, self.wv, self.wa, self.e = cells, visual_weight, auditory_weight, enhancement

    def priority_map(self, visual, auditory) -> np.ndarray:
        v, a = np.asarray(visual, np.float32), np.asarray(auditory, np.float32)
        return self.wv * v + self.wa * a + self.e * np.maximum(v, 0) * np.maximum(a, 0)

    def orient(self, visual, auditory, visited: Set[int] = frozenset()) -> int:
        p = self.priority_map(visual, auditory)
        cand = [i for i in range(self.n) if i not in visited]
        return max(cand, key=lambda i: (p[i], -i)) if cand else -1

    def scan(self, visual, auditory, targets: int) -> List[int]:
        seen: Set[int] = set()
        out = []
        for _ in range(min(targets, self.n)):
            i = self.orient(visual, auditory, seen)
            if i < 0:
                break
            seen.add(i)
            out.append(i)
        return out


class FrontalEyeFields:
    """Saccade planning over a retinotopic grid: saliency = patch contrast energy, inhibition of return."""

    def __init__(self, retinotopy: RetinotopicMap):
        self.map = retinotopy

    def saliency_map(self, image) -> np.ndarray:
        return np.array([float(p.var()) for p in self.map.extract(image)], np.float32)

    def patch_position(self, index: int) -> Tuple[int, int]:
        return (index // self.map.gw) * self.map.s, (index % self.map.gw) * self.map.s

    def next_saccade(self, image, visited: Set[int] = frozenset()) -> int:
        s = self.saliency_map(image)
        cand = [i for i in range(len(s)) if i not in visited]
        return max(cand, key=lambda i: (s[i], -i)) if cand else -1

    def scan(self, image, fixations: int) -> List[int]:
        seen: Set[int] = set()
        path = []
        for _ in range(fixations):
            i = self.next_saccade(image, seen)
            if i < 0:
                break
            seen.add(i)
            path.append(i)
        return path


class InferiorColliculus:
    """Per-band log energy of an audio frame (equal-width bands of the magnitude spectrum)."""

    def __init__(self, bands: int = 16):
        self.bands = bands

    def process(self, samples) -> torch.Tensor:
        mag = torch.fft.rfft(_t(samples)).abs()
        chunks = torch.tensor_split(mag, self.bands)
        return torch.stack([torch.log1p((c * c).sum()) for c in chunks])


class OlfactoryBulb:
    """Glomerular normalisation and k-winners-take-all sparsification of a receptor vector."""

    def __init__(self, k: int = 8):
        self.k = k

    def process(self, receptors) -> torch.Tensor:
        x = _t(receptors)
        x = x / (x.norm() + 1e-12)
        out = torch.zeros_like(x)
        idx = torch.topk(x, min(self.k, x.numel())).indices
        out[idx] = x[idx]
        return out


class AuditoryCortex(_NetArea):
    pass


class SomatosensoryCortex(_NetArea):
    pass


class FusiformFaceArea(_NetArea):
    pass


class SuperiorTemporalSulcus:
    """Audio-visual integration: concatenated latents classified by one network."""

    def __init__(self, cfg: NetworkConfig, seed: int = 0):
        self.net = Network(cfg, seed=seed)

    def integrate(self, a, b) -> torch.Tensor:
        return torch.cat([_t(a), _t(b)])

    def learn(self, a, b, label, steps: int) -> None:
        self.net.learn(self.integrate(a, b), label, steps)

    def classify(self, a, b, steps: int) -> int:
        return self.net.predict(self.integrate(a, b), steps)


class DorsalStream:
    """Motion: frame differences fed to a temporal network that predicts the next difference."""

    def __init__(self, cfg: NetworkConfig, seed: int = 0, temporal_precision: float = 0.5):
        self.tn = TemporalNetwork(Network(cfg, seed=seed), temporal_precision)
        self.prev: Optional[torch.Tensor] = None

    def learn_sequence(self, frames: Sequence, steps: int) -> None:
        self.tn.reset()
        prev = None
        for f in frames:
            f = _t(f)
            if prev is not None:
                d = f - prev
                self.tn.base.learn_unsupervised(d, steps)
            prev = f

    def predict_motion(self, frame_a, frame_b, steps: int) -> torch.Tensor:
        net = self.tn.base
        return net.generate(net.infer_get_top(_t(frame_b) - _t(frame_a), steps), steps)


class GustatoryCortex(_PatternMemory):
    learn = _PatternMemory.memorize


class VestibularSystem:
    def __init__(self, cfg: DeepRecurrentNetworkConfig, seed: int = 0):
        self.integrator = DeepRecurrentNetwork(cfg, seed=seed)

    def integrate(self, motion, steps: int) -> torch.Tensor:
        return self.integrator.step(motion, steps)

    def head_direction(self, motion, steps: int) -> torch.Tensor:
        return self.integrator.encode(motion, steps)

    def reset(self) -> None:
        self.integrator.reset()


# ---------------------------------------------------------------- memory
class GridCellEncoder:
    """Modules of hexagonal grid cells: three plane waves at 60 degrees per cell, module frequencies
    in geometric progression, cell phases tiling each module's period."""

    def __init__(self, modules: int, cells_per_module: int, base_frequency: float, ratio: float, seed: int = 0):
        if modules < 1 or cells_per_module < 1:
            raise ValueError("modules and cells_per_module must be >= 1")
        rng = np.random.default_rng(seed)
        self.m, self.k = modules, cells_per_module
        self.freq = base_frequency * ratio ** np.arange(modules)
        side = max(1, round(math.sqrt(cells_per_module)))
        per = 2 * math.pi / self.freq
        kk = np.arange(cells_per_module)
        self.px = np.concatenate([((kk % side) + 0.5) / side * per[m] + rng.uniform(0, 0.01, self.k)
                                  for m in range(modules)])
        self.py = np.concatenate([((kk // side) + 0.5) / side * per[m] + rng.uniform(0, 0.01, self.k)
                                  for m in range(modules)])
        self.dirs = np.array([[1, 0], [-0.5, math.sqrt(3) / 2], [-0.5, -math.sqrt(3) / 2]])

    @property
    def code_dim(self) -> int:
        return self.m * self.k

    def encode(self, x: float, y: float) -> torch.Tensor:
        f = np.repeat(self.freq, self.k)
        dx, dy = x - self.px, y - self.py
        s = sum(np.cos(f * (d[0] * dx + d[1] * dy)) for d in self.dirs)
        return torch.tensor((s + 1.5) / 4.5, dtype=torch.float32)


class EntorhinalCortex:
    """Grid code of a position -> network that predicts the observation seen there."""

    def __init__(self, grid: GridCellEncoder, cfg: NetworkConfig, seed: int = 0):
        if cfg.layer_sizes[0] != grid.code_dim:
            raise ValueError("network input must equal the grid code size")
        self.grid, self.net = grid, Network(cfg, seed=seed)

    def encode_position(self, x: float, y: float) -> torch.Tensor:
        return self.grid.encode(x, y)

    def learn(self, x: float, y: float, observation, steps: int) -> None:
        self.net.learn(self.grid.encode(x, y), observation, steps)

    def predict_observation(self, x: float, y: float, steps: int) -> torch.Tensor:
        return self.net.infer_get_top(self.grid.encode(x, y), steps)


@dataclass(frozen=True)
class HippocampalFormationConfig:
    hippocampus: HopfieldNetworkConfig = field(default_factory=HopfieldNetworkConfig)
    neocortex: NetworkConfig = field(default_factory=NetworkConfig)
    max_episodes: int = 256


class HippocampalFormation:
    """Fast episodic storage (Hopfield) plus slow neocortical consolidation by replay."""

    def __init__(self, cfg: HippocampalFormationConfig, seed: int = 0):
        if cfg.neocortex.layer_sizes[0] != cfg.hippocampus.network_config.layer_sizes[0]:
            raise ValueError("neocortex input must equal the hippocampal input")
        self.cfg = cfg
        self.hpc = HopfieldNetwork(cfg.hippocampus, seed=seed)
        self.neo = Network(cfg.neocortex, seed=seed + 1)
        self.episodes: List[torch.Tensor] = []

    @property
    def episode_count(self) -> int:
        return len(self.episodes)

    def experience(self, x, steps: int) -> None:
        self.hpc.learn(x, steps)
        self.hpc.store(x, steps)
        self.episodes.append(_t(x).clone())
        if len(self.episodes) > self.cfg.max_episodes:
            self.episodes.pop(0)

    def recall(self, cue, steps: int) -> torch.Tensor:
        return self.hpc.recall(cue, steps)

    def replay(self, rounds: int, steps: int, seed: int = 0) -> None:
        rng = np.random.default_rng(seed)
        for _ in range(rounds):
            for i in rng.permutation(len(self.episodes)):
                self.neo.learn_unsupervised(self.episodes[i], steps)

    def neocortical_encode(self, x, steps: int) -> torch.Tensor:
        return self.neo.infer_get_top(x, steps)


class ParahippocampalCortex(_NetArea):
    def __init__(self, cfg: NetworkConfig, seed: int = 0, threshold: float = 0.9):
        super().__init__(cfg, seed)
        self.places = _PatternMemory(threshold)

    def encode_scene(self, x, steps: int) -> torch.Tensor:
        return self.encode(x, steps)

    def remember_place(self, x, place, steps: int) -> None:
        self.places.memorize(self.encode(x, steps), place)

    def recognize_place(self, x, steps: int):
        return self.places.recognize(self.encode(x, steps))


class PerirhinalCortex(_NetArea):
    def __init__(self, cfg: NetworkConfig, seed: int = 0, novelty_threshold: float = 0.9):
        super().__init__(cfg, seed)
        self.memory = _PatternMemory(novelty_threshold)

    def remember(self, x, steps: int, label=None) -> None:
        self.memory.memorize(self.encode(x, steps), label)

    def familiarity(self, x, steps: int) -> float:
        return self.memory.familiarity(self.encode(x, steps))

    def is_novel(self, x, steps: int) -> bool:
        return self.memory.is_novel(self.encode(x, steps))


class PiriformCortex(_PatternMemory):
    learn = _PatternMemory.memorize


# ---------------------------------------------------------------- limbic
class Amygdala(_NetArea):
    def appraise(self, stimulus, steps: int) -> torch.Tensor:
        return self.encode(stimulus, steps)

    def learn(self, stimulus, affect, steps: int) -> None:    # supervised: stimulus -> affect
        self.net.learn(stimulus, affect, steps)

    def salience_gain(self, stimulus, steps: int, base_gain: float = 1.0) -> float:
        return base_gain * (1.0 + float(self.appraise(stimulus, steps).abs().max()))


class CingulateCortex:
    def __init__(self, temperature: float = 1.0):
        self.temperature = temperature

    @staticmethod
    def surprise(energies: Sequence[float]) -> float:
        return float(sum(energies))

    def conflict(self, energies: Sequence[float]) -> float:
        n = len(energies)
        if n <= 1:
            return 0.0
        g = _softmax_gates(energies, self.temperature)
        return -sum(x * math.log(x) for x in g if x > 0) / math.log(n)

    def monitor(self, energies):
        return self.surprise(energies), self.conflict(energies)

    def needs_control(self, energies, threshold: float = 0.8) -> bool:
        return self.conflict(energies) >= threshold


class Hypothalamus:
    def __init__(self, set_points: Sequence[float]):
        self.set_points = np.asarray(set_points, np.float32)

    def drive(self, current) -> np.ndarray:
        return self.set_points - np.asarray(current, np.float32)

    def need_level(self, current) -> float:
        return float(np.linalg.norm(self.drive(current)))

    def goal(self) -> torch.Tensor:
        return torch.tensor(self.set_points)


class InsularCortex:
    """Interoceptive feeling: exponentially smoothed homeostatic need."""

    def __init__(self, hypothalamus: Hypothalamus, smoothing: float = 0.2):
        self.h, self.a = hypothalamus, smoothing
        self.feeling = 0.0

    def experience(self, body_state) -> float:
        self.feeling += self.a * (self.h.need_level(body_state) - self.feeling)
        return self.feeling

    def feel(self) -> float:
        return self.feeling

    def reset(self) -> None:
        self.feeling = 0.0


class NucleusAccumbens:
    """Incentive salience = value x (1 + need); option gates by softmax of salience."""

    def __init__(self, temperature: float = 1.0):
        self.temperature = temperature

    @staticmethod
    def incentive_salience(values: Sequence[float], need: float) -> List[float]:
        return [v * (1.0 + need) for v in values]

    def gate_weights(self, values, need: float) -> List[float]:
        return _softmax_gates([-s for s in self.incentive_salience(values, need)], self.temperature)

    def select(self, values, need: float) -> int:
        s = self.incentive_salience(values, need)
        return max(range(len(s)), key=lambda i: (s[i], -i))


class OrbitofrontalCortex(_NetArea):
    def estimate_value(self, x, steps: int) -> float:
        return float(self.encode(x, steps).mean())

    def learn(self, x, value, steps: int) -> None:
        self.net.learn(x, _t(value) * torch.ones(self.net.config.layer_sizes[-1]), steps)


class PeriaqueductalGray:
    """Defensive response by threat level: none / freeze / flight / fight."""

    def __init__(self, freeze: float = 0.3, flight: float = 0.6, fight: float = 0.9):
        self.t = (freeze, flight, fight)

    def respond(self, threat: float) -> str:
        if threat >= self.t[2]:
            return "fight"
        if threat >= self.t[1]:
            return "flight"
        if threat >= self.t[0]:
            return "freeze"
        return "none"


# ---------------------------------------------------------------- executive
@dataclass(frozen=True)
class CerebellarCortexConfig:
    state_dim: int
    command_dim: int
    forward_model: NetworkConfig


class CerebellarCortex:
    def __init__(self, cfg: CerebellarCortexConfig, seed: int = 0):
        if cfg.forward_model.layer_sizes[0] != cfg.state_dim + cfg.command_dim \
                or cfg.forward_model.layer_sizes[-1] != cfg.state_dim:
            raise ValueError("forward model must map [state | command] -> next state")
        self.cfg, self.net = cfg, Network(cfg.forward_model, seed=seed)

    def _in(self, s, c) -> torch.Tensor:
        return torch.cat([_t(s), _t(c)])

    def predict(self, state, command, steps: int) -> torch.Tensor:
        return self.net.infer_get_top(self._in(state, command), steps)

    def learn(self, state, command, actual_next, steps: int) -> None:
        self.net.learn(self._in(state, command), actual_next, steps)

    def prediction_error(self, state, command, actual_next, steps: int) -> float:
        return 0.5 * float(((self.predict(state, command, steps) - _t(actual_next)) ** 2).sum())


class MotorCortex:
    """Commands chosen by the cerebellar forward model: the candidate whose predicted outcome is
    closest to the goal."""

    def __init__(self, cerebellum: CerebellarCortex, commands: Sequence):
        self.cb, self.commands = cerebellum, [_t(c) for c in commands]

    def predict_outcome(self, state, k: int, steps: int) -> torch.Tensor:
        return self.cb.predict(state, self.commands[k], steps)

    def select_command(self, state, goal, steps: int) -> int:
        d = [float(((self.predict_outcome(state, k, steps) - _t(goal)) ** 2).sum()) for k in range(len(self.commands))]
        return min(range(len(d)), key=lambda i: (d[i], i))

    def learn(self, state, k: int, actual_next, steps: int) -> None:
        self.cb.learn(state, self.commands[k], actual_next, steps)

    def reach_goal(self, state, goal, environment, steps: int, max_moves: int = 20, tol: float = 1e-2):
        path = []
        s = _t(state)
        for _ in range(max_moves):
            k = self.select_command(s, goal, steps)
            s = _t(environment(s, self.commands[k]))
            path.append(k)
            if float(((s - _t(goal)) ** 2).sum()) < tol:
                break
        return path, s


class PremotorCortex:
    """Action sequences: a temporal network predicts the next action code from the current one."""

    def __init__(self, cfg: NetworkConfig, seed: int = 0, temporal_precision: float = 0.5):
        self.tn = TemporalNetwork(Network(cfg, seed=seed), temporal_precision)

    def learn_step(self, action, next_action, steps: int) -> None:
        self.tn.step(action, next_action, steps)

    def next_action(self, action, steps: int) -> int:
        return self.tn.predict(action, steps)

    def reset(self) -> None:
        self.tn.reset()


@dataclass(frozen=True)
class PrefrontalCortexConfig:
    working_memory: GatedStateNetworkConfig
    task_experts: HierarchicalMoEConfig


class PrefrontalCortex:
    def __init__(self, cfg: PrefrontalCortexConfig, seed: int = 0):
        self.wm = GatedStateNetwork(cfg.working_memory, seed=seed)
        self.experts = HierarchicalMixtureOfExperts(cfg.task_experts, seed=seed + 1)

    def step(self, x, steps: int) -> torch.Tensor:
        return self.wm.step(x, steps)

    def learn(self, x, label, steps: int) -> None:
        self.experts.learn(self.wm.step(x, steps), label, steps)

    def decide(self, x, steps: int) -> int:
        return self.experts.predict(self.wm.step(x, steps), steps)

    def reset(self) -> None:
        self.wm.reset()


class FrontopolarCortex:
    """Holds a pending alternative goal and switches when its accumulated advantage exceeds a bound."""

    def __init__(self, switch_threshold: float = 1.0, decay: float = 0.9):
        self.threshold, self.decay = switch_threshold, decay
        self.held = None
        self.evidence = 0.0

    def hold(self, goal) -> None:
        self.held = goal
        self.evidence = 0.0

    def should_switch(self, current_energy: float, alternative_energy: float) -> bool:
        self.evidence = self.decay * self.evidence + (current_energy - alternative_energy)
        return self.held is not None and self.evidence > self.threshold

    def clear(self) -> None:
        self.held = None
        self.evidence = 0.0


# ---------------------------------------------------------------- control
class BasalGanglia:
    def __init__(self, temperature: float = 1.0, no_go_threshold: Optional[float] = None):
        if temperature <= 0:
            raise ValueError("temperature must be > 0")
        self.temperature, self.no_go = temperature, no_go_threshold

    def select(self, energies: Sequence[float]):
        if not energies:
            raise ValueError("At least one candidate action is required.")
        g = _softmax_gates(energies, self.temperature)
        best = min(range(len(energies)), key=lambda i: (energies[i], i))
        if self.no_go is not None and energies[best] > self.no_go:
            return -1, g
        return best, g


class Thalamus:
    def __init__(self, temperature: float = 1.0, base_precision: float = 1.0):
        self.temperature, self.base = temperature, base_precision

    def allocate(self, energies: Sequence[float]) -> List[float]:
        if not energies:
            return []
        return [self.base * len(energies) * g for g in _softmax_gates(energies, self.temperature)]

    def modulate(self, areas: Sequence[Network]) -> List[float]:
        p = self.allocate([a.compute_energy() for a in areas])
        for a, pi in zip(areas, p):
            a.set_top_layer_prior(None, pi)
        return p


class Pulvinar(Thalamus):
    """Attention allocation across areas by the same energy softmax (relayed precision)."""


class Claustrum:
    @staticmethod
    def coherence(latents: Sequence) -> float:
        xs = [_t(v) for v in latents]
        if len(xs) < 2:
            return 1.0
        sims = [float(torch.dot(a, b) / (a.norm() * b.norm() + 1e-12)) for i, a in enumerate(xs) for b in xs[i + 1:]]
        return sum(sims) / len(sims)

    @staticmethod
    def synchronize(latents: Sequence) -> torch.Tensor:
        return torch.stack([_t(v) for v in latents]).mean(0)


class TemporoparietalJunction:
    def __init__(self, threshold: float = 2.0, adaptation: float = 0.1):
        self.threshold, self.a = threshold, adaptation
        self.expected = None

    def reorient_signal(self, surprise: float) -> float:
        if self.expected is None:
            self.expected = surprise
            return 0.0
        sig = surprise / (self.expected + 1e-12)
        self.expected += self.a * (surprise - self.expected)
        return sig

    def should_reorient(self, surprise: float) -> bool:
        return self.reorient_signal(surprise) > self.threshold


class PosteriorParietalCortex(_NetArea):
    """Coordinate transform learned as a supervised map (e.g. eye-centred -> body-centred)."""

    def learn(self, x, target, steps: int) -> None:
        self.net.learn(x, target, steps)

    def transform(self, x, steps: int) -> torch.Tensor:
        return self.encode(x, steps)

    def locate(self, x, steps: int) -> int:
        return int(self.transform(x, steps).argmax())


class DefaultModeNetwork:
    """Imagination by generating from latents of past experience."""

    def __init__(self, cfg: NetworkConfig, seed: int = 0):
        self.net = Network(cfg, seed=seed)
        self.latents: List[torch.Tensor] = []

    def learn_from_experience(self, x, steps: int) -> None:
        self.net.learn_unsupervised(x, steps)
        self.latents.append(self.net.infer_get_top(x, steps))

    def imagine(self, steps: int, seed: int = 0, mix: float = 0.5) -> torch.Tensor:
        g = torch.Generator().manual_seed(seed)
        if len(self.latents) >= 2:
            i, j = torch.randint(len(self.latents), (2,), generator=g).tolist()
            z = (1 - mix) * self.latents[i] + mix * self.latents[j]
        else:
            z = torch.randn(self.net.config.layer_sizes[-1], generator=g)
        return self.net.generate(z, steps)

    def imagine_sequence(self, n: int, steps: int) -> List[torch.Tensor]:
        return [self.imagine(steps, seed=k) for k in range(n)]


class AssociationCortex:
    """Binds two modality latents; cross-modal prediction by a network trained a -> b."""

    def __init__(self, cfg_ab: NetworkConfig, seed: int = 0):
        self.net = Network(cfg_ab, seed=seed)

    @staticmethod
    def bind(a, b) -> torch.Tensor:
        return torch.cat([_t(a), _t(b)])

    def learn(self, a, b, steps: int) -> None:
        self.net.learn(a, b, steps)

    def cross_modal(self, a, steps: int) -> torch.Tensor:
        return self.net.infer_get_top(a, steps)

    def predict(self, a, steps: int) -> int:
        return int(self.cross_modal(a, steps).argmax())


# ---------------------------------------------------------------- language
class WernickeArea(_NetArea):
    """Comprehension: utterance -> meaning latent; surprise = settled energy."""

    def learn_utterance(self, utterance, meaning, steps: int) -> None:
        self.net.learn(utterance, meaning, steps)

    def comprehend(self, utterance, steps: int) -> torch.Tensor:
        return self.encode(utterance, steps)

    def listen(self, utterance, steps: int) -> Tuple[torch.Tensor, float]:
        m = self.encode(utterance, steps)
        return m, self.net.compute_energy()

    def surprise(self, utterance, steps: int) -> float:
        return self.listen(utterance, steps)[1]


class BrocaArea:
    """Production: meaning latent -> utterance (generative direction of a PC network)."""

    def __init__(self, cfg: NetworkConfig, seed: int = 0):
        self.net = Network(cfg, seed=seed)

    def learn_utterance(self, utterance, meaning, steps: int) -> None:
        self.net.learn(utterance, meaning, steps)

    def produce_from_meaning(self, meaning, steps: int) -> torch.Tensor:
        return self.net.generate(meaning, steps)

    def produce(self, meaning, steps: int) -> int:
        return int(self.produce_from_meaning(meaning, steps).argmax())

    def produce_sequence(self, meanings: Sequence, steps: int) -> List[int]:
        return [self.produce(m, steps) for m in meanings]


class AngularGyrus:
    """Relational association: learns pairs (a, b); relational energy of a new pair."""

    def __init__(self, cfg: NetworkConfig, seed: int = 0):
        self.net = Network(cfg, seed=seed)

    def learn(self, a, b, steps: int) -> None:
        self.net.learn(a, b, steps)

    def associate(self, a, steps: int) -> torch.Tensor:
        return self.net.infer_get_top(a, steps)

    def relational_energy(self, a, b, steps: int) -> float:
        return self.net.infer_energy(a, b, steps)


class VisualWordFormArea(_NetArea):
    def learn(self, image, word_label, steps: int) -> None:
        self.net.learn(image, word_label, steps)


# ---------------------------------------------------------------- neuromodulation
class DopaminergicSystem:
    def __init__(self, discount: float = 0.95, tonic_level: float = 0.1, baseline_lr: float = 0.05):
        if not 0 <= discount <= 1 or tonic_level < 0 or not 0 < baseline_lr <= 1:
            raise ValueError("invalid dopamine parameters")
        self.discount, self.tonic, self.lr = discount, tonic_level, baseline_lr
        self.baseline = 0.0

    def reward_prediction_error(self, reward: float, v_now: float, v_next: Optional[float] = None) -> float:
        return reward - v_now if v_next is None else reward + self.discount * v_next - v_now

    def step(self, reward: float) -> float:
        d = reward - self.baseline
        self.baseline += self.lr * d
        return d

    def modulate_learning_rate(self, base_lr: float, rpe: float) -> float:
        if base_lr < 0:
            raise ValueError("base learning rate must be >= 0")
        return base_lr * (self.tonic + abs(rpe))

    def reset(self) -> None:
        self.baseline = 0.0


class Habenula:
    def __init__(self, gain: float = 1.0):
        self.gain = gain

    @staticmethod
    def disappointment(reward: float, expected: float) -> float:
        return expected - reward

    @staticmethod
    def negative_prediction_error(reward: float, expected: float) -> float:
        return max(0.0, expected - reward)

    def suppress_dopamine(self, dopamine: float, reward: float, expected: float) -> float:
        return dopamine - self.gain * self.negative_prediction_error(reward, expected)


class LocusCoeruleus:
    def __init__(self, adaptation: float = 0.1, phasic_threshold: float = 1.5, phasic_gain: float = 4.0,
                 tonic_gain: float = 1.0):
        if not 0 < adaptation <= 1 or phasic_threshold <= 1 or phasic_gain <= 0 or tonic_gain <= 0:
            raise ValueError("invalid locus coeruleus parameters")
        self.a, self.th, self.pg, self.tg = adaptation, phasic_threshold, phasic_gain, tonic_gain
        self.expected = 0.0
        self.init = False

    def process(self, surprise: float) -> Tuple[bool, float]:
        if surprise < 0:
            raise ValueError("surprise must be >= 0")
        if not self.init:
            self.expected, self.init, burst = surprise, True, False
        else:
            burst = surprise > self.th * self.expected
            self.expected += self.a * (surprise - self.expected)
        return burst, (self.pg if burst else self.tg)

    @staticmethod
    def global_surprise(areas: Sequence[Network]) -> float:
        return sum(a.compute_energy() for a in areas)

    def modulate(self, areas: Sequence[Network]) -> float:
        _, g = self.process(self.global_surprise(areas))
        for a in areas:
            a.set_top_layer_prior(None, g)
        return g

    def reset(self) -> None:
        self.expected, self.init = 0.0, False


class NucleusBasalis:
    def __init__(self, areas: int, adaptation: float = 0.1, gain: float = 1.0):
        if areas <= 0 or not 0 < adaptation <= 1 or gain < 0:
            raise ValueError("invalid nucleus basalis parameters")
        self.n, self.a, self.gain = areas, adaptation, gain
        self.expected = np.zeros(areas, np.float32)
        self.init = False

    def update(self, energies) -> np.ndarray:
        e = np.asarray([x.compute_energy() if isinstance(x, Network) else x for x in energies], np.float32)
        if len(e) != self.n:
            raise ValueError("one energy per area")
        self.expected = self.expected + self.a * (e - self.expected) if self.init else e.copy()
        self.init = True
        return self.gain * self.expected

    def modulate_learning_rates(self, base_lr: float, energies) -> np.ndarray:
        return base_lr * (1 + self.update(energies))

    def reset(self) -> None:
        self.expected[:] = 0
        self.init = False


class RapheNuclei:
    def __init__(self, level: float = 0.5):
        self.level = level

    @property
    def level(self) -> float:
        return self._level

    @level.setter
    def level(self, v: float) -> None:
        self._level = min(max(v, 0.0), 1.0)

    def discount_factor(self, min_gamma: float = 0.5, max_gamma: float = 0.99) -> float:
        return min_gamma + self._level * (max_gamma - min_gamma)

    def time_horizon(self, min_gamma: float = 0.5, max_gamma: float = 0.99) -> float:
        return 1.0 / (1.0 - self.discount_factor(min_gamma, max_gamma))


AREAS = {c.__name__: c for c in (
    RetinaLgn, SuperiorColliculus, FrontalEyeFields, InferiorColliculus, OlfactoryBulb, AuditoryCortex,
    SomatosensoryCortex, FusiformFaceArea, SuperiorTemporalSulcus, DorsalStream, GustatoryCortex, VestibularSystem,
    EntorhinalCortex, HippocampalFormation, ParahippocampalCortex, PerirhinalCortex, PiriformCortex, Amygdala,
    CingulateCortex, Hypothalamus, InsularCortex, NucleusAccumbens, OrbitofrontalCortex, PeriaqueductalGray,
    CerebellarCortex, MotorCortex, PremotorCortex, PrefrontalCortex, FrontopolarCortex, BasalGanglia, Thalamus,
    Pulvinar, Claustrum, TemporoparietalJunction, PosteriorParietalCortex, DefaultModeNetwork, AssociationCortex,
    WernickeArea, BrocaArea, AngularGyrus, VisualWordFormArea, DopaminergicSystem, Habenula, LocusCoeruleus,
    NucleusBasalis, RapheNuclei, VisualCortex, RetinotopicMap, GridCellEncoder)}
