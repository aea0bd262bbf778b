"""The predictive-coding network (per-sample engine; the CPU oracle).

Reference: PredicitiveCoding/Networks/Network.cs:23-1365, NetworkConfig.cs:5-133,
EffortLevel.cs:14-40.  Semantics reproduced exactly:

* inference is Jacobi-synchronous: every layer predicts the layer below from the
  *old* states, all errors are formed, then every unclamped layer updates
  (Network.cs:75-119);
* ``learn`` clamps input and label, settles, then applies the Hebbian update using
  the last prediction and the updated states, and persists the layers (:139-156);
* ``predict`` is argmin over one-hot label candidates of the free energy, re-running
  the winner so the stored state is the best explanation (:369-435);
* inference calls work on transient copies (the store is not changed) except where
  the reference persists (learn / predict / learn_unsupervised ...).

The store is :class:`LayerStore` (in memory, with optional on-disk persistence in
the reference's LayerSerializer record format).  A reentrant lock serialises
writers against readers the way the reference's ReaderWriterLockSlim does.
"""
from __future__ import annotations

import os
import threading
from dataclasses import dataclass, field, replace
from typing import List, Optional, Sequence, Tuple

import torch

from .layer import ACTIVATIONS, Layer
from .store import LayerStore

EFFORT_PRESETS = {"low": (10, 1e-3), "medium": (30, 1e-4), "high": (100, 1e-5)}


@dataclass
class NetworkConfig:
    """Reference NetworkConfig (NetworkConfig.cs:5-133) with the same defaults."""
    layer_sizes: Sequence[int] = (20, 64, 32, 4)
    activation: str = "tanh"
    state_lr: float = 0.1
    weight_lr: float = 1e-3
    weight_decay: float = 0.0
    use_diagonal_precision: bool = False
    lazy_persistence: bool = False
    use_feedforward_gist_init: bool = False
    activity_regularization: float = 0.0
    input_shape: Optional[Sequence[int]] = None
    output_shape: Optional[Sequence[int]] = None
    path: Optional[str] = None

    @property
    def input_size(self) -> int:
        if self.input_shape is None:
            return self.layer_sizes[0]
        n = 1
        for d in self.input_shape:
            n *= d
        return n

    @property
    def output_size(self) -> int:
        if self.output_shape is None:
            return self.layer_sizes[-1]
        n = 1
        for d in self.output_shape:
            n *= d
        return n

    def validate(self) -> None:
        if len(self.layer_sizes) < 2:
            raise ValueError("LayerSizes must have at least 2 elements.")
        if self.state_lr < 0:
            raise ValueError("StateLearningRate must be >= 0.")
        if self.weight_lr < 0:
            raise ValueError("WeightLearningRate must be >= 0.")
        if self.weight_decay < 0:
            raise ValueError("WeightDecay must be >= 0.")
        if self.activity_regularization < 0:
            raise ValueError("ActivityRegularization must be >= 0.")
        if self.activation not in ACTIVATIONS:
            raise ValueError(f"unknown activation {self.activation!r}")
        if self.input_shape is not None:
            if any(d <= 0 for d in self.input_shape):
                raise ValueError("All InputShape dimensions must be > 0.")
            if self.input_size != self.layer_sizes[0]:
                raise ValueError(f"InputShape product ({self.input_size}) must equal LayerSizes[0] "
                                 f"({self.layer_sizes[0]}).")
        if self.output_shape is not None:
            if any(d <= 0 for d in self.output_shape):
                raise ValueError("All OutputShape dimensions must be > 0.")
            if self.output_size != self.layer_sizes[-1]:
                raise ValueError(f"OutputShape product ({self.output_size}) must equal LayerSizes[^1] "
                                 f"({self.layer_sizes[-1]}).")
        if self.path is not None:
            os.makedirs(self.path, exist_ok=True)


@dataclass
class GenerativeSnapshot:
    """Read-only export consumed by the batched engine (Networks/GenerativeSnapshot.cs:15-23)."""
    layer_sizes: List[int]
    activation: str
    state_lr: float
    activity_regularization: float
    use_feedforward_gist_init: bool
    weights: List[torch.Tensor]     # W_l [lower, size], l = 1..L-1
    biases: List[torch.Tensor]      # b_l [lower]
    precisions: List[float]         # Pi_l, l = 0..L-1


class Network:
    """Predictive-coding network with the reference's public API (snake_case)."""

    def __init__(self, config: NetworkConfig, seed: int = 0, store: Optional[LayerStore] = None):
        config.validate()
        self.config = config
        self._lock = threading.RLock()
        if store is None:
            gen = torch.Generator().manual_seed(seed)
            sizes = list(config.layer_sizes)
            layers = []
            for l, s in enumerate(sizes):
                lower = sizes[l - 1] if l > 0 else 0
                L = Layer.create(l, s, lower, config.activation, gen, state_lr=config.state_lr,
                                 weight_lr=config.weight_lr, weight_decay=config.weight_decay)
                if config.use_diagonal_precision:
                    L.init_diagonal_precision()
                layers.append(L)
            store = LayerStore(layers, path=config.path, lazy=config.lazy_persistence)
        self._store = store

    @property
    def layer_count(self) -> int:
        return len(self.config.layer_sizes)

    # ------------------------------------------------------------ helpers
    def _read_all(self) -> List[Layer]:
        return [self._store.read(l) for l in range(self.layer_count)]

    def _flatten(self, x: torch.Tensor) -> torch.Tensor:
        x = torch.as_tensor(x, dtype=torch.float32).reshape(-1)
        if x.numel() != self.config.layer_sizes[0]:
            raise ValueError(f"Input has {x.numel()} elements but the network expects "
                             f"{self.config.layer_sizes[0]} (LayerSizes[0]).")
        return x

    def _flatten_label(self, y: torch.Tensor) -> torch.Tensor:
        y = torch.as_tensor(y, dtype=torch.float32).reshape(-1)
        if y.numel() != self.config.layer_sizes[-1]:
            raise ValueError(f"Label has {y.numel()} elements but the top layer has "
                             f"{self.config.layer_sizes[-1]} units.")
        return y

    @staticmethod
    def _clamp(layers: List[Layer], i: int, value: torch.Tensor) -> None:
        layers[i].mu = value.clone().float()
        layers[i].is_clamped = True

    def _ffg(self, layers: List[Layer]) -> None:
        """Feed-forward gist warm start: one top-down sweep seeding hidden states (Network.cs:121-137)."""
        for l in range(len(layers) - 1, 0, -1):
            layers[l].compute_prediction()
            if l > 1 and not layers[l - 1].is_clamped:
                layers[l - 1].mu = layers[l].pred.clone()

    # ---- override points for architecture variants (attention gates, skips, ...)
    def _lower_error(self, layers: List[Layer], l: int) -> torch.Tensor:
        """Error of layer l-1 as seen by layer l's state and weight updates."""
        return layers[l - 1].eps

    def _after_predictions(self, layers: List[Layer]) -> None:
        """Hook between the top-down predictions and the error computation."""

    def _after_state_updates(self, layers: List[Layer]) -> None:
        """Hook after the state updates of a relaxation step."""

    def _after_learn(self, layers: List[Layer], lr_scale: float) -> None:
        """Hook after the Hebbian weight updates of a learning step."""

    def _update_weights(self, layers: List[Layer], lr: float) -> None:
        for l in range(1, len(layers)):
            layers[l].update_weights(self._lower_error(layers, l), lr)
            layers[l].W_half = None
            self._store.write(l, layers[l])

    def _relax_step(self, layers: List[Layer]) -> None:
        L = len(layers)
        for l in range(L - 1, 0, -1):
            layers[l].compute_prediction()
        self._after_predictions(layers)
        for l in range(1, L):
            layers[l - 1].set_prediction_error(layers[l].pred)
        layers[-1].set_prediction_error(None)
        for l in range(1, L):
            if not layers[l].is_clamped:
                layers[l].update_state(self._lower_error(layers, l), self.config.state_lr,
                                       self.config.activity_regularization)
        self._after_state_updates(layers)

    def _infer_core(self, layers, x, steps, clamp_top, label) -> None:
        self._clamp(layers, 0, self._flatten(x))
        if clamp_top and label is not None:
            self._clamp(layers, len(layers) - 1, self._flatten_label(label))
        else:
            layers[-1].is_clamped = False
        if self.config.use_feedforward_gist_init:
            self._ffg(layers)
        for _ in range(steps):
            self._relax_step(layers)

    @staticmethod
    def _energy(layers: List[Layer]) -> float:
        return sum(layers[l].local_energy() for l in range(len(layers) - 1))

    def _write_back(self, layers, which) -> None:
        for l in which:
            self._store.write(l, layers[l])

    # ------------------------------------------------------------ inference
    def infer(self, x, steps: int, clamp_top: bool = False, label=None) -> None:
        with self._lock:
            self._infer_core(self._read_all(), x, steps, clamp_top, label)

    def infer_mixed(self, x, steps: int, clamp_top: bool = False, label=None) -> None:
        with self._lock:
            layers = self._read_all()
            for L in layers[1:]:
                L.quantize_weights()
            self._infer_core(layers, x, steps, clamp_top, label)

    def infer_energy(self, x, label, steps: int) -> float:
        with self._lock:
            layers = self._read_all()
            self._infer_core(layers, x, steps, True, label)
            return self._energy(layers)

    def infer_get_top(self, x, steps: int, reset_state: bool = False, mixed: bool = False) -> torch.Tensor:
        """Free inference (top unclamped); returns the top state (Network.cs:1068-1100)."""
        with self._lock:
            layers = self._read_all()
            if mixed:
                for L in layers[1:]:
                    L.quantize_weights()
            if reset_state:
                for L in layers[1:]:
                    L.mu = torch.zeros_like(L.mu)
            self._infer_core(layers, x, steps, False, None)
            return layers[-1].mu.clone()

    def infer_trace(self, x, steps: int) -> List[float]:
        """Free inference returning the energy after every step (Network.cs:700-735)."""
        with self._lock:
            layers = self._read_all()
            self._clamp(layers, 0, self._flatten(x))
            layers[-1].is_clamped = False
            if self.config.use_feedforward_gist_init:
                self._ffg(layers)
            out = []
            for _ in range(steps):
                self._relax_step(layers)
                out.append(self._energy(layers))
            return out

    def _settle_adaptive(self, layers, max_steps: int, epsilon: float) -> Tuple[int, float]:
        previous = float("inf")
        energy = 0.0
        step = 0
        while step < max_steps:
            self._relax_step(layers)
            step += 1
            energy = self._energy(layers)
            if epsilon > 0 and previous != float("inf") and previous - energy < epsilon * max(previous, 1e-12):
                break
            previous = energy
        return step, energy

    def infer_adaptive(self, x, max_steps: int = 30, epsilon: float = 1e-4, effort: Optional[str] = None):
        """Energy-based early exit (Network.cs:760-800); returns (top, steps_used, energy)."""
        if effort is not None:
            max_steps, epsilon = EFFORT_PRESETS[effort]
        if max_steps < 1:
            raise ValueError("max_steps must be >= 1.")
        with self._lock:
            layers = self._read_all()
            for L in layers[1:]:
                L.mu = torch.zeros_like(L.mu)
            self._clamp(layers, 0, self._flatten(x))
            layers[-1].is_clamped = False
            if self.config.use_feedforward_gist_init:
                self._ffg(layers)
            steps, energy = self._settle_adaptive(layers, max_steps, epsilon)
            return layers[-1].mu.clone(), steps, energy

    # ------------------------------------------------------------ learning
    def learn(self, x, label, steps: int, mixed: bool = False, gate: float = 1.0) -> float:
        """Clamp both ends, settle, Hebbian update, persist (Network.cs:139-232).  Returns the energy."""
        with self._lock:
            layers = self._read_all()
            if mixed:
                for L in layers[1:]:
                    L.quantize_weights(force=True)
            self._infer_core(layers, x, steps, True, label)
            energy = self._energy(layers)
            if gate > 0:
                self._update_weights(layers, self.config.weight_lr * gate)
                self._after_learn(layers, gate)
            return energy

    def learn_gated(self, x, label, steps: int, gate: float) -> float:
        """MoE expert learning scaled by its gate; gate == 0 is a pure energy probe (Network.cs:200-232)."""
        return self.learn(x, label, steps, gate=gate)

    def learn_unsupervised(self, x, steps: int) -> None:
        with self._lock:
            layers = self._read_all()
            self._infer_core(layers, x, steps, False, None)
            for l in range(1, len(layers)):
                layers[l].update_weights(layers[l - 1].eps, self.config.weight_lr)
                self._store.write(l, layers[l])

    # ------------------------------------------------------------ prediction
    def class_energies(self, x, steps: int, mixed: bool = False) -> List[float]:
        with self._lock:
            layers = self._read_all()
            if mixed:
                for L in layers[1:]:
                    L.quantize_weights()
            n = layers[-1].size
            out = []
            flat = self._flatten(x)
            for c in range(n):
                for L in layers[1:-1]:
                    L.mu = torch.zeros_like(L.mu)
                lab = torch.zeros(n)
                lab[c] = 1.0
                self._infer_core(layers, flat, steps, True, lab)
                out.append(self._energy(layers))
            return out

    def predict_with_energy(self, x, steps: int, mixed: bool = False) -> Tuple[int, float]:
        """argmin_c F(x, onehot(c)), winner re-run and persisted (Network.cs:369-435)."""
        with self._lock:
            layers = self._read_all()
            if mixed:
                for L in layers[1:]:
                    L.quantize_weights()
            n = layers[-1].size
            flat = self._flatten(x)
            best_e, best_c = float("inf"), 0
            for c in range(n):
                for L in layers[1:-1]:
                    L.mu = torch.zeros_like(L.mu)
                lab = torch.zeros(n)
                lab[c] = 1.0
                self._infer_core(layers, flat, steps, True, lab)
                e = self._energy(layers)
                if e < best_e:
                    best_e, best_c = e, c
            for L in layers[1:-1]:
                L.mu = torch.zeros_like(L.mu)
            lab = torch.zeros(n)
            lab[best_c] = 1.0
            self._infer_core(layers, flat, steps, True, lab)
            winner = self._energy(layers)
            for L in layers:
                L.W_half = None
            self._write_back(layers, range(len(layers)))
            return best_c, winner

    def predict(self, x, steps: int, mixed: bool = False) -> int:
        return self.predict_with_energy(x, steps, mixed)[0]

    def predict_adaptive(self, x, max_steps: int = 30, epsilon: float = 1e-4,
                         effort: Optional[str] = None) -> Tuple[int, float, int]:
        """Adaptive settling per candidate (Network.cs:802-860); returns (class, energy, total steps)."""
        if effort is not None:
            max_steps, epsilon = EFFORT_PRESETS[effort]
        with self._lock:
            layers = self._read_all()
            n = layers[-1].size
            flat = self._flatten(x)

            def settle(c):
                for L in layers[1:-1]:
                    L.mu = torch.zeros_like(L.mu)
                lab = torch.zeros(n)
                lab[c] = 1.0
                self._clamp(layers, 0, flat)
                self._clamp(layers, len(layers) - 1, lab)
                if self.config.use_feedforward_gist_init:
                    self._ffg(layers)
                return self._settle_adaptive(layers, max_steps, epsilon)

            best_e, best_c, total = float("inf"), 0, 0
            for c in range(n):
                s, e = settle(c)
                total += s
                if e < best_e:
                    best_e, best_c = e, c
            s, winner = settle(best_c)
            total += s
            self._write_back(layers, range(len(layers)))
            return best_c, winner, total

    # ------------------------------------------------------------ temporal
    def _inject_temporal(self, layers, priors, precision) -> None:
        hidden = len(layers) - 2
        if len(priors) != hidden:
            raise ValueError(f"Expected {hidden} temporal prior(s) (one per hidden layer) but got {len(priors)}.")
        for i in range(hidden):
            layers[i + 1].temporal_prior = torch.as_tensor(priors[i]).float().clone()
            layers[i + 1].temporal_precision = precision

    @staticmethod
    def _hidden_states(layers) -> List[torch.Tensor]:
        return [layers[i + 1].mu.clone() for i in range(len(layers) - 2)]

    def learn_temporal(self, x, label, steps, priors=None, precision: float = 1.0) -> List[torch.Tensor]:
        with self._lock:
            layers = self._read_all()
            if priors is not None:
                self._inject_temporal(layers, priors, precision)
            self._infer_core(layers, x, steps, True, label)
            for l in range(1, len(layers)):
                layers[l].update_weights(layers[l - 1].eps, self.config.weight_lr)
                self._store.write(l, layers[l])
            return self._hidden_states(layers)

    def infer_temporal(self, x, steps, priors=None, precision: float = 1.0, clamp_top=False, label=None):
        with self._lock:
            layers = self._read_all()
            if priors is not None:
                self._inject_temporal(layers, priors, precision)
            self._infer_core(layers, x, steps, clamp_top, label)
            return self._hidden_states(layers)

    def predict_temporal(self, x, steps, priors=None, precision: float = 1.0) -> int:
        with self._lock:
            layers = self._read_all()
            n = layers[-1].size
            flat = self._flatten(x)
            best_e, best_c = float("inf"), 0
            for c in range(n):
                for L in layers[1:-1]:
                    L.mu = torch.zeros_like(L.mu)
                if priors is not None:
                    self._inject_temporal(layers, priors, precision)
                lab = torch.zeros(n)
                lab[c] = 1.0
                self._infer_core(layers, flat, steps, True, lab)
                e = self._energy(layers)
                if e < best_e:
                    best_e, best_c = e, c
            for L in layers[1:-1]:
                L.mu = torch.zeros_like(L.mu)
            if priors is not None:
                self._inject_temporal(layers, priors, precision)
            lab = torch.zeros(n)
            lab[best_c] = 1.0
            self._infer_core(layers, flat, steps, True, lab)
            self._write_back(layers, range(len(layers)))
            return best_c

    def infer_energy_temporal(self, x, label, steps, priors=None, precision: float = 1.0) -> float:
        with self._lock:
            layers = self._read_all()
            if priors is not None:
                self._inject_temporal(layers, priors, precision)
            self._infer_core(layers, x, steps, True, label)
            return self._energy(layers)

    def learn_temporal_gated(self, x, label, steps, priors=None, precision: float = 1.0, gate: float = 1.0):
        """Temporal learning with the weight lr scaled by ``gate``; returns (hidden states, energy)."""
        with self._lock:
            layers = self._read_all()
            if priors is not None:
                self._inject_temporal(layers, priors, precision)
            self._infer_core(layers, x, steps, True, label)
            energy = self._energy(layers)
            if gate > 0:
                for l in range(1, len(layers)):
                    layers[l].update_weights(layers[l - 1].eps, self.config.weight_lr * gate)
                    self._store.write(l, layers[l])
            return self._hidden_states(layers), energy

    def predict_with_energy_temporal(self, x, steps, priors=None, precision: float = 1.0):
        with self._lock:
            layers = self._read_all()
            n = layers[-1].size
            flat = self._flatten(x)
            best_e, best_c = float("inf"), 0
            for c in range(n):
                for L in layers[1:-1]:
                    L.mu = torch.zeros_like(L.mu)
                if priors is not None:
                    self._inject_temporal(layers, priors, precision)
                lab = torch.zeros(n)
                lab[c] = 1.0
                self._infer_core(layers, flat, steps, True, lab)
                e = self._energy(layers)
                if e < best_e:
                    best_e, best_c = e, c
            for L in layers[1:-1]:
                L.mu = torch.zeros_like(L.mu)
            if priors is not None:
                self._inject_temporal(layers, priors, precision)
            lab = torch.zeros(n)
            lab[best_c] = 1.0
            self._infer_core(layers, flat, steps, True, lab)
            winner = self._energy(layers)
            self._write_back(layers, range(len(layers)))
            return best_c, winner

    def learn_unsupervised_temporal(self, x, steps, priors=None, precision: float = 1.0):
        with self._lock:
            layers = self._read_all()
            if priors is not None:
                self._inject_temporal(layers, priors, precision)
            self._infer_core(layers, x, steps, False, None)
            for l in range(1, len(layers)):
                layers[l].update_weights(layers[l - 1].eps, self.config.weight_lr)
                self._store.write(l, layers[l])
            return layers[-1].mu.clone(), self._hidden_states(layers)

    def infer_get_top_temporal(self, x, steps, priors=None, precision: float = 1.0):
        with self._lock:
            layers = self._read_all()
            if priors is not None:
                self._inject_temporal(layers, priors, precision)
            self._infer_core(layers, x, steps, False, None)
            return layers[-1].mu.clone(), self._hidden_states(layers)

    # ------------------------------------------------------------ generation / priors
    def generate(self, latent, steps: int) -> torch.Tensor:
        """Clamp the top to ``latent``, settle the free input layer from zero (Network.cs:1181-1222)."""
        latent = torch.as_tensor(latent, dtype=torch.float32).reshape(-1)
        if latent.numel() != self.config.layer_sizes[-1]:
            raise ValueError(f"Latent vector has {latent.numel()} elements; top layer expects "
                             f"{self.config.layer_sizes[-1]}.")
        with self._lock:
            layers = self._read_all()
            self._clamp(layers, len(layers) - 1, latent)
            layers[0].mu = torch.zeros_like(layers[0].mu)
            layers[0].is_clamped = False
            eta, lam = self.config.state_lr, self.config.activity_regularization
            for _ in range(steps):
                for l in range(len(layers) - 1, 0, -1):
                    layers[l].compute_prediction()
                for l in range(1, len(layers)):
                    layers[l - 1].set_prediction_error(layers[l].pred)
                layers[-1].set_prediction_error(None)
                for l in range(1, len(layers) - 1):
                    if not layers[l].is_clamped:
                        layers[l].update_state(layers[l - 1].eps, eta, lam)
                if not layers[0].is_clamped:
                    layers[0].mu = layers[0].mu - eta * layers[0].eps
            return layers[0].mu.clone()

    def set_top_layer_prior(self, prior, precision: float = 1.0) -> None:
        with self._lock:
            top = self._store.read(self.layer_count - 1)
            top.prior_mean = None if prior is None else torch.as_tensor(prior).float().clone()
            top.precision = precision
            self._store.write(self.layer_count - 1, top)

    # ------------------------------------------------------------ energy / diagnostics
    def compute_energy(self) -> float:
        with self._lock:
            return sum(self._store.read(l).local_energy() for l in range(self.layer_count - 1))

    def compute_layer_energies(self) -> List[float]:
        with self._lock:
            return [self._store.read(l).local_energy() for l in range(self.layer_count - 1)]

    def average_weight_norm(self) -> float:
        with self._lock:
            if self.layer_count < 2:
                return 0.0
            return sum(self._store.read(l).weight_norm() for l in range(1, self.layer_count)) / (self.layer_count - 1)

    def layer(self, i: int) -> Layer:
        """A copy of stored layer ``i``."""
        return self._store.read(i)

    def update_precisions(self, eta: float) -> None:
        """Precision learning on every stored layer (scalar or diagonal)."""
        with self._lock:
            for l in range(self.layer_count):
                L = self._store.read(l)
                if L.diag_precision is not None:
                    L.update_diagonal_precision(eta)
                else:
                    L.update_precision(eta)
                self._store.write(l, L)

    # ------------------------------------------------------------ persistence / export
    def flush_store(self) -> None:
        with self._lock:
            self._store.flush()

    def persist_weights_quantized(self, precision: str = "half") -> None:
        with self._lock:
            for l in range(self.layer_count):
                self._store.write_quantized(l, self._store.read(l), precision)

    def persist_weights_as_half(self) -> None:
        self.persist_weights_quantized("half")

    def export_generative_snapshot(self) -> GenerativeSnapshot:
        """Export for the batched engine; diagonal precision / priors are rejected (Network.cs:1328-1358)."""
        with self._lock:
            layers = self._read_all()
            for L in layers:
                if L.diag_precision is not None or L.prior_mean is not None:
                    raise NotImplementedError("export_generative_snapshot does not support diagonal precision or "
                                              "informative priors.")
            return GenerativeSnapshot(list(self.config.layer_sizes), self.config.activation, self.config.state_lr,
                                      self.config.activity_regularization, self.config.use_feedforward_gist_init,
                                      [L.W.clone() for L in layers[1:]], [L.b.clone() for L in layers[1:]],
                                      [L.precision for L in layers])

    def import_weights(self, weights: Sequence[torch.Tensor], biases: Sequence[torch.Tensor]) -> None:
        """Overwrite W_l / b_l (l = 1..L-1), e.g. after batched training on the GPU."""
        with self._lock:
            for l in range(1, self.layer_count):
                L = self._store.read(l)
                L.W = weights[l - 1].detach().float().cpu().clone()
                L.b = biases[l - 1].detach().float().cpu().clone()
                self._store.write(l, L)

    def close(self) -> None:
        self._store.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
