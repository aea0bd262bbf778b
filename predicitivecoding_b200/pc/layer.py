"""One predictive-coding layer and the activation functions it uses.

Reference: PredicitiveCoding/Model/Layer.cs:34-465 and Core/Activation.cs:19-150.

Layer ``l`` holds its state ``mu`` (size ``size``), its precision-weighted
prediction error ``eps``, and — for ``l >= 1`` — the generative weights
``W [lower, size]`` and bias ``b [lower]`` with which it predicts the layer
below: ``pred = f(W mu + b)``.

One deliberate difference: the reference never writes ``PreActivation`` in
``ComputePrediction`` (Layer.cs:212-220), so its ReLU derivative, which reads the
pre-activation, is always 0.  Here the pre-activation is stored and the ReLU
derivative is the true one; tanh / sigmoid / linear (whose derivatives use the
activation output) are unaffected.  ``reference_relu_quirk=True`` restores the
reference behaviour exactly.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import torch

ACTIVATIONS = ("linear", "tanh", "relu", "sigmoid")


def activate(x: torch.Tensor, kind: str) -> torch.Tensor:
    if kind == "tanh":
        return torch.tanh(x)
    if kind == "relu":
        return torch.relu(x)
    if kind == "sigmoid":
        return torch.sigmoid(x)
    if kind == "linear":
        return x.clone()
    raise ValueError(f"unknown activation {kind!r}")


def derivative(pre: torch.Tensor, act: Optional[torch.Tensor], kind: str) -> torch.Tensor:
    """f'(x) as the reference computes it: from y for tanh (1-y^2) and sigmoid (y(1-y))."""
    if kind == "linear":
        return torch.ones_like(pre)
    if kind == "tanh":
        y = act if act is not None else torch.tanh(pre)
        return 1.0 - y * y
    if kind == "relu":
        return (pre > 0).to(pre.dtype)
    if kind == "sigmoid":
        y = act if act is not None else torch.sigmoid(pre)
        return y * (1.0 - y)
    raise ValueError(f"unknown activation {kind!r}")


def softmax(x: torch.Tensor) -> torch.Tensor:
    return torch.softmax(x, dim=-1)


def init_weights(fan_in: int, fan_out: int, kind: str, gen: torch.Generator) -> torch.Tensor:
    """[fan_out, fan_in]: He for ReLU, Xavier-uniform for linear, Xavier-normal otherwise
    (Core/RandomUtils.cs:60-99)."""
    if kind == "relu":
        return torch.randn(fan_out, fan_in, generator=gen) * math.sqrt(2.0 / fan_in)
    if kind == "linear":
        a = math.sqrt(6.0 / (fan_in + fan_out))
        return (torch.rand(fan_out, fan_in, generator=gen) * 2 - 1) * a
    return torch.randn(fan_out, fan_in, generator=gen) * math.sqrt(2.0 / (fan_in + fan_out))


@dataclass
class Layer:
    index: int
    size: int
    lower_size: int
    activation: str = "tanh"
    state_lr: float = 0.1
    weight_lr: float = 1e-3
    weight_decay: float = 0.0
    precision: float = 1.0
    is_clamped: bool = False
    mu: torch.Tensor = None
    eps: torch.Tensor = None
    W: Optional[torch.Tensor] = None
    b: Optional[torch.Tensor] = None
    pre: Optional[torch.Tensor] = None
    pred: Optional[torch.Tensor] = None
    diag_precision: Optional[torch.Tensor] = None
    prior_mean: Optional[torch.Tensor] = None
    temporal_prior: Optional[torch.Tensor] = None
    temporal_precision: float = 0.0
    W_half: Optional[torch.Tensor] = None  # transient low-precision copy (mixed precision)
    reference_relu_quirk: bool = False

    # ------------------------------------------------------------ construction
    @staticmethod
    def create(index: int, size: int, lower_size: int, activation: str, gen: torch.Generator,
               **kw) -> "Layer":
        """Layer.Initialize (Layer.cs:167-178): mu ~ N(0, 0.01^2), W by fan-based init, b = 0."""
        L = Layer(index, size, lower_size, activation, **kw)
        L.mu = torch.randn(size, generator=gen) * 0.01
        L.eps = torch.zeros(size)
        if lower_size > 0:
            L.W = init_weights(size, lower_size, activation, gen)
            L.b = torch.zeros(lower_size)
            L.pre = torch.zeros(lower_size)
            L.pred = torch.zeros(lower_size)
        return L

    def init_diagonal_precision(self) -> None:
        self.diag_precision = torch.ones(self.size)

    def quantize_weights(self, dtype=torch.float16, force: bool = False) -> None:
        """Transient Half/bf16 copy of W used by the mixed-precision forward (Layer.cs:197-201)."""
        if self.W is None:
            self.W_half = None
            return
        if force or self.W_half is None:
            self.W_half = self.W.to(dtype)

    def clone(self) -> "Layer":
        c = Layer(self.index, self.size, self.lower_size, self.activation, self.state_lr, self.weight_lr,
                  self.weight_decay, self.precision, self.is_clamped)
        for name in ("mu", "eps", "W", "b", "pre", "pred", "diag_precision", "prior_mean", "temporal_prior",
                     "W_half"):
            v = getattr(self, name)
            setattr(c, name, None if v is None else v.clone())
        c.temporal_precision = self.temporal_precision
        c.reference_relu_quirk = self.reference_relu_quirk
        return c

    # ------------------------------------------------------------ dynamics
    def compute_prediction(self) -> None:
        """pred = f(W mu + b)  (Layer.cs:212-220)."""
        if self.W is None:
            return
        if self.W_half is not None:
            pre = (self.W_half.float() @ self.mu.to(self.W_half.dtype).float())
        else:
            pre = self.W @ self.mu
        pre = pre + self.b
        if not self.reference_relu_quirk:
            self.pre = pre
        self.pred = activate(pre, self.activation)

    def set_prediction_error(self, pred_from_above: Optional[torch.Tensor]) -> None:
        """eps = Pi (mu - pred_above);  top layer: Pi (mu - prior) or 0 (Layer.cs:234-262)."""
        if pred_from_above is None:
            if self.prior_mean is None:
                self.eps = torch.zeros_like(self.mu)
                return
            residual = self.mu - self.prior_mean
        else:
            residual = self.mu - pred_from_above
        if self.diag_precision is not None:
            self.eps = residual * self.diag_precision
        elif self.precision == 1.0:
            self.eps = residual.clone()
        else:
            self.eps = residual * self.precision

    def update_state(self, lower_error: Optional[torch.Tensor], eta: float, activity_reg: float = 0.0) -> None:
        """mu -= eta (eps - W^T (f'(pre) * eps_below) + lambda sign(mu) + Pi_t (mu - mu_prev))  (Layer.cs:273-309)."""
        if self.is_clamped or self.W is None:
            return
        if lower_error is not None:
            delta = derivative(self.pre, self.pred, self.activation) * lower_error
            if self.W_half is not None:
                wt = self.W_half.float().T @ delta.to(self.W_half.dtype).float()
            else:
                wt = self.W.T @ delta
            grad = self.eps - wt
        else:
            grad = self.eps.clone()
        if activity_reg > 0:
            grad = grad + activity_reg * torch.sign(self.mu)
        if self.temporal_precision > 0 and self.temporal_prior is not None:
            grad = grad + self.temporal_precision * (self.mu - self.temporal_prior)
        self.mu = self.mu - eta * grad

    def update_weights(self, lower_error: Optional[torch.Tensor], eta_w: float) -> None:
        """W += eta (f'(pre) * eps_below) (x) mu;  b += eta delta;  W -= eta*lambda*W  (Layer.cs:320-333)."""
        if self.W is None or lower_error is None:
            return
        delta = derivative(self.pre, self.pred, self.activation) * lower_error
        self.W = self.W + eta_w * torch.outer(delta, self.mu)
        self.b = self.b + eta_w * delta
        if self.weight_decay > 0:
            self.W = self.W - eta_w * self.weight_decay * self.W

    def update_precision(self, eta: float) -> None:
        """Gradient step on scalar precision with the log-normaliser (Layer.cs:340-347)."""
        ss = float((self.eps * self.eps).sum()) / (self.precision * self.precision)
        grad = 0.5 * ss - 0.5 * self.size / self.precision
        self.precision = max(1e-6, self.precision - eta * grad)

    def update_diagonal_precision(self, eta: float) -> None:
        """Per-unit precision update (Huang & Rao 2011; Layer.cs:352-366)."""
        if self.diag_precision is None:
            raise RuntimeError("Call init_diagonal_precision() before update_diagonal_precision().")
        pi = self.diag_precision
        r2 = torch.where(pi > 0, (self.eps / pi) ** 2, torch.zeros_like(pi))
        grad = 0.5 * r2 - 0.5 / pi
        self.diag_precision = torch.clamp(pi - eta * grad, min=1e-6)

    # ------------------------------------------------------------ diagnostics
    def weight_norm(self) -> float:
        return 0.0 if self.W is None else float(torch.sqrt((self.W * self.W).sum()))

    def local_energy(self) -> float:
        """1/2 ||eps||^2 / Pi (or per-unit Pi) (Layer.cs:437-450)."""
        if self.diag_precision is not None:
            pi = self.diag_precision
            return 0.5 * float(torch.where(pi > 0, self.eps * self.eps / pi, torch.zeros_like(pi)).sum())
        return 0.5 * float((self.eps * self.eps).sum()) / self.precision

    def __repr__(self) -> str:
        s = f"PCLayer[{self.index}] Size={self.size}"
        s += f" LowerSize={self.lower_size}" if self.lower_size > 0 else " (input)"
        s += f" Act={self.activation}"
        if self.diag_precision is not None:
            s += " [diag-Pi]"
        elif self.precision != 1.0:
            s += f" Pi={self.precision:.3f}"
        if self.is_clamped:
            s += " [CLAMPED]"
        return s
