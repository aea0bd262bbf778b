"""Optimizers and schedules with the reference's exact update order.

Reference: PredictiveCoding.LLM/Training/Optimizers.cs:12-116 (Adam/AdamW with per-tensor
moments, decoupled decay applied after the Adam step on the updated weight, moment
get/set for checkpointing; global-norm clipping that zeroes non-finite gradients) and
LrSchedule.cs:9-27 (linear warmup (step+1)/W, then cosine to MinLr).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import torch


class Adam:
    """Adam/AdamW over a list of tensors; moments keyed by tensor identity."""

    def __init__(self, beta1: float = 0.9, beta2: float = 0.999, eps: float = 1e-8, weight_decay: float = 0.0):
        self.beta1, self.beta2, self.eps, self.weight_decay = beta1, beta2, eps, weight_decay
        self.t = 0
        self._m: Dict[int, torch.Tensor] = {}
        self._v: Dict[int, torch.Tensor] = {}

    @property
    def step_count(self) -> int:
        return self.t

    @torch.no_grad()
    def step(self, params: Sequence[torch.Tensor], lr: float) -> None:
        """w -= lr * mhat / (sqrt(vhat) + eps); then w -= lr * wd * w (reference order)."""
        self.t += 1
        bc1 = 1.0 - self.beta1 ** self.t
        bc2 = 1.0 - self.beta2 ** self.t
        for p in params:
            if p.grad is None:
                continue
            g = p.grad
            m = self._m.get(id(p))
            if m is None:
                m = self._m[id(p)] = torch.zeros_like(p)
                self._v[id(p)] = torch.zeros_like(p)
            v = self._v[id(p)]
            m.mul_(self.beta1).add_(g, alpha=1 - self.beta1)
            v.mul_(self.beta2).addcmul_(g, g, value=1 - self.beta2)
            p.sub_(lr * (m / bc1) / ((v / bc2).sqrt() + self.eps))
            if self.weight_decay > 0:
                p.sub_(lr * self.weight_decay * p)

    def moments_for(self, p: torch.Tensor) -> Optional[Tuple[torch.Tensor, torch.Tensor]]:
        m = self._m.get(id(p))
        return None if m is None else (m, self._v[id(p)])

    def set_moments(self, p: torch.Tensor, m: torch.Tensor, v: torch.Tensor) -> None:
        self._m[id(p)] = m.to(p.device, p.dtype).clone()
        self._v[id(p)] = v.to(p.device, p.dtype).clone()

    def restore_step_count(self, t: int) -> None:
        self.t = int(t)


@torch.no_grad()
def clip_global_norm(params: Iterable[torch.Tensor], max_norm: float) -> float:
    """Zero non-finite gradient entries, then scale so the global L2 norm <= max_norm; returns the norm."""
    grads = [p.grad for p in params if p.grad is not None]
    total = 0.0
    for g in grads:
        g.nan_to_num_(nan=0.0, posinf=0.0, neginf=0.0)
        total += float((g.float() * g.float()).sum())
    norm = math.sqrt(total)
    if max_norm > 0 and norm > max_norm:
        s = max_norm / norm
        for g in grads:
            g.mul_(s)
    return norm


@dataclass
class LrSchedule:
    peak_lr: float = 3e-4
    min_lr: float = 0.0
    warmup_steps: int = 100
    total_steps: int = 1000

    def at(self, step: int) -> float:
        if step < self.warmup_steps:
            return self.peak_lr * (step + 1) / max(1, self.warmup_steps)
        if step >= self.total_steps:
            return self.min_lr
        progress = (step - self.warmup_steps) / max(1, self.total_steps - self.warmup_steps)
        return self.min_lr + 0.5 * (self.peak_lr - self.min_lr) * (1.0 + math.cos(math.pi * progress))
