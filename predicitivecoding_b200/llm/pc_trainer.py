"""Incremental predictive coding (iPC) for the decoder: block-boundary latents learn locally.

Reference: PredictiveCoding.LLM/Training/PcDecoderTrainer.cs:29-192.  Latents mu_b live
between blocks (mu_0 = the embedding, mu_b warm-started by the feed-forward pass); a light
relaxation ``mu_b -= eta (eps_b + topdown_b)`` with eps_b = mu_b - f_b(mu_{b-1}) and topdown_b
the VJP of the block above (or of the cross-entropy at the top), both clipped; then each
block learns from its own error only, ``theta_b += lr * VJP_{f_b}(eps_b)`` (clipped per
tensor, non-finite entries zeroed); embedding / output head / final norm follow the CE
gradient; every ``anchor_every`` steps a short burst of backprop + fresh Adam re-centres the
weights on the true loss.  Gradients are zeroed before every VJP here (the reference lets
relaxation-phase gradients leak into the weight update through its accumulating autograd).
"""
from __future__ import annotations

from typing import List

import torch

from ..models.decoder_lm import DecoderLM, cross_entropy_masked, rms_norm
from ..optim.adam import Adam
from .trainer import step as adam_step

DEFAULT_ANCHOR_EVERY = 2048


def _clip_(v: torch.Tensor, max_norm: float) -> torch.Tensor:
    v.nan_to_num_(nan=0.0, posinf=0.0, neginf=0.0)
    n = float(v.norm())
    if n > max_norm and n > 0:
        v.mul_(max_norm / n)
    return v


class PcDecoderTrainer:
    def __init__(self, model: DecoderLM, relax_steps: int = 1, eta_state: float = 0.1, lr_weights: float = 0.3,
                 clip_norm: float = 1.0, anchor_every: int = DEFAULT_ANCHOR_EVERY, anchor_burst: int = 3,
                 anchor_lr: float = 0.01):
        c = model.cfg
        if c.num_loops != 1 or c.num_experts != 0 or c.mtp_weight != 0 or c.use_plan or c.block_pattern is not None:
            raise NotImplementedError("PcDecoderTrainer needs a plain dense preset (no loops/MoE/MTP/plan).")
        if not c.use_rope or not c.use_rms_norm:
            raise NotImplementedError("PcDecoderTrainer assumes RMSNorm + RoPE.")
        self.m = model
        self.relax_steps, self.eta_state, self.lr_weights, self.clip_norm = relax_steps, eta_state, lr_weights, clip_norm
        self.anchor_every, self.anchor_burst, self.anchor_lr = anchor_every, anchor_burst, anchor_lr
        self.steps = 0

    def _f(self, x, b):
        m = self.m
        from ..models.decoder_lm import rope_tables
        S = x.shape[1]
        rope = rope_tables(S, m.cfg.head_dim, 0, device=x.device)
        return m.blocks[b](x, m.attn_scale, rope, False)

    def _zero(self):
        for p in self.m.parameters():
            p.grad = None

    def step(self, tokens, targets) -> float:
        m = self.m
        dev = m.wemb.device
        t = torch.as_tensor(tokens, device=dev).long().view(1, -1)
        y = torch.as_tensor(targets, device=dev).long().view(1, -1)
        B = len(m.blocks)
        with torch.no_grad():
            mu = [m.wemb[t].clone()]
            for b in range(B):
                mu.append(self._f(mu[b], b).clone())
        for _ in range(self.relax_steps):
            for b in range(1, B + 1):
                with torch.no_grad():
                    eps = mu[b] - self._f(mu[b - 1], b - 1)
                hc = mu[b].clone().requires_grad_(True)
                self._zero()
                if b < B:
                    f = self._f(hc, b)
                    f.backward((mu[b + 1] - f).detach())
                else:
                    loss = cross_entropy_masked(rms_norm(hc, m.lnf_g, m.cfg.eps) @ m.wout, y, -1)
                    loss.backward()
                with torch.no_grad():
                    stp = _clip_(eps + hc.grad, self.clip_norm)
                    mu[b] = mu[b] - self.eta_state * stp
        for b in range(1, B + 1):
            self._zero()
            f = self._f(mu[b - 1], b - 1)
            f.backward((mu[b] - f).detach())
            with torch.no_grad():
                for p in m.blocks[b - 1].parameters():
                    if p.grad is not None:
                        p.add_(self.lr_weights * _clip_(p.grad, self.clip_norm))
        self._zero()
        ce = m.loss(t, y)
        ce.backward()
        with torch.no_grad():
            for p in (m.wemb, m.wout, m.lnf_g):
                if p.grad is not None:
                    p.sub_(self.lr_weights * _clip_(p.grad, self.clip_norm))
        self._zero()
        self.steps += 1
        if self.anchor_every > 0 and self.steps % self.anchor_every == 0:
            self.anchor(tokens, targets)
        return float(ce)

    def anchor(self, tokens, targets) -> None:
        opt = Adam()
        ps = list(self.m.parameters())
        for _ in range(self.anchor_burst):
            adam_step(ps, [(tokens, targets)], lambda a, b, tr: self.m.loss(a.view(1, -1), b.view(1, -1), -1, tr),
                      opt, self.anchor_lr, clip_norm=1.0)
