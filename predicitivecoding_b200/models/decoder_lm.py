"""Trainable decoder LM (PyTorch autograd path).

Reference: PredictiveCoding.LLM/Autograd/DecoderLM.cs:132-753.  Every mechanism of
the reference model is here: pre-norm attention blocks (LayerNorm or RMSNorm,
sinusoidal positions or RoPE), dense GELU FFN with biases, sparse top-k MoE FFN
with the Switch balance loss, gated-recurrence 'T' blocks, weight-tied loops with
an early exit at inference, a multi-token-prediction head and a latent plan.

This module is the CPU oracle and the generic GPU path (any config).  The dense
RMSNorm+RoPE family additionally runs on :class:`FusedDecoderTrainer`, which
executes the same maths with hand-written sm_100a kernels.

Weight layout: matrices are stored the reference's way, ``[in, out]`` so that
``y = x @ W`` (DecoderLM.cs:465-473).  Heads are packed: ``wq[:, h*hd:(h+1)*hd]``
is the reference's ``_wq[h]`` and ``wo[h*hd:(h+1)*hd, :]`` is ``_wo[h]``;
:meth:`DecoderLM.reference_parameters` unpacks them in the reference's
``Parameters()`` order (the checkpoint contract, DecoderLM.cs:182-193, 497-517).
"""
from __future__ import annotations

import math
from typing import List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .config import DecoderLmConfig

GELU_C = 0.7978845608
GELU_A = 0.044715


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    """tanh-approximation GELU with the reference constants (Autograd.cs:303-328)."""
    return 0.5 * x * (1.0 + torch.tanh(GELU_C * (x + GELU_A * x * x * x)))


def rms_norm(x: torch.Tensor, g: torch.Tensor, eps: float) -> torch.Tensor:
    """y = x * g / sqrt(mean(x^2) + eps)  (Autograd.cs:435-472)."""
    inv = torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return x * inv * g


def layer_norm(x: torch.Tensor, g: torch.Tensor, b: torch.Tensor, eps: float) -> torch.Tensor:
    """Biased-variance layer norm (Autograd.cs:382-433)."""
    mean = x.mean(-1, keepdim=True)
    var = (x - mean).pow(2).mean(-1, keepdim=True)
    return (x - mean) * torch.rsqrt(var + eps) * g + b


def rope_tables(seq: int, head_dim: int, base_pos: int = 0, device=None, dtype=torch.float32):
    """cos/sin [seq, hd/2] with freq_i = 10000^(-2i/hd), angle = (base_pos + row) * freq_i."""
    half = head_dim // 2
    i = torch.arange(half, dtype=torch.float64)
    freq = 1.0 / torch.pow(10000.0, 2.0 * i / head_dim)
    pos = torch.arange(base_pos, base_pos + seq, dtype=torch.float64)
    ang = pos[:, None] * freq[None, :]
    return torch.cos(ang).to(device=device, dtype=dtype), torch.sin(ang).to(device=device, dtype=dtype)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate interleaved pairs (2i, 2i+1) of the last dim (Autograd.cs:475-508).  x: [..., S, hd]."""
    x0 = x[..., 0::2]
    x1 = x[..., 1::2]
    o0 = x0 * cos - x1 * sin
    o1 = x0 * sin + x1 * cos
    return torch.stack((o0, o1), dim=-1).flatten(-2)


def sinusoidal_positions(seq: int, dim: int, device=None) -> torch.Tensor:
    """Sinusoidal positional encoding of the non-RoPE path (Autograd/AgPositional.cs:13-32)."""
    pos = torch.arange(seq, dtype=torch.float64)[:, None]
    i = torch.arange(dim, dtype=torch.float64)[None, :]
    angle = pos / torch.pow(10000.0, (2 * torch.div(i, 2, rounding_mode="floor")) / dim)
    pe = torch.where((i % 2) == 0, torch.sin(angle), torch.cos(angle))
    return pe.to(device=device, dtype=torch.float32)


def _randn(gen: torch.Generator, *shape) -> torch.Tensor:
    # 0.02 * N(0, 1) (AgInit.Randn, DecoderLM.cs:712-752); seeded torch generator, not .NET's Random
    return torch.randn(*shape, generator=gen) * 0.02


class AttentionBlock(nn.Module):
    """Pre-norm attention block + dense or MoE FFN (DecoderLM.cs:445-615)."""

    def __init__(self, cfg: DecoderLmConfig, gen: torch.Generator):
        super().__init__()
        D, F_ = cfg.dim, cfg.ff_dim
        self.cfg = cfg
        self.ln1_g = nn.Parameter(torch.ones(D))
        self.ln1_b = None if cfg.use_rms_norm else nn.Parameter(torch.zeros(D))
        self.wq = nn.Parameter(_randn(gen, D, D))
        self.wk = nn.Parameter(_randn(gen, D, D))
        self.wv = nn.Parameter(_randn(gen, D, D))
        self.wo = nn.Parameter(_randn(gen, D, D))
        self.ln2_g = nn.Parameter(torch.ones(D))
        self.ln2_b = None if cfg.use_rms_norm else nn.Parameter(torch.zeros(D))
        self.router = None
        if cfg.num_experts > 0:
            E = cfg.num_experts
            self.router = nn.Parameter(_randn(gen, D, E))
            self.ew1 = nn.ParameterList([nn.Parameter(_randn(gen, D, F_)) for _ in range(E)])
            self.eb1 = nn.ParameterList([nn.Parameter(torch.zeros(F_)) for _ in range(E)])
            self.ew2 = nn.ParameterList([nn.Parameter(_randn(gen, F_, D)) for _ in range(E)])
            self.eb2 = nn.ParameterList([nn.Parameter(torch.zeros(D)) for _ in range(E)])
        elif cfg.ffn == "gelu":
            self.w1 = nn.Parameter(_randn(gen, D, F_))
            self.b1 = nn.Parameter(torch.zeros(F_))
            self.w2 = nn.Parameter(_randn(gen, F_, D))
            self.b2 = nn.Parameter(torch.zeros(D))
        else:  # swiglu
            self.w1 = nn.Parameter(_randn(gen, D, F_))  # gate
            self.w3 = nn.Parameter(_randn(gen, D, F_))  # up
            self.w2 = nn.Parameter(_randn(gen, F_, D))

    def norm1(self, x):
        c = self.cfg
        return rms_norm(x, self.ln1_g, c.eps) if c.use_rms_norm else layer_norm(x, self.ln1_g, self.ln1_b, c.eps)

    def norm2(self, x):
        c = self.cfg
        return rms_norm(x, self.ln2_g, c.eps) if c.use_rms_norm else layer_norm(x, self.ln2_g, self.ln2_b, c.eps)

    def reference_parameters(self) -> List[torch.Tensor]:
        """Tensors in the reference Block.Parameters() order, per-head matrices unpacked."""
        c = self.cfg
        hd = c.head_dim
        out = [self.ln1_g.view(1, -1)]
        if self.ln1_b is not None:
            out.append(self.ln1_b.view(1, -1))
        for h in range(c.num_heads):
            s = slice(h * hd, (h + 1) * hd)
            out += [self.wq[:, s], self.wk[:, s], self.wv[:, s], self.wo[s, :]]
        out.append(self.ln2_g.view(1, -1))
        if self.ln2_b is not None:
            out.append(self.ln2_b.view(1, -1))
        if self.router is not None:
            out.append(self.router)
            for k in range(c.num_experts):
                out += [self.ew1[k], self.eb1[k].view(1, -1), self.ew2[k], self.eb2[k].view(1, -1)]
        elif c.ffn == "gelu":
            out += [self.w1, self.b1.view(1, -1), self.w2, self.b2.view(1, -1)]
        else:
            out += [self.w1, self.w3, self.w2]
        return out

    def attention(self, h: torch.Tensor, attn_scale: float, rope: Optional[Tuple[torch.Tensor, torch.Tensor]],
                  probe=None, block_index: int = 0) -> torch.Tensor:
        c = self.cfg
        B, S, D = h.shape
        H, hd = c.num_heads, c.head_dim
        q = (h @ self.wq).view(B, S, H, hd).transpose(1, 2)
        k = (h @ self.wk).view(B, S, H, hd).transpose(1, 2)
        v = (h @ self.wv).view(B, S, H, hd).transpose(1, 2)
        if rope is not None:
            q = apply_rope(q, *rope)
            k = apply_rope(k, *rope)
        if probe is None and h.is_cuda:
            o = F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=attn_scale)
        else:
            scores = (q @ k.transpose(-1, -2)) * attn_scale
            mask = torch.ones(S, S, dtype=torch.bool, device=h.device).triu(1)
            probs = torch.softmax(scores.masked_fill(mask, float("-inf")), dim=-1)
            if probe is not None:
                probe.record_causal_attention(block_index, probs.detach())
            o = probs @ v
        o = o.transpose(1, 2).reshape(B, S, D)
        return o @ self.wo

    def dense_ffn(self, h):
        if self.cfg.ffn == "gelu":
            return gelu_tanh(h @ self.w1 + self.b1) @ self.w2 + self.b2
        return (F.silu(h @ self.w1) * (h @ self.w3)) @ self.w2

    def moe_ffn(self, h, aux_losses: Optional[list], probe=None):
        """Top-k gated experts; only routed rows run (DecoderLM.cs:556-615)."""
        c = self.cfg
        B, S, D = h.shape
        x = h.reshape(B * S, D)
        gates = torch.softmax(x @ self.router, dim=-1)  # [rows, E]
        rows, E = gates.shape
        topi = torch.topk(gates.detach(), c.moe_top_k, dim=-1).indices
        mask = torch.zeros_like(gates).scatter_(1, topi, 1.0)
        kept = gates * mask
        out = torch.zeros_like(x)
        for e in range(E):
            routed = torch.nonzero(mask[:, e] > 0, as_tuple=False).flatten()
            if routed.numel() == 0:
                continue
            if probe is not None:
                probe.moe_rows_computed += int(routed.numel())
            sub = x.index_select(0, routed)
            y = gelu_tanh(sub @ self.ew1[e] + self.eb1[e]) @ self.ew2[e] + self.eb2[e]
            y = y * kept.index_select(0, routed)[:, e:e + 1]
            out = out.index_add(0, routed, y)
        if aux_losses is not None:
            frac = mask.sum(0) / (rows * c.moe_top_k)
            bal = (gates.mean(0) * frac).sum() * E
            aux_losses.append(bal)
        return out.view(B, S, D)

    def forward(self, x, attn_scale, rope, training, aux_losses=None, probe=None, block_index=0):
        c = self.cfg
        a = self.attention(self.norm1(x), attn_scale, rope, probe, block_index)
        x = x + F.dropout(a, c.dropout, training)
        h2 = self.norm2(x)
        ff = self.dense_ffn(h2) if self.router is None else self.moe_ffn(h2, aux_losses, probe)
        return x + F.dropout(ff, c.dropout, training)


def recurrent_scan(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """s_t = a_t * s_{t-1} + b_t along the sequence axis (Autograd.cs:741-767).  [B, S, D].

    On a CUDA device the scan runs as one kernel per direction (forward scan, reverse-scan backward).
    """
    if a.is_cuda:
        from .. import ops
        return ops.LinearScan.apply(a, b)
    out = []
    s = torch.zeros_like(b[:, 0])
    for t in range(b.shape[1]):
        s = a[:, t] * s + b[:, t]
        out.append(s)
    return torch.stack(out, dim=1)


class TemporalBlock(nn.Module):
    """Gated diagonal linear recurrence in place of attention (DecoderLM.cs:619-703)."""

    def __init__(self, cfg: DecoderLmConfig, gen: torch.Generator):
        super().__init__()
        D, F_ = cfg.dim, cfg.ff_dim
        self.cfg = cfg
        self.ln1_g = nn.Parameter(torch.ones(D))
        self.ln1_b = nn.Parameter(torch.zeros(D))
        self.wa = nn.Parameter(_randn(gen, D, D)); self.ba = nn.Parameter(torch.zeros(D))
        self.wi = nn.Parameter(_randn(gen, D, D)); self.bi = nn.Parameter(torch.zeros(D))
        self.wu = nn.Parameter(_randn(gen, D, D)); self.bu = nn.Parameter(torch.zeros(D))
        self.wo = nn.Parameter(_randn(gen, D, D)); self.bo = nn.Parameter(torch.zeros(D))
        self.ln2_g = nn.Parameter(torch.ones(D))
        self.ln2_b = nn.Parameter(torch.zeros(D))
        self.w1 = nn.Parameter(_randn(gen, D, F_)); self.b1 = nn.Parameter(torch.zeros(F_))
        self.w2 = nn.Parameter(_randn(gen, F_, D)); self.b2 = nn.Parameter(torch.zeros(D))

    def reference_parameters(self):
        r = lambda t: t.view(1, -1)
        return [r(self.ln1_g), r(self.ln1_b), self.wa, r(self.ba), self.wi, r(self.bi), self.wu, r(self.bu),
                self.wo, r(self.bo), r(self.ln2_g), r(self.ln2_b), self.w1, r(self.b1), self.w2, r(self.b2)]

    def forward(self, x, attn_scale, rope, training, aux_losses=None, probe=None, block_index=0):
        c = self.cfg
        h1 = layer_norm(x, self.ln1_g, self.ln1_b, c.eps)
        a = torch.sigmoid(h1 @ self.wa + self.ba)
        i = torch.sigmoid(h1 @ self.wi + self.bi)
        u = h1 @ self.wu + self.bu
        s = recurrent_scan(a, i * u)
        t = s @ self.wo + self.bo
        x = x + F.dropout(t, c.dropout, training)
        h2 = layer_norm(x, self.ln2_g, self.ln2_b, c.eps)
        ff = gelu_tanh(h2 @ self.w1 + self.b1) @ self.w2 + self.b2
        return x + F.dropout(ff, c.dropout, training)


class DecoderLM(nn.Module):
    """Decoder LM with the reference DecoderLM's mechanisms (DecoderLM.cs:132-420)."""

    def __init__(self, cfg: DecoderLmConfig, seed: int = 42):
        super().__init__()
        cfg.validate()
        self.cfg = cfg
        gen = torch.Generator().manual_seed(seed)
        self.attn_scale = 1.0 / math.sqrt(cfg.head_dim)
        D, V = cfg.dim, cfg.vocab
        self.wemb = nn.Parameter(_randn(gen, V, D))
        blocks = []
        for b in range(cfg.num_blocks):
            if cfg.block_pattern is not None and cfg.block_pattern[b] == "T":
                blocks.append(TemporalBlock(cfg, gen))
            else:
                blocks.append(AttentionBlock(cfg, gen))
        self.blocks = nn.ModuleList(blocks)
        self.loop_bias = (nn.ParameterList([nn.Parameter(torch.zeros(D)) for _ in range(cfg.num_loops)])
                          if cfg.num_loops > 1 else None)
        self.lnf_g = nn.Parameter(torch.ones(D))
        self.lnf_b = None if cfg.use_rms_norm else nn.Parameter(torch.zeros(D))
        self.wout = nn.Parameter(_randn(gen, D, V))
        self.wout_mtp = nn.Parameter(_randn(gen, D, V)) if cfg.mtp_weight > 0 else None
        self.plan = nn.Parameter(torch.zeros(D)) if cfg.use_plan else None
        self.forward_tokens = 0

    # ------------------------------------------------------------ parameter contract
    def reference_parameters(self) -> List[torch.Tensor]:
        """All trainable tensors in the reference Parameters() order (DecoderLM.cs:182-193)."""
        ps = [self.wemb]
        for b in self.blocks:
            ps += b.reference_parameters()
        if self.loop_bias is not None:
            ps += [p.view(1, -1) for p in self.loop_bias]
        ps.append(self.lnf_g.view(1, -1))
        if self.lnf_b is not None:
            ps.append(self.lnf_b.view(1, -1))
        ps.append(self.wout)
        if self.wout_mtp is not None:
            ps.append(self.wout_mtp)
        if self.plan is not None:
            ps.append(self.plan.view(1, -1))
        return ps

    @torch.no_grad()
    def load_reference_parameters(self, tensors) -> None:
        """Overwrite every parameter from tensors given in the reference Parameters() order
        (per-head matrices unpacked), e.g. a legacy LLM1 checkpoint or a FASTER store's tensors."""
        dst = self.reference_parameters()
        if len(tensors) != len(dst):
            raise ValueError(f"expected {len(dst)} tensors in reference order, got {len(tensors)}")
        for i, (d, src) in enumerate(zip(dst, tensors)):
            src = torch.as_tensor(src, dtype=torch.float32)
            if src.numel() != d.numel():
                raise ValueError(f"tensor {i}: shape {tuple(src.shape)} vs model {tuple(d.shape)}")
            d.copy_(src.reshape(d.shape).to(d.device))

    @property
    def parameter_count(self) -> int:
        return sum(p.numel() for p in self.parameters())

    @property
    def active_parameter_count_per_token(self) -> int:
        c = self.cfg
        if c.num_experts == 0:
            return self.parameter_count
        per_expert = c.dim * c.ff_dim + c.ff_dim + c.ff_dim * c.dim + c.dim
        attn_blocks = c.block_pattern.count("A") if c.block_pattern else c.num_blocks
        return self.parameter_count - attn_blocks * (c.num_experts - c.moe_top_k) * per_expert

    # ------------------------------------------------------------ forward
    def hidden(self, tokens: torch.Tensor, training: bool = False, probe=None,
               aux_losses: Optional[list] = None, base_pos: int = 0) -> torch.Tensor:
        """Embedding -> (looped) block stack -> final norm.  tokens: [B, S] or [S]."""
        c = self.cfg
        squeeze = tokens.dim() == 1
        if squeeze:
            tokens = tokens[None]
        B, S = tokens.shape
        if S > c.max_seq:
            raise ValueError(f"Sequence length {S} exceeds MaxSeq {c.max_seq}.")
        self.forward_tokens += B * S
        x = self.wemb[tokens]
        dev = x.device
        rope = None
        if c.use_rope:
            rope = rope_tables(S, c.head_dim, base_pos, device=dev)
        else:
            x = x + sinusoidal_positions(S, c.dim, device=dev)
        if self.plan is not None:
            x = x + self.plan
        previous = None
        loops_used = 0
        for k in range(c.num_loops):
            if self.loop_bias is not None:
                x = x + self.loop_bias[k]
            for bi, blk in enumerate(self.blocks):
                x = blk(x, self.attn_scale, rope, training, aux_losses, probe, bi)
                if probe is not None:
                    probe.record_block(bi, x.detach())
            loops_used = k + 1
            if not training and c.loop_exit_tau > 0 and k < c.num_loops - 1:
                if previous is not None:
                    rel = (x - previous).norm() / (previous.norm() + 1e-12)
                    if float(rel) < c.loop_exit_tau:
                        break
                previous = x.detach().clone()
        if probe is not None:
            probe.loops_used = loops_used
        x = rms_norm(x, self.lnf_g, c.eps) if c.use_rms_norm else layer_norm(x, self.lnf_g, self.lnf_b, c.eps)
        return x[0] if squeeze else x

    def heads(self, tokens, training=False, probe=None, aux_losses=None):
        xf = self.hidden(tokens, training, probe, aux_losses)
        main = xf @ self.wout
        mtp = xf @ self.wout_mtp if self.wout_mtp is not None else None
        return main, mtp

    def forward(self, tokens: torch.Tensor, training: bool = False, probe=None) -> torch.Tensor:
        """Logits [.., S, V]."""
        return self.hidden(tokens, training, probe) @ self.wout

    def loss(self, tokens: torch.Tensor, targets: torch.Tensor, ignore_index: int = -1,
             training: bool = False) -> torch.Tensor:
        """Masked next-token CE (+ MTP aux head + MoE balance), DecoderLM.cs:320-350."""
        c = self.cfg
        aux = [] if c.num_experts > 0 and c.moe_balance_weight > 0 else None
        main, mtp = self.heads(tokens, training, None, aux)
        loss = cross_entropy_masked(main, targets, ignore_index)
        if mtp is not None:
            aux_t = mtp_targets(targets, c.mtp_horizon, ignore_index)
            if bool((aux_t != ignore_index).any()):
                loss = loss + c.mtp_weight * cross_entropy_masked(mtp, aux_t, ignore_index)
        if aux:
            loss = loss + c.moe_balance_weight * torch.stack(aux).sum()
        return loss

    # ------------------------------------------------------------ latent plan
    def settle_plan(self, prompt: torch.Tensor, steps: int, lr: float) -> List[float]:
        """Gradient steps on the plan vector alone (DecoderLM.cs:385-407)."""
        if self.plan is None:
            raise RuntimeError("settle_plan needs a model built with use_plan=True.")
        if prompt.numel() < 2:
            raise ValueError("Settling needs a prompt of at least 2 tokens.")
        if steps < 1:
            raise ValueError("steps must be >= 1.")
        tokens, targets = prompt[:-1], prompt[1:]
        trace = []
        for _ in range(steps):
            loss = cross_entropy_masked(self.forward(tokens), targets, -10**9)
            g, = torch.autograd.grad(loss, [self.plan])
            with torch.no_grad():
                self.plan -= lr * g
            trace.append(float(loss))
        return trace


def cross_entropy_masked(logits: torch.Tensor, targets: torch.Tensor, ignore_index: int = -1) -> torch.Tensor:
    """Mean CE over rows whose target != ignore_index; 0 if none (Autograd.cs:550-590).

    The CPU reference adds 1e-12 inside the log; at fp32 this changes nothing
    measurable for non-degenerate rows, so the pure log-softmax form is used.
    """
    V = logits.shape[-1]
    lg = logits.reshape(-1, V)
    lg = lg if lg.dtype == torch.float64 else lg.float()
    t = targets.reshape(-1)
    keep = t != ignore_index
    if not bool(keep.any()):
        return lg.sum() * 0.0
    return F.cross_entropy(lg[keep], t[keep].long())


def mtp_targets(targets: torch.Tensor, horizon: int, ignore_index: int) -> torch.Tensor:
    """Targets shifted horizon-1 further into the future; missing tail rows masked."""
    shift = horizon - 1
    t = targets.clone()
    if t.dim() == 1:
        t[:-shift] = targets[shift:]
        t[-shift:] = ignore_index
    else:
        t[:, :-shift] = targets[:, shift:]
        t[:, -shift:] = ignore_index
    return t
