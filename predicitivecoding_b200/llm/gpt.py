"""Configurable GPT inference family: GQA, RoPE/ALiBi/sinusoidal, QK-norm, soft-caps, latent (MLA)
attention, sliding window with sink tokens, fp16 KV cache, recurrent 'T' blocks and MoE FFNs.

Reference: PredictiveCoding.LLM/Model/TransformerConfig.cs:1-203 (config + validation),
ModernPresets.cs:1-74 (Llama-3 / Nemotron / DeepSeek style presets), GptModel.cs:1-90,
TransformerBlock.cs:1-149, Attention.cs:1-455, RecurrentLayer.cs:1-79, Layers.cs:1-259.

The reference runs one token for one sequence per call with per-head ``List<float[]>`` caches.
Here every call is batched: ``forward`` runs a whole prompt for B sequences at once (masked
attention, GEMM-shaped), ``step`` decodes one token for all B sequences against a tensor KV cache
``[B, Hkv, T, hd]``; eviction for the sliding window keeps the sink prefix and the newest
``window`` entries exactly as the reference's ``KvCacheLayer.Evict``.
"""
from __future__ import annotations

import json
import math
from dataclasses import asdict, dataclass, replace
from typing import List, Optional, Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..pc.layer import init_weights


@dataclass(frozen=True)
class TransformerConfig:
    vocab_size: int = 260
    max_seq_len: int = 256
    embed_dim: int = 128
    num_heads: int = 4
    num_kv_heads: int = 0            # 0 -> num_heads
    num_layers: int = 4
    feed_forward_dim: int = 512
    layer_norm_eps: float = 1e-5
    tie_embeddings: bool = True
    positional: str = "sinusoidal"   # sinusoidal | rotary | alibi
    norm: str = "layernorm"          # layernorm | rmsnorm
    use_flash_attention: bool = False
    ffn: str = "gelu"                # gelu | swiglu
    attention: str = "multihead"     # multihead | latent
    use_qk_norm: bool = False
    attn_logit_softcap: float = 0.0
    final_logit_softcap: float = 0.0
    kv_latent_dim: int = 64
    rope_head_dim: int = 16
    window_size: int = 0
    num_sink_tokens: int = 0
    kv_cache_half: bool = False
    block_pattern: Optional[str] = None
    num_experts: int = 0
    moe_top_k: int = 1

    @property
    def head_dim(self) -> int:
        return self.embed_dim // self.num_heads

    @property
    def kv_heads(self) -> int:
        return self.num_heads if self.num_kv_heads <= 0 else self.num_kv_heads

    @property
    def kv_group_size(self) -> int:
        return self.num_heads // self.kv_heads

    def validate(self) -> None:
        def bad(msg):
            raise ValueError(msg)
        if self.vocab_size < 2:
            bad("vocab_size must be >= 2.")
        if self.max_seq_len < 1 or self.embed_dim < 1 or self.num_heads < 1:
            bad("max_seq_len, embed_dim and num_heads must be >= 1.")
        if self.embed_dim % self.num_heads:
            bad(f"embed_dim ({self.embed_dim}) must be divisible by num_heads ({self.num_heads}).")
        if self.kv_heads < 1 or self.num_heads % self.kv_heads:
            bad(f"num_heads ({self.num_heads}) must be divisible by kv_heads ({self.kv_heads}).")
        if self.positional not in ("sinusoidal", "rotary", "alibi"):
            bad(f"unknown positional kind {self.positional!r}")
        if self.norm not in ("layernorm", "rmsnorm") or self.ffn not in ("gelu", "swiglu"):
            bad("norm must be layernorm|rmsnorm and ffn gelu|swiglu")
        if self.attention not in ("multihead", "latent"):
            bad(f"unknown attention kind {self.attention!r}")
        if self.positional == "rotary" and self.head_dim % 2:
            bad("RoPE requires an even head_dim.")
        if self.attention == "latent":
            if self.kv_latent_dim < 1:
                bad("kv_latent_dim must be >= 1 for latent attention.")
            if self.rope_head_dim < 2 or self.rope_head_dim % 2:
                bad("rope_head_dim must be a positive even number for latent attention.")
        if self.attn_logit_softcap < 0 or self.final_logit_softcap < 0:
            bad("Soft-cap values must be >= 0 (0 disables).")
        if self.window_size < 0 or self.num_sink_tokens < 0:
            bad("window_size and num_sink_tokens must be >= 0.")
        if self.num_sink_tokens > 0 and self.window_size == 0:
            bad("num_sink_tokens needs window_size > 0.")
        if self.window_size > 0 and self.attention == "latent":
            bad("Sliding-window attention applies to the standard KV path.")
        if self.block_pattern is not None:
            if len(self.block_pattern) != self.num_layers:
                bad("block_pattern length must equal num_layers.")
            if set(self.block_pattern) - {"A", "T"}:
                bad("block_pattern may only contain 'A' and 'T'.")
        if self.num_experts < 0 or (self.num_experts > 0 and not 1 <= self.moe_top_k <= self.num_experts):
            bad("moe_top_k must be in [1, num_experts].")
        if self.num_layers < 1 or self.feed_forward_dim < 1 or self.layer_norm_eps <= 0:
            bad("num_layers, feed_forward_dim >= 1 and layer_norm_eps > 0 required.")

    def to_json(self) -> str:
        return json.dumps(asdict(self))

    @staticmethod
    def from_json(s: str) -> "TransformerConfig":
        return TransformerConfig(**json.loads(s))

    def with_(self, **kw) -> "TransformerConfig":
        return replace(self, **kw)


class ModernPresets:
    @staticmethod
    def llama3_style(vocab=260, max_seq=256, embed=128, heads=4, kv_heads=2, layers=4, ff=512) -> TransformerConfig:
        return TransformerConfig(vocab, max_seq, embed, heads, kv_heads, layers, ff, norm="rmsnorm", ffn="swiglu",
                                 positional="rotary")

    @staticmethod
    def nemotron_style(vocab=260, max_seq=256, embed=128, heads=4, kv_heads=2, layers=4, ff=512) -> TransformerConfig:
        pattern = "".join("A" if (l + 1) % 4 == 0 else "T" for l in range(layers))
        return TransformerConfig(vocab, max_seq, embed, heads, kv_heads, layers, ff, norm="rmsnorm", ffn="swiglu",
                                 positional="rotary", block_pattern=pattern)

    @staticmethod
    def deepseek_style(vocab=260, max_seq=256, embed=128, heads=4, layers=4, ff=512) -> TransformerConfig:
        rope = max(2, (embed // heads) // 2)
        rope -= rope % 2
        return TransformerConfig(vocab, max_seq, embed, heads, 0, layers, ff, norm="rmsnorm", ffn="swiglu",
                                 positional="rotary", use_qk_norm=True, attn_logit_softcap=50.0,
                                 final_logit_softcap=30.0, attention="latent", kv_latent_dim=max(1, embed // 2),
                                 rope_head_dim=rope)


# ---------------------------------------------------------------- building blocks
class Linear(nn.Module):
    """y = W x + b with W [out, in]; init by the activation that follows (He for ReLU-like gates)."""

    def __init__(self, d_in: int, d_out: int, gen: torch.Generator, init: str = "linear"):
        super().__init__()
        self.weight = nn.Parameter(init_weights(d_in, d_out, init, gen))
        self.bias = nn.Parameter(torch.zeros(d_out))

    def forward(self, x):
        return F.linear(x, self.weight, self.bias)


class Norm(nn.Module):
    def __init__(self, cfg: TransformerConfig):
        super().__init__()
        self.rms = cfg.norm == "rmsnorm"
        self.eps = cfg.layer_norm_eps
        self.gamma = nn.Parameter(torch.ones(cfg.embed_dim))
        self.beta = None if self.rms else nn.Parameter(torch.zeros(cfg.embed_dim))

    def forward(self, x):
        if self.rms:
            return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + self.eps) * self.gamma
        return F.layer_norm(x, x.shape[-1:], self.gamma, self.beta, self.eps)


def _rms_heads(x, eps):
    return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps)


def rope_rotate(x: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
    """Interleaved-pair rotation of the last dim; theta_i = pos * 10000^(-2i/d).  positions: [..T] broadcast."""
    d = x.shape[-1]
    i = torch.arange(d // 2, device=x.device, dtype=torch.float32)
    inv = torch.pow(torch.tensor(10000.0, device=x.device), -(2 * i) / d)
    ang = positions.to(torch.float32)[..., None] * inv
    c, s = torch.cos(ang).to(x.dtype), torch.sin(ang).to(x.dtype)
    x0, x1 = x[..., 0::2], x[..., 1::2]
    return torch.stack([x0 * c - x1 * s, x0 * s + x1 * c], -1).flatten(-2)


def sinusoidal(positions: torch.Tensor, dim: int) -> torch.Tensor:
    """pe[2j] = sin(p / 10000^(2j/d)), pe[2j+1] = cos(same angle)."""
    i = torch.arange(0, dim, 2, device=positions.device, dtype=torch.float32)
    ang = positions.to(torch.float32)[:, None] / torch.pow(torch.tensor(10000.0, device=positions.device), i / dim)
    pe = torch.zeros(positions.numel(), dim, device=positions.device)
    pe[:, 0::2] = torch.sin(ang)
    pe[:, 1::2] = torch.cos(ang)[:, : dim // 2]
    return pe


class LayerCache:
    """K/V of one attention layer for B sequences: k, v [B, Hkv, T, hd]; positions [T] (shared)."""

    def __init__(self, half: bool = False):
        self.k = self.v = None
        self.positions: List[int] = []
        self.half = half

    @property
    def length(self) -> int:
        return len(self.positions)

    @property
    def bytes_used(self) -> int:
        return 0 if self.k is None else self.k.numel() * self.k.element_size() * 2

    def append(self, k, v, positions: Sequence[int]) -> None:
        dt = torch.float16 if self.half else k.dtype
        k, v = k.to(dt), v.to(dt)
        self.k = k if self.k is None else torch.cat([self.k, k], 2)
        self.v = v if self.v is None else torch.cat([self.v, v], 2)
        self.positions.extend(int(p) for p in positions)

    def evict(self, sinks: int, window: int) -> None:
        n = self.length
        if n <= sinks + window:
            return
        keep = list(range(sinks)) + list(range(n - window, n))
        idx = torch.tensor(keep, device=self.k.device)
        self.k, self.v = self.k.index_select(2, idx), self.v.index_select(2, idx)
        self.positions = [self.positions[i] for i in keep]

    def clone(self) -> "LayerCache":
        c = LayerCache(self.half)
        c.k = None if self.k is None else self.k.clone()
        c.v = None if self.v is None else self.v.clone()
        c.positions = list(self.positions)
        return c


class LatentCache(LayerCache):
    """MLA cache: the compressed latent c_kv [B, T, dc] and the shared RoPE key k_R [B, T, dr]."""


class RecurrentCache:
    def __init__(self, state: Optional[torch.Tensor] = None, length: int = 0):
        self.state, self.length_ = state, length

    @property
    def length(self) -> int:
        return self.length_

    @property
    def bytes_used(self) -> int:
        return 0 if self.state is None else self.state.numel() * 4

    def clone(self):
        return RecurrentCache(None if self.state is None else self.state.clone(), self.length_)


class KvCache:
    def __init__(self, layers):
        self.layers = layers

    @property
    def length(self) -> int:
        return self.layers[0].length if self.layers else 0

    @property
    def bytes_used(self) -> int:
        return sum(l.bytes_used for l in self.layers)

    def clone(self) -> "KvCache":
        return KvCache([l.clone() for l in self.layers])


def _softmax_attend(q, k, v, bias, softcap, scale):
    """q [B,H,Tq,d], k/v [B,H,Tk,d], bias [Tq,Tk] (+ per-head [H,Tq,Tk]) additive (-inf masks)."""
    s = torch.matmul(q, k.transpose(-1, -2)) * scale
    if softcap > 0:
        s = softcap * torch.tanh(s / softcap)
    s = s + bias
    return torch.matmul(torch.softmax(s, -1), v)


class MultiHeadAttention(nn.Module):
    def __init__(self, cfg: TransformerConfig, gen: torch.Generator):
        super().__init__()
        self.cfg = cfg
        H, G, hd = cfg.num_heads, cfg.kv_heads, cfg.head_dim
        self.q = Linear(cfg.embed_dim, H * hd, gen)
        self.k = Linear(cfg.embed_dim, G * hd, gen)
        self.v = Linear(cfg.embed_dim, G * hd, gen)
        self.o = Linear(H * hd, cfg.embed_dim, gen)
        self.register_buffer("slopes", torch.tensor([2.0 ** (-(8.0 / H) * (h + 1)) for h in range(H)]),
                             persistent=False)

    def create_cache(self):
        return LayerCache(self.cfg.kv_cache_half)

    def forward(self, x, cache: Optional[LayerCache], positions: torch.Tensor):
        """x [B,T,D] at absolute ``positions`` [T]; attends to the cache (if any) plus itself, causally."""
        c = self.cfg
        B, T, _ = x.shape
        H, G, hd = c.num_heads, c.kv_heads, c.head_dim
        q = self.q(x).view(B, T, H, hd).transpose(1, 2)
        k = self.k(x).view(B, T, G, hd).transpose(1, 2)
        v = self.v(x).view(B, T, G, hd).transpose(1, 2)
        if c.use_qk_norm:
            q, k = _rms_heads(q, c.layer_norm_eps), _rms_heads(k, c.layer_norm_eps)
        if c.positional == "rotary":
            q, k = rope_rotate(q, positions), rope_rotate(k, positions)
        if cache is not None:
            outs = []
            # token by token when a window evicts mid-prompt, so every query sees exactly the
            # entries the cache holds at its own step
            chunks = [(t, t + 1) for t in range(T)] if c.window_size > 0 else [(0, T)]
            for a, b in chunks:
                cache.append(k[:, :, a:b], v[:, :, a:b], positions[a:b].tolist())
                if c.window_size > 0:
                    cache.evict(c.num_sink_tokens, c.window_size)
                kp = torch.tensor(cache.positions, device=x.device)
                outs.append(self._attend(q[:, :, a:b], cache.k.to(q.dtype), cache.v.to(q.dtype),
                                         positions[a:b], kp))
            ctx = torch.cat(outs, 2)
        else:
            ctx = self._attend(q, k, v, positions, positions)
        return self.o(ctx.transpose(1, 2).reshape(B, T, H * hd))

    def _attend(self, q, k, v, qpos, kpos):
        c = self.cfg
        g = c.kv_group_size
        if g > 1:
            k, v = k.repeat_interleave(g, 1), v.repeat_interleave(g, 1)
        dist = (qpos[:, None] - kpos[None, :]).to(q.dtype)                     # [Tq, Tk]
        allowed = dist >= 0
        if c.window_size > 0:
            allowed &= (dist < c.window_size) | (kpos[None, :] < c.num_sink_tokens)
        bias = torch.zeros_like(dist).masked_fill(~allowed, float("-inf"))
        if c.positional == "alibi":
            bias = bias - self.slopes.to(q.dtype)[:, None, None] * dist.clamp(min=0)
        return _softmax_attend(q, k, v, bias, c.attn_logit_softcap, 1.0 / math.sqrt(c.head_dim))


class LatentAttention(nn.Module):
    """Multi-head latent attention: cache c_kv = W_dkv h [dc] and a shared RoPE key k_R [dr]."""

    def __init__(self, cfg: TransformerConfig, gen: torch.Generator):
        super().__init__()
        self.cfg = cfg
        H, hd, dc, dr = cfg.num_heads, cfg.head_dim, cfg.kv_latent_dim, cfg.rope_head_dim
        D = cfg.embed_dim
        self.w_dkv = Linear(D, dc, gen)
        self.w_uk = Linear(dc, H * hd, gen)
        self.w_uv = Linear(dc, H * hd, gen)
        self.w_q = Linear(D, H * hd, gen)
        self.w_kr = Linear(D, dr, gen)
        self.w_qr = Linear(D, H * dr, gen)
        self.w_o = Linear(H * hd, D, gen)

    def create_cache(self):
        return LatentCache()

    def forward(self, x, cache, positions):
        c = self.cfg
        B, T, _ = x.shape
        H, hd, dr = c.num_heads, c.head_dim, c.rope_head_dim
        ckv = self.w_dkv(x)                                                    # [B,T,dc]
        kr = rope_rotate(self.w_kr(x), positions)                              # [B,T,dr]
        q = self.w_q(x).view(B, T, H, hd).transpose(1, 2)
        qr = rope_rotate(self.w_qr(x).view(B, T, H, dr).transpose(1, 2), positions)
        if cache is not None:
            cache.append(ckv[:, None], kr[:, None], positions.tolist())       # stored as [B,1,T,*]
            ckv_all, kr_all = cache.k[:, 0], cache.v[:, 0]
            kpos = torch.tensor(cache.positions, device=x.device)
        else:
            ckv_all, kr_all, kpos = ckv, kr, positions
        Tk = ckv_all.shape[1]
        k = self.w_uk(ckv_all).view(B, Tk, H, hd).transpose(1, 2)
        v = self.w_uv(ckv_all).view(B, Tk, H, hd).transpose(1, 2)
        s = (torch.matmul(q, k.transpose(-1, -2)) + torch.matmul(qr, kr_all[:, None].transpose(-1, -2)))
        s = s / math.sqrt(hd + dr)
        if c.attn_logit_softcap > 0:
            s = c.attn_logit_softcap * torch.tanh(s / c.attn_logit_softcap)
        s = s.masked_fill(positions[:, None] < kpos[None, :], float("-inf"))
        ctx = torch.matmul(torch.softmax(s, -1), v)
        return self.w_o(ctx.transpose(1, 2).reshape(B, T, H * hd))


class RecurrentTemporalLayer(nn.Module):
    """h_t = sigmoid(W_a x) * h_{t-1} + sigmoid(W_i x) * (W_u x);  out = W_o h_t."""

    def __init__(self, cfg: TransformerConfig, gen: torch.Generator):
        super().__init__()
        D = cfg.embed_dim
        self.wa, self.wi, self.wu, self.wo = (Linear(D, D, gen) for _ in range(4))

    def create_cache(self):
        return RecurrentCache()

    def forward(self, x, cache, positions):
        a, i, u = torch.sigmoid(self.wa(x)), torch.sigmoid(self.wi(x)), self.wu(x)
        h = cache.state if cache is not None and cache.state is not None else torch.zeros_like(x[:, 0])
        outs = []
        for t in range(x.shape[1]):
            h = a[:, t] * h + i[:, t] * u[:, t]
            outs.append(h)
        if cache is not None:
            cache.state, cache.length_ = h, cache.length_ + x.shape[1]
        return self.wo(torch.stack(outs, 1))


class FeedForward(nn.Module):
    def __init__(self, cfg: TransformerConfig, gen: torch.Generator):
        super().__init__()
        self.fc1 = Linear(cfg.embed_dim, cfg.feed_forward_dim, gen, "relu")
        self.fc2 = Linear(cfg.feed_forward_dim, cfg.embed_dim, gen)

    def forward(self, x):
        return self.fc2(F.gelu(self.fc1(x), approximate="tanh"))


class SwiGluFeedForward(nn.Module):
    def __init__(self, cfg: TransformerConfig, gen: torch.Generator):
        super().__init__()
        self.gate = Linear(cfg.embed_dim, cfg.feed_forward_dim, gen, "relu")
        self.up = Linear(cfg.embed_dim, cfg.feed_forward_dim, gen)
        self.down = Linear(cfg.feed_forward_dim, cfg.embed_dim, gen)

    def forward(self, x):
        return self.down(F.silu(self.gate(x)) * self.up(x))


class MoeFeedForward(nn.Module):
    """Softmax router; the top-k experts (GELU FFNs) are summed weighted by their raw gate."""

    def __init__(self, cfg: TransformerConfig, gen: torch.Generator):
        super().__init__()
        self.router = Linear(cfg.embed_dim, cfg.num_experts, gen)
        self.experts = nn.ModuleList(FeedForward(cfg, gen) for _ in range(cfg.num_experts))
        self.top_k = cfg.moe_top_k

    def forward(self, x):
        gates = torch.softmax(self.router(x), -1)
        g, idx = gates.topk(self.top_k, -1)
        flat = x.reshape(-1, x.shape[-1])
        out = torch.zeros_like(flat)
        gf, idf = g.reshape(-1, self.top_k), idx.reshape(-1, self.top_k)
        for e, ex in enumerate(self.experts):
            rows, slot = (idf == e).nonzero(as_tuple=True)
            if rows.numel():
                out.index_add_(0, rows, gf[rows, slot, None] * ex(flat[rows]))
        return out.view_as(x)


class TransformerBlock(nn.Module):
    def __init__(self, cfg: TransformerConfig, gen: torch.Generator, temporal: bool = False):
        super().__init__()
        self.ln1, self.ln2 = Norm(cfg), Norm(cfg)
        if temporal:
            self.attn = RecurrentTemporalLayer(cfg, gen)
        elif cfg.attention == "latent":
            self.attn = LatentAttention(cfg, gen)
        else:
            self.attn = MultiHeadAttention(cfg, gen)
        if cfg.num_experts > 0 and not temporal:
            self.ffn = MoeFeedForward(cfg, gen)
        elif cfg.ffn == "swiglu" and not (temporal and cfg.num_experts > 0):
            self.ffn = SwiGluFeedForward(cfg, gen)
        else:
            self.ffn = FeedForward(cfg, gen)

    def create_cache(self):
        return self.attn.create_cache()

    def forward(self, x, cache, positions):
        h = x + self.attn(self.ln1(x), cache, positions)
        return h + self.ffn(self.ln2(h))


class GptModel(nn.Module):
    def __init__(self, cfg: TransformerConfig, seed: int = 0):
        super().__init__()
        cfg.validate()
        self.cfg = cfg
        gen = torch.Generator().manual_seed(seed)
        self.embedding = nn.Parameter(torch.randn(cfg.vocab_size, cfg.embed_dim, generator=gen) * 0.02)
        pat = cfg.block_pattern
        self.blocks = nn.ModuleList(TransformerBlock(cfg, gen, temporal=pat is not None and pat[l] == "T")
                                    for l in range(cfg.num_layers))
        self.ln_final = Norm(cfg)
        self.lm_head = None if cfg.tie_embeddings else Linear(cfg.embed_dim, cfg.vocab_size, gen)
        self.forward_tokens = 0

    @property
    def vocab_size(self) -> int:
        return self.cfg.vocab_size

    @property
    def max_seq_len(self) -> int:
        return self.cfg.max_seq_len

    def create_cache(self) -> KvCache:
        return KvCache([b.create_cache() for b in self.blocks])

    def forward(self, tokens: torch.Tensor, cache: Optional[KvCache] = None, start: int = 0, probe=None):
        """tokens [B, T] (or [T]) at positions start..start+T-1 -> logits [B, T, V]."""
        if tokens.dim() == 1:
            tokens = tokens[None]
        B, T = tokens.shape
        if int(tokens.min()) < 0 or int(tokens.max()) >= self.cfg.vocab_size:
            raise ValueError("token out of range")
        dev = self.embedding.device
        tokens = tokens.to(dev)
        positions = torch.arange(start, start + T, device=dev)
        x = self.embedding[tokens]
        if self.cfg.positional == "sinusoidal":
            x = x + sinusoidal(positions, self.cfg.embed_dim).to(x.dtype)
        for l, blk in enumerate(self.blocks):
            x = blk(x, None if cache is None else cache.layers[l], positions)
            if probe is not None:
                probe.record_block(l, x[0, -1].detach().float().cpu())
        x = self.ln_final(x)
        logits = x @ self.embedding.T if self.lm_head is None else self.lm_head(x)
        if self.cfg.final_logit_softcap > 0:
            cap = self.cfg.final_logit_softcap
            logits = cap * torch.tanh(logits / cap)
        self.forward_tokens += B * T
        return logits

    @torch.no_grad()
    def step(self, token, position: int, cache: KvCache, probe=None) -> torch.Tensor:
        """One decode step for B sequences: token [B] (or int) at ``position`` -> logits [B, V] (or [V])."""
        scalar = isinstance(token, int)
        t = torch.tensor([[token]]) if scalar else torch.as_tensor(token).view(-1, 1)
        out = self.forward(t, cache, position, probe)[:, -1]
        return out[0] if scalar else out

    @torch.no_grad()
    def generate(self, prompt: Sequence[int], max_new: int, eos: Optional[int] = None) -> List[int]:
        cache = self.create_cache()
        logits = self.forward(torch.tensor(prompt)[None], cache, 0)[0, -1]
        out = list(prompt)
        for _ in range(max_new):
            nxt = int(logits.argmax())
            out.append(nxt)
            if nxt == eos or len(out) >= self.cfg.max_seq_len:
                break
            logits = self.step(nxt, len(out) - 1, cache)
        return out
