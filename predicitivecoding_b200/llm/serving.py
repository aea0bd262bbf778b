"""KV-cache inference model, exporter and server.

Reference: PredictiveCoding.LLM/Serving/GptExporter.cs:30-193 (positional parameter walk of a
trained DecoderLM into the inference stack), Serving/LlmServer.cs:16-95 (O(n) decoding with a
KV cache), Model/Attention.cs:40-184 (per-layer KV cache with optional half-precision storage
and sliding-window eviction keeping attention sinks), Model/GptModel.cs:67-89 (single-token step).

``InferenceModel`` decodes a whole batch at once: prefill runs the prompt through the
blocks and fills a preallocated cache [layers, batch, heads, max_seq, head_dim]; each
``step`` appends one token per sequence.  It supports the dense attention family (RMSNorm
or LayerNorm, RoPE or sinusoidal positions, GELU or SwiGLU FFN, MoE FFN).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

from .. import ops

from ..models.decoder_lm import (AttentionBlock, DecoderLM, apply_rope, gelu_tanh, layer_norm, rms_norm,
                                 rope_tables, sinusoidal_positions)


@dataclass
class KvCache:
    k: torch.Tensor          # [L, B, H, S_max, hd]
    v: torch.Tensor
    length: int = 0
    sinks: int = 0           # tokens kept forever at the front when the window slides
    window: Optional[int] = None
    position: int = 0        # absolute position of the next token (RoPE angle), unaffected by eviction

    def evict(self) -> None:
        """Sliding window with attention sinks (Attention.cs:98-109): keep the first ``sinks``
        positions and the most recent ``window - sinks``."""
        if self.window is None or self.length <= self.window:
            return
        keep_recent = self.window - self.sinks
        src = slice(self.length - keep_recent, self.length)
        dst = slice(self.sinks, self.sinks + keep_recent)
        self.k[:, :, :, dst] = self.k[:, :, :, src].clone()
        self.v[:, :, :, dst] = self.v[:, :, :, src].clone()
        self.length = self.window


class InferenceModel:
    """Exported decoder for batched KV-cache decoding."""

    def __init__(self, model: DecoderLM, device=None, dtype: Optional[torch.dtype] = None,
                 kv_dtype: Optional[torch.dtype] = None):
        cfg = model.cfg
        if cfg.block_pattern is not None or cfg.num_loops != 1:
            raise NotImplementedError("InferenceModel runs dense attention stacks; recurrent 'T' blocks are served "
                                      "by export_gpt (step-by-step), looped models cannot be exported.")
        self.cfg = cfg
        self.device = torch.device(device) if device is not None else model.wemb.device
        self.dtype = dtype or (torch.bfloat16 if self.device.type == "cuda" else torch.float32)
        self.kv_dtype = kv_dtype or self.dtype
        self.model = model
        self.forward_tokens = 0
        # the decode kernel reads bf16 caches with head_dim 64 or 128 on the GPU
        self._fast_decode = (self.device.type == "cuda" and self.kv_dtype == torch.bfloat16
                             and cfg.head_dim in (64, 128))
        cast = lambda t: None if t is None else t.detach().to(self.device, self.dtype).contiguous()
        self._tc = self.device.type == "cuda" and self.dtype == torch.bfloat16 and ops.available()
        # the plan vector conditions every position identically: fold it into the embedding rows
        self.wemb = cast(model.wemb + model.plan if cfg.use_plan else model.wemb)
        self.wout = cast(model.wout)
        self.lnf = (cast(model.lnf_g), cast(model.lnf_b))
        self.blocks = []
        for b in model.blocks:
            blk = {}
            for name, p in b.named_parameters():
                blk[name] = cast(p)
            blk["_ref"] = b
            if (self._tc and cfg.ffn == "swiglu" and cfg.num_experts == 0 and "w1" in blk and "w3" in blk
                    and blk["w1"].shape[1] % 16 == 0 and blk["w1"].shape[0] % 8 == 0):
                # gate and up in alternating 16-column blocks: one projection launch with SwiGLU in its epilogue
                blk["w13"] = ops.interleave16(blk.pop("w1"), blk.pop("w3")).contiguous()
            self.blocks.append(blk)

    # ------------------------------------------------------------ pieces
    def _norm(self, x, g, b):
        c = self.cfg
        return rms_norm(x, g, c.eps) if c.use_rms_norm else layer_norm(x, g, b, c.eps)

    def _mm(self, x, w):
        """Projection on the tcgen05 GEMM when the shapes allow it (bf16 on the GPU), else torch."""
        return ops.linear(x, w) if self._tc and ops.linear_ok(x, w) else x @ w

    def _ffn(self, blk, h):
        c = self.cfg
        if c.num_experts > 0:
            return blk["_ref"].moe_ffn(h.float(), None).to(h.dtype)
        if c.ffn == "gelu":
            return self._mm(gelu_tanh(self._mm(h, blk["w1"]) + blk["b1"]), blk["w2"]) + blk["b2"]
        if "w13" in blk:
            return self._mm(ops.linear_swiglu(h.contiguous(), blk["w13"]), blk["w2"])
        return self._mm(F.silu(self._mm(h, blk["w1"])) * self._mm(h, blk["w3"]), blk["w2"])

    def new_cache(self, batch: int, max_len: Optional[int] = None, window: Optional[int] = None,
                  sinks: int = 0) -> KvCache:
        c = self.cfg
        S = max_len or c.max_seq
        shape = (c.num_blocks, batch, c.num_heads, S, c.head_dim)
        return KvCache(torch.zeros(shape, device=self.device, dtype=self.kv_dtype),
                       torch.zeros(shape, device=self.device, dtype=self.kv_dtype), 0, sinks, window)

    @torch.no_grad()
    def _run(self, tokens: torch.Tensor, cache: KvCache) -> torch.Tensor:
        """tokens [B, T] appended at cache.length; returns logits of every new position [B, T, V]."""
        c = self.cfg
        B, T = tokens.shape
        pos0 = cache.length
        if pos0 + T > cache.k.shape[3]:
            raise ValueError("KV cache full: evict or enlarge max_len")
        self.forward_tokens += B * T
        x = self.wemb[tokens]
        rope = None
        if c.use_rope:
            cos, sin = rope_tables(T, c.head_dim, cache.position, device=self.device)
            rope = (cos.to(self.dtype), sin.to(self.dtype))
        else:
            p0 = cache.position
            x = x + sinusoidal_positions(p0 + T, c.dim, device=self.device)[p0:].to(self.dtype)
        H, hd = c.num_heads, c.head_dim
        scale = 1.0 / math.sqrt(hd)
        lens = None
        for l, blk in enumerate(self.blocks):
            h = self._norm(x, blk["ln1_g"], blk.get("ln1_b"))
            q = self._mm(h, blk["wq"]).view(B, T, H, hd).transpose(1, 2)
            k = self._mm(h, blk["wk"]).view(B, T, H, hd).transpose(1, 2)
            v = self._mm(h, blk["wv"]).view(B, T, H, hd).transpose(1, 2)
            if rope is not None:
                q = apply_rope(q, *rope)
                k = apply_rope(k, *rope)
            cache.k[l, :, :, pos0:pos0 + T] = k.to(self.kv_dtype)
            cache.v[l, :, :, pos0:pos0 + T] = v.to(self.kv_dtype)
            if T == 1 and self._fast_decode:
                # one new token per sequence: split-KV decode kernel straight on the cache
                if lens is None:
                    lens = torch.full((B,), pos0 + 1, dtype=torch.int32, device=self.device)
                o = ops.decode_attn(q[:, :, 0].contiguous(), cache.k[l], cache.v[l], lens, scale)[:, :, None]
            elif pos0 == 0 and self._tc and T % 128 == 0 and hd in (64, 128):
                # prompt prefill on an empty cache: causal flash attention over the prompt
                qkv = torch.cat([t.transpose(1, 2).reshape(B * T, c.dim) for t in (q, k, v)], 1).contiguous()
                o2 = torch.empty(B * T, c.dim, device=self.device, dtype=torch.bfloat16)
                lse_buf = torch.empty(B * H, T, device=self.device)
                ops.attn_fwd(qkv, o2, lse_buf, B, T, H, hd, scale)
                o = o2.view(B, T, H, hd).transpose(1, 2)
            else:
                K = cache.k[l, :, :, :pos0 + T].to(self.dtype)
                V = cache.v[l, :, :, :pos0 + T].to(self.dtype)
                # causal over the new positions, full over the cached prefix
                mask = torch.ones(T, pos0 + T, dtype=torch.bool, device=self.device).tril(pos0)
                o = F.scaled_dot_product_attention(q, K, V, attn_mask=mask, scale=scale)
            x = x + self._mm(o.transpose(1, 2).reshape(B, T, c.dim).contiguous(), blk["wo"])
            x = x + self._ffn(blk, self._norm(x, blk["ln2_g"], blk.get("ln2_b")))
        cache.length = pos0 + T
        cache.position += T
        x = self._norm(x, *self.lnf)
        if self._tc and ops.linear_ok(x, self.wout):
            return ops.linear(x, self.wout, fp32=True)
        return (x @ self.wout).float()

    def prefill(self, tokens: torch.Tensor, cache: KvCache) -> torch.Tensor:
        if tokens.dim() == 1:
            tokens = tokens[None]
        return self._run(tokens.to(self.device), cache)

    def step(self, tokens: torch.Tensor, cache: KvCache) -> torch.Tensor:
        """One token per sequence [B] -> logits [B, V]."""
        if cache.window is not None and cache.length >= cache.window:
            cache.evict()
        return self._run(tokens.to(self.device).view(-1, 1), cache)[:, -1]

    @torch.no_grad()
    def generate(self, prompts: Sequence[Sequence[int]], max_new_tokens: int, eos: int = -1) -> List[List[int]]:
        """Greedy batched generation (prompts padded on the left to a common length)."""
        B = len(prompts)
        T = max(len(p) for p in prompts)
        pad = [[p[0]] * (T - len(p)) + list(p) for p in prompts]
        cache = self.new_cache(B, min(self.cfg.max_seq, T + max_new_tokens))
        logits = self.prefill(torch.tensor(pad), cache)[:, -1]
        out = [[] for _ in range(B)]
        done = [False] * B
        for _ in range(max_new_tokens):
            nxt = torch.argmax(logits, -1)
            for i, t in enumerate(nxt.tolist()):
                if not done[i]:
                    out[i].append(t)
                    done[i] = t == eos
            if all(done) or cache.length >= cache.k.shape[3]:
                break
            logits = self.step(nxt, cache)
        return out


def export(model: DecoderLM, device=None, dtype=None):
    """GptExporter.Export: a trained DecoderLM becomes a KV-cache inference model.  Dense attention
    stacks (with or without plan and MoE) get the batched device model; stacks with recurrent 'T'
    blocks get the step-by-step ``GptModel`` behind the same ``generate`` interface."""
    if model.cfg.block_pattern is not None and "T" in model.cfg.block_pattern:
        return StepModelServer(export_gpt(model), device)
    return InferenceModel(model, device, dtype)


class StepModelServer:
    """Batched ``generate`` over a step-by-step KV-cache model (each sequence keeps its own cache)."""

    def __init__(self, gpt, device=None):
        self.gpt = gpt.to(device) if device is not None else gpt
        self.cfg = gpt.cfg

    @torch.no_grad()
    def generate(self, prompts: Sequence[Sequence[int]], max_new_tokens: int, eos: int = -1) -> List[List[int]]:
        outs = []
        for p in prompts:
            cache = self.gpt.create_cache()
            pos, logits = 0, None
            for t in p:
                logits = self.gpt.step(int(t), pos, cache)
                pos += 1
            out = []
            while len(out) < max_new_tokens and pos < self.cfg.max_seq_len:
                nxt = int(torch.argmax(logits.reshape(-1)))
                out.append(nxt)
                if nxt == eos:
                    break
                logits = self.gpt.step(nxt, pos, cache)
                pos += 1
            outs.append(out)
        return outs


class LlmServer:
    """O(n) decoding over a KV cache (Serving/LlmServer.cs:16-95)."""

    def __init__(self, model: InferenceModel, tokenizer):
        self.model, self.tok = model, tokenizer
        self.prompted = 0
        self.generated = 0

    def generate(self, prompt: str, max_new_tokens: int = 64, stop_at_eos: bool = True) -> str:
        ids = self.tok.encode(prompt, add_bos=True)
        out = self.model.generate([ids], max_new_tokens, self.tok.eos if stop_at_eos else -1)[0]
        if stop_at_eos and out and out[-1] == self.tok.eos:
            out = out[:-1]
        self.prompted += len(ids)
        self.generated += len(out)
        return self.tok.decode(out)

    def generate_batch(self, prompts: Sequence[str], max_new_tokens: int = 64) -> List[str]:
        ids = [self.tok.encode(p, add_bos=True) for p in prompts]
        outs = self.model.generate(ids, max_new_tokens, self.tok.eos)
        return [self.tok.decode([t for t in o if t != self.tok.eos]) for o in outs]


@torch.no_grad()
def export_gpt(model: DecoderLM):
    """GptExporter.Export (Serving/GptExporter.cs:32-150): a trained DecoderLM becomes the step-by-step
    KV-cache ``GptModel`` of ``llm.gpt``, by walking the reference parameter order.

    Covers every block family the trainer has: attention blocks (per-head q/k/v/o slices), recurrent
    'T' blocks (wa/wi/wu/wo with biases, LayerNorm, GELU FFN), MoE FFNs (router + GELU experts) and the
    plan vector, which conditions every position identically and is therefore added into every row of
    the embedding table.  The multi-token head is skipped (the main head serves).  Looped models are
    refused, as in the reference (the serving stack is single-pass).
    """
    from .gpt import FeedForward, GptModel, Norm, TransformerConfig
    c = model.cfg
    if c.num_loops > 1:
        raise NotImplementedError("looped models (num_loops > 1) cannot be exported: serving is single-pass")
    tc = TransformerConfig(vocab_size=c.vocab, max_seq_len=c.max_seq, embed_dim=c.dim, num_heads=c.num_heads,
                           num_layers=c.num_blocks, feed_forward_dim=c.ff_dim, layer_norm_eps=c.eps,
                           tie_embeddings=False, positional="rotary" if c.use_rope else "sinusoidal",
                           norm="rmsnorm" if c.use_rms_norm else "layernorm", ffn=c.ffn,
                           block_pattern=c.block_pattern, num_experts=c.num_experts, moe_top_k=c.moe_top_k)
    gpt = GptModel(tc, seed=0)
    ps = [p.detach().float().cpu() for p in model.reference_parameters()]
    cur = [0]

    def nxt(rows, cols, what):
        if cur[0] >= len(ps):
            raise ValueError(f"exporter ran out of parameters at {what!r} (layout drift)")
        t = ps[cur[0]]
        cur[0] += 1
        t2 = t.view(1, -1) if t.dim() == 1 else t
        if tuple(t2.shape) != (rows, cols):
            raise ValueError(f"exporter shape mismatch at {what!r}: expected [{rows},{cols}], found {list(t2.shape)}")
        return t2

    def linear(lin, w, b=None):            # trainable y = x W ([in, out]) -> Linear weight [out, in]
        lin.weight.copy_(w.T)
        if b is not None:
            lin.bias.copy_(b.reshape(-1))

    def norm(n, g, b):
        if (b is None) != n.rms:
            raise ValueError("norm import mismatch: trained and served configs disagree")
        n.gamma.copy_(g.reshape(-1))
        if b is not None:
            n.beta.copy_(b.reshape(-1))

    D, hd, F_, H = c.dim, c.head_dim, c.ff_dim, c.num_heads
    rms = c.use_rms_norm
    wemb = nxt(c.vocab, D, "wemb")
    for bi, blk in enumerate(gpt.blocks):
        temporal = c.block_pattern is not None and c.block_pattern[bi] == "T"
        if temporal:
            # the trained recurrent block always uses LayerNorm and a GELU FFN with biases
            ln = TransformerConfig(**{**tc.__dict__, "norm": "layernorm"})
            blk.ln1, blk.ln2 = Norm(ln), Norm(ln)
            blk.ffn = FeedForward(tc, torch.Generator().manual_seed(0))
            norm(blk.ln1, nxt(1, D, "ln1G"), nxt(1, D, "ln1B"))
            for name in ("wa", "wi", "wu", "wo"):
                linear(getattr(blk.attn, name), nxt(D, D, name), nxt(1, D, "b" + name[1]))
        else:
            norm(blk.ln1, nxt(1, D, "ln1G"), None if rms else nxt(1, D, "ln1B"))
            a = blk.attn
            for h in range(H):
                s = slice(h * hd, (h + 1) * hd)
                a.q.weight[s].copy_(nxt(D, hd, "wq").T)
                a.k.weight[s].copy_(nxt(D, hd, "wk").T)
                a.v.weight[s].copy_(nxt(D, hd, "wv").T)
                a.o.weight[:, s].copy_(nxt(hd, D, "wo").T)
            for lin in (a.q, a.k, a.v, a.o):
                lin.bias.zero_()
        norm(blk.ln2, nxt(1, D, "ln2G"), None if (rms and not temporal) else nxt(1, D, "ln2B"))
        if c.num_experts > 0 and not temporal:
            linear(blk.ffn.router, nxt(D, c.num_experts, "router"))
            blk.ffn.router.bias.zero_()
            for ex in blk.ffn.experts:
                linear(ex.fc1, nxt(D, F_, "ew1"), nxt(1, F_, "eb1"))
                linear(ex.fc2, nxt(F_, D, "ew2"), nxt(1, D, "eb2"))
        elif temporal or c.ffn == "gelu":
            linear(blk.ffn.fc1, nxt(D, F_, "w1"), nxt(1, F_, "b1"))
            linear(blk.ffn.fc2, nxt(F_, D, "w2"), nxt(1, D, "b2"))
        else:
            f = blk.ffn
            linear(f.gate, nxt(D, F_, "w1"))
            linear(f.up, nxt(D, F_, "w3"))
            linear(f.down, nxt(F_, D, "w2"))
            for lin in (f.gate, f.up, f.down):
                lin.bias.zero_()
    norm(gpt.ln_final, nxt(1, D, "lnFG"), None if rms else nxt(1, D, "lnFB"))
    linear(gpt.lm_head, nxt(D, c.vocab, "wout"))
    gpt.lm_head.bias.zero_()
    if c.mtp_weight > 0:
        nxt(D, c.vocab, "woutMtp")
    plan = nxt(1, D, "plan").reshape(-1) if c.use_plan else torch.zeros(D)
    if cur[0] != len(ps):
        raise ValueError(f"exporter left {len(ps) - cur[0]} parameter(s) unconsumed (layout drift)")
    gpt.embedding.copy_(wemb + plan)
    return gpt
