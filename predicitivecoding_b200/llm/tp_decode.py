"""Tensor-parallel KV-cache decoding of the dense RMSNorm + RoPE + SwiGLU decoder (one process per GPU).

Reference: the reference decodes on the CPU, one token at a time over a KV cache (GptModel.Step,
Model/GptModel.cs:67-89; LlmServer, Serving/LlmServer.cs:16-95), and its only tensor parallelism is a
CPU column/row split of one matvec (Infrastructure/TensorParallel.cs:88-131).  Here the Megatron
layout runs on T GPUs:

* rank t owns heads [t*H/T, (t+1)*H/T) (column-parallel W_qkv, row-parallel W_o), FFN columns
  [t*F/T, (t+1)*F/T) (column-parallel W_1/W_3, row-parallel W_2) and vocabulary slice
  [t*V/T, (t+1)*V/T) of the LM head; the embedding and the norm gains are replicated;
* each rank keeps the KV cache of its own heads ([B, H/T, capacity, hd] bf16 per layer);
* each row-parallel product lands in this rank's half of a double-buffered symmetric buffer; after
  one device barrier a single kernel reads every rank's partial over NVLink, sums them in rank
  order, adds the fp32 residual (replicated on every rank) and writes the next RMSNorm's bf16
  input -- all-reduce, residual add and norm in one launch;
* prefill runs the prompt through the causal attention kernel; each decode step rotates q/k and
  appends k/v to the cache in one kernel, then runs the flash-decoding split-KV kernel; greedy sampling takes the per-rank vocabulary
  maxima and gathers them (value, index) over the ranks;
* one decode step is captured in a CUDA graph and replayed, so a step costs one graph launch.
"""
from __future__ import annotations

import math
import os
from typing import Optional

import torch
import torch.distributed as dist

from .. import ops
from ..models.config import DecoderLmConfig
from ..models.decoder_lm import DecoderLM, rope_tables


_ROW_SYNC = os.environ.get("PCB_TP_ROW_SYNC", "1") != "0"   # 0: device barrier + all-reduce kernel


def tp_decode_supports(cfg: DecoderLmConfig, world: int) -> bool:
    return (cfg.use_rms_norm and cfg.use_rope and cfg.ffn == "swiglu" and cfg.num_experts == 0
            and cfg.block_pattern is None and cfg.num_loops == 1 and not cfg.use_plan
            and cfg.num_heads % world == 0 and cfg.ff_dim % (16 * world) == 0 and cfg.vocab % world == 0
            and cfg.head_dim in (64, 128))


class TensorParallelDecoder:
    def __init__(self, cfg: DecoderLmConfig, batch: int, capacity: int, *, process_group=None, device="cuda",
                 model: Optional[DecoderLM] = None, seed: int = 42, use_graph: bool = True):
        from ..parallel.collectives import Communicator
        self.pg = process_group
        self.T = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.t = dist.get_rank(process_group) if dist.is_initialized() else 0
        if not tp_decode_supports(cfg, self.T):
            raise NotImplementedError("TensorParallelDecoder needs a dense RMSNorm+RoPE+SwiGLU config whose heads, "
                                      "FFN width and vocabulary divide by the TP size")
        self.cfg, self.B = cfg, batch
        self.cap = (capacity + 127) // 128 * 128
        self.device = dev = torch.device(device)
        T, t = self.T, self.t
        D, F_, V, L, H, hd = cfg.dim, cfg.ff_dim, cfg.vocab, cfg.num_blocks, cfg.num_heads, cfg.head_dim
        self.Hl, self.Fl, self.Vl = H // T, F_ // T, V // T
        self.Dl = self.Hl * hd
        bf16 = torch.bfloat16
        self.W = {}
        if model is not None:
            self._import(model)
        else:
            self._random(seed)
        from ..parallel.peer import PeerGroup
        self.comm = Communicator(self.pg, backend="peer", device=dev, capacity_bytes=1 << 20) if T > 1 else None
        self.peer = PeerGroup(self.pg, dev)
        self.pbuf = [self.peer.symmetric(batch * D, bf16) for _ in range(2)]   # decode partials
        # per-row handshake of the decode all-reduce (replaces a device barrier before each one)
        self.row_flags = self.peer.symmetric(batch * T, torch.int32) if T > 1 else None
        self.row_epoch = torch.zeros(batch, device=dev, dtype=torch.int32) if T > 1 else None
        self.pbuf_prefill = None
        self._flip = 0
        self.kc = [torch.zeros(batch, self.Hl, self.cap, hd, device=dev, dtype=bf16) for _ in range(L)]
        self.vc = [torch.zeros(batch, self.Hl, self.cap, hd, device=dev, dtype=bf16) for _ in range(L)]
        cos, sin = rope_tables(self.cap, hd, 0, device=dev)
        self.rope_cs = torch.stack((cos, sin), dim=-1).contiguous()          # [cap, hd/2, 2]
        self.scale = 1.0 / math.sqrt(hd)
        # decode-step state (static buffers so the step can be captured)
        # key splits per (sequence, head): one split (the attention kernel then writes the output itself, no
        # merge launch) while the (sequence, head) pairs fit one wave of the kernel (3 CTAs per SM), two
        # beyond; measured on B200 at 640 cached keys: 256 pairs 13.9 us with 1 split (16.8 + merge with 2);
        # 512 pairs 35.1 us + merge with 2 against 38.5 us with 1 (decode step 2.09 against 2.15 ms)
        nsplit = max(1, min(1 if batch * self.Hl <= 3 * 148 else 2, self.cap // 64))
        self.nsplit = nsplit
        self.pacc = torch.empty(batch * self.Hl * nsplit * hd, device=dev)
        self.pml = torch.empty(batch * self.Hl * nsplit * 2, device=dev)
        self.tok = torch.zeros(batch, device=dev, dtype=torch.int64)
        self.qbuf = torch.zeros(batch, self.Hl, hd, device=dev, dtype=bf16)
        self.pos = torch.zeros(1, device=dev, dtype=torch.int64)
        self.lens = torch.zeros(batch, device=dev, dtype=torch.int32)
        self.out_tokens = torch.zeros(batch, self.cap, device=dev, dtype=torch.int64)
        self.gather_in = torch.zeros(batch * 2, device=dev, dtype=torch.float32)
        self.gather_out = torch.zeros(T * batch * 2, device=dev, dtype=torch.float32)
        self.graph = None
        self.use_graph = use_graph
        self.launches_per_step = None

    # ------------------------------------------------------------------ weights
    def _shard(self, name, full: torch.Tensor):
        self.W[name] = full.to(self.device, torch.bfloat16).contiguous()

    def _import(self, model: DecoderLM) -> None:
        t, Dl, Fl, Vl, hd = self.t, self.Dl, self.Fl, self.Vl, self.cfg.head_dim
        hs = slice(t * Dl, (t + 1) * Dl)
        fs = slice(t * Fl, (t + 1) * Fl)
        with torch.no_grad():
            self._shard("wemb", model.wemb)
            self._shard("lnf", model.lnf_g)
            self._shard("wout", model.wout[:, t * Vl:(t + 1) * Vl])
            for l, blk in enumerate(model.blocks):
                self._shard(f"b{l}.ln1", blk.ln1_g)
                self._shard(f"b{l}.ln2", blk.ln2_g)
                self._shard(f"b{l}.wqkv", torch.cat((blk.wq[:, hs], blk.wk[:, hs], blk.wv[:, hs]), 1))
                self._shard(f"b{l}.wo", blk.wo[hs, :])
                # gate and up in alternating 16-column blocks: the decode projection applies SwiGLU in its
                # epilogue (each warp of the skinny kernel holds both halves of 16 features)
                self._shard(f"b{l}.w13", ops.interleave16(blk.w1[:, fs], blk.w3[:, fs]))
                self._shard(f"b{l}.w2", blk.w2[fs, :])

    def _random(self, seed: int) -> None:
        """Random-init shards straight on the device (replicated tensors from a shared seed)."""
        cfg, dev = self.cfg, self.device
        D, L = cfg.dim, cfg.num_blocks
        shared = torch.Generator(device=dev).manual_seed(seed)
        own = torch.Generator(device=dev).manual_seed(seed * 1009 + 7 + self.t)

        def rn(gen, *shape, std=0.02):
            return (torch.randn(*shape, device=dev, generator=gen) * std).to(torch.bfloat16)

        self.W["wemb"] = rn(shared, cfg.vocab, D, std=1.0)
        self.W["lnf"] = torch.ones(D, device=dev, dtype=torch.bfloat16)
        self.W["wout"] = rn(own, D, self.Vl)
        for l in range(L):
            self.W[f"b{l}.ln1"] = torch.ones(D, device=dev, dtype=torch.bfloat16)
            self.W[f"b{l}.ln2"] = torch.ones(D, device=dev, dtype=torch.bfloat16)
            self.W[f"b{l}.wqkv"] = rn(own, D, 3 * self.Dl)
            self.W[f"b{l}.wo"] = rn(own, self.Dl, D)
            self.W[f"b{l}.w13"] = rn(own, D, 2 * self.Fl)   # random: already "interleaved"
            self.W[f"b{l}.w2"] = rn(own, self.Fl, D)

    # ------------------------------------------------------------------ pieces
    def _norm(self, x: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
        y = torch.empty(x.shape, device=self.device, dtype=torch.bfloat16)
        ops.rmsnorm_fwd(x, g, y, None, self.cfg.eps)
        return y

    def _row_parallel(self, a: torch.Tensor, w: torch.Tensor, x: torch.Tensor, gamma: torch.Tensor,
                      bufs) -> torch.Tensor:
        """x += sum over ranks of a @ w; returns rmsnorm(x) * gamma in bf16."""
        buf = bufs[self._flip]
        self._flip ^= 1
        rows = a.shape[0]
        ops.linear(a, w, out=buf.local[:rows * self.cfg.dim].view(rows, self.cfg.dim))
        y = torch.empty(x.shape, device=self.device, dtype=torch.bfloat16)
        if self.T > 1 and rows == self.B and _ROW_SYNC:
            # decode: the kernel does a per-row handshake with the peers before reading their partials
            rc = ops.ext().tp_allreduce_norm(buf.ptrs, self.T, x, gamma, y, self.cfg.eps, self.row_flags.ptrs,
                                             self.row_epoch, self.t, self.peer.err)
        else:
            if self.T > 1:
                self.peer.barrier()
            rc = ops.ext().tp_allreduce_norm(buf.ptrs, self.T, x, gamma, y, self.cfg.eps)
        if rc != 0:
            raise RuntimeError(f"tp_allreduce_norm failed with status {rc}")
        return y

    def _layer(self, x: torch.Tensor, h: torch.Tensor, l: int, attn, bufs) -> torch.Tensor:
        """One block on normalised input h (residual x updated in place); returns the next norm's output."""
        W, L = self.W, self.cfg.num_blocks
        o = attn(h, W[f"b{l}.wqkv"], l)
        h2 = self._row_parallel(o, W[f"b{l}.wo"], x, W[f"b{l}.ln2"], bufs)
        a = ops.linear_swiglu(h2, W[f"b{l}.w13"])
        nxt = W[f"b{l + 1}.ln1"] if l + 1 < L else W["lnf"]
        return self._row_parallel(a, W[f"b{l}.w2"], x, nxt, bufs)

    def _argmax_tokens(self, hf: torch.Tensor) -> torch.Tensor:
        """Greedy next tokens from the final normalised rows [B, D] (vocabulary split over ranks)."""
        logits = ops.linear(hf, self.W["wout"], fp32=True)      # [B, V/T]
        val, idx = logits.max(dim=-1)
        if self.comm is None:
            return idx
        self.gather_in.view(self.B, 2)[:, 0] = val
        self.gather_in.view(self.B, 2)[:, 1] = (idx + self.t * self.Vl).float()
        self.comm.all_gather(self.gather_out, self.gather_in)
        g = self.gather_out.view(self.T, self.B, 2)
        best = g[:, :, 0].argmax(dim=0)                          # lowest rank wins ties, like a global argmax
        return g[:, :, 1].gather(0, best[None]).squeeze(0).long()

    # ------------------------------------------------------------------ prefill
    @torch.no_grad()
    def prefill(self, prompt: torch.Tensor) -> torch.Tensor:
        """Run the prompt [B, P] (P % 128 == 0) through the model, fill the caches, return the first
        generated token of each row."""
        cfg, B = self.cfg, self.B
        P = prompt.shape[1]
        if prompt.shape[0] != B or P % 128 or P >= self.cap:
            raise ValueError("prompt must be [batch, P] with P % 128 == 0 and P < capacity")
        D, Dl, Hl, hd = cfg.dim, self.Dl, self.Hl, cfg.head_dim
        M = B * P
        if self.pbuf_prefill is None or self.pbuf_prefill[0].local.numel() < M * D:
            self.pbuf_prefill = [self.peer.symmetric(M * D, torch.bfloat16) for _ in range(2)]
        tok = prompt.to(self.device, torch.int32).reshape(-1)
        x = torch.empty(M, D, device=self.device)
        ops.embed_fwd(tok, self.W["wemb"], x)
        out = torch.empty(M, Dl, device=self.device, dtype=torch.bfloat16)
        lse = torch.empty(B * Hl, P, device=self.device)
        cs = self.rope_cs[:P].contiguous()

        def attn(h, w_qkv, l):
            qkv = ops.linear(h, w_qkv)                         # [M, 3*Dl] = q | k | v column blocks
            ops.rope(qkv, cs, P, Dl, hd, 2, 1.0)
            kv = qkv.view(B, P, 3, Hl, hd)
            self.kc[l][:, :, :P].copy_(kv[:, :, 1].transpose(1, 2))
            self.vc[l][:, :, :P].copy_(kv[:, :, 2].transpose(1, 2))
            ops.attn_fwd(qkv, out, lse, B, P, Hl, hd, self.scale)
            return out

        self._flip = 0
        h = self._norm(x, self.W["b0.ln1"])
        for l in range(cfg.num_blocks):
            h = self._layer(x, h, l, attn, self.pbuf_prefill)
        last = h.view(B, P, D)[:, -1].contiguous()             # lnf already applied
        nxt = self._argmax_tokens(last)
        self.tok.copy_(nxt)
        self.pos.fill_(P)
        self.lens.fill_(P)
        self.out_tokens[:, 0] = nxt
        self.prompt_len = P
        return nxt

    # ------------------------------------------------------------------ decode
    def _step_body(self) -> None:
        """One token for every row: reads self.tok at position self.pos, writes the next token."""
        cfg, B = self.cfg, self.B
        D, Dl, Hl, hd = cfg.dim, self.Dl, self.Hl, cfg.head_dim
        x = self.W["wemb"].index_select(0, self.tok).float()   # [B, D]
        self.lens.add_(1)

        def attn(h, w_qkv, l):
            # projection, RoPE on q and k at self.pos, q -> self.qbuf, k / v appended to the caches (one launch)
            ops.qkv_rope_append(h, w_qkv, self.rope_cs, self.pos, self.qbuf, self.kc[l], self.vc[l])
            o = ops.decode_attn(self.qbuf, self.kc[l], self.vc[l], self.lens, self.scale, nsplit=self.nsplit,
                                scratch=(self.pacc, self.pml))
            return o.view(B, Dl)

        self._flip = 0
        h = self._norm(x, self.W["b0.ln1"])
        for l in range(cfg.num_blocks):
            h = self._layer(x, h, l, attn, self.pbuf)
        nxt = self._argmax_tokens(h)
        self.tok.copy_(nxt)
        self.pos.add_(1)
        self.out_tokens.index_copy_(1, self.pos - self.prompt_len, nxt[:, None])

    def _capture(self) -> None:
        # warm the allocator and the kernels outside the graph on a copy of the state, then restore
        saved = (self.tok.clone(), self.pos.clone(), self.lens.clone())
        before = ops.launch_count()
        self._step_body()
        self.launches_per_step = ops.launch_count() - before
        torch.cuda.synchronize(self.device)
        self.tok.copy_(saved[0]); self.pos.copy_(saved[1]); self.lens.copy_(saved[2])
        if self.T > 1:
            self.peer.barrier()
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            with torch.cuda.graph(self.graph, stream=s):
                self._step_body()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)

    @torch.no_grad()
    def decode(self, steps: int) -> None:
        """Generate `steps` more tokens per row (after prefill); tokens land in out_tokens[:, 1:]."""
        if int(self.pos) + steps > self.cap:
            raise ValueError("decode would run past the KV-cache capacity")
        if self.use_graph and self.graph is None:
            self._capture()
        for _ in range(steps):
            if self.graph is not None:
                self.graph.replay()
            else:
                self._step_body()

    @torch.no_grad()
    def generate(self, prompt: torch.Tensor, new_tokens: int) -> torch.Tensor:
        """Greedy continuation: [B, new_tokens] token ids (on the host)."""
        self.prefill(prompt)
        self.decode(new_tokens - 1)
        return self.out_tokens[:, :new_tokens].cpu()

    def check(self) -> None:
        self.peer.check()
        if self.comm is not None:
            self.comm.check()

    def release(self) -> None:
        self.graph = None
        torch.cuda.synchronize(self.device)
