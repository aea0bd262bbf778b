"""Device-resident decoder trainer on the hand-written sm_100a kernels.

The B200 counterpart of the reference's ``DeviceDecoderTrainer``
(PredictiveCoding.Device/Training/DeviceDecoderTrainer.cs:40-575): weights, Adam
state and every activation live in preallocated device buffers; a step is one
forward, one fused cross-entropy, one backward and one AdamW, with the loss as
the only value read back.  Differences by design:

* true batches: the reference trains one sequence per launch chain and
  accumulates windows; here one step processes ``batch`` sequences at once;
* bf16 tensor-core GEMMs (tcgen05) with fused epilogues (residual add, GELU /
  SwiGLU, their backward), fp32 residual stream and fp32 master weights;
* one flat parameter arena (fp32 master, grads, moments, bf16 working copy),
  sharded over data-parallel ranks (ZeRO-1): gradients are reduce-scattered,
  each rank runs AdamW on its shard, bf16 weights are all-gathered;
* the whole step is captured into one CUDA graph (single rank) so the ~280
  launches of a 12-layer step cost one graph launch on the host.

Supported family: RMSNorm + RoPE dense decoders (GELU FFN with biases, as the
reference trains, or SwiGLU without biases), head_dim 64/128, seq % 128 == 0 —
the same restriction as the reference's ``Supports`` (DeviceDecoderTrainer.cs:104-110)
plus the SwiGLU extension.
"""
from __future__ import annotations

import math
import os
import time
from typing import Dict, List, Optional, Sequence

import torch

from .. import ops
from ..ops import moe as moe_ops
from ..utils.trace import nvtx_range
from ..models.config import DecoderLmConfig
from ..models.decoder_lm import DecoderLM, rope_tables
from .arena import ParamArena, ParamSpec


def supports(cfg: DecoderLmConfig, seq: Optional[int] = None) -> bool:
    """True when ``cfg`` can run on the fused device path."""
    s = seq or cfg.max_seq
    moe_ok = cfg.num_experts == 0 or moe_ops.supported(cfg.dim, cfg.ff_dim, cfg.num_experts, cfg.moe_top_k)
    return (cfg.use_rms_norm and cfg.use_rope and cfg.block_pattern is None and moe_ok
            and cfg.num_loops == 1 and cfg.mtp_weight == 0 and not cfg.use_plan and cfg.dropout == 0
            and cfg.head_dim in (64, 128) and s % 128 == 0 and cfg.dim % 64 == 0 and cfg.ff_dim % 64 == 0)


def _interleave_gate_up(gate_t: torch.Tensor, up_t: torch.Tensor) -> torch.Tensor:
    """[F, D] gate and up rows -> [2F, D] with 64-row groups [gate_g | up_g] (the SwiGLU epilogue layout)."""
    F_, D = gate_t.shape
    g = gate_t.reshape(F_ // 64, 64, D)
    u = up_t.reshape(F_ // 64, 64, D)
    return torch.stack((g, u), dim=1).reshape(2 * F_, D)


def _split_gate_up(w13: torch.Tensor):
    F2, D = w13.shape
    x = w13.reshape(F2 // 128, 2, 64, D)
    return x[:, 0].reshape(F2 // 2, D), x[:, 1].reshape(F2 // 2, D)


class FusedDecoderTrainer:
    """One data-parallel rank of the fused decoder training step."""

    def __init__(self, cfg: DecoderLmConfig, batch: int, seq: Optional[int] = None, *, device="cuda",
                 lr: float = 3e-4, weight_decay: float = 0.1, betas=(0.9, 0.999), eps: float = 1e-8,
                 clip_norm: float = 0.0, seed: int = 42, model: Optional[DecoderLM] = None,
                 decay_all: bool = True, process_group=None, grad_sync: str = "auto", use_graph: bool = True):
        seq = seq or cfg.max_seq
        if not supports(cfg, seq):
            raise NotImplementedError("FusedDecoderTrainer needs an RMSNorm+RoPE config (head_dim 64/128, "
                                      "seq % 128 == 0; with experts: dim and ff_dim % 256 == 0, <= 64 experts, "
                                      "top-k <= 8); use the autograd path.")
        self.cfg, self.B, self.S = cfg, batch, seq
        self.M = batch * seq
        self.device = torch.device(device)
        self.lr, self.wd, self.betas, self.eps, self.clip_norm = lr, weight_decay, betas, eps, clip_norm
        self.t = 0
        self.use_graph = use_graph
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.tokens_seen = 0

        # ---------------- data parallel
        self.pg = process_group
        if self.pg is not None:
            import torch.distributed as dist
            self.world, self.rank = dist.get_world_size(self.pg), dist.get_rank(self.pg)
        else:
            self.world, self.rank = 1, 0
        if grad_sync == "auto":
            grad_sync = "fused" if self.world > 1 else "none"
        if self.world == 1:
            grad_sync = "none"
        if grad_sync not in ("none", "zero", "fused"):
            raise ValueError(f"grad_sync must be 'none', 'zero' (NCCL) or 'fused' (peer memory), got {grad_sync!r}")
        self.grad_sync = grad_sync
        self.peer = None

        # ---------------- parameters
        D, F_, L = cfg.dim, cfg.ff_dim, cfg.num_blocks
        # vocabulary rows padded to a multiple of 8 (16-byte TMA strides); the padded rows stay zero
        # and the cross-entropy only sees the real columns
        self.Vr = cfg.vocab
        V = self.Vp = (cfg.vocab + 7) // 8 * 8
        specs = [ParamSpec("wemb", (V, D))]
        for l in range(L):
            specs.append(ParamSpec(f"b{l}.wqkv", (3 * D, D)))
            specs.append(ParamSpec(f"b{l}.wo", (D, D)))
            if cfg.num_experts > 0:
                # expert e's blocks: router row e, W1_e^T rows [e F, (e+1) F), W2_e^T rows [e D, (e+1) D)
                E = cfg.num_experts
                specs.append(ParamSpec(f"b{l}.router", (E, D)))
                specs.append(ParamSpec(f"b{l}.ew1", (E * F_, D)))
                specs.append(ParamSpec(f"b{l}.ew2", (E * D, F_)))
                continue
            if cfg.ffn == "swiglu":
                specs.append(ParamSpec(f"b{l}.w13", (2 * F_, D)))
            else:
                specs.append(ParamSpec(f"b{l}.w1", (F_, D)))
            specs.append(ParamSpec(f"b{l}.w2", (D, F_)))
        specs.append(ParamSpec("wout", (V, D)))
        for l in range(L):
            specs.append(ParamSpec(f"b{l}.ln1", (D,), decay_all))
            specs.append(ParamSpec(f"b{l}.ln2", (D,), decay_all))
            if cfg.num_experts > 0:
                specs.append(ParamSpec(f"b{l}.eb1", (cfg.num_experts * F_,), decay_all))
                specs.append(ParamSpec(f"b{l}.eb2", (cfg.num_experts * D,), decay_all))
            elif cfg.ffn == "gelu":
                specs.append(ParamSpec(f"b{l}.b1", (F_,), decay_all))
                specs.append(ParamSpec(f"b{l}.b2", (D,), decay_all))
        specs.append(ParamSpec("lnf", (D,), decay_all))
        # fused data parallel: one bucket per group of tensors whose gradients become final together,
        # in backward order; every rank owns an equal piece of every bucket
        self.arena = ParamArena(specs, self.world, buckets=self._bucket_names() if grad_sync == "fused" else None)
        A = self.arena
        dev = self.device
        f32, bf16 = torch.float32, torch.bfloat16
        if grad_sync == "fused":
            # bf16 weights, gradient staging and the clip-norm slots live in IPC-shared buffers: during the
            # backward the copy engines push each finished bucket's pieces into their owners' staging slots;
            # after it, each owner reduces its pieces, clips, runs AdamW and stores bf16 weights to every peer
            from ..parallel.peer import PeerGroup
            self.peer = PeerGroup(self.pg, dev)
            self._w16_sym = self.peer.symmetric(A.total, bf16)
            self._stage_sym = self.peer.symmetric(self.world * A.shard, f32)
            self._norm_sym = self.peer.symmetric(self.world, torch.float64)
            self.w16 = self._w16_sym.local
            self.grad = torch.zeros(A.total, device=dev, dtype=f32)      # this rank's full local gradient
            self.gshard = torch.zeros(A.shard, device=dev, dtype=f32)    # reduced gradient of the owned pieces
            self.sumsq = torch.zeros(1, device=dev, dtype=torch.float64)
            self._tab = torch.tensor([list(p) for p in A.pieces(self.rank)], dtype=torch.int64, device=dev)
            self._plans = [self.push_plan(A, self.rank, b) for b in range(len(A.buckets))]
            self._push_stream = torch.cuda.Stream(dev, priority=-1)
            self._bucket_events = [torch.cuda.Event() for _ in A.buckets]
        else:
            self.w16 = torch.zeros(A.total, device=dev, dtype=bf16)      # full bf16 working copy (replicated)
            self.grad = torch.zeros(A.total, device=dev, dtype=f32)      # full gradient (local, then reduced)
        lo, hi = self.rank * A.shard, (self.rank + 1) * A.shard
        self.shard_lo, self.shard_hi = lo, hi
        self.w32 = torch.zeros(A.shard, device=dev, dtype=f32)       # fp32 master shard
        self.m = torch.zeros(A.shard, device=dev, dtype=f32)
        self.v = torch.zeros(A.shard, device=dev, dtype=f32)
        self.grad_shard = self.grad[lo:hi] if self.world == 1 else torch.zeros(A.shard, device=dev, dtype=f32)
        self.n_decay_local = max(0, min(A.n_decay - lo, A.shard))
        self.hyper_host = torch.zeros(8, dtype=f32).pin_memory()
        self._hyper_np = self.hyper_host.numpy()   # host writes through numpy: no torch op per field
        # the pinned staging buffers are rewritten only after the copies that read them have run
        self._h2d_ev = torch.cuda.Event() if torch.device(device).type == "cuda" else None
        self._h2d_pending = False
        self.hyper = torch.zeros(8, device=dev, dtype=f32)
        self.clip_buf = torch.zeros(1, device=dev, dtype=f32)
        self.W = A.views(self.w16)   # bf16 views by name
        self.G = A.views(self.grad)  # fp32 grad views by name

        if model is None:
            model = DecoderLM(cfg, seed=seed)
        self.import_model(model)

        # ---------------- activations
        M, S, H, hd = self.M, seq, cfg.num_heads, cfg.head_dim
        z = lambda *shape, dt=bf16: torch.empty(*shape, device=dev, dtype=dt)
        self.tok = torch.zeros(M, device=dev, dtype=torch.int32)
        self.tgt = torch.zeros(M, device=dev, dtype=torch.int32)
        self.tok_pin = torch.zeros(M, dtype=torch.int32).pin_memory()
        self.tgt_pin = torch.zeros(M, dtype=torch.int32).pin_memory()
        self.loss_pin = torch.zeros(1, dtype=f32).pin_memory()
        # step_pipelined: each step's loss leaves through one of two pinned slots, read one step later
        self._loss_slots = [torch.zeros(1, dtype=f32).pin_memory() for _ in range(2)]
        self._loss_ev = [torch.cuda.Event() for _ in range(2)] if torch.device(dev).type == "cuda" else None
        self._pipe_pending: Optional[int] = None
        self._pipe_n = 0
        self.x = [z(M, D, dt=f32) for _ in range(L + 1)]
        self.xmid = [z(M, D, dt=f32) for _ in range(L)]
        self.n1 = [z(M, D) for _ in range(L)]
        self.n2 = [z(M, D) for _ in range(L)]
        self.inv1 = [z(M, dt=f32) for _ in range(L)]
        self.inv2 = [z(M, dt=f32) for _ in range(L)]
        self.qkv = [z(M, 3 * D) for _ in range(L)]
        self.ao = [z(M, D) for _ in range(L)]
        self.lse = [z(batch * H, S, dt=f32) for _ in range(L)]
        fpre = 2 * F_ if cfg.ffn == "swiglu" else F_
        if cfg.num_experts > 0:
            E, k = cfg.num_experts, cfg.moe_top_k
            self.moe = [moe_ops.MoEBuffers.allocate(M, D, F_, E, k, dev) for _ in range(L)]
            self.moe_scr = moe_ops.MoEScratch.allocate(M, D, F_, E, k, dev)
            self.moe_aux = z(1, dt=f32)   # weighted balance losses of the step (in summed-row units)
            self.pre, self.act = [], []
        else:
            self.moe = None
            self.pre = [z(M, fpre) for _ in range(L)]
            self.act = [z(M, F_) for _ in range(L)]
        self.nf = z(M, D)
        self.invf = z(M, dt=f32)
        self.logits = z(M, V)
        self.loss_rows = z(M, dt=f32)
        self.loss_sum = z(1, dt=f32)
        # backward scratch
        self.dx = z(M, D, dt=f32)
        self.dx16 = z(M, D)
        self.dn = z(M, D, dt=f32)
        self.dpre = z(M, fpre) if cfg.num_experts == 0 else None
        self.dao = z(M, D)
        self.dqkv = z(M, 3 * D)
        self.dq_acc = z(M, D, dt=f32)
        self.dvec = z(batch * H, S, dt=f32)
        cos, sin = rope_tables(S, hd, 0, device=dev)
        self.rope_cs = torch.stack((cos, sin), dim=-1).contiguous()  # [S, hd/2, 2]
        self.attn_scale = 1.0 / math.sqrt(hd)
        self.launches_per_step = None
        # Weight-gradient GEMMs on a second stream (SwiGLU dense blocks): they feed only the optimizer, so
        # they fill the SMs that the chain of input gradients, norms and attention leaves idle (tails of
        # persistent grids, memory-bound kernels).  The bf16 gradient buffers they read come in two
        # copies, so the chain writes one while a weight-gradient GEMM still reads the other.
        # PCB_WGRAD_STREAM=0 keeps every GEMM on one stream.
        self._wg_stream = None
        self._wg_read: Dict[tuple, torch.cuda.Event] = {}
        if (torch.device(dev).type == "cuda" and os.environ.get("PCB_WGRAD_STREAM", "1") != "0"
                and cfg.num_experts == 0 and cfg.ffn == "swiglu"):
            self._wg_stream = torch.cuda.Stream(dev)
            self.dx16_pp = [self.dx16, z(M, D)]
            self.dpre_pp = [self.dpre, z(M, fpre)]
            self.dqkv_pp = [self.dqkv, z(M, 3 * D)]

    def _bucket_names(self) -> List[List[str]]:
        """Tensor groups in the order the backward finishes their gradients: LM head + final norm,
        then the blocks from last to first, then the embedding."""
        cfg = self.cfg
        out = [["wout", "lnf"]]
        for l in reversed(range(cfg.num_blocks)):
            names = [f"b{l}.wqkv", f"b{l}.wo", f"b{l}.ln1", f"b{l}.ln2"]
            if cfg.num_experts > 0:
                names += [f"b{l}.router", f"b{l}.ew1", f"b{l}.ew2", f"b{l}.eb1", f"b{l}.eb2"]
            elif cfg.ffn == "swiglu":
                names += [f"b{l}.w2", f"b{l}.w13"]
            else:
                names += [f"b{l}.w2", f"b{l}.w1", f"b{l}.b1", f"b{l}.b2"]
            out.append(names)
        out.append(["wemb"])
        return out

    @staticmethod
    def push_plan(arena: ParamArena, rank: int, b: int):
        """Copies that send this rank's finished bucket ``b`` to the other ranks:
        (owner rank q, element offset in q's staging buffer, element offset in the local gradient,
        element count).  Owner q's staging buffer holds one slot of ``arena.shard`` elements per source
        rank, in q's local (pieces) order."""
        world = arena.world
        start, end, _ = arena.buckets[b]
        c = (end - start) // world
        loff = arena.pieces(rank)[b][0]
        plan = []
        for k in range(1, world):          # start with the next rank, so the ranks spread their pushes
            q = (rank + k) % world
            plan.append((q, rank * arena.shard + loff, start + q * c, c))
        return plan

    def _bucket_done(self, b: int) -> None:
        """Bucket ``b``'s gradient is final on this rank: push its pieces to their owners (copy engines,
        on the push stream, ordered after the kernels that produced them)."""
        if self.grad_sync != "fused":
            return
        ev = self._bucket_events[b]
        ev.record(torch.cuda.current_stream(self.device))
        s = self._push_stream
        s.wait_event(ev)
        if self._wg_stream is not None:
            s.wait_stream(self._wg_stream)   # the bucket's weight gradients come from the side stream
        base = self.grad.data_ptr()
        with torch.cuda.stream(s):
            for q, dst, src, n in self._plans[b]:
                ops.ext().memcpy_d2d(self._stage_sym.host_ptrs[q] + 4 * dst, base + 4 * src, 4 * n)

    # ------------------------------------------------------------------ weights in/out
    def _model_to_flat(self, model: DecoderLM) -> torch.Tensor:
        """DecoderLM tensors (reference [in,out] layout) -> flat fp32 arena (cpu)."""
        cfg = self.cfg
        full = torch.zeros(self.arena.total, dtype=torch.float32)
        V = self.arena.views(full)
        V["wemb"][:self.Vr].copy_(model.wemb.detach().float().cpu())
        for l, blk in enumerate(model.blocks):
            V[f"b{l}.wqkv"].copy_(torch.cat([blk.wq.T, blk.wk.T, blk.wv.T], 0).detach().cpu())
            V[f"b{l}.wo"].copy_(blk.wo.detach().T.cpu())
            V[f"b{l}.ln1"].copy_(blk.ln1_g.detach().cpu())
            V[f"b{l}.ln2"].copy_(blk.ln2_g.detach().cpu())
            if cfg.num_experts > 0:
                E, D, F_ = cfg.num_experts, cfg.dim, cfg.ff_dim
                V[f"b{l}.router"].copy_(blk.router.detach().T.cpu())
                for e in range(E):
                    V[f"b{l}.ew1"][e * F_:(e + 1) * F_].copy_(blk.ew1[e].detach().T.cpu())
                    V[f"b{l}.ew2"][e * D:(e + 1) * D].copy_(blk.ew2[e].detach().T.cpu())
                    V[f"b{l}.eb1"][e * F_:(e + 1) * F_].copy_(blk.eb1[e].detach().cpu())
                    V[f"b{l}.eb2"][e * D:(e + 1) * D].copy_(blk.eb2[e].detach().cpu())
                continue
            if cfg.ffn == "swiglu":
                V[f"b{l}.w13"].copy_(_interleave_gate_up(blk.w1.detach().T.cpu(), blk.w3.detach().T.cpu()))
            else:
                V[f"b{l}.w1"].copy_(blk.w1.detach().T.cpu())
                V[f"b{l}.b1"].copy_(blk.b1.detach().cpu())
                V[f"b{l}.b2"].copy_(blk.b2.detach().cpu())
            V[f"b{l}.w2"].copy_(blk.w2.detach().T.cpu())
        V["lnf"].copy_(model.lnf_g.detach().cpu())
        V["wout"][:self.Vr].copy_(model.wout.detach().T.cpu())
        return full

    @torch.no_grad()
    def import_model(self, model: DecoderLM) -> None:
        """Copy a DecoderLM's weights (reference [in,out] layout) into the arena."""
        full_d = self._model_to_flat(model).to(self.device)
        self.w32.copy_(self.arena.gather_local(full_d, self.rank))
        self.w16.copy_(full_d.to(torch.bfloat16))
        self.m.zero_()
        self.v.zero_()
        self.t = 0

    @torch.no_grad()
    def master_weights(self) -> torch.Tensor:
        """Full fp32 master buffer (all-gathered across ranks)."""
        return self._gather_full(self.w32)

    @torch.no_grad()
    def _flat_to_model(self, flat: torch.Tensor, model: DecoderLM) -> DecoderLM:
        cfg = self.cfg
        V = self.arena.views(flat.cpu())
        model.wemb.copy_(V["wemb"][:self.Vr])
        D = cfg.dim
        for l, blk in enumerate(model.blocks):
            wqkv = V[f"b{l}.wqkv"]
            blk.wq.copy_(wqkv[:D].T)
            blk.wk.copy_(wqkv[D:2 * D].T)
            blk.wv.copy_(wqkv[2 * D:].T)
            blk.wo.copy_(V[f"b{l}.wo"].T)
            blk.ln1_g.copy_(V[f"b{l}.ln1"])
            blk.ln2_g.copy_(V[f"b{l}.ln2"])
            if cfg.num_experts > 0:
                E, F_ = cfg.num_experts, cfg.ff_dim
                blk.router.copy_(V[f"b{l}.router"].T)
                for e in range(E):
                    blk.ew1[e].copy_(V[f"b{l}.ew1"][e * F_:(e + 1) * F_].T)
                    blk.ew2[e].copy_(V[f"b{l}.ew2"][e * D:(e + 1) * D].T)
                    blk.eb1[e].copy_(V[f"b{l}.eb1"][e * F_:(e + 1) * F_])
                    blk.eb2[e].copy_(V[f"b{l}.eb2"][e * D:(e + 1) * D])
                continue
            if cfg.ffn == "swiglu":
                g, u = _split_gate_up(V[f"b{l}.w13"])
                blk.w1.copy_(g.T)
                blk.w3.copy_(u.T)
            else:
                blk.w1.copy_(V[f"b{l}.w1"].T)
                blk.b1.copy_(V[f"b{l}.b1"])
                blk.b2.copy_(V[f"b{l}.b2"])
            blk.w2.copy_(V[f"b{l}.w2"].T)
        model.lnf_g.copy_(V["lnf"])
        model.wout.copy_(V["wout"][:self.Vr].T)
        return model

    @torch.no_grad()
    def export_model(self, model: Optional[DecoderLM] = None) -> DecoderLM:
        """Write the fp32 master weights back into a DecoderLM (reference layout)."""
        return self._flat_to_model(self.master_weights(), model if model is not None else DecoderLM(self.cfg))

    def _gather_full(self, shard: torch.Tensor) -> torch.Tensor:
        """Full flat buffer from every rank's local shard (the ranks' pieces put back in place)."""
        if self.world == 1:
            return shard.clone()
        import torch.distributed as dist
        A = self.arena
        out = torch.empty(self.world * A.shard, device=self.device, dtype=torch.float32)
        dist.all_gather_into_tensor(out, shard.contiguous(), group=self.pg)
        if not A.buckets:
            return out
        full = torch.zeros(A.total, device=self.device, dtype=torch.float32)
        for r in range(self.world):
            A.scatter_local(out[r * A.shard:(r + 1) * A.shard], r, full)
        return full

    @torch.no_grad()
    def save_state(self, path: str) -> None:
        """Adam moments and step count in the device-trainer state file (DAM1), tensors in the
        reference Parameters() order and layout (DeviceDecoderTrainer.SaveState)."""
        from ..io.checkpoint import save_dam1
        moms = []
        for buf in (self._gather_full(self.m), self._gather_full(self.v)):
            moms.append([t.detach().reshape(-1).numpy().copy() for t in
                         self._flat_to_model(buf, DecoderLM(self.cfg)).reference_parameters()])
        if self.rank == 0:
            save_dam1(path, self.t, list(zip(moms[0], moms[1])))

    @torch.no_grad()
    def load_state(self, path: str) -> None:
        from ..io.checkpoint import load_dam1
        ref = DecoderLM(self.cfg)
        counts = [p.numel() for p in ref.reference_parameters()]
        t, moms = load_dam1(path, counts)
        for k, buf in ((0, self.m), (1, self.v)):
            tensors = [torch.from_numpy(mv[k].copy()).view_as(p) for mv, p in zip(moms, ref.reference_parameters())]
            ref.load_reference_parameters([x.numpy() for x in tensors])
            full = self._model_to_flat(ref).to(self.device)
            buf.copy_(self.arena.gather_local(full, self.rank))
        self.t = int(t)

    # ------------------------------------------------------------------ the step
    def _forward(self, write_grad: bool = True) -> None:
        cfg = self.cfg
        W = self.W
        B, S, M, D, H, hd = self.B, self.S, self.M, cfg.dim, cfg.num_heads, cfg.head_dim
        ops.embed_fwd(self.tok, W["wemb"], self.x[0])
        if self.moe is not None:
            self.moe_aux.zero_()
        for l in range(cfg.num_blocks):
            ops.rmsnorm_fwd(self.x[l], W[f"b{l}.ln1"], self.n1[l], self.inv1[l], cfg.eps)
            ops.gemm(self.n1[l], W[f"b{l}.wqkv"], epi=ops.EPI_BF16, c=self.qkv[l],
                     rope=(self.rope_cs, S, hd, 2 * D))
            ops.attn_fwd(self.qkv[l], self.ao[l], self.lse[l], B, S, H, hd, self.attn_scale)
            ops.gemm(self.ao[l], W[f"b{l}.wo"], epi=ops.EPI_RESID_F32, c=self.xmid[l], aux=self.x[l])
            ops.rmsnorm_fwd(self.xmid[l], W[f"b{l}.ln2"], self.n2[l], self.inv2[l], cfg.eps)
            if self.moe is not None:
                moe_ops.forward(self.n2[l], self.xmid[l], self.x[l + 1], W[f"b{l}.router"], W[f"b{l}.ew1"],
                                W[f"b{l}.eb1"], W[f"b{l}.ew2"], W[f"b{l}.eb2"], cfg.moe_top_k, self.moe[l],
                                self.moe_aux, cfg.moe_balance_weight * M)
            elif cfg.ffn == "swiglu":
                ops.gemm(self.n2[l], W[f"b{l}.w13"], epi=ops.EPI_SWIGLU, c=self.pre[l], d=self.act[l])
                ops.gemm(self.act[l], W[f"b{l}.w2"], epi=ops.EPI_RESID_F32, c=self.x[l + 1], aux=self.xmid[l])
            else:
                ops.gemm(self.n2[l], W[f"b{l}.w1"], epi=ops.EPI_GELU, c=self.pre[l], d=self.act[l],
                         bias=W[f"b{l}.b1"])
                ops.gemm(self.act[l], W[f"b{l}.w2"], epi=ops.EPI_RESID_F32, c=self.x[l + 1], aux=self.xmid[l],
                         bias=W[f"b{l}.b2"])
        L = cfg.num_blocks
        ops.rmsnorm_fwd(self.x[L], W["lnf"], self.nf, self.invf, cfg.eps)
        ops.gemm(self.nf, W["wout"], epi=ops.EPI_BF16, c=self.logits)
        ops.cross_entropy(self.logits[:, :self.Vr], self.tgt, self.loss_rows, 1.0 / M, write_grad)
        self.loss_sum.zero_()
        ops.sumsq(self.loss_rows, self.loss_sum, square=False)
        if self.moe is not None:
            ops.sumsq(self.moe_aux, self.loss_sum, square=False)

    def _backward(self) -> None:
        if self._wg_stream is not None:
            self._backward_two_streams()
            return
        cfg = self.cfg
        W, G = self.W, self.G
        B, S, D, H, hd = self.B, self.S, cfg.dim, cfg.num_heads, cfg.head_dim
        L = cfg.num_blocks
        RED = ops.EPI_RED_F32
        dl = self.logits  # holds dlogits after the fused CE
        ops.gemm(dl, self.nf, a_mn=True, b_mn=True, epi=RED, c=G["wout"])           # dWout = dL^T nf
        ops.gemm(dl, W["wout"], b_mn=True, epi=ops.EPI_F32, c=self.dn)              # dnf = dL Wout
        ops.rmsnorm_bwd(self.dn, self.x[L], W["lnf"], self.invf, self.dx, G["lnf"], False, self.dx16)
        self._bucket_done(0)
        for l in reversed(range(L)):
            # ---- FFN: x_{l+1} = xmid + ffn(norm2(xmid))
            if self.moe is not None:
                moe_ops.backward(self.dx, self.n2[l], self.dn, W[f"b{l}.router"], W[f"b{l}.ew1"], W[f"b{l}.ew2"],
                                 cfg.moe_top_k, self.moe[l], self.moe_scr, G[f"b{l}.router"], G[f"b{l}.ew1"],
                                 G[f"b{l}.eb1"], G[f"b{l}.ew2"], G[f"b{l}.eb2"], cfg.moe_balance_weight)
            elif cfg.ffn == "swiglu":
                ops.gemm(self.dx16, self.act[l], a_mn=True, b_mn=True, epi=RED, c=G[f"b{l}.w2"])
                ops.gemm(self.dx16, W[f"b{l}.w2"], b_mn=True, epi=ops.EPI_SWIGLU_BWD, c=self.dpre, aux=self.pre[l])
                ops.gemm(self.dpre, self.n2[l], a_mn=True, b_mn=True, epi=RED, c=G[f"b{l}.w13"])
                ops.gemm(self.dpre, W[f"b{l}.w13"], b_mn=True, epi=ops.EPI_F32, c=self.dn)
            else:
                ops.gemm(self.dx16, self.act[l], a_mn=True, b_mn=True, epi=RED, c=G[f"b{l}.w2"])
                ops.colsum(self.dx16, G[f"b{l}.b2"])
                ops.gemm(self.dx16, W[f"b{l}.w2"], b_mn=True, epi=ops.EPI_GELU_BWD, c=self.dpre, aux=self.pre[l])
                ops.colsum(self.dpre, G[f"b{l}.b1"])
                ops.gemm(self.dpre, self.n2[l], a_mn=True, b_mn=True, epi=RED, c=G[f"b{l}.w1"])
                ops.gemm(self.dpre, W[f"b{l}.w1"], b_mn=True, epi=ops.EPI_F32, c=self.dn)
            ops.rmsnorm_bwd(self.dn, self.xmid[l], W[f"b{l}.ln2"], self.inv2[l], self.dx, G[f"b{l}.ln2"], True,
                            self.dx16)
            # ---- attention: xmid = x + attn(norm1(x)) Wo
            ops.gemm(self.dx16, self.ao[l], a_mn=True, b_mn=True, epi=RED, c=G[f"b{l}.wo"])
            ops.gemm(self.dx16, W[f"b{l}.wo"], b_mn=True, epi=ops.EPI_BF16, c=self.dao)
            ops.attn_bwd(self.qkv[l], self.ao[l], self.dao, self.lse[l], self.dvec, self.dq_acc, self.dqkv,
                         B, S, H, hd, self.attn_scale, self.rope_cs)
            ops.gemm(self.dqkv, self.n1[l], a_mn=True, b_mn=True, epi=RED, c=G[f"b{l}.wqkv"])
            ops.gemm(self.dqkv, W[f"b{l}.wqkv"], b_mn=True, epi=ops.EPI_F32, c=self.dn)
            ops.rmsnorm_bwd(self.dn, self.x[l], W[f"b{l}.ln1"], self.inv1[l], self.dx, G[f"b{l}.ln1"], True,
                            self.dx16)
            self._bucket_done(L - l)
        ops.embed_bwd(self.tok, self.dx, G["wemb"])
        self._bucket_done(L + 1)

    def _backward_two_streams(self) -> None:
        """The SwiGLU backward of ``_backward`` with every weight-gradient GEMM (dW += dY^T X, fp32
        reduce epilogue) on the side stream.  Each one forks from the main stream after its inputs are
        written; before the main stream rewrites a bf16 gradient copy it waits for the weight-gradient
        GEMM that last read it; the main stream joins the side stream at the end."""
        cfg = self.cfg
        W, G = self.W, self.G
        B, S, D, H, hd = self.B, self.S, cfg.dim, cfg.num_heads, cfg.head_dim
        L = cfg.num_blocks
        RED = ops.EPI_RED_F32
        main = torch.cuda.current_stream(self.device)
        side = self._wg_stream
        read = self._wg_read

        def wgrad(dy, x, g, key):
            side.wait_stream(main)
            with torch.cuda.stream(side):
                ops.gemm(dy, x, a_mn=True, b_mn=True, epi=RED, c=g)
            if key is not None:
                ev = torch.cuda.Event()
                ev.record(side)
                read[key] = ev

        def claim(key):
            ev = read.pop(key, None)
            if ev is not None:
                main.wait_event(ev)

        dx16, dpre, dqkv = self.dx16_pp, self.dpre_pp, self.dqkv_pp
        dl = self.logits  # holds dlogits after the fused CE (not rewritten during the backward)
        wgrad(dl, self.nf, G["wout"], None)                                           # dWout = dL^T nf
        ops.gemm(dl, W["wout"], b_mn=True, epi=ops.EPI_F32, c=self.dn)                # dnf = dL Wout
        k = 0
        claim(("dx16", k))
        ops.rmsnorm_bwd(self.dn, self.x[L], W["lnf"], self.invf, self.dx, G["lnf"], False, dx16[k])
        self._bucket_done(0)
        for l in reversed(range(L)):
            p = l & 1
            wgrad(dx16[k], self.act[l], G[f"b{l}.w2"], ("dx16", k))
            claim(("dpre", p))
            ops.gemm(dx16[k], W[f"b{l}.w2"], b_mn=True, epi=ops.EPI_SWIGLU_BWD, c=dpre[p], aux=self.pre[l])
            wgrad(dpre[p], self.n2[l], G[f"b{l}.w13"], ("dpre", p))
            ops.gemm(dpre[p], W[f"b{l}.w13"], b_mn=True, epi=ops.EPI_F32, c=self.dn)
            k ^= 1
            claim(("dx16", k))
            ops.rmsnorm_bwd(self.dn, self.xmid[l], W[f"b{l}.ln2"], self.inv2[l], self.dx, G[f"b{l}.ln2"], True,
                            dx16[k])
            wgrad(dx16[k], self.ao[l], G[f"b{l}.wo"], ("dx16", k))
            ops.gemm(dx16[k], W[f"b{l}.wo"], b_mn=True, epi=ops.EPI_BF16, c=self.dao)
            claim(("dqkv", p))
            ops.attn_bwd(self.qkv[l], self.ao[l], self.dao, self.lse[l], self.dvec, self.dq_acc, dqkv[p],
                         B, S, H, hd, self.attn_scale, self.rope_cs)
            wgrad(dqkv[p], self.n1[l], G[f"b{l}.wqkv"], ("dqkv", p))
            ops.gemm(dqkv[p], W[f"b{l}.wqkv"], b_mn=True, epi=ops.EPI_F32, c=self.dn)
            k ^= 1
            claim(("dx16", k))
            ops.rmsnorm_bwd(self.dn, self.x[l], W[f"b{l}.ln1"], self.inv1[l], self.dx, G[f"b{l}.ln1"], True,
                            dx16[k])
            self._bucket_done(L - l)
        ops.embed_bwd(self.tok, self.dx, G["wemb"])
        self._bucket_done(L + 1)
        main.wait_stream(side)   # every weight gradient is complete before the optimizer
        read.clear()

    def _optimizer(self) -> None:
        """Gradient sync (data parallel) + AdamW on this rank's shard + bf16 weight refresh."""
        if self.grad_sync == "fused":
            A = self.arena
            torch.cuda.current_stream(self.device).wait_stream(self._push_stream)
            self.peer.barrier()   # every rank's pushes into every staging buffer are complete
            self.sumsq.zero_()
            ops.ext().dp_reduce_sumsq(self.grad, self._stage_sym.local, A.shard, self._tab, self.rank, self.world,
                                      self.gshard, self.sumsq)
            slots = None
            if self.clip_norm > 0:
                ops.ext().dp_norm_push(self.sumsq, self._norm_sym.ptrs, self.rank, self.world)
                self.peer.barrier()   # every rank's partial sum of squares has arrived
                slots = self._norm_sym.local
            ops.ext().dp_adamw_ag(self.gshard, self.w32, self.m, self.v, self._w16_sym.ptrs, A.shard, self._tab,
                                  self.hyper, self.betas[0], self.betas[1], self.eps, slots, float(self.clip_norm),
                                  self.world)
            self.peer.barrier()   # every rank's weights are written before anyone's next forward
            return
        if self.world > 1:
            import torch.distributed as dist
            dist.reduce_scatter_tensor(self.grad_shard, self.grad, group=self.pg)
        clip = None
        if self.clip_norm > 0:
            self.clip_buf.zero_()
            ops.sumsq(self.grad_shard, self.clip_buf, square=True)
            if self.world > 1:
                import torch.distributed as dist
                dist.all_reduce(self.clip_buf, group=self.pg)
            clip = self.clip_buf
        w16_shard = self.w16[self.shard_lo:self.shard_hi]
        ops.adamw(self.w32, self.grad_shard, self.m, self.v, w16_shard, self.n_decay_local, self.hyper,
                  self.betas[0], self.betas[1], self.eps, clip, self.clip_norm)
        if self.world > 1:
            import torch.distributed as dist
            dist.all_gather_into_tensor(self.w16, w16_shard, group=self.pg)

    def _upload(self) -> None:
        """Enqueue the host-to-device copies of the staged step (tokens, targets, hyper-parameters)."""
        self.tok.copy_(self.tok_pin, non_blocking=True)
        self.tgt.copy_(self.tgt_pin, non_blocking=True)
        self.hyper.copy_(self.hyper_host, non_blocking=True)
        if self._h2d_ev is not None:
            self._h2d_ev.record(torch.cuda.current_stream(self.device))
            self._h2d_pending = True

    def _host_writable(self) -> None:
        """Wait until the last upload has read the pinned buffers (the GPU may be a step behind)."""
        if self._h2d_pending:
            self._h2d_ev.synchronize()
            self._h2d_pending = False

    def _step_body(self) -> None:
        self._upload()
        self._device_step()

    def _device_step(self) -> None:
        """Everything of a step after the uploads: captured as one CUDA graph."""
        self.grad.zero_()
        with nvtx_range("forward"):
            self._forward(True)
        with nvtx_range("backward"):
            self._backward()
        with nvtx_range("optimizer"):
            self._optimizer()
        self.loss_pin.copy_(self.loss_sum, non_blocking=True)

    def _set_hyper(self, lr: float) -> None:
        self._host_writable()
        self.t += 1
        b1, b2 = self.betas
        h = self._hyper_np
        h[0] = lr
        h[1] = self.wd
        h[2] = 1.0 - b1 ** self.t
        h[3] = 1.0 - b2 ** self.t
        # gradients are sums over ranks of per-rank means: fold the 1/world mean here
        h[4] = 1.0 / self.world

    def stage(self, tokens: torch.Tensor, targets: torch.Tensor) -> None:
        """Copy one step's [B, S] int tokens/targets into the pinned staging buffers."""
        self._host_writable()
        self.tok_pin.copy_(tokens.reshape(-1))      # copy_ converts the dtype in place
        self.tgt_pin.copy_(targets.reshape(-1))

    def launch(self, lr: Optional[float] = None) -> None:
        """Enqueue one full training step on the current stream (no host sync)."""
        self._set_hyper(self.lr if lr is None else lr)
        if self.use_graph and self.grad_sync in ("none", "fused"):
            if self.graph is None:
                self._capture()
            self._upload()
            self.graph.replay()
        else:
            self._step_body()
        self.tokens_seen += self.M

    def _capture(self) -> None:
        # one eager step first: sets kernel attributes and driver entry points outside capture,
        # then restore the state it touched so the captured step starts from the same place
        w32, w16, m, v = self.w32.clone(), self.w16.clone(), self.m.clone(), self.v.clone()
        before = ops.launch_count()
        self._step_body()
        torch.cuda.synchronize(self.device)
        self.launches_per_step = ops.launch_count() - before
        self.w32.copy_(w32); self.w16.copy_(w16); self.m.copy_(m); self.v.copy_(v)
        del w32, w16, m, v
        self.graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            with torch.cuda.graph(self.graph, stream=s):
                self._device_step()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)

    def read_loss(self) -> float:
        """Synchronise and return the mean loss of the last launched step."""
        torch.cuda.current_stream(self.device).synchronize()
        return float(self.loss_pin[0]) / self.M

    def step(self, tokens: torch.Tensor, targets: torch.Tensor, lr: Optional[float] = None) -> float:
        """Public API: one training step on host tokens/targets [B, S]; returns the mean loss."""
        self.stage(tokens, targets)
        self.launch(lr)
        return self.read_loss()

    def step_pipelined(self, tokens: torch.Tensor, targets: torch.Tensor,
                       lr: Optional[float] = None) -> Optional[float]:
        """Public API for a training loop that never leaves the GPU waiting on the host: stage and launch
        this step, then return the mean loss of the previous one (None on the first call; ``flush()``
        returns the last).  The host prepares step i+1 while step i runs.  Every step still copies its
        tokens and targets from pinned memory to the device, and its loss comes back to the host: a
        4-byte copy, ordered after the step, into one of two pinned slots that alternate, so the slot
        read for step i is not rewritten before step i+2 is launched."""
        self.stage(tokens, targets)
        self.launch(lr)
        slot = self._pipe_n & 1
        self._pipe_n += 1
        self._loss_slots[slot].copy_(self.loss_sum, non_blocking=True)
        self._loss_ev[slot].record(torch.cuda.current_stream(self.device))
        prev, self._pipe_pending = self._pipe_pending, slot
        if prev is None:
            return None
        self._loss_ev[prev].synchronize()
        return float(self._loss_slots[prev][0]) / self.M

    def flush(self) -> Optional[float]:
        """Mean loss of the last step launched by ``step_pipelined`` (waits for that step only)."""
        prev, self._pipe_pending = self._pipe_pending, None
        if prev is None:
            return None
        self._loss_ev[prev].synchronize()
        return float(self._loss_slots[prev][0]) / self.M

    @torch.no_grad()
    def evaluate_loss(self, tokens: torch.Tensor, targets: torch.Tensor) -> float:
        """Mean CE without touching gradients or weights (DeviceDecoderTrainer.EvaluateLoss)."""
        self.stage(tokens, targets)
        self._upload()
        self._forward(write_grad=False)
        self.loss_pin.copy_(self.loss_sum, non_blocking=True)
        return self.read_loss()

    # ------------------------------------------------------------------ optimizer state
    def adam_state(self):
        return self.t, self.m, self.v

    def flops_per_step(self) -> float:
        """Model FLOPs of one step (6*N*T for the matmuls + causal attention fwd/bwd)."""
        cfg = self.cfg
        D, F_, V, L = cfg.dim, cfg.ff_dim, cfg.vocab, cfg.num_blocks
        if cfg.num_experts > 0:
            ffn = cfg.moe_top_k * 2 * D * F_ + D * cfg.num_experts   # k routed experts + the router
        else:
            ffn = (3 if cfg.ffn == "swiglu" else 2) * D * F_
        mat = L * (4 * D * D + ffn) + V * D
        attn = L * 2 * 2 * self.S * D / 2  # QK^T and PV, causal half, per token
        return 6.0 * mat * self.M + 3.0 * attn * self.M
