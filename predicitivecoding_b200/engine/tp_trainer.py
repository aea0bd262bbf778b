"""Tensor-parallel (+ sequence-parallel) decoder training step with the collectives fused into the GEMMs.

Reference: the reference's only tensor parallelism is a CPU column/row split of one matvec
(PredictiveCoding.LLM/Infrastructure/TensorParallel.cs:20-141: ``ShardedLinear.ForwardColumnParallel``
and ``ForwardRowParallel`` with ``DeviceMesh.AllReduceSum``).  This trainer runs the Megatron
layout for the dense RMSNorm/RoPE/SwiGLU decoder on T GPUs (one process each):

* attention heads and the FFN width are split across ranks (column-parallel W_qkv and W_13,
  row-parallel W_o and W_2); embeddings, LM head and norm gains are replicated;
* the residual stream is sequence-parallel: rank t owns rows [t*R, (t+1)*R) of the B*S tokens;
* column-parallel GEMMs read their input from a symmetric "gather" buffer: each rank writes its
  own normalised rows there, and the tcgen05 GEMM kernel itself copies the other ranks' rows over
  NVLink (epilogue warps, chunk by chunk in ring order, with per-chunk ready counters) while its
  first tiles compute on local rows -- the all-gather never exists as a separate collective;
* row-parallel GEMMs store each output tile directly into the owning rank's slot buffer (bf16,
  remote stores from the epilogue); the owner sums the T slots in rank order, adds the residual
  and applies the next RMSNorm in one kernel that writes straight into the next gather buffer;
* the backward mirrors it (dgrad of a row-parallel GEMM is a gather-GEMM, of a column-parallel
  one a reduce-scatter GEMM); replicated parameters' gradients are summed over ranks with the
  peer-memory all-reduce, then every rank runs AdamW on its parameters;
* with a data-parallel group (TP x DP, e.g. 4 x 2 on 8 GPUs) every TP replica trains its own batch;
  before AdamW the replicated and the sharded gradients are summed across the replicas (ranks with the
  same TP index) by the peer-memory all-reduce, and AdamW folds the 1/DP mean into its gradient scale.

All cross-rank ordering is by the bounded device barrier; nothing waits on the host.
"""
from __future__ import annotations

import math
import os
from typing import Optional

import torch
import torch.distributed as dist

from .. import ops
from ..utils.trace import nvtx_range
from ..models.config import DecoderLmConfig
from ..models.decoder_lm import DecoderLM, rope_tables
from .arena import ParamArena, ParamSpec


def _pad64(x: int) -> int:
    return (x + 63) // 64 * 64


def _interleave(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    F_, D = gate.shape
    return torch.stack((gate.reshape(F_ // 64, 64, D), up.reshape(F_ // 64, 64, D)), 1).reshape(2 * F_, D)


def tp_supports(cfg: DecoderLmConfig, batch: int, seq: int, world: int) -> bool:
    return (cfg.use_rms_norm and cfg.use_rope and cfg.ffn == "swiglu" and cfg.num_experts == 0
            and cfg.block_pattern is None and cfg.num_loops == 1 and not cfg.use_plan and cfg.mtp_weight == 0
            and cfg.head_dim in (64, 128) and cfg.num_heads % world == 0 and seq % 128 == 0
            and (batch * seq) % (256 * world) == 0 and cfg.dim % 8 == 0)


class TensorParallelTrainer:
    def __init__(self, cfg: DecoderLmConfig, batch: int, seq: Optional[int] = None, *, process_group=None,
                 device="cuda", lr: float = 3e-4, weight_decay: float = 0.1, betas=(0.9, 0.999), eps: float = 1e-8,
                 seed: int = 42, model: Optional[DecoderLM] = None, decay_all: bool = True, use_graph: bool = True,
                 dp_group=None):
        from ..parallel.collectives import Communicator
        from ..parallel.peer import PeerGroup
        seq = seq or cfg.max_seq
        self.pg = process_group
        self.T = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.t = dist.get_rank(process_group) if dist.is_initialized() else 0
        if not tp_supports(cfg, batch, seq, self.T):
            raise NotImplementedError("TensorParallelTrainer needs a dense RMSNorm+RoPE+SwiGLU config, heads "
                                      "divisible by the TP size and B*S divisible by 256*T")
        self.cfg, self.B, self.S = cfg, batch, seq
        self.M = batch * seq
        self.R = self.M // self.T
        self.device = torch.device(device)
        self.lr, self.wd, self.betas, self.eps = lr, weight_decay, betas, eps
        self.step_count = 0
        self.use_graph = use_graph
        self.graph = None
        T, t, dev = self.T, self.t, self.device
        D, F_, V, L, H, hd = cfg.dim, cfg.ff_dim, cfg.vocab, cfg.num_blocks, cfg.num_heads, cfg.head_dim
        self.Hl = H // T
        self.Dl = self.Hl * hd
        self.Fl = _pad64(-(-F_ // T))          # local FFN width, padded to the 64-column SwiGLU groups
        Dl, Fl = self.Dl, self.Fl
        f32, bf16 = torch.float32, torch.bfloat16

        # ---------------- parameters: replicated and sharded arenas
        rep = [ParamSpec("wemb", (V, D)), ParamSpec("wout", (V, D))]
        for l in range(L):
            rep += [ParamSpec(f"b{l}.ln1", (D,), decay_all), ParamSpec(f"b{l}.ln2", (D,), decay_all)]
        rep.append(ParamSpec("lnf", (D,), decay_all))
        shd = []
        for l in range(L):
            shd += [ParamSpec(f"b{l}.wqkv", (3 * Dl, D)), ParamSpec(f"b{l}.wo", (D, Dl)),
                    ParamSpec(f"b{l}.w13", (2 * Fl, D)), ParamSpec(f"b{l}.w2", (D, Fl))]
        self.rep, self.shd = ParamArena(rep), ParamArena(shd)
        self.w32 = {k: torch.zeros(a.total, device=dev, dtype=f32) for k, a in (("rep", self.rep), ("shd", self.shd))}
        self.w16 = {k: torch.zeros(a.total, device=dev, dtype=bf16) for k, a in (("rep", self.rep), ("shd", self.shd))}
        self.grad = {k: torch.zeros(a.total, device=dev, dtype=f32) for k, a in (("rep", self.rep), ("shd", self.shd))}
        self.m = {k: torch.zeros_like(v) for k, v in self.w32.items()}
        self.v = {k: torch.zeros_like(v) for k, v in self.w32.items()}
        self.W = {**self.rep.views(self.w16["rep"]), **self.shd.views(self.w16["shd"])}
        self.G = {**self.rep.views(self.grad["rep"]), **self.shd.views(self.grad["shd"])}
        self.hyper_host = torch.zeros(8, dtype=f32).pin_memory()
        self._hyper_np = self.hyper_host.numpy()
        self.hyper = torch.zeros(8, device=dev, dtype=f32)
        # the pinned staging buffers are rewritten only after the copies that read them have run
        self._h2d_ev = torch.cuda.Event()
        self._h2d_pending = False

        # ---------------- peer memory: gather buffers, reduce-scatter slots, barrier, all-reduce
        self.peer = PeerGroup(self.pg, dev)
        M, R = self.M, self.R
        self.G1 = [self.peer.symmetric(M * D, bf16) for _ in range(L)]
        self.G2 = [self.peer.symmetric(M * D, bf16) for _ in range(L)]
        self.GD = self.peer.symmetric(M * D, bf16)
        self.slots = self.peer.symmetric(M * D, bf16)       # [T, R, D]: slot s holds rank s's partials
        self.ready = torch.zeros(max(T, 1), device=dev, dtype=torch.int32)
        self.comm = Communicator(self.pg, backend="peer", device=dev, capacity_bytes=64 << 20) if T > 1 else None
        self.dp_group = dp_group
        self.dp = dist.get_world_size(dp_group) if (dp_group is not None and dist.is_initialized()) else 1
        self.dp_comm = Communicator(dp_group, backend="peer", device=dev, capacity_bytes=64 << 20) \
            if self.dp > 1 else None

        if model is None:
            model = DecoderLM(cfg, seed=seed)
        self.import_model(model)

        # ---------------- activations
        z = lambda *shape, dt=bf16: torch.empty(*shape, device=dev, dtype=dt)
        self.tok = torch.zeros(M, device=dev, dtype=torch.int32)
        self.tgt = torch.zeros(M, device=dev, dtype=torch.int32)
        self.tok_pin = torch.zeros(M, dtype=torch.int32).pin_memory()
        self.tgt_pin = torch.zeros(M, dtype=torch.int32).pin_memory()
        self.loss_pin = torch.zeros(1, dtype=f32).pin_memory()
        self.x = [z(R, D, dt=f32) for _ in range(L + 1)]
        self.xmid = [z(R, D, dt=f32) for _ in range(L)]
        self.inv1 = [z(R, dt=f32) for _ in range(L)]
        self.inv2 = [z(R, dt=f32) for _ in range(L)]
        self.qkv = [z(M, 3 * Dl) for _ in range(L)]
        self.ao = [z(M, Dl) for _ in range(L)]
        self.lse = [z(batch * self.Hl, seq, dt=f32) for _ in range(L)]
        self.pre = [z(M, 2 * Fl) for _ in range(L)]
        self.act = [z(M, Fl) for _ in range(L)]
        self.nf = z(R, D)
        self.invf = z(R, dt=f32)
        self.logits = z(R, V)
        self.loss_rows = z(R, dt=f32)
        self.loss_sum = z(1, dt=f32)
        self.dx = z(R, D, dt=f32)
        self.dn = z(R, D, dt=f32)
        self.dpre = z(M, 2 * Fl)
        self.dao = z(M, Dl)
        self.dqkv = z(M, 3 * Dl)
        self.dq_acc = z(M, Dl, dt=f32)
        self.dvec = z(batch * self.Hl, seq, dt=f32)
        cos, sin = rope_tables(seq, hd, 0, device=dev)
        self.rope_cs = torch.stack((cos, sin), dim=-1).contiguous()
        self.attn_scale = 1.0 / math.sqrt(hd)
        self.launches_per_step = None
        # Weight-gradient GEMMs on a second stream: at tensor-parallel widths the per-rank products are
        # narrow, and the dW GEMMs (which only feed the optimizer) fill the SMs the gather/reduce-scatter
        # chain leaves idle.  The buffers they read that the backward rewrites (the gathered output
        # gradient, dpre, dqkv) come in two copies; every rank alternates them in the same order, so the
        # symmetric gather buffer a peer reads is always the one this rank wrote for that use.
        # PCB_WGRAD_STREAM=0 keeps one stream (and one copy of each buffer).
        self._wg_stream = None
        self._wg_read = {}
        self.GD_pp, self.dpre_pp, self.dqkv_pp = [self.GD, self.GD], [self.dpre, self.dpre], [self.dqkv, self.dqkv]
        if self.device.type == "cuda" and os.environ.get("PCB_WGRAD_STREAM", "1") != "0":
            self._wg_stream = torch.cuda.Stream(dev)
            self.GD_pp[1] = self.peer.symmetric(M * D, bf16)
            self.dpre_pp[1] = z(M, 2 * Fl)
            self.dqkv_pp[1] = z(M, 3 * Dl)

    # ------------------------------------------------------------------ weights
    def _shard_full(self, model: DecoderLM):
        """Full-model tensors in this rank's shard layout (cpu fp32)."""
        cfg, t, Dl, Fl = self.cfg, self.t, self.Dl, self.Fl
        F_ = cfg.ff_dim
        f0, f1 = t * (-(-F_ // self.T)), min(F_, (t + 1) * (-(-F_ // self.T)))
        out = {"wemb": model.wemb.detach().float().cpu(), "wout": model.wout.detach().T.float().cpu(),
               "lnf": model.lnf_g.detach().float().cpu()}
        for l, blk in enumerate(model.blocks):
            q, k, v = blk.wq.detach().T.cpu(), blk.wk.detach().T.cpu(), blk.wv.detach().T.cpu()   # [D_out, D_in]
            sl = slice(t * Dl, (t + 1) * Dl)
            out[f"b{l}.wqkv"] = torch.cat([q[sl], k[sl], v[sl]], 0)
            out[f"b{l}.wo"] = blk.wo.detach().T.cpu()[:, sl]
            gate = torch.zeros(Fl, cfg.dim)
            up = torch.zeros(Fl, cfg.dim)
            gate[:f1 - f0] = blk.w1.detach().T.cpu()[f0:f1]
            up[:f1 - f0] = blk.w3.detach().T.cpu()[f0:f1]
            out[f"b{l}.w13"] = _interleave(gate, up)
            w2 = torch.zeros(cfg.dim, Fl)
            w2[:, :f1 - f0] = blk.w2.detach().T.cpu()[:, f0:f1]
            out[f"b{l}.w2"] = w2
            out[f"b{l}.ln1"] = blk.ln1_g.detach().float().cpu()
            out[f"b{l}.ln2"] = blk.ln2_g.detach().float().cpu()
        return out

    @torch.no_grad()
    def import_model(self, model: DecoderLM) -> None:
        full = self._shard_full(model)
        for key, arena in (("rep", self.rep), ("shd", self.shd)):
            host = torch.zeros(arena.total)
            for name, view in arena.views(host).items():
                view.copy_(full[name])
            self.w32[key].copy_(host)
            self.w16[key].copy_(host.to(torch.bfloat16))
            self.m[key].zero_()
            self.v[key].zero_()
        self.step_count = 0

    @torch.no_grad()
    def local_weights(self):
        """This rank's fp32 tensors by name (sharded ones are the local shards)."""
        return {**self.rep.views(self.w32["rep"]), **self.shd.views(self.w32["shd"])}

    # ------------------------------------------------------------------ fused GEMM helpers
    def _own(self, buf):
        return buf.local.view(self.M, self.cfg.dim)[self.t * self.R:(self.t + 1) * self.R]

    def _ag_gemm(self, gbuf, b, **kw):
        """C = gather(gbuf) @ op(b): the kernel copies the other ranks' rows of gbuf itself."""
        a = gbuf.local.view(self.M, self.cfg.dim)
        if self.T == 1:
            return ops.gemm(a, b, err=self.peer.err, **kw)
        self.ready.zero_()
        return ops.gemm(a, b, err=self.peer.err,
                        tp=(gbuf.ptrs.data_ptr(), self.ready.data_ptr(), self.R, self.t, self.T, 0, 0, 0), **kw)

    def _rs_gemm(self, a, b, b_mn=False):
        """Partial products of every row land in the owning rank's slot ``self.t``."""
        ops.gemm(a, b, b_mn=b_mn, epi=ops.EPI_RS_BF16, c=self.slots.local.view(self.M, self.cfg.dim),
                 err=self.peer.err, tp=(0, 0, 0, 0, 0, self.slots.ptrs.data_ptr(), self.R, self.t))

    def _barrier(self):
        if self.T > 1:
            self.peer.barrier()

    # ------------------------------------------------------------------ the step
    def _forward(self, write_grad: bool = True) -> None:
        cfg, W, T = self.cfg, self.W, self.T
        B, S, R, hd = self.B, self.S, self.R, cfg.head_dim
        L, eps = cfg.num_blocks, cfg.eps
        sl = slice(self.t * R, (self.t + 1) * R)
        ops.embed_fwd(self.tok[sl], W["wemb"], self.x[0])
        ops.rmsnorm_fwd(self.x[0], W["b0.ln1"], self._own(self.G1[0]), self.inv1[0], eps)
        for l in range(L):
            self._barrier()
            self._ag_gemm(self.G1[l], W[f"b{l}.wqkv"], epi=ops.EPI_BF16, c=self.qkv[l],
                          rope=(self.rope_cs, S, hd, 2 * self.Dl))
            ops.attn_fwd(self.qkv[l], self.ao[l], self.lse[l], B, S, self.Hl, hd, self.attn_scale)
            self._rs_gemm(self.ao[l], W[f"b{l}.wo"])
            self._barrier()
            ops.ext().tp_reduce_norm(self.slots.local, T, self.x[l], self.xmid[l], False, W[f"b{l}.ln2"],
                                     self._own(self.G2[l]), self.inv2[l], eps)
            self._barrier()
            self._ag_gemm(self.G2[l], W[f"b{l}.w13"], epi=ops.EPI_SWIGLU, c=self.pre[l], d=self.act[l])
            self._rs_gemm(self.act[l], W[f"b{l}.w2"])
            self._barrier()
            if l + 1 < L:
                gamma, y, inv = W[f"b{l + 1}.ln1"], self._own(self.G1[l + 1]), self.inv1[l + 1]
            else:
                gamma, y, inv = W["lnf"], self.nf, self.invf
            ops.ext().tp_reduce_norm(self.slots.local, T, self.xmid[l], self.x[l + 1], False, gamma, y, inv, eps)
        ops.gemm(self.nf, W["wout"], epi=ops.EPI_BF16, c=self.logits)
        ops.cross_entropy(self.logits, self.tgt[sl], self.loss_rows, 1.0 / self.M, write_grad)
        self.loss_sum.zero_()
        ops.sumsq(self.loss_rows, self.loss_sum, square=False)

    def _backward(self) -> None:
        cfg, W, G, T = self.cfg, self.W, self.G, self.T
        B, S, R, hd = self.B, self.S, self.R, cfg.head_dim
        L = cfg.num_blocks
        RED = ops.EPI_RED_F32
        sl = slice(self.t * R, (self.t + 1) * R)
        main = torch.cuda.current_stream(self.device)
        side, read = self._wg_stream, self._wg_read

        def wgrad(dy, x, g, key):
            """dW += dy^T x (fp32 reduce epilogue), on the side stream when there is one."""
            if side is None:
                ops.gemm(dy, x, a_mn=True, b_mn=True, epi=RED, c=g)
                return
            side.wait_stream(main)
            with torch.cuda.stream(side):
                ops.gemm(dy, x, a_mn=True, b_mn=True, epi=RED, c=g)
            if key is not None:
                ev = torch.cuda.Event()
                ev.record(side)
                read[key] = ev

        def claim(key):
            """The main stream is about to rewrite buffer ``key``: wait for the dW GEMM that read it."""
            ev = read.pop(key, None)
            if ev is not None:
                main.wait_event(ev)

        GD, dpre, dqkv = self.GD_pp, self.dpre_pp, self.dqkv_pp
        dl = self.logits
        wgrad(dl, self.nf, G["wout"], None)
        ops.gemm(dl, W["wout"], b_mn=True, epi=ops.EPI_F32, c=self.dn)
        k = 0
        claim(("GD", k))
        ops.rmsnorm_bwd(self.dn, self.x[L], W["lnf"], self.invf, self.dx, G["lnf"], False, self._own(GD[k]))
        for l in reversed(range(L)):
            p = l & 1
            # ---- FFN (row-parallel W2, column-parallel W13)
            self._barrier()
            claim(("dpre", p))
            self._ag_gemm(GD[k], W[f"b{l}.w2"], b_mn=True, epi=ops.EPI_SWIGLU_BWD, c=dpre[p], aux=self.pre[l])
            wgrad(GD[k].local.view(self.M, cfg.dim), self.act[l], G[f"b{l}.w2"], ("GD", k))
            wgrad(dpre[p], self.G2[l].local.view(self.M, cfg.dim), G[f"b{l}.w13"], ("dpre", p))
            self._rs_gemm(dpre[p], W[f"b{l}.w13"], b_mn=True)
            self._barrier()
            ops.ext().tp_reduce_norm(self.slots.local, T, None, self.dn, False, None, None, None, cfg.eps)
            k ^= 1
            claim(("GD", k))
            ops.rmsnorm_bwd(self.dn, self.xmid[l], W[f"b{l}.ln2"], self.inv2[l], self.dx, G[f"b{l}.ln2"], True,
                            self._own(GD[k]))
            # ---- attention (row-parallel Wo, column-parallel Wqkv)
            self._barrier()
            self._ag_gemm(GD[k], W[f"b{l}.wo"], b_mn=True, epi=ops.EPI_BF16, c=self.dao)
            wgrad(GD[k].local.view(self.M, cfg.dim), self.ao[l], G[f"b{l}.wo"], ("GD", k))
            claim(("dqkv", p))
            ops.attn_bwd(self.qkv[l], self.ao[l], self.dao, self.lse[l], self.dvec, self.dq_acc, dqkv[p],
                         B, S, self.Hl, hd, self.attn_scale, self.rope_cs)
            wgrad(dqkv[p], self.G1[l].local.view(self.M, cfg.dim), G[f"b{l}.wqkv"], ("dqkv", p))
            self._rs_gemm(dqkv[p], W[f"b{l}.wqkv"], b_mn=True)
            self._barrier()
            ops.ext().tp_reduce_norm(self.slots.local, T, None, self.dn, False, None, None, None, cfg.eps)
            k ^= 1
            claim(("GD", k))
            ops.rmsnorm_bwd(self.dn, self.x[l], W[f"b{l}.ln1"], self.inv1[l], self.dx, G[f"b{l}.ln1"], True,
                            self._own(GD[k]))
        ops.embed_bwd(self.tok[sl], self.dx, G["wemb"])
        if side is not None:
            main.wait_stream(side)   # every weight gradient is complete before the optimizer
            read.clear()

    def _optimizer(self) -> None:
        if self.comm is not None:
            self.comm.all_reduce(self.grad["rep"])       # replicated parameters: sum of row partials
        if self.dp_comm is not None:                     # data-parallel replicas: sum, AdamW scales by 1/DP
            self.dp_comm.all_reduce(self.grad["rep"])
            self.dp_comm.all_reduce(self.grad["shd"])
        for key, arena in (("rep", self.rep), ("shd", self.shd)):
            ops.adamw(self.w32[key], self.grad[key], self.m[key], self.v[key], self.w16[key], arena.n_decay,
                      self.hyper, self.betas[0], self.betas[1], self.eps)
        self._barrier()   # nobody's next forward reads a weight before every rank has written its own

    def _upload(self) -> None:
        """Enqueue the host-to-device copies of the staged step (tokens, targets, hyper-parameters)."""
        self.tok.copy_(self.tok_pin, non_blocking=True)
        self.tgt.copy_(self.tgt_pin, non_blocking=True)
        self.hyper.copy_(self.hyper_host, non_blocking=True)
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
        self.grad["rep"].zero_()
        self.grad["shd"].zero_()
        with nvtx_range("tp_forward"):
            self._forward(True)
        with nvtx_range("tp_backward"):
            self._backward()
        with nvtx_range("tp_optimizer"):
            self._optimizer()
        self.loss_pin.copy_(self.loss_sum, non_blocking=True)

    def _set_hyper(self, lr: float) -> None:
        self._host_writable()
        self.step_count += 1
        b1, b2 = self.betas
        h = self._hyper_np
        h[0] = lr
        h[1] = self.wd
        h[2] = 1.0 - b1 ** self.step_count
        h[3] = 1.0 - b2 ** self.step_count
        h[4] = 1.0 / self.dp

    def stage(self, tokens: torch.Tensor, targets: torch.Tensor) -> None:
        self._host_writable()
        self.tok_pin.copy_(tokens.reshape(-1))      # copy_ converts the dtype in place
        self.tgt_pin.copy_(targets.reshape(-1))

    def launch(self, lr: Optional[float] = None) -> None:
        self._set_hyper(self.lr if lr is None else lr)
        if self.use_graph:
            if self.graph is None:
                self._capture()
            self._upload()
            self.graph.replay()
        else:
            self._step_body()

    def _capture(self) -> None:
        saved = {k: (self.w32[k].clone(), self.w16[k].clone(), self.m[k].clone(), self.v[k].clone())
                 for k in self.w32}
        before = ops.launch_count()
        self._step_body()
        torch.cuda.synchronize(self.device)
        self.launches_per_step = ops.launch_count() - before
        for k, (a, b, c, d) in saved.items():
            self.w32[k].copy_(a); self.w16[k].copy_(b); self.m[k].copy_(c); self.v[k].copy_(d)
        self._barrier()
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            with torch.cuda.graph(self.graph, stream=s):
                self._device_step()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)

    def read_loss(self) -> float:
        """Mean loss over all B*S tokens (sum of the ranks' row sums; one small host all-reduce)."""
        torch.cuda.current_stream(self.device).synchronize()
        v = torch.tensor([float(self.loss_pin[0])], dtype=torch.float64)
        if self.T > 1:
            v = v.to(self.device)
            dist.all_reduce(v, group=self.pg)
        if self.dp > 1:
            v = v.to(self.device)
            dist.all_reduce(v, group=self.dp_group)
        return float(v) / (self.M * self.dp)

    def step(self, tokens: torch.Tensor, targets: torch.Tensor, lr: Optional[float] = None) -> float:
        self.stage(tokens, targets)
        self.launch(lr)
        return self.read_loss()

    def check(self) -> None:
        self.peer.check()
        if self.dp_comm is not None:
            self.dp_comm.check()

    def release(self) -> None:
        """Drop the CUDA graph (it holds peer-memory kernels) before the process group goes away."""
        self.graph = None
        torch.cuda.synchronize(self.device)

    def flops_per_step(self) -> float:
        cfg = self.cfg
        D, F_, V, L = cfg.dim, cfg.ff_dim, cfg.vocab, cfg.num_blocks
        mat = L * (4 * D * D + 3 * D * F_) + V * D
        attn = L * 2 * 2 * self.S * D / 2
        return 6.0 * mat * self.M + 3.0 * attn * self.M
