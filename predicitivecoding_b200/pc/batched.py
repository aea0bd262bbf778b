"""Batched predictive-coding relaxation and learning.

Reference: PredictiveCoding.Device/BatchedPcForward.cs:28-178 (``InferGetTopBatch``).
The reference runs the two GEMMs of each step on the GPU but the bias,
activation, error, derivative and state update on the host, copying both
operands over PCIe for every GEMM (:74-128; CudaGemmProvider.cs:30-59).  Here
everything is device resident and every relaxation step is exactly two GEMM
launches per layer, with the element-wise work fused into their epilogues:

    prediction GEMM (layer l):  pre = M_l W_l^T + b_l ;  pred = f(pre)
                                E_{l-1} = Pi_{l-1} (M_{l-1} - pred)        (error of the layer below)
                                Delta_l = f'(pre) * E_{l-1}                 (bf16, next GEMM's operand)
    state GEMM (layer l):       M_l -= eta (E_l - Delta_l W_l + lambda sign(M_l))   (+ bf16 copy)

All prediction GEMMs of a step run before any state GEMM, which keeps the
reference's Jacobi-synchronous semantics.  Learning adds one GEMM per layer:
``W_l = (W_l + eta_w/B Delta_l^T M_l)(1 - eta_w lambda)`` in the epilogue, and
``b_l += eta_w mean(Delta_l)``.  The batch-mean Hebbian update replaces the
reference's per-sample online ``Learn`` (Network.cs:139-156); with B = 1 they are
the same rule.

:class:`BatchedPCReference` is the same maths in plain PyTorch fp32 (any device):
the oracle for the fused engine and the PyTorch baseline of the benchmark.
"""
from __future__ import annotations

import math
from typing import List, Optional, Sequence

import torch

from .. import ops
from .layer import activate, derivative, init_weights


def _init_params(sizes, activation, seed):
    gen = torch.Generator().manual_seed(seed)
    W, b = [], []
    for l in range(1, len(sizes)):
        W.append(init_weights(sizes[l], sizes[l - 1], activation, gen))
        b.append(torch.zeros(sizes[l - 1]))
    return W, b


class BatchedPCReference:
    """Batched PC engine in plain PyTorch (fp32 by default)."""

    def __init__(self, layer_sizes: Sequence[int], activation: str = "tanh", state_lr: float = 0.1,
                 weight_lr: float = 1e-3, weight_decay: float = 0.0, activity_reg: float = 0.0,
                 precisions: Optional[Sequence[float]] = None, ffg: bool = False, seed: int = 0,
                 weights=None, biases=None, device="cpu", dtype=torch.float32):
        self.sizes = list(layer_sizes)
        self.act, self.eta, self.eta_w, self.wd, self.lam = activation, state_lr, weight_lr, weight_decay, activity_reg
        self.pi = list(precisions) if precisions is not None else [1.0] * len(self.sizes)
        self.ffg = ffg
        if weights is None:
            weights, biases = _init_params(self.sizes, activation, seed)
        self.W = [w.to(device, dtype).clone() for w in weights]
        self.b = [x.to(device, dtype).clone() for x in biases]
        self.device, self.dtype = device, dtype
        self.last_energy: List[float] = []

    def _relax(self, M, steps, clamp_top):
        L = len(self.sizes)
        pre = [None] * L
        pred = [None] * L

        def top_down(l):
            pre[l] = M[l] @ self.W[l - 1].T + self.b[l - 1]
            pred[l] = activate(pre[l], self.act)

        if self.ffg:
            for l in range(L - 1, 0, -1):
                top_down(l)
                if l > 1:
                    M[l - 1] = pred[l].clone()
        E = [None] * L
        for _ in range(steps):
            for l in range(L - 1, 0, -1):
                top_down(l)
            for l in range(L - 1):
                E[l] = self.pi[l] * (M[l] - pred[l + 1])
            E[L - 1] = torch.zeros_like(M[L - 1])
            deltas = [None] * L
            for l in range(1, L):
                deltas[l] = derivative(pre[l], pred[l], self.act) * E[l - 1]
            for l in range(1, L):
                if clamp_top and l == L - 1:
                    continue
                grad = E[l] - deltas[l] @ self.W[l - 1]
                if self.lam > 0:
                    grad = grad + self.lam * torch.sign(M[l])
                M[l] = M[l] - self.eta * grad
        self.last_energy = [0.5 * float((E[l] * E[l]).sum()) / self.pi[l] for l in range(L - 1)]
        return M, pre, pred, E

    def _states(self, inputs, targets):
        B = inputs.shape[0]
        M = [inputs.to(self.device, self.dtype).clone()]
        for s in self.sizes[1:]:
            M.append(torch.zeros(B, s, device=self.device, dtype=self.dtype))
        if targets is not None:
            M[-1] = targets.to(self.device, self.dtype).clone()
        return M

    def infer_get_top(self, inputs: torch.Tensor, steps: int) -> torch.Tensor:
        """Batched twin of Network.infer_get_top(reset_state=True) (BatchedPcForward.cs:36-139)."""
        M, _, _, _ = self._relax(self._states(inputs, None), steps, clamp_top=False)
        return M[-1]

    def learn(self, inputs: torch.Tensor, targets: torch.Tensor, steps: int) -> float:
        """Clamp input and target, settle, apply the batch-mean Hebbian update.  Returns the energy."""
        B = inputs.shape[0]
        M, pre, pred, E = self._relax(self._states(inputs, targets), steps, clamp_top=True)
        # the last relaxation step's prediction and the updated states, as Network.Learn does
        L = len(self.sizes)
        for l in range(1, L):
            delta = derivative(pre[l], pred[l], self.act) * E[l - 1]
            self.W[l - 1] = (self.W[l - 1] + (self.eta_w / B) * delta.T @ M[l]) * (1 - self.eta_w * self.wd)
            self.b[l - 1] = self.b[l - 1] + (self.eta_w / B) * delta.sum(0)
        return sum(self.last_energy)


class BatchedPC:
    """Fused GPU batched PC engine (tcgen05 GEMMs with PC epilogues); optional data parallelism.

    With ``process_group`` every rank relaxes its own ``batch`` samples and the
    per-layer Hebbian deltas are summed over ranks and applied by one fused
    peer-memory kernel (all-reduce + weight update + bf16 refresh on every rank).
    """

    def __init__(self, layer_sizes: Sequence[int], batch: int, activation: str = "tanh", state_lr: float = 0.1,
                 weight_lr: float = 1e-3, weight_decay: float = 0.0, activity_reg: float = 0.0,
                 precisions: Optional[Sequence[float]] = None, ffg: bool = False, seed: int = 0,
                 weights=None, biases=None, device="cuda", process_group=None):
        self.sizes = list(layer_sizes)
        for s in self.sizes:
            if s % 8:
                raise ValueError("BatchedPC needs every layer size to be a multiple of 8 (TMA row alignment)")
        self.B = batch
        self.act, self.eta, self.eta_w, self.wd, self.lam = activation, state_lr, weight_lr, weight_decay, activity_reg
        self.pi = list(precisions) if precisions is not None else [1.0] * len(self.sizes)
        self.ffg = ffg
        self.device = torch.device(device)
        dev = self.device
        self.pg = process_group
        if process_group is not None:
            import torch.distributed as dist
            self.world, self.rank = dist.get_world_size(process_group), dist.get_rank(process_group)
        else:
            self.world, self.rank = 1, 0
        if weights is None:
            weights, biases = _init_params(self.sizes, activation, seed)
        L = len(self.sizes)
        # flat parameter arena: W_1..W_{L-1} then b_1..b_{L-1} (fp32); bf16 copy of the W region
        self.w_off, off = [], 0
        for l in range(1, L):
            self.w_off.append(off)
            off += self.sizes[l - 1] * self.sizes[l]
        self.n_w = off
        self.b_off = []
        for l in range(1, L):
            self.b_off.append(off)
            off += self.sizes[l - 1]
        self.n_total = off
        if self.world > 1:
            from ..parallel.peer import PeerGroup
            self.peer = PeerGroup(process_group, dev)
            self._p32 = self.peer.symmetric(self.n_total, torch.float32)
            self._p16 = self.peer.symmetric(self.n_w, torch.bfloat16)
            self._dlt = self.peer.symmetric(self.n_total, torch.float32)
            self.p32, self.p16, self.delta_flat = self._p32.local, self._p16.local, self._dlt.local
        else:
            self.peer = None
            self.p32 = torch.zeros(self.n_total, device=dev)
            self.p16 = torch.zeros(self.n_w, device=dev, dtype=torch.bfloat16)
            self.delta_flat = None
        self.W32 = [self.p32[o:o + self.sizes[l] * self.sizes[l + 1]].view(self.sizes[l], self.sizes[l + 1])
                    for l, o in enumerate(self.w_off)]
        self.W16 = [self.p16[o:o + self.sizes[l] * self.sizes[l + 1]].view(self.sizes[l], self.sizes[l + 1])
                    for l, o in enumerate(self.w_off)]
        self.b32 = [self.p32[o:o + self.sizes[l]] for l, o in enumerate(self.b_off)]
        for l in range(L - 1):
            self.W32[l].copy_(weights[l].to(dev, torch.float32))
            self.b32[l].copy_(biases[l].to(dev, torch.float32))
        self.p16.copy_(self.p32[:self.n_w].to(torch.bfloat16))
        if self.delta_flat is not None:
            self.dW = [self.delta_flat[o:o + self.sizes[l] * self.sizes[l + 1]].view(self.sizes[l], self.sizes[l + 1])
                       for l, o in enumerate(self.w_off)]
            self.db = [self.delta_flat[o:o + self.sizes[l]] for l, o in enumerate(self.b_off)]
        # states and per-step buffers
        B = batch
        self.M32 = [torch.zeros(B, s, device=dev) for s in self.sizes]
        self.M16 = [None] + [torch.zeros(B, s, device=dev, dtype=torch.bfloat16) for s in self.sizes[1:]]
        self.E = [torch.zeros(B, s, device=dev) for s in self.sizes]
        self.D16 = [None] + [torch.zeros(B, self.sizes[l - 1], device=dev, dtype=torch.bfloat16) for l in range(1, L)]
        self.energy = torch.zeros(L, device=dev)
        self.graph = None
        self.launches = 0

    # ------------------------------------------------------------ kernels
    def _pred(self, l: int, with_energy: bool) -> None:
        ops.gemm_pc(self.M16[l], self.W16[l - 1], epi=ops.EPI_PC_PRED, c=self.E[l - 1], d=self.D16[l],
                    aux=self.M32[l - 1], bias=self.b32[l - 1], act=self.act, pi=self.pi[l - 1],
                    energy=self.energy[l - 1:l] if with_energy else None)

    def _state(self, l: int, top_free: bool) -> None:
        aux = None if (l == len(self.sizes) - 1 and top_free) else self.E[l]
        ops.gemm_pc(self.D16[l], self.W16[l - 1], b_mn=True, epi=ops.EPI_PC_STATE, c=self.M32[l], d=self.M16[l],
                    aux=aux, eta=self.eta, actreg=self.lam)

    def _ffg_sweep(self, top_clamped: bool) -> None:
        L = len(self.sizes)
        for l in range(L - 1, 0, -1):
            if l > 1:
                # the prediction of layer l becomes the state of layer l-1 (fp32 and bf16)
                ops.gemm_pc(self.M16[l], self.W16[l - 1], epi=ops.EPI_PC_PRED, aux=self.M32[l - 1],
                            bias=self.b32[l - 1], act=self.act, pred_out=self.M32[l - 1], pred_bf16=self.M16[l - 1])

    def _relax(self, steps: int, top_clamped: bool, energy_last: bool = True) -> None:
        L = len(self.sizes)
        if self.ffg:
            self._ffg_sweep(top_clamped)
        for s in range(steps):
            last = energy_last and s == steps - 1
            if last:
                self.energy.zero_()
            for l in range(L - 1, 0, -1):
                self._pred(l, last)
            for l in range(1, L):
                if top_clamped and l == L - 1:
                    continue
                self._state(l, top_free=not top_clamped)

    def _load(self, inputs: torch.Tensor, targets: Optional[torch.Tensor]) -> None:
        self.M32[0].copy_(inputs, non_blocking=True)
        for l in range(1, len(self.sizes)):
            self.M32[l].zero_()
            self.M16[l].zero_()
        if targets is not None:
            self.M32[-1].copy_(targets, non_blocking=True)
            self.M16[-1].copy_(self.M32[-1])

    def _update(self) -> None:
        """Hebbian weight update from the last step's deltas and the updated states."""
        L = len(self.sizes)
        Bg = self.B * self.world
        decay = 1.0 - self.eta_w * self.wd
        if self.world == 1:
            for l in range(1, L):
                ops.gemm_pc(self.D16[l], self.M16[l], a_mn=True, b_mn=True, epi=ops.EPI_PC_WUPD, c=self.W32[l - 1],
                            d=self.W16[l - 1], alpha=self.eta_w / Bg, decay=decay)
                ops.colsum(self.D16[l], self.b32[l - 1], self.eta_w / Bg)
            return
        # data parallel: partial deltas -> symmetric buffer; fused all-reduce + update on each rank's shard
        self.delta_flat[self.n_w:].zero_()
        for l in range(1, L):
            ops.gemm(self.D16[l], self.M16[l], a_mn=True, b_mn=True, epi=ops.EPI_F32, c=self.dW[l - 1],
                     alpha=self.eta_w / Bg)
            ops.colsum(self.D16[l], self.db[l - 1], self.eta_w / Bg)
        self.peer.barrier()
        for lo_all, hi_all, dec, w16 in ((0, self.n_w, decay, self._p16.ptrs), (self.n_w, self.n_total, 1.0, None)):
            n = hi_all - lo_all
            per = ((n + self.world - 1) // self.world + 3) // 4 * 4
            lo = min(hi_all, lo_all + self.rank * per)
            hi = min(hi_all, lo + per)
            if hi > lo:
                ops.ext().pc_allreduce_update(self._dlt.ptrs, self._p32.ptrs, w16, lo, hi, 1.0, dec, self.world,
                                              self.rank)
        self.peer.barrier()

    # ------------------------------------------------------------ public API
    @torch.no_grad()
    def infer_get_top(self, inputs: torch.Tensor, steps: int) -> torch.Tensor:
        """Free-top inference from zero states; returns the top states [B, top]."""
        self._load(inputs, None)
        self._relax(steps, top_clamped=False)
        return self.M32[-1].clone()

    @torch.no_grad()
    def learn(self, inputs: torch.Tensor, targets: torch.Tensor, steps: int) -> None:
        """Clamp both ends, settle ``steps``, apply the (all-reduced) batch-mean Hebbian update."""
        self._load(inputs, targets)
        self._relax(steps, top_clamped=True)
        self._update()

    def energy_value(self) -> float:
        """Free energy of the last relaxation step (sum over layers of 1/2 ||E||^2 / Pi)."""
        e = self.energy.cpu().tolist()
        return sum(0.5 * e[l] / self.pi[l] for l in range(len(self.sizes) - 1))

    def capture(self, steps: int) -> None:
        """Capture learn(steps) on the current staged inputs into a CUDA graph (replay with ``replay``)."""
        self._stage_in = torch.zeros_like(self.M32[0])
        self._stage_tg = torch.zeros_like(self.M32[-1])
        before = ops.launch_count()
        self.learn(self._stage_in, self._stage_tg, steps)   # warm-up outside capture
        torch.cuda.synchronize(self.device)
        self._graph_launches = ops.launch_count() - before
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
            self.learn(self._stage_in, self._stage_tg, steps)
        torch.cuda.current_stream(self.device).wait_stream(s)
        self.graph = g

    def replay(self, inputs: torch.Tensor, targets: torch.Tensor) -> None:
        self._stage_in.copy_(inputs, non_blocking=True)
        self._stage_tg.copy_(targets, non_blocking=True)
        self.graph.replay()

    def weights(self):
        return [w.detach().cpu().clone() for w in self.W32], [b.detach().cpu().clone() for b in self.b32]

    def flops_per_learn(self, steps: int) -> float:
        """GEMM FLOPs of one learn(): per step, prediction + state GEMMs, then the weight-update GEMMs."""
        B, s = self.B, self.sizes
        pred = sum(2 * B * s[l] * s[l - 1] for l in range(1, len(s)))
        state = sum(2 * B * s[l] * s[l - 1] for l in range(1, len(s) - 1))
        return steps * (pred + state) + pred
