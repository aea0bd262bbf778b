"""Collectives: AllReduce / Broadcast / ReduceScatter / AllGather with Sum / Prod / Max / Min.

Reference: PredictiveCoding.Device/Nccl/NcclProvider.cs:1-109 — one provider over a set of
devices whose four collectives take one ``float[]`` per rank and run on the host ("mock NCCL").

Three implementations with one contract:

* ``HostCollectives``: the reference's semantics over in-process per-rank buffers (CPU tensors or
  arrays); the oracle for the others and the path for a single process that holds every rank.
* ``MultiDeviceCollectives``: one process driving several GPUs, per-device tensors, through
  NCCL's single-process communicators (``torch.cuda.nccl``).
* ``Communicator``: one process per GPU (the production shape).  ``backend="peer"`` runs the
  extension's NVLink peer-memory kernels over IPC-mapped symmetric buffers with bounded device
  barriers — one-shot all-reduce for small payloads (every rank reads every peer), two-shot
  (reduce-scatter into its own shard, barrier, all-gather of the shards) for large ones;
  ``backend="nccl"`` calls ``torch.distributed`` (the baseline); ``backend="gloo"`` is the CPU
  path used by the multi-process tests.
"""
from __future__ import annotations

import enum
from typing import Tuple, List, Optional, Sequence

import torch
import torch.distributed as dist


class ReduceOp(enum.IntEnum):
    SUM = 0
    PROD = 1
    MAX = 2
    MIN = 3


def _op(op) -> ReduceOp:
    if isinstance(op, str):
        return ReduceOp[op.upper()]
    return ReduceOp(int(op))


def _combine(a: torch.Tensor, b: torch.Tensor, op: ReduceOp) -> torch.Tensor:
    if op == ReduceOp.SUM:
        return a + b
    if op == ReduceOp.PROD:
        return a * b
    if op == ReduceOp.MAX:
        return torch.maximum(a, b)
    return torch.minimum(a, b)


_DIST_OP = {ReduceOp.SUM: dist.ReduceOp.SUM, ReduceOp.PROD: dist.ReduceOp.PRODUCT, ReduceOp.MAX: dist.ReduceOp.MAX,
            ReduceOp.MIN: dist.ReduceOp.MIN}


# ------------------------------------------------------------------------------------ host
class HostCollectives:
    """Per-rank buffers in one process; results written in place, rank order 0..n-1."""

    def __init__(self, rank_count: int):
        if rank_count < 1:
            raise ValueError("At least one rank is required.")
        self.rank_count = rank_count

    def _uniform(self, bufs: Sequence[torch.Tensor]) -> None:
        if len(bufs) != self.rank_count:
            raise ValueError(f"Expected {self.rank_count} per-rank buffers.")
        if any(b.numel() != bufs[0].numel() for b in bufs):
            raise ValueError("All rank buffers must be the same length.")

    def all_reduce(self, bufs: Sequence[torch.Tensor], op=ReduceOp.SUM) -> None:
        self._uniform(bufs)
        op = _op(op)
        acc = bufs[0].clone()
        for b in bufs[1:]:
            acc = _combine(acc, b, op)
        for b in bufs:
            b.copy_(acc)

    def broadcast(self, bufs: Sequence[torch.Tensor], root: int) -> None:
        self._uniform(bufs)
        if not 0 <= root < self.rank_count:
            raise ValueError("root out of range")
        src = bufs[root].clone()
        for b in bufs:
            b.copy_(src)

    def reduce_scatter(self, send: Sequence[torch.Tensor], recv: Sequence[torch.Tensor], op=ReduceOp.SUM) -> None:
        self._uniform(send)
        total = send[0].numel()
        if total % self.rank_count:
            raise ValueError("Send length must divide evenly across ranks.")
        chunk = total // self.rank_count
        op = _op(op)
        acc = send[0].reshape(-1).clone()
        for s in send[1:]:
            acc = _combine(acc, s.reshape(-1), op)
        for r, out in enumerate(recv):
            if out.numel() != chunk:
                raise ValueError(f"recv[{r}] must have length {chunk}.")
            out.reshape(-1).copy_(acc[r * chunk:(r + 1) * chunk])

    def all_gather(self, send: Sequence[torch.Tensor], recv: Sequence[torch.Tensor]) -> None:
        self._uniform(send)
        n = send[0].numel()
        for r, out in enumerate(recv):
            if out.numel() != n * self.rank_count:
                raise ValueError(f"recv[{r}] must have length {n * self.rank_count}.")
            out.reshape(-1).copy_(torch.cat([s.reshape(-1) for s in send]).to(out.device))


# ------------------------------------------------------------------------------------ one process, many GPUs
class MultiDeviceCollectives(HostCollectives):
    """Per-device CUDA tensors held by one process; NCCL single-process communicators."""

    def __init__(self, devices: Sequence[int]):
        super().__init__(len(devices))
        self.devices = list(devices)

    @staticmethod
    def for_all_devices() -> "MultiDeviceCollectives":
        return MultiDeviceCollectives(list(range(max(1, torch.cuda.device_count()))))

    def _nccl_ok(self, bufs) -> bool:
        return (all(b.is_cuda for b in bufs) and len({b.device for b in bufs}) == len(bufs)
                and torch.cuda.nccl.is_available(list(bufs)))

    def all_reduce(self, bufs, op=ReduceOp.SUM) -> None:
        if self._nccl_ok(bufs):
            self._uniform(bufs)
            torch.cuda.nccl.all_reduce(list(bufs), op=int(_op(op)))
        else:
            super().all_reduce(bufs, op)

    def broadcast(self, bufs, root: int) -> None:
        if self._nccl_ok(bufs):
            self._uniform(bufs)
            torch.cuda.nccl.broadcast(list(bufs), root=root)
        else:
            super().broadcast(bufs, root)

    def all_gather(self, send, recv) -> None:
        if self._nccl_ok(send) and self._nccl_ok(recv):
            self._uniform(send)
            torch.cuda.nccl.all_gather(list(send), list(recv))
        else:
            super().all_gather(send, recv)

    def reduce_scatter(self, send, recv, op=ReduceOp.SUM) -> None:
        if self._nccl_ok(send) and self._nccl_ok(recv):
            self._uniform(send)
            torch.cuda.nccl.reduce_scatter(list(send), list(recv), op=int(_op(op)))
        else:
            super().reduce_scatter(send, recv, op)


# ------------------------------------------------------------------------------------ one process per GPU
def two_shot_shard(n: int, world: int, rank: int) -> Tuple[int, int]:
    """[a, b) of an n-element message that `rank` reduces in the two-shot all-reduce.

    Shards are ceil(n / world) rounded up to a multiple of 8 elements, so every shard starts on a
    16-byte boundary for both fp32 and bf16 (the kernel's vector path); the last shards may be short or
    empty. Together the shards of ranks 0..world-1 cover [0, n) exactly once.
    """
    per = -(-n // world)
    per += (-per) % 8
    return min(n, rank * per), min(n, (rank + 1) * per)


class Communicator:
    """Collectives among the ranks of a process group (one rank per GPU, or gloo ranks on CPU)."""

    ONE_SHOT_MAX_BYTES = 512 * 1024

    def __init__(self, pg=None, backend: str = "auto", device: Optional[torch.device] = None,
                 capacity_bytes: int = 64 << 20):
        self.pg = pg
        self.world = dist.get_world_size(pg) if dist.is_initialized() else 1
        self.rank = dist.get_rank(pg) if dist.is_initialized() else 0
        if backend == "auto":
            backend = "peer" if torch.cuda.is_available() and (device is None or torch.device(device).type == "cuda") \
                else "gloo"
        if backend not in ("peer", "nccl", "gloo"):
            raise ValueError(f"unknown backend {backend!r}")
        self.backend = backend
        self.device = torch.device(device) if device is not None else (
            torch.device("cuda", torch.cuda.current_device()) if backend != "gloo" else torch.device("cpu"))
        self._peer = None
        self._stage = {}
        self.capacity = capacity_bytes
        if backend == "peer":
            from .peer import PeerGroup
            self._peer = PeerGroup(pg, self.device)

    # -------------------------------------------------------------- staging buffers (peer backend)
    def _stage_buf(self, dtype: torch.dtype):
        if dtype not in self._stage:
            elt = torch.tensor([], dtype=dtype).element_size()
            self._stage[dtype] = self._peer.symmetric(self.capacity // elt, dtype)
        return self._stage[dtype]

    def _chunks(self, n: int, elt: int):
        cap = (self.capacity // elt) // max(1, self.world) * max(1, self.world)
        cap -= cap % (8 * self.world) if cap > 8 * self.world else 0
        i = 0
        while i < n:
            yield i, min(n, i + cap)
            i += cap

    @staticmethod
    def _check_dtype(t: torch.Tensor) -> None:
        if t.dtype not in (torch.float32, torch.bfloat16):
            raise TypeError("peer collectives support fp32 and bf16 tensors")

    # -------------------------------------------------------------- API
    def all_reduce(self, t: torch.Tensor, op=ReduceOp.SUM) -> torch.Tensor:
        op = _op(op)
        if self.backend != "peer":
            if self.world > 1:
                dist.all_reduce(t, op=_DIST_OP[op], group=self.pg)
            return t
        self._check_dtype(t)
        from .. import ops
        flat = t.view(-1)
        buf = self._stage_buf(t.dtype)
        P = self._peer
        for lo, hi in self._chunks(flat.numel(), t.element_size()):
            n = hi - lo
            buf.local[:n].copy_(flat[lo:hi])
            P.barrier()
            if n * t.element_size() <= self.ONE_SHOT_MAX_BYTES or self.world == 1:
                ops.ext().coll_reduce(buf.ptrs, flat[lo:hi], 0, n, self.world, int(op), 1.0)
                P.barrier()
            else:
                # two-shot in one pass: rank r reduces shard r over every rank's buffer and stores the
                # result into shard r of every rank's buffer (peer stores); after a barrier each rank's
                # buffer holds the whole reduced vector
                a, b = two_shot_shard(n, self.world, self.rank)
                if b > a:
                    ops.ext().coll_reduce_push(buf.ptrs, buf.ptrs, buf.local, a, b, self.world, int(op), 1.0)
                P.barrier()
                flat[lo:hi].copy_(buf.local[:n])
                P.barrier()
        return t

    def broadcast(self, t: torch.Tensor, root: int = 0) -> torch.Tensor:
        if not 0 <= root < self.world:
            raise ValueError("root out of range")
        if self.backend != "peer":
            if self.world > 1:
                dist.broadcast(t, src=dist.get_global_rank(self.pg, root) if self.pg is not None else root,
                               group=self.pg)
            return t
        self._check_dtype(t)
        from .. import ops
        flat = t.view(-1)
        buf = self._stage_buf(t.dtype)
        for lo, hi in self._chunks(flat.numel(), t.element_size()):
            n = hi - lo
            if self.rank == root:
                buf.local[:n].copy_(flat[lo:hi])
            self._peer.barrier()
            if self.rank != root:
                ops.ext().coll_gather(buf.ptrs[root:root + 1], flat[lo:hi], n, 0, 1)
            self._peer.barrier()
        return t

    def reduce_scatter(self, out: torch.Tensor, inp: torch.Tensor, op=ReduceOp.SUM) -> torch.Tensor:
        op = _op(op)
        if inp.numel() != out.numel() * self.world:
            raise ValueError("input must hold world * output elements")
        if self.backend != "peer":
            if self.world > 1:
                dist.reduce_scatter_tensor(out, inp, op=_DIST_OP[op], group=self.pg)
            else:
                out.copy_(inp.view_as(out))
            return out
        self._check_dtype(inp)
        from .. import ops
        chunk = out.numel()
        if inp.numel() * inp.element_size() > self.capacity:
            raise ValueError("reduce_scatter payload exceeds the staging capacity")
        buf = self._stage_buf(inp.dtype)
        buf.local[:inp.numel()].copy_(inp.view(-1))
        self._peer.barrier()
        ops.ext().coll_reduce(buf.ptrs, out.view(-1), self.rank * chunk, (self.rank + 1) * chunk, self.world,
                              int(op), 1.0)
        self._peer.barrier()
        return out

    def all_gather(self, out: torch.Tensor, inp: torch.Tensor) -> torch.Tensor:
        if out.numel() != inp.numel() * self.world:
            raise ValueError("output must hold world * input elements")
        if self.backend != "peer":
            if self.world > 1:
                dist.all_gather_into_tensor(out, inp, group=self.pg)
            else:
                out.copy_(inp.view_as(out))
            return out
        self._check_dtype(inp)
        from .. import ops
        n = inp.numel()
        if n * inp.element_size() > self.capacity:
            raise ValueError("all_gather payload exceeds the staging capacity")
        buf = self._stage_buf(inp.dtype)
        buf.local[:n].copy_(inp.view(-1))
        self._peer.barrier()
        ops.ext().coll_gather(buf.ptrs, out.view(-1), n, 0, self.world)
        self._peer.barrier()
        return out

    def check(self) -> None:
        if self._peer is not None:
            self._peer.check()

    def close(self) -> None:
        if self._peer is not None:
            self._peer.close()
