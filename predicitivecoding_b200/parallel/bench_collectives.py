"""Device timing of the fused peer-memory collectives against their NVLink roofline.

Run one process per GPU, e.g. on 8 GPUs:

    timeout -k 60 600 python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \\
        --master-port 29541 -m predicitivecoding_b200.parallel.bench_collectives

Cases (each timed with CUDA events on the launching stream after warm-up, max over ranks):

* ``rs_adamw_ag``: the data-parallel optimizer step of the 124M decoder (134,105,856 parameters):
  every rank reads its 1/T shard of every rank's fp32 gradients over NVLink, runs AdamW on it and
  writes the bf16 weights of the shard into every rank's weight buffer;
* ``pc_allreduce_update``: the PC data-parallel weight step (64 Mi fp32 weights): sum of every
  rank's delta-W shard, weight update, fp32 + bf16 weights written to every rank;
* ``all_reduce``: the Communicator's peer all-reduce (one-shot below 512 KiB, two-shot above);
* ``dp_bucket_push`` / ``dp_post_backward``: the trainer's bucketed data-parallel step on the same
  124M arena, split as it runs: the copy-engine pushes of every bucket's pieces to their owners (in the
  trainer they overlap the backward; here they are timed alone), and what runs after the backward
  (barrier, owner reduce + sum of squares, clip-norm exchange, AdamW + bf16 weights to every rank,
  barrier).

Bytes that must cross each GPU's links, per direction: a rank's inbound link carries what it pulls from
the others and what the others push to it, and its outbound link the mirror image, so for T ranks the
per-direction volume is (T-1)/T * N * 6 for ``rs_adamw_ag`` (4-byte gradients pulled, 2-byte weights
pushed), (T-1)/T * N * 10 for ``pc_allreduce_update`` (4 pulled, 4 + 2 pushed) and 2 (T-1)/T * S for
an all-reduce of S bytes. The roofline time is that volume at the measured 770 GB/s per direction per
GPU; each line reports achieved / roofline. Every case includes the device barriers it needs in the
trainer (before: all inputs written; after: all outputs written).
"""
from __future__ import annotations

import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist

LINK_GBS = 770.0   # measured peer copy per direction per GPU on this pool


def nvlink_bytes_per_direction(case: str, n: int, world: int) -> float:
    """Bytes that must cross each rank's links in one direction for one call.

    ``n`` is the parameter count for ``rs_adamw_ag`` (fp32 gradients pulled, bf16 weights pushed) and
    ``pc_allreduce_update`` (fp32 deltas pulled, fp32 + bf16 weights pushed), and the message size in
    bytes for ``all_reduce``. What a rank pulls and what the others push to it share its inbound link.
    """
    if world <= 1:
        return 0.0
    f = (world - 1) / world
    per_elem = {"rs_adamw_ag": 4 + 2, "pc_allreduce_update": 4 + 6, "all_reduce": 2, "dp_bucket_push": 4,
                "dp_post_backward": 2}
    if case not in per_elem:
        raise ValueError(f"unknown case {case!r}")
    return f * n * per_elem[case]


def _time(fn, iters: int, dev) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize(dev)
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s = torch.cuda.current_stream(dev)
    a.record(s)
    for _ in range(iters):
        fn()
    b.record(s)
    torch.cuda.synchronize(dev)
    t = torch.tensor([a.elapsed_time(b) / iters], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def main() -> None:
    from .. import ops
    from .collectives import Communicator
    from .peer import PeerGroup
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    rank, T = dist.get_rank(), dist.get_world_size()
    peer = PeerGroup(None, dev)
    out = []

    # ---- data-parallel AdamW step of the 124M decoder
    N = 134_105_856
    N -= N % (8 * T)
    grad = peer.symmetric(N, torch.float32)
    w16 = peer.symmetric(N, torch.bfloat16)
    grad.local.normal_()
    per = N // T
    lo, hi = rank * per, (rank + 1) * per
    w32 = torch.randn(per, device=dev)
    m = torch.zeros(per, device=dev)
    v = torch.zeros(per, device=dev)
    hyper = torch.tensor([1e-4, 0.1, 0.1, 0.001, 1.0 / T, 0, 0, 0], device=dev)

    def dp_step():
        peer.barrier()
        ops.ext().rs_adamw_ag(grad.ptrs, w16.ptrs, w32, m, v, lo, hi, hi, hyper, 0.9, 0.999, 1e-8, T)
        peer.barrier()

    ms = _time(dp_step, 10, dev)
    per_dir = nvlink_bytes_per_direction("rs_adamw_ag", N, T)
    roof = per_dir / (LINK_GBS * 1e9) * 1e3
    out.append({"case": "rs_adamw_ag (124M params, fp32 grads in, bf16 weights out)", "world": T,
                "ms": round(ms, 3), "nvlink_gb_per_direction": round(per_dir / 1e9, 3),
                "roofline_ms": round(roof, 3), "of_roofline": round(roof / ms, 3) if T > 1 else None})
    del grad, w16, w32, m, v

    # ---- bucketed data-parallel step (the trainer's path): pushes, then the post-backward kernels
    from ..engine.arena import ParamArena, ParamSpec
    from ..engine.fused_trainer import FusedDecoderTrainer
    from ..models.config import DecoderLmConfig
    cfg = DecoderLmConfig.gpt2_small_swiglu()
    D, F_, L, V = cfg.dim, cfg.ff_dim, cfg.num_blocks, cfg.vocab
    specs = [ParamSpec("wemb", (V, D)), ParamSpec("wout", (V, D)), ParamSpec("lnf", (D,))]
    buckets = [["wout", "lnf"]]
    for l in reversed(range(L)):
        names = [f"b{l}.wqkv", f"b{l}.wo", f"b{l}.w13", f"b{l}.w2", f"b{l}.ln1", f"b{l}.ln2"]
        shapes = [(3 * D, D), (D, D), (2 * F_, D), (D, F_), (D,), (D,)]
        specs += [ParamSpec(n, sh) for n, sh in zip(names, shapes)]
        buckets.append(names)
    buckets.append(["wemb"])
    A = ParamArena(specs, T, buckets=buckets)
    gradb = torch.randn(A.total, device=dev)
    stage = peer.symmetric(T * A.shard, torch.float32)
    w16c = peer.symmetric(A.total, torch.bfloat16)
    norm = peer.symmetric(T, torch.float64)
    tab = torch.tensor([list(p) for p in A.pieces(rank)], dtype=torch.int64, device=dev)
    plans = [FusedDecoderTrainer.push_plan(A, rank, b) for b in range(len(A.buckets))]
    gsh, w32b = torch.zeros(A.shard, device=dev), torch.randn(A.shard, device=dev)
    mb, vb = torch.zeros(A.shard, device=dev), torch.zeros(A.shard, device=dev)
    sumsq = torch.zeros(1, device=dev, dtype=torch.float64)

    def pushes():
        base = gradb.data_ptr()
        for plan in plans:
            for q, dst, src, n in plan:
                ops.ext().memcpy_d2d(stage.host_ptrs[q] + 4 * dst, base + 4 * src, 4 * n)
        peer.barrier()

    def post_backward():
        peer.barrier()
        sumsq.zero_()
        ops.ext().dp_reduce_sumsq(gradb, stage.local, A.shard, tab, rank, T, gsh, sumsq)
        ops.ext().dp_norm_push(sumsq, norm.ptrs, rank, T)
        peer.barrier()
        ops.ext().dp_adamw_ag(gsh, w32b, mb, vb, w16c.ptrs, A.shard, tab, hyper, 0.9, 0.999, 1e-8, norm.local, 1.0, T)
        peer.barrier()

    for name, fn in (("dp_bucket_push", pushes), ("dp_post_backward", post_backward)):
        ms = _time(fn, 10, dev)
        per_dir = nvlink_bytes_per_direction(name, A.total, T)
        roof = per_dir / (LINK_GBS * 1e9) * 1e3
        label = ("dp_bucket_push (copy engines, all buckets, timed alone)" if name == "dp_bucket_push" else
                 "dp_post_backward (reduce + clip + AdamW + bf16 all-gather)")
        out.append({"case": label, "world": T, "ms": round(ms, 3), "nvlink_gb_per_direction": round(per_dir / 1e9, 3),
                    "roofline_ms": round(roof, 3), "of_roofline": round(roof / ms, 3) if T > 1 else None})
    del gradb, stage, w16c, norm, gsh, w32b, mb, vb

    # ---- PC data-parallel delta-W all-reduce + update
    N2 = 64 << 20
    dlt = peer.symmetric(N2, torch.float32)
    wts = peer.symmetric(N2, torch.float32)
    w16b = peer.symmetric(N2, torch.bfloat16)
    dlt.local.normal_()
    wts.local.normal_()
    per2 = N2 // T
    lo2, hi2 = rank * per2, (rank + 1) * per2

    def pc_step():
        peer.barrier()
        ops.ext().pc_allreduce_update(dlt.ptrs, wts.ptrs, w16b.ptrs, lo2, hi2, 1e-6, 1.0, T, rank)
        peer.barrier()

    ms = _time(pc_step, 10, dev)
    per_dir = nvlink_bytes_per_direction("pc_allreduce_update", N2, T)
    roof = per_dir / (LINK_GBS * 1e9) * 1e3
    out.append({"case": "pc_allreduce_update (64 Mi fp32 weights)", "world": T, "ms": round(ms, 3),
                "nvlink_gb_per_direction": round(per_dir / 1e9, 3),
                "roofline_ms": round(roof, 3), "of_roofline": round(roof / ms, 3) if T > 1 else None})
    del dlt, wts, w16b

    # ---- Communicator all-reduce (fp32)
    comm = Communicator(None, backend="peer", device=dev, capacity_bytes=256 << 20)
    for nbytes in (256 << 10, 32 << 20, 256 << 20):
        x = torch.randn(nbytes // 4, device=dev)
        ms = _time(lambda: comm.all_reduce(x), 10, dev)
        roof = nvlink_bytes_per_direction("all_reduce", nbytes, T) / (LINK_GBS * 1e9) * 1e3
        out.append({"case": f"all_reduce fp32 {nbytes >> 10} KiB", "world": T, "ms": round(ms, 4),
                    "bus_gbs": round(2 * (T - 1) / T * nbytes / (ms * 1e-3) / 1e9, 1),
                    "roofline_ms": round(roof, 4), "of_roofline": round(roof / ms, 3) if T > 1 else None})
    peer.check()
    comm.check()
    if rank == 0:
        for o in out:
            print(json.dumps(o), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
