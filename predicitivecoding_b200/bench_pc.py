"""Benchmark of the wide predictive-coding MLP (samples/s), used by ``bench.py --workload pc``.

Layers 4096-8192x6-1024 (tanh), T=32 relaxation steps with state lr 0.1, weight lr 1e-3;
each step clamps seeded N(0,1) inputs (4096) and targets (1024), settles, and applies
the batch-mean Hebbian update, all-reduced over ranks by the fused peer-memory kernel.
Batch 4096 per GPU, bf16 GEMM operands with fp32 states and weights.
"""
from __future__ import annotations

import time

import torch

PC_SIZES = [4096] + [8192] * 6 + [1024]
PC_STEPS = 32


def run_pc_bench(args, dev, rank, world, pg):
    from predicitivecoding_b200 import ops
    from predicitivecoding_b200.pc.batched import BatchedPC, BatchedPCReference
    from predicitivecoding_b200.utils.clocks import ClockSampler

    B = args.batch or 4096
    g = torch.Generator().manual_seed(100 + rank)
    pool = [(torch.randn(B, PC_SIZES[0], generator=g).pin_memory(), torch.randn(B, PC_SIZES[-1], generator=g).pin_memory())
            for _ in range(2)]
    if args.impl == "torch":
        eng = BatchedPCReference(PC_SIZES, "tanh", 0.1, 1e-3, seed=0, device=dev, dtype=torch.bfloat16)

        def step(x, y, sync=True):
            eng.learn(x.to(dev, non_blocking=True), y.to(dev, non_blocking=True), PC_STEPS)
            if world > 1:
                import torch.distributed as dist
                for w in eng.W + eng.b:
                    dist.all_reduce(w)
                    w.div_(world)
            if sync:
                torch.cuda.synchronize(dev)
        flops = None
    else:
        eng = BatchedPC(PC_SIZES, B, "tanh", 0.1, 1e-3, seed=0, device=dev, process_group=pg)
        use_graph = not args.no_graph
        if use_graph:
            eng.capture(PC_STEPS)

        def step(x, y, sync=True):
            if use_graph:
                eng.replay(x, y)
            else:
                eng.learn(x.to(dev, non_blocking=True), y.to(dev, non_blocking=True), PC_STEPS)
            if sync:
                e = eng.energy[:1].to("cpu")   # the step's result read back on the host
                return float(e)
        flops = eng.flops_per_learn(PC_STEPS)

    for i in range(max(3, args.warmup)):
        step(*pool[i % 2])
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0 = ops.launch_count() if args.impl != "torch" else 0
    with ClockSampler(dev.index) as clk:
        start.record()
        for i in range(args.steps):
            step(*pool[i % 2], sync=False)
        end.record()
        torch.cuda.synchronize(dev)
    ms = start.elapsed_time(end)
    launched = (ops.launch_count() - l0) if args.impl != "torch" else 0
    if args.impl != "torch" and getattr(eng, "graph", None) is not None:
        # replays launch the captured kernels: count them once per replay
        per = eng._graph_launches if hasattr(eng, "_graph_launches") else None
        if per:
            launched = per * args.steps
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t)
    ms_step = ms / args.steps
    samples = world * B * args.steps / (ms / 1e3)

    ek = args.e2e_steps or args.steps
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for i in range(ek):
        step(*pool[i % 2], sync=True)
    e2e = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e = float(t)
    from bench import REF_PC_SAMPLES
    res = {
        "metric": "PC-net train samples/s (max over ranks)",
        "value": round(samples, 1), "unit": "samples/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": round(ms_step, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": round(samples / REF_PC_SAMPLES, 2),
        "vs_baseline_basis": "closest published reference figure: BatchedPcForward 64 samples x "
                             "[3072,512,128,10], 20 steps in 75 ms on one RTX 4070 SUPER (ROADMAP-MixedPrecision.md:99)",
        "dtype": "bf16", "data": "synthetic (seeded N(0,1) inputs and targets, random-init weights)",
        "impl": args.impl,
        "config": {"model": "pc-mlp-4096-8192x6-1024", "global_batch": B * world, "seq_len": None,
                   "relax_steps": PC_STEPS, "parallelism": f"dp{world}", "batch_per_gpu": B,
                   "l2": "no flush needed: per-step working set (states 7x128 MB fp32, weights 1.5 GB) >> 126 MB L2"},
        "clocks": clk.summary(),
        "e2e": {"value": round(world * B * ek / e2e, 1), "unit": "samples/s",
                "h2d_bytes_per_step": B * (PC_SIZES[0] + PC_SIZES[-1]) * 4, "d2h_bytes_per_step": 4,
                "api": "BatchedPC.replay(inputs, targets) + energy read-back"},
        "gpu_launches": int(launched),
    }
    if flops:
        res["model_tflops_per_gpu"] = round(flops / (ms_step / 1e3) / 1e12, 1)
    return res
