"""Float32 vs mixed precision, measured in-house (median of 5 after warm-up).

Reference: tools/MixedPrecisionBench/Program.cs (MatVec / MatVecT float vs half weights, PC network
inference float vs mixed at CIFAR scale, GEMM 1024^3 CPU float vs CPU mixed vs CUDA).  Here the GPU
rows use the tcgen05 GEMM (bf16 in, fp32 accumulate) timed with CUDA events.
"""
from __future__ import annotations

import statistics
import time

import torch


def median_ms(fn, reps: int = 5, warmup: int = 2) -> float:
    for _ in range(warmup):
        fn()
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        ts.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(ts)


def cuda_ms(fn, reps: int = 5, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ts = []
    for _ in range(reps):
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


def run(rows=None) -> list:
    from ..pc.network import Network, NetworkConfig
    out = []
    g = torch.Generator().manual_seed(1)
    for n in (512, 2048):
        w = torch.randn(n, n, generator=g) * 0.05
        wh = w.half()
        v = torch.randn(n, generator=g)
        out.append(("MatVec", f"{n}x{n}", median_ms(lambda: w @ v), median_ms(lambda: (wh.float() @ v))))
        out.append(("MatVecT", f"{n}x{n}", median_ms(lambda: w.T @ v), median_ms(lambda: (wh.float().T @ v))))
    net = Network(NetworkConfig(layer_sizes=(3072, 512, 128, 10), state_lr=0.05), seed=0)
    x = torch.randn(3072, generator=g)
    out.append(("PC infer (20 steps)", "3072-512-128-10", median_ms(lambda: net.infer_get_top(x, 20, True), 3, 1),
                median_ms(lambda: net.infer_get_top(x, 20, True, mixed=True), 3, 1)))
    a = torch.randn(1024, 1024, generator=g)
    b = torch.randn(1024, 1024, generator=g)
    row = ["GEMM", "1024^3", median_ms(lambda: a @ b), median_ms(lambda: a.half().float() @ b.half().float())]
    if torch.cuda.is_available():
        from .. import ops
        a16, b16 = a.cuda().bfloat16(), b.cuda().bfloat16().T.contiguous()
        row.append(cuda_ms(lambda: ops.gemm(a16, b16, epi=ops.EPI_F32)))
    out.append(tuple(row))
    return out


def main() -> None:
    print("| op | size | float32 ms | mixed ms | B200 tcgen05 ms |")
    print("|----|------|-----------:|---------:|----------------:|")
    for r in run():
        print(f"| {r[0]} | {r[1]} | {r[2]:.3f} | {r[3]:.3f} | {r[4]:.4f} |" if len(r) > 4 else
              f"| {r[0]} | {r[1]} | {r[2]:.3f} | {r[3]:.3f} | - |")


if __name__ == "__main__":
    main()
