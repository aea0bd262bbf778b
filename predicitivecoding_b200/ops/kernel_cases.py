"""Single-GPU cases, one per fused kernel family, for timing and profiler captures.

``python -m predicitivecoding_b200.ops.kernel_cases <case> [--time N]`` runs three launches
of the case's kernel (what a profiler capture with ``-s 1 -c 1`` expects); with ``--time N`` it
also times N launches with CUDA events after the warm-up and prints achieved TFLOP/s.
Inputs are sized above L2 where that is the point of the case (the PC GEMMs read a 128 MiB
weight) and kept to a few GB on the device.
"""
from __future__ import annotations

import argparse
import json

import torch

from . import ext, gemm, gemm_pc, attn_fwd, attn_bwd, EPI_SWIGLU, EPI_RED_F32, EPI_PC_PRED, EPI_PC_STATE

CASES = ("gemm_swiglu", "gemm_dw", "pc_pred", "pc_state", "attn_fwd", "attn_fwd_mma", "attn_bwd")


def build(which: str, dev: str = "cuda"):
    """Return (launch_fn, flops_per_launch) for one case."""
    bf = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(0)

    def rn(*s, scale=1.0):
        return (torch.randn(*s, device=dev, generator=g) * scale)

    if which == "gemm_swiglu":          # decoder W13 forward at the 124M shape, 8 sequences of 1024
        M, D, F = 8192, 768, 2048
        x, w = rn(M, D).to(bf), rn(2 * F, D, scale=0.03).to(bf)
        pre = torch.empty(M, 2 * F, device=dev, dtype=bf)
        act = torch.empty(M, F, device=dev, dtype=bf)
        return (lambda: gemm(x, w, epi=EPI_SWIGLU, c=pre, d=act)), 2 * M * 2 * F * D
    if which == "gemm_dw":              # weight-gradient GEMM: MN-major operands, split-K fp32 atomics
        M, N, K = 2048, 768, 8192
        a, b = rn(K, M).to(bf), rn(K, N).to(bf)
        c = torch.zeros(M, N, device=dev)
        return (lambda: gemm(a, b, a_mn=True, b_mn=True, epi=EPI_RED_F32, c=c)), 2 * M * N * K
    if which in ("pc_pred", "pc_state"):  # PC 8192 -> 8192 layer, batch 2048
        B, S = 2048, 8192
        w = rn(S, S, scale=0.01).to(bf)
        if which == "pc_pred":
            m16, mb = rn(B, S).to(bf), rn(B, S)
            e = torch.empty(B, S, device=dev)
            d = torch.empty(B, S, device=dev, dtype=bf)
            bias = torch.zeros(S, device=dev)
            fn = lambda: gemm_pc(m16, w, epi=EPI_PC_PRED, c=e, d=d, aux=mb, bias=bias, act="tanh")
        else:
            d, mu, e = rn(B, S).to(bf), rn(B, S), rn(B, S)
            mu16 = torch.empty(B, S, device=dev, dtype=bf)
            fn = lambda: gemm_pc(d, w, b_mn=True, epi=EPI_PC_STATE, c=mu, d=mu16, aux=e, eta=0.1)
        return fn, 2 * B * S * S
    if which in ("attn_fwd", "attn_fwd_mma", "attn_bwd"):  # causal attention, 8 x 1024 tokens, 12 heads of 64
        B, S, H, hd = 8, 1024, 12, 64
        D = H * hd
        qkv = rn(B * S, 3 * D).to(bf)
        o = torch.empty(B * S, D, device=dev, dtype=bf)
        lse = torch.empty(B * H, S, device=dev)
        causal_mm = B * H * S * S * hd          # one causal S x S x hd matmul = 2 * (S^2 / 2) * hd per head
        attn_fwd(qkv, o, lse, B, S, H, hd, 0.125)
        if which in ("attn_fwd", "attn_fwd_mma"):
            impl = "mma" if which == "attn_fwd_mma" else "tc"
            return (lambda: attn_fwd(qkv, o, lse, B, S, H, hd, 0.125, impl=impl)), 2 * causal_mm
        do = rn(B * S, D).to(bf)
        dq = torch.empty(B * S, D, device=dev)
        dv = torch.empty(B * H, S, device=dev)
        dqkv = torch.empty_like(qkv)
        return (lambda: attn_bwd(qkv, o, do, lse, dv, dq, dqkv, B, S, H, hd, 0.125)), 5 * causal_mm
    raise ValueError(f"unknown case {which!r}; one of {CASES}")


def time_case(which: str, iters: int = 20) -> dict:
    fn, flops = build(which)
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(iters):
        fn()
    t1.record()
    torch.cuda.synchronize()
    us = t0.elapsed_time(t1) * 1e3 / iters
    return {"case": which, "us": round(us, 2), "tflops": round(flops / us * 1e-6, 1)}


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("case", choices=CASES + ("all",))
    p.add_argument("--time", type=int, default=0, help="time N launches after warm-up")
    a = p.parse_args()
    ext()
    for c in (CASES if a.case == "all" else (a.case,)):
        if a.time:
            print(json.dumps(time_case(c, a.time)))
        else:
            fn, _ = build(c)
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            print("ok", c)


if __name__ == "__main__":
    main()
