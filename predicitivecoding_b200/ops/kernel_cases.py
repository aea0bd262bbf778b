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

from . import (ext, gemm, gemm_pc, attn_fwd, attn_bwd, EPI_BF16, EPI_F32, EPI_RESID_F32, EPI_SWIGLU, EPI_SWIGLU_BWD,
               EPI_RED_F32, EPI_PC_PRED, EPI_PC_STATE)

CASES = ("gemm_swiglu", "gemm_lmhead", "gemm_dw", "pc_pred", "pc_state", "attn_fwd", "attn_fwd_mma", "attn_bwd",
         "attn_fwd_d128", "attn_fwd_mma_d128", "attn_bwd_d128", "moe_fwd", "moe_layer", "skinny_qkv",
         "decode_attn_b32")


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
    if which == "gemm_lmhead":          # decoder LM head (vocabulary 32000, d 768) on 4 sequences of 1024
        M, D, V = 4096, 768, 32000
        x, w = rn(M, D).to(bf), rn(V, D, scale=0.03).to(bf)
        logits = torch.empty(M, V, device=dev, dtype=bf)
        return (lambda: gemm(x, w, epi=EPI_BF16, c=logits)), 2 * M * V * D
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
    if which.startswith("attn_"):
        # causal attention: 8 x 1024 tokens, 12 heads of 64 (the 124M decoder), or with the _d128 suffix
        # 8 x 2048 tokens, 16 heads of 128 (the 1.3B decoder)
        B, S, H, hd = (8, 2048, 16, 128) if which.endswith("_d128") else (8, 1024, 12, 64)
        which = which.replace("_d128", "")
        D = H * hd
        qkv = rn(B * S, 3 * D).to(bf)
        o = torch.empty(B * S, D, device=dev, dtype=bf)
        lse = torch.empty(B * H, S, device=dev)
        causal_mm = B * H * S * S * hd          # one causal S x S x hd matmul = 2 * (S^2 / 2) * hd per head
        sc = hd ** -0.5
        attn_fwd(qkv, o, lse, B, S, H, hd, sc)
        if which in ("attn_fwd", "attn_fwd_mma"):
            impl = "mma" if which == "attn_fwd_mma" else "tc"
            return (lambda: attn_fwd(qkv, o, lse, B, S, H, hd, sc, impl=impl)), 2 * causal_mm
        do = rn(B * S, D).to(bf)
        dq = torch.empty(B * S, D, device=dev)
        dv = torch.empty(B * H, S, device=dev)
        dqkv = torch.empty_like(qkv)
        return (lambda: attn_bwd(qkv, o, do, lse, dv, dq, dqkv, B, S, H, hd, sc)), 5 * causal_mm
    if which in ("moe_fwd", "moe_layer"):
        # mixture-of-experts FFN layer: 16 x 1024 tokens, d 768, 8 GELU experts of 3072, top-2
        from . import moe
        M, D, F_, E, k = 16384, 768, 3072, 8, 2
        x = rn(M, D).to(bf)
        router, w1, w2 = rn(E, D, scale=0.05).to(bf), rn(E * F_, D, scale=0.03).to(bf), rn(E * D, F_, scale=0.02).to(bf)
        b1, b2 = torch.zeros(E * F_, device=dev), torch.zeros(E * D, device=dev)
        res, out = rn(M, D), torch.empty(M, D, device=dev)
        buf = moe.MoEBuffers.allocate(M, D, F_, E, k, dev)
        flops = k * M * 2 * 2 * D * F_
        if which == "moe_fwd":
            return (lambda: moe.forward(x, res, out, router, w1, b1, w2, b2, k, buf)), flops
        scr = moe.MoEScratch.allocate(M, D, F_, E, k, dev)
        dx, dn = rn(M, D), torch.empty(M, D, device=dev)
        grads = [torch.zeros(E, D, device=dev), torch.zeros(E * F_, D, device=dev), torch.zeros(E * F_, device=dev),
                 torch.zeros(E * D, F_, device=dev), torch.zeros(E * D, device=dev)]

        def layer():
            moe.forward(x, res, out, router, w1, b1, w2, b2, k, buf)
            moe.backward(dx, x, dn, router, w1, w2, k, buf, scr, *grads, 0.01)
        return layer, 3 * flops
    if which == "skinny_qkv":           # decode projection of the 1.3B decoder: 32 rows, K 2048, N 6144
        x, w = rn(32, 2048).to(bf), rn(2048, 6144, scale=0.02).to(bf)
        y = torch.empty(32, 6144, device=dev, dtype=bf)
        from . import linear
        return (lambda: linear(x, w, out=y)), 2 * 32 * 2048 * 6144
    if which == "decode_attn_b32":      # decode attention: batch 32, 16 heads of 128, 640 cached keys
        from . import decode_attn
        B, H, hd, L, cap = 32, 16, 128, 640, 768
        q = rn(B, H, hd).to(bf)
        kc, vc = rn(B, H, cap, hd).to(bf), rn(B, H, cap, hd).to(bf)
        lens = torch.full((B,), L, dtype=torch.int32, device=dev)
        return (lambda: decode_attn(q, kc, vc, lens, hd ** -0.5)), 4 * B * H * L * hd
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


def decoder_gemm_table(iters: int = 20) -> list:
    """Every GEMM of one layer of the 124M decoder step (micro-batch 16 x 1024 tokens) plus the LM head,
    with the epilogue the fused trainer uses; CUDA-event time per launch and TFLOP/s."""
    dev = "cuda"
    M, D, F, V = 16384, 768, 2048, 32000
    bf = torch.bfloat16

    def rn(*shape, dt=bf):
        return torch.randn(*shape, device=dev).to(dt)

    rows = []

    def t(fn, flops, name, it=iters):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(it):
            fn()
        b.record()
        torch.cuda.synchronize()
        us = a.elapsed_time(b) * 1e3 / it
        rows.append({"gemm": name, "us": round(us, 1), "tflops": round(flops / us * 1e-6, 1)})

    n1, x = rn(M, D), rn(M, D, dt=torch.float32)
    wqkv, wo, w13, w2, wout = rn(3 * D, D), rn(D, D), rn(2 * F, D), rn(D, F), rn(V, D)
    qkv = torch.empty(M, 3 * D, device=dev, dtype=bf)
    xo = torch.empty(M, D, device=dev)
    pre = torch.empty(M, 2 * F, device=dev, dtype=bf)
    act = torch.empty(M, F, device=dev, dtype=bf)
    logits = torch.empty(M, V, device=dev, dtype=bf)
    dn = torch.empty(M, D, device=dev)
    t(lambda: gemm(n1, wqkv, epi=EPI_BF16, c=qkv), 2 * M * D * 3 * D, "qkv fwd [M,2304,768] bf16")
    ao = rn(M, D)
    t(lambda: gemm(ao, wo, epi=EPI_RESID_F32, c=xo, aux=x), 2 * M * D * D, "o fwd [M,768,768] +resid f32")
    t(lambda: gemm(n1, w13, epi=EPI_SWIGLU, c=pre, d=act), 2 * M * D * 2 * F, "w13 fwd [M,4096,768] swiglu")
    t(lambda: gemm(act, w2, epi=EPI_RESID_F32, c=xo, aux=x), 2 * M * F * D, "w2 fwd [M,768,2048] +resid f32")
    t(lambda: gemm(n1, wout, epi=EPI_BF16, c=logits), 2 * M * D * V, "lm head [M,32000,768]", 5)
    t(lambda: gemm(logits, wout, b_mn=True, epi=EPI_F32, c=dn), 2 * M * D * V, "lm dgrad [M,768,32000]", 5)
    gW = torch.zeros(V, D, device=dev)
    t(lambda: gemm(logits, n1, a_mn=True, b_mn=True, epi=EPI_RED_F32, c=gW), 2 * M * D * V, "lm wgrad [32000,768,M]", 5)
    dx16, dpre = rn(M, D), torch.empty(M, 2 * F, device=dev, dtype=bf)
    t(lambda: gemm(dx16, w2, b_mn=True, epi=EPI_SWIGLU_BWD, c=dpre, aux=pre), 2 * M * D * F,
      "w2 dgrad [M,2048,768] swiglu bwd")
    g2 = torch.zeros(D, F, device=dev)
    t(lambda: gemm(dx16, act, a_mn=True, b_mn=True, epi=EPI_RED_F32, c=g2), 2 * M * D * F, "w2 wgrad [768,2048,M]")
    g13 = torch.zeros(2 * F, D, device=dev)
    t(lambda: gemm(dpre, n1, a_mn=True, b_mn=True, epi=EPI_RED_F32, c=g13), 2 * M * D * 2 * F, "w13 wgrad [4096,768,M]")
    t(lambda: gemm(dpre, w13, b_mn=True, epi=EPI_F32, c=dn), 2 * M * D * 2 * F, "w13 dgrad [M,768,4096] f32")
    dao = torch.empty(M, D, device=dev, dtype=bf)
    t(lambda: gemm(dx16, wo, b_mn=True, epi=EPI_BF16, c=dao), 2 * M * D * D, "o dgrad [M,768,768] bf16")
    go = torch.zeros(D, D, device=dev)
    t(lambda: gemm(dx16, ao, a_mn=True, b_mn=True, epi=EPI_RED_F32, c=go), 2 * M * D * D, "o wgrad [768,768,M]")
    dqkv = rn(M, 3 * D)
    gq = torch.zeros(3 * D, D, device=dev)
    t(lambda: gemm(dqkv, n1, a_mn=True, b_mn=True, epi=EPI_RED_F32, c=gq), 2 * M * D * 3 * D, "qkv wgrad [2304,768,M]")
    t(lambda: gemm(dqkv, wqkv, b_mn=True, epi=EPI_F32, c=dn), 2 * M * D * 3 * D, "qkv dgrad [M,768,2304] f32")
    return rows


def decode_linear_table(iters: int = 50) -> list:
    """Decode-sized projections (<= 32 rows) of the 1.3B decoder on the skinny tcgen05 kernel, on the
    regular tcgen05 GEMM, through ops.linear (which picks one of the two) and on torch.matmul (cuBLAS,
    for reference): device time per launch from CUDA
    events around one replay of a CUDA graph of `iters` launches (launch overhead out, programmatic
    launch overlap in)."""
    from . import linear
    import predicitivecoding_b200.ops as ops_mod
    dev = "cuda"

    def graph_us(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        g, s = torch.cuda.CUDAGraph(), torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for _ in range(iters):
                    fn()
        torch.cuda.current_stream().wait_stream(s)
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) * 1e3 / iters

    rows = []
    for name, (M, K, N) in (("qkv", (32, 2048, 6144)), ("o", (32, 2048, 2048)), ("w13", (32, 2048, 11008)),
                            ("w2", (32, 5504, 2048)), ("lm head", (32, 2048, 32000)), ("qkv, 8 rows", (8, 2048, 6144)),
                            ("124M qkv", (32, 768, 2304))):
        x = torch.randn(M, K, device=dev).to(torch.bfloat16)
        w = (torch.randn(K, N, device=dev) * 0.02).to(torch.bfloat16)
        y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        sk = graph_us(lambda: ext().skinny_gemm(x, w, y))
        keep = ops_mod.SKINNY_MAX_ROWS
        try:
            ops_mod.SKINNY_MAX_ROWS = 0
            reg = graph_us(lambda: linear(x, w, out=y))
            ops_mod.SKINNY_MAX_ROWS = 32
            routed = graph_us(lambda: linear(x, w, out=y))
        finally:
            ops_mod.SKINNY_MAX_ROWS = keep
        tm = graph_us(lambda: torch.matmul(x, w, out=y))
        rows.append({"shape": name, "M": M, "K": K, "N": N, "skinny_us": round(sk, 2), "tcgen05_gemm_us": round(reg, 2),
                     "ops_linear_us": round(routed, 2), "torch_matmul_us": round(tm, 2),
                     "skinny_weight_TBps": round(K * N * 2 / sk / 1e6, 2)})
    return rows


def decode_attn_split_table(iters: int = 20) -> list:
    """Split-KV decode attention of the 1.3B decoder's decode step (batch 32, 640 cached keys of hd 128;
    16 heads at TP=1, 8 at TP=2) for each key-split count: device time per call from CUDA events around
    one replay of a CUDA graph of `iters` calls, and the K/V stream rate."""
    from . import decode_attn
    dev = "cuda"
    rows = []
    for (B, H, hd, L, cap) in ((32, 16, 128, 640, 768), (32, 8, 128, 640, 768)):
        q = torch.randn(B, H, hd, device=dev).to(torch.bfloat16)
        kc = torch.randn(B, H, cap, hd, device=dev).to(torch.bfloat16)
        vc = torch.randn(B, H, cap, hd, device=dev).to(torch.bfloat16)
        lens = torch.full((B,), L, dtype=torch.int32, device=dev)
        out = torch.empty_like(q)
        for ns in (1, 2, 3, 4, 8):
            scratch = (torch.empty(B * H * ns * hd, device=dev), torch.empty(B * H * ns * 2, device=dev))
            fn = lambda: decode_attn(q, kc, vc, lens, hd ** -0.5, nsplit=ns, out=out, scratch=scratch)
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            g, st = torch.cuda.CUDAGraph(), torch.cuda.Stream()
            st.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(st):
                with torch.cuda.graph(g, stream=st):
                    for _ in range(iters):
                        fn()
            torch.cuda.current_stream().wait_stream(st)
            g.replay()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            g.replay()
            b.record()
            torch.cuda.synchronize()
            us = a.elapsed_time(b) * 1e3 / iters
            rows.append({"batch": B, "heads": H, "hd": hd, "keys": L, "nsplit": ns, "us": round(us, 2),
                         "kv_TBps": round(2 * B * H * L * hd * 2 / us / 1e6, 2)})
    return rows


def step_breakdown(steps: int = 2) -> list:
    """Device time per kernel of one step of the 124M decoder trainer (micro-batch 16 x 1024), from the
    CUDA activity records of torch.profiler over `steps` steps after 3 warm-up steps; eager launches
    (no CUDA graph) so that every kernel record is attributed. Returns rows sorted by time."""
    from ..engine.fused_trainer import FusedDecoderTrainer
    from ..models.config import DecoderLmConfig
    from ..utils.data import zipf_windows
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = DecoderLmConfig.gpt2_small_swiglu()
    B, S = 16, cfg.max_seq
    tok, tgt = zipf_windows(B, S, cfg.vocab, 1.1, seed=1)
    tok, tgt = tok.to(torch.int32).pin_memory(), tgt.to(torch.int32).pin_memory()
    tr = FusedDecoderTrainer(cfg, B, S, device=dev, lr=3e-4, weight_decay=0.1, use_graph=False)
    tr.stage(tok, tgt)
    for _ in range(3):
        tr.step(tok, tgt)
    torch.cuda.synchronize()
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        for _ in range(steps):
            tr.step(tok, tgt)
        torch.cuda.synchronize()
    rows = []
    for e in prof.key_averages():
        t = getattr(e, "device_time_total", 0.0)
        if t > 0:
            rows.append({"kernel": e.key[:120], "us_per_step": round(t / steps, 1), "launches_per_step": e.count // steps})
    rows.sort(key=lambda r: -r["us_per_step"])
    return rows


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("case", choices=CASES + ("all", "decoder_gemms", "decode_linears", "decode_attn_splits",
                                            "step_breakdown"))
    p.add_argument("--time", type=int, default=0, help="time N launches after warm-up")
    a = p.parse_args()
    ext()
    if a.case == "decoder_gemms":
        for row in decoder_gemm_table():
            print(json.dumps(row))
        return
    if a.case == "decode_attn_splits":
        for row in decode_attn_split_table():
            print(json.dumps(row))
        return
    if a.case == "decode_linears":
        for row in decode_linear_table():
            print(json.dumps(row))
        return
    if a.case == "step_breakdown":
        rows = step_breakdown()
        print(json.dumps({"kernel_us_per_step": round(sum(r["us_per_step"] for r in rows), 1)}))
        for row in rows:
            print(json.dumps(row))
        return
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
