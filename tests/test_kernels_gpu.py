"""Numerics of every sm_100a kernel against a plain PyTorch fp32 reference of the same op.

Tolerances follow the reference's own GPU parity tests: bf16 GEMM within 0.02
relative (TEST/PredicitiveCoding.UnitTests/LlmDeviceTrainTests.cs:302-335), fused
attention forward/backward vs autograd (:90-182, loosened from 1e-4 for bf16 operands).
"""
import math

import pytest
import torch

from predicitivecoding_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-12))


def _operands(M, N, K, a_mn, b_mn, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    A = torch.randn(M, K, generator=g).to(DEV, torch.bfloat16)       # logical [M, K]
    B = torch.randn(K, N, generator=g).to(DEV, torch.bfloat16)       # logical [K, N]
    a_st = A.t().contiguous() if a_mn else A.contiguous()            # stored [K,M] or [M,K]
    b_st = B.contiguous() if b_mn else B.t().contiguous()            # stored [K,N] or [N,K]
    ref = A.float() @ B.float()
    return a_st, b_st, ref


@pytest.fixture(params=["single", "pair"])
def gemm_mode(request):
    ops.ext().set_gemm_mode(1 if request.param == "single" else 2)
    yield request.param
    ops.ext().set_gemm_mode(-1)


@pytest.mark.parametrize("a_mn", [False, True])
@pytest.mark.parametrize("b_mn", [False, True])
@pytest.mark.parametrize("shape", [(256, 256, 128), (384, 512, 320), (200, 136, 72), (1024, 768, 2048),
                                   (640, 384, 192)])
def test_gemm_layouts(a_mn, b_mn, shape, gemm_mode):
    M, N, K = shape
    a, b, ref = _operands(M, N, K, a_mn, b_mn)
    out = torch.empty(M, N, device=DEV, dtype=torch.float32)
    ops.gemm(a, b, a_mn=a_mn, b_mn=b_mn, epi=ops.EPI_F32, c=out)
    torch.cuda.synchronize()
    assert rel_err(out, ref) < 1e-3, rel_err(out, ref)


@pytest.mark.parametrize("bn", [128, 256])
def test_gemm_pair_epilogues(bn, gemm_mode):
    M, N, K = 768, 512, 320
    a, b, ref = _operands(M, N, K, False, False, seed=9)
    x = torch.randn(M, N, device=DEV)
    out = torch.empty_like(x)
    ops.gemm(a, b, epi=ops.EPI_RESID_F32, c=out, aux=x, bn=bn)
    red = torch.zeros(M, N, device=DEV)
    a2, b2, ref2 = _operands(M, N, 4096, True, True, seed=10)
    ops.gemm(a2, b2, a_mn=True, b_mn=True, epi=ops.EPI_RED_F32, c=red, splits=4, bn=bn)
    torch.cuda.synchronize()
    assert rel_err(out, ref + x) < 1e-3
    assert rel_err(red, ref2) < 1e-3


@pytest.mark.parametrize("bn", [128, 256])
@pytest.mark.parametrize("shape", [(512, 512, 256), (200, 136, 72), (1000, 100, 128), (768, 2304, 192)])
def test_gemm_bf16_out_and_bias(bn, shape, gemm_mode):
    # (200, 136): TMA-store boxes clipped at the row and column edges; (1000, 100): a row stride that is
    # not a multiple of 16 bytes, so the epilogue stores without a tensor map
    M, N, K = shape
    a, b, ref = _operands(M, N, K, False, False, seed=1)
    bias = torch.randn(N, device=DEV)
    padded = torch.full((M, N + 8), 7.0, device=DEV, dtype=torch.bfloat16)
    out = padded[:, :N]
    ops.gemm(a, b, epi=ops.EPI_BF16, c=out, bias=bias, alpha=0.5, bn=bn)
    torch.cuda.synchronize()
    assert rel_err(out, 0.5 * ref + bias) < 0.02
    assert bool((padded[:, N:] == 7.0).all()), "bf16 epilogue wrote past the last column"


@pytest.mark.parametrize("bn", [128, 256])
def test_gemm_bf16_fused_rope(bn, gemm_mode):
    # the q/k columns [0, 2D) of a fused qkv projection rotated in the epilogue, v columns untouched
    from predicitivecoding_b200.models.decoder_lm import rope_tables
    S, hd, D = 256, 64, 256
    M, N, K = 2 * S, 3 * D, 192
    a, b, ref = _operands(M, N, K, False, False, seed=4)
    cos, sin = rope_tables(S, hd, device=DEV)
    cs = torch.stack((cos, sin), -1).contiguous()
    out = ops.gemm(a, b, epi=ops.EPI_BF16, bn=bn, rope=(cs, S, hd, 2 * D))
    expect = ref.to(torch.bfloat16)
    ops.rope(expect, cs, S, D, hd, 2, 1.0)
    torch.cuda.synchronize()
    assert rel_err(out, expect.float()) < 0.02


def test_gemm_split_k_red():
    M, N, K = 256, 384, 4096
    a, b, ref = _operands(M, N, K, True, True, seed=2)
    out = torch.ones(M, N, device=DEV)
    ops.gemm(a, b, a_mn=True, b_mn=True, epi=ops.EPI_RED_F32, c=out, splits=8)
    torch.cuda.synchronize()
    assert rel_err(out, ref + 1.0) < 1e-3


@pytest.mark.parametrize("shape", [(512, 256, 192), (200, 136, 72), (300, 102, 64)])
@pytest.mark.parametrize("with_bias", [False, True])
def test_gemm_resid(shape, with_bias, gemm_mode):
    # (200, 136): TMA boxes clipped at both edges; (300, 102): rows of 408 bytes, no tensor maps
    M, N, K = shape
    a, b, ref = _operands(M, N, K, False, False, seed=3)
    x = torch.randn(M, N, device=DEV)
    bias = torch.randn(N, device=DEV) if with_bias else None
    padded = torch.full((M, N + 4), 5.0, device=DEV)
    out = padded[:, :N]
    ops.gemm(a, b, epi=ops.EPI_RESID_F32, c=out, aux=x, bias=bias, alpha=0.5)
    torch.cuda.synchronize()
    expect = 0.5 * ref + x + (bias if with_bias else 0.0)
    assert rel_err(out, expect) < 1e-3
    assert bool((padded[:, N:] == 5.0).all())


def _gelu(x):
    return 0.5 * x * (1 + torch.tanh(0.7978845608 * (x + 0.044715 * x ** 3)))


def test_gemm_gelu_and_bwd(gemm_mode):
    M, N, K = 512, 512, 256
    a, b, ref = _operands(M, N, K, False, False, seed=4)
    ref = ref / 16
    bias = torch.randn(N, device=DEV) * 0.1
    pre = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    act = torch.empty_like(pre)
    ops.gemm(a, b, epi=ops.EPI_GELU, c=pre, d=act, bias=bias, alpha=1 / 16)
    torch.cuda.synchronize()
    assert rel_err(pre, ref + bias) < 0.02
    assert rel_err(act, _gelu(pre.float())) < 0.02
    # backward: d(pre) = (dact) * gelu'(pre), dact = a2 @ b2
    a2, b2, dact = _operands(M, N, K, False, True, seed=5)
    dpre = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    ops.gemm(a2, b2, b_mn=True, epi=ops.EPI_GELU_BWD, c=dpre, aux=pre)
    x = pre.float().requires_grad_()
    _gelu(x).backward(dact)
    torch.cuda.synchronize()
    assert rel_err(dpre, x.grad) < 0.02


@pytest.mark.parametrize("shape", [(512, 256, 192), (200, 384, 128)])
def test_gemm_swiglu_and_bwd(shape, gemm_mode):
    M, F, D = shape
    g = torch.Generator().manual_seed(6)
    x = torch.randn(M, D, generator=g).to(DEV, torch.bfloat16)
    wg = (torch.randn(F, D, generator=g) / 8).to(DEV, torch.bfloat16)
    wu = (torch.randn(F, D, generator=g) / 8).to(DEV, torch.bfloat16)
    from predicitivecoding_b200.engine.fused_trainer import _interleave_gate_up
    w13 = _interleave_gate_up(wg, wu).contiguous()
    pre = torch.empty(M, 2 * F, device=DEV, dtype=torch.bfloat16)
    act = torch.empty(M, F, device=DEV, dtype=torch.bfloat16)
    ops.gemm(x, w13, epi=ops.EPI_SWIGLU, c=pre, d=act)
    gr = x.float() @ wg.float().t()
    ur = x.float() @ wu.float().t()
    ref = torch.nn.functional.silu(gr) * ur
    torch.cuda.synchronize()
    assert rel_err(act, ref) < 0.02
    assert rel_err(pre, x.float() @ w13.float().t()) < 0.01
    # backward through the interleaved layout
    dh = torch.randn(M, F, device=DEV)
    w2 = torch.randn(D, F, device=DEV).to(torch.bfloat16)  # stored [K=D? no] -> use dact = y @ w2
    y = torch.randn(M, D, device=DEV).to(torch.bfloat16)
    dact = y.float() @ w2.float()
    dpre = torch.empty_like(pre)
    ops.gemm(y, w2, b_mn=True, epi=ops.EPI_SWIGLU_BWD, c=dpre, aux=pre)
    pre_f = pre.float().view(M, F // 64, 2, 64)
    gg = pre_f[:, :, 0].reshape(M, F).requires_grad_()
    uu = pre_f[:, :, 1].reshape(M, F).requires_grad_()
    (torch.nn.functional.silu(gg) * uu).backward(dact)
    torch.cuda.synchronize()
    d = dpre.float().view(M, F // 64, 2, 64)
    assert rel_err(d[:, :, 0].reshape(M, F), gg.grad) < 0.02
    assert rel_err(d[:, :, 1].reshape(M, F), uu.grad) < 0.02


@pytest.mark.parametrize("D", [768, 2048, 3072])
def test_rmsnorm_fwd_bwd(D):
    M = 1000
    x = torch.randn(M, D, device=DEV)
    g = (1 + 0.1 * torch.randn(D, device=DEV)).to(torch.bfloat16)
    y = torch.empty(M, D, device=DEV, dtype=torch.bfloat16)
    inv = torch.empty(M, device=DEV)
    ops.rmsnorm_fwd(x, g, y, inv, 1e-5)
    xr = x.clone().requires_grad_()
    gr = g.float().clone().requires_grad_()
    ref = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-5) * gr
    assert rel_err(y, ref) < 0.01
    dy = torch.randn(M, D, device=DEV)
    ref.backward(dy)
    dx = torch.ones(M, D, device=DEV)
    dx16 = torch.empty(M, D, device=DEV, dtype=torch.bfloat16)
    dg = torch.zeros(D, device=DEV)
    ops.rmsnorm_bwd(dy, x, g, inv, dx, dg, accumulate=True, dx16=dx16)
    torch.cuda.synchronize()
    assert rel_err(dx, xr.grad + 1) < 1e-4
    assert rel_err(dx16, xr.grad + 1) < 0.01
    assert rel_err(dg, gr.grad) < 1e-4


def test_rope_roundtrip_and_values():
    from predicitivecoding_b200.models.decoder_lm import apply_rope, rope_tables
    B, S, H, hd = 2, 128, 4, 64
    D = H * hd
    qkv = torch.randn(B * S, 3 * D, device=DEV).to(torch.bfloat16)
    cos, sin = rope_tables(S, hd, device=DEV)
    cs = torch.stack((cos, sin), -1).contiguous()
    out = qkv.clone()
    ops.rope(out, cs, S, D, hd, 2, 1.0)
    q = qkv[:, :D].float().view(B, S, H, hd).transpose(1, 2)
    ref = apply_rope(q, cos, sin).transpose(1, 2).reshape(B * S, D)
    torch.cuda.synchronize()
    assert rel_err(out[:, :D], ref) < 0.01
    assert torch.equal(out[:, 2 * D:], qkv[:, 2 * D:])
    ops.rope(out, cs, S, D, hd, 2, -1.0)
    torch.cuda.synchronize()
    assert rel_err(out, qkv) < 0.02


@pytest.mark.parametrize("V", [32000, 1000, 4104, 50257])
def test_cross_entropy_fused(V):
    # 32000 / 1000 / 4104: register-resident rows (8, 1 and 2 vectors per thread); 50257: streaming path
    M = 300
    logits = (torch.randn(M, V, device=DEV) * 2).to(torch.bfloat16)
    tgt = torch.randint(0, V, (M,), device=DEV, dtype=torch.int32)
    tgt[5] = -1
    loss = torch.empty(M, device=DEV)
    lg = logits.float().clone().requires_grad_()
    keep = tgt >= 0
    ref_rows = torch.nn.functional.cross_entropy(lg, tgt.long().clamp(min=0), reduction="none") * keep
    (ref_rows.sum() / M).backward()
    buf = logits.clone()
    ops.cross_entropy(buf, tgt, loss, 1.0 / M, True)
    torch.cuda.synchronize()
    assert rel_err(loss, ref_rows) < 1e-3
    assert rel_err(buf, lg.grad) < 0.02
    assert float(buf[5].float().abs().max()) == 0.0


def test_adamw_matches_reference_order():
    n = 10000
    w = torch.randn(n, device=DEV)
    g = torch.randn(n, device=DEV)
    m = torch.zeros(n, device=DEV)
    v = torch.zeros(n, device=DEV)
    w16 = torch.empty(n, device=DEV, dtype=torch.bfloat16)
    lr, wd, b1, b2, eps = 1e-2, 0.1, 0.9, 0.999, 1e-8
    wr, mr, vr = w.clone(), m.clone(), v.clone()
    for t in range(1, 4):
        hyper = torch.tensor([lr, wd, 1 - b1 ** t, 1 - b2 ** t, 1.0, 0, 0, 0], device=DEV)
        ops.adamw(w, g, m, v, w16, n // 2, hyper, b1, b2, eps)
        mr = b1 * mr + (1 - b1) * g
        vr = b2 * vr + (1 - b2) * g * g
        wr = wr - lr * (mr / (1 - b1 ** t)) / ((vr / (1 - b2 ** t)).sqrt() + eps)
        wr[: n // 2] = wr[: n // 2] - lr * wd * wr[: n // 2]
    torch.cuda.synchronize()
    assert rel_err(w, wr) < 1e-6
    assert rel_err(w16, wr) < 0.01


@pytest.mark.parametrize("impl", ["tc", "mma"])
@pytest.mark.parametrize("hd", [64, 128])
def test_attention_fwd_bwd(hd, impl):
    B, S, H = 2, 256, 2
    D = H * hd
    qkv = (torch.randn(B * S, 3 * D, device=DEV)).to(torch.bfloat16)
    out = torch.empty(B * S, D, device=DEV, dtype=torch.bfloat16)
    lse = torch.empty(B * H, S, device=DEV)
    scale = 1 / math.sqrt(hd)
    ops.attn_fwd(qkv, out, lse, B, S, H, hd, scale, impl=impl)
    q, k, v = (qkv.float()[:, i * D:(i + 1) * D].view(B, S, H, hd).transpose(1, 2).clone().requires_grad_()
               for i in range(3))
    s = (q @ k.transpose(-1, -2)) * scale
    mask = torch.ones(S, S, dtype=torch.bool, device=DEV).triu(1)
    s = s.masked_fill(mask, float("-inf"))
    p = torch.softmax(s, -1)
    o = (p @ v)
    ref = o.transpose(1, 2).reshape(B * S, D)
    torch.cuda.synchronize()
    assert rel_err(out, ref) < 0.02
    assert rel_err(lse.view(B, H, S), torch.logsumexp(s, -1)) < 1e-3
    do = torch.randn(B * S, D, device=DEV).to(torch.bfloat16)
    o.backward(do.float().view(B, S, H, hd).transpose(1, 2))
    dqkv = torch.zeros(B * S, 3 * D, device=DEV, dtype=torch.bfloat16)
    dvec = torch.empty(B * H, S, device=DEV)
    dq_acc = torch.empty(B * S, D, device=DEV)
    ops.attn_bwd(qkv, out, do, lse, dvec, dq_acc, dqkv, B, S, H, hd, scale, impl=impl)
    torch.cuda.synchronize()
    for i, t in enumerate((q, k, v)):
        ref_g = t.grad.transpose(1, 2).reshape(B * S, D)
        assert rel_err(dqkv[:, i * D:(i + 1) * D], ref_g) < 0.03, ("qkv"[i], rel_err(dqkv[:, i * D:(i + 1) * D], ref_g))


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("S,mag", [(1024, 1.5), (512, 4.0), (2048, 0.5)])
def test_attention_tc_long_sequence(S, mag, hd):
    """Many key tiles per tile pair: the K/V ring, both softmax warpgroups, diagonal masking, the early
    release of S (head dim 64) or P over S (head dim 128), and (large magnitudes) the lazy rescaling of O
    in tensor memory; several items per CTA (B * H * S / 256 > 148 for S = 2048 at B = 2, H = 3 is not,
    so the persistent loop is covered by the decoder-shaped case below)."""
    B, H = 2, 3
    D = H * hd
    g = torch.Generator(device=DEV).manual_seed(S)
    qkv = (torch.randn(B * S, 3 * D, device=DEV, generator=g) * mag).to(torch.bfloat16)
    out = torch.empty(B * S, D, device=DEV, dtype=torch.bfloat16)
    lse = torch.empty(B * H, S, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    scale = 1 / math.sqrt(hd)
    assert ops.tc_attention_supported(S, hd)
    assert ops.ext().attn_fwd_tc(qkv, out, lse, B, S, H, hd, scale, err) == 0
    q, k, v = (qkv.float()[:, i * D:(i + 1) * D].view(B, S, H, hd).transpose(1, 2) for i in range(3))
    s = (q @ k.transpose(-1, -2)) * scale
    s = s.masked_fill(torch.ones(S, S, dtype=torch.bool, device=DEV).triu(1), float("-inf"))
    ref = (torch.softmax(s, -1) @ v).transpose(1, 2).reshape(B * S, D)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert rel_err(out, ref) < 0.02
    assert rel_err(lse.view(B, H, S), torch.logsumexp(s, -1)) < 1e-3


@pytest.mark.parametrize("hd", [64, 128])
def test_attention_fwd_tc_persistent_items(hd):
    """More tile pairs than CTAs (B * H * S / 256 = 384 > 148): each persistent CTA runs several items,
    reusing Q buffers, the K/V ring and the TMEM accumulators across them."""
    B, S, H = 16, 1024, 6
    D = H * hd
    g = torch.Generator(device=DEV).manual_seed(hd)
    qkv = torch.randn(B * S, 3 * D, device=DEV, generator=g).to(torch.bfloat16)
    out = torch.empty(B * S, D, device=DEV, dtype=torch.bfloat16)
    lse = torch.empty(B * H, S, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    scale = 1 / math.sqrt(hd)
    assert ops.ext().attn_fwd_tc(qkv, out, lse, B, S, H, hd, scale, err) == 0
    q, k, v = (qkv.float()[:, i * D:(i + 1) * D].view(B, S, H, hd).transpose(1, 2) for i in range(3))
    s = (q @ k.transpose(-1, -2)) * scale
    s = s.masked_fill(torch.ones(S, S, dtype=torch.bool, device=DEV).triu(1), float("-inf"))
    ref = (torch.softmax(s, -1) @ v).transpose(1, 2).reshape(B * S, D)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert rel_err(out, ref) < 0.02
    assert rel_err(lse.view(B, H, S), torch.logsumexp(s, -1)) < 1e-3


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("S,B,H", [(1024, 2, 3), (384, 3, 2)])
def test_attention_bwd_tc_matches_autograd(S, B, H, hd):
    """tcgen05 backward over many key/query tiles (persistent CTAs, the Q/dO ring, dQ reductions),
    with and without the RoPE rotation of dq/dk; head dim 128 uses 64-query tiles and the transposed
    dQ product."""
    D = H * hd
    g = torch.Generator(device=DEV).manual_seed(S + B)
    qkv = torch.randn(B * S, 3 * D, device=DEV, generator=g).to(torch.bfloat16)
    scale = 1 / math.sqrt(hd)
    out = torch.empty(B * S, D, device=DEV, dtype=torch.bfloat16)
    lse = torch.empty(B * H, S, device=DEV)
    ops.attn_fwd(qkv, out, lse, B, S, H, hd, scale, impl="mma")
    do = torch.randn(B * S, D, device=DEV, generator=g).to(torch.bfloat16)
    q, k, v = (qkv.float()[:, i * D:(i + 1) * D].view(B, S, H, hd).transpose(1, 2).clone().requires_grad_()
               for i in range(3))
    s = ((q @ k.transpose(-1, -2)) * scale).masked_fill(
        torch.ones(S, S, dtype=torch.bool, device=DEV).triu(1), float("-inf"))
    (torch.softmax(s, -1) @ v).backward(do.float().view(B, S, H, hd).transpose(1, 2))
    ref = [t.grad.transpose(1, 2).reshape(B * S, D) for t in (q, k, v)]
    pos = torch.arange(S, device=DEV, dtype=torch.float32)
    inv = 10000.0 ** (-torch.arange(0, hd, 2, device=DEV, dtype=torch.float32) / hd)
    ang = pos[:, None] * inv[None, :]
    cs = torch.stack([ang.cos(), ang.sin()], -1).contiguous()          # [S, hd/2, 2]
    for rope in (None, cs):
        dqkv = torch.zeros(B * S, 3 * D, device=DEV, dtype=torch.bfloat16)
        dvec = torch.empty(B * H, S, device=DEV)
        dq_acc = torch.empty(B * S, D, device=DEV)
        err = torch.zeros(1, dtype=torch.int32, device=DEV)
        rc = ops.ext().attn_bwd_tc(qkv, out, do, lse, dvec, dq_acc, dqkv, B, S, H, hd, scale, rope, err)
        torch.cuda.synchronize()
        assert rc == 0 and int(err.item()) == 0
        got = [dqkv[:, i * D:(i + 1) * D].float() for i in range(3)]
        if rope is not None:  # rotate the reference dq, dk by -theta
            c, s_ = cs[..., 0].repeat(B, 1), cs[..., 1].repeat(B, 1)
            for i in (0, 1):
                x = ref[i].view(B * S, H, hd // 2, 2)
                a, b = x[..., 0], x[..., 1]
                ref_i = torch.stack([a * c[:, None] + b * s_[:, None], -a * s_[:, None] + b * c[:, None]], -1)
                assert rel_err(got[i], ref_i.reshape(B * S, D)) < 0.03
        else:
            for i in range(3):
                assert rel_err(got[i], ref[i]) < 0.03, ("qkv"[i], rel_err(got[i], ref[i]))


def test_embed_fwd_bwd():
    V, D, M = 500, 256, 1000
    W = torch.randn(V, D, device=DEV).to(torch.bfloat16)
    tok = torch.randint(0, V, (M,), device=DEV, dtype=torch.int32)
    x = torch.empty(M, D, device=DEV)
    ops.embed_fwd(tok, W, x)
    dx = torch.randn(M, D, device=DEV)
    dW = torch.zeros(V, D, device=DEV)
    ops.embed_bwd(tok, dx, dW)
    ref = torch.zeros(V, D, device=DEV).index_add_(0, tok.long(), dx)
    torch.cuda.synchronize()
    assert torch.equal(x, W.float()[tok.long()])
    assert rel_err(dW, ref) < 1e-5


@pytest.mark.parametrize("M,K,N", [(1, 2048, 768), (32, 2048, 768), (7, 688, 2048), (32, 2048, 1376), (32, 5504, 2048),
                                   (32, 104, 1000), (16, 2048, 32000), (2, 256, 512), (5, 1216, 512),
                                   (32, 1216, 512)])
@pytest.mark.parametrize("fp32", [False, True])
def test_skinny_linear_matches_fp32(M, K, N, fp32):
    """Decode-sized projections (<= 32 rows) on the tcgen05 skinny kernel against an fp32 matmul, including
    K and N tails and K split over clusters of 1 to 16 CTAs (with few rows, some CTAs of the cluster own
    no rows to store); repeated runs give the same bits (fixed-order cluster reduction)."""
    g = torch.Generator(device=DEV).manual_seed(M * 7 + K)
    x = torch.randn(M, K, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(K, N, device=DEV, generator=g) * K ** -0.5).to(torch.bfloat16)
    ref = x.float() @ w.float()
    ys = []
    for _ in range(3):
        y = torch.empty(M, N, device=DEV, dtype=torch.float32 if fp32 else torch.bfloat16)
        ops.ext().skinny_gemm(x, w, y)
        ys.append(y)
    ys.append(ops.linear(x, w, fp32=fp32))     # the routed path (skinny or, for the widest, the regular GEMM)
    torch.cuda.synchronize()
    for y in ys:
        assert y.dtype == (torch.float32 if fp32 else torch.bfloat16)
        assert rel_err(y, ref) < (1e-3 if fp32 else 1e-2)
    for y in ys[1:3]:
        assert torch.equal(y, ys[0])


@pytest.mark.parametrize("case", ["skinny_qkv", "decode_attn_b32", "gemm_swiglu", "moe_fwd"])
def test_profiling_cases_run(case):
    """The profiler-capture cases build and launch (what an ncu capture of them relies on)."""
    from predicitivecoding_b200.ops import kernel_cases
    fn, flops = kernel_cases.build(case)
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    assert flops > 0


@pytest.mark.parametrize("M,K,F", [(1, 2048, 2752), (32, 2048, 5504), (7, 512, 688), (64, 512, 688)])
def test_linear_swiglu_matches_fp32(M, K, F):
    """silu(x W_gate) * (x W_up) from the interleaved [K, 2F] weight: the skinny kernel's SwiGLU epilogue
    (<= 32 rows) and the GEMM + SwiGLU-pass fallback (64 rows) against fp32."""
    g = torch.Generator(device=DEV).manual_seed(M + K + F)
    x = torch.randn(M, K, device=DEV, generator=g).to(torch.bfloat16)
    wg = (torch.randn(K, F, device=DEV, generator=g) * K ** -0.5).to(torch.bfloat16)
    wu = (torch.randn(K, F, device=DEV, generator=g) * K ** -0.5).to(torch.bfloat16)
    ref = torch.nn.functional.silu(x.float() @ wg.float()) * (x.float() @ wu.float())
    a = ops.linear_swiglu(x, ops.interleave16(wg, wu))
    torch.cuda.synchronize()
    assert a.shape == (M, F) and a.dtype == torch.bfloat16
    assert rel_err(a, ref) < 2e-2


@pytest.mark.parametrize("B,H,hd", [(4, 4, 64), (32, 16, 128), (3, 2, 128)])
@pytest.mark.parametrize("fused", [True, False])
def test_qkv_rope_append_matches_fp32(B, H, hd, fused):
    """Decode qkv projection + RoPE at position pos + KV-cache append: the skinny kernel's RoPE epilogue and
    the GEMM + RoPE/append kernel against fp32 (adjacent-pair rotation), other cache rows untouched."""
    D, K, cap, p = H * hd, 256, 64, 37
    g = torch.Generator(device=DEV).manual_seed(B * H + hd)
    x = torch.randn(B, K, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(K, 3 * D, device=DEV, generator=g) * K ** -0.5).to(torch.bfloat16)
    ang = torch.arange(cap, device=DEV, dtype=torch.float32)[:, None] * \
        (10000.0 ** (-torch.arange(0, hd, 2, device=DEV, dtype=torch.float32) / hd))[None]
    cs = torch.stack((ang.cos(), ang.sin()), -1).contiguous()            # [cap, hd/2, 2]
    pos = torch.tensor(p, device=DEV, dtype=torch.int64)
    q = torch.zeros(B, H, hd, device=DEV, dtype=torch.bfloat16)
    kc = torch.full((B, H, cap, hd), 7.0, device=DEV, dtype=torch.bfloat16)
    vc = torch.full((B, H, cap, hd), 7.0, device=DEV, dtype=torch.bfloat16)
    keep = ops.FUSED_ROPE
    try:
        ops.FUSED_ROPE = fused
        ops.qkv_rope_append(x, w, cs, pos, q, kc, vc)
    finally:
        ops.FUSED_ROPE = keep
    torch.cuda.synchronize()
    y = x.float() @ w.float()
    c, s = cs[p, :, 0], cs[p, :, 1]

    def rot(t):                                                           # [B, H, hd]
        a, b = t[..., 0::2], t[..., 1::2]
        out = torch.empty_like(t)
        out[..., 0::2] = a * c - b * s
        out[..., 1::2] = a * s + b * c
        return out
    qr = rot(y[:, :D].view(B, H, hd))
    kr = rot(y[:, D:2 * D].view(B, H, hd))
    vr = y[:, 2 * D:].view(B, H, hd)
    assert rel_err(q, qr) < 1e-2
    assert rel_err(kc[:, :, p], kr) < 1e-2
    assert rel_err(vc[:, :, p], vr) < 1e-2
    others = torch.ones(cap, dtype=torch.bool)
    others[p] = False
    assert bool((kc[:, :, others] == 7.0).all()) and bool((vc[:, :, others] == 7.0).all())
