"""Serving / small-op kernels against plain fp32 PyTorch references."""
import math

import pytest
import torch

from predicitivecoding_b200 import ops

pytestmark = pytest.mark.gpu


def _ref_decode(q, k, v, lens, scale, softcap):
    B, H, hd = q.shape
    Hkv = k.shape[1]
    G = H // Hkv
    out = torch.zeros(B, H, hd)
    for b in range(B):
        n = int(lens[b])
        if n == 0:
            continue
        kk = k[b, :, :n].float().repeat_interleave(G, 0)      # [H, n, hd]
        vv = v[b, :, :n].float().repeat_interleave(G, 0)
        s = torch.einsum("hd,hnd->hn", q[b].float(), kk) * scale
        if softcap > 0:
            s = softcap * torch.tanh(s / softcap)
        out[b] = torch.einsum("hn,hnd->hd", torch.softmax(s, -1), vv)
    return out


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("G", [1, 2, 4, 8])
def test_decode_attention(hd, G):
    g = torch.Generator(device="cuda").manual_seed(hd + G)
    B, Hkv, cap = 3, 2, 700
    H = Hkv * G
    q = torch.randn(B, H, hd, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, cap, hd, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, cap, hd, device="cuda", generator=g).to(torch.bfloat16)
    lens = torch.tensor([1, 333, 700], dtype=torch.int32, device="cuda")
    for softcap in (0.0, 5.0):
        for nsplit in (1, 3, 8, None):
            out = ops.decode_attn(q, k, v, lens, 1 / math.sqrt(hd), softcap, nsplit=nsplit)
            ref = _ref_decode(q.cpu(), k.cpu(), v.cpu(), lens.cpu(), 1 / math.sqrt(hd), softcap)
            assert (out.float().cpu() - ref).abs().max() < 2e-2


def test_decode_attention_empty_sequence():
    q = torch.randn(2, 4, 64, device="cuda").to(torch.bfloat16)
    k = torch.randn(2, 4, 64, 64, device="cuda").to(torch.bfloat16)
    lens = torch.tensor([0, 5], dtype=torch.int32, device="cuda")
    out = ops.decode_attn(q, k, k, lens, 0.125)
    assert float(out[0].float().abs().max()) == 0.0 and torch.isfinite(out.float()).all()


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("nb", [1, 3, 8, 11])
def test_weight_only_gemv(bits, nb):
    from predicitivecoding_b200.llm.quant import Int4Matrix, Int8Matrix
    g = torch.Generator().manual_seed(bits * 100 + nb)
    w = torch.randn(333, 512, generator=g)
    x = torch.randn(nb, 512, generator=g)
    m = Int8Matrix(w) if bits == 8 else Int4Matrix(w)
    ref = x @ m.to_float().T
    mq = m.q.cuda() if bits == 8 else m.packed.cuda()
    y = ops.wq_matmul(x.cuda(), mq, m.scale.cuda(), bits)
    assert (y.cpu() - ref).abs().max() < 1e-3 * ref.abs().max() + 1e-4


def test_quant_matrices_use_the_kernel_on_gpu():
    from predicitivecoding_b200.llm.quant import Int8Matrix
    m = Int8Matrix(torch.randn(64, 128).cuda())
    before = ops.launch_count()
    y = m.matvec(torch.randn(2, 128, device="cuda"))
    assert ops.launch_count() == before + 1 and y.shape == (2, 64)


def test_softmax_rows_fwd_bwd():
    x = torch.randn(37, 1000, device="cuda")
    x[0, :500] = float("-inf")
    y = ops.softmax_rows(x, 0.5)
    ref = torch.softmax(x.cpu() * 0.5, -1)
    assert (y.cpu() - ref).abs().max() < 1e-6
    dy = torch.randn_like(x)
    dx = ops.softmax_rows_bwd(y, dy, 0.5)
    xr = (x.cpu() * 1.0).requires_grad_()
    torch.softmax(xr * 0.5, -1).backward(dy.cpu())
    assert (dx.cpu() - xr.grad).abs().max() < 1e-5


def test_linear_scan_fwd_bwd_matches_loop():
    from predicitivecoding_b200.models.decoder_lm import recurrent_scan
    a = torch.rand(3, 50, 96).requires_grad_()
    b = torch.randn(3, 50, 96).requires_grad_()
    s_ref = recurrent_scan(a, b)
    gs = torch.randn_like(s_ref)
    s_ref.backward(gs)
    ac, bc = a.detach().cuda().requires_grad_(), b.detach().cuda().requires_grad_()
    s = recurrent_scan(ac, bc)
    s.backward(gs.cuda())
    assert (s.detach().cpu() - s_ref.detach()).abs().max() < 1e-5
    assert (ac.grad.cpu() - a.grad).abs().max() < 1e-4 and (bc.grad.cpu() - b.grad).abs().max() < 1e-4


def test_serving_decode_kernel_matches_sdpa_path():
    from predicitivecoding_b200.llm.serving import export
    from predicitivecoding_b200.models.config import DecoderLmConfig
    from predicitivecoding_b200.models.decoder_lm import DecoderLM
    cfg = DecoderLmConfig(256, 256, 2, 4, 512, 128, use_rms_norm=True, use_rope=True, ffn="swiglu")
    m = DecoderLM(cfg, seed=5).eval()
    inf = export(m, "cuda", torch.bfloat16)
    assert inf._fast_decode
    toks = torch.tensor([[1, 2, 3, 4, 5], [7, 8, 9, 10, 11]], device="cuda")
    logits = {}
    for fast in (True, False):
        inf._fast_decode = fast
        c = inf.new_cache(2)
        inf.prefill(toks, c)
        before = ops.launch_count()
        outs = [inf.step(toks[:, i % 5], c) for i in range(6)]
        if fast:
            assert ops.launch_count() >= before + 6 * cfg.num_blocks * 2
        logits[fast] = torch.stack(outs)
    assert (logits[True] - logits[False]).abs().max() < 5e-2 * logits[False].abs().max()


def test_serving_swiglu_projection_matches_autograd_model():
    """The exported bf16 model (w1/w3 interleaved for the fused SwiGLU projection) against the fp32 autograd
    model: prefill logits of a prompt and the logits of decode steps."""
    from predicitivecoding_b200.llm.serving import export
    from predicitivecoding_b200.models.config import DecoderLmConfig
    from predicitivecoding_b200.models.decoder_lm import DecoderLM
    cfg = DecoderLmConfig(256, 256, 2, 4, 512, 128, use_rms_norm=True, use_rope=True, ffn="swiglu")
    m = DecoderLM(cfg, seed=6).eval()
    inf = export(m, "cuda", torch.bfloat16)
    assert all("w13" in blk for blk in inf.blocks)
    toks = torch.randint(0, 256, (2, 9), generator=torch.Generator().manual_seed(3))
    with torch.no_grad():
        ref = m(toks).float()                                   # [2, 9, V] fp32 on the CPU
    c = inf.new_cache(2)
    pre = inf.prefill(toks[:, :5].cuda(), c).float().cpu()
    steps = [inf.step(toks[:, i].cuda(), c).float().cpu() for i in range(5, 9)]
    got = torch.cat([pre, torch.stack(steps, 1)], 1)
    err = float((got - ref).norm() / ref.norm())
    assert err < 3e-2, err
