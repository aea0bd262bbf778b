"""Device mixture-of-experts FFN (routing, expert-sorted dispatch, grouped tcgen05 GEMMs, combine and
their backward) against an fp32 PyTorch statement of the same layer, and the fused trainer with experts
against the autograd DecoderLM (DecoderLM.cs:556-615)."""
import pytest
import torch

from predicitivecoding_b200 import ops
from predicitivecoding_b200.ops import moe
from predicitivecoding_b200.models.config import DecoderLmConfig
from predicitivecoding_b200.models.decoder_lm import DecoderLM
from predicitivecoding_b200.engine.fused_trainer import FusedDecoderTrainer

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel(a, b):
    a, b = a.detach().float(), b.detach().float()
    return float((a - b).norm() / (b.norm() + 1e-12))


def bf16_exact(t):
    return t.to(torch.bfloat16).float()


def layer(M=512, D=256, F_=512, E=4, k=2, seed=0, skew=None):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, D, generator=g)
    router = torch.randn(E, D, generator=g) * 0.05
    if skew is not None:       # a shared direction in every row that only the experts in `skew` like
        u = torch.randn(D, generator=g)
        u /= u.norm()
        x += 4.0 * u
        for e in range(E):
            router[e] += (3.0 if e in skew else -3.0) * u
    x, router = bf16_exact(x), bf16_exact(router)
    w1 = bf16_exact(torch.randn(E * F_, D, generator=g) * D ** -0.5)
    b1 = torch.randn(E * F_, generator=g) * 0.1
    w2 = bf16_exact(torch.randn(E * D, F_, generator=g) * F_ ** -0.5)
    b2 = torch.randn(E * D, generator=g) * 0.1
    return [t.to(DEV) for t in (x, router, w1, b1, w2, b2)]


def run_device(x, router, w1, b1, w2, b2, k, dx, weight):
    M, D = x.shape
    E, F_ = router.shape[0], w1.shape[0] // router.shape[0]
    buf = moe.MoEBuffers.allocate(M, D, F_, E, k, DEV)
    scr = moe.MoEScratch.allocate(M, D, F_, E, k, DEV)
    res = torch.randn(M, D, device=DEV)
    out = torch.empty(M, D, device=DEV)
    loss = torch.zeros(1, device=DEV)
    bf = lambda t: t.to(torch.bfloat16).contiguous()
    moe.forward(bf(x), res, out, bf(router), bf(w1), b1, bf(w2), b2, k, buf, loss, weight)
    dn = torch.empty(M, D, device=DEV)
    grads = [torch.zeros_like(t) for t in (router, w1, b1, w2, b2)]
    moe.backward(dx, bf(x), dn, bf(router), bf(w1), bf(w2), k, buf, scr, *grads[:3], grads[3], grads[4], weight)
    torch.cuda.synchronize()
    return buf, res, out, float(loss), dn, grads


@pytest.mark.parametrize("skew", [None, (0, 1)])
def test_moe_layer_matches_fp32_reference(skew):
    k, weight = 2, 0.01
    x, router, w1, b1, w2, b2 = layer(skew=skew)
    M, D = x.shape
    dx = torch.randn(M, D, device=DEV)
    buf, res, out, loss, dn, grads = run_device(x, router, w1, b1, w2, b2, k, dx, weight)
    # the reference uses the device's routing so near-ties cannot split the two
    leaves = [t.clone().requires_grad_(True) for t in (x, router, w1, b1, w2, b2)]
    y, bal, _ = moe.reference(*leaves, k, topi=buf.topi)
    assert rel(out - res, y) < 2e-2
    assert abs(loss - weight * float(bal)) < 1e-4 * max(1.0, abs(loss))
    ((y * dx).sum() + weight * bal).backward()
    assert rel(dn, leaves[0].grad) < 3e-2
    for name, got, leaf in zip(("router", "w1", "b1", "w2", "b2"), grads, leaves[1:]):
        assert rel(got, leaf.grad) < 3e-2, name
    if skew is not None:
        counts = torch.bincount(buf.topi.view(-1).long(), minlength=4)
        assert int(counts[2]) == 0 and int(counts[3]) == 0   # empty experts exercised


def test_dispatch_is_a_stable_padded_sort():
    k, E = 2, 4
    x, router, w1, b1, w2, b2 = layer(M=1000 // 8 * 8, E=E)
    M = x.shape[0]
    buf = moe.MoEBuffers.allocate(M, x.shape[1], w1.shape[0] // E, E, k, DEV)
    ops.ext().moe_route(x.to(torch.bfloat16), router.to(torch.bfloat16), k, buf.gates, buf.topi)
    ops.ext().moe_dispatch(buf.topi, buf.gates, k, buf.seg, buf.pos, buf.src, buf.rgate, buf.coef, None, 0.0)
    torch.cuda.synchronize()
    gates_ref = torch.softmax(x.to(torch.bfloat16).float() @ router.to(torch.bfloat16).float().T, -1)
    assert rel(buf.gates, gates_ref) < 1e-3
    topi = buf.topi.view(-1).long().cpu()
    seg = buf.seg.cpu().tolist()
    counts = torch.bincount(topi, minlength=E).tolist()
    for e in range(E):
        assert seg[e] % 256 == 0
        assert seg[e + 1] - seg[e] == (counts[e] + 255) // 256 * 256
    pos = buf.pos.view(-1).cpu()
    src = buf.src.cpu()
    for e in range(E):
        idx = torch.nonzero(topi == e).flatten()         # assignment order
        p = pos[idx]
        assert torch.equal(p, torch.arange(seg[e], seg[e] + counts[e]))   # stable, contiguous
        assert torch.equal(src[p], idx // k)
        assert bool((src[seg[e] + counts[e]:seg[e + 1]] == -1).all())


def moe_model_cfg():
    return DecoderLmConfig(vocab=512, dim=256, num_blocks=2, num_heads=4, ff_dim=512, max_seq=128,
                           use_rms_norm=True, use_rope=True, num_experts=4, moe_top_k=2, moe_balance_weight=0.01)


def test_fused_trainer_with_experts_matches_autograd(monkeypatch):
    cfg = moe_model_cfg()
    model = DecoderLM(cfg, seed=11)
    with torch.no_grad():
        for blk in model.blocks:
            for e in range(cfg.num_experts):
                blk.eb1[e].normal_(0, 0.05)
                blk.eb2[e].normal_(0, 0.05)
    tr = FusedDecoderTrainer(cfg, batch=2, model=model, use_graph=False)
    gen = torch.Generator().manual_seed(0)
    t = torch.randint(0, cfg.vocab, (2, cfg.max_seq + 1), generator=gen)
    tok, tgt = t[:, :-1].contiguous(), t[:, 1:].contiguous()
    tr.stage(tok, tgt)
    tr.tok.copy_(tr.tok_pin)
    tr.tgt.copy_(tr.tgt_pin)
    tr.grad.zero_()
    tr._forward(True)
    tr._backward()
    torch.cuda.synchronize()
    loss_dev = float(tr.loss_sum) / tr.M
    ref = model.to(DEV)
    # the autograd model routes with the device's top-k choices: bf16 and fp32 logits may order a near-tie
    # differently, and one re-routed row moves the router gradient by a few percent
    device_topi = iter([tr.moe[l].topi.long() for l in range(cfg.num_blocks)])

    def topk_as_device(x, k, *args, **kwargs):
        idx = next(device_topi)
        return torch.return_types.topk((x.gather(-1, idx), idx))

    monkeypatch.setattr(torch, "topk", topk_as_device)
    loss = ref.loss(tok.to(DEV), tgt.to(DEV))
    monkeypatch.undo()
    loss.backward()
    assert abs(loss_dev - float(loss)) / float(loss) < 5e-3
    G = tr.G
    E, D, F_ = cfg.num_experts, cfg.dim, cfg.ff_dim
    for l, blk in enumerate(ref.blocks):
        assert rel(G[f"b{l}.router"], blk.router.grad.T) < 0.06
        w1 = torch.cat([blk.ew1[e].grad.T for e in range(E)], 0)
        w2 = torch.cat([blk.ew2[e].grad.T for e in range(E)], 0)
        assert rel(G[f"b{l}.ew1"], w1) < 0.05
        assert rel(G[f"b{l}.ew2"], w2) < 0.05
        assert rel(G[f"b{l}.eb1"], torch.cat([blk.eb1[e].grad for e in range(E)])) < 0.05
        assert rel(G[f"b{l}.eb2"], torch.cat([blk.eb2[e].grad for e in range(E)])) < 0.05
        assert rel(G[f"b{l}.ln2"], blk.ln2_g.grad) < 0.05
    assert rel(G["wemb"], ref.wemb.grad) < 0.05


def test_fused_trainer_with_experts_trains_in_a_graph():
    cfg = moe_model_cfg()
    tr = FusedDecoderTrainer(cfg, batch=2, seed=2, use_graph=True, lr=1e-3)
    gen = torch.Generator().manual_seed(1)
    t = torch.randint(0, 64, (2, cfg.max_seq + 1), generator=gen)   # a small alphabet: learnable
    tok, tgt = t[:, :-1].contiguous(), t[:, 1:].contiguous()
    losses = [tr.step(tok, tgt) for _ in range(12)]
    assert all(l == l for l in losses)
    assert losses[-1] < losses[0]
    # export round trip keeps the experts
    m = tr.export_model()
    assert len(m.blocks[0].ew1) == cfg.num_experts
