"""Weight-gradient GEMMs on a second stream give the same step as one stream.

The fused trainer forks every dW GEMM of a SwiGLU block onto a side stream and double-buffers the bf16
gradient inputs those GEMMs read (PCB_WGRAD_STREAM, on by default).  Both schedules accumulate the same
products into the fp32 gradient arena, so after a step the gradients agree up to the summation order of
the split-K fp32 atomics: the first step's gradients (same weights) agree to fp32 rounding.  Later
steps start from weights that already differ by that rounding, which AdamW's normalised update
magnifies for near-zero gradient entries, so from then on the losses are compared and the gradients
only loosely.  Run eagerly and as a captured CUDA graph, over three steps so the double buffers are
reused across steps.
"""
import pytest
import torch

from predicitivecoding_b200.engine.fused_trainer import FusedDecoderTrainer
from predicitivecoding_b200.models.config import DecoderLmConfig
from predicitivecoding_b200.models.decoder_lm import DecoderLM

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.double() - b.double()).norm() / (b.double().norm() + 1e-30))


@pytest.mark.parametrize("use_graph", [False, True])
def test_two_stream_backward_matches_one_stream(monkeypatch, use_graph):
    cfg = DecoderLmConfig(vocab=1024, dim=256, num_blocks=3, num_heads=4, ff_dim=512, max_seq=256,
                          use_rms_norm=True, use_rope=True, ffn="swiglu")
    B = 4
    g = torch.Generator().manual_seed(7)
    data = [torch.randint(0, cfg.vocab, (B, cfg.max_seq + 1), generator=g) for _ in range(3)]
    out = {}
    for ws in ("1", "0"):
        monkeypatch.setenv("PCB_WGRAD_STREAM", ws)
        tr = FusedDecoderTrainer(cfg, batch=B, model=DecoderLM(cfg, seed=5), device="cuda:0", lr=1e-3,
                                 weight_decay=0.1, clip_norm=1.0, use_graph=use_graph)
        assert (tr._wg_stream is not None) == (ws == "1")
        losses, g_first = [], None
        for t in data:
            losses.append(tr.step(t[:, :-1], t[:, 1:]))
            if g_first is None:
                g_first = tr.grad.clone()
        torch.cuda.synchronize()
        out[ws] = (losses, g_first, tr.grad.clone())
        del tr
    (l1, f1, g1), (l0, f0, g0) = out["1"], out["0"]
    assert l1[0] == pytest.approx(l0[0], rel=1e-6)          # same forward, same weights
    assert torch.isfinite(f1).all() and f1.abs().max() > 0
    assert _rel(f1, f0) < 1e-4, _rel(f1, f0)                # same weights: summation order only
    for a, b in zip(l1[1:], l0[1:]):
        assert a == pytest.approx(b, rel=1e-3)
    assert _rel(g1, g0) < 5e-2, _rel(g1, g0)
