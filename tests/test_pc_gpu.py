"""Fused batched PC engine (PC GEMM epilogues) against the fp32 PyTorch oracle.

Tolerances follow the reference's mixed-precision twin test (batched mixed within
5e-2 of fp32, TEST/PredicitiveCoding.UnitTests/BatchedPcForwardTests.cs:45-111): the
fused engine keeps fp32 states and weights but multiplies bf16 operands.
"""
import pytest
import torch

from predicitivecoding_b200.pc.batched import BatchedPC, BatchedPCReference

pytestmark = pytest.mark.gpu


def rel(a, b):
    return float((a.float().cpu() - b.float().cpu()).norm() / (b.float().cpu().norm() + 1e-12))


@pytest.mark.parametrize("act", ["tanh", "sigmoid", "linear"])
@pytest.mark.parametrize("ffg", [False, True])
def test_infer_get_top_matches_reference(act, ffg):
    sizes = [256, 384, 128, 64]
    ref = BatchedPCReference(sizes, act, 0.1, activity_reg=0.001, ffg=ffg, seed=3, precisions=[1.0, 1.5, 1.0, 1.0])
    eng = BatchedPC(sizes, 256, act, 0.1, activity_reg=0.001, ffg=ffg, weights=ref.W, biases=ref.b,
                    precisions=[1.0, 1.5, 1.0, 1.0])
    X = torch.randn(256, 256, generator=torch.Generator().manual_seed(0))
    top_ref = ref.infer_get_top(X, 15)
    top = eng.infer_get_top(X.cuda(), 15)
    torch.cuda.synchronize()
    assert rel(top, top_ref) < 5e-2


def test_learn_matches_reference_weights_and_energy():
    sizes = [256, 512, 512, 128]
    ref = BatchedPCReference(sizes, "tanh", 0.1, weight_lr=0.05, weight_decay=0.01, seed=4)
    eng = BatchedPC(sizes, 512, "tanh", 0.1, weight_lr=0.05, weight_decay=0.01, weights=ref.W, biases=ref.b)
    g = torch.Generator().manual_seed(1)
    for _ in range(3):
        X = torch.randn(512, 256, generator=g)
        Y = torch.randn(512, 128, generator=g)
        e_ref = ref.learn(X, Y, 12)
        eng.learn(X.cuda(), Y.cuda(), 12)
        torch.cuda.synchronize()
        assert abs(eng.energy_value() - e_ref) / e_ref < 5e-2
    W, b = eng.weights()
    W0 = BatchedPCReference(sizes, "tanh", seed=4).W
    for l in range(3):
        # compare the weight *changes* (the update is small relative to W)
        assert rel(W[l] - W0[l], ref.W[l] - W0[l]) < 5e-2
        assert rel(b[l], ref.b[l]) < 5e-2


def test_graph_replay_equals_eager():
    sizes = [128, 256, 64]
    a = BatchedPC(sizes, 128, "tanh", 0.1, weight_lr=0.01, seed=5)
    b = BatchedPC(sizes, 128, "tanh", 0.1, weight_lr=0.01, seed=5)
    X = torch.randn(128, 128, device="cuda")
    Y = torch.randn(128, 64, device="cuda")
    b.capture(8)                         # runs one learn on zeros during capture warm-up
    a.learn(torch.zeros_like(X), torch.zeros_like(Y), 8)
    a.learn(X, Y, 8)
    b.replay(X, Y)
    torch.cuda.synchronize()
    for wa, wb in zip(a.W32, b.W32):
        assert rel(wb, wa) < 1e-5
