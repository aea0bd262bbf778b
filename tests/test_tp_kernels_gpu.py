"""Tensor-parallel GEMM fusions on one GPU: the in-kernel all-gather of A and the reduce-scatter
epilogue, with the 'peers' emulated by separate buffers on the same device (one kernel launch, so
no cross-launch waiting), against fp32 PyTorch references."""
import pytest
import torch

from predicitivecoding_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world,rank,N", [(2, 0, 256), (4, 1, 384), (4, 3, 1024)])
def test_fused_allgather_gemm(world, rank, N):
    rows, K = 256, 512
    g = torch.Generator(device="cuda").manual_seed(world * 10 + rank)
    X = torch.randn(world * rows, K, device="cuda", generator=g).to(torch.bfloat16)
    W = (torch.randn(N, K, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    local = torch.zeros_like(X)
    local[rank * rows:(rank + 1) * rows] = X[rank * rows:(rank + 1) * rows]
    peers = []
    for c in range(world):
        if c == rank:
            peers.append(local)
        else:
            p = torch.zeros_like(X)
            p[c * rows:(c + 1) * rows] = X[c * rows:(c + 1) * rows]
            peers.append(p)
    table = torch.tensor([p.data_ptr() for p in peers], dtype=torch.int64, device="cuda")
    ready = torch.zeros(world, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = ops.gemm(local, W, epi=ops.EPI_F32, err=err,
                   tp=(table.data_ptr(), ready.data_ptr(), rows, rank, world, 0, 0, 0))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(local, X)                      # the gathered buffer now holds every chunk
    ref = X.float() @ W.float().T
    assert (out - ref).abs().max() < 2e-2 * ref.abs().max()
    assert int(ready.sum()) > 0


@pytest.mark.parametrize("world", [2, 4])
def test_reduce_scatter_epilogue_and_owner_reduce(world):
    rows, K, N = 256, 256, 512
    g = torch.Generator(device="cuda").manual_seed(world)
    slots = [torch.zeros(world * rows, N, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
    table = torch.tensor([s.data_ptr() for s in slots], dtype=torch.int64, device="cuda")
    parts = []
    for src in range(world):                          # every "rank" writes its partial product
        A = torch.randn(world * rows, K, device="cuda", generator=g).to(torch.bfloat16)
        B = (torch.randn(N, K, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
        ops.gemm(A, B, epi=ops.EPI_RS_BF16, tp=(0, 0, 0, 0, 0, table.data_ptr(), rows, src))
        parts.append(A.float() @ B.float().T)
    torch.cuda.synchronize()
    for owner in range(world):
        for src in range(world):
            got = slots[owner][src * rows:(src + 1) * rows].float()
            ref = parts[src][owner * rows:(owner + 1) * rows]
            assert (got - ref).abs().max() < 2e-2 * ref.abs().max() + 1e-3
    # owner-side reduction + residual + RMSNorm into a gather buffer
    owner = world - 1
    resid = torch.randn(rows, N, device="cuda")
    x = torch.empty(rows, N, device="cuda")
    gamma = (1 + 0.1 * torch.randn(N, device="cuda")).to(torch.bfloat16)
    y = torch.empty(rows, N, device="cuda", dtype=torch.bfloat16)
    inv = torch.empty(rows, device="cuda")
    ops.ext().tp_reduce_norm(slots[owner], world, resid, x, False, gamma, y, inv, 1e-5)
    ref_x = resid + sum(slots[owner][s * rows:(s + 1) * rows].float() for s in range(world))
    assert (x - ref_x).abs().max() < 1e-4
    ref_inv = torch.rsqrt((ref_x * ref_x).mean(1) + 1e-5)
    ref_y = ref_x * ref_inv[:, None] * gamma.float()
    assert (inv - ref_inv).abs().max() < 1e-5 * ref_inv.abs().max() + 1e-6
    assert (y.float() - ref_y).abs().max() < 1e-2 * ref_y.abs().max()
    # plain reduction with accumulate
    acc = torch.ones(rows, N, device="cuda")
    ops.ext().tp_reduce_norm(slots[owner], world, None, acc, True, None, None, None, 1e-5)
    assert (acc - (1 + ref_x - resid)).abs().max() < 1e-4
