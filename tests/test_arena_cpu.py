"""Bucketed parameter arena and the data-parallel push plan, emulated on the CPU.

Every rank owns an equal piece of every gradient bucket.  Applying each rank's
push plan (the copies its copy engines issue during the backward) and then the
owner's reduction (own gradient + staged slots) must give, for every rank, the sum
over ranks of the gradient on exactly the elements it owns.
"""
import torch

from predicitivecoding_b200.engine.arena import ParamArena, ParamSpec
from predicitivecoding_b200.engine.fused_trainer import FusedDecoderTrainer


def _specs():
    return [ParamSpec("emb", (50, 8)), ParamSpec("w0", (24, 8)), ParamSpec("g0", (8,), False),
            ParamSpec("w1", (24, 8)), ParamSpec("g1", (8,), False), ParamSpec("head", (50, 8))]


def test_bucketed_layout_pieces_and_decay_ends():
    A = ParamArena(_specs(), 4, buckets=[["head"], ["w1", "g1"], ["w0", "g0"], ["emb"]])
    assert A.total == 4 * A.shard and all((e - s) % (4 * 64) == 0 for s, e, _ in A.buckets)
    for (s, e, d), name in zip(A.buckets, ["head", "w1", "w0", "emb"]):
        assert s <= A.offsets[name] < d <= e          # decayed tensors first in each bucket
    loc = [p[0] for p in A.pieces(2)]
    assert loc == sorted(loc) and sum(p[2] for p in A.pieces(2)) == A.shard
    flat = torch.arange(A.total, dtype=torch.float32)
    for r in range(4):
        local = A.gather_local(flat, r)
        back = torch.full((A.total,), -1.0)
        A.scatter_local(local, r, back)
        mask = back >= 0
        assert torch.equal(back[mask], flat[mask]) and int(mask.sum()) == A.shard


def test_push_plan_then_owner_reduce_is_a_reduce_scatter():
    world = 4
    A = ParamArena(_specs(), world, buckets=[["head"], ["w1", "g1"], ["w0", "g0"], ["emb"]])
    g = torch.Generator().manual_seed(0)
    grads = [torch.randn(A.total, generator=g) for _ in range(world)]
    staging = [torch.zeros(world * A.shard) for _ in range(world)]
    for r in range(world):
        for b in range(len(A.buckets)):
            for q, dst, src, n in FusedDecoderTrainer.push_plan(A, r, b):
                staging[q][dst:dst + n] = grads[r][src:src + n]
    total = sum(grads)
    for r in range(world):
        own = A.gather_local(grads[r], r)
        red = own + sum(staging[r][p * A.shard:(p + 1) * A.shard] for p in range(world) if p != r)
        assert torch.allclose(red, A.gather_local(total, r), atol=1e-5)
