"""Data-parallel fused trainer on 2 GPUs (skipped with fewer devices).

Each rank trains on half of a global batch; the fused peer-memory path (bucketed
gradient pushes overlapped with the backward, then reduce + clip + AdamW + bf16
all-gather) and the NCCL ZeRO-1 baseline must both track a single-GPU trainer
that sees the whole batch, with global-norm clipping off and on.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cfg():
    from predicitivecoding_b200.models.config import DecoderLmConfig
    return DecoderLmConfig(vocab=512, dim=128, num_blocks=2, num_heads=2, ff_dim=256, max_seq=128,
                           use_rms_norm=True, use_rope=True, ffn="swiglu")


def _data(step):
    g = torch.Generator().manual_seed(1000 + step)
    t = torch.randint(0, 512, (4, 129), generator=g)
    return t[:, :-1].contiguous(), t[:, 1:].contiguous()


def _worker(rank, world, port, mode, clip, out_q):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    try:
        from predicitivecoding_b200.engine.fused_trainer import FusedDecoderTrainer
        from predicitivecoding_b200.models.decoder_lm import DecoderLM
        cfg = _cfg()
        tr = FusedDecoderTrainer(cfg, batch=2, model=DecoderLM(cfg, seed=7), device=dev, lr=1e-3, clip_norm=clip,
                                 process_group=dist.group.WORLD, grad_sync=mode, use_graph=(mode == "fused"))
        losses = []
        for s in range(4):
            tok, tgt = _data(s)
            half = slice(2 * rank, 2 * rank + 2)
            losses.append(tr.step(tok[half], tgt[half]))
        # mean loss over ranks = loss of the whole batch
        t = torch.tensor(losses, device=dev)
        dist.all_reduce(t)
        w = torch.cat([p.detach().reshape(-1) for p in tr.export_model().reference_parameters()])
        if rank == 0:
            out_q.put(((t / world).tolist(), w.cpu()))
        if tr.peer is not None:
            tr.peer.check()
        tr.graph = None
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _run(mode, clip):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, clip, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("clip", [0.0, 0.05])
@pytest.mark.parametrize("mode", ["fused", "zero"])
def test_dp_matches_single_gpu(mode, clip):
    """clip 0.05 is far below this model's gradient norm, so the clip scale is active on every step."""
    from predicitivecoding_b200.engine.fused_trainer import FusedDecoderTrainer
    from predicitivecoding_b200.models.decoder_lm import DecoderLM
    dp_losses, dp_w = _run(mode, clip)
    cfg = _cfg()
    single = FusedDecoderTrainer(cfg, batch=4, model=DecoderLM(cfg, seed=7), device="cuda:0", lr=1e-3,
                                 clip_norm=clip, use_graph=False)
    ref = [single.step(*_data(s)) for s in range(4)]
    for a, b in zip(dp_losses, ref):
        assert abs(a - b) / b < 5e-3, (dp_losses, ref)
    w = torch.cat([p.detach().reshape(-1) for p in single.export_model().reference_parameters()]).cpu()
    rel = float((dp_w - w).norm() / w.norm())
    assert rel < 2e-3, rel
