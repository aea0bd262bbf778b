"""Tensor-parallel trainer: T=1 on one GPU and T=2 on two GPUs track the single-GPU fused trainer."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _cfg():
    from predicitivecoding_b200.models.config import DecoderLmConfig
    return DecoderLmConfig(vocab=512, dim=256, num_blocks=2, num_heads=4, ff_dim=512, max_seq=256,
                           use_rms_norm=True, use_rope=True, ffn="swiglu")


def _data(step):
    g = torch.Generator().manual_seed(500 + step)
    t = torch.randint(0, 512, (2, 257), generator=g)
    return t[:, :-1].contiguous(), t[:, 1:].contiguous()


def _close(a, b):
    # Adam moves every weight by up to lr per step; entries whose gradient is ~0 may flip sign between
    # summation orders, so bound the mean tightly and the max by 2 * lr * steps
    d = (a - b).abs()
    assert d.mean() < 1e-4 and d.max() < 6e-3, (float(d.mean()), float(d.max()))


def _reference(steps=3):
    from predicitivecoding_b200.engine.fused_trainer import FusedDecoderTrainer
    from predicitivecoding_b200.models.decoder_lm import DecoderLM
    cfg = _cfg()
    tr = FusedDecoderTrainer(cfg, batch=2, model=DecoderLM(cfg, seed=11), device="cuda:0", lr=1e-3, use_graph=False)
    losses = [tr.step(*_data(s)) for s in range(steps)]
    return losses, tr.export_model()


def test_tp_trainer_single_rank_matches_fused_trainer():
    from predicitivecoding_b200.engine.tp_trainer import TensorParallelTrainer
    from predicitivecoding_b200.models.decoder_lm import DecoderLM
    cfg = _cfg()
    ref_losses, ref_model = _reference()
    tp = TensorParallelTrainer(cfg, batch=2, model=DecoderLM(cfg, seed=11), device="cuda:0", lr=1e-3, use_graph=True)
    losses = [tp.step(*_data(s)) for s in range(3)]
    tp.check()
    for a, b in zip(losses, ref_losses):
        assert abs(a - b) < 2e-3 * abs(b)
    w = tp.local_weights()
    _close(w["b1.wqkv"][:256].cpu(), ref_model.blocks[1].wq.detach().T)
    _close(w["wemb"].cpu(), ref_model.wemb.detach())
    assert tp.launches_per_step is not None and tp.launches_per_step > 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    tp = None
    try:
        from predicitivecoding_b200.engine.tp_trainer import TensorParallelTrainer
        from predicitivecoding_b200.models.decoder_lm import DecoderLM
        cfg = _cfg()
        tp = TensorParallelTrainer(cfg, batch=2, model=DecoderLM(cfg, seed=11), device=dev, lr=1e-3,
                                   process_group=dist.group.WORLD, use_graph=True)
        losses = [tp.step(*_data(s)) for s in range(3)]
        tp.check()
        w = {k: v.detach().cpu() for k, v in tp.local_weights().items() if k in ("b1.wqkv", "b0.wo", "wemb", "b1.w2")}
        q.put((rank, losses, w))
    finally:
        if tp is not None:
            tp.release()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_matches_single_gpu():
    ref_losses, ref = _reference()
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, losses, w = q.get(timeout=600)
        res[r] = (losses, w)
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    for r in range(world):
        for a, b in zip(res[r][0], ref_losses):
            assert abs(a - b) < 3e-3 * abs(b)
    Dl = 128
    for r in range(world):
        w = res[r][1]
        q_ref = ref.blocks[1].wq.detach().T[r * Dl:(r + 1) * Dl]
        _close(w["b1.wqkv"][:Dl], q_ref)
        _close(w["b0.wo"], ref.blocks[0].wo.detach().T[:, r * Dl:(r + 1) * Dl])
        _close(w["b1.w2"][:, :256], ref.blocks[1].w2.detach().T[:, r * 256:(r + 1) * 256])
        _close(w["wemb"], ref.wemb.detach())


def _dp_worker(rank, world, port, q):
    """TP=1 x DP=2: each rank trains on its half of the batch; gradients are averaged over the replicas."""
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    tp = None
    try:
        from predicitivecoding_b200.engine.tp_trainer import TensorParallelTrainer
        from predicitivecoding_b200.models.decoder_lm import DecoderLM
        cfg = _cfg()
        singles = [dist.new_group([r]) for r in range(world)]
        tp = TensorParallelTrainer(cfg, batch=1, model=DecoderLM(cfg, seed=11), device=dev, lr=1e-3,
                                   process_group=singles[rank], dp_group=dist.group.WORLD, use_graph=True)
        losses = []
        for s in range(3):
            tok, tgt = _data(s)
            losses.append(tp.step(tok[rank:rank + 1], tgt[rank:rank + 1]))
        tp.check()
        w = {k: v.detach().cpu() for k, v in tp.local_weights().items() if k in ("b1.wqkv", "wemb", "b1.w2")}
        q.put((rank, losses, w))
    finally:
        if tp is not None:
            tp.release()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp1_dp2_matches_single_gpu():
    ref_losses, ref = _reference()
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_dp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, losses, w = q.get(timeout=600)
        res[r] = (losses, w)
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    for r in range(world):
        for a, b in zip(res[r][0], ref_losses):
            assert abs(a - b) < 3e-3 * abs(b)
        w = res[r][1]
        _close(w["b1.wqkv"][:256], ref.blocks[1].wq.detach().T)
        _close(w["wemb"], ref.wemb.detach())
    assert torch.equal(res[0][1]["b1.w2"], res[1][1]["b1.w2"])   # replicas stay identical
