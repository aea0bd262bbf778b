"""PC data parallel on 2 GPUs (skipped with fewer devices): two ranks with half the batch each, their
Hebbian deltas all-reduced and applied by the fused peer-memory kernel, must give the weights of one
GPU learning on the whole batch (bf16 operands, fp32 weights)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SIZES = [256, 512, 256, 128]
B = 256


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _data(step):
    g = torch.Generator().manual_seed(100 + step)
    return torch.randn(B, SIZES[0], generator=g), torch.randn(B, SIZES[-1], generator=g)


def _init():
    from predicitivecoding_b200.pc.batched import BatchedPCReference
    ref = BatchedPCReference(SIZES, "tanh", 0.1, weight_lr=0.05, weight_decay=0.01, seed=9)
    return ref.W, ref.b


def _worker(rank, world, port, out_q):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    try:
        from predicitivecoding_b200.pc.batched import BatchedPC
        W, b = _init()
        eng = BatchedPC(SIZES, B // world, "tanh", 0.1, weight_lr=0.05, weight_decay=0.01, weights=W, biases=b,
                        device=dev, process_group=dist.group.WORLD)
        half = slice(rank * B // world, (rank + 1) * B // world)
        for s in range(3):
            x, y = _data(s)
            eng.learn(x[half].to(dev), y[half].to(dev), 10)
        torch.cuda.synchronize()
        eng.peer.check()
        if rank == 0:
            out_q.put(eng.weights())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_pc_data_parallel_matches_single_gpu_after_three_learn_steps():
    from predicitivecoding_b200.pc.batched import BatchedPC
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    dp_w, dp_b = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    W, b = _init()
    single = BatchedPC(SIZES, B, "tanh", 0.1, weight_lr=0.05, weight_decay=0.01, weights=W, biases=b)
    for s in range(3):
        x, y = _data(s)
        single.learn(x.cuda(), y.cuda(), 10)
    torch.cuda.synchronize()
    sw, sb = single.weights()
    for a, r in zip(dp_w + dp_b, sw + sb):
        d = float((a - r).norm() / (r.norm() + 1e-12))
        assert d < 1e-2, d
    # and the update did move the weights
    assert float((sw[0] - W[0].float()).norm()) > 0
