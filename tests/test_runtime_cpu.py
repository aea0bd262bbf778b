"""Device runtime and collectives on the CPU (host semantics and gloo ranks)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from predicitivecoding_b200.parallel.collectives import Communicator, HostCollectives, ReduceOp
from predicitivecoding_b200.runtime import Device, DeviceKind, DeviceRegistry, DeviceRuntime, DeviceTensor, TensorOps


def test_device_resolution_without_gpu():
    if DeviceRuntime.cuda_available():
        pytest.skip("host has a GPU")
    assert DeviceRuntime.resolve(Device.cuda(0)).is_cpu
    assert DeviceRuntime.resolve(Device.cuda_multi()).is_cpu
    assert DeviceRuntime.resolve(Device.rocm(0)).is_cpu and DeviceRuntime.resolve(Device.metal(0)).is_cpu
    assert str(Device.cuda(3)) == "cuda:3" and str(Device.cpu()) == "cpu"
    assert Device.cuda_multi().is_cuda and Device.rocm().is_gpu and not Device.cpu().is_gpu
    assert DeviceRegistry.auto_select().is_cpu and not DeviceRegistry.enable_rocm()


def test_device_tensor_and_ops_on_cpu():
    a = DeviceTensor.from_host(torch.arange(6.0).view(2, 3))
    b = DeviceTensor.from_host(torch.ones(3, 2))
    c = TensorOps.matmul(a, b)
    assert torch.equal(c.to_host(), torch.tensor([[3.0, 3.0], [12.0, 12.0]]))
    assert a.size_in_bytes == 24 and a.element_count == 6 and not a.is_on_device
    s = TensorOps.softmax_rows(a)
    assert torch.allclose(s.to_host().sum(1), torch.ones(2))
    with pytest.raises(ValueError):
        TensorOps.matmul(a, a)


def _ranks():
    return [torch.tensor([1.0, 2.0, 3.0]), torch.tensor([4.0, -5.0, 6.0]), torch.tensor([0.5, 8.0, -9.0])]


@pytest.mark.parametrize("op,expect", [("sum", [5.5, 5.0, 0.0]), ("prod", [2.0, -80.0, -162.0]),
                                        ("max", [4.0, 8.0, 6.0]), ("min", [0.5, -5.0, -9.0])])
def test_host_all_reduce_ops(op, expect):
    bufs = _ranks()
    HostCollectives(3).all_reduce(bufs, op)
    for b in bufs:
        assert torch.allclose(b, torch.tensor(expect))


def test_host_broadcast_scatter_gather():
    hc = HostCollectives(3)
    bufs = _ranks()
    hc.broadcast(bufs, 1)
    assert all(torch.equal(b, torch.tensor([4.0, -5.0, 6.0])) for b in bufs)
    send = [torch.arange(6.0) + r for r in range(3)]
    recv = [torch.zeros(2) for _ in range(3)]
    hc.reduce_scatter(send, recv)
    assert torch.equal(recv[1], torch.tensor([9.0, 12.0]))
    out = [torch.zeros(9) for _ in range(3)]
    hc.all_gather(_ranks(), out)
    assert torch.equal(out[2][3:6], torch.tensor([4.0, -5.0, 6.0]))
    with pytest.raises(ValueError):
        hc.all_reduce(_ranks()[:2])
    with pytest.raises(ValueError):
        hc.reduce_scatter([torch.zeros(4)] * 3, [torch.zeros(1)] * 3)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _gloo_worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        c = Communicator(backend="gloo")
        res = {}
        for op in ReduceOp:
            t = torch.tensor([1.0 + rank, 2.0 - 3 * rank, 0.5 * rank])
            c.all_reduce(t, op)
            res[op.name] = t
        b = torch.tensor([float(rank)] * 3)
        c.broadcast(b, root=1)
        res["bcast"] = b
        out = torch.zeros(2)
        c.reduce_scatter(out, torch.arange(4.0) * (rank + 1))
        res["rs"] = out
        g = torch.zeros(4)
        c.all_gather(g, torch.tensor([rank, rank + 10.0]))
        res["ag"] = g
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_communicator_gloo_matches_host_semantics():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    for op in ReduceOp:
        bufs = [torch.tensor([1.0 + r, 2.0 - 3 * r, 0.5 * r]) for r in range(world)]
        HostCollectives(world).all_reduce(bufs, op)
        for r in range(world):
            assert torch.allclose(got[r][op.name], bufs[r])
    for r in range(world):
        assert torch.equal(got[r]["bcast"], torch.ones(3))
        assert torch.equal(got[r]["ag"], torch.tensor([0.0, 10.0, 1.0, 11.0]))
    assert torch.equal(got[0]["rs"], torch.tensor([0.0, 3.0])) and torch.equal(got[1]["rs"], torch.tensor([6.0, 9.0]))


def test_collective_roofline_counts_both_directions():
    from predicitivecoding_b200.parallel.bench_collectives import nvlink_bytes_per_direction as vol
    n = 134_105_856
    # 2 ranks: half of the gradients pulled in (4 B) and half of the weights pushed in (2 B) per parameter
    assert vol("rs_adamw_ag", n, 2) == 0.5 * n * 6
    assert abs(vol("rs_adamw_ag", n, 8) - 7 / 8 * n * 6) < 1
    assert vol("pc_allreduce_update", 64 << 20, 8) == 7 / 8 * (64 << 20) * 10
    assert vol("all_reduce", 1 << 28, 4) == 2 * 3 / 4 * (1 << 28)
    assert vol("rs_adamw_ag", n, 1) == 0.0
    with pytest.raises(ValueError):
        vol("broadcast", 1, 2)


def test_two_shot_shards_cover_message_once_and_align():
    from predicitivecoding_b200.parallel.collectives import two_shot_shard
    for world in (1, 2, 3, 4, 8):
        for n in (1, 7, 8, 9, 63, 64, 1000, 4097, 1 << 20, (1 << 20) + 5):
            shards = [two_shot_shard(n, world, r) for r in range(world)]
            covered = []
            for a, b in shards:
                assert 0 <= a <= b <= n
                if b > a:
                    assert a % 8 == 0          # 16-byte aligned start for fp32 and bf16
                covered.extend(range(a, b)) if n < 5000 else None
            if n < 5000:
                assert covered == list(range(n))
            assert sum(b - a for a, b in shards) == n
