"""Native allocator, stream pool, device tensors and the peer collectives on the GPU."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from predicitivecoding_b200 import ops

pytestmark = pytest.mark.gpu


def test_caching_allocator_reuses_blocks():
    from predicitivecoding_b200.runtime import DeviceAllocator
    a = DeviceAllocator(0)
    a.empty_cache()
    s0 = a.stats()
    t = a.alloc((1000,), torch.float32)
    t.fill_(3.0)
    ptr = t.data_ptr()
    del t
    u = a.alloc((900,), torch.float32)          # same 4 KiB class -> the cached block
    s1 = a.stats()
    assert u.data_ptr() == ptr and s1.cache_hits >= s0.cache_hits + 1
    big = a.alloc((3 << 20,), torch.float32)
    assert a.stats().reserved >= s1.reserved + (12 << 20) and a.stats().peak >= a.stats().allocated
    del big, u
    torch.cuda.synchronize()
    a.empty_cache()
    assert a.stats().reserved <= s0.reserved + 4096


def test_allocator_stream_safety_with_record_stream():
    from predicitivecoding_b200.runtime import DeviceAllocator, StreamManager
    a = DeviceAllocator(0)
    side = StreamManager.shared().create_stream(0)
    t = a.alloc((1 << 20,), torch.float32)
    t.fill_(1.0)
    ev = torch.cuda.Event()
    ev.record()
    with torch.cuda.stream(side):
        side.wait_event(ev)
        torch.cuda._sleep(100_000_000)
        t.mul_(2.0)
    a.record_stream(t, side)
    ptr = t.data_ptr()
    del t
    busy = not side.query()
    u = a.alloc((1 << 20,), torch.float32)      # side stream may still use the old block
    if busy:
        assert u.data_ptr() != ptr
    torch.cuda.synchronize()
    del u
    w = a.alloc((1 << 20,), torch.float32)      # once the side stream is done the block comes back
    assert w.data_ptr() in (ptr,) or busy


def test_stream_pool_streams_run_kernels():
    from predicitivecoding_b200.runtime import StreamManager
    sm = StreamManager.shared()
    s1, s2 = sm.create_stream(0), sm.create_stream(0, high_priority=True)
    assert s1.cuda_stream != torch.cuda.default_stream().cuda_stream and s1.cuda_stream != s2.cuda_stream
    a = torch.randn(256, 128, device="cuda").to(torch.bfloat16)
    b = torch.randn(64, 128, device="cuda").to(torch.bfloat16)
    with torch.cuda.stream(s1):
        c = ops.gemm(a, b, epi=ops.EPI_F32)
    s1.synchronize()
    assert torch.allclose(c, a.float() @ b.float().T, atol=0.05, rtol=0.02)
    assert sm.thread_stream(0) is sm.thread_stream(0)


def test_device_tensor_matmul_on_tensor_cores():
    from predicitivecoding_b200.runtime import Device, DeviceTensor, TensorOps
    a = DeviceTensor.from_host(torch.randn(64, 32), Device.cuda(0))
    b = DeviceTensor.from_host(torch.randn(32, 48), Device.cuda(0))
    before = ops.launch_count()
    c = TensorOps.matmul(a, b)
    assert ops.launch_count() == before + 1 and c.is_on_device
    assert torch.allclose(c.to_host(), a.to_host() @ b.to_host(), atol=0.1, rtol=0.02)
    assert DeviceTensor.from_host(torch.ones(3), Device.cuda_multi()).device == Device.cuda(0)


def test_peer_collectives_single_rank_kernels():
    from predicitivecoding_b200.parallel.collectives import Communicator
    c = Communicator(backend="peer", capacity_bytes=1 << 20)
    for dt in (torch.float32, torch.bfloat16):
        x = torch.randn(100_003, device="cuda").to(dt)      # > capacity for bf16? 200 KB, two chunks for fp32
        y = x.clone()
        c.all_reduce(y)
        assert torch.equal(y, x)
        out = torch.empty_like(x)
        c.all_gather(out, x)
        assert torch.equal(out, x)
    c.check()


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
    try:
        from predicitivecoding_b200.parallel.collectives import Communicator, ReduceOp
        peer = Communicator(backend="peer", capacity_bytes=8 << 20)
        nccl = Communicator(backend="nccl")
        errs = []
        for n in (1000, 3_000_001):                 # one-shot and two-shot (and chunked) paths
            for dt in (torch.float32, torch.bfloat16):
                g = torch.Generator(device=dev).manual_seed(rank * 7 + n)
                x = torch.randn(n, device=dev, generator=g).to(dt)
                for op in (ReduceOp.SUM, ReduceOp.MAX, ReduceOp.MIN) if n == 1000 else (ReduceOp.SUM,):
                    a, b = x.clone(), x.clone()
                    peer.all_reduce(a, op)
                    nccl.all_reduce(b, op)
                    errs.append(float((a.float() - b.float()).abs().max()))
        x = torch.randn(4096 * world, device=dev)
        a, b = torch.empty(4096, device=dev), torch.empty(4096, device=dev)
        peer.reduce_scatter(a, x)
        nccl.reduce_scatter(b, x.clone())
        errs.append(float((a - b).abs().max()))
        y = torch.randn(5000, device=dev)
        a, b = torch.empty(5000 * world, device=dev), torch.empty(5000 * world, device=dev)
        peer.all_gather(a, y)
        nccl.all_gather(b, y)
        errs.append(float((a - b).abs().max()))
        z = torch.full((777,), float(rank), device=dev)
        peer.broadcast(z, root=1)
        errs.append(float((z - 1.0).abs().max()))
        peer.check()
        torch.cuda.synchronize()
        q.put((rank, errs))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_collectives_match_nccl_two_ranks():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    for r in range(world):
        # sums over 2 ranks are order-independent except bf16 rounding of the result
        assert max(res[r]) < 2e-2, res[r]


def test_runtime_kernel_saxpy_matches_torch():
    from predicitivecoding_b200.runtime.kernel import RuntimeKernel
    src = r'''
extern "C" __global__ void saxpy(float a, const float* x, float* y, int n) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = a * x[i] + y[i];
}'''
    k = RuntimeKernel(src, "saxpy")
    x = torch.randn(100_003, device="cuda")
    y = torch.randn(100_003, device="cuda")
    ref = 1.5 * x + y
    k.launch_1d(x.numel(), [1.5, x, y, x.numel()], sync=True)
    # the kernel fuses the multiply-add; torch rounds twice: allow one rounding near zero
    assert torch.allclose(y, ref, rtol=1e-5, atol=1e-6)
    k.close()


def test_canary_allocator_detects_overrun():
    from predicitivecoding_b200.runtime.allocator import CanaryAllocator
    a = CanaryAllocator(0)
    good = a.alloc((1000,), torch.float32)
    bad = a.alloc((1000,), torch.float32)
    good.fill_(1.0)
    bad.fill_(2.0)
    assert a.verify() == []
    # write past the end of `bad` through its underlying storage (as an out-of-bounds kernel would)
    torch.as_strided(bad, (1002,), (1,)).fill_(3.0)
    assert a.verify() == [1]


def test_deterministic_weight_gradient_is_bitwise_repeatable():
    from predicitivecoding_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(1)
    dy = torch.randn(4096, 768, device="cuda", generator=g).to(torch.bfloat16)
    x = torch.randn(4096, 768, device="cuda", generator=g).to(torch.bfloat16)
    ops.set_deterministic(True)
    try:
        outs = []
        for _ in range(2):
            c = torch.zeros(768, 768, device="cuda")
            ops.gemm(dy, x, a_mn=True, b_mn=True, epi=ops.EPI_RED_F32, c=c)
            outs.append(c)
        torch.cuda.synchronize()
        assert torch.equal(outs[0], outs[1])
        ref = dy.float().T @ x.float()
        assert float((outs[0] - ref).norm() / ref.norm()) < 1e-2
    finally:
        ops.set_deterministic(False)
