"""The allocation-free attention backward, called through its exported C symbol.

pcb_attn_bwd_noalloc is for callers that cannot allocate device memory where
they call attention (a host that owns all device memory through its own pool, a
loop that must not take cudaMalloc's implicit synchronisation, a foreign-language
host with only a C ABI).  Its gradients are checked against a plain fp32 PyTorch
attention backward and against the regular entry point (caller-allocated
scratch), on two calls in a row so that stale scratch from the first call would
show up in the second.  The shapes include one that fills the built-in scratch
almost exactly and one just beyond it.  This file is collected last on purpose.
"""
import ctypes
import math

import pytest
import torch

from predicitivecoding_b200 import ops

pytestmark = pytest.mark.gpu

SCRATCH_FLOATS = 16 * 1024 * 1024 // 4


def _symbol():
    lib = ctypes.CDLL(ops.ext().__file__)
    f = lib.pcb_attn_bwd_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong,
                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                  ctypes.c_int, ctypes.c_float, ctypes.c_void_p]
    return f


def _need(B, S, H, hd):
    return (B * S * H * hd + 63) // 64 * 64 + B * H * S


def _inputs(B, S, H, hd, seed):
    g = torch.Generator().manual_seed(seed)
    D = H * hd
    qkv = torch.randn(B * S, 3 * D, generator=g).to("cuda", torch.bfloat16)
    dout = torch.randn(B * S, D, generator=g).to("cuda", torch.bfloat16)
    out = torch.empty(B * S, D, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B * H, S, device="cuda")
    ops.attn_fwd(qkv, out, lse, B, S, H, hd, 1 / math.sqrt(hd))
    return qkv, out, dout, lse


def _fp32_reference(qkv, dout, B, S, H, hd):
    """dq | dk | dv of causal softmax attention in fp32 autograd, on the same bf16 inputs."""
    D = H * hd
    x = qkv.float().view(B, S, 3, H, hd).permute(2, 0, 3, 1, 4)      # [3, B, H, S, hd]
    q, k, v = (t.detach().clone().requires_grad_(True) for t in x)
    s = (q @ k.transpose(-1, -2)) / math.sqrt(hd)
    mask = torch.ones(S, S, dtype=torch.bool, device=qkv.device).triu(1)
    o = torch.softmax(s.masked_fill(mask, float("-inf")), dim=-1) @ v
    o.backward(dout.float().view(B, S, H, hd).permute(0, 2, 1, 3))
    grads = [t.grad.permute(0, 2, 1, 3).reshape(B * S, D) for t in (q, k, v)]
    return torch.cat(grads, dim=1)


def _regular(qkv, out, dout, lse, B, S, H, hd):
    D = H * hd
    dqkv = torch.zeros(B * S, 3 * D, device="cuda", dtype=torch.bfloat16)
    dvec = torch.empty(B * H, S, device="cuda")
    dq_acc = torch.empty(B * S, D, device="cuda")
    ops.attn_bwd(qkv, out, dout, lse, dvec, dq_acc, dqkv, B, S, H, hd, 1 / math.sqrt(hd))
    return dqkv


def _noalloc(f, qkv, out, dout, lse, B, S, H, hd):
    D = H * hd
    dqkv = torch.zeros(B * S, 3 * D, device="cuda", dtype=torch.bfloat16)
    stream = torch.cuda.current_stream().cuda_stream
    rc = f(qkv.data_ptr(), qkv.stride(0), out.data_ptr(), dout.data_ptr(), dout.stride(0), lse.data_ptr(),
           dqkv.data_ptr(), dqkv.stride(0), B, S, H, hd, 1 / math.sqrt(hd), stream)
    assert rc == 0, rc
    return dqkv


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


@pytest.mark.parametrize("B,S,H,hd", [(2, 256, 2, 64), (2, 256, 2, 128),
                                      (4, 128, 126, 64),     # fills all but 1 Ki floats of the scratch
                                      (2, 128, 127, 128)])   # fills all but 256 floats
def test_noalloc_matches_fp32_reference_and_regular_entry_on_two_calls(B, S, H, hd):
    assert _need(B, S, H, hd) <= SCRATCH_FLOATS
    f = _symbol()
    a = _inputs(B, S, H, hd, seed=11)
    b = _inputs(B, S, H, hd, seed=12)
    got_a = _noalloc(f, *a, B, S, H, hd)
    got_b = _noalloc(f, *b, B, S, H, hd)      # second call: the scratch still holds call one's dQ partials
    torch.cuda.synchronize()
    for got, inp in ((got_a, a), (got_b, b)):
        qkv, out, dout, lse = inp
        assert _rel(got, _fp32_reference(qkv, dout, B, S, H, hd)) < 0.03
        assert _rel(got, _regular(qkv, out, dout, lse, B, S, H, hd)) < 0.02


@pytest.mark.parametrize("B,S,H,hd", [(4, 128, 127, 64), (2, 128, 128, 128), (64, 1024, 16, 64),
                                      (1 << 30, 1 << 30, 16, 64)])   # the last one overflows 64-bit products
def test_noalloc_rejects_problems_beyond_its_scratch(B, S, H, hd):
    f = _symbol()
    if B * S * H < 1 << 40:
        assert _need(B, S, H, hd) > SCRATCH_FLOATS
    rc = f(0, 3 * H * hd, 0, 0, H * hd, 0, 0, 3 * H * hd, B, S, H, hd, 0.125, torch.cuda.current_stream().cuda_stream)
    assert rc == -7


def test_noalloc_rejects_misaligned_operands():
    f = _symbol()
    B, S, H, hd = 1, 128, 1, 64
    qkv, out, dout, lse = _inputs(B, S, H, hd, seed=3)
    dqkv = torch.zeros(B * S * 3 * H * hd + 8, device="cuda", dtype=torch.bfloat16)
    rc = f(qkv.data_ptr(), qkv.stride(0), out.data_ptr(), dout.data_ptr(), dout.stride(0), lse.data_ptr(),
           dqkv.data_ptr() + 2, 3 * H * hd, B, S, H, hd, 0.125, torch.cuda.current_stream().cuda_stream)
    assert rc == -10
