"""The allocation-free attention backward, called through its exported C symbol.

pcb_attn_bwd_noalloc is for callers that cannot allocate device memory where
they call attention (a host that owns all device memory through its own pool, a
loop that must not take cudaMalloc's implicit synchronisation, a foreign-language
host with only a C ABI).  It must give the same gradients as the regular entry
point, which takes caller-allocated scratch, and must not carry stale scratch
from one call into the next.  This file is collected last on purpose.
"""
import ctypes
import math

import pytest
import torch

from predicitivecoding_b200 import ops

pytestmark = pytest.mark.gpu


def _symbol():
    lib = ctypes.CDLL(ops.ext().__file__)
    f = lib.pcb_attn_bwd_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong,
                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                  ctypes.c_int, ctypes.c_float, ctypes.c_void_p]
    return f


def _inputs(B, S, H, hd, seed):
    g = torch.Generator().manual_seed(seed)
    D = H * hd
    qkv = torch.randn(B * S, 3 * D, generator=g).to("cuda", torch.bfloat16)
    dout = torch.randn(B * S, D, generator=g).to("cuda", torch.bfloat16)
    out = torch.empty(B * S, D, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B * H, S, device="cuda")
    ops.attn_fwd(qkv, out, lse, B, S, H, hd, 1 / math.sqrt(hd))
    return qkv, out, dout, lse


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


@pytest.mark.parametrize("hd", [64, 128])
def test_noalloc_matches_regular_entry_on_two_calls(hd):
    f = _symbol()
    B, S, H = 2, 256, 2
    a = _inputs(B, S, H, hd, seed=11)
    b = _inputs(B, S, H, hd, seed=12)
    got_a = _noalloc(f, *a, B, S, H, hd)
    got_b = _noalloc(f, *b, B, S, H, hd)      # second call: scratch holds call one's dQ partials
    torch.cuda.synchronize()
    ref_a = _regular(*a, B, S, H, hd)
    ref_b = _regular(*b, B, S, H, hd)
    torch.cuda.synchronize()
    assert _rel(got_a, ref_a) < 0.03
    assert _rel(got_b, ref_b) < 0.03


def test_noalloc_rejects_problems_beyond_its_scratch():
    f = _symbol()
    # 64 x 1024 tokens x 1024 features of fp32 dQ accumulator = 256 MiB > 16 MiB built-in scratch
    B, S, H, hd = 64, 1024, 16, 64
    rc = f(0, 3 * H * hd, 0, 0, H * hd, 0, 0, 3 * H * hd, B, S, H, hd, 0.125, torch.cuda.current_stream().cuda_stream)
    assert rc == -7
