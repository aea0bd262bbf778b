"""Mixture-of-experts FFN on the device: router, expert-sorted dispatch, grouped tcgen05 GEMMs, combine,
and the backward of all of it.

Semantics (PredictiveCoding.LLM/Autograd/DecoderLM.cs:556-615): gates = softmax(x R) over all E experts;
each row runs its top-k experts, y = sum_{e in topk} gate_e * (gelu_tanh(x W1_e + b1_e) W2_e + b2_e) with
the gates not renormalised; the Switch balance loss is E * sum_e mean_t(gate[t, e]) * frac_e with
frac_e = (rows routed to e) / (rows * k), added to the loss with weight ``MoeBalanceWeight``.

Device plan per layer (no host synchronisation, so the whole step stays one CUDA graph):

    moe_route     one warp per token: logits, softmax, top-k                      -> gates [M, E], topi [M, k]
    moe_dispatch  one CTA: stable counting sort of the M*k assignments by expert   -> seg, pos, src, rgate
                  (segments padded to 256 rows, the CTA-pair tile), balance terms
    moe_gather    xs[p] = x[src[p]]                                                 [cap, D] bf16
    grouped GEMM  pre, act = gelu(xs W1_e^T + b1_e) per 256-row tile of expert e    [cap, F] bf16
    grouped GEMM  ys = act W2_e^T + b2_e                                            [cap, D] fp32
    moe_combine   out[t] = res[t] + sum_j gate_j ys[pos_j]                          [M, D] fp32

Backward: moe_combine_bwd (dys = gate * dx per sorted row, dgate = <dx, ys>), grouped dgrad GEMMs with the
GELU backward epilogue, grouped weight-gradient GEMMs whose K range is each expert's segment, per-expert
column sums for the bias gradients, and moe_router_bwd (softmax backward incl. the balance term, the
scatter of the expert input gradients back to the tokens, and dx += dlogits R) plus the router's weight
gradient.

Weights as the kernels read them (nn.Linear layout, K-major): router [E, D]; w1 [E*F, D] (block e =
W1_e^T); w2 [E*D, F] (block e = W2_e^T); b1 [E*F]; b2 [E*D].  Gradients are fp32 with the same shapes and
are accumulated (atomically) into zeroed buffers.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn.functional as F

from . import EPI_F32, EPI_GELU, EPI_GELU_BWD, EPI_RED_F32, ext

SEG = 256   # expert segments are padded to the CTA-pair GEMM's 256-row tile
MAX_EXPERTS = 64
MAX_TOP_K = 8


def capacity(M: int, k: int, E: int) -> int:
    """Rows of the expert-sorted buffer: every assignment plus the worst-case padding of E segments."""
    return (M * k + E * (SEG - 1) + SEG - 1) // SEG * SEG


def supported(D: int, F_: int, E: int, k: int) -> bool:
    """Shapes the device MoE path handles (grouped GEMM tiles may not straddle experts)."""
    return 1 <= E <= MAX_EXPERTS and 1 <= k <= min(E, MAX_TOP_K) and D % SEG == 0 and F_ % SEG == 0


@dataclass
class MoEBuffers:
    """Per-layer routing state and activations kept from the forward for the backward."""
    gates: torch.Tensor
    topi: torch.Tensor
    pos: torch.Tensor
    src: torch.Tensor
    rgate: torch.Tensor
    seg: torch.Tensor
    coef: torch.Tensor
    xs: torch.Tensor
    pre: torch.Tensor
    act: torch.Tensor
    ys: torch.Tensor

    @staticmethod
    def allocate(M: int, D: int, F_: int, E: int, k: int, device) -> "MoEBuffers":
        cap = capacity(M, k, E)
        f32, i32, bf16 = torch.float32, torch.int32, torch.bfloat16
        return MoEBuffers(
            gates=torch.zeros(M, E, device=device, dtype=f32), topi=torch.zeros(M, k, device=device, dtype=i32),
            pos=torch.zeros(M, k, device=device, dtype=i32), src=torch.full((cap,), -1, device=device, dtype=i32),
            rgate=torch.zeros(cap, device=device, dtype=f32), seg=torch.zeros(E + 1, device=device, dtype=i32),
            coef=torch.zeros(E, device=device, dtype=f32), xs=torch.zeros(cap, D, device=device, dtype=bf16),
            pre=torch.zeros(cap, F_, device=device, dtype=bf16), act=torch.zeros(cap, F_, device=device, dtype=bf16),
            ys=torch.zeros(cap, D, device=device, dtype=f32))


@dataclass
class MoEScratch:
    """Backward scratch, shared by all layers."""
    dys: torch.Tensor
    dgate: torch.Tensor
    dpre: torch.Tensor
    dxs: torch.Tensor
    dlogits: torch.Tensor

    @staticmethod
    def allocate(M: int, D: int, F_: int, E: int, k: int, device) -> "MoEScratch":
        cap = capacity(M, k, E)
        return MoEScratch(dys=torch.zeros(cap, D, device=device, dtype=torch.bfloat16),
                          dgate=torch.zeros(cap, device=device, dtype=torch.float32),
                          dpre=torch.zeros(cap, F_, device=device, dtype=torch.bfloat16),
                          dxs=torch.zeros(cap, D, device=device, dtype=torch.float32),
                          dlogits=torch.zeros(M, E, device=device, dtype=torch.float32))


def gemm_grouped(a, b, *, b_mn=False, epi, seg, count, mode, c=None, d=None, aux=None, bias=None, err=None):
    ext().gemm_grouped(a, b, bool(b_mn), int(epi), seg, int(count), int(mode), c, d, aux, bias, err)


def forward(x: torch.Tensor, res: torch.Tensor, out: torch.Tensor, router: torch.Tensor, w1: torch.Tensor,
            b1: torch.Tensor, w2: torch.Tensor, b2: torch.Tensor, k: int, buf: MoEBuffers,
            loss_acc: Optional[torch.Tensor] = None, loss_weight: float = 0.0) -> None:
    """out = res + MoE(x).  x: [M, D] bf16 (the normalised input), res/out: [M, D] fp32.  Adds
    ``loss_weight * balance`` to ``loss_acc`` (device fp32 scalar) when given."""
    E = router.shape[0]
    ext().moe_route(x, router, int(k), buf.gates, buf.topi)
    ext().moe_dispatch(buf.topi, buf.gates, int(k), buf.seg, buf.pos, buf.src, buf.rgate, buf.coef, loss_acc,
                       float(loss_weight))
    ext().moe_gather(x, buf.src, buf.seg, buf.xs)
    gemm_grouped(buf.xs, w1, epi=EPI_GELU, seg=buf.seg, count=E, mode=1, c=buf.pre, d=buf.act, bias=b1)
    gemm_grouped(buf.act, w2, epi=EPI_F32, seg=buf.seg, count=E, mode=1, c=buf.ys, bias=b2)
    ext().moe_combine(res, buf.ys, buf.pos, buf.rgate, int(k), out)


def backward(dx: torch.Tensor, x: torch.Tensor, dn: torch.Tensor, router: torch.Tensor, w1: torch.Tensor,
             w2: torch.Tensor, k: int, buf: MoEBuffers, scr: MoEScratch, g_router: torch.Tensor, g_w1: torch.Tensor,
             g_b1: torch.Tensor, g_w2: torch.Tensor, g_b2: torch.Tensor, balance_weight: float = 0.0) -> None:
    """Given dx = dL/d(out) [M, D] fp32, writes dn = dL/dx [M, D] fp32 and accumulates the weight
    gradients (fp32, same shapes as the weights) into g_*.  The loss holds ``balance_weight * balance``
    (the balance's gradient is added to the router's)."""
    E = router.shape[0]
    ext().moe_combine_bwd(dx, buf.ys, buf.src, buf.rgate, buf.seg, scr.dys, scr.dgate)
    ext().moe_seg_colsum(scr.dys, buf.seg, g_b2)
    gemm_grouped(scr.dys, buf.act, b_mn=True, epi=EPI_RED_F32, seg=buf.seg, count=E, mode=2, c=g_w2)
    gemm_grouped(scr.dys, w2, b_mn=True, epi=EPI_GELU_BWD, seg=buf.seg, count=E, mode=1, c=scr.dpre, aux=buf.pre)
    ext().moe_seg_colsum(scr.dpre, buf.seg, g_b1)
    gemm_grouped(scr.dpre, buf.xs, b_mn=True, epi=EPI_RED_F32, seg=buf.seg, count=E, mode=2, c=g_w1)
    gemm_grouped(scr.dpre, w1, b_mn=True, epi=EPI_F32, seg=buf.seg, count=E, mode=1, c=scr.dxs)
    ext().moe_router_bwd(buf.gates, buf.topi, buf.pos, scr.dgate, buf.coef, float(balance_weight), scr.dxs, router,
                         int(k), scr.dlogits, dn)
    ext().moe_router_wgrad(scr.dlogits, x, g_router)


KERNELS_PER_FORWARD = 6
KERNELS_PER_BACKWARD = 9


# ---------------------------------------------------------------------------------------------- reference
def reference(x: torch.Tensor, router: torch.Tensor, w1: torch.Tensor, b1: torch.Tensor, w2: torch.Tensor,
              b2: torch.Tensor, k: int, topi: Optional[torch.Tensor] = None):
    """fp32 PyTorch statement of the same layer (differentiable): returns (y [M, D], balance, topi).
    Weights in the kernels' layout (router [E, D], w1 [E*F, D], w2 [E*D, F]).  ``topi`` fixes the
    routing (so a bf16 device run and this fp32 reference agree on near-ties)."""
    E = router.shape[0]
    D = x.shape[1]
    F_ = w1.shape[0] // E
    gates = torch.softmax(x @ router.t(), dim=-1)
    if topi is None:
        topi = torch.topk(gates.detach(), k, dim=-1).indices
    topi = topi.long()
    mask = torch.zeros_like(gates).scatter_(1, topi, 1.0)
    y = torch.zeros_like(x)
    for e in range(E):
        rows = torch.nonzero(mask[:, e] > 0, as_tuple=False).flatten()
        if rows.numel() == 0:
            continue
        sub = x.index_select(0, rows)
        h = F.gelu(sub @ w1[e * F_:(e + 1) * F_].t() + b1[e * F_:(e + 1) * F_], approximate="tanh")
        o = h @ w2[e * D:(e + 1) * D].t() + b2[e * D:(e + 1) * D]
        y = y.index_add(0, rows, o * gates.index_select(0, rows)[:, e:e + 1])
    frac = mask.sum(0) / (x.shape[0] * k)
    balance = (gates.mean(0) * frac).sum() * E
    return y, balance, topi
