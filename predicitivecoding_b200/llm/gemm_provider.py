"""Pluggable GEMM provider for the autograd LLM stack, with route tracking.

Reference: PredictiveCoding.LLM/Infrastructure/Gemm.cs:1-136 (``IGemmProvider.MatMul`` /
``MatMulMixed`` with a CPU provider whose mixed path rounds both operands to fp16 first; a static
``Gemm.Provider`` that the autograd MatMul calls; ``BatchedMatMul``; ``MatVec``).

``TorchGemmProvider`` is the host path.  ``B200GemmProvider`` sends bf16 operands through the
extension's tcgen05 GEMM (fp32 accumulate) and falls back to nothing: it raises if the extension
is missing.  ``Gemm.calls`` counts which provider served each call so tests can assert the route.
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

import torch


class TorchGemmProvider:
    name = "torch"

    def matmul(self, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
        return a.float() @ b.float()

    def matmul_mixed(self, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
        return a.to(torch.float16).float() @ b.to(torch.float16).float()


class B200GemmProvider:
    """C[M,N] = A[M,K] @ B[K,N] on the tensor cores (bf16 in, fp32 out)."""
    name = "b200"

    def matmul(self, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
        from .. import ops
        a16 = a.to(device="cuda", dtype=torch.bfloat16).contiguous()
        b16 = b.to(device="cuda", dtype=torch.bfloat16).contiguous()
        return ops.gemm(a16, b16, b_mn=True, epi=ops.EPI_F32)

    matmul_mixed = matmul


class Gemm:
    provider = TorchGemmProvider()
    calls = {}

    @classmethod
    def set_provider(cls, p) -> None:
        cls.provider = p

    @classmethod
    def _note(cls):
        cls.calls[cls.provider.name] = cls.calls.get(cls.provider.name, 0) + 1

    @classmethod
    def matmul(cls, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
        if a.shape[-1] != b.shape[0]:
            raise ValueError("inner dimensions differ")
        cls._note()
        return cls.provider.matmul(a, b)

    @classmethod
    def matmul_mixed(cls, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
        if a.shape[-1] != b.shape[0]:
            raise ValueError("inner dimensions differ")
        cls._note()
        return cls.provider.matmul_mixed(a, b)

    @classmethod
    def batched_matmul(cls, batch: Sequence[Tuple[torch.Tensor, torch.Tensor]]) -> List[torch.Tensor]:
        return [cls.matmul(a, b) for a, b in batch]

    @staticmethod
    def matvec(w: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        if x.numel() != w.shape[1]:
            raise ValueError(f"x has {x.numel()} elements; expected {w.shape[1]}.")
        return w.float() @ x.float().reshape(-1)


class GemmMatMul(torch.autograd.Function):
    """Autograd matmul routed through ``Gemm`` for the forward and both backward products."""

    @staticmethod
    def forward(ctx, a, b):
        ctx.save_for_backward(a, b)
        return Gemm.matmul(a, b).to(a.device)

    @staticmethod
    def backward(ctx, g):
        a, b = ctx.saved_tensors
        return Gemm.matmul(g, b.T).to(a.device), Gemm.matmul(a.T, g).to(b.device)


def auto_route(device: torch.device) -> None:
    """Pick the tensor-core provider when a CUDA device is in use, the torch provider otherwise."""
    Gemm.set_provider(B200GemmProvider() if device.type == "cuda" else TorchGemmProvider())
