"""Weight compression for inference: 16-bit (fp16/bf16) matrices and per-row symmetric int8/int4.

Reference: PredictiveCoding.LLM/Infrastructure/Precision.cs:1-87 (BFloat16 by round-to-nearest-even
with NaN kept quiet, LowPrecisionMatrix) and Quantization.cs:1-135 (Int8Matrix: scale = max|w|/127,
q = clamp(round(w/scale), -127, 127); Int4Matrix: scale = max|w|/7, two's-complement nibbles, even
column in the low nibble; both accumulate q*x then multiply by the row scale).

On a GPU the matrices stay resident and ``matvec``/``matmul`` run the weight-only kernels of the
extension (dequantise in registers, fp32 accumulate); on the CPU they run the same arithmetic in torch.
"""
from __future__ import annotations

import torch


def bf16_bits(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> bf16 bit patterns (int32 holding uint16) by round-to-nearest-even; NaN stays NaN."""
    b = x.float().contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    rounded = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) & 0xFFFF
    nan = ((b >> 16) | 0x40) & 0xFFFF
    return torch.where(torch.isnan(x.float()), nan, rounded).to(torch.int32)


def bf16_from_bits(bits: torch.Tensor) -> torch.Tensor:
    return (bits.to(torch.int64) << 16).to(torch.int32).view(torch.float32)


class LowPrecisionMatrix:
    def __init__(self, w: torch.Tensor, precision: str = "bf16"):
        if w.dim() != 2:
            raise ValueError("weight must be a [rows, cols] matrix.")
        if precision not in ("fp16", "bf16"):
            raise ValueError("precision must be fp16 or bf16")
        self.precision = precision
        self.rows, self.cols = w.shape
        if precision == "fp16":
            self.data = w.to(torch.float16)
        else:
            self.data = bf16_from_bits(bf16_bits(w.float())).to(torch.bfloat16) if w.device.type == "cpu" \
                else w.to(torch.bfloat16)

    @property
    def memory_bytes(self) -> int:
        return self.data.numel() * 2

    def to_float(self) -> torch.Tensor:
        return self.data.float()

    def matvec(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.cols:
            raise ValueError(f"x has {x.shape[-1]} elements; expected {self.cols}.")
        return x.float() @ self.data.float().T


class Int8Matrix:
    def __init__(self, w: torch.Tensor):
        if w.dim() != 2:
            raise ValueError("weight must be [rows, cols].")
        w = w.float()
        self.rows, self.cols = w.shape
        amax = w.abs().amax(1).clamp(min=1e-12)
        self.scale = amax / 127.0
        self.q = torch.clamp(torch.round(w / self.scale[:, None]), -127, 127).to(torch.int8)

    @property
    def memory_bytes(self) -> int:
        return self.q.numel() + self.scale.numel() * 4

    def to_float(self) -> torch.Tensor:
        return self.q.float() * self.scale[:, None]

    def matvec(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.cols:
            raise ValueError(f"x has {x.shape[-1]} elements; expected {self.cols}.")
        if x.is_cuda and self.q.is_cuda:
            from .. import ops
            return ops.wq_matmul(x, self.q, self.scale, bits=8)
        return (x.float() @ self.q.float().T) * self.scale


class Int4Matrix:
    def __init__(self, w: torch.Tensor):
        if w.dim() != 2:
            raise ValueError("weight must be [rows, cols].")
        w = w.float()
        self.rows, self.cols = w.shape
        amax = w.abs().amax(1).clamp(min=1e-12)
        self.scale = amax / 7.0
        q = torch.clamp(torch.round(w / self.scale[:, None]), -7, 7).to(torch.int32)
        if self.cols % 2:
            q = torch.cat([q, torch.zeros(self.rows, 1, dtype=torch.int32, device=q.device)], 1)
        nib = q & 0xF
        self.packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).to(torch.uint8)

    @property
    def memory_bytes(self) -> int:
        return self.packed.numel() + self.scale.numel() * 4

    def unpack(self) -> torch.Tensor:
        p = self.packed.to(torch.int32)
        lo, hi = p & 0xF, (p >> 4) & 0xF
        q = torch.stack([lo, hi], -1).flatten(-2)[:, : self.cols]
        return torch.where(q >= 8, q - 16, q)

    def to_float(self) -> torch.Tensor:
        return self.unpack().float() * self.scale[:, None]

    def matvec(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.cols:
            raise ValueError(f"x has {x.shape[-1]} elements; expected {self.cols}.")
        if x.is_cuda and self.packed.is_cuda and self.cols % 2 == 0:
            from .. import ops
            return ops.wq_matmul(x, self.packed, self.scale, bits=4)
        return (x.float() @ self.unpack().float().T) * self.scale
