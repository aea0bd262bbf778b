"""Binary record of one PC layer, byte-compatible with the reference LayerSerializer.

Layout (PredicitiveCoding/Model/LayerSerializer.cs:10-41), little endian:

    0   int32  Size            4  int32  LowerSize
    8   f32    Precision      12  f32    WeightDecay
    16  f32    StateLR        20  f32    WeightLR
    24  u8     IsClamped      25  u8     flags (bit0 diag-Pi, bit1 prior, bit2 Half W, bit3 bf16 W, bit4 int8 W)
    26  2 pad
    28  Mu[Size] f32, PredictionError[Size] f32
    if LowerSize > 0: W in the stored precision, then Bias, PreActivation, Prediction (f32 [LowerSize] each)
    if diag: DiagonalPrecision[Size] f32;  if prior: PriorMean[Size] f32

int8 weights are affine per row: f32 scales[rows], i8 zero points[rows], i8 codes[rows*cols];
s = (max-min)/255, z = round(-min/s) - 128 (round half to even, as .NET MathF.Round), q = clamp(round(w/s)+z);
a constant row uses s = max(|min|, 1e-12)/127, z = 0.  bf16 rounding is round-to-nearest-even with NaN kept.
"""
from __future__ import annotations

import enum

import struct

import numpy as np
import torch

from ..pc.layer import Layer

_HDR = struct.Struct("<iiffff BB 2x")
PRECISIONS = ("float32", "half", "bfloat16", "int8")


class WeightStoragePrecision(str, enum.Enum):
    """Stored weight precision (Model/WeightStoragePrecision.cs:12); members compare equal to the strings
    accepted everywhere a precision is taken."""
    FLOAT32 = "float32"
    HALF = "half"
    BFLOAT16 = "bfloat16"
    INT8 = "int8"
_FLAG = {"float32": 0, "half": 4, "bfloat16": 8, "int8": 16}


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns, NaN preserved (Core/TensorUtils.cs:379-393)."""
    bits = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = np.uint32(0x7FFF) + ((bits >> np.uint32(16)) & np.uint32(1))
    out = ((bits + rounding) >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out[nan] = ((bits[nan] >> np.uint32(16)) | np.uint32(0x0040)).astype(np.uint16)
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << np.uint32(16)).view(np.float32)


def quantize_int8_rows(w: np.ndarray):
    rows = w.shape[0]
    scales = np.empty(rows, np.float32)
    zeros = np.empty(rows, np.int8)
    codes = np.empty(w.shape, np.int8)
    for r in range(rows):
        row = w[r].astype(np.float32)
        mn, mx = np.float32(row.min()), np.float32(row.max())
        if mx - mn < np.float32(1e-12):
            s = np.float32(max(abs(float(mn)), 1e-12) / 127.0)
            z = 0
        else:
            s = np.float32((mx - mn) / np.float32(255.0))
            z = int(np.clip(int(np.rint(-mn / s)) - 128, -128, 127))
        scales[r] = s
        zeros[r] = z
        codes[r] = np.clip(np.rint(row / s).astype(np.int64) + z, -128, 127).astype(np.int8)
    return scales, zeros, codes


def dequantize_int8_rows(scales, zeros, codes) -> np.ndarray:
    return ((codes.astype(np.float32) - zeros.astype(np.float32)[:, None]) * scales[:, None]).astype(np.float32)


def byte_length(size: int, lower: int, has_diag: bool, has_prior: bool, precision: str = "float32") -> int:
    n = 28 + size * 8
    if lower > 0:
        n += {"half": lower * size * 2, "bfloat16": lower * size * 2,
              "int8": lower * 4 + lower + lower * size}.get(precision, lower * size * 4)
        n += lower * 12
    if has_diag:
        n += size * 4
    if has_prior:
        n += size * 4
    return n


def _f32(t) -> bytes:
    return np.ascontiguousarray(t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else t,
                                dtype="<f4").tobytes()


def serialize(layer: Layer, precision: str = "float32") -> bytes:
    if precision not in PRECISIONS:
        raise ValueError(f"precision must be one of {PRECISIONS}")
    if layer.lower_size == 0:
        precision = "float32"
    has_diag = layer.diag_precision is not None
    has_prior = layer.prior_mean is not None
    flags = (1 if has_diag else 0) | (2 if has_prior else 0) | _FLAG[precision]
    out = bytearray(_HDR.pack(layer.size, layer.lower_size, layer.precision, layer.weight_decay, layer.state_lr,
                              layer.weight_lr, 1 if layer.is_clamped else 0, flags))
    out += _f32(layer.mu)
    out += _f32(layer.eps)
    if layer.lower_size > 0:
        W = layer.W.detach().cpu().float().numpy()
        if precision == "half":
            out += W.astype("<f2").tobytes()
        elif precision == "bfloat16":
            out += f32_to_bf16_bits(W).astype("<u2").tobytes()
        elif precision == "int8":
            s, z, q = quantize_int8_rows(W)
            out += s.astype("<f4").tobytes() + z.tobytes() + q.tobytes()
        else:
            out += W.astype("<f4").tobytes()
        pre = layer.pre if layer.pre is not None else torch.zeros(layer.lower_size)
        pred = layer.pred if layer.pred is not None else torch.zeros(layer.lower_size)
        out += _f32(layer.b) + _f32(pre) + _f32(pred)
    if has_diag:
        out += _f32(layer.diag_precision)
    if has_prior:
        out += _f32(layer.prior_mean)
    assert len(out) == byte_length(layer.size, layer.lower_size, has_diag, has_prior, precision)
    return bytes(out)


def deserialize(buf: bytes, index: int, activation: str) -> Layer:
    size, lower, prec, wd, slr, wlr, clamped, flags = _HDR.unpack_from(buf, 0)
    pos = 28

    def take_f32(n):
        nonlocal pos
        a = np.frombuffer(buf, dtype="<f4", count=n, offset=pos).astype(np.float32)
        pos += 4 * n
        return torch.from_numpy(a.copy())

    L = Layer(index, size, lower, activation, slr, wlr, wd, prec, bool(clamped))
    L.mu = take_f32(size)
    L.eps = take_f32(size)
    if lower > 0:
        n = lower * size
        if flags & 4:
            h = np.frombuffer(buf, dtype="<f2", count=n, offset=pos)
            pos += 2 * n
            L.W_half = torch.from_numpy(h.astype(np.float16).reshape(lower, size).copy())
            L.W = L.W_half.float()
        elif flags & 8:
            b = np.frombuffer(buf, dtype="<u2", count=n, offset=pos)
            pos += 2 * n
            L.W = torch.from_numpy(bf16_bits_to_f32(b).reshape(lower, size).copy())
        elif flags & 16:
            s = np.frombuffer(buf, dtype="<f4", count=lower, offset=pos)
            pos += 4 * lower
            z = np.frombuffer(buf, dtype=np.int8, count=lower, offset=pos)
            pos += lower
            q = np.frombuffer(buf, dtype=np.int8, count=n, offset=pos).reshape(lower, size)
            pos += n
            L.W = torch.from_numpy(dequantize_int8_rows(s, z, q))
        else:
            L.W = take_f32(n).view(lower, size)
        L.b = take_f32(lower)
        L.pre = take_f32(lower)
        L.pred = take_f32(lower)
    if flags & 1:
        L.diag_precision = take_f32(size)
    if flags & 2:
        L.prior_mean = take_f32(size)
    return L
