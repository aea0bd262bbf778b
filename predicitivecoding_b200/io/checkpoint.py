"""LLM checkpoint formats.

* Tensor blob (PredictiveCoding.LLM/Training/Checkpoint.cs:86-173):
  ``[int32 rows][int32 cols][uint8 precision][data]`` with precision 0 fp32, 1 fp16,
  2 bf16 (round-to-nearest-even), 3 int8 per-row "min + scale" (float scales[rows],
  float mins[rows], int8 codes: q = clamp(round((w-min)/s) - 128), w = (q+128) s + min).
* Model store (PredictiveLlm.cs:630-771): one FASTER-layout key/value store under a
  directory, plus a 4-byte ``pagesize`` hint file.  Keys: 0..N-1 tensors in
  ``Parameters()`` order; -100 format version (int 1); -1 config JSON; -2 tokenizer
  manifest JSON; -3 BPE header ``[u8 word_split][i32 vocab][i32 merges]``; 4_000_000+m one
  merge ``(a, b, id)`` per record; -4 odometer JSON; -5 memory header ``[key_dim][capacity]
  [count]``; 3_000_000+i one memory entry ``[key f32 * dim][i32 len][utf8]``; -6 online-Adam
  step; 1_000_000+i / 2_000_000+i online-Adam moments m / v (fp32).
* ``optimizer.bin`` "OPT1" (OptimizerCheckpoint.cs:18-76): magic 0x4F505431, int32 t,
  int32 count, then per parameter ``[int32 len][m f32 * len][v f32 * len]``.
* ``adam-device.bin`` "DAM1" (DeviceDecoderTrainer.cs:503-543): magic 0x44414D31, int32 t,
  then per parameter in the device-packed order (wemb; per block G1, Wq, Wk, Wv, Wo, G2,
  W1, B1, W2, B2; gF; wout) ``[int32 count][m f32][v f32]``.
* Legacy "LLM1" (magic 0x4C4C4D31): ``int32 count`` then per tensor ``[rows][cols][f32...]``.
"""
from __future__ import annotations

import json
import os
import struct
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from .faster import FasterKV
from .layer_serializer import bf16_bits_to_f32, f32_to_bf16_bits

PRECISION_CODES = {"float32": 0, "half": 1, "bfloat16": 2, "int8": 3}
PRECISION_NAMES = {v: k for k, v in PRECISION_CODES.items()}

FORMAT_VERSION = 1
VERSION_KEY = -100
CONFIG_KEY = -1
TOKENIZER_MANIFEST_KEY = -2
TOKENIZER_HEADER_KEY = -3
ODOMETER_KEY = -4
MEMORY_HEADER_KEY = -5
OPTIMIZER_STEP_KEY = -6
MOMENT_M_BASE = 1_000_000
MOMENT_V_BASE = 2_000_000
MEMORY_ENTRY_BASE = 3_000_000
MERGE_BASE = 4_000_000
PAGE_SIZE_HINT = "pagesize"
LOG_NAME = "weights.log"
OPT1_MAGIC = 0x4F505431
DAM1_MAGIC = 0x44414D31
LLM1_MAGIC = 0x4C4C4D31


def _as2d(t: torch.Tensor) -> np.ndarray:
    a = t.detach().float().cpu().numpy()
    return a.reshape(1, -1) if a.ndim == 1 else a.reshape(a.shape[0], -1)


def tensor_blob(t: torch.Tensor, precision: str = "float32") -> bytes:
    a = _as2d(t)
    rows, cols = a.shape
    head = struct.pack("<iiB", rows, cols, PRECISION_CODES[precision])
    if precision == "float32":
        return head + a.astype("<f4").tobytes()
    if precision == "half":
        return head + a.astype("<f2").tobytes()
    if precision == "bfloat16":
        return head + f32_to_bf16_bits(a).astype("<u2").tobytes()
    scales = np.empty(rows, np.float32)
    mins = np.empty(rows, np.float32)
    codes = np.empty((rows, cols), np.int8)
    for r in range(rows):
        mn, mx = np.float32(a[r].min()), np.float32(a[r].max())
        s = np.float32(1e-12) if mx - mn < np.float32(1e-12) else np.float32((mx - mn) / np.float32(255.0))
        scales[r], mins[r] = s, mn
        codes[r] = np.clip(np.rint((a[r] - mn) / s).astype(np.int64) - 128, -128, 127).astype(np.int8)
    return head + scales.astype("<f4").tobytes() + mins.astype("<f4").tobytes() + codes.tobytes()


def read_tensor_blob(b: bytes) -> Tuple[np.ndarray, str]:
    rows, cols, code = struct.unpack_from("<iiB", b, 0)
    pos = 9
    n = rows * cols
    prec = PRECISION_NAMES[code]
    if prec == "float32":
        a = np.frombuffer(b, "<f4", n, pos)
    elif prec == "half":
        a = np.frombuffer(b, "<f2", n, pos).astype(np.float32)
    elif prec == "bfloat16":
        a = bf16_bits_to_f32(np.frombuffer(b, "<u2", n, pos))
    else:
        scales = np.frombuffer(b, "<f4", rows, pos)
        mins = np.frombuffer(b, "<f4", rows, pos + 4 * rows)
        codes = np.frombuffer(b, np.int8, n, pos + 8 * rows).reshape(rows, cols)
        a = (codes.astype(np.float32) + 128.0) * scales[:, None] + mins[:, None]
    return np.array(a, dtype=np.float32).reshape(rows, cols), prec


def page_size_bits_for(max_payload_len: int) -> int:
    """Checkpoint.cs:215-221: record = payload + 4 (length prefix) + 32 (header); >= 22 bits."""
    rec = max_payload_len + 4 + 32
    bits = 22
    while (1 << bits) < rec:
        bits += 1
    return bits


class CheckpointStore:
    """Keyed blob store over a directory (``weights.log`` + ``checkpoints/``)."""

    def __init__(self, directory: str, page_size_bits: int = 22, recover: bool = True, segment_bits: int = 0):
        os.makedirs(directory, exist_ok=True)
        self.dir = directory
        self.page_size_bits = page_size_bits
        self.kv = FasterKV(os.path.join(directory, LOG_NAME), os.path.join(directory, "checkpoints"), recover=recover,
                           page_bits=page_size_bits, segment_bits=segment_bits or max(30, page_size_bits))

    def put_blob(self, key: int, data: bytes) -> None:
        self.kv.upsert(key, bytes(data))

    def get_blob(self, key: int) -> Optional[bytes]:
        return self.kv.read(key)

    def upsert_tensor(self, key: int, t: torch.Tensor, precision: str = "float32") -> None:
        self.put_blob(key, tensor_blob(t, precision))

    def commit(self) -> None:
        self.kv.checkpoint()

    def close(self) -> None:
        self.kv.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def save_parameters(directory: str, tensors: Sequence[torch.Tensor], precision: str = "float32") -> None:
    """Parameters only, keys 0..N-1 (the plain ``Checkpoint.Save(dir, params)`` layout)."""
    blobs = [tensor_blob(t, precision) for t in tensors]
    bits = page_size_bits_for(max((len(b) for b in blobs), default=0))
    clear_store(directory)
    os.makedirs(directory, exist_ok=True)
    write_page_size_hint(directory, bits)
    with CheckpointStore(directory, bits, recover=False) as st:
        for i, b in enumerate(blobs):
            st.put_blob(i, b)
        st.commit()


def load_parameters(directory: str) -> List[torch.Tensor]:
    bits = read_page_size_hint(directory)
    out = []
    with CheckpointStore(directory, bits, recover=True) as st:
        i = 0
        while (b := st.get_blob(i)) is not None:
            out.append(torch.from_numpy(read_tensor_blob(b)[0].copy()))
            i += 1
    return out


def clear_store(directory: str) -> None:
    import glob
    import shutil
    for f in glob.glob(os.path.join(directory, LOG_NAME + "*")):
        os.remove(f)
    shutil.rmtree(os.path.join(directory, "checkpoints"), ignore_errors=True)


def write_page_size_hint(directory: str, bits: int) -> None:
    with open(os.path.join(directory, PAGE_SIZE_HINT), "wb") as f:
        f.write(struct.pack("<i", bits))


def read_page_size_hint(directory: str) -> int:
    p = os.path.join(directory, PAGE_SIZE_HINT)
    if not os.path.exists(p):
        raise FileNotFoundError(f"No LLM checkpoint found under '{directory}' (missing page-size hint).")
    b = open(p, "rb").read()
    if len(b) < 4:
        raise ValueError(f"Corrupt page-size hint under '{directory}'.")
    return struct.unpack("<i", b[:4])[0]


def is_checkpoint(directory: str) -> bool:
    """A saved model is recognised by its own format marker (the page-size hint + version record)."""
    try:
        bits = read_page_size_hint(directory)
        with CheckpointStore(directory, bits) as st:
            v = st.get_blob(VERSION_KEY)
            return v is not None and struct.unpack("<i", v[:4])[0] == FORMAT_VERSION
    except Exception:
        return False


# --------------------------------------------------------------------------- OPT1 / DAM1 / LLM1
def save_opt1(path: str, params: Sequence[torch.Tensor], t: int, moments: Sequence[Optional[Tuple]]) -> None:
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    with open(path, "wb") as f:
        f.write(struct.pack("<Iii", OPT1_MAGIC, int(t), len(params)))
        for p, mv in zip(params, moments):
            n = p.numel()
            m = np.zeros(n, np.float32) if mv is None else mv[0].detach().float().cpu().numpy().reshape(-1)
            v = np.zeros(n, np.float32) if mv is None else mv[1].detach().float().cpu().numpy().reshape(-1)
            f.write(struct.pack("<i", n))
            f.write(m.astype("<f4").tobytes())
            f.write(v.astype("<f4").tobytes())


def load_opt1(path: str, params: Sequence[torch.Tensor]):
    b = open(path, "rb").read()
    magic, t, count = struct.unpack_from("<Iii", b, 0)
    if magic != OPT1_MAGIC:
        raise ValueError(f"'{path}' is not an optimizer checkpoint.")
    if count != len(params):
        raise ValueError(f"Optimizer checkpoint has {count} parameters; model has {len(params)}.")
    pos = 12
    out = []
    for i, p in enumerate(params):
        n = struct.unpack_from("<i", b, pos)[0]
        pos += 4
        if n != p.numel():
            raise ValueError(f"Optimizer moment length {n} != parameter {i} length {p.numel()}.")
        m = np.frombuffer(b, "<f4", n, pos).copy()
        pos += 4 * n
        v = np.frombuffer(b, "<f4", n, pos).copy()
        pos += 4 * n
        out.append((torch.from_numpy(m).view_as(p.detach().cpu()), torch.from_numpy(v).view_as(p.detach().cpu())))
    return t, out


def save_dam1(path: str, t: int, moments: Sequence[Tuple[np.ndarray, np.ndarray]]) -> None:
    with open(path, "wb") as f:
        f.write(struct.pack("<Ii", DAM1_MAGIC, int(t)))
        for m, v in moments:
            m = np.asarray(m, np.float32).reshape(-1)
            v = np.asarray(v, np.float32).reshape(-1)
            f.write(struct.pack("<i", m.size))
            f.write(m.astype("<f4").tobytes())
            f.write(v.astype("<f4").tobytes())


def load_dam1(path: str, counts: Sequence[int]):
    b = open(path, "rb").read()
    magic, t = struct.unpack_from("<Ii", b, 0)
    if magic != DAM1_MAGIC:
        raise ValueError("Not a device Adam state file.")
    pos = 8
    out = []
    for c in counts:
        n = struct.unpack_from("<i", b, pos)[0]
        pos += 4
        if n != c:
            raise ValueError(f"Adam state shape mismatch: {n} vs {c}.")
        m = np.frombuffer(b, "<f4", n, pos).copy()
        pos += 4 * n
        v = np.frombuffer(b, "<f4", n, pos).copy()
        pos += 4 * n
        out.append((m, v))
    return t, out


def read_llm1(path: str) -> List[np.ndarray]:
    """Legacy flat checkpoint: magic "LLM1", int32 count, then [rows][cols][f32...] per tensor."""
    b = open(path, "rb").read()
    magic, count = struct.unpack_from("<Ii", b, 0)
    if magic != LLM1_MAGIC:
        raise ValueError("Not an LLM1 checkpoint.")
    pos = 8
    out = []
    for _ in range(count):
        rows, cols = struct.unpack_from("<ii", b, pos)
        pos += 8
        a = np.frombuffer(b, "<f4", rows * cols, pos).reshape(rows, cols).copy()
        pos += 4 * rows * cols
        out.append(a)
    return out


def write_llm1(path: str, tensors: Sequence[torch.Tensor]) -> None:
    with open(path, "wb") as f:
        f.write(struct.pack("<Ii", LLM1_MAGIC, len(tensors)))
        for t in tensors:
            a = _as2d(t)
            f.write(struct.pack("<ii", *a.shape))
            f.write(a.astype("<f4").tobytes())
