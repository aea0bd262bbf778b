"""Layer store of a PC network: in-memory layers with optional on-disk persistence.

Reference: PredicitiveCoding/Model/LayerStore.cs:45-371 keeps one record per layer in
a FASTER key-value log (key = layer index, value = LayerSerializer record), with
eager or lazy persistence and recover-on-open.  Here the records are the same
LayerSerializer bytes; on disk they live in a FASTER-format hybrid log
(``io.faster``) under ``path`` (``layers.log`` + ``checkpoints/``), written on every
write (eager) or on ``flush`` (lazy), and recovered when a store is opened on an
existing path.
"""
from __future__ import annotations

import os
import threading
from typing import List, Optional

from ..io import layer_serializer as ser
from .layer import Layer


def page_size_bits(layer_sizes) -> int:
    """LayerStore.cs:354-369: the smallest page (>= 2^22 bytes) that holds the largest layer record
    plus ~32 bytes of record header, for records without diagonal precision or prior."""
    biggest = 0
    for l, size in enumerate(layer_sizes):
        lower = layer_sizes[l - 1] if l > 0 else 0
        biggest = max(biggest, ser.byte_length(size, lower, False, False))
    bits = 22
    while (1 << bits) < biggest + 32:
        bits += 1
    return bits


def _open_kv(path: str, sizes, page_bits: int = 0, segment_bits: int = 0) -> "object":
    from ..io.faster import DEFAULT_SEGMENT_BITS, FasterKV
    if page_bits:
        return FasterKV(os.path.join(path, "layers.log"), os.path.join(path, "checkpoints"), page_bits=page_bits,
                        segment_bits=segment_bits or max(DEFAULT_SEGMENT_BITS, page_bits))
    # records with a diagonal precision or prior are larger than the reference's sizing assumes:
    # grow the page until the largest possible record fits
    bits = page_size_bits(sizes)
    biggest = max(ser.byte_length(s, sizes[l - 1] if l else 0, True, True) for l, s in enumerate(sizes))
    while (1 << bits) < biggest + 40:
        bits += 1
    return FasterKV(os.path.join(path, "layers.log"), os.path.join(path, "checkpoints"), page_bits=bits)


class LayerStore:
    def __init__(self, layers: List[Layer], path: Optional[str] = None, lazy: bool = False, page_bits: int = 0,
                 segment_bits: int = 0):
        """``page_bits`` / ``segment_bits`` override the log geometry (0 = the reference's sizing:
        pages just large enough for the largest layer, 1 GiB segments)."""
        self._layers = [L.clone() for L in layers]
        self._dirty = set()
        self._lock = threading.RLock()
        self.path = path
        self.lazy = lazy
        self._kv = None
        self._quantized = {}
        if path is not None:
            os.makedirs(path, exist_ok=True)
            self._kv = _open_kv(path, [L.size for L in self._layers], page_bits, segment_bits)
            if self._kv.count() > 0:
                self._recover()
            else:
                for i in range(len(self._layers)):
                    self._persist(i)
                self._kv.checkpoint()

    @classmethod
    def open(cls, path: str, activation: str, lazy: bool = False, page_bits: int = 0,
             segment_bits: int = 0) -> "LayerStore":
        """Recover a store written earlier at ``path`` (``page_bits`` 0 = find the page size from the log)."""
        from ..io.faster import DEFAULT_SEGMENT_BITS, FasterKV, probe_page_bits
        bits = page_bits or probe_page_bits(os.path.join(path, "layers.log"))
        kv = FasterKV(os.path.join(path, "layers.log"), os.path.join(path, "checkpoints"), page_bits=bits,
                      segment_bits=segment_bits or max(DEFAULT_SEGMENT_BITS, bits))
        recs = kv.items()
        layers = [ser.deserialize(recs[k], k, activation) for k in sorted(recs)]
        st = cls.__new__(cls)
        st._layers, st._dirty, st._lock = layers, set(), threading.RLock()
        st.path, st.lazy, st._kv, st._quantized = path, lazy, kv, {}
        return st

    def _recover(self) -> None:
        recs = self._kv.items()
        act = self._layers[0].activation
        for k, buf in recs.items():
            if 0 <= k < len(self._layers):
                self._layers[k] = ser.deserialize(buf, k, act)

    def _persist(self, i: int) -> None:
        prec = self._quantized.get(i, "float32")
        self._kv.upsert(i, ser.serialize(self._layers[i], prec))

    def read(self, i: int) -> Layer:
        with self._lock:
            return self._layers[i].clone()

    def write(self, i: int, layer: Layer) -> None:
        with self._lock:
            self._layers[i] = layer.clone()
            self._layers[i].W_half = None if i not in self._quantized else self._layers[i].W_half
            if self._kv is not None:
                if self.lazy:
                    self._dirty.add(i)
                else:
                    self._persist(i)

    def write_quantized(self, i: int, layer: Layer, precision: str) -> None:
        """Persist layer ``i`` with its weights rounded to ``precision``; the live copy is rounded too."""
        with self._lock:
            rec = ser.serialize(layer, precision)
            q = ser.deserialize(rec, i, layer.activation)
            self._layers[i] = q
            if precision != "float32":
                self._quantized[i] = precision
            else:
                self._quantized.pop(i, None)
            if self._kv is not None:
                self._kv.upsert(i, rec)

    def flush(self) -> None:
        with self._lock:
            if self._kv is None:
                return
            for i in sorted(self._dirty):
                self._persist(i)
            self._dirty.clear()
            self._kv.checkpoint()

    def close(self) -> None:
        if self._kv is not None:
            self.flush()
            self._kv.close()
            self._kv = None

    def __len__(self) -> int:
        return len(self._layers)
