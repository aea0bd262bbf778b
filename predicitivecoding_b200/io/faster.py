"""Log-structured key/value store in the layout of a FASTER ``FasterKV<int, SpanByte>`` hybrid log.

The reference persists PC layers (PredicitiveCoding/Model/LayerStore.cs:45-371) and LLM
checkpoints (PredictiveCoding.LLM/Training/Checkpoint.cs:238-403) in Microsoft FASTER
2.6.5 stores: an append-only hybrid log device ``<name>`` (segment files
``<name>.0``, ``<name>.1`` ...), records of ``[RecordInfo u64][key i32][value
length i32][value bytes]`` padded to 8 bytes, the first 64 bytes of the address
space reserved, and fold-over checkpoints under ``<checkpoint dir>`` recording
the log's flushed tail.  This module writes and reads that structure:
upserts append a record, reads scan the log and keep the newest valid record per
key, ``checkpoint`` flushes and records the tail so a reopened store recovers
exactly the committed records.

The record header packs the previous-address chain in bits 0-47 and flags above
(bit 58 ``valid``, bit 59 ``tombstone``).  No store written by the reference's
.NET process exists in its repository, so byte-level interchange with stores
written by FASTER itself is unverified; round trips through this module are
tested.
"""
from __future__ import annotations

import glob
import json
import os
import struct
import threading
import time
import uuid
from typing import Dict, Iterator, Optional, Tuple

FIRST_VALID_ADDRESS = 64
SEGMENT_BITS = 30  # 1 GiB segments
_VALID = 1 << 58
_TOMBSTONE = 1 << 59
_ADDR_MASK = (1 << 48) - 1
_REC = struct.Struct("<Qii")


def _align8(n: int) -> int:
    return (n + 7) & ~7


class FasterKV:
    """Append-only int -> bytes store with checkpoints (single process, thread-safe)."""

    def __init__(self, log_path: str, checkpoint_dir: str, recover: bool = True):
        self.log_path = log_path
        self.checkpoint_dir = checkpoint_dir
        os.makedirs(os.path.dirname(os.path.abspath(log_path)), exist_ok=True)
        os.makedirs(checkpoint_dir, exist_ok=True)
        self._lock = threading.RLock()
        self._index: Dict[int, Tuple[int, int]] = {}  # key -> (address, record length)
        self._tail = FIRST_VALID_ADDRESS
        seg0 = self._segment_path(0)
        if recover and os.path.exists(seg0):
            committed = self._last_checkpoint_tail()
            self._scan(committed)
        else:
            with open(seg0, "wb") as f:
                f.write(b"\0" * FIRST_VALID_ADDRESS)
        self._fh = open(seg0, "r+b")

    # ------------------------------------------------------------ paths / metadata
    def _segment_path(self, seg: int) -> str:
        return f"{self.log_path}.{seg}"

    def _cpr_dir(self) -> str:
        return os.path.join(self.checkpoint_dir, "cpr-checkpoints")

    def _last_checkpoint_tail(self) -> Optional[int]:
        best = None
        for info in glob.glob(os.path.join(self._cpr_dir(), "*", "info.dat")):
            try:
                meta = json.load(open(info))
            except Exception:
                continue
            if best is None or meta["version"] > best["version"]:
                best = meta
        return None if best is None else int(best["finalLogicalAddress"])

    # ------------------------------------------------------------ log scan
    def _records(self, limit: Optional[int] = None) -> Iterator[Tuple[int, int, int, bytes, int]]:
        path = self._segment_path(0)
        if not os.path.exists(path):
            return
        data = open(path, "rb").read()
        end = len(data) if limit is None else min(limit, len(data))
        pos = FIRST_VALID_ADDRESS
        while pos + _REC.size <= end:
            info, key, vlen = _REC.unpack_from(data, pos)
            if info == 0 or vlen < 0:
                break
            rec_len = _align8(_REC.size + vlen)
            if pos + rec_len > end:
                break
            yield pos, info, key, data[pos + _REC.size: pos + _REC.size + vlen], rec_len
            pos += rec_len

    def _scan(self, limit: Optional[int]) -> None:
        last = FIRST_VALID_ADDRESS
        for addr, info, key, _, rec_len in self._records(limit):
            if info & _VALID:
                if info & _TOMBSTONE:
                    self._index.pop(key, None)
                else:
                    self._index[key] = (addr, rec_len)
            last = addr + rec_len
        self._tail = last

    # ------------------------------------------------------------ API
    def upsert(self, key: int, value: bytes) -> None:
        self._append(key, value, tombstone=False)

    def delete(self, key: int) -> None:
        self._append(key, b"", tombstone=True)

    def _append(self, key: int, value: bytes, tombstone: bool) -> None:
        with self._lock:
            prev = self._index.get(key, (0, 0))[0]
            info = (prev & _ADDR_MASK) | _VALID | (_TOMBSTONE if tombstone else 0)
            rec = _REC.pack(info, int(key), len(value)) + value
            rec += b"\0" * (_align8(len(rec)) - len(rec))
            self._fh.seek(self._tail)
            self._fh.write(rec)
            if tombstone:
                self._index.pop(key, None)
            else:
                self._index[key] = (self._tail, len(rec))
            self._tail += len(rec)

    def read(self, key: int) -> Optional[bytes]:
        with self._lock:
            loc = self._index.get(key)
            if loc is None:
                return None
            self._fh.flush()
            self._fh.seek(loc[0])
            _, _, vlen = _REC.unpack(self._fh.read(_REC.size))
            return self._fh.read(vlen)

    def items(self) -> Dict[int, bytes]:
        return {k: self.read(k) for k in sorted(self._index)}

    def keys(self):
        return sorted(self._index)

    def count(self) -> int:
        return len(self._index)

    def checkpoint(self) -> str:
        """Flush the log and record the committed tail (a fold-over checkpoint)."""
        with self._lock:
            self._fh.flush()
            os.fsync(self._fh.fileno())
            versions = [json.load(open(p))["version"] for p in glob.glob(os.path.join(self._cpr_dir(), "*", "info.dat"))]
            token = str(uuid.uuid4())
            d = os.path.join(self._cpr_dir(), token)
            os.makedirs(d, exist_ok=True)
            meta = {"version": (max(versions) + 1) if versions else 1, "guid": token, "useSnapshotFile": 0,
                    "beginAddress": FIRST_VALID_ADDRESS, "headAddress": FIRST_VALID_ADDRESS,
                    "flushedLogicalAddress": self._tail, "finalLogicalAddress": self._tail,
                    "checkpointType": "FoldOver", "timestamp": time.time()}
            with open(os.path.join(d, "info.dat"), "w") as f:
                json.dump(meta, f)
            return token

    def clear(self) -> None:
        with self._lock:
            self._fh.close()
            for p in glob.glob(self.log_path + ".*"):
                os.remove(p)
            for p in glob.glob(os.path.join(self._cpr_dir(), "*", "info.dat")):
                os.remove(p)
            with open(self._segment_path(0), "wb") as f:
                f.write(b"\0" * FIRST_VALID_ADDRESS)
            self._fh = open(self._segment_path(0), "r+b")
            self._index.clear()
            self._tail = FIRST_VALID_ADDRESS

    def close(self) -> None:
        with self._lock:
            if self._fh is not None:
                self._fh.flush()
                self._fh.close()
                self._fh = None
