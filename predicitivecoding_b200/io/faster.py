"""Key/value store in the on-disk layout of a FASTER 2.x ``FasterKV<int, SpanByte>``.

The reference persists PC layers (PredicitiveCoding/Model/LayerStore.cs:100-131, 320-340) and LLM
checkpoints (PredictiveCoding.LLM/Training/Checkpoint.cs:238-403) in Microsoft FASTER 2.6.5 stores
created with ``Devices.CreateLogDevice(<dir>/<name>.log)``, ``LogSettings.PageSizeBits`` sized so the
largest record fits one page, an index of ``1 << 20`` hash buckets, and full fold-over checkpoints
(``TakeFullCheckpointAsync(CheckpointType.FoldOver)``).  This module writes and reads that layout:

Hybrid log (FASTER ``Allocator/VarLenBlittableAllocator.cs``, ``Device/LocalStorageDevice.cs``)
    A logical address space split into segment files ``<log>.<n>`` of ``1 << segment_bits`` bytes
    (address >> segment_bits picks the file).  Addresses below 64 are reserved (the begin address
    is 64).  Pages are ``1 << page_bits`` bytes and no record crosses a page: a record that does not
    fit the rest of its page starts the next page, and the skipped bytes stay zero.  A record is
    ``RecordInfo`` (8 bytes) | key (int32, padded to 8) | SpanByte value (int32 length + payload),
    the whole rounded up to 8 bytes.

RecordInfo (``Index/Common/RecordInfo.cs``)
    bits 0-47 previous address in the hash chain (bit 47 marks the read cache), 48-54 spare,
    55 tombstone, 56 valid, 57 sealed, 58 tentative, 59 dirty, 60 filler, 61 in-new-version,
    62 modified.  A word of zero marks the unused tail of a page.

Index (``Index/Common/HashBucket.cs``, ``Index/FASTER/FASTERBase.cs``)
    ``size`` buckets of 8 words; words 0-6 are entries (address bits 0-47, 14-bit tag bits 48-61,
    pending 62, tentative 63), word 7 the overflow-bucket pointer.  A key hashes with FASTER's
    64-bit integer hash (``Utilities/Utility.cs`` ``GetHashCode(long)``): bucket = hash & (size-1),
    tag = hash >> 50.  Records chain per (bucket, tag), newest first.

Checkpoints (``Index/Recovery/Checkpoint.cs``, ``Index/CheckpointManagement/DefaultCheckpointNamingScheme.cs``,
``DeviceLogCommitCheckpointManager.cs``)
    ``<ckpt>/index-checkpoints/<token>/{info.dat, ht.dat, ofb.dat}`` and
    ``<ckpt>/cpr-checkpoints/<token>/info.dat``.  Each ``info.dat`` is an int32 byte count followed by
    the recovery-info text (one value per line) and zero padding to a 512-byte sector.  The log
    recovery info carries, in order: format version, checksum, token, use-snapshot flag, version,
    next version, flushed / start / final / snapshot-final logical address, head, begin and
    delta-tail address, manual-locking flag, session count (and per-session lines), object-log
    segment count.  The index info: token, table size, hash-table bytes, overflow bytes, bucket
    count, start and final logical address.

Recovery picks the cpr checkpoint with the highest version and rebuilds the index by scanning the
log up to its final logical address (the same records the saved index points at); the reader also
accepts the JSON ``info.dat`` that earlier versions of this package wrote.  No store written by the
reference's .NET process exists in its repository, so byte-level interchange with FASTER itself
rests on the structures above, not on a test against FASTER-written files.
"""
from __future__ import annotations

import glob
import json
import os
import struct
import threading
import uuid
from typing import Dict, Iterator, List, Optional, Tuple

FIRST_VALID_ADDRESS = 64
DEFAULT_SEGMENT_BITS = 30          # 1 GiB segment files (LogSettings.SegmentSizeBits default)
DEFAULT_PAGE_BITS = 22
DEFAULT_INDEX_BUCKETS = 1 << 20    # the reference's FasterKV(size: 1L << 20)
SECTOR = 512
LOG_CHECKPOINT_FORMAT = 5

_ADDR_MASK = (1 << 48) - 1
_TOMBSTONE = 1 << 55
_VALID = 1 << 56
_TAG_BITS = 14
_TAG_SHIFT_ENTRY = 48
_TAG_SHIFT_HASH = 64 - _TAG_BITS
_ENTRIES = 7                       # entries per bucket (word 7 is the overflow pointer)
_M64 = (1 << 64) - 1


def _align8(n: int) -> int:
    return (n + 7) & ~7


def _s64(x: int) -> int:
    x &= _M64
    return x - (1 << 64) if x >> 63 else x


def key_hash(key: int) -> int:
    """FASTER's 64-bit integer hash (16-bit limbs folded with multiplier 40343, then rotated right 45)."""
    x = key & _M64
    h = 8
    h = (40343 * h + (x & 0xFFFF)) & _M64
    h = (40343 * h + ((x >> 16) & 0xFFFF)) & _M64
    h = (40343 * h + ((x >> 32) & 0xFFFF)) & _M64
    h = (40343 * h + (x >> 48)) & _M64
    h = (40343 * h) & _M64
    return ((h >> 45) | (h << 19)) & _M64


def record_size(value_len: int) -> int:
    """RecordInfo + key (int32 padded to 8) + SpanByte (int32 length + payload), rounded to 8."""
    return 8 + 8 + _align8(4 + value_len)


def _sector_blob(text: str) -> bytes:
    body = text.encode("utf-8")
    raw = struct.pack("<i", len(body)) + body
    return raw + b"\0" * (-len(raw) % SECTOR)


def _read_sector_blob(path: str) -> Optional[List[str]]:
    data = open(path, "rb").read()
    if len(data) >= 4:
        n = struct.unpack_from("<i", data)[0]
        if 0 < n <= len(data) - 4:
            try:
                return data[4:4 + n].decode("utf-8").splitlines()
            except UnicodeDecodeError:
                return None
    return None


def _guid_longs(token: str) -> Tuple[int, int]:
    """The two int64 halves of a .NET Guid's byte order (first three fields little-endian)."""
    b = uuid.UUID(token).bytes_le
    return struct.unpack("<qq", b)


class FasterKV:
    """int -> bytes store over a FASTER-layout hybrid log with full fold-over checkpoints.

    Single process, thread-safe.  ``page_bits`` must be large enough for the largest record (the
    reference sizes it that way, LayerStore.cs:354-369 / Checkpoint.cs:195-221).
    """

    def __init__(self, log_path: str, checkpoint_dir: str, recover: bool = True, page_bits: int = DEFAULT_PAGE_BITS,
                 segment_bits: int = DEFAULT_SEGMENT_BITS, index_buckets: int = DEFAULT_INDEX_BUCKETS):
        if segment_bits < page_bits:
            raise ValueError("segment_bits must be >= page_bits")
        if index_buckets & (index_buckets - 1):
            raise ValueError("index_buckets must be a power of two")
        self.log_path = log_path
        self.checkpoint_dir = checkpoint_dir
        self.page_bits, self.segment_bits, self.index_buckets = page_bits, segment_bits, index_buckets
        self.page_size = 1 << page_bits
        os.makedirs(os.path.dirname(os.path.abspath(log_path)), exist_ok=True)
        os.makedirs(checkpoint_dir, exist_ok=True)
        self._lock = threading.RLock()
        self._files: Dict[int, object] = {}
        self._chain: Dict[Tuple[int, int], int] = {}     # (bucket, tag) -> newest address
        self._index: Dict[int, Tuple[int, int]] = {}     # key -> (address, value length)
        self._tail = FIRST_VALID_ADDRESS
        self.version = 1
        if recover and os.path.exists(self._segment_path(0)):
            meta = self._latest_checkpoint()
            if meta is not None:
                self.version = meta["version"] + 1
                self._scan(meta["final"])
            else:
                self._scan(None)
        else:
            for p in glob.glob(self.log_path + ".*"):
                if p[len(self.log_path) + 1:].isdigit():
                    os.remove(p)

    # ------------------------------------------------------------ segments
    def _segment_path(self, seg: int) -> str:
        return f"{self.log_path}.{seg}"

    def _file(self, seg: int):
        f = self._files.get(seg)
        if f is None:
            p = self._segment_path(seg)
            f = open(p, "r+b") if os.path.exists(p) else open(p, "w+b")
            self._files[seg] = f
        return f

    def _write_at(self, addr: int, data: bytes) -> None:
        seg, off = addr >> self.segment_bits, addr & ((1 << self.segment_bits) - 1)
        f = self._file(seg)
        f.seek(off)
        f.write(data)

    def _read_at(self, addr: int, n: int) -> bytes:
        seg, off = addr >> self.segment_bits, addr & ((1 << self.segment_bits) - 1)
        p = self._segment_path(seg)
        if seg not in self._files and not os.path.exists(p):
            return b""
        f = self._file(seg)
        f.flush()
        f.seek(off)
        return f.read(n)

    # ------------------------------------------------------------ log scan
    def _records(self, limit: Optional[int]) -> Iterator[Tuple[int, int, int, int, int]]:
        """(address, record info, key, value length, record size) of every record below ``limit``."""
        addr = FIRST_VALID_ADDRESS
        while limit is None or addr < limit:
            room = self.page_size - (addr & (self.page_size - 1))
            if room < 24:
                addr += room
                continue
            head = self._read_at(addr, 20)
            if len(head) < 20:
                if limit is None or not os.path.exists(self._segment_path((addr + room) >> self.segment_bits)):
                    return
                addr += room                   # a short segment file: its last page tail was never written
                continue
            info, key, vlen = struct.unpack_from("<Qi4xi", head)
            if info == 0:                      # unused tail of the page: the next record starts a page
                addr += room
                continue
            size = record_size(vlen)
            if vlen < 0 or size > room:
                return
            yield addr, info, key, vlen, size
            addr += size

    def _scan(self, limit: Optional[int]) -> None:
        end = FIRST_VALID_ADDRESS
        for addr, info, key, vlen, size in self._records(limit):
            end = addr + size
            if not info & _VALID:
                continue
            h = key_hash(key)
            self._chain[(h & (self.index_buckets - 1), h >> _TAG_SHIFT_HASH)] = addr
            if info & _TOMBSTONE:
                self._index.pop(key, None)
            else:
                self._index[key] = (addr, vlen)
        self._tail = end

    # ------------------------------------------------------------ API
    def upsert(self, key: int, value: bytes) -> None:
        self._append(key, bytes(value), tombstone=False)

    def delete(self, key: int) -> None:
        self._append(key, b"", tombstone=True)

    def _append(self, key: int, value: bytes, tombstone: bool) -> None:
        size = record_size(len(value))
        if size > self.page_size:
            raise ValueError(f"record of {size} bytes exceeds the {self.page_size}-byte page (raise page_bits)")
        with self._lock:
            room = self.page_size - (self._tail & (self.page_size - 1))
            if size > room:              # the page's unused tail is written as zeros, as a page flush would
                self._write_at(self._tail, b"\0" * room)
                self._tail += room
            h = key_hash(key)
            slot = (h & (self.index_buckets - 1), h >> _TAG_SHIFT_HASH)
            prev = self._chain.get(slot, 0)
            info = (prev & _ADDR_MASK) | _VALID | (_TOMBSTONE if tombstone else 0)
            rec = struct.pack("<Qi4xi", info, int(key), len(value)) + value
            rec += b"\0" * (size - len(rec))
            addr = self._tail
            self._write_at(addr, rec)
            self._chain[slot] = addr
            if tombstone:
                self._index.pop(key, None)
            else:
                self._index[key] = (addr, len(value))
            self._tail = addr + size

    def read(self, key: int) -> Optional[bytes]:
        with self._lock:
            loc = self._index.get(key)
            if loc is None:
                return None
            return self._read_at(loc[0] + 20, loc[1])

    def items(self) -> Dict[int, bytes]:
        return {k: self.read(k) for k in sorted(self._index)}

    def keys(self):
        return sorted(self._index)

    def count(self) -> int:
        return len(self._index)

    @property
    def tail_address(self) -> int:
        return self._tail

    # ------------------------------------------------------------ checkpoints
    def _cpr_dir(self) -> str:
        return os.path.join(self.checkpoint_dir, "cpr-checkpoints")

    def _index_dir(self) -> str:
        return os.path.join(self.checkpoint_dir, "index-checkpoints")

    def _latest_checkpoint(self) -> Optional[dict]:
        best = None
        for info in glob.glob(os.path.join(self._cpr_dir(), "*", "info.dat")):
            meta = self._parse_log_info(info)
            if meta is not None and (best is None or meta["version"] > best["version"]):
                best = meta
        return best

    @staticmethod
    def _parse_log_info(path: str) -> Optional[dict]:
        lines = _read_sector_blob(path)
        try:
            if lines is not None and len(lines) >= 13:
                return {"version": int(lines[4]), "final": int(lines[8]), "token": lines[2].strip()}
            meta = json.load(open(path))            # the JSON form written by earlier versions of this package
            return {"version": int(meta["version"]), "final": int(meta["finalLogicalAddress"]),
                    "token": meta.get("guid", "")}
        except (ValueError, KeyError, OSError, UnicodeDecodeError):
            return None

    def _log_info_text(self, token: str, tail: int) -> str:
        version, begin, head = self.version, FIRST_VALID_ADDRESS, tail    # fold-over: everything flushed
        sessions, object_segments = 0, 0
        lo, hi = _guid_longs(token)
        checksum = _s64(lo ^ hi ^ version ^ tail ^ tail ^ tail ^ head ^ begin ^ sessions ^ object_segments)
        # format, checksum, token, snapshot flag, version, next version, flushed / start / final / snapshot-final
        # address, head, begin, delta tail, manual locking, sessions, object-log segments
        fields = [LOG_CHECKPOINT_FORMAT, checksum, token, 0, version, version + 1, tail, tail, tail,
                  tail, head, begin, -1, "False", sessions, object_segments]
        return "".join(f"{v}\r\n" for v in fields)

    def _write_index_checkpoint(self, token: str, tail: int) -> None:
        d = os.path.join(self._index_dir(), token)
        os.makedirs(d, exist_ok=True)
        buckets: Dict[int, List[Tuple[int, int]]] = {}
        for (b, tag), addr in self._chain.items():
            buckets.setdefault(b, []).append((tag, addr))
        overflow: List[bytes] = []
        ht_bytes = self.index_buckets * 64
        with open(os.path.join(d, "ht.dat"), "wb") as f:
            f.truncate(ht_bytes)                       # sparse: untouched buckets read as zero
            for b, entries in sorted(buckets.items()):
                entries.sort()
                words, chunks = [], [entries[i:i + _ENTRIES] for i in range(0, len(entries), _ENTRIES)]
                for ci, chunk in enumerate(chunks):
                    w = [(addr & _ADDR_MASK) | (tag << _TAG_SHIFT_ENTRY) for tag, addr in chunk]
                    w += [0] * (_ENTRIES - len(w))
                    nxt = len(overflow) + 1 if ci + 1 < len(chunks) else 0   # 1-based overflow bucket
                    block = struct.pack("<8Q", *(w + [nxt]))
                    if ci == 0:
                        words = block
                    else:
                        overflow.append(block)
                f.seek(b * 64)
                f.write(words)
        with open(os.path.join(d, "ofb.dat"), "wb") as f:
            f.write(b"".join(overflow))
        text = "".join(f"{v}\r\n" for v in [token, self.index_buckets, ht_bytes, 64 * len(overflow),
                                             self.index_buckets, FIRST_VALID_ADDRESS, tail])
        with open(os.path.join(d, "info.dat"), "wb") as f:
            f.write(_sector_blob(text))

    def checkpoint(self) -> str:
        """Full fold-over checkpoint: flush the log, write the index and the log recovery info."""
        with self._lock:
            for f in self._files.values():
                f.flush()
                os.fsync(f.fileno())
            token = str(uuid.uuid4())
            tail = self._tail
            self._write_index_checkpoint(token, tail)
            d = os.path.join(self._cpr_dir(), token)
            os.makedirs(d, exist_ok=True)
            with open(os.path.join(d, "info.dat"), "wb") as f:
                f.write(_sector_blob(self._log_info_text(token, tail)))
            self.version += 1
            return token

    def clear(self) -> None:
        with self._lock:
            self._close_files()
            for p in glob.glob(self.log_path + ".*"):
                if p[len(self.log_path) + 1:].isdigit():
                    os.remove(p)
            import shutil
            shutil.rmtree(self._cpr_dir(), ignore_errors=True)
            shutil.rmtree(self._index_dir(), ignore_errors=True)
            self._index.clear()
            self._chain.clear()
            self._tail = FIRST_VALID_ADDRESS
            self.version = 1

    def _close_files(self) -> None:
        for f in self._files.values():
            f.flush()
            f.close()
        self._files.clear()

    def close(self) -> None:
        with self._lock:
            self._close_files()


def read_index_checkpoint(checkpoint_dir: str, token: str) -> Dict[Tuple[int, int], int]:
    """(bucket, tag) -> address of an index checkpoint's ht.dat / ofb.dat (for inspection and tests)."""
    d = os.path.join(checkpoint_dir, "index-checkpoints", token)
    lines = _read_sector_blob(os.path.join(d, "info.dat")) or []
    size = int(lines[1]) if len(lines) > 1 else DEFAULT_INDEX_BUCKETS
    import numpy as np
    ofb = open(os.path.join(d, "ofb.dat"), "rb").read()
    ht = np.fromfile(os.path.join(d, "ht.dat"), dtype="<u8")[:size * 8].reshape(-1, 8)
    out: Dict[Tuple[int, int], int] = {}

    def take(words, b):
        for w in words[:_ENTRIES]:
            w = int(w)
            if w:
                out[(b, (w >> _TAG_SHIFT_ENTRY) & ((1 << _TAG_BITS) - 1))] = w & _ADDR_MASK
        return int(words[_ENTRIES])

    for b in np.nonzero(ht.any(axis=1))[0].tolist():
        nxt = take(ht[b], b)
        while nxt:
            nxt = take(struct.unpack_from("<8Q", ofb, (nxt - 1) * 64), b)
    return out


def probe_page_bits(log_path: str, lo: int = 9, hi: int = 34, segment_bits: int = DEFAULT_SEGMENT_BITS) -> int:
    """Page size of an existing log, for callers that do not know how it was configured: the page
    bits (smallest first) under which a scan of the log reaches furthest.  FASTER itself does not
    record the page size in a checkpoint; its owners recompute it (LayerStore.cs:354-369)."""
    best_bits, best_end = DEFAULT_PAGE_BITS, -1
    for bits in range(lo, hi + 1):
        kv = FasterKV.__new__(FasterKV)
        if bits > segment_bits:
            break
        kv.log_path, kv.page_bits, kv.segment_bits = log_path, bits, segment_bits
        kv.page_size, kv._files = 1 << bits, {}
        end = FIRST_VALID_ADDRESS
        try:
            for addr, _, _, _, size in kv._records(None):
                end = addr + size
        finally:
            kv._close_files()
        if end > best_end:
            best_bits, best_end = bits, end
    return best_bits
