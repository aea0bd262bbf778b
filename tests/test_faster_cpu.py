"""FASTER hybrid-log layout: round trips through the store wrappers, checked in both directions
against a reader and a writer of the documented on-disk format written here from scratch.

Geometry is shrunk (pages of 2^10-2^12 bytes, segments of 2^12-2^14) so a handful of records spans
several pages and several segment files, which exercises the page-skip and segment-split rules.
"""
import os
import struct
import tempfile
import uuid

import numpy as np
import torch

from predicitivecoding_b200.io import checkpoint as ck
from predicitivecoding_b200.io.faster import (FIRST_VALID_ADDRESS, FasterKV, key_hash, probe_page_bits,
                                              read_index_checkpoint, record_size)
from predicitivecoding_b200.pc.layer import Layer
from predicitivecoding_b200.pc.store import LayerStore, page_size_bits


# ------------------------------------------------------------------ an independent reader / writer
def parse_log(log_path, page_bits, segment_bits, limit):
    """Newest value per key, by walking pages in address order (no use of the package's scanner)."""
    page, seg = 1 << page_bits, 1 << segment_bits
    data = bytearray()
    n = 0
    while os.path.exists(f"{log_path}.{n}"):
        blob = open(f"{log_path}.{n}", "rb").read()
        data += blob + b"\0" * (seg - len(blob))
        n += 1
    out, addr, records = {}, FIRST_VALID_ADDRESS, 0
    while addr < limit:
        room = page - addr % page
        word = int.from_bytes(data[addr:addr + 8], "little") if room >= 24 else 0
        if word == 0:
            addr += room
            continue
        key, vlen = struct.unpack_from("<i4xi", data, addr + 8)
        assert (addr % page) + record_size(vlen) <= page, "record crosses a page"
        assert word >> 56 & 1, "valid bit"
        if word >> 55 & 1:
            out.pop(key, None)
        else:
            out[key] = bytes(data[addr + 20:addr + 20 + vlen])
        addr += record_size(vlen)
        records += 1
    return out, records


def final_address(ckpt_dir):
    best = None
    for tok in os.listdir(os.path.join(ckpt_dir, "cpr-checkpoints")):
        raw = open(os.path.join(ckpt_dir, "cpr-checkpoints", tok, "info.dat"), "rb").read()
        n = struct.unpack_from("<i", raw)[0]
        assert len(raw) % 512 == 0
        lines = raw[4:4 + n].decode().splitlines()
        assert lines[2] == tok and int(lines[5]) == int(lines[4]) + 1
        lo, hi = struct.unpack("<qq", uuid.UUID(tok).bytes_le)
        v, fl, st, fi, hd, bg = (int(lines[i]) for i in (4, 6, 7, 8, 10, 11))
        chk = lo ^ hi ^ v ^ fl ^ st ^ fi ^ hd ^ bg ^ int(lines[14]) ^ int(lines[15])
        assert int(lines[1]) == chk
        if best is None or v > best[0]:
            best = (v, fi)
    return best[1]


def write_log(log_path, ckpt_dir, page_bits, segment_bits, records):
    """Write records (key, value) the way the documented layout prescribes, plus a fold-over
    checkpoint, without the package's writer."""
    page, seg = 1 << page_bits, 1 << segment_bits
    data = bytearray(FIRST_VALID_ADDRESS)
    heads = {}
    for key, value in records:
        size = record_size(len(value))
        if len(data) % page + size > page:
            data += b"\0" * (page - len(data) % page)
        h = key_hash(key)
        slot = (h & ((1 << 20) - 1), h >> 50)
        info = heads.get(slot, 0) | (1 << 56)
        heads[slot] = len(data)
        rec = struct.pack("<Qi4xi", info, key, len(value)) + value
        data += rec + b"\0" * (size - len(rec))
    for n in range(0, len(data), seg):
        with open(f"{log_path}.{n // seg}", "wb") as f:
            f.write(data[n:n + seg])
    tok = str(uuid.uuid4())
    d = os.path.join(ckpt_dir, "cpr-checkpoints", tok)
    os.makedirs(d)
    tail = len(data)
    lo, hi = struct.unpack("<qq", uuid.UUID(tok).bytes_le)
    chk = lo ^ hi ^ 1 ^ tail ^ tail ^ tail ^ tail ^ 64
    text = "".join(f"{v}\n" for v in [5, chk, tok, 0, 1, 2, tail, tail, tail, tail, tail, 64, -1, "False", 0, 0])
    raw = struct.pack("<i", len(text)) + text.encode()
    with open(os.path.join(d, "info.dat"), "wb") as f:
        f.write(raw + b"\0" * (-len(raw) % 512))


# ------------------------------------------------------------------ tests
def test_records_span_pages_and_segments_and_reopen():
    with tempfile.TemporaryDirectory() as d:
        log, cp = os.path.join(d, "s.log"), os.path.join(d, "ck")
        kv = FasterKV(log, cp, page_bits=10, segment_bits=12)
        vals = {k: bytes([k % 251]) * (37 * k % 700) for k in range(60)}
        for k, v in vals.items():
            kv.upsert(k, v)
        kv.delete(5)
        kv.upsert(6, b"six")
        tok = kv.checkpoint()
        kv.upsert(7, b"not committed")
        kv.close()
        assert len([f for f in os.listdir(d) if f.startswith("s.log.")]) >= 5
        vals.pop(5)
        vals[6] = b"six"
        got, n = parse_log(log, 10, 12, final_address(cp))
        assert got == vals and n == 62
        kv2 = FasterKV(log, cp, page_bits=10, segment_bits=12)
        assert kv2.items() == vals
        assert read_index_checkpoint(cp, tok) == kv2._chain
        assert probe_page_bits(log, segment_bits=12) == 10


def test_store_reads_a_log_written_from_the_format_description():
    with tempfile.TemporaryDirectory() as d:
        log, cp = os.path.join(d, "w.log"), os.path.join(d, "ck")
        recs = [(k, os.urandom(100 + 53 * k % 900)) for k in range(30)] + [(3, b"three")]
        write_log(log, cp, 11, 13, recs)
        want = dict(recs)
        kv = FasterKV(log, cp, page_bits=11, segment_bits=13)
        assert kv.items() == want
        kv.close()


def test_layer_store_round_trip_across_pages_and_segments():
    with tempfile.TemporaryDirectory() as d:
        g = torch.Generator().manual_seed(0)
        sizes = [24, 30, 16]
        layers = [Layer.create(i, s, sizes[i - 1] if i else 0, "tanh", g) for i, s in enumerate(sizes)]
        st = LayerStore(layers, path=d, page_bits=12, segment_bits=13)
        L1 = st.read(1)
        L1.W += 1.0
        st.write(1, L1)
        st.close()
        from predicitivecoding_b200.io import layer_serializer as ser
        got, _ = parse_log(os.path.join(d, "layers.log"), 12, 13, final_address(os.path.join(d, "checkpoints")))
        assert sorted(got) == [0, 1, 2]
        assert torch.allclose(ser.deserialize(got[1], 1, "tanh").W, L1.W)
        back = LayerStore.open(d, "tanh", page_bits=12, segment_bits=13)
        assert torch.allclose(back.read(1).W, L1.W) and torch.allclose(back.read(2).W, layers[2].W)


def test_layer_store_page_size_follows_the_reference_rule():
    assert page_size_bits([784, 256, 256, 10]) == 22          # every record fits 4 MiB
    assert page_size_bits([4096, 8192]) == 28                 # 8192 x 4096 fp32 weights need 2^28 bytes


def test_checkpoint_store_round_trip_across_pages_and_segments():
    with tempfile.TemporaryDirectory() as d:
        ts = [torch.randn(7, 33), torch.randn(50, 20), torch.randn(3)]
        with ck.CheckpointStore(d, page_size_bits=12, recover=False, segment_bits=13) as st:
            for i, t in enumerate(ts):
                st.upsert_tensor(i, t)
            st.commit()
        got, _ = parse_log(os.path.join(d, ck.LOG_NAME), 12, 13, final_address(os.path.join(d, "checkpoints")))
        for i, t in enumerate(ts):
            a, _ = ck.read_tensor_blob(got[i])
            assert np.allclose(a.reshape(-1), t.numpy().reshape(-1))
        with ck.CheckpointStore(d, page_size_bits=12, segment_bits=13) as st:
            assert np.allclose(ck.read_tensor_blob(st.get_blob(1))[0], ts[1].numpy())


def test_reader_accepts_the_earlier_json_checkpoint_metadata():
    import json
    with tempfile.TemporaryDirectory() as d:
        log, cp = os.path.join(d, "j.log"), os.path.join(d, "ck")
        kv = FasterKV(log, cp, page_bits=12)
        kv.upsert(1, b"a")
        kv.close()
        os.makedirs(os.path.join(cp, "cpr-checkpoints", "old"))
        with open(os.path.join(cp, "cpr-checkpoints", "old", "info.dat"), "w") as f:
            json.dump({"version": 1, "finalLogicalAddress": kv.tail_address, "guid": "old"}, f)
        assert FasterKV(log, cp, page_bits=12).items() == {1: b"a"}
