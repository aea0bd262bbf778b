"""Data-format readers byte by byte (the checks of PredictiveCoding.UnitTests' CsvLoader, MnistDataset,
RssReader, EdfReader, NiftiReader, MidiReader and Spectrogram tests, restated for this package). Every
fixture is built here from the format's published layout."""
import gzip
import struct
import xml.etree.ElementTree as ET

import numpy as np
import pytest
import torch

from predicitivecoding_b200.systems import data as D


# ---------------------------------------------------------------- CSV
def test_csv_with_header_reads_values_and_columns():
    t = D.load_csv("a,b,c\n1,2,3\n4,5,6\n")
    assert t.columns == ["a", "b", "c"] and t.numeric().tolist() == [[1, 2, 3], [4, 5, 6]]


def test_csv_without_header_subset_and_tabs(tmp_path):
    t = D.load_csv("1,2\n3,4\n", header=False)
    assert len(t.rows) == 2 and t.numeric(["c1"]).tolist() == [[2.0], [4.0]]
    tsv = D.load_csv("x\ty\n7\t8\n", delimiter="\t")
    assert tsv.column("y") == ["8"]
    p = tmp_path / "t.csv"
    p.write_text("u,v\n9,10\n")
    assert D.load_csv(str(p)).numeric().tolist() == [[9.0, 10.0]]
    with pytest.raises(ValueError):
        D.load_csv("a\nhello\n").numeric()


# ---------------------------------------------------------------- IDX (MNIST)
def idx(arr: np.ndarray, code: int) -> bytes:
    return bytes([0, 0, code, arr.ndim]) + struct.pack(f">{arr.ndim}I", *arr.shape) + arr.astype(">u1").tobytes()


def test_mnist_images_are_normalised_and_labels_read(tmp_path):
    imgs = np.arange(2 * 4 * 4, dtype=np.uint8).reshape(2, 4, 4) * 7
    labels = np.array([3, 9], np.uint8)
    (tmp_path / "i.gz").write_bytes(gzip.compress(idx(imgs, 0x08)))
    (tmp_path / "l").write_bytes(idx(labels, 0x08))
    ds = D.load_mnist(str(tmp_path / "i.gz"), str(tmp_path / "l"))
    assert ds.images.shape == (2, 1, 4, 4) and float(ds.images.max()) <= 1.0
    assert torch.allclose(ds.images[1, 0], torch.from_numpy(imgs[1] / 255.0).float())
    assert ds.labels.tolist() == [3, 9] and ds.one_hot(0)[3] == 1
    assert D.read_idx(idx(imgs, 0x08)).dtype == np.dtype(">u1")
    with pytest.raises(ValueError):
        D.read_idx(b"\x01\x00\x08\x01\x00\x00\x00\x01\x05")


# ---------------------------------------------------------------- RSS / Atom
RSS = """<?xml version="1.0"?><rss version="2.0"><channel><title>c</title>
<item><title>First</title><description>Body one</description><link>http://a/1</link></item>
<item><title>Second</title><description>Body two</description></item></channel></rss>"""
ATOM = """<?xml version="1.0"?><feed xmlns="http://www.w3.org/2005/Atom"><title>f</title>
<entry><title>E1</title><summary>S1</summary><link href="http://b/1"/></entry></feed>"""


def test_rss2_and_atom_items():
    items = D.read_rss(RSS)
    assert [i["title"] for i in items] == ["First", "Second"] and items[0]["link"] == "http://a/1"
    atom = D.read_rss(ATOM)
    assert atom[0]["title"] == "E1" and atom[0]["link"] == "http://b/1"
    with pytest.raises(ET.ParseError):
        D.read_rss("<rss><channel>")


# ---------------------------------------------------------------- EDF
def edf(labels, samples_per_record, records, pmin=-100.0, pmax=100.0, dmin=-32768, dmax=32767):
    ns = len(labels)
    f = lambda s, w: s.ljust(w)[:w].encode("ascii")
    head = f("0", 8) + f("patient", 80) + f("rec", 80) + f("01.01.01", 8) + f("00.00.00", 8)
    head += f(str(256 + 256 * ns), 8) + f("", 44) + f(str(len(records)), 8) + f("1", 8) + f(str(ns), 4)
    sig = b"".join(f(l, 16) for l in labels) + f("", 80) * ns + f("uV", 8) * ns
    sig += f(str(pmin), 8) * ns + f(str(pmax), 8) * ns + f(str(dmin), 8) * ns + f(str(dmax), 8) * ns
    sig += f("", 80) * ns + b"".join(f(str(n), 8) for n in samples_per_record) + f("", 32) * ns
    body = b"".join(np.asarray(r, "<i2").tobytes() for r in records)
    return head + sig + body


def test_edf_metadata_and_physical_scaling():
    rec = D.read_edf(edf(["EEG Fz", "EEG Cz"], [2, 2], [[0, 32767, -32768, 0], [100, 200, 300, 400]]))
    assert rec.labels == ["EEG Fz", "EEG Cz"] and rec.sample_rates == [2.0, 2.0]
    # each data record holds signal 0's samples, then signal 1's
    fz, cz = rec.signals
    assert fz.tolist() == pytest.approx([0.0015, 100.0, 0.3067, 0.6119], abs=1e-3)
    assert cz[:2].tolist() == pytest.approx([-100.0, 0.0015], abs=1e-3) and len(cz) == 4


# ---------------------------------------------------------------- NIfTI-1
def nifti(vol: np.ndarray, slope=0.0, inter=0.0) -> bytes:
    h = bytearray(352)
    struct.pack_into("<i", h, 0, 348)
    dims = [vol.ndim] + list(vol.shape) + [1] * (7 - vol.ndim)
    struct.pack_into("<8h", h, 40, *dims)
    struct.pack_into("<h", h, 70, 16)                       # float32
    struct.pack_into("<h", h, 72, 32)
    struct.pack_into("<8f", h, 76, 1.0, 0.5, 0.5, 2.0, 1, 1, 1, 1)
    struct.pack_into("<f", h, 108, 352.0)
    struct.pack_into("<2f", h, 112, slope, inter)
    h[344:348] = b"n+1\x00"
    return bytes(h) + vol.astype("<f4").T.tobytes()


def test_nifti_dimensions_voxels_and_scaling():
    vol = np.arange(24, dtype=np.float32).reshape(2, 3, 4)
    arr, pix = D.read_nifti(nifti(vol))
    assert arr.shape == (2, 3, 4) and np.array_equal(arr, vol) and pix == pytest.approx((0.5, 0.5, 2.0))
    scaled, _ = D.read_nifti(nifti(vol, slope=2.0, inter=1.0))
    assert np.array_equal(scaled, vol * 2 + 1)


# ---------------------------------------------------------------- MIDI
def midi(events: bytes, division=96) -> bytes:
    track = events + b"\x00\xff\x2f\x00"
    return b"MThd" + struct.pack(">IHHH", 6, 0, 1, division) + b"MTrk" + struct.pack(">I", len(track)) + track


def test_midi_reads_notes_with_running_status_and_meta_events():
    ev = b"\x00\xff\x51\x03\x07\xa1\x20"            # tempo meta event
    ev += b"\x00\x90\x3c\x64"                         # note on C4 at 0
    ev += b"\x60\x3c\x00"                             # running status: velocity 0 = note off at 96
    ev += b"\x00\x90\x40\x50\x83\x00\x80\x40\x00"     # E4 on at 96, off 384 ticks later (VLQ 0x83 0x00)
    division, notes = D.read_midi(midi(ev))
    assert division == 96
    assert [(n.pitch, n.velocity, n.start_tick, n.end_tick) for n in notes] == [(60, 100, 0, 96), (64, 80, 96, 480)]
    with pytest.raises(ValueError):
        D.read_midi(b"RIFF0000")


# ---------------------------------------------------------------- spectrogram
def test_spectrogram_is_frequency_by_time_and_finds_the_tone():
    sr, f0 = 8000, 1000
    t = np.arange(4096) / sr
    s = D.spectrogram(np.sin(2 * np.pi * f0 * t), n_fft=256, hop=128, log=False)
    assert s.shape[0] == 129 and s.shape[1] == 4096 // 128 + 1
    assert int(s.mean(1).argmax()) == round(f0 / sr * 256)
