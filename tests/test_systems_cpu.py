"""Imaging codecs and the people-counting stack on the CPU."""
import numpy as np
import pytest

from predicitivecoding_b200.systems import imaging as im
from predicitivecoding_b200.systems import vision as vi


def _img():
    rng = np.random.default_rng(0)
    return im.RgbImage.from_pixel_data(rng.integers(0, 256, (7, 9, 3), dtype=np.uint8), 9, 7)


def test_netpbm_ascii_binary_and_16bit():
    p3 = b"P3\n# comment\n2 1\n255\n255 0 0  0 255 0\n"
    a = im.RgbImage.load(p3)
    assert a[0, 0] == (255, 0, 0) and a[1, 0] == (0, 255, 0)
    p5 = b"P5 2 2 65535\n" + bytes([0xFF, 0xFF, 0, 0, 0x80, 0, 0x40, 0])
    g = im.RgbImage.load(p5)
    assert g[0, 0] == (255, 255, 255) and g[1, 0] == (0, 0, 0) and g[0, 1][0] == 0x8000 * 255 // 65535
    with pytest.raises(ValueError):
        im.decode_netpbm(b"P6 2 2 255\n" + b"\x00" * 5)


def test_png_bmp_roundtrip_and_ops(tmp_path):
    a = _img()
    for ext in ("png", "bmp"):
        p = str(tmp_path / f"x.{ext}")
        getattr(a, f"save_as_{ext}")(p)
        b = im.RgbImage.load(p)
        assert np.array_equal(a.pixels, b.pixels)
    c = a.crop(2, 1, 4, 3)
    assert (c.width, c.height) == (4, 3) and c[0, 0] == a[2, 1]
    r = a.resize(18, 14)
    assert (r.width, r.height) == (18, 14)
    gray = a.to_gray()
    assert gray.shape == (7, 9) and gray.dtype == np.uint8


def test_gif_exact_palette_and_quantised(tmp_path):
    f1 = im.RgbImage(4, 3, im.Rgb24(10, 20, 30))
    f2 = f1.clone()
    f2[1, 1] = im.Rgb24(200, 100, 50)
    data = im.encode_gif([f1, f2], 5)
    assert data[:6] == b"GIF89a" and b"NETSCAPE2.0" in data and data[-1] == 0x3B
    frames = im.decode_gif_indices(data)
    assert len(frames) == 2 and len(frames[0]) == 12 and frames[1][1 * 4 + 1] != frames[1][0]
    big = im.RgbImage.from_pixel_data(np.arange(300 * 3, dtype=np.uint32).astype(np.uint8).reshape(30, 10, 3) * 0
                                      + np.random.default_rng(1).integers(0, 256, (30, 10, 3), dtype=np.uint8), 10, 30)
    q = im.decode_gif_indices(im.encode_gif([big]))[0]
    p = big.pixels.reshape(-1, 3).astype(int)
    assert np.array_equal(q, (p[:, 0] & 0xE0) | ((p[:, 1] >> 3) & 0x1C) | (p[:, 2] >> 6))
    with pytest.raises(ValueError):
        im.encode_gif([f1, im.RgbImage(3, 3)])


def test_nms_and_iou():
    a = vi.Detection(0, 0, 10, 10, 0.9)
    b = vi.Detection(1, 1, 11, 11, 0.8)
    c = vi.Detection(20, 20, 30, 30, 0.7)
    assert vi.iou(a, b) == pytest.approx(81 / 119)
    assert vi.nms([c, b, a], 0.5) == [a, c]


def test_sort_tracker_confirms_counts_and_expires():
    tr = vi.SortTracker(iou_threshold=0.3, max_age=2, min_hits=3)
    for f in range(5):
        out = tr.update([vi.Detection(10 + 2 * f, 10, 30 + 2 * f, 50)])
        assert len(out) == (1 if f >= 2 else 0)
    assert tr.unique_count == 1 and tr.current_count == 1
    for _ in range(4):
        tr.update([])
    assert tr.tracks == [] and tr.unique_count == 1


def test_line_and_zone_counters_and_smoother():
    lc = vi.LineCounter(0, 5, 10, 5)
    lc.update([(1, 5, 2), (2, 5, 8)])
    lc.update([(1, 5, 8), (2, 5, 2)])
    assert (lc.inbound, lc.outbound, lc.net) == (1, 1, 0)
    z = vi.ZoneCounter([(0, 0), (10, 0), (10, 10), (0, 10)])
    z.update([(1, 5, 5), (2, 20, 5)])
    z.update([(1, 6, 5)])
    assert z.occupancy == 1 and z.entered == 1 and z.dwell_frames(1) == 2
    sm = vi.CountSmoother(3)
    assert [sm.add(v) for v in (5, 1, 9, 2)] == [5, 5, 5, 2]


def test_reid_gallery_and_hog():
    frame = im.RgbImage(20, 20, im.Rgb24(200, 10, 10))
    emb = vi.ColorHistogramEmbedder(8, 0.6)
    e1 = emb.embed(frame, vi.Detection(2, 2, 12, 12))
    assert e1.shape == (24,) and abs(np.linalg.norm(e1) - 1) < 1e-6
    g = vi.PersonGallery(0.9)
    assert g.identify_or_register(e1) == 1 and g.identify_or_register(e1) == 1
    other = im.RgbImage(20, 20, im.Rgb24(10, 10, 200))
    assert g.identify_or_register(emb.embed(other, vi.Detection(2, 2, 12, 12))) == 2
    hog = vi.HogDescriptor(16, 16, 8, 9)
    x = np.tile(np.arange(16, dtype=np.float32), (16, 1))
    f = hog.compute_gray(x)
    assert f.shape == (hog.dimension,) == (36,) and f.max() > 0


def test_counting_pipeline_and_cpu_annotation():
    boxes = [vi.Detection(5, 5, 15, 25)]
    pipe = vi.PeopleCountingPipeline(lambda fr: boxes, vi.SortTracker(min_hits=2), detect_every_n=2)
    res = [pipe.process(im.RgbImage(32, 32)) for _ in range(4)]
    assert [r.detected for r in res] == [True, False, True, False] and res[-1].current_count == 1
    ann = vi.Annotator(2).draw_boxes(boxes).draw_line(0, 31, 31, 0).draw_zone([(2, 2), (29, 2), (29, 29)])
    img = ann.render_cpu(im.RgbImage(32, 32))
    assert img[5, 5] == vi.DET_COLOR or img[5, 5] in (vi.LINE_COLOR, vi.ZONE_COLOR)
    assert img[10, 15] == (0, 0, 0)
    assert (img.pixels != 0).any(axis=2).sum() > 100


# ---------------------------------------------------------------- Thousand Brains
from predicitivecoding_b200.systems import brain as br


def test_sdr_ops_and_encoders():
    a, b = br.Sdr(10, [1, 3, 3, 5]), br.Sdr(10, [3, 5, 7])
    assert a.bits == (1, 3, 5) and a.overlap(b) == 2 and a.union(b).bits == (1, 3, 5, 7)
    assert a.intersect(b).bits == (3, 5) and abs(a.overlap_score(b) - 2 / 3) < 1e-6
    with pytest.raises(ValueError):
        br.Sdr(4, [4])
    rng = np.random.default_rng(0)
    r = br.Sdr.random(100, 10, rng)
    n = r.add_noise(0.3, rng)
    assert n.cardinality == 10 and r.overlap(n) == 7
    se = br.ScalarEncoder(0, 1, 20, 5)
    assert se.encode(0).bits == (0, 1, 2, 3, 4) and se.encode(1).bits[-1] == 19
    assert se.encode(0.5).overlap(se.encode(0.55)) >= 4
    pe = br.PoseEncoder(0, 10, 0, 10, 50, 5, 8, 3)
    assert pe.encode(1, 2, 90).cardinality == 13 and pe.size == 124
    pi = br.PathIntegrator()
    pi.move(1.0)
    pi.move(1.0, 90)
    dx, dy = pi.displacement(0, 2)
    assert abs(dx - 1) < 1e-9 and abs(dy - 1) < 1e-9


def test_spatial_pooler_and_temporal_memory_learn_a_sequence():
    sp = br.SpatialPooler(br.SpatialPoolerConfig(200, 256, 10, seed=1))
    rng = np.random.default_rng(2)
    x = br.Sdr.random(200, 20, rng)
    out1 = sp.compute(x, True)
    for _ in range(5):
        sp.compute(x, True)
    assert out1.cardinality == 10 and sp.compute(x, False).overlap(out1) >= 8
    tm = br.TemporalMemory(br.TemporalMemoryConfig(64, 4, activation_threshold=3, min_threshold=2,
                                                   max_new_synapse_count=8))
    seq = [br.Sdr(64, range(i * 8, i * 8 + 5)) for i in range(4)]
    anomalies = []
    for rep in range(8):
        tm.reset()
        anomalies.append([tm.compute(s, True).anomaly for s in seq])
    assert anomalies[0][1:] == [1.0, 1.0, 1.0] and max(anomalies[-1][1:]) == 0.0


def test_multi_column_recognition():
    data = br.SyntheticObjectDataset(n_objects=6, points=8, seed=3)
    tbs = br.ThousandBrainsSystem(data.size, data.size, n_columns=3, columns=256)
    rep = br.recognition_benchmark(tbs, data)
    assert rep.n == 6 and rep.accuracy >= 0.8
    cons = br.Consensus(0.5).compute([[1, 2], [2], [2, 3]])
    assert cons.candidates == [2] and cons.reached
    lv = br.LateralVoting(4, "ring")
    assert lv.neighbors(0) == [1, 3]
    assert br.k_winners([0.1, 0.9, 0.5, 0.9], 2) == [1, 3]


# ---------------------------------------------------------------- cortex
import torch

from predicitivecoding_b200.pc.network import NetworkConfig
from predicitivecoding_b200.pc.networks import HierarchicalNetworkConfig, HopfieldNetworkConfig
from predicitivecoding_b200.systems import cortex as cx


def test_retinotopic_map_roundtrip_and_visual_cortex():
    m = cx.RetinotopicMap(1, 8, 8, 4, 2)
    img = torch.arange(64, dtype=torch.float32)
    patches = m.extract(img)
    assert len(patches) == 9 and torch.allclose(m.assemble(patches), img)
    cfg = cx.VisualCortexConfig(1, 8, 8, 4, 4, NetworkConfig(layer_sizes=(16, 8, 4)),
                                HierarchicalNetworkConfig([NetworkConfig(layer_sizes=(16, 8, 3))]),
                                NetworkConfig(layer_sizes=(3, 6, 2)))
    vc = cx.VisualCortex(cfg)
    x = torch.rand(64)
    vc.learn_supervised(x, torch.tensor([1.0, 0.0]), 5)
    assert vc.encode(x, 5).shape == (3,) and vc.predict(x, 5) in (0, 1)
    assert vc.reconstruct(x, 5).shape == (64,) and len(vc.encode_areas(x, 5)) == 2


def test_scalar_areas():
    bg = cx.BasalGanglia(1.0, no_go_threshold=5.0)
    a, g = bg.select([3.0, 1.0, 2.0])
    assert a == 1 and abs(sum(g) - 1) < 1e-6 and bg.select([6.0, 7.0])[0] == -1
    th = cx.Thalamus(1.0, 1.0).allocate([1.0, 1.0])
    assert th == pytest.approx([1.0, 1.0])
    cc = cx.CingulateCortex()
    assert cc.conflict([1.0, 1.0, 1.0]) == pytest.approx(1.0) and cc.conflict([0.0, 50.0]) < 0.01
    da = cx.DopaminergicSystem(0.9)
    assert da.reward_prediction_error(1.0, 0.5, 1.0) == pytest.approx(1.4) and da.step(1.0) == 1.0
    lc = cx.LocusCoeruleus()
    assert lc.process(1.0) == (False, 1.0) and lc.process(10.0) == (True, 4.0)
    assert cx.Habenula().suppress_dopamine(1.0, 0.0, 0.5) == 0.5
    assert cx.RapheNuclei(1.0).time_horizon() == pytest.approx(100.0)
    nb = cx.NucleusBasalis(2)
    assert list(nb.update([1.0, 2.0])) == [1.0, 2.0]
    hy = cx.Hypothalamus([1.0, 1.0])
    assert hy.need_level([1.0, 0.0]) == 1.0
    assert cx.PeriaqueductalGray().respond(0.7) == "flight"
    sc = cx.SuperiorColliculus(4, enhancement=1.0)
    assert sc.scan([0.1, 0.9, 0.2, 0.0], [0.0, 0.0, 0.9, 0.0], 2) == [2, 1]
    assert cx.Claustrum.coherence([[1, 0], [1, 0]]) == pytest.approx(1.0)
    ret = cx.RetinaLgn(1, 9, 9)
    flat = ret.process(torch.ones(81))
    spot = torch.zeros(81)
    spot[40] = 1
    assert flat.abs().max() < 1e-5 and ret.process(spot)[40] > 0
    gc = cx.GridCellEncoder(2, 9, 1.0, 1.4)
    assert gc.encode(0.3, 0.7).shape == (18,)
    assert cx.OlfactoryBulb(2).process([0.1, 3.0, 0.2, 2.0]).count_nonzero() == 2
    assert cx.InferiorColliculus(4).process(torch.sin(torch.arange(64.0))).shape == (4,)


def test_network_backed_areas():
    am = cx.Amygdala(NetworkConfig(layer_sizes=(4, 6, 2)))
    am.learn(torch.ones(4), torch.tensor([1.0, 0.0]), 5)
    assert am.salience_gain(torch.ones(4), 5) >= 1.0
    cb = cx.CerebellarCortex(cx.CerebellarCortexConfig(2, 1, NetworkConfig(layer_sizes=(3, 8, 2))))
    cb.learn([0.0, 0.0], [1.0], [0.5, 0.5], 5)
    assert cb.prediction_error([0.0, 0.0], [1.0], [0.5, 0.5], 5) >= 0
    mc = cx.MotorCortex(cb, [[1.0], [-1.0]])
    assert mc.select_command([0.0, 0.0], [0.5, 0.5], 5) in (0, 1)
    hf = cx.HippocampalFormation(cx.HippocampalFormationConfig(
        HopfieldNetworkConfig(NetworkConfig(layer_sizes=(4, 6, 3))), NetworkConfig(layer_sizes=(4, 6, 3))))
    for k in range(3):
        hf.experience(torch.eye(4)[k], 5)
    hf.replay(1, 3)
    assert hf.episode_count == 3 and hf.recall(torch.eye(4)[0], 5).shape == (4,)
    pr = cx.PerirhinalCortex(NetworkConfig(layer_sizes=(4, 6, 3)))
    pr.remember(torch.eye(4)[0], 5)
    assert not pr.is_novel(torch.eye(4)[0], 5)
    pc = cx.PiriformCortex()
    pc.memorize([1, 0, 0], "rose")
    assert pc.recognize([0.9, 0.1, 0]) == "rose"
    we = cx.WernickeArea(NetworkConfig(layer_sizes=(5, 6, 2)))
    we.learn_utterance(torch.ones(5), torch.tensor([0.0, 1.0]), 5)
    assert we.surprise(torch.ones(5), 5) >= 0
    assert cx.BrocaArea(NetworkConfig(layer_sizes=(5, 6, 2))).produce(torch.tensor([0.0, 1.0]), 5) in range(5)
    dm = cx.DefaultModeNetwork(NetworkConfig(layer_sizes=(4, 6, 3)))
    dm.learn_from_experience(torch.ones(4), 3)
    dm.learn_from_experience(torch.zeros(4), 3)
    assert len(dm.imagine_sequence(2, 3)) == 2
    assert len(cx.AREAS) >= 49


# ---------------------------------------------------------------- ONNX subset
from predicitivecoding_b200.systems import onnx as ox


def _graph():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(4, 3, 3, 3, generator=g)
    b = torch.randn(4, generator=g)
    sc, bi = torch.rand(4, generator=g) + 0.5, torch.randn(4, generator=g)
    mu, var = torch.randn(4, generator=g), torch.rand(4, generator=g) + 0.5
    fc = torch.randn(4 * 4 * 4, 5, generator=g)
    T = ox.TensorData.from_torch
    A = lambda name, typ, **kw: ox.Attribute(name, typ, **kw)
    nodes = [
        ox.Node("c", "Conv", ["x", "w", "b"], ["c"], {"pads": A("pads", ox.A_INTS, ints=[1, 1, 1, 1])}),
        ox.Node("bn", "BatchNormalization", ["c", "sc", "bi", "mu", "var"], ["n"]),
        ox.Node("r", "Relu", ["n"], ["r"]),
        ox.Node("p", "MaxPool", ["r"], ["p"], {"kernel_shape": A("kernel_shape", ox.A_INTS, ints=[2, 2]),
                                                "strides": A("strides", ox.A_INTS, ints=[2, 2])}),
        ox.Node("k", "Constant", [], ["shape"], {"value": A("value", ox.A_TENSOR, t=T("", torch.tensor([1, -1])))}),
        ox.Node("f", "Reshape", ["p", "shape"], ["f"]),
        ox.Node("id", "Identity", ["f"], ["fi"]),
        ox.Node("g", "Gemm", ["fi", "fc"], ["g"]),
        ox.Node("s", "Softmax", ["g"], ["y"], {"axis": A("axis", ox.A_INT, i=1)}),
        ox.Node("dead", "Relu", ["g"], ["unused"]),
    ]
    inits = {k: T(k, v) for k, v in dict(w=w, b=b, sc=sc, bi=bi, mu=mu, var=var, fc=fc).items()}
    gr = ox.Graph("tiny", 13, nodes, inits, [ox.ValueInfo("x", [1, 3, 8, 8])], [ox.ValueInfo("y", [1, 5])])

    def ref(x):
        c = torch.nn.functional.conv2d(x, w, b, padding=1)
        n = (c - mu.view(1, -1, 1, 1)) / torch.sqrt(var.view(1, -1, 1, 1) + 1e-5) * sc.view(1, -1, 1, 1) + bi.view(1, -1, 1, 1)
        p = torch.nn.functional.max_pool2d(torch.relu(n), 2, 2)
        return torch.softmax(p.reshape(1, -1) @ fc, 1)
    return gr, ref


def test_onnx_protobuf_roundtrip_execution_optimizer_and_pcnx(tmp_path):
    gr, ref = _graph()
    blob = ox.encode_model(gr)
    m = ox.OnnxModel.load(blob)
    assert m.input_names == ["x"] and m.output_names == ["y"] and m.graph.opset == 13
    x = torch.randn(1, 3, 8, 8)
    y = m.run({"x": x})["y"]
    assert torch.allclose(y, ref(x), atol=1e-5)
    opt = ox.optimize_graph(m.graph)
    ops = [n.op_type for n in opt.nodes]
    assert "Constant" not in ops and "Identity" not in ops and "Reshape" in ops and len(ops) == 7
    p = str(tmp_path / "tiny.pcnx")
    m.save(p)
    back = ox.OnnxModel.load(p)
    assert torch.equal(back.run({"x": x})["y"], ox.OnnxModel(opt).run({"x": x})["y"])
    assert torch.allclose(back.run({"x": x})["y"], y, atol=1e-6)
    with pytest.raises(ValueError):
        ox.read_pcnx(b"NOPE" + b"\x00" * 16)


# ---------------------------------------------------------------- data sources
import gzip
import json
import struct as st

from predicitivecoding_b200.systems import data as dt


def test_idx_mnist_and_cifar(tmp_path):
    imgs = np.arange(2 * 3 * 3, dtype=np.uint8).reshape(2, 3, 3)
    (tmp_path / "i.gz").write_bytes(gzip.compress(b"\x00\x00\x08\x03" + st.pack(">3I", 2, 3, 3) + imgs.tobytes()))
    (tmp_path / "l").write_bytes(b"\x00\x00\x08\x01" + st.pack(">I", 2) + bytes([3, 7]))
    ds = dt.load_mnist(str(tmp_path / "i.gz"), str(tmp_path / "l"))
    assert ds.images.shape == (2, 1, 3, 3) and ds.labels.tolist() == [3, 7] and ds.one_hot(1)[7] == 1
    rec = bytes([5]) + bytes(range(256)) * 12
    (tmp_path / "c.bin").write_bytes(rec * 2)
    cf = dt.load_cifar10([str(tmp_path / "c.bin")])
    assert len(cf) == 2 and cf.images.shape == (2, 3, 32, 32) and int(cf.labels[0]) == 5


def test_csv_sqlite_and_shards(tmp_path):
    t = dt.load_csv("a,b\n1,2\n3,4\n")
    assert t.numeric().tolist() == [[1, 2], [3, 4]] and t.column("b") == ["2", "4"]
    import sqlite3
    db = str(tmp_path / "x.db")
    con = sqlite3.connect(db)
    con.execute("create table t(x int, y text)")
    con.execute("insert into t values (1, 'a'), (2, 'b')")
    con.commit()
    con.close()
    assert dt.sqlite_table(db, "select * from t where x > ?", (1,)).rows == [["2", "b"]]
    w = dt.ShardedCorpusWriter(str(tmp_path / "sh"), 1024)
    for i in range(60):
        w.append([f"document {i} line one", "  second   line "])
    w.close()
    assert len(w.shards()) > 1 and w.documents == 60
    w2 = dt.ShardedCorpusWriter(str(tmp_path / "sh"), 1024)
    lines = list(w2.lines())
    assert lines[0] == "document 0 line one" and lines[1] == "second line" and len(lines) == 120


def test_html_rss_and_language_id(tmp_path):
    page = "<html><script>x=1</script><h1>Title &amp; more</h1><p>Para <b>one</b>.</p><p>Two</p></html>"
    assert dt.html_to_text(page) == ["Title & more", "Para one .", "Two"]
    rss = "<rss><channel><item><title>A</title><link>u</link></item><item><title>B</title></item></channel></rss>"
    assert [i["title"] for i in dt.read_rss(rss)] == ["A", "B"]
    tr = dt.NGramLanguageClassifierTrainer()
    tr.add("en", "the quick brown fox jumps over the lazy dog and the cat sat on the mat with the hat")
    tr.add("it", "il gatto nero dorme sul divano e la casa della nonna era piena di gente allegra")
    clf = tr.train()
    assert clf.predict("the dog and the hat") == "en" and clf.predict("la gatta della casa") == "it"
    p = str(tmp_path / "lid.bin")
    clf.save(p)
    assert dt.NGramLanguageClassifier.load(p).predict("the cat") == "en"


def test_signal_formats():
    s = dt.spectrogram(torch.sin(torch.arange(2048.0) * 0.3))
    assert s.shape[0] == 129
    # EDF: one signal, 2 records of 4 samples
    ns = 1
    hdr = (b"0".ljust(8) + b"pat".ljust(80) + b"rec".ljust(80) + b"01.01.01" + b"00.00.00" + b"512".ljust(8)
           + b"".ljust(44) + b"2".ljust(8) + b"1".ljust(8) + b"1".ljust(4))
    sh = (b"EEG".ljust(16) + b"".ljust(80) + b"uV".ljust(8) + b"-100".ljust(8) + b"100".ljust(8) + b"-32768".ljust(8)
          + b"32767".ljust(8) + b"".ljust(80) + b"4".ljust(8) + b"".ljust(32))
    body = np.array([0, 32767, -32768, 0, 1, 2, 3, 4], "<i2").tobytes()
    rec = dt.read_edf(hdr + sh + body)
    assert rec.labels == ["EEG"] and rec.sample_rates == [4.0] and abs(rec.signals[0][1] - 100) < 0.01
    # NIfTI-1: 2x3x1 float volume
    h = bytearray(352)
    st.pack_into("<i", h, 0, 348)
    st.pack_into("<8h", h, 40, 3, 2, 3, 1, 1, 1, 1, 1)
    st.pack_into("<h", h, 70, 16)
    st.pack_into("<8f", h, 76, 1, 1, 2, 3, 1, 1, 1, 1)
    st.pack_into("<f", h, 108, 352.0)
    st.pack_into("<2f", h, 112, 1.0, 0.0)
    vol, pix = dt.read_nifti(bytes(h) + np.arange(6, dtype="<f4").tobytes())
    assert vol.shape == (2, 3, 1) and vol[1, 0, 0] == 1 and pix == (1.0, 2.0, 3.0)
    # MIDI: one track, note 60 on at 0, off at 96
    trk = b"\x00\x90\x3c\x40" + b"\x60\x80\x3c\x00" + b"\x00\xff\x2f\x00"
    mid = b"MThd" + st.pack(">IHHH", 6, 0, 1, 96) + b"MTrk" + st.pack(">I", len(trk)) + trk
    div, notes = dt.read_midi(mid)
    assert div == 96 and notes == [dt.MidiNote(0, 0, 60, 64, 0, 96)]


def test_web_sources_with_injected_fetch():
    pages = {"https://en.wikipedia.org/w/api.php?action=query&prop=extracts&explaintext=1&format=json&titles=Cat":
             json.dumps({"query": {"pages": {"1": {"extract": "Cats purr.\n\nThey nap."}}}}),
             "https://hacker-news.firebaseio.com/v0/topstories.json": "[1, 2]",
             "https://hacker-news.firebaseio.com/v0/item/1.json": '{"title": "A"}',
             "https://hacker-news.firebaseio.com/v0/item/2.json": '{"title": "B"}'}
    assert dt.WikipediaSource(pages.__getitem__).article("Cat") == ["Cats purr.", "They nap."]
    assert [s["title"] for s in dt.HackerNewsSource(pages.__getitem__).top_stories(2)] == ["A", "B"]
    atom = ("<feed xmlns='http://www.w3.org/2005/Atom'><entry><title> Paper\n one </title><summary>S</summary>"
            "<id>x</id></entry></feed>")
    assert dt.ArxivSource(lambda u: atom).search("pc")[0]["title"] == "Paper one"


# ---------------------------------------------------------------- faces
from predicitivecoding_b200.systems import faces as fc


def _face(seed, person):
    rng = np.random.default_rng(1000 * person + seed)
    base = np.random.default_rng(person).integers(0, 256, (16, 16, 3)).astype(np.float64)
    noisy = np.clip(base + rng.normal(0, 12, base.shape), 0, 255).astype(np.uint8)
    big = np.kron(noisy, np.ones((8, 8, 1), np.uint8))
    return im.RgbImage.from_pixel_data(big, 128, 128)


def test_lbp_descriptor_and_tan_triggs():
    assert (fc.UNIFORM < 58).sum() == 58 and fc.UNIFORM[0b01010101] == 58
    g = fc.face_pixels(_face(0, 1))
    d = fc.lbp_descriptor(g)
    assert d.shape == (fc.DIMENSION,) and abs(np.linalg.norm(d) - 1) < 1e-5
    t = fc.tan_triggs(g)
    assert t.dtype == np.uint8 and t.min() == 0 and t.max() == 255


def test_pca_whitening_and_embedders_and_benchmarks():
    rng = np.random.default_rng(0)
    X = rng.normal(size=(200, 20)) @ np.diag(np.linspace(5, 0.1, 20))
    p = fc.PcaProjector().fit(X, 5)
    z = p.project(X).numpy()
    assert z.shape == (200, 5) and np.allclose(z.var(0, ddof=1), 1, atol=0.05)
    people = [0, 1, 2]
    imgs = [_face(s, pp) for pp in people for s in range(3)]
    lbp = fc.LbpEmbedder()
    db = fc.FaceDatabase(lbp, threshold=0.0)
    for pp in people:
        db.enroll(f"p{pp}", _face(0, pp))
    assert db.identify(_face(5, 1))[0] == "p1"
    pairs = [(_face(1, a), _face(2, b), a == b) for a in people for b in people]
    res = fc.verification_benchmark(lbp, pairs, folds=3)
    assert res.auc_roc > 0.9 and res.mean_same > res.mean_diff
    assert fc.identification_benchmark(lbp, {f"p{pp}": _face(0, pp) for pp in people},
                                       [(f"p{pp}", _face(4, pp)) for pp in people]) == 1.0
    enh = fc.EnhancedLbpEmbedder(target_dim=4)
    enh.fit(imgs)
    assert enh.embed(imgs[0]).shape == (4,)
    pce = fc.PcFaceEmbedder(latent_dim=8, inference_steps=2, epochs=1, hidden=16)
    pce.fit(imgs[:3])
    fused = fc.FusedEmbedder([lbp, pce])
    assert fused.embed(imgs[0]).shape == (fc.DIMENSION + 8,)
    assert fc.auc_roc([0.9, 0.8, 0.1], [True, True, False]) == 1.0
