"""Detectors and face embedders over the in-house ONNX executor, with small synthetic ONNX graphs as
model fixtures (the reference downloads YOLOX / SCRFD / ArcFace models; none ship with it)."""
import os
import tempfile

import numpy as np
import pytest
import torch

from predicitivecoding_b200.systems import onnx as ox
from predicitivecoding_b200.systems.imaging import RgbImage
from predicitivecoding_b200.systems.vision_models import (
    ArcFaceOnnxEmbedder, FaceCountDetector, FrameStream, LfwDataset, PcDistilledFaceEmbedder, RetinaFaceDetector,
    YoloPersonDetector, align_face, similarity_transform, TEMPLATE_X, TEMPLATE_Y)


def _const_model(inp, in_shape, outs):
    """A graph whose outputs are constants (input -> ReduceMean -> * 0 -> + constant), serialised with the
    package's ONNX writer and parsed back."""
    g = ox.Graph(name="fixture", opset=13, inputs=[ox.ValueInfo(inp, list(in_shape))])
    g.initializers["zero"] = ox.TensorData.from_torch("zero", torch.zeros(1))
    g.nodes.append(ox.Node("m", "ReduceMean", [inp], ["mean"], {"keepdims": ox.Attribute("keepdims", 2, i=0)}))
    g.nodes.append(ox.Node("z", "Mul", ["mean", "zero"], ["z0"]))
    for name, t in outs.items():
        g.initializers[name + "_c"] = ox.TensorData.from_torch(name + "_c", t)
        g.nodes.append(ox.Node("a" + name, "Add", ["z0", name + "_c"], [name]))
        g.outputs.append(ox.ValueInfo(name, list(t.shape)))
    return ox.OnnxModel.load(ox.encode_model(g))


def test_yolox_decoding_letterbox_and_nms():
    out = torch.full((1, 8400, 85), -1.0)
    out[..., 4] = 0.0
    # stride 8 cell (gx=10, gy=20): centre ((0.5 + 10) * 8, (0.5 + 20) * 8) = (84, 164), size e^2 * 8
    a = 20 * 80 + 10
    out[0, a, :4] = torch.tensor([0.5, 0.5, 2.0, 2.0])
    out[0, a, 4], out[0, a, 5] = 0.9, 0.8
    out[0, a + 1] = out[0, a]                              # a near-duplicate one cell right: NMS drops it
    out[0, a + 1, 4] = 0.85
    det = YoloPersonDetector(_const_model("images", (1, 3, 640, 640), {"output": out}))
    frame = RgbImage(1280, 640)                            # r = 0.5: boxes scale by 2
    got = det.detect(frame)
    assert len(got) == 1 and got[0].label == "person" and abs(got[0].score - 0.72) < 1e-5
    w = float(np.exp(2.0) * 8)
    assert abs(got[0].x1 - (84 - w / 2) / 0.5) < 1e-3 and abs(got[0].y2 - (164 + w / 2) / 0.5) < 1e-3
    t, r = det.preprocess(RgbImage(320, 160, fill=(10, 20, 30)))
    assert r == 2.0 and t[0, :, 0, 0].tolist() == [30.0, 20.0, 10.0] and float(t[0, 0, 639, 639]) == 114.0
    # the transposed [1, 85, N] layout decodes the same
    det2 = YoloPersonDetector(_const_model("images", (1, 3, 640, 640), {"output": out.transpose(1, 2).contiguous()}))
    assert len(det2.detect(frame)) == 1


def _face_outputs(hits):
    outs = {}
    for s in (8, 16, 32):
        n = (640 // s) ** 2 * 2
        sc, bb, kp = torch.full((1, n, 1), -9.0), torch.zeros(1, n, 4), torch.zeros(1, n, 10)
        for (stride, cell, anchor, score, box, kps) in hits:
            if stride == s:
                a = cell * 2 + anchor
                sc[0, a, 0], bb[0, a] = score, torch.tensor(box)
                kp[0, a] = torch.tensor(kps)
        outs[f"score{s}"], outs[f"bbox{s}"], outs[f"kps{s}"] = sc, bb, kp
    return outs


def test_face_detector_decoding_counting_and_alignment():
    kps = [-10, -8, 10, -8, 0, 2, -8, 12, 8, 12]
    cell = 5 * 40 + 7                                       # stride 16: column 7, row 5 -> centre (112, 80)
    hits = [(16, cell, 0, 4.0, [20, 24, 20, 24], kps), (16, cell, 1, 3.0, [19, 24, 21, 24], kps)]
    model = _const_model("input.1", (1, 3, 640, 640), _face_outputs(hits))
    det = RetinaFaceDetector(model)
    faces = det.detect_all(RgbImage(1280, 640))            # scale x 2, y 1
    assert len(faces) == 1
    f = faces[0]
    assert abs(f.x1 - (112 - 20) * 2) < 1e-4 and abs(f.y1 - (80 - 24)) < 1e-4 and abs(f.score - 1 / (1 + np.exp(-4))) < 1e-5
    assert abs(f.landmarks[0] - (112 - 10) * 2) < 1e-4
    assert [d.label for d in FaceCountDetector(det).detect(RgbImage(1280, 640))] == ["face"]
    # alignment: landmarks exactly at the template map every template point to itself
    img = RgbImage.from_pixel_data(np.random.default_rng(0).integers(0, 255, (112, 112, 3)).astype(np.uint8), 112, 112)
    lm = [v for p in zip(TEMPLATE_X, TEMPLATE_Y) for v in p]
    out = align_face(img, lm)
    assert np.abs(out.pixels.astype(int) - img.pixels.astype(int)).max() <= 1
    a, b, tx, ty = similarity_transform([(0, 0), (1, 0)], [(2, 2), (2, 4)])   # rotate 90, scale 2, shift
    assert np.allclose([a, b, tx, ty], [0, 2, 2, 2])


def _arcface_model(dim=16):
    """Flatten -> Gemm: a linear 'embedding network' over 3x112x112 inputs."""
    g = ox.Graph(name="arc", opset=13, inputs=[ox.ValueInfo("data", [-1, 3, 112, 112])])
    w = torch.randn(dim, 3 * 112 * 112, generator=torch.Generator().manual_seed(0)) * 0.01
    g.initializers["W"] = ox.TensorData.from_torch("W", w)
    g.nodes.append(ox.Node("f", "Flatten", ["data"], ["flat"], {"axis": ox.Attribute("axis", 2, i=1)}))
    g.nodes.append(ox.Node("g", "Gemm", ["flat", "W"], ["fc1"], {"transB": ox.Attribute("transB", 2, i=1)}))
    g.outputs.append(ox.ValueInfo("fc1", [-1, dim]))
    return ox.OnnxModel.load(ox.encode_model(g))


def _faces(n, seed=0):
    rng = np.random.default_rng(seed)
    return [RgbImage.from_pixel_data(rng.integers(0, 255, (96, 96, 3)).astype(np.uint8), 96, 96) for _ in range(n)]


def test_arcface_embedder_normalises_and_batches():
    emb = ArcFaceOnnxEmbedder(_arcface_model())
    ims = _faces(5)
    batch = emb.embed_batch(ims)
    one = emb.embed(ims[2])
    assert emb.dimension == 16 and np.allclose(batch[2], one, atol=1e-5)
    assert all(abs(np.linalg.norm(v) - 1) < 1e-5 for v in batch)


def test_pc_distilled_embedder_trains_persists_and_checks_its_probe():
    teacher = ArcFaceOnnxEmbedder(_arcface_model(8))
    ims = _faces(12, seed=1)
    with tempfile.TemporaryDirectory() as d:
        st = PcDistilledFaceEmbedder(d, teacher, hidden_dim=16, inference_steps=3, epochs=2, max_train=12)
        st.fit(ims)
        v = st.embed(ims[0])
        assert v.shape == (8,) and abs(np.linalg.norm(v) - 1) < 1e-4 and st.dimension == 8
        st.net.close()
        again = PcDistilledFaceEmbedder(d)                   # teacher-free reload
        assert np.allclose(again.embed(ims[0]), v, atol=1e-4)
        again.net.close()
        import json
        m = json.load(open(os.path.join(d, "distilled.json")))
        m["Probe"] = [p + 1.0 for p in m["Probe"]]
        json.dump(m, open(os.path.join(d, "distilled.json"), "w"))
        with pytest.raises(RuntimeError):
            PcDistilledFaceEmbedder(d).embed(ims[0])


def test_lfw_pairs_and_frame_stream():
    with tempfile.TemporaryDirectory() as d:
        with open(os.path.join(d, "pairs.txt"), "w") as f:
            f.write("2\t1\nAnn\t1\t2\nBob\t1\t3\nAnn\t1\tBob\t2\nCid\t4\tAnn\t3\n")
        ds = LfwDataset(os.path.join(d, "lfw"), os.path.join(d, "pairs.txt"))
        assert ds.fold_count == 2 and ds.total_pairs == 4
        f0 = ds.folds[0]
        assert f0[0] == (os.path.join(d, "lfw", "Ann", "Ann_0001.jpg"), os.path.join(d, "lfw", "Ann", "Ann_0002.jpg"), True)
        assert f0[1][2] is False and f0[1][1].endswith("Bob_0002.jpg")
        fr = os.path.join(d, "frames")
        os.makedirs(fr)
        for i in range(5):
            RgbImage(8, 4, fill=(i, 0, 0)).save_as_png(os.path.join(fr, f"{i:03d}.png"))
        got = [im.pixels[0, 0, 0] for im in FrameStream.read(fr, frame_stride=2)]
        assert got == [0, 2, 4] and FrameStream.grab_one(fr).width == 8
        with pytest.raises(RuntimeError):
            list(FrameStream.read("0"))
