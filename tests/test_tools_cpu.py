"""In-house HOG detectors, distillation, ONNX packing and language identification tools (CPU)."""
import random

import numpy as np
import pytest
import torch

from predicitivecoding_b200.cli import detector_distiller, lang_detect_smoke, onnx_pack
from predicitivecoding_b200.systems import onnx as ox
from predicitivecoding_b200.systems.data import LanguageDetector, LanguageProfile, default_language_classifier
from predicitivecoding_b200.systems.detectors import HogDetector, HogTrainer, LinearModel, LinearRegressor, rect_iou
from predicitivecoding_b200.systems.imaging import RgbImage
from predicitivecoding_b200.systems.vision import HogDescriptor


def _scene(rng, boxes, w=160, h=200):
    px = (rng.random((h, w, 3)) * 60).astype(np.uint8)
    for x, y, bw, bh in boxes:
        px[y:y + bh, x:x + bw] = 230
        px[y + bh // 4:y + 3 * bh // 4, x + bw // 4:x + 3 * bw // 4] = 20
    return RgbImage.from_pixel_data(px, w, h)


def test_hog_batch_equals_single_windows():
    rng = np.random.default_rng(0)
    img = _scene(rng, [(10, 20, 64, 128)])
    hog = HogDescriptor(64, 128)
    feats, corners = hog.windows(img, 8)
    for k in (0, 5, len(corners) - 1):
        x, y = corners[k]
        np.testing.assert_allclose(feats[k], hog.from_window(img, int(x), int(y)), atol=1e-6)


def test_linear_model_and_regressor_roundtrip(tmp_path):
    rng = np.random.default_rng(1)
    X = rng.normal(size=(200, 12)).astype(np.float32)
    y = np.where(X[:, 0] + 0.5 * X[:, 3] > 0, 1, -1)
    m = LinearModel(12, "thing")
    m.fit(list(zip(X, y)), epochs=20, lr=0.05)
    acc = np.mean([(m.score(x) >= 0) == (t > 0) for x, t in zip(X, y)])
    assert acc > 0.95
    m.save(tmp_path / "m.txt")
    m2 = LinearModel.load(tmp_path / "m.txt")
    assert m2.label == "thing" and np.allclose(m2.weights, m.weights) and m2.bias == pytest.approx(m.bias)
    np.testing.assert_allclose(m.score_batch(X[:5]), [m.score(x) for x in X[:5]], rtol=1e-5, atol=1e-5)
    W = rng.normal(size=(3, 12)).astype(np.float32)
    r = LinearRegressor(12, 3)
    r.fit([(x, W @ x) for x in X], epochs=30, lr=0.02)
    assert np.abs(r.predict(X[0]) - W @ X[0]).max() < 0.05
    assert np.linalg.norm(r.predict_normalized(X[0])) == pytest.approx(1.0, abs=1e-5)
    r.save(tmp_path / "r.txt")
    np.testing.assert_allclose(LinearRegressor.load(tmp_path / "r.txt").predict(X[1]), r.predict(X[1]), atol=1e-5)


def test_trainer_negatives_avoid_positives_and_detector_finds_object():
    rng = np.random.default_rng(2)
    prng = random.Random(3)
    hog = HogDescriptor(32, 64)
    tr = HogTrainer(hog)
    for _ in range(12):
        x, y = int(rng.integers(0, 100)), int(rng.integers(0, 100))
        box = (x, y, 32, 64)
        img = _scene(rng, [box])
        tr.add_positive(img, box)
        assert tr.add_random_negatives(img, [box], 4, prng) > 0
    assert tr.positive_count == 12 and tr.negative_count > 0
    model = tr.train("object", epochs=15)
    det = HogDetector(hog, model, score_threshold=0.0, pyramid_scale=1.5)
    truth = (72, 96, 32, 64)
    found = det.detect(_scene(rng, [truth]))
    assert found
    best = max(found, key=lambda d: d.score)
    assert rect_iou((int(best.x1), int(best.y1), int(best.width), int(best.height)), truth) > 0.5


def test_distill_writes_models(tmp_path):
    rng = np.random.default_rng(4)
    frames, boxes = [], []
    for i in range(12):
        b = (int(rng.integers(0, 90)), int(rng.integers(0, 60)), 64, 128)
        frames.append(_scene(rng, [b]))
        boxes.append(b)
    face_box = {id(f): (b[0] + 8, b[1] + 8, 48, 48) for f, b in zip(frames, boxes)}
    rep = detector_distiller.distill(
        frames, lambda f: [boxes[frames.index(f)]], lambda f: [face_box[id(f)]],
        lambda f, b: rng.normal(size=8).tolist(), str(tmp_path), neg_per_frame=3, epochs=3)
    names = sorted(p.split("/")[-1] for p in rep.written)
    assert names == ["face-embedder.txt", "hog-face.txt", "hog-person.txt"]
    assert LinearModel.load(str(tmp_path / "hog-person.txt")).dimension == HogDescriptor(64, 128).dimension


def test_onnx_pack_cli(tmp_path, capsys):
    w = torch.randn(4, 3)
    # the inner Identity is elided; the one producing the graph output "y" is kept
    g = ox.Graph("g", 13, [ox.Node("id0", "Identity", ["x"], ["u"]), ox.Node("mm", "MatMul", ["u", "w"], ["t"]),
                           ox.Node("id", "Identity", ["t"], ["y"])],
                 {"w": ox.TensorData("w", ox.FLOAT, [4, 3], w.numpy().reshape(-1))},
                 [ox.ValueInfo("x", [2, 4])], [ox.ValueInfo("y", [2, 3])])
    src = tmp_path / "m.onnx"
    src.write_bytes(ox.encode_model(g))
    assert onnx_pack.main([str(src)]) == 0
    out = capsys.readouterr().out
    assert "nodes        : 3 -> 2" in out
    x = torch.randn(2, 4)
    np.testing.assert_allclose(ox.OnnxModel.load(str(tmp_path / "m.pcnx")).run({"x": x})["y"], x @ w, rtol=1e-5)
    assert onnx_pack.main([str(src), str(src)]) == 1
    assert onnx_pack.main(["--bogus", str(src)]) == 1


def test_language_detectors(tmp_path):
    d = LanguageDetector.create_default(seed=42)
    assert d.detect("Questo testo è scritto in italiano e parla della città.") == "Italian"
    assert d.detect("Wir gehen morgen früh mit den Kindern in die Stadt.") == "German"
    assert d.detect("12345 !!!") == "Unknown"
    probs = d.detect_all("The children are reading the newspaper in the garden.")
    assert probs[0].language == "English" and probs[0].probability > 0.5
    prof = LanguageProfile.from_texts("xx", ["abc abd"])
    prof.save(str(tmp_path / "xx"))
    again = LanguageProfile.load(str(tmp_path / "xx"))
    assert again.freq == prof.freq and again.n_words == prof.n_words
    assert default_language_classifier().predict("la casa è molto bella e il giardino è grande") == "Italian"
    assert lang_detect_smoke.main([]) == 0
