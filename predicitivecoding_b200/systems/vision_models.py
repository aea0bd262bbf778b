"""ONNX-model detectors and face embedders on the in-house ONNX executor, face alignment, the
predictive-coding distilled face embedder, LFW pair lists and frame streams.

Reference:
  PredictiveCoding.Vision/Detection/YoloPersonDetector.cs:21-170 (YOLOX: 640 letterbox filled with 114,
      B/G/R planes in 0-255, anchors at strides 8/16/32, score = objectness x P(person), NMS 0.45),
  Detection/FaceCountDetector.cs:14-34, Capture/FrameStream.cs,
  PredictiveCoding.FaceRecognition/FaceAlignment/RetinaFaceDetector.cs:24-260 (640x640, (c-127.5)/128,
      9 outputs grouped by last dimension 1/4/10 and sorted by anchor count, 2 anchors per cell,
      distance boxes and 5 keypoints from the anchor centre, score 0.5, NMS 0.4),
  FaceAlignment/FaceAligner.cs (least-squares similarity transform onto the 112x112 ArcFace landmark
      template, inverse bilinear warp, black outside the source),
  ArcFaceOnnxEmbedder.cs:23-200 (aligned or centre-cropped 112x112, (c-127.5)/127.5, L2-normalised),
  PcDistilledFaceEmbedder.cs:22-301 (supervised PC regression from LBP descriptors to teacher
      embeddings, persisted with a manifest and a probe that detects a silently reseeded store),
  Datasets/LfwDataset.cs (pairs.txt folds).

No model files ship with the reference (it downloads them); here every model is an ``OnnxModel``
the caller loads from a file or builds, so nothing touches the network.  The YOLOX template and the
ArcFace landmark template are published conventions kept as the models expect them.
"""
from __future__ import annotations

import json
import math
import os
import random
import shutil
from dataclasses import dataclass
from typing import Callable, Dict, Iterator, List, Optional, Sequence, Tuple

import numpy as np
import torch

from .imaging import RgbImage
from .onnx import OnnxModel
from .vision import Detection, nms

INPUT = 640
STRIDES = (8, 16, 32)


def _as_model(model) -> OnnxModel:
    return model if isinstance(model, OnnxModel) else OnnxModel.load(model)


# ----------------------------------------------------------------------------- YOLOX persons
class YoloPersonDetector:
    """YOLOX full-body detector: letterbox to 640 (padding value 114), B/G/R planes in raw 0-255,
    grid-anchor decoding at strides 8/16/32 (box centre = (offset + cell) * stride, size =
    exp(log-size) * stride), score = objectness * P(person), boxes back in frame pixels, NMS."""

    def __init__(self, model, score_threshold: float = 0.45, nms_threshold: float = 0.45, person_class: int = 0,
                 num_classes: int = 80):
        self.model = _as_model(model)
        self.score_threshold, self.nms_threshold = score_threshold, nms_threshold
        self.person_class, self.attrs = person_class, 5 + num_classes
        self.name = "YOLOX full-body (COCO person) - in-house runtime"

    @staticmethod
    def preprocess(frame: RgbImage) -> Tuple[torch.Tensor, float]:
        r = min(INPUT / frame.height, INPUT / frame.width)
        nw, nh = max(1, int(round(frame.width * r))), max(1, int(round(frame.height * r)))
        t = torch.full((1, 3, INPUT, INPUT), 114.0)
        px = torch.from_numpy(frame.resize(nw, nh).pixels.astype(np.float32))       # [h, w, RGB]
        t[0, :, :nh, :nw] = px.permute(2, 0, 1).flip(0)                            # B, G, R planes
        return t, r

    def _rows(self, out: torch.Tensor) -> Optional[torch.Tensor]:
        a = self.attrs
        if out.dim() == 3 and out.shape[2] == a:
            return out[0]
        if out.dim() == 3 and out.shape[1] == a:
            return out[0].T
        if out.dim() == 2 and out.shape[1] == a:
            return out
        return None

    def decode(self, out: torch.Tensor, r: float, width: int, height: int) -> List[Detection]:
        rows = self._rows(out)
        if rows is None:
            return []
        rows = rows.float()
        cand, anchor = [], 0
        for s in STRIDES:
            g = INPUT // s
            n = min(g * g, rows.shape[0] - anchor)
            if n <= 0:
                break
            blk = rows[anchor:anchor + n]
            gy, gx = torch.div(torch.arange(n), g, rounding_mode="floor"), torch.arange(n) % g
            score = blk[:, 4] * blk[:, 5 + self.person_class]
            keep = score >= self.score_threshold
            cx, cy = (blk[:, 0] + gx) * s, (blk[:, 1] + gy) * s
            w, h = torch.exp(blk[:, 2]) * s, torch.exp(blk[:, 3]) * s
            for i in torch.nonzero(keep).flatten().tolist():
                cand.append(Detection(min(max((cx[i] - w[i] / 2).item() / r, 0), width - 1),
                                      min(max((cy[i] - h[i] / 2).item() / r, 0), height - 1),
                                      min(max((cx[i] + w[i] / 2).item() / r, 0), width - 1),
                                      min(max((cy[i] + h[i] / 2).item() / r, 0), height - 1),
                                      float(score[i]), "person"))
            anchor += g * g
        return nms(cand, self.nms_threshold)

    def detect(self, frame: RgbImage) -> List[Detection]:
        t, r = self.preprocess(frame)
        out = self.model.run({self.model.input_names[0]: t})[self.model.output_names[0]]
        return self.decode(out, r, frame.width, frame.height)


# ----------------------------------------------------------------------------- faces
@dataclass
class FaceDetection:
    x1: float
    y1: float
    x2: float
    y2: float
    score: float
    landmarks: List[float]          # x0, y0, ..., x4, y4: eyes, nose, mouth corners

    @property
    def area(self) -> float:
        return (self.x2 - self.x1) * (self.y2 - self.y1)


class RetinaFaceDetector:
    """Anchor-free face detector with five keypoints (the SCRFD / RetinaFace family the reference
    loads): 640x640 input, (c - 127.5) / 128 in R/G/B planes; per stride a score map, a distance box
    map and a keypoint map, two anchors per cell at the cell's corner."""

    ANCHORS = 2

    def __init__(self, model, score_threshold: float = 0.5, nms_threshold: float = 0.4):
        self.model = _as_model(model)
        self.score_threshold, self.nms_threshold = score_threshold, nms_threshold

    @staticmethod
    def preprocess(image: RgbImage) -> torch.Tensor:
        px = torch.from_numpy(image.resize(INPUT, INPUT).pixels.astype(np.float32))
        return ((px - 127.5) / 128.0).permute(2, 0, 1)[None].contiguous()

    def detect_all(self, image: RgbImage) -> List[FaceDetection]:
        sx, sy = image.width / INPUT, image.height / INPUT
        outs = self.model.run({self.model.input_names[0]: self.preprocess(image)})
        known = {(INPUT // s) ** 2 * self.ANCHORS for s in STRIDES}
        groups: Dict[int, List[Tuple[int, torch.Tensor]]] = {1: [], 4: [], 10: []}
        for t in outs.values():
            if not t.is_floating_point():
                continue
            d = list(t.shape)
            if len(d) == 3:
                n, last = d[1], d[2]
            elif len(d) == 2:
                n, last = (d[1], 1) if d[0] == 1 and d[1] in known else (d[0], d[1])
            elif len(d) == 1:
                n, last = d[0], 1
            else:
                continue
            if n in known and last in groups:
                groups[last].append((n, t.reshape(n, last).float()))
        for g in groups.values():
            g.sort(key=lambda x: -x[0])
        if any(len(g) < 3 for g in groups.values()):
            return []
        cand = []
        for si, s in enumerate(STRIDES):
            w = INPUT // s
            (n, score), (_, box), (_, kps) = groups[1][si], groups[4][si], groups[10][si]
            p = torch.sigmoid(score[:, 0])
            for a in torch.nonzero(p >= self.score_threshold).flatten().tolist():
                cell = a // self.ANCHORS
                cx, cy = (cell % w) * s, (cell // w) * s
                b = box[a].tolist()
                k = kps[a].tolist()
                lm = []
                for j in range(5):
                    lm += [(cx + k[2 * j]) * sx, (cy + k[2 * j + 1]) * sy]
                cand.append(FaceDetection((cx - b[0]) * sx, (cy - b[1]) * sy, (cx + b[2]) * sx, (cy + b[3]) * sy,
                                          float(p[a]), lm))
        cand.sort(key=lambda f: -f.score)
        kept: List[FaceDetection] = []
        for f in cand:
            if all(_iou(f, k) <= self.nms_threshold for k in kept):
                kept.append(f)
        return kept

    def detect(self, image: RgbImage) -> Optional[FaceDetection]:
        """The most confident face, or None."""
        faces = self.detect_all(image)
        return faces[0] if faces else None


def _iou(a, b) -> float:
    ix = max(0.0, min(a.x2, b.x2) - max(a.x1, b.x1))
    iy = max(0.0, min(a.y2, b.y2) - max(a.y1, b.y1))
    inter = ix * iy
    union = a.area + b.area - inter
    return inter / union if union > 0 else 0.0


class FaceCountDetector:
    """Faces as people (head counting): every face box becomes a 'face' detection."""

    def __init__(self, detector: RetinaFaceDetector):
        self.detector = detector
        self.name = "RetinaFace (face / head count)"

    def detect(self, frame: RgbImage) -> List[Detection]:
        return [Detection(f.x1, f.y1, f.x2, f.y2, f.score, "face") for f in self.detector.detect_all(frame)]


# landmark template of 112x112 ArcFace inputs (left eye, right eye, nose tip, left / right mouth corner)
TEMPLATE_X = (38.2946, 73.5318, 56.0252, 41.5493, 70.7299)
TEMPLATE_Y = (51.6963, 51.5014, 71.7366, 92.3655, 92.2041)


def similarity_transform(src: Sequence[Tuple[float, float]], dst: Sequence[Tuple[float, float]]):
    """Least-squares rotation + isotropic scale + translation mapping src points onto dst:
    x' = a x - b y + tx, y' = b x + a y + ty (closed form from the centred point sets)."""
    s, d = np.asarray(src, np.float64), np.asarray(dst, np.float64)
    ms, md = s.mean(0), d.mean(0)
    sc, dc = s - ms, d - md
    den = (sc ** 2).sum()
    a = (sc[:, 0] * dc[:, 0] + sc[:, 1] * dc[:, 1]).sum() / den if den > 1e-10 else 1.0
    b = (sc[:, 0] * dc[:, 1] - sc[:, 1] * dc[:, 0]).sum() / den if den > 1e-10 else 0.0
    tx = md[0] - (a * ms[0] - b * ms[1])
    ty = md[1] - (b * ms[0] + a * ms[1])
    return a, b, tx, ty


def align_face(image: RgbImage, landmarks: Sequence[float], out_size: int = 112) -> RgbImage:
    """Warp a face onto the ArcFace template: similarity transform from the five detected landmarks,
    then each output pixel samples the source bilinearly (black outside it)."""
    k = out_size / 112.0
    src = [(landmarks[2 * i], landmarks[2 * i + 1]) for i in range(5)]
    dst = [(TEMPLATE_X[i] * k, TEMPLATE_Y[i] * k) for i in range(5)]
    a, b, tx, ty = similarity_transform(src, dst)
    det = a * a + b * b + 1e-10
    yd, xd = np.mgrid[0:out_size, 0:out_size].astype(np.float64)
    u, v = xd - tx, yd - ty
    xs, ys = (a * u + b * v) / det, (-b * u + a * v) / det
    px = image.pixels.astype(np.float64)
    H, W = image.height, image.width
    inside = (xs >= 0) & (ys >= 0) & (xs <= W - 1) & (ys <= H - 1)
    x0, y0 = np.clip(np.floor(xs).astype(int), 0, W - 1), np.clip(np.floor(ys).astype(int), 0, H - 1)
    x1, y1 = np.minimum(x0 + 1, W - 1), np.minimum(y0 + 1, H - 1)
    fx, fy = (xs - x0)[..., None], (ys - y0)[..., None]
    out = (px[y0, x0] * (1 - fx) * (1 - fy) + px[y0, x1] * fx * (1 - fy) + px[y1, x0] * (1 - fx) * fy
           + px[y1, x1] * fx * fy)
    out = np.where(inside[..., None], out, 0.0)
    return RgbImage.from_pixel_data(np.clip(np.rint(out), 0, 255).astype(np.uint8), out_size, out_size)


def _l2n(v: np.ndarray) -> np.ndarray:
    n = float(np.sqrt((v.astype(np.float64) ** 2).sum()))
    return (v / n).astype(np.float32) if n > 0 else v.astype(np.float32)


class ArcFaceOnnxEmbedder:
    """Teacher face embedder: detect + align (when a detector is given) or centre-crop, 112x112,
    (c - 127.5) / 127.5 in R/G/B planes, the model's embedding L2-normalised."""

    def __init__(self, model, detector: Optional[RetinaFaceDetector] = None, crop_fraction: float = 0.5,
                 batch_size: int = 64):
        self.model = _as_model(model)
        self.detector, self.crop, self.batch = detector, crop_fraction, batch_size
        self.dimension: Optional[int] = None
        self.name = "ArcFace" + (" +align" if detector is not None else "") + " - in-house runtime"

    def fit(self, images: Sequence[RgbImage]) -> None:   # pretrained: nothing to learn
        pass

    def preprocess(self, image: RgbImage) -> torch.Tensor:
        face = None
        if self.detector is not None:
            det = self.detector.detect(image)
            if det is not None:
                face = align_face(image, det.landmarks)
        if face is None:
            side = max(1, int(min(image.width, image.height) * self.crop))
            face = image.crop((image.width - side) // 2, (image.height - side) // 2, side, side).resize(112, 112)
        px = torch.from_numpy(face.pixels.astype(np.float32))
        return ((px - 127.5) / 127.5).permute(2, 0, 1).contiguous()

    def embed_batch(self, images: Sequence[RgbImage]) -> List[np.ndarray]:
        out: List[np.ndarray] = []
        for i in range(0, len(images), self.batch):
            x = torch.stack([self.preprocess(im) for im in images[i:i + self.batch]])
            y = self.model.run({self.model.input_names[0]: x})[self.model.output_names[0]]
            y = y.reshape(x.shape[0], -1).float().numpy()
            self.dimension = y.shape[1]
            out += [_l2n(r) for r in y]
        return out

    def embed(self, image: RgbImage) -> np.ndarray:
        return self.embed_batch([image])[0]


class PcDistilledFaceEmbedder:
    """A teacher's face embeddings distilled into a predictive-coding network (no backprop, no ONNX at
    inference): input clamped to the LBP descriptor, top clamped to the teacher's embedding, Hebbian
    learning; the embedding is the free-settled top state, L2-normalised.  The trained network lives in
    ``store_dir`` (a LayerStore plus ``distilled.json``), and the manifest keeps a probe - the first
    values of the embedding of a fixed reference input - that is recomputed on load so a missing or
    reseeded store is detected instead of serving random embeddings."""

    MANIFEST = "distilled.json"
    PROBE_LEN, PROBE_TOL = 8, 1e-3

    def __init__(self, store_dir: str, teacher=None, hidden_dim: int = 1024, inference_steps: int = 8,
                 epochs: int = 10, max_train: int = 2000, descriptor: Optional[Callable] = None):
        if hidden_dim < 1 or inference_steps < 1 or epochs < 1 or max_train < 1:
            raise ValueError("hidden_dim, inference_steps, epochs and max_train must be >= 1")
        from .faces import face_pixels, lbp_descriptor
        self.store_dir, self.teacher = store_dir, teacher
        self.hidden, self.steps, self.epochs, self.max_train = hidden_dim, inference_steps, epochs, max_train
        self.descriptor = descriptor or (lambda im: lbp_descriptor(face_pixels(im)))
        self.net = None
        self.manifest: Optional[dict] = None

    @property
    def dimension(self) -> int:
        m = self.manifest or self._peek()
        if m is not None:
            return m["OutputDim"]
        if self.teacher is not None and getattr(self.teacher, "dimension", None):
            return self.teacher.dimension
        raise RuntimeError(f"embedding dimension unknown: no trained store in {self.store_dir!r} and no teacher")

    def _peek(self) -> Optional[dict]:
        p = os.path.join(self.store_dir, self.MANIFEST)
        return json.load(open(p)) if os.path.exists(p) else None

    def _open(self, m: dict):
        from ..pc.network import Network, NetworkConfig
        cfg = NetworkConfig(layer_sizes=(m["InputDim"], m["HiddenDim"], m["OutputDim"]), activation="tanh",
                            state_lr=0.1, weight_lr=0.01, path=os.path.join(self.store_dir, "net"))
        return Network(cfg, seed=5)

    def _probe(self, m: dict) -> List[float]:
        ref = np.linspace(-1.0, 1.0, m["InputDim"], dtype=np.float32)
        top = self.net.infer_get_top(torch.from_numpy(ref), m["InferenceSteps"])
        return [float(v) for v in _l2n(top.numpy())[: self.PROBE_LEN]]

    def _try_load(self) -> bool:
        m = self._peek()
        if m is None:
            return False
        self.net = self._open(m)
        if any(abs(a - b) > self.PROBE_TOL for a, b in zip(self._probe(m), m["Probe"])):
            self.net.close()
            self.net = None
            raise RuntimeError(f"distilled store in {self.store_dir!r} does not reproduce its probe "
                               "(missing or corrupt weights); delete it and distil again")
        self.manifest = m
        return True

    def fit(self, images: Sequence[RgbImage]) -> None:
        if self.net is not None or self._try_load():
            return
        if self.teacher is None:
            raise RuntimeError(f"no trained model in {self.store_dir!r} and no teacher to distil from")
        rng = random.Random(7)
        sample = list(images)
        rng.shuffle(sample)
        sample = sample[: self.max_train]
        self.teacher.fit(sample)
        targets = self.teacher.embed_batch(sample)
        pairs = [(self.descriptor(im), t) for im, t in zip(sample, targets) if t is not None]
        if not pairs:
            raise RuntimeError("distillation produced no (descriptor, teacher embedding) pairs")
        shutil.rmtree(os.path.join(self.store_dir, "net"), ignore_errors=True)
        os.makedirs(self.store_dir, exist_ok=True)
        m = {"Version": 1, "InputDim": int(pairs[0][0].size), "HiddenDim": self.hidden,
             "OutputDim": int(pairs[0][1].size), "InferenceSteps": self.steps,
             "TeacherName": getattr(self.teacher, "name", "teacher"), "SampleCount": len(pairs),
             "Epochs": self.epochs, "Probe": []}
        try:
            self.net = self._open(m)
            xs = [torch.from_numpy(np.asarray(d, np.float32)) for d, _ in pairs]
            ys = [torch.from_numpy(np.asarray(t, np.float32)) for _, t in pairs]
            order = list(range(len(pairs)))
            shuf = random.Random(11)
            for _ in range(self.epochs):
                shuf.shuffle(order)
                for i in order:
                    self.net.learn(xs[i], ys[i], self.steps)
                self.net.flush_store()
            self.net.close()                 # durable now: reopen from the store
            self.net = self._open(m)
            m["Probe"] = self._probe(m)
            with open(os.path.join(self.store_dir, self.MANIFEST), "w") as f:
                json.dump(m, f)
            self.manifest = m
        except Exception:
            if self.net is not None:
                self.net.close()
            self.net = None
            shutil.rmtree(os.path.join(self.store_dir, "net"), ignore_errors=True)
            raise

    def embed(self, image: RgbImage) -> np.ndarray:
        if self.net is None and not self._try_load():
            raise RuntimeError("call fit() first")
        d = torch.from_numpy(np.asarray(self.descriptor(image), np.float32))
        return _l2n(self.net.infer_get_top(d, self.manifest["InferenceSteps"]).numpy())

    def embed_batch(self, images: Sequence[RgbImage]) -> List[np.ndarray]:
        return [self.embed(im) for im in images]


# ----------------------------------------------------------------------------- datasets and streams
class LfwDataset:
    """LFW verification folds from a pairs file: first line '<folds>\\t<pairs per fold>', then the
    matched pairs '<name>\\t<i1>\\t<i2>', then the mismatched '<n1>\\t<i1>\\t<n2>\\t<i2>'; pair k
    belongs to fold k // pairs_per_fold; images are <root>/<name>/<name>_<iiii>.jpg."""

    def __init__(self, images_root: str, pairs_file: str):
        self.root = images_root
        lines = open(pairs_file).read().splitlines()
        folds_n, per = (int(v) for v in lines[0].split("\t")[:2])
        total = folds_n * per
        self.folds: List[List[Tuple[str, str, bool]]] = [[] for _ in range(folds_n)]
        for i in range(total):
            if 1 + i < len(lines) and len(p := lines[1 + i].split("\t")) >= 3:
                self.folds[i // per].append((self._img(p[0], p[1]), self._img(p[0], p[2]), True))
        for i in range(total):
            if 1 + total + i < len(lines) and len(p := lines[1 + total + i].split("\t")) >= 4:
                self.folds[i // per].append((self._img(p[0], p[1]), self._img(p[2], p[3]), False))

    def _img(self, name: str, idx: str) -> str:
        return os.path.join(self.root, name, f"{name}_{int(idx):04d}.jpg")

    @property
    def fold_count(self) -> int:
        return len(self.folds)

    @property
    def total_pairs(self) -> int:
        return sum(len(f) for f in self.folds)

    def all_pairs(self) -> Iterator[Tuple[str, str, bool]]:
        for f in self.folds:
            yield from f

    def all_images(self) -> Iterator[Tuple[str, str]]:
        for name in sorted(os.listdir(self.root)):
            d = os.path.join(self.root, name)
            if os.path.isdir(d):
                for f in sorted(os.listdir(d)):
                    yield name, os.path.join(d, f)


class FrameStream:
    """Frames from a source, every ``frame_stride``-th one: a directory of images (Netpbm, PNG or BMP,
    sorted by name).  Camera indices, video files and network streams need a video-capture library,
    which this package does not bundle: those sources raise."""

    @staticmethod
    def _frames(source: str) -> Iterator[RgbImage]:
        if os.path.isdir(source):
            for f in sorted(os.listdir(source)):
                p = os.path.join(source, f)
                if os.path.isfile(p):
                    try:
                        yield RgbImage.load(p)
                    except ValueError:
                        continue
            return
        raise RuntimeError(f"could not open capture source {source!r}: pass a directory of images "
                           "(camera, video-file and network capture are not available in this package)")

    @classmethod
    def read(cls, source: str, frame_stride: int = 1) -> Iterator[RgbImage]:
        stride = max(1, frame_stride)
        for i, fr in enumerate(cls._frames(source)):
            if i % stride == 0:
                yield fr

    @classmethod
    def grab_one(cls, source: str) -> Optional[RgbImage]:
        try:
            return next(iter(cls._frames(source)), None)
        except RuntimeError:
            return None
