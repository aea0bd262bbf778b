"""In-house HOG detectors: linear hinge-loss model, linear regressor, sample trainer, sliding-window detector.

Reference: PredictiveCoding.Vision/Detection/Hog/LinearModel.cs (hinge SGD with L2 shrink,
``hoglinear v1 <label> <dim> <bias>`` text format), LinearRegressor.cs (squared-error SGD,
``linreg v1 <in> <out>`` rows of bias + weights), HogTrainer.cs (positives from teacher boxes,
random negatives with IoU <= 0.1 against them, aspect kept), HogPersonDetector.cs (image pyramid at
scale 1.2, stride of one cell, threshold, NMS 0.4).

The detector scores every window of a pyramid level with one matrix product (on the GPU when one
is present) instead of one dot product per window; the HOG of all windows of a level is computed
in one batched pass.
"""
from __future__ import annotations

import random
from typing import List, Optional, Sequence, Tuple

import numpy as np
import torch

from .imaging import RgbImage
from .vision import Detection, HogDescriptor, nms

Box = Tuple[int, int, int, int]  # x, y, w, h


def _fmt(v: float) -> str:
    return repr(float(np.float32(v)))


def _shuffle_order(n: int, rng: random.Random) -> List[int]:
    order = list(range(n))
    for i in range(n - 1, 0, -1):
        j = rng.randrange(i + 1)
        order[i], order[j] = order[j], order[i]
    return order


class LinearModel:
    """Linear classifier trained by hinge-loss SGD: score = w.x + b."""

    def __init__(self, dimension: int, label: str = "object"):
        if dimension < 1:
            raise ValueError("dimension must be >= 1")
        self.weights = np.zeros(dimension, np.float32)
        self.bias = 0.0
        self.label = label

    @property
    def dimension(self) -> int:
        return self.weights.size

    def score(self, features) -> float:
        f = np.asarray(features, np.float32)
        if f.size != self.dimension:
            raise ValueError(f"Expected {self.dimension} features, got {f.size}.")
        return float(np.dot(self.weights, f) + self.bias)

    def score_batch(self, features: np.ndarray) -> np.ndarray:
        f = np.asarray(features, np.float32)
        if torch.cuda.is_available() and f.shape[0] >= 256:
            w = torch.from_numpy(self.weights).cuda()
            return (torch.from_numpy(f).cuda() @ w + self.bias).cpu().numpy()
        return f @ self.weights + np.float32(self.bias)

    def predict(self, features, threshold: float = 0.0) -> bool:
        return self.score(features) >= threshold

    def train_step(self, features, label: int, lr: float, l2: float = 1e-4) -> None:
        f = np.asarray(features, np.float32)
        margin = label * self.score(f)
        self.weights *= np.float32(1.0 - lr * l2)
        if margin < 1.0:
            self.weights += np.float32(lr * label) * f
            self.bias += lr * label

    def fit(self, samples: Sequence[Tuple[np.ndarray, int]], epochs: int = 10, lr: float = 0.01,
            l2: float = 1e-4, seed: int = 1) -> None:
        rng = random.Random(seed)
        for _ in range(epochs):
            for k in _shuffle_order(len(samples), rng):
                f, y = samples[k]
                self.train_step(f, 1 if y >= 0 else -1, lr, l2)

    def save(self, path: str) -> None:
        with open(path, "w") as fh:
            fh.write(f"hoglinear v1 {self.label} {self.dimension} {_fmt(self.bias)}\n")
            for w in self.weights:
                fh.write(_fmt(w) + "\n")

    @staticmethod
    def load(path: str) -> "LinearModel":
        lines = open(path).read().split("\n")
        h = lines[0].split()
        if len(h) != 5 or h[0] != "hoglinear":
            raise ValueError("Bad linear-model header.")
        m = LinearModel(int(h[3]), h[2])
        m.bias = float(h[4])
        vals = [float(x) for x in lines[1:1 + m.dimension]]
        if len(vals) != m.dimension:
            raise ValueError("Truncated linear model.")
        m.weights = np.asarray(vals, np.float32)
        return m


class LinearRegressor:
    """Multi-output linear regression by squared-error SGD (used to distil embeddings)."""

    def __init__(self, input_dim: int, output_dim: int):
        if input_dim < 1 or output_dim < 1:
            raise ValueError("dimensions must be >= 1")
        self.w = np.zeros((output_dim, input_dim), np.float32)
        self.b = np.zeros(output_dim, np.float32)

    @property
    def input_dim(self) -> int:
        return self.w.shape[1]

    @property
    def output_dim(self) -> int:
        return self.w.shape[0]

    def predict(self, x) -> np.ndarray:
        x = np.asarray(x, np.float32)
        if x.size != self.input_dim:
            raise ValueError(f"Expected {self.input_dim} inputs, got {x.size}.")
        return self.w @ x + self.b

    def predict_normalized(self, x) -> np.ndarray:
        y = self.predict(x)
        n = float(np.sqrt((y.astype(np.float64) ** 2).sum()))
        return (y / n).astype(np.float32) if n > 1e-8 else y

    def train_step(self, x, target, lr: float, l2: float = 1e-5) -> None:
        x = np.asarray(x, np.float32)
        t = np.asarray(target, np.float32)
        if t.size != self.output_dim:
            raise ValueError("Target length mismatch.")
        err = self.predict(x) - t
        self.w -= np.float32(lr) * (err[:, None] * x[None, :] + np.float32(l2) * self.w)
        self.b -= np.float32(lr) * err

    def fit(self, samples: Sequence[Tuple[np.ndarray, np.ndarray]], epochs: int = 20, lr: float = 1e-3,
            l2: float = 1e-5, seed: int = 1) -> None:
        rng = random.Random(seed)
        for _ in range(epochs):
            for k in _shuffle_order(len(samples), rng):
                self.train_step(samples[k][0], samples[k][1], lr, l2)

    def save(self, path: str) -> None:
        with open(path, "w") as fh:
            fh.write(f"linreg v1 {self.input_dim} {self.output_dim}\n")
            for o in range(self.output_dim):
                fh.write(" ".join([_fmt(self.b[o])] + [_fmt(v) for v in self.w[o]]) + "\n")

    @staticmethod
    def load(path: str) -> "LinearRegressor":
        lines = open(path).read().split("\n")
        h = lines[0].split()
        if len(h) != 4 or h[0] != "linreg":
            raise ValueError("Bad regressor header.")
        r = LinearRegressor(int(h[2]), int(h[3]))
        for o in range(r.output_dim):
            row = [float(v) for v in lines[1 + o].split()]
            if len(row) != r.input_dim + 1:
                raise ValueError("Truncated regressor.")
            r.b[o], r.w[o] = row[0], row[1:]
        return r


def rect_iou(a: Box, b: Box) -> float:
    ix = max(0, min(a[0] + a[2], b[0] + b[2]) - max(a[0], b[0]))
    iy = max(0, min(a[1] + a[3], b[1] + b[3]) - max(a[1], b[1]))
    inter = ix * iy
    union = a[2] * a[3] + b[2] * b[3] - inter
    return inter / union if union > 0 else 0.0


class HogTrainer:
    """Collects labelled HOG samples (teacher boxes as positives, random boxes as negatives)."""

    def __init__(self, hog: HogDescriptor):
        self.hog = hog
        self.samples: List[Tuple[np.ndarray, int]] = []
        self.positive_count = 0
        self.negative_count = 0

    def add_positive(self, image: RgbImage, box: Box) -> None:
        self.samples.append((self.hog.from_crop(image, box), 1))
        self.positive_count += 1

    def add_negative(self, image: RgbImage, box: Box) -> None:
        self.samples.append((self.hog.from_crop(image, box), -1))
        self.negative_count += 1

    def add_sample(self, features, label: int) -> None:
        f = np.asarray(features, np.float32)
        if f.size != self.hog.dimension:
            raise ValueError("Feature length mismatch.")
        self.samples.append((f, 1 if label >= 0 else -1))
        if label >= 0:
            self.positive_count += 1
        else:
            self.negative_count += 1

    def add_random_negatives(self, image: RgbImage, avoid: Sequence[Box], count: int, rng: random.Random,
                             max_iou: float = 0.1, max_attempts: int = 0) -> int:
        ww, wh = self.hog.ww, self.hog.wh
        if image.width < ww or image.height < wh:
            return 0
        aspect = ww / wh
        added = attempts = 0
        limit = max_attempts if max_attempts > 0 else count * 20
        while added < count and attempts < limit:
            attempts += 1
            h = rng.randint(wh, image.height)
            w = min(max(int(h * aspect), ww), image.width)
            x = rng.randint(0, image.width - w)
            y = rng.randint(0, image.height - h)
            box = (x, y, w, h)
            if any(rect_iou(box, a) > max_iou for a in avoid):
                continue
            self.add_negative(image, box)
            added += 1
        return added

    def train(self, label: str, epochs: int = 15, lr: float = 0.01, l2: float = 1e-4, seed: int = 1) -> LinearModel:
        if not self.samples:
            raise ValueError("No samples to train on.")
        m = LinearModel(self.hog.dimension, label)
        m.fit(self.samples, epochs, lr, l2, seed)
        return m


class HogDetector:
    """Sliding-window detector over an image pyramid with a linear HOG model."""

    def __init__(self, hog: HogDescriptor, model: LinearModel, score_threshold: float = 0.0,
                 pyramid_scale: float = 1.2, stride_cells: int = 1, nms_iou: float = 0.4):
        if model.dimension != hog.dimension:
            raise ValueError("Model dimension does not match the HOG descriptor.")
        if pyramid_scale <= 1.0:
            raise ValueError("pyramid_scale must be > 1")
        if stride_cells < 1:
            raise ValueError("stride_cells must be >= 1")
        self.hog, self.model, self.threshold = hog, model, score_threshold
        self.scale, self.stride, self.nms_iou = pyramid_scale, stride_cells * hog.cell, nms_iou

    @property
    def name(self) -> str:
        return f"hog-{self.model.label}"

    def detect(self, frame: RgbImage) -> List[Detection]:
        raw: List[Detection] = []
        scale = 1.0
        while True:
            sw, sh = int(frame.width / scale), int(frame.height / scale)
            if sw < self.hog.ww or sh < self.hog.wh:
                break
            work = frame if scale == 1.0 else frame.resize(sw, sh)
            feats, corners = self.hog.windows(work, self.stride)
            if len(feats):
                scores = self.model.score_batch(feats)
                for (x, y), s in zip(corners, scores):
                    if s >= self.threshold:
                        ox, oy = x * scale, y * scale
                        raw.append(Detection(float(ox), float(oy), float(ox + self.hog.ww * scale),
                                             float(oy + self.hog.wh * scale), float(s), self.model.label))
            scale *= self.scale
        return nms(raw, self.nms_iou)
