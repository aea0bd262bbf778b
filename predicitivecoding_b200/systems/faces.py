"""Face recognition: uniform-LBP grid descriptors, Tan-Triggs illumination normalisation, PCA with
whitening (randomised subspace iteration, runs on the GPU when given CUDA tensors), predictive-coding
latent embedders, fused embedders, a face database, and LFW-style verification / identification
benchmarks.

Reference: PredictiveCoding.FaceRecognition/FaceDescriptor.cs:1-116 (central 62% square crop,
128x128 grey, 8x8 cells of 59-bin uniform LBP, per-cell Hellinger (sqrt of L1-normalised) then global
L2), Descriptors/FacePreprocessor.cs:1-126 (gamma 0.2, box-blur DoG radii 2/4, contrast equalisation
alpha 0.1, tau 10 tanh, min-max to bytes), Descriptors/PcaProjector.cs:1-222, EnhancedLbpEmbedder.cs,
PcFaceEmbedder.cs:1-103 (GenerativeNetwork [descriptor, 128, latent], prior 0.1), FusedEmbedder.cs,
Recognition/FaceDatabase.cs, Benchmark/FaceVerificationBenchmark.cs:1-182 (10-fold best-threshold
accuracy, AUC-ROC), FaceIdentificationBenchmark.cs.  Detection and ONNX teachers (RetinaFace, ArcFace)
are out of scope without model files; the ``systems.onnx`` runtime loads such models when present.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from ..pc.network import NetworkConfig
from ..pc.networks import GenerativeNetwork, GenerativeNetworkConfig
from .imaging import RgbImage

SIZE, GRID, BINS, CROP = 128, 8, 59, 0.62
DIMENSION = GRID * GRID * BINS


def _uniform_map() -> np.ndarray:
    m = np.full(256, 58, np.int64)
    nxt = 0
    for code in range(256):
        t = sum(((code >> i) & 1) != ((code >> ((i + 1) % 8)) & 1) for i in range(8))
        if t <= 2:
            m[code] = nxt
            nxt += 1
    return m


UNIFORM = _uniform_map()


def face_pixels(image: RgbImage) -> np.ndarray:
    side = max(1, int(min(image.width, image.height) * CROP))
    x0, y0 = (image.width - side) // 2, (image.height - side) // 2
    return image.crop(x0, y0, side, side).resize(SIZE, SIZE).to_gray()


def lbp_descriptor(gray: np.ndarray) -> np.ndarray:
    g = np.asarray(gray, np.int32).reshape(SIZE, SIZE)
    c = g[1:-1, 1:-1]
    nb = [g[:-2, :-2], g[:-2, 1:-1], g[:-2, 2:], g[1:-1, 2:], g[2:, 2:], g[2:, 1:-1], g[2:, :-2], g[1:-1, :-2]]
    code = sum((n >= c).astype(np.int64) << i for i, n in enumerate(nb))
    cell = SIZE // GRID
    ys, xs = np.meshgrid(np.arange(1, SIZE - 1), np.arange(1, SIZE - 1), indexing="ij")
    ci = np.minimum(ys // cell, GRID - 1) * GRID + np.minimum(xs // cell, GRID - 1)
    feat = np.zeros(DIMENSION, np.float64)
    np.add.at(feat, ci.ravel() * BINS + UNIFORM[code.ravel()], 1.0)
    f = feat.reshape(GRID * GRID, BINS)
    s = f.sum(1, keepdims=True)
    f = np.where(s > 0, np.sqrt(f / np.maximum(s, 1e-30)), 0).reshape(-1)
    n = np.linalg.norm(f)
    return (f / n if n > 0 else f).astype(np.float32)


def _box_blur(img: np.ndarray, r: int) -> np.ndarray:
    n = img.shape[0]
    idx = np.clip(np.arange(n)[:, None] + np.arange(-r, r + 1)[None], 0, n - 1)
    t = img[:, idx].mean(-1)
    return t[idx, :].mean(1)


def tan_triggs(gray: np.ndarray, gamma: float = 0.2, alpha: float = 0.1, tau: float = 10.0) -> np.ndarray:
    img = np.power(np.asarray(gray, np.float64).reshape(SIZE, SIZE) + 0.5, gamma)
    img = _box_blur(img, 2) - _box_blur(img, 4)
    scale = np.mean(np.power(np.abs(img) + 1e-6, alpha)) ** (1 / alpha)
    if scale > 1e-8:
        img = img / scale
    img = tau * np.tanh(img / tau)
    lo, hi = img.min(), img.max()
    if hi - lo <= 1e-8:
        return np.full(SIZE * SIZE, 128, np.uint8)
    return np.rint((img - lo) / (hi - lo) * 255).astype(np.uint8).reshape(-1)


class PcaProjector:
    """Top-k principal directions by subspace iteration with re-orthonormalisation, whitened."""

    def __init__(self):
        self.mean = self.components = self.scales = None

    @property
    def is_fit(self) -> bool:
        return self.components is not None

    def fit(self, data, target_dim: int, max_samples: int = 2000, iterations: int = 12, seed: int = 17):
        X = torch.as_tensor(np.asarray(data) if not torch.is_tensor(data) else data, dtype=torch.float32)
        g = torch.Generator().manual_seed(seed)
        if X.shape[0] > max_samples:
            X = X[torch.randperm(X.shape[0], generator=g)[:max_samples].to(X.device)]
        n, d = X.shape
        k = min(target_dim, n - 1, d)
        self.mean = X.mean(0)
        Xc = X - self.mean
        V = torch.linalg.qr(torch.randn(d, k, generator=g).to(X.device) * 2 - 1)[0]
        for _ in range(iterations):
            V = torch.linalg.qr(Xc.T @ (Xc @ V))[0]
        Z = Xc @ V
        var = (Z * Z).sum(0) / max(1, n - 1)
        order = torch.argsort(var, descending=True)
        self.components = V[:, order].T.contiguous()
        self.scales = 1.0 / torch.sqrt(var[order] + 1e-8)
        return self

    @property
    def output_dim(self) -> int:
        return self.components.shape[0]

    def project(self, x, whiten: bool = True) -> torch.Tensor:
        x = torch.as_tensor(np.asarray(x) if not torch.is_tensor(x) else x, dtype=torch.float32).to(self.mean.device)
        z = (x - self.mean) @ self.components.T
        return z * self.scales if whiten else z


def cosine(a, b) -> float:
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    d = np.linalg.norm(a) * np.linalg.norm(b)
    return float(a @ b / d) if d > 1e-12 else 0.0


class LbpEmbedder:
    name = "LBP 8x8x59"
    dimension = DIMENSION

    def fit(self, images: Sequence[RgbImage]) -> None:
        pass

    def embed(self, image: RgbImage) -> np.ndarray:
        return lbp_descriptor(face_pixels(image))


class EnhancedLbpEmbedder:
    def __init__(self, target_dim: int = 200, max_train: int = 2000):
        self.target_dim, self.max_train = target_dim, max_train
        self.pca = PcaProjector()
        self.name = f"Enhanced LBP (DoG + PCA {target_dim}-D)"

    def _desc(self, image: RgbImage) -> np.ndarray:
        return lbp_descriptor(tan_triggs(face_pixels(image)))

    def fit(self, images: Sequence[RgbImage]) -> None:
        self.pca.fit(np.stack([self._desc(im) for im in images[: self.max_train]]), self.target_dim, self.max_train)

    def embed(self, image: RgbImage) -> np.ndarray:
        if not self.pca.is_fit:
            raise RuntimeError("call fit() first")
        return self.pca.project(self._desc(image)).numpy()


class PcFaceEmbedder:
    """Latent of a generative PC network trained on LBP descriptors."""

    def __init__(self, latent_dim: int = 128, inference_steps: int = 8, epochs: int = 8, hidden: int = 128, seed: int = 1):
        self.latent, self.steps, self.epochs, self.hidden, self.seed = latent_dim, inference_steps, epochs, hidden, seed
        self.net: Optional[GenerativeNetwork] = None
        self.name = f"Predictive Coding latent ({latent_dim}-D)"

    def fit(self, images: Sequence[RgbImage]) -> None:
        cfg = GenerativeNetworkConfig(NetworkConfig(layer_sizes=(DIMENSION, self.hidden, self.latent),
                                                    activation="tanh", state_lr=0.1, weight_lr=0.01), 0.1)
        self.net = GenerativeNetwork(cfg, seed=self.seed)
        descs = [lbp_descriptor(face_pixels(im)) for im in images]
        rng = np.random.default_rng(7)
        for _ in range(self.epochs):
            for i in rng.permutation(len(descs)):
                self.net.learn(descs[i], self.steps)

    def embed(self, image: RgbImage) -> np.ndarray:
        if self.net is None:
            raise RuntimeError("call fit() first")
        return self.net.encode(lbp_descriptor(face_pixels(image)), self.steps).numpy()


class FusedEmbedder:
    """L2-normalised concatenation of several embedders (optionally weighted)."""

    def __init__(self, parts: Sequence, weights: Optional[Sequence[float]] = None):
        self.parts, self.weights = list(parts), list(weights or [1.0] * len(parts))
        self.name = " + ".join(p.name for p in self.parts)

    def fit(self, images) -> None:
        for p in self.parts:
            p.fit(images)

    def embed(self, image) -> np.ndarray:
        vs = []
        for p, w in zip(self.parts, self.weights):
            v = np.asarray(p.embed(image), np.float64)
            vs.append(w * v / (np.linalg.norm(v) + 1e-12))
        out = np.concatenate(vs)
        return (out / (np.linalg.norm(out) + 1e-12)).astype(np.float32)


class FaceDatabase:
    """Enrolled identities (mean embedding per person) with open-set identification."""

    def __init__(self, embedder, threshold: float = 0.5):
        self.embedder, self.threshold = embedder, threshold
        self.people: Dict[str, List[np.ndarray]] = {}

    def enroll(self, name: str, image: RgbImage) -> None:
        self.people.setdefault(name, []).append(self.embedder.embed(image))

    def identify(self, image: RgbImage) -> Tuple[Optional[str], float]:
        q = self.embedder.embed(image)
        best, score = None, -1.0
        for name, es in self.people.items():
            s = cosine(q, np.mean(es, 0))
            if s > score:
                best, score = name, s
        return (best if score >= self.threshold else None), score

    def remove(self, name: str) -> bool:
        return self.people.pop(name, None) is not None


@dataclass(frozen=True)
class VerificationResult:
    accuracy: float
    accuracy_std: float
    auc_roc: float
    best_threshold: float
    mean_same: float
    mean_diff: float
    pairs: int


def auc_roc(scores: Sequence[float], labels: Sequence[bool]) -> float:
    """Probability that a random positive scores above a random negative (ties count half)."""
    s = np.asarray(scores)
    y = np.asarray(labels, bool)
    pos, neg = s[y], s[~y]
    if len(pos) == 0 or len(neg) == 0:
        return float("nan")
    order = np.argsort(np.concatenate([pos, neg]), kind="mergesort")
    allv = np.concatenate([pos, neg])[order]
    ranks = np.empty(len(allv))
    i = 0
    while i < len(allv):
        j = i
        while j + 1 < len(allv) and allv[j + 1] == allv[i]:
            j += 1
        ranks[i:j + 1] = (i + j) / 2 + 1
        i = j + 1
    r = np.empty(len(allv))
    r[order] = ranks
    return float((r[:len(pos)].sum() - len(pos) * (len(pos) + 1) / 2) / (len(pos) * len(neg)))


def verification_benchmark(embedder, pairs: Sequence[Tuple[RgbImage, RgbImage, bool]], folds: int = 10
                           ) -> VerificationResult:
    scores = np.array([cosine(embedder.embed(a), embedder.embed(b)) for a, b, _ in pairs])
    labels = np.array([s for _, _, s in pairs], bool)
    idx = np.arange(len(pairs))
    accs, ths = [], []
    for f in range(folds):
        test = idx[f::folds]
        train = np.setdiff1d(idx, test)
        cand = np.unique(scores[train]) if len(train) else np.array([0.5])
        th = max(cand, key=lambda t: ((scores[train] >= t) == labels[train]).mean())
        ths.append(th)
        if len(test):
            accs.append(((scores[test] >= th) == labels[test]).mean())
    return VerificationResult(float(np.mean(accs)), float(np.std(accs)), auc_roc(scores, labels), float(np.mean(ths)),
                              float(scores[labels].mean()) if labels.any() else float("nan"),
                              float(scores[~labels].mean()) if (~labels).any() else float("nan"), len(pairs))


def identification_benchmark(embedder, gallery: Dict[str, RgbImage], probes: Sequence[Tuple[str, RgbImage]]) -> float:
    g = {n: embedder.embed(im) for n, im in gallery.items()}
    hits = 0
    for name, im in probes:
        q = embedder.embed(im)
        hits += max(g, key=lambda k: cosine(q, g[k])) == name
    return hits / max(1, len(probes))
