"""People counting and tracking: detections, NMS, a SORT-style tracker with alpha-beta box filters,
line and zone counters, a median count smoother, colour-histogram re-identification with a person
gallery, HOG descriptors, the counting pipeline, and annotation (CPU drawing and a CUDA rasteriser).

Reference: PredictiveCoding.Vision/Detection/Detection.cs, Nms.cs:1-40 (score-sorted greedy NMS),
Tracking/Track.cs:1-80 (centre alpha 0.85, velocity beta 0.30, size alpha 0.50),
Tracking/SortTracker.cs:1-104 (greedy IoU matching, min_hits confirmation, max_age removal, unique
count), Counting/LineCounter.cs:1-88 (proper segment intersection, side by cross product),
ZoneCounter.cs:1-84 (even-odd point-in-polygon on the box's bottom-centre, dwell frames),
CountSmoother.cs (running median), ReId/ColorHistogramEmbedder.cs:1-68, PersonGallery.cs:1-80,
Detection/Hog/HogDescriptor.cs:1-143 (unsigned-gradient 9-bin cells, 2x2-cell L2-Hys-free L2 blocks),
Runtime/PeopleCountingPipeline.cs:1-133, Annotate.cs:11-117.
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass
from typing import Callable, Dict, Iterable, List, Optional, Sequence, Tuple

import numpy as np
import torch

from .imaging import Rgb24, RgbImage


@dataclass(frozen=True)
class Detection:
    x1: float
    y1: float
    x2: float
    y2: float
    score: float = 1.0
    label: str = "person"

    @property
    def width(self) -> float:
        return self.x2 - self.x1

    @property
    def height(self) -> float:
        return self.y2 - self.y1

    @property
    def area(self) -> float:
        return self.width * self.height

    @property
    def center_x(self) -> float:
        return (self.x1 + self.x2) * 0.5

    @property
    def center_y(self) -> float:
        return (self.y1 + self.y2) * 0.5


def iou(a: Detection, b: Detection) -> float:
    ix1, iy1 = max(a.x1, b.x1), max(a.y1, b.y1)
    ix2, iy2 = min(a.x2, b.x2), min(a.y2, b.y2)
    inter = max(0.0, ix2 - ix1) * max(0.0, iy2 - iy1)
    union = a.area + b.area - inter
    return inter / union if union > 0 else 0.0


def nms(boxes: List[Detection], iou_threshold: float) -> List[Detection]:
    kept: List[Detection] = []
    for d in sorted(boxes, key=lambda d: -d.score):
        if all(iou(d, k) <= iou_threshold for k in kept):
            kept.append(d)
    return kept


class Track:
    ALPHA, BETA, SIZE_ALPHA = 0.85, 0.30, 0.50

    def __init__(self, tid: int, d: Detection):
        self.id = tid
        self.cx, self.cy, self.w, self.h = d.center_x, d.center_y, d.width, d.height
        self.vcx = self.vcy = 0.0
        self.label = d.label
        self.hits, self.age, self.time_since_update = 1, 1, 0
        self.confirmed = False
        self.counted_unique = False

    x1 = property(lambda s: s.cx - s.w * 0.5)
    y1 = property(lambda s: s.cy - s.h * 0.5)
    x2 = property(lambda s: s.cx + s.w * 0.5)
    y2 = property(lambda s: s.cy + s.h * 0.5)
    center_x = property(lambda s: s.cx)
    center_y = property(lambda s: s.cy)

    def predict(self) -> None:
        self.cx += self.vcx
        self.cy += self.vcy
        self.age += 1
        self.time_since_update += 1

    def update(self, d: Detection) -> None:
        rx, ry = d.center_x - self.cx, d.center_y - self.cy
        self.cx += self.ALPHA * rx
        self.cy += self.ALPHA * ry
        self.vcx += self.BETA * rx
        self.vcy += self.BETA * ry
        self.w += self.SIZE_ALPHA * (d.width - self.w)
        self.h += self.SIZE_ALPHA * (d.height - self.h)
        self.label = d.label
        self.hits += 1
        self.time_since_update = 0

    def to_detection(self) -> Detection:
        return Detection(self.x1, self.y1, self.x2, self.y2, 1.0, self.label)


class SortTracker:
    def __init__(self, iou_threshold: float = 0.3, max_age: int = 30, min_hits: int = 3):
        self.iou_threshold, self.max_age, self.min_hits = iou_threshold, max(1, max_age), max(1, min_hits)
        self.tracks: List[Track] = []
        self.next_id = 1
        self.unique_count = 0

    @property
    def active_tracks(self) -> List[Track]:
        return [t for t in self.tracks if t.confirmed and t.time_since_update == 0]

    @property
    def current_count(self) -> int:
        return len(self.active_tracks)

    def update(self, dets: Sequence[Detection]) -> List[Track]:
        for t in self.tracks:
            t.predict()
        pairs = [(iou(d, t.to_detection()), i, k) for i, d in enumerate(dets) for k, t in enumerate(self.tracks)]
        pairs = sorted((p for p in pairs if p[0] >= self.iou_threshold), key=lambda p: -p[0])
        md, mt = set(), set()
        for _, i, k in pairs:
            if i in md or k in mt:
                continue
            md.add(i)
            mt.add(k)
            self.tracks[k].update(dets[i])
        for i, d in enumerate(dets):
            if i not in md:
                self.tracks.append(Track(self.next_id, d))
                self.next_id += 1
        for t in self.tracks:
            if not t.confirmed and t.hits >= self.min_hits:
                t.confirmed = True
            if t.confirmed and not t.counted_unique:
                t.counted_unique = True
                self.unique_count += 1
        self.tracks = [t for t in self.tracks if t.time_since_update <= self.max_age]
        return self.active_tracks

    def reset(self) -> None:
        self.tracks.clear()
        self.next_id = 1
        self.unique_count = 0


def _cross(ux, uy, vx, vy):
    return ux * vy - uy * vx


class LineCounter:
    def __init__(self, ax: float, ay: float, bx: float, by: float):
        if ax == bx and ay == by:
            raise ValueError("Line endpoints must differ.")
        self.a, self.b = (ax, ay), (bx, by)
        self.prev: Dict[int, Tuple[float, float]] = {}
        self.inbound = self.outbound = 0

    @property
    def net(self) -> int:
        return self.inbound - self.outbound

    @staticmethod
    def _intersect(p1, p2, p3, p4) -> bool:
        d1 = _cross(p4[0] - p3[0], p4[1] - p3[1], p1[0] - p3[0], p1[1] - p3[1])
        d2 = _cross(p4[0] - p3[0], p4[1] - p3[1], p2[0] - p3[0], p2[1] - p3[1])
        d3 = _cross(p2[0] - p1[0], p2[1] - p1[1], p3[0] - p1[0], p3[1] - p1[1])
        d4 = _cross(p2[0] - p1[0], p2[1] - p1[1], p4[0] - p1[0], p4[1] - p1[1])
        return ((d1 > 0 > d2) or (d1 < 0 < d2)) and ((d3 > 0 > d4) or (d3 < 0 < d4))

    def update(self, items) -> None:
        centres = [(t.id, t.center_x, t.center_y) if isinstance(t, Track) else t for t in items]
        (ax, ay), (bx, by) = self.a, self.b
        for tid, x, y in centres:
            p = self.prev.get(tid)
            if p is not None and self._intersect(p, (x, y), self.a, self.b):
                side = _cross(bx - ax, by - ay, x - ax, y - ay)
                if side > 0:
                    self.inbound += 1
                elif side < 0:
                    self.outbound += 1
            self.prev[tid] = (x, y)

    def forget(self, tid: int) -> None:
        self.prev.pop(tid, None)

    def reset(self) -> None:
        self.prev.clear()
        self.inbound = self.outbound = 0


class ZoneCounter:
    def __init__(self, polygon: Sequence[Tuple[float, float]]):
        if len(polygon) < 3:
            raise ValueError("A zone needs at least 3 vertices.")
        self.poly = list(polygon)
        self.ever_entered = set()
        self.dwell: Dict[int, int] = {}
        self.occupancy = 0

    @property
    def entered(self) -> int:
        return len(self.ever_entered)

    def dwell_frames(self, tid: int) -> int:
        return self.dwell.get(tid, 0)

    def is_inside(self, x: float, y: float) -> bool:
        inside = False
        n = len(self.poly)
        j = n - 1
        for i in range(n):
            xi, yi = self.poly[i]
            xj, yj = self.poly[j]
            if (yi > y) != (yj > y) and x < (xj - xi) * (y - yi) / (yj - yi) + xi:
                inside = not inside
            j = i
        return inside

    def update(self, items) -> None:
        pts = [(t.id, t.center_x, t.y2) if isinstance(t, Track) else t for t in items]
        occ = 0
        for tid, x, y in pts:
            if not self.is_inside(x, y):
                continue
            occ += 1
            self.ever_entered.add(tid)
            self.dwell[tid] = self.dwell.get(tid, 0) + 1
        self.occupancy = occ

    def reset(self) -> None:
        self.ever_entered.clear()
        self.dwell.clear()
        self.occupancy = 0


class CountSmoother:
    def __init__(self, window: int = 5):
        self.window = [0] * max(1, window)
        self.filled = self.head = 0

    def add(self, v: int) -> int:
        self.window[self.head] = v
        self.head = (self.head + 1) % len(self.window)
        self.filled = min(self.filled + 1, len(self.window))
        return sorted(self.window[:self.filled])[self.filled // 2]


class ColorHistogramEmbedder:
    name = "color-histogram"

    def __init__(self, bins_per_channel: int = 8, central_crop: float = 0.6):
        if not 1 <= bins_per_channel <= 256 or not 0 < central_crop <= 1:
            raise ValueError("invalid embedder parameters")
        self.bins, self.crop = bins_per_channel, central_crop

    @property
    def dimension(self) -> int:
        return 3 * self.bins

    def embed(self, frame: RgbImage, box: Detection) -> np.ndarray:
        mx, my = box.width * (1 - self.crop) * 0.5, box.height * (1 - self.crop) * 0.5
        cl = lambda v, hi: int(min(max(v, 0), hi))
        x0, y0 = cl(round(box.x1 + mx), frame.width - 1), cl(round(box.y1 + my), frame.height - 1)
        x1, y1 = cl(round(box.x2 - mx), frame.width - 1), cl(round(box.y2 - my), frame.height - 1)
        hist = np.zeros(3 * self.bins, np.float32)
        reg = frame.pixels[y0:y1 + 1, x0:x1 + 1].reshape(-1, 3).astype(np.int64)
        if reg.size == 0:
            return hist
        b = np.minimum(self.bins - 1, reg * self.bins // 256)
        for c in range(3):
            hist[c * self.bins:(c + 1) * self.bins] += np.bincount(b[:, c], minlength=self.bins)
        n = float(np.sqrt((hist.astype(np.float64) ** 2).sum()))
        return hist / n if n > 1e-8 else hist


class PersonGallery:
    def __init__(self, match_threshold: float = 0.6):
        if not 0 <= match_threshold <= 1:
            raise ValueError("match_threshold must be in [0, 1]")
        self.people: List[Tuple[int, np.ndarray]] = []
        self.threshold = match_threshold
        self.next_id = 1

    @property
    def count(self) -> int:
        return len(self.people)

    @staticmethod
    def _cos(a, b) -> float:
        d = float(np.linalg.norm(a) * np.linalg.norm(b))
        return float(np.dot(a, b)) / d if d > 1e-12 else 0.0

    def identify(self, emb) -> Optional[Tuple[int, float]]:
        if not self.people:
            return None
        return max(((pid, self._cos(emb, e)) for pid, e in self.people), key=lambda p: p[1])

    def identify_or_register(self, emb) -> int:
        m = self.identify(emb)
        if m is not None and m[1] >= self.threshold:
            return m[0]
        pid = self.next_id
        self.next_id += 1
        self.people.append((pid, np.array(emb, np.float32)))
        return pid

    def reset(self) -> None:
        self.people.clear()
        self.next_id = 1


class HogDescriptor:
    def __init__(self, window_width: int = 64, window_height: int = 128, cell_size: int = 8, bins: int = 9):
        if cell_size < 2 or bins < 2 or window_width % cell_size or window_height % cell_size:
            raise ValueError("invalid HOG geometry")
        self.ww, self.wh, self.cell, self.bins = window_width, window_height, cell_size, bins
        self.cx, self.cy = window_width // cell_size, window_height // cell_size
        self.dimension = max(0, self.cx - 1) * max(0, self.cy - 1) * 4 * bins
        if self.dimension == 0:
            raise ValueError("Window too small for a 2x2 block grid.")

    def compute_gray(self, gray: np.ndarray) -> np.ndarray:
        return self.compute_gray_batch(np.asarray(gray, np.float32).reshape(1, self.wh, self.ww))[0]

    def compute_gray_batch(self, grays: np.ndarray) -> np.ndarray:
        """HOG of N windows at once: [N, wh, ww] luma -> [N, dimension] (clamped central differences,
        unsigned 9-bin orientation, 2x2-cell blocks, L2 normalisation)."""
        g = np.asarray(grays, np.float32).reshape(-1, self.wh, self.ww)
        n = g.shape[0]
        xp, xm = np.clip(np.arange(self.ww) + 1, 0, self.ww - 1), np.clip(np.arange(self.ww) - 1, 0, self.ww - 1)
        yp, ym = np.clip(np.arange(self.wh) + 1, 0, self.wh - 1), np.clip(np.arange(self.wh) - 1, 0, self.wh - 1)
        gx = g[:, :, xp] - g[:, :, xm]
        gy = g[:, yp, :] - g[:, ym, :]
        mag = np.sqrt(gx * gx + gy * gy)
        ang = np.degrees(np.arctan2(gy, gx))
        ang = np.where(ang < 0, ang + 180, ang)
        ang = np.where(ang >= 180, ang - 180, ang)
        b = np.minimum(self.bins - 1, (ang / (180.0 / self.bins)).astype(np.int64))
        cell_idx = (np.arange(self.wh)[:, None] // self.cell) * self.cx + np.arange(self.ww)[None, :] // self.cell
        flat = (np.arange(n)[:, None, None] * (self.cy * self.cx) + cell_idx[None]) * self.bins + b
        hist = np.bincount(flat.reshape(-1), weights=mag.reshape(-1).astype(np.float64),
                           minlength=n * self.cy * self.cx * self.bins).reshape(n, self.cy, self.cx, self.bins)
        blk = np.concatenate([hist[:, :-1, :-1], hist[:, :-1, 1:], hist[:, 1:, :-1], hist[:, 1:, 1:]], axis=-1)
        # block layout: cells (y, x), (y, x+1), (y+1, x), (y+1, x+1), bins innermost
        norm = np.sqrt((blk * blk).sum(-1, keepdims=True) + 1e-6 ** 2)
        return (blk / norm).reshape(n, -1).astype(np.float32)

    @staticmethod
    def _luma(pixels: np.ndarray) -> np.ndarray:
        p = pixels.astype(np.float32)
        return 0.299 * p[..., 0] + 0.587 * p[..., 1] + 0.114 * p[..., 2]

    def from_window(self, image: RgbImage, x0: int, y0: int) -> np.ndarray:
        """HOG of the window whose top-left corner is (x0, y0) (HogDescriptor.cs:109-120)."""
        return self.compute_gray(self._luma(image.pixels[y0:y0 + self.wh, x0:x0 + self.ww]))

    def from_crop(self, image: RgbImage, box: Tuple[int, int, int, int]) -> np.ndarray:
        """HOG of an (x, y, w, h) box cropped and resized to the window (HogDescriptor.cs:124-140)."""
        x, y, w, h = box
        x0, y0 = max(0, x), max(0, y)
        x1, y1 = min(image.width, x + w), min(image.height, y + h)
        if x1 <= x0 or y1 <= y0:
            return np.zeros(self.dimension, np.float32)
        crop = image.crop(x0, y0, x1 - x0, y1 - y0).resize(self.ww, self.wh)
        return self.compute_gray(self._luma(crop.pixels))

    def windows(self, image: RgbImage, stride: int) -> Tuple[np.ndarray, np.ndarray]:
        """Every window at the given stride: ([N, dimension] features, [N, 2] top-left corners)."""
        lum = self._luma(image.pixels)
        ys = np.arange(0, image.height - self.wh + 1, stride)
        xs = np.arange(0, image.width - self.ww + 1, stride)
        if len(ys) == 0 or len(xs) == 0:
            return np.zeros((0, self.dimension), np.float32), np.zeros((0, 2), np.int64)
        view = np.lib.stride_tricks.sliding_window_view(lum, (self.wh, self.ww))[ys][:, xs]
        corners = np.stack(np.meshgrid(xs, ys), -1).reshape(-1, 2)
        return self.compute_gray_batch(view.reshape(-1, self.wh, self.ww)), corners


@dataclass(frozen=True)
class PipelineResult:
    frame_index: int
    detected: bool
    tracks: List[Track]
    current_count: int
    unique_count: int


class PeopleCountingPipeline:
    def __init__(self, detector: Callable[[RgbImage], List[Detection]], tracker: SortTracker, detect_every_n: int = 1):
        if detect_every_n < 1:
            raise ValueError("detect_every_n must be >= 1")
        self.detector, self.tracker, self.every = detector, tracker, detect_every_n
        self.processed = self.detection_frames = 0
        self.last: List[Detection] = []
        self.t0 = None

    @property
    def fps(self) -> float:
        dt = time.perf_counter() - self.t0 if self.t0 else 0
        return self.processed / dt if dt > 1e-6 else 0.0

    def process(self, frame: RgbImage) -> PipelineResult:
        if self.t0 is None:
            self.t0 = time.perf_counter()
        det = self.processed % self.every == 0
        if det:
            self.last = self.detector(frame)
            self.detection_frames += 1
        tracks = self.tracker.update(self.last)
        idx = self.processed
        self.processed += 1
        return PipelineResult(idx, det, tracks, self.tracker.current_count, self.tracker.unique_count)

    def run(self, frames: Iterable[RgbImage], on_result: Optional[Callable] = None) -> None:
        for f in frames:
            r = self.process(f)
            if on_result:
                on_result(r)


# ---------------------------------------------------------------- annotation
DET_COLOR = Rgb24(0, 255, 0)
LINE_COLOR = Rgb24(255, 220, 32)
ZONE_COLOR = Rgb24(32, 230, 230)
PALETTE = [Rgb24(255, 64, 64), Rgb24(64, 255, 64), Rgb24(64, 160, 255), Rgb24(255, 220, 32),
           Rgb24(255, 64, 255), Rgb24(32, 230, 230), Rgb24(255, 150, 40), Rgb24(170, 110, 255)]


def _clamped_box(img: RgbImage, x1, y1, x2, y2):
    c = lambda v, hi: min(max(int(v), 0), hi)
    return c(x1, img.width - 1), c(y1, img.height - 1), c(x2, img.width - 1), c(y2, img.height - 1)


def _line_segments(ax, ay, bx, by, thickness) -> List[Tuple[int, int, int, int]]:
    dx, dy = bx - ax, by - ay
    ln = math.sqrt(dx * dx + dy * dy)
    if ln < 1e-3:
        return []
    px, py = -dy / ln, dx / ln
    half = max(0, thickness // 2)
    r = lambda v: int(round(v))          # round half to even, as the reference's MathF.Round
    return [(r(ax + px * o), r(ay + py * o), r(bx + px * o), r(by + py * o)) for o in range(-half, half + 1)]


class Annotator:
    """Collects boxes and lines in drawing order; ``render_cpu`` draws them the reference way,
    ``render_cuda`` rasterises them on the GPU with identical pixels."""

    def __init__(self, thickness: int = 2):
        self.t = thickness
        self.boxes: List[Tuple[Tuple[float, float, float, float], Rgb24]] = []
        self.segments: List[Tuple[Tuple[int, int, int, int], Rgb24]] = []

    def draw_boxes(self, dets: Sequence[Detection]) -> "Annotator":
        self.boxes += [((d.x1, d.y1, d.x2, d.y2), DET_COLOR) for d in dets]
        return self

    def draw_tracks(self, tracks: Sequence[Track]) -> "Annotator":
        self.boxes += [((t.x1, t.y1, t.x2, t.y2), PALETTE[t.id % len(PALETTE)]) for t in tracks]
        return self

    def draw_line(self, ax, ay, bx, by, color: Optional[Rgb24] = None, thickness: Optional[int] = None) -> "Annotator":
        c = color or LINE_COLOR
        self.segments += [(s, c) for s in _line_segments(ax, ay, bx, by, thickness or self.t)]
        return self

    def draw_zone(self, polygon, color: Optional[Rgb24] = None) -> "Annotator":
        for i in range(len(polygon)):
            (ax, ay), (bx, by) = polygon[i], polygon[(i + 1) % len(polygon)]
            self.draw_line(ax, ay, bx, by, color or ZONE_COLOR)
        return self

    def render_cpu(self, img: RgbImage) -> RgbImage:
        p = img.pixels
        H, W = img.height, img.width
        for (x1, y1, x2, y2), c in self.boxes:
            x1, y1, x2, y2 = _clamped_box(img, x1, y1, x2, y2)
            for k in range(self.t):
                for y in (y1 + k, y2 - k):
                    if 0 <= y < H and x2 >= x1:
                        p[y, max(0, x1):min(W - 1, x2) + 1] = c
                for x in (x1 + k, x2 - k):
                    if 0 <= x < W and y2 >= y1:
                        p[max(0, y1):min(H - 1, y2) + 1, x] = c
        for (x0, y0, x1, y1), c in self.segments:
            dx, sx = abs(x1 - x0), 1 if x0 < x1 else -1
            dy, sy = -abs(y1 - y0), 1 if y0 < y1 else -1
            err = dx + dy
            while True:
                if 0 <= x0 < W and 0 <= y0 < H:
                    p[y0, x0] = c
                if x0 == x1 and y0 == y1:
                    break
                e2 = 2 * err
                if e2 >= dy:
                    err += dy
                    x0 += sx
                if e2 <= dx:
                    err += dx
                    y0 += sy
        return img

    def render_cuda(self, img: torch.Tensor) -> torch.Tensor:
        """img: [H, W, 3] uint8 CUDA tensor, drawn in place."""
        from .. import ops
        H, W = img.shape[0], img.shape[1]
        cl = lambda v, hi: min(max(int(v), 0), hi)
        boxes = [(cl(a, W - 1), cl(b, H - 1), cl(c, W - 1), cl(d, H - 1)) for (a, b, c, d), _ in self.boxes]
        dev = img.device
        bt = torch.tensor(boxes, dtype=torch.int32, device=dev).reshape(-1)
        st = torch.tensor([s for s, _ in self.segments], dtype=torch.int32, device=dev).reshape(-1)
        cols = torch.tensor([list(c) for _, c in self.boxes] + [list(c) for _, c in self.segments],
                            dtype=torch.uint8, device=dev).reshape(-1)
        owner = torch.empty(H * W, dtype=torch.int32, device=dev)
        ops.ext().annotate(img, bt, self.t, st, cols if cols.numel() else torch.zeros(3, dtype=torch.uint8, device=dev),
                           owner)
        return img
