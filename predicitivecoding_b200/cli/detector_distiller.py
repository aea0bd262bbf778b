"""Distil teacher detections into in-house HOG detectors and a face embedder.

Reference: tools/DetectorDistiller/Program.cs (YOLOX person boxes -> HOG person detector, RetinaFace
face boxes -> HOG face detector, ArcFace embeddings -> linear regressor from face HOG; outputs
``hog-person.txt``, ``hog-face.txt``, ``face-embedder.txt``).  The teachers are callables
(``frame -> boxes`` / ``(frame, box) -> embedding``); the command line reads their labels from a
JSON file produced offline: ``{"<image file>": {"person": [[x,y,w,h],...], "face": [[x,y,w,h],...],
"face_embedding": [[...], ...]}}`` with one embedding per face box.
"""
from __future__ import annotations

import json
import os
import random
import sys
from dataclasses import dataclass
from typing import Callable, Iterable, List, Optional, Sequence, Tuple

import numpy as np

from ..systems.detectors import Box, HogTrainer, LinearRegressor
from ..systems.imaging import RgbImage
from ..systems.vision import HogDescriptor

Teacher = Callable[[RgbImage], Sequence[Box]]
Embedder = Callable[[RgbImage, Box], Optional[Sequence[float]]]


@dataclass
class DistillReport:
    frames: int
    person_pos: int
    person_neg: int
    face_pos: int
    face_neg: int
    embed_pairs: int
    written: List[str]


def distill(frames: Iterable[RgbImage], person_teacher: Optional[Teacher], face_teacher: Optional[Teacher],
            embed_teacher: Optional[Embedder], out_dir: str, neg_per_frame: int = 5, epochs: int = 20,
            seed: int = 7) -> DistillReport:
    os.makedirs(out_dir, exist_ok=True)
    rng = random.Random(seed)
    hog_p, hog_f = HogDescriptor(64, 128), HogDescriptor(48, 48)
    tp, tf = HogTrainer(hog_p), HogTrainer(hog_f)
    pairs: List[Tuple[np.ndarray, np.ndarray]] = []
    n = 0
    for frame in frames:
        n += 1
        if person_teacher is not None:
            boxes = list(person_teacher(frame))
            for b in boxes:
                tp.add_positive(frame, b)
            tp.add_random_negatives(frame, boxes, neg_per_frame, rng)
        if face_teacher is not None:
            boxes = list(face_teacher(frame))
            for b in boxes:
                tf.add_positive(frame, b)
            tf.add_random_negatives(frame, boxes, neg_per_frame, rng)
            if embed_teacher is not None:
                for b in boxes:
                    e = embed_teacher(frame, b)
                    if e is not None:
                        pairs.append((hog_f.from_crop(frame, b), np.asarray(e, np.float32)))
    written = []
    if tp.positive_count:
        p = os.path.join(out_dir, "hog-person.txt")
        tp.train("person", epochs=epochs).save(p)
        written.append(p)
    if tf.positive_count:
        p = os.path.join(out_dir, "hog-face.txt")
        tf.train("face", epochs=epochs).save(p)
        written.append(p)
    if len(pairs) >= 10:
        p = os.path.join(out_dir, "face-embedder.txt")
        reg = LinearRegressor(hog_f.dimension, pairs[0][1].size)
        reg.fit(pairs, epochs=30, lr=1e-3)
        reg.save(p)
        written.append(p)
    return DistillReport(n, tp.positive_count, tp.negative_count, tf.positive_count, tf.negative_count, len(pairs),
                         written)


def _arg(argv, key, default=None):
    return argv[argv.index(key) + 1] if key in argv and argv.index(key) + 1 < len(argv) else default


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    src, labels = _arg(argv, "--source"), _arg(argv, "--labels")
    if src is None or labels is None:
        print("Distil teacher boxes / embeddings into in-house HOG detectors and a face embedder.\n\n"
              "  Usage: python -m predicitivecoding_b200.cli.detector_distiller --source <imageFolder> "
              "--labels <teacher.json> [--frames N] [--neg K] [--out <outDir>]")
        return 0
    out = _arg(argv, "--out", "vision-inhouse")
    max_frames, neg = int(_arg(argv, "--frames", 200)), int(_arg(argv, "--neg", 5))
    lab = json.load(open(labels))
    names = sorted(f for f in os.listdir(src) if f in lab)[:max_frames]
    frames = [(f, RgbImage.load(os.path.join(src, f))) for f in names]
    by_id = {id(im): lab[f] for f, im in frames}

    def face_embed(frame, box):
        entry = by_id[id(frame)]
        i = [tuple(b) for b in entry.get("face", [])].index(tuple(box))
        embs = entry.get("face_embedding", [])
        return embs[i] if i < len(embs) else None

    rep = distill((im for _, im in frames), lambda im: [tuple(b) for b in by_id[id(im)].get("person", [])],
                  lambda im: [tuple(b) for b in by_id[id(im)].get("face", [])], face_embed, out, neg)
    print(f"  Collected over {rep.frames} frames:")
    print(f"    person  {rep.person_pos} pos / {rep.person_neg} neg")
    print(f"    face    {rep.face_pos} pos / {rep.face_neg} neg")
    print(f"    embed   {rep.embed_pairs} distillation pairs")
    for p in rep.written:
        print(f"  wrote {p}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
