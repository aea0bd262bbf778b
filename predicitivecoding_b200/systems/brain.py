"""Thousand-Brains sensorimotor recognition: sparse distributed representations, scalar / category /
pose encoders, an HTM spatial pooler and temporal memory, cortical columns that store
feature-at-location object models, lateral voting and consensus across columns, 2-D path
integration, a synthetic object dataset and a recognition benchmark.

Reference: PredictiveCoding.Brain/Sdr/Sdr.cs:1-234, ScalarEncoder.cs, CategoryEncoder.cs,
ReferenceFrames/PoseEncoder.cs:1-91, PathIntegrator.cs, ObjectFrame.cs:1-89, Columns/ObjectMemory.cs:1-69,
CorticalColumn.cs:1-197, KWinners.cs, Sequence/SpatialPooler.cs:1-150, TemporalMemory.cs:1-305,
Voting/LateralVoting.cs:1-124, Consensus.cs:1-89, MultiColumnSystem.cs:1-174,
System/ThousandBrainsSystem.cs:1-249, Eval/SyntheticObjectDataset.cs, RecognitionBenchmark.cs.
Same algorithms (HTM-style: overlap-ranked column winners with permanence learning; per-cell
distal segments with active / matching thresholds, bursting, least-used-cell growth; object
hypotheses intersected over observations; consensus = objects voted by at least a fraction of
columns).  Sets and sorted lists replace the reference's arrays; randomness is seeded numpy.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, Iterable, List, Optional, Sequence, Set, Tuple

import numpy as np


# ---------------------------------------------------------------- SDR
class Sdr:
    __slots__ = ("size", "bits")

    def __init__(self, size: int, active: Iterable[int] = ()):
        if size <= 0:
            raise ValueError("Size must be positive.")
        bits = sorted(set(int(b) for b in active))
        if bits and (bits[0] < 0 or bits[-1] >= size):
            raise ValueError(f"Active bit index out of range [0,{size}).")
        self.size = size
        self.bits: Tuple[int, ...] = tuple(bits)

    @property
    def cardinality(self) -> int:
        return len(self.bits)

    @property
    def sparsity(self) -> float:
        return len(self.bits) / self.size

    def is_active(self, bit: int) -> bool:
        return bit in set(self.bits)

    def _same(self, o: "Sdr") -> None:
        if o.size != self.size:
            raise ValueError(f"Size mismatch: {self.size} vs {o.size}.")

    def overlap(self, o: "Sdr") -> int:
        self._same(o)
        return len(set(self.bits) & set(o.bits))

    def overlap_score(self, o: "Sdr") -> float:
        m = min(self.cardinality, o.cardinality)
        return 0.0 if m == 0 else self.overlap(o) / m

    def matches(self, o: "Sdr", min_overlap: int) -> bool:
        return self.overlap(o) >= min_overlap

    def union(self, o: "Sdr") -> "Sdr":
        self._same(o)
        return Sdr(self.size, set(self.bits) | set(o.bits))

    def intersect(self, o: "Sdr") -> "Sdr":
        self._same(o)
        return Sdr(self.size, set(self.bits) & set(o.bits))

    def add_noise(self, fraction: float, rng: np.random.Generator) -> "Sdr":
        if fraction <= 0 or not self.bits:
            return self
        k = min(int(round(fraction * self.cardinality)), self.cardinality, self.size - self.cardinality)
        if k <= 0:
            return self
        removed = set(rng.choice(self.bits, k, replace=False).tolist())
        keep = set(self.bits) - removed
        orig = set(self.bits)
        while len(keep) < self.cardinality:
            c = int(rng.integers(self.size))
            if c not in orig:
                keep.add(c)
        return Sdr(self.size, keep)

    def subsample(self, n: int, rng: np.random.Generator) -> "Sdr":
        if n >= self.cardinality:
            return self
        return Sdr(self.size, rng.choice(self.bits, max(0, n), replace=False).tolist())

    def to_dense(self) -> np.ndarray:
        d = np.zeros(self.size, np.float32)
        d[list(self.bits)] = 1
        return d

    @staticmethod
    def from_dense(v, threshold: float = 0.5) -> "Sdr":
        v = np.asarray(v)
        return Sdr(max(1, v.size), np.nonzero(v >= threshold)[0].tolist())

    @staticmethod
    def empty(size: int) -> "Sdr":
        return Sdr(size)

    @staticmethod
    def random(size: int, cardinality: int, rng: np.random.Generator) -> "Sdr":
        if not 0 <= cardinality <= size:
            raise ValueError("Cardinality must be in [0, size].")
        return Sdr(size, rng.choice(size, cardinality, replace=False).tolist())

    def __eq__(self, o) -> bool:
        return isinstance(o, Sdr) and o.size == self.size and o.bits == self.bits

    def __hash__(self) -> int:
        return hash((self.size, self.bits))

    def __repr__(self) -> str:
        return f"Sdr({self.size}, {list(self.bits)})"


class ScalarEncoder:
    """A contiguous window of w bits slides over n positions as the value goes from min to max."""

    def __init__(self, lo: float, hi: float, n: int, w: int):
        if n <= 0 or not 0 < w < n or hi < lo:
            raise ValueError("invalid scalar encoder")
        self.lo, self.hi, self.n, self.w = lo, hi, n, w
        self.buckets = n - w + 1

    @property
    def size(self) -> int:
        return self.n

    def encode(self, v: float) -> Sdr:
        c = min(max(v, self.lo), self.hi)
        frac = (c - self.lo) / (self.hi - self.lo) if self.hi > self.lo else 0.0
        s = min(max(int(math.floor(frac * (self.buckets - 1) + 0.5)), 0), self.buckets - 1)
        return Sdr(self.n, range(s, s + self.w))


class CategoryEncoder:
    def __init__(self, categories: int, w: int):
        if categories <= 0 or w <= 0:
            raise ValueError("invalid category encoder")
        self.categories, self.w = categories, w

    @property
    def size(self) -> int:
        return self.categories * self.w

    def encode(self, c: int) -> Sdr:
        if not 0 <= c < self.categories:
            raise ValueError(f"category must be in [0, {self.categories}).")
        return Sdr(self.size, range(c * self.w, (c + 1) * self.w))


class PoseEncoder:
    def __init__(self, min_x, max_x, min_y, max_y, position_bits=100, position_active=10, orientation_buckets=8,
                 orientation_active=5):
        if orientation_buckets < 2:
            raise ValueError("orientation_buckets must be >= 2")
        self.x = ScalarEncoder(min_x, max_x, position_bits, position_active)
        self.y = ScalarEncoder(min_y, max_y, position_bits, position_active)
        self.theta = CategoryEncoder(orientation_buckets, orientation_active)
        self.buckets = orientation_buckets

    @property
    def size(self) -> int:
        return self.x.size + self.y.size + self.theta.size

    def encode_xy(self, x: float, y: float) -> Sdr:
        return Sdr(self.x.size + self.y.size,
                   list(self.x.encode(x).bits) + [b + self.x.size for b in self.y.encode(y).bits])

    def encode_theta(self, deg: float) -> Sdr:
        nrm = ((deg % 360.0) + 360.0) % 360.0
        return self.theta.encode(int(nrm / 360.0 * self.buckets) % self.buckets)

    def encode(self, x: float, y: float, deg: float) -> Sdr:
        xy = self.encode_xy(x, y)
        off = self.x.size + self.y.size
        return Sdr(self.size, list(xy.bits) + [b + off for b in self.encode_theta(deg).bits])


@dataclass
class Pose2D:
    x: float = 0.0
    y: float = 0.0
    theta_deg: float = 0.0

    def moved(self, forward: float, turn_deg: float = 0.0) -> "Pose2D":
        th = self.theta_deg + turn_deg
        r = math.radians(th)
        return Pose2D(self.x + forward * math.cos(r), self.y + forward * math.sin(r), th % 360.0)


class PathIntegrator:
    """Dead-reckoning location in an object's frame from a stream of motor commands."""

    def __init__(self, start: Pose2D = Pose2D()):
        self.pose = start
        self.history: List[Pose2D] = [start]

    def move(self, forward: float, turn_deg: float = 0.0) -> Pose2D:
        self.pose = self.pose.moved(forward, turn_deg)
        self.history.append(self.pose)
        return self.pose

    def displacement(self, a: int, b: int) -> Tuple[float, float]:
        pa, pb = self.history[a], self.history[b]
        return pb.x - pa.x, pb.y - pa.y

    def reset(self, start: Pose2D = Pose2D()) -> None:
        self.__init__(start)


def k_winners(scores: Sequence[float], k: int, boosts: Optional[Sequence[float]] = None) -> List[int]:
    """Indices of the k largest (boosted) scores, ties by lower index."""
    s = np.asarray(scores, np.float64) * (np.asarray(boosts) if boosts is not None else 1.0)
    order = sorted(range(len(s)), key=lambda i: (-s[i], i))
    return sorted(order[:max(0, k)])


# ---------------------------------------------------------------- spatial pooler
@dataclass(frozen=True)
class SpatialPoolerConfig:
    input_size: int
    columns: int
    active_columns: int = 0
    potential_pct: float = 0.5
    connected_permanence: float = 0.5
    permanence_increment: float = 0.05
    permanence_decrement: float = 0.02
    stimulus_threshold: int = 1
    seed: int = 42


class SpatialPooler:
    def __init__(self, cfg: SpatialPoolerConfig):
        if cfg.input_size <= 0 or cfg.columns <= 0:
            raise ValueError("input_size and columns must be positive.")
        self.cfg = cfg
        self.k = min(cfg.active_columns, cfg.columns) if cfg.active_columns > 0 else max(1, round(cfg.columns * 0.02))
        rng = np.random.default_rng(cfg.seed)
        npot = min(max(round(cfg.potential_pct * cfg.input_size), 1), cfg.input_size)
        self.potential = np.stack([np.sort(rng.choice(cfg.input_size, npot, replace=False)) for _ in range(cfg.columns)])
        self.perm = np.clip(cfg.connected_permanence + rng.uniform(-0.1, 0.1, self.potential.shape), 0, 1).astype(
            np.float32)

    def compute(self, x: Sdr, learn: bool) -> Sdr:
        if x.size != self.cfg.input_size:
            raise ValueError("input size mismatch")
        active = x.to_dense().astype(bool)
        on = active[self.potential]
        overlaps = ((self.perm >= self.cfg.connected_permanence) & on).sum(1)
        eligible = [c for c in range(self.cfg.columns) if overlaps[c] >= self.cfg.stimulus_threshold]
        eligible.sort(key=lambda c: (-overlaps[c], c))
        winners = eligible[: self.k]
        if learn:
            for c in winners:
                self.perm[c] = np.clip(np.where(on[c], self.perm[c] + self.cfg.permanence_increment,
                                                self.perm[c] - self.cfg.permanence_decrement), 0, 1)
        return Sdr(self.cfg.columns, winners)


# ---------------------------------------------------------------- temporal memory
@dataclass(frozen=True)
class TemporalMemoryConfig:
    columns: int
    cells_per_column: int = 8
    activation_threshold: int = 13
    min_threshold: int = 10
    connected_permanence: float = 0.5
    initial_permanence: float = 0.21
    permanence_increment: float = 0.10
    permanence_decrement: float = 0.10
    predicted_segment_decrement: float = 0.0
    max_new_synapse_count: int = 20
    seed: int = 42


@dataclass(frozen=True)
class TemporalMemoryResult:
    active_cells: List[int]
    winner_cells: List[int]
    predictive_cells: List[int]
    anomaly: float


class _Segment:
    __slots__ = ("cell", "syn")

    def __init__(self, cell: int):
        self.cell = cell
        self.syn: Dict[int, float] = {}   # presynaptic cell -> permanence (insertion ordered)


class TemporalMemory:
    def __init__(self, cfg: TemporalMemoryConfig):
        if cfg.columns <= 0 or cfg.cells_per_column <= 0 or cfg.activation_threshold <= 0 or cfg.min_threshold <= 0:
            raise ValueError("invalid temporal memory config")
        self.cfg = cfg
        self.segments: Dict[int, List[_Segment]] = {}
        self.rng = np.random.default_rng(cfg.seed)
        self.reset()

    def reset(self) -> None:
        self.prev_active: Set[int] = set()
        self.prev_winner: Set[int] = set()
        self.active_segs: List[_Segment] = []
        self.matching_segs: List[_Segment] = []
        self.num_potential: Dict[_Segment, int] = {}

    def _col(self, cell: int) -> int:
        return cell // self.cfg.cells_per_column

    def _adapt(self, seg: _Segment, pre: Set[int], inc: float, dec: float) -> None:
        for c in seg.syn:
            seg.syn[c] = min(max(seg.syn[c] + (inc if c in pre else -dec), 0.0), 1.0)

    def _grow(self, seg: _Segment, cand: Set[int], n: int) -> None:
        pool = [c for c in sorted(cand) if c != seg.cell and c not in seg.syn]
        for i in range(min(n, len(pool))):
            j = int(self.rng.integers(i, len(pool)))
            pool[i], pool[j] = pool[j], pool[i]
            seg.syn[pool[i]] = self.cfg.initial_permanence

    def _learn(self, seg: _Segment) -> None:
        self._adapt(seg, self.prev_active, self.cfg.permanence_increment, self.cfg.permanence_decrement)
        g = self.cfg.max_new_synapse_count - self.num_potential.get(seg, 0)
        if g > 0:
            self._grow(seg, self.prev_winner, g)

    def _least_used(self, col: int) -> int:
        cpc = self.cfg.cells_per_column
        return min(range(col * cpc, (col + 1) * cpc), key=lambda c: (len(self.segments.get(c, [])), c))

    def compute(self, active_columns: Sdr, learn: bool) -> TemporalMemoryResult:
        cfg = self.cfg
        if active_columns.size != cfg.columns:
            raise ValueError("active column SDR has the wrong size")
        by_col_active: Dict[int, List[_Segment]] = {}
        for s in self.active_segs:
            by_col_active.setdefault(self._col(s.cell), []).append(s)
        by_col_match: Dict[int, List[_Segment]] = {}
        for s in self.matching_segs:
            by_col_match.setdefault(self._col(s.cell), []).append(s)
        active: Set[int] = set()
        winner: Set[int] = set()
        bursting = 0
        for col in active_columns.bits:
            segs = by_col_active.get(col)
            if segs:
                for s in segs:
                    active.add(s.cell)
                    winner.add(s.cell)
                if learn:
                    for s in segs:
                        self._learn(s)
                continue
            bursting += 1
            active.update(range(col * cfg.cells_per_column, (col + 1) * cfg.cells_per_column))
            learning = None
            cand = by_col_match.get(col)
            if cand:
                learning = max(cand, key=lambda s: (self.num_potential.get(s, 0), -s.cell))
                w = learning.cell
            else:
                w = self._least_used(col)
                if learn and self.prev_winner:
                    learning = _Segment(w)
                    self.segments.setdefault(w, []).append(learning)
            winner.add(w)
            if learn and learning is not None:
                self._learn(learning)
        if learn and cfg.predicted_segment_decrement > 0:
            cols = set(active_columns.bits)
            for s in self.matching_segs:
                if self._col(s.cell) not in cols:
                    self._adapt(s, self.prev_active, -cfg.predicted_segment_decrement, 0.0)
        new_active, new_match, pot, predictive = [], [], {}, set()
        for segs in self.segments.values():
            for s in segs:
                n_pot = n_con = 0
                for c, p in s.syn.items():
                    if c in active:
                        n_pot += 1
                        n_con += p >= cfg.connected_permanence
                if n_con >= cfg.activation_threshold:
                    new_active.append(s)
                    predictive.add(s.cell)
                if n_pot >= cfg.min_threshold:
                    new_match.append(s)
                if n_pot > 0:
                    pot[s] = n_pot
        anomaly = bursting / active_columns.cardinality if active_columns.cardinality else 0.0
        self.prev_active, self.prev_winner = active, winner
        self.active_segs, self.matching_segs, self.num_potential = new_active, new_match, pot
        return TemporalMemoryResult(sorted(active), sorted(winner), sorted(predictive), anomaly)


# ---------------------------------------------------------------- object models and columns
class ObjectFrame:
    def __init__(self, object_id: int, min_overlap: int = 3):
        if min_overlap < 1:
            raise ValueError("min_overlap must be >= 1")
        self.object_id, self.min_overlap = object_id, min_overlap
        self.points: List[Tuple[Sdr, Sdr]] = []

    def add_point(self, location: Sdr, feature: Sdr) -> None:
        self.points.append((location, feature))

    def votes_for(self, location: Sdr, feature: Sdr) -> int:
        return sum(1 for l, f in self.points if l.size == location.size and f.size == feature.size
                   and l.matches(location, self.min_overlap) and f.matches(feature, self.min_overlap))

    def matching_features(self, location: Sdr) -> List[Sdr]:
        return [f for l, f in self.points if l.size == location.size and l.matches(location, self.min_overlap)]

    def matching_locations(self, feature: Sdr) -> List[Sdr]:
        return [l for l, f in self.points if f.size == feature.size and f.matches(feature, self.min_overlap)]


class ObjectMemory:
    def __init__(self, min_overlap: int = 3):
        self.min_overlap = min_overlap
        self.frames: Dict[int, ObjectFrame] = {}

    @property
    def object_count(self) -> int:
        return len(self.frames)

    def add_point(self, oid: int, location: Sdr, feature: Sdr) -> None:
        self.frames.setdefault(oid, ObjectFrame(oid, self.min_overlap)).add_point(location, feature)

    def intersecting_object_ids(self, location: Sdr, feature: Sdr) -> List[int]:
        return [oid for oid, f in self.frames.items() if f.votes_for(location, feature) > 0]


@dataclass(frozen=True)
class CorticalColumnConfig:
    input_size: int
    columns: int
    cells_per_column: int = 8
    sparsity: float = 0.02
    min_overlap: int = 3
    seed: int = 42


@dataclass(frozen=True)
class CorticalColumnOutput:
    active_cells: Sdr
    object_hypotheses: List[int]
    converged: bool
    anomaly: float


class CorticalColumn:
    def __init__(self, cfg: CorticalColumnConfig):
        self.cfg = cfg
        k = max(1, round(cfg.sparsity * cfg.columns))
        self.sp = SpatialPooler(SpatialPoolerConfig(cfg.input_size, cfg.columns, k, seed=cfg.seed))
        self.tm = TemporalMemory(TemporalMemoryConfig(cfg.columns, cfg.cells_per_column, seed=cfg.seed + 1))
        self.memory = ObjectMemory(cfg.min_overlap)
        self.hypotheses: Set[int] = set()
        self.steps = 0
        self.next_id = 0
        self.learning_id = -1

    @property
    def object_count(self) -> int:
        return self.memory.object_count

    def start_new_object(self) -> int:
        self.learning_id = self.next_id
        self.next_id += 1
        return self.learning_id

    def compute(self, feature: Sdr, location: Sdr, learn: bool) -> CorticalColumnOutput:
        cols = self.sp.compute(feature, learn)
        tm = self.tm.compute(cols, learn)
        if learn:
            if self.learning_id < 0:
                raise RuntimeError("Call start_new_object() before learning.")
            self.memory.add_point(self.learning_id, location, cols)
            hyp = [self.learning_id]
        else:
            cand = set(self.memory.intersecting_object_ids(location, cols))
            self.hypotheses = cand if self.steps == 0 else self.hypotheses & cand
            self.steps += 1
            hyp = sorted(self.hypotheses)
        return CorticalColumnOutput(Sdr(self.cfg.columns * self.cfg.cells_per_column, tm.active_cells), hyp,
                                    len(hyp) == 1, tm.anomaly)

    def constrain(self, candidates: Iterable[int]) -> None:
        self.hypotheses &= set(candidates)

    def reset(self) -> None:
        self.tm.reset()
        self.hypotheses = set()
        self.steps = 0

    def learn_object(self, observations: Sequence[Tuple[Sdr, Sdr]]) -> int:
        oid = self.start_new_object()
        self.tm.reset()
        for f, l in observations:
            self.compute(f, l, True)
        return oid

    def infer(self, observations: Sequence[Tuple[Sdr, Sdr]]) -> List[CorticalColumnOutput]:
        self.reset()
        return [self.compute(f, l, False) for f, l in observations]


# ---------------------------------------------------------------- voting
class LateralVoting:
    def __init__(self, n: int, topology: str = "all", radius: int = 2):
        if n < 2 or radius < 1:
            raise ValueError("at least 2 columns and radius >= 1")
        self.n, self.topology, self.radius = n, topology, radius

    def neighbors(self, i: int) -> List[int]:
        if self.topology == "ring":
            return sorted({(i - 1) % self.n, (i + 1) % self.n} - {i})
        if self.topology == "local":
            return [j for j in range(max(0, i - self.radius), min(self.n, i + self.radius + 1)) if j != i]
        return [j for j in range(self.n) if j != i]

    def lateral_sdr(self, i: int, cells: Sequence[Sdr]) -> Sdr:
        nb = self.neighbors(i)
        if not nb:
            return Sdr.empty(cells[i].size)
        s = cells[nb[0]]
        for j in nb[1:]:
            s = s.union(cells[j])
        return s

    def broadcast(self, cells: Sequence[Sdr]) -> List[Sdr]:
        return [self.lateral_sdr(i, cells) for i in range(self.n)]


@dataclass(frozen=True)
class ConsensusResult:
    candidates: List[int]
    score: float
    reached: bool
    round: int


class Consensus:
    def __init__(self, min_agreement: float = 1.0):
        if not 0 < min_agreement <= 1:
            raise ValueError("min_agreement must be in (0, 1]")
        self.min_agreement = min_agreement

    def compute(self, hypotheses: Sequence[Sequence[int]], rnd: int = 0) -> ConsensusResult:
        n = len(hypotheses)
        if n == 0:
            return ConsensusResult([], 0.0, False, rnd)
        votes: Dict[int, int] = {}
        for h in hypotheses:
            for oid in h:
                votes[oid] = votes.get(oid, 0) + 1
        cand = sorted(o for o, v in votes.items() if v / n >= self.min_agreement)
        score = sum(votes[o] / n for o in cand) / len(cand) if cand else 0.0
        return ConsensusResult(cand, score, bool(cand), rnd)


class MultiColumnSystem:
    def __init__(self, configs: Sequence[CorticalColumnConfig], topology: str = "all", min_agreement: float = 0.5):
        if len(configs) < 2:
            raise ValueError("At least 2 column configs required.")
        self.columns = [CorticalColumn(c) for c in configs]
        self.lateral = LateralVoting(len(configs), topology)
        self.consensus = Consensus(min_agreement)
        self.current: Optional[ConsensusResult] = None

    @property
    def object_count(self) -> int:
        return self.columns[0].object_count

    def learn_object(self, per_column: Sequence[Sequence[Tuple[Sdr, Sdr]]]) -> int:
        ids = {c.start_new_object() for c in self.columns}
        if len(ids) != 1:
            raise RuntimeError("columns out of sync")
        for c, obs in zip(self.columns, per_column):
            c.tm.reset()
            for f, l in obs:
                c.compute(f, l, True)
        return ids.pop()

    def vote_step(self, inputs: Sequence[Tuple[Sdr, Sdr]]) -> ConsensusResult:
        outs = [c.compute(f, l, False) for c, (f, l) in zip(self.columns, inputs)]
        self.lateral.broadcast([o.active_cells for o in outs])
        self.current = self.consensus.compute([o.object_hypotheses for o in outs])
        if self.current.candidates:
            for c in self.columns:
                c.constrain(self.current.candidates)
        return self.current

    def run_to_consensus(self, inputs, max_rounds: int = 20) -> ConsensusResult:
        r = ConsensusResult([], 0.0, False, 0)
        for _ in range(max_rounds):
            r = self.vote_step(inputs)
            if len(r.candidates) == 1:
                break
        return r

    def propagate_constraint(self, external_candidates: Sequence[int]) -> None:
        """Restrict every column's hypotheses to candidates another area holds (MultiColumnSystem.cs:141-148)."""
        ext = list(external_candidates)
        if ext:
            for c in self.columns:
                c.constrain(ext)

    def reset(self) -> None:
        for c in self.columns:
            c.reset()
        self.current = None


class ThousandBrainsSystem:
    """N columns that see the same object from different sensor patches; recognition succeeds when
    the columns' intersected hypotheses agree on one object."""

    def __init__(self, feature_size: int, location_size: int, n_columns: int = 3, columns: int = 256,
                 min_agreement: float = 0.5, seed: int = 42):
        cfgs = [CorticalColumnConfig(feature_size, columns, 4, 0.04, 2, seed + 17 * i) for i in range(n_columns)]
        self.system = MultiColumnSystem(cfgs, "all", min_agreement)
        self.learned = 0

    def teach_object(self, observations: Sequence[Tuple[Sdr, Sdr]]) -> int:
        self.learned += 1
        return self.system.learn_object([observations] * len(self.system.columns))

    def recognize(self, observations: Sequence[Tuple[Sdr, Sdr]]) -> Optional[int]:
        self.system.reset()
        n = len(self.system.columns)
        result = None
        for i in range(0, len(observations), n):
            step = [observations[(i + k) % len(observations)] for k in range(n)]
            result = self.system.vote_step(step)
            if len(result.candidates) == 1:
                return result.candidates[0]
        return result.candidates[0] if result and len(result.candidates) == 1 else None


# ---------------------------------------------------------------- evaluation
class SyntheticObjectDataset:
    """Objects = random sets of (location, feature) pairs drawn from shared feature / location pools."""

    def __init__(self, n_objects: int = 10, points: int = 10, n_features: int = 20, n_locations: int = 30,
                 size: int = 400, active: int = 12, seed: int = 0):
        rng = np.random.default_rng(seed)
        self.features = [Sdr.random(size, active, rng) for _ in range(n_features)]
        self.locations = [Sdr.random(size, active, rng) for _ in range(n_locations)]
        self.objects = []
        for _ in range(n_objects):
            locs = rng.choice(n_locations, points, replace=False)
            feats = rng.integers(0, n_features, points)
            self.objects.append([(self.features[f], self.locations[l]) for f, l in zip(feats, locs)])
        self.size = size


@dataclass(frozen=True)
class RecognitionReport:
    accuracy: float
    mean_steps: float
    n: int


def recognition_benchmark(system: ThousandBrainsSystem, data: SyntheticObjectDataset, noise: float = 0.0,
                          seed: int = 1) -> RecognitionReport:
    rng = np.random.default_rng(seed)
    ids = [system.teach_object(o) for o in data.objects]
    correct, steps = 0, 0
    for oid, obs in zip(ids, data.objects):
        order = rng.permutation(len(obs))
        noisy = [(obs[i][0].add_noise(noise, rng), obs[i][1]) for i in order]
        got = system.recognize(noisy)
        correct += got == oid
        steps += len(noisy)
    return RecognitionReport(correct / len(ids), steps / len(ids), len(ids))
