"""Thousand-Brains extensions: 3D reference frames, displacement recognition, composition,
heterarchical message passing, object-model persistence and the headless HTML visualiser.

Reference (PredictiveCoding.Brain):
  ReferenceFrames/Pose2D.cs, Pose3D.cs, PoseEncoder3D.cs, PathIntegrator3D.cs, DisplacementModule.cs,
  DisplacementRecognizer.cs, DisplacementRecognizer3D.cs;
  Composition/FeaturePoint*.cs, CompositeObject.cs, BehaviorSequence.cs, ConceptualFrame.cs,
  CompositionLibrary.cs;
  Connectivity/ConnectionType.cs, AreaNode.cs, AreaOutput.cs, LongRangeConnection.cs,
  HeterarchicalGraph.cs:14-96, HeterarchicalMessagePassing.cs:1-180;
  Persistence/SdrCodec.cs, ObjectModelStore.cs:18-94; Viz/VizData.cs, HtmlVisualizer.cs:27-387.

Rotations use unit quaternions (w, x, y, z) with the Hamilton product, matching the reference's
System.Numerics conventions: yaw about +Z, pitch about -Y, roll about +X, composed yaw * pitch * roll.
The HTML page is this package's own design: one self-contained file, data embedded as JSON with '<'
escaped so no value can close the script element, no external resources.
"""
from __future__ import annotations

import html
import json
import math
import time
from dataclasses import asdict, dataclass, field
from enum import Enum
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

from .brain import CategoryEncoder, ConsensusResult, MultiColumnSystem, PoseEncoder, ScalarEncoder, Sdr


# ----------------------------------------------------------------------------- quaternions and poses
@dataclass(frozen=True)
class Quaternion:
    w: float = 1.0
    x: float = 0.0
    y: float = 0.0
    z: float = 0.0

    @staticmethod
    def from_axis_angle(ax: Tuple[float, float, float], angle: float) -> "Quaternion":
        s, c = math.sin(angle / 2), math.cos(angle / 2)
        return Quaternion(c, ax[0] * s, ax[1] * s, ax[2] * s)

    def __mul__(self, o: "Quaternion") -> "Quaternion":
        a, b = self, o
        return Quaternion(a.w * b.w - a.x * b.x - a.y * b.y - a.z * b.z,
                          a.w * b.x + a.x * b.w + a.y * b.z - a.z * b.y,
                          a.w * b.y - a.x * b.z + a.y * b.w + a.z * b.x,
                          a.w * b.z + a.x * b.y - a.y * b.x + a.z * b.w)

    def norm2(self) -> float:
        return self.w * self.w + self.x * self.x + self.y * self.y + self.z * self.z

    def normalized(self) -> "Quaternion":
        n = math.sqrt(self.norm2()) or 1.0
        return Quaternion(self.w / n, self.x / n, self.y / n, self.z / n)

    def inverse(self) -> "Quaternion":
        n = self.norm2() or 1.0
        return Quaternion(self.w / n, -self.x / n, -self.y / n, -self.z / n)

    def rotate(self, v: Tuple[float, float, float]) -> Tuple[float, float, float]:
        p = self * Quaternion(0.0, *v) * self.inverse()
        return p.x, p.y, p.z


def _ypr_quaternion(yaw_deg: float, pitch_deg: float, roll_deg: float) -> Quaternion:
    r = math.radians
    return (Quaternion.from_axis_angle((0, 0, 1), r(yaw_deg)) * Quaternion.from_axis_angle((0, -1, 0), r(pitch_deg))
            * Quaternion.from_axis_angle((1, 0, 0), r(roll_deg)))


def _quaternion_ypr(q: Quaternion) -> Tuple[float, float, float]:
    q = q.normalized()
    x, y, z, w = q.x, q.y, q.z, q.w
    sp = max(-1.0, min(1.0, 2 * (x * z - w * y)))
    if abs(sp) > 0.99999:      # gimbal lock: roll folds into yaw
        yaw = math.atan2(2 * (w * z - x * y), 1 - 2 * (x * x + z * z))
        return math.degrees(yaw), math.copysign(90.0, sp), 0.0
    yaw = math.atan2(2 * (x * y + w * z), 1 - 2 * (y * y + z * z))
    roll = math.atan2(2 * (y * z + w * x), 1 - 2 * (x * x + y * y))
    return math.degrees(yaw), math.degrees(math.asin(sp)), math.degrees(roll)


@dataclass(frozen=True)
class RigidPose2D:
    """Translation + rotation in the plane (Pose2D.cs): apply, compose (child in parent), inverse."""
    x: float = 0.0
    y: float = 0.0
    theta_deg: float = 0.0

    @staticmethod
    def _rot(px, py, deg):
        r = math.radians(deg)
        c, s = math.cos(r), math.sin(r)
        return px * c - py * s, px * s + py * c

    def apply(self, px: float, py: float) -> Tuple[float, float]:
        rx, ry = self._rot(px, py, self.theta_deg)
        return self.x + rx, self.y + ry

    def compose(self, child: "RigidPose2D") -> "RigidPose2D":
        cx, cy = self.apply(child.x, child.y)
        return RigidPose2D(cx, cy, self.theta_deg + child.theta_deg)

    def inverse(self) -> "RigidPose2D":
        ix, iy = self._rot(-self.x, -self.y, -self.theta_deg)
        return RigidPose2D(ix, iy, -self.theta_deg)

    def normalized(self) -> "RigidPose2D":
        return RigidPose2D(self.x, self.y, ((self.theta_deg % 360.0) + 360.0) % 360.0)


@dataclass(frozen=True)
class Pose3D:
    """Translation + unit-quaternion rotation (Pose3D.cs)."""
    x: float = 0.0
    y: float = 0.0
    z: float = 0.0
    rotation: Quaternion = Quaternion()

    @staticmethod
    def from_translation(dx, dy, dz) -> "Pose3D":
        return Pose3D(dx, dy, dz)

    @staticmethod
    def from_yaw_pitch_roll(yaw, pitch, roll) -> "Pose3D":
        return Pose3D(0.0, 0.0, 0.0, _ypr_quaternion(yaw, pitch, roll))

    def apply(self, px, py, pz) -> Tuple[float, float, float]:
        rx, ry, rz = self.rotation.rotate((px, py, pz))
        return self.x + rx, self.y + ry, self.z + rz

    def compose(self, child: "Pose3D") -> "Pose3D":
        cx, cy, cz = self.apply(child.x, child.y, child.z)
        return Pose3D(cx, cy, cz, self.rotation * child.rotation)

    def inverse(self) -> "Pose3D":
        inv = self.rotation.inverse()
        ix, iy, iz = inv.rotate((-self.x, -self.y, -self.z))
        return Pose3D(ix, iy, iz, inv)

    def normalized(self) -> "Pose3D":
        return Pose3D(self.x, self.y, self.z, self.rotation.normalized())

    def to_yaw_pitch_roll(self) -> Tuple[float, float, float]:
        return _quaternion_ypr(self.rotation)


class PoseEncoder3D:
    """x, y, z scalar codes + yaw / pitch / roll bucket codes, concatenated (PoseEncoder3D.cs)."""

    def __init__(self, min_x, max_x, min_y, max_y, min_z, max_z, position_bits=100, position_active=10,
                 orientation_buckets=8, orientation_active=5):
        if max_x < min_x or max_y < min_y or max_z < min_z:
            raise ValueError("each axis needs max >= min")
        if orientation_buckets < 2:
            raise ValueError("orientation_buckets must be >= 2")
        self.axes = [ScalarEncoder(a, b, position_bits, position_active)
                     for a, b in ((min_x, max_x), (min_y, max_y), (min_z, max_z))]
        self.angles = [CategoryEncoder(orientation_buckets, orientation_active) for _ in range(3)]
        self.buckets = orientation_buckets

    @property
    def size(self) -> int:
        return sum(e.size for e in self.axes) + sum(e.size for e in self.angles)

    @staticmethod
    def _concat(parts: Sequence[Tuple[Sdr, int]]) -> Sdr:
        bits, off = [], 0
        for sdr, size in parts:
            bits += [b + off for b in sdr.bits]
            off += size
        return Sdr(off, bits)

    def encode_xyz(self, x, y, z) -> Sdr:
        return self._concat([(e.encode(v), e.size) for e, v in zip(self.axes, (x, y, z))])

    def _angle(self, enc, deg):
        nrm = ((deg % 360.0) + 360.0) % 360.0
        return enc.encode(int(nrm / 360.0 * self.buckets) % self.buckets)

    def encode_orientation(self, yaw, pitch, roll) -> Sdr:
        return self._concat([(self._angle(e, v), e.size) for e, v in zip(self.angles, (yaw, pitch, roll))])

    def encode(self, x, y, z, yaw, pitch, roll) -> Sdr:
        xyz = self.encode_xyz(x, y, z)
        return self._concat([(xyz, xyz.size), (self.encode_orientation(yaw, pitch, roll),
                                               sum(e.size for e in self.angles))])


class PathIntegrator3D:
    """Dead reckoning in 3D: world-frame steps, forward steps along the heading, and body-frame turns
    composed onto the orientation (PathIntegrator3D.cs)."""

    def __init__(self, encoder: PoseEncoder3D, x0=0.0, y0=0.0, z0=0.0, yaw0=0.0, pitch0=0.0, roll0=0.0):
        self.encoder = encoder
        self.reset(x0, y0, z0, yaw0, pitch0, roll0)

    def reset(self, x=0.0, y=0.0, z=0.0, yaw=0.0, pitch=0.0, roll=0.0) -> None:
        self.x, self.y, self.z = x, y, z
        self.orientation = _ypr_quaternion(yaw, pitch, roll).normalized()

    @property
    def pose(self) -> Pose3D:
        return Pose3D(self.x, self.y, self.z, self.orientation)

    @property
    def location_code(self) -> Sdr:
        yaw, pitch, roll = _quaternion_ypr(self.orientation)
        return self.encoder.encode(self.x, self.y, self.z, yaw, pitch, roll)

    def step(self, dx, dy, dz) -> Sdr:
        self.x += dx
        self.y += dy
        self.z += dz
        return self.location_code

    def step_forward(self, distance: float) -> Sdr:
        fx, fy, fz = self.orientation.rotate((1.0, 0.0, 0.0))
        return self.step(distance * fx, distance * fy, distance * fz)

    def rotate(self, yaw, pitch, roll) -> Sdr:
        self.orientation = (self.orientation * _ypr_quaternion(yaw, pitch, roll)).normalized()
        return self.location_code


# ----------------------------------------------------------------------------- displacement recognition
@dataclass(frozen=True)
class FeaturePoint:
    x: float
    y: float
    feature: Sdr

    def transformed(self, pose: RigidPose2D) -> "FeaturePoint":
        return FeaturePoint(*pose.apply(self.x, self.y), self.feature)


@dataclass(frozen=True)
class FeaturePoint3D:
    x: float
    y: float
    z: float
    feature: Sdr

    def transformed(self, pose: Pose3D) -> "FeaturePoint3D":
        return FeaturePoint3D(*pose.apply(self.x, self.y, self.z), self.feature)


class DisplacementModule:
    """Encodes a 2D displacement (dx, dy) as an SDR and applies / inverts / measures them
    (DisplacementModule.cs)."""

    def __init__(self, max_abs: float, bits_per_axis: int = 60, active_per_axis: int = 10):
        if max_abs <= 0:
            raise ValueError("max_abs must be positive")
        self.dx = ScalarEncoder(-max_abs, max_abs, bits_per_axis, active_per_axis)
        self.dy = ScalarEncoder(-max_abs, max_abs, bits_per_axis, active_per_axis)

    @property
    def sdr_size(self) -> int:
        return self.dx.size + self.dy.size

    def encode(self, dx, dy) -> Sdr:
        return Sdr(self.sdr_size, list(self.dx.encode(dx).bits) + [b + self.dx.size for b in self.dy.encode(dy).bits])

    @staticmethod
    def apply(sx, sy, dx, dy):
        return sx + dx, sy + dy

    @staticmethod
    def invert(dx, dy):
        return -dx, -dy

    @staticmethod
    def between(x1, y1, x2, y2):
        return x2 - x1, y2 - y1


@dataclass(frozen=True)
class RecognitionScore:
    object_id: int
    matching_pairs: int
    confidence: float


class DisplacementRecognizer:
    """Pose-invariant recognition from pairwise landmark distances: an object is the set of
    (feature A, feature B, |A-B|) descriptors of its landmarks; an observation votes for a stored
    object once per observed descriptor that matches a stored one (features overlap >= min_overlap,
    distance within tolerance, either order) (DisplacementRecognizer.cs / DisplacementRecognizer3D.cs)."""

    def __init__(self, min_overlap: int = 12, distance_tolerance: float = 0.6):
        if min_overlap < 1 or distance_tolerance < 0:
            raise ValueError("min_overlap >= 1 and distance_tolerance >= 0")
        self.min_overlap, self.tol = min_overlap, distance_tolerance
        self.objects: Dict[int, List[Tuple[Sdr, Sdr, float]]] = {}

    @property
    def object_count(self) -> int:
        return len(self.objects)

    @staticmethod
    def _coords(p) -> Tuple[float, ...]:
        return (p.x, p.y, p.z) if isinstance(p, FeaturePoint3D) else (p.x, p.y)

    def _descriptors(self, pts) -> List[Tuple[Sdr, Sdr, float]]:
        out = []
        for i in range(len(pts)):
            for j in range(i + 1, len(pts)):
                out.append((pts[i].feature, pts[j].feature, math.dist(self._coords(pts[i]), self._coords(pts[j]))))
        return out

    def learn(self, object_id: int, landmarks: Sequence) -> None:
        self.objects[object_id] = self._descriptors(list(landmarks))

    def _match(self, o, s) -> bool:
        m = self.min_overlap
        return ((o[0].matches(s[0], m) and o[1].matches(s[1], m)) or
                (o[0].matches(s[1], m) and o[1].matches(s[0], m)))

    def rank(self, observed: Sequence) -> List[RecognitionScore]:
        obs = self._descriptors(list(observed))
        scores = []
        for oid, stored in self.objects.items():
            n = sum(1 for o in obs if any(abs(o[2] - s[2]) <= self.tol and self._match(o, s) for s in stored))
            scores.append(RecognitionScore(oid, n, n / len(obs) if obs else 0.0))
        scores.sort(key=lambda r: -r.matching_pairs)
        return scores

    def recognize(self, observed: Sequence) -> Optional[int]:
        r = self.rank(observed)
        return r[0].object_id if r and r[0].matching_pairs > 0 else None


DisplacementRecognizer3D = DisplacementRecognizer   # the 3D form takes FeaturePoint3D landmarks


# ----------------------------------------------------------------------------- composition
@dataclass(frozen=True)
class ObjectPart:
    child_id: int
    pose_in_parent: RigidPose2D


class CompositeObject:
    """An object made of other objects, each placed by a pose in the parent's frame (CompositeObject.cs)."""

    def __init__(self, object_id: int):
        self.object_id = object_id
        self.parts: List[ObjectPart] = []

    def add_part(self, child_id: int, x: float = 0.0, y: float = 0.0, rotation_deg: float = 0.0,
                 pose: Optional[RigidPose2D] = None) -> "CompositeObject":
        if child_id == self.object_id:
            raise ValueError("a composite object cannot contain itself")
        self.parts.append(ObjectPart(child_id, pose or RigidPose2D(x, y, rotation_deg)))
        return self


class BehaviorSequence:
    """An ordered list of state SDRs: a behaviour is an object whose 'location' is time
    (BehaviorSequence.cs)."""

    def __init__(self, behavior_id: int):
        self.behavior_id = behavior_id
        self.steps: List[Sdr] = []

    def __len__(self) -> int:
        return len(self.steps)

    def append(self, state: Sdr) -> "BehaviorSequence":
        self.steps.append(state)
        return self

    def at(self, step: int) -> Optional[Sdr]:
        return self.steps[step] if 0 <= step < len(self.steps) else None

    def predict_next(self, current: int) -> Optional[Sdr]:
        return self.at(current + 1)

    def to_object_points(self, position: ScalarEncoder) -> List[Tuple[Sdr, Sdr]]:
        return [(position.encode(i), s) for i, s in enumerate(self.steps)]

    def match_score(self, observed: Sequence[Sdr], min_overlap: int) -> float:
        if not observed:
            return 0.0
        hits = sum(1 for a, b in zip(observed, self.steps) if a.size == b.size and a.matches(b, min_overlap))
        return hits / len(observed)


class ConceptualFrame:
    """An abstract N-dimensional space of concepts: locations are scalar codes per axis, recall is the
    nearest stored concept, movement adds a displacement (ConceptualFrame.cs)."""

    def __init__(self, axes: Sequence[Tuple[float, float]], bits_per_axis: int = 100, active_per_axis: int = 10):
        if len(axes) < 1:
            raise ValueError("at least one axis")
        self.axes = [ScalarEncoder(lo, hi, bits_per_axis, active_per_axis) for lo, hi in axes]
        self.concepts: List[Tuple[List[float], Sdr]] = []

    @property
    def dimensions(self) -> int:
        return len(self.axes)

    @property
    def location_size(self) -> int:
        return sum(a.size for a in self.axes)

    def _vec(self, c) -> List[float]:
        c = [float(v) for v in c]
        if len(c) != self.dimensions:
            raise ValueError(f"expected {self.dimensions} coordinates, got {len(c)}")
        return c

    def encode_location(self, coords) -> Sdr:
        c, bits, off = self._vec(coords), [], 0
        for a, v in zip(self.axes, c):
            bits += [b + off for b in a.encode(v).bits]
            off += a.size
        return Sdr(self.location_size, bits)

    def add_concept(self, coords, concept: Sdr) -> None:
        self.concepts.append((self._vec(coords), concept))

    def nearest(self, coords):
        if not self.concepts:
            return None
        q = self._vec(coords)
        c, s = min(self.concepts, key=lambda cs: math.dist(q, cs[0]))
        return c, s, math.dist(q, c)

    def recall(self, coords) -> Optional[Sdr]:
        n = self.nearest(coords)
        return None if n is None else n[1]

    def move(self, frm, displacement) -> List[float]:
        return [a + b for a, b in zip(self._vec(frm), self._vec(displacement))]


class CompositionLibrary:
    """Primitives (landmark sets) and composites (parts placed by poses), resolved recursively into
    landmarks in the root frame, with cycle and depth checks (CompositionLibrary.cs)."""

    def __init__(self, max_depth: int = 32):
        if max_depth < 1:
            raise ValueError("max_depth >= 1")
        self.max_depth = max_depth
        self.primitives: Dict[int, List[FeaturePoint]] = {}
        self.composites: Dict[int, CompositeObject] = {}

    def contains(self, i: int) -> bool:
        return i in self.primitives or i in self.composites

    def _unused(self, i: int) -> None:
        if self.contains(i):
            raise ValueError(f"object id {i} is already registered")

    def add_primitive(self, i: int, points: Sequence[FeaturePoint]) -> None:
        self._unused(i)
        self.primitives[i] = list(points)

    def add_composite(self, c: CompositeObject) -> None:
        self._unused(c.object_id)
        self.composites[c.object_id] = c

    def create_composite(self, i: int) -> CompositeObject:
        self._unused(i)
        c = CompositeObject(i)
        self.composites[i] = c
        return c

    def resolve(self, i: int) -> List[FeaturePoint]:
        acc: List[FeaturePoint] = []
        self._resolve(i, RigidPose2D(), acc, set(), 0)
        return acc

    def _resolve(self, i, to_root, acc, path, depth) -> None:
        if depth > self.max_depth:
            raise RuntimeError(f"composition nesting exceeded max depth {self.max_depth} at object {i}")
        if i in path:
            raise RuntimeError(f"cyclic composition detected at object {i}")
        path.add(i)
        if i in self.primitives:
            acc += [p.transformed(to_root) for p in self.primitives[i]]
        elif i in self.composites:
            for part in self.composites[i].parts:
                self._resolve(part.child_id, to_root.compose(part.pose_in_parent), acc, path, depth + 1)
        else:
            raise KeyError(f"object id {i} is not a registered primitive or composite")
        path.discard(i)

    def to_observations(self, i: int, pose: PoseEncoder) -> List[Tuple[Sdr, Sdr]]:
        return [(p.feature, pose.encode_xy(p.x, p.y)) for p in self.resolve(i)]


# ----------------------------------------------------------------------------- heterarchy
class ConnectionType(Enum):
    FEED_FORWARD = "FeedForward"
    FEED_BACK = "FeedBack"
    LATERAL = "Lateral"
    HETERARCHICAL = "Heterarchical"


@dataclass(frozen=True)
class LongRangeConnection:
    connection_id: int
    source_area_id: int
    target_area_id: int
    type: ConnectionType
    weight: float

    def __post_init__(self):
        if not 0 < self.weight <= 1:
            raise ValueError("weight must be in (0, 1]")


class AreaNode:
    def __init__(self, area_id: int, system: MultiColumnSystem, name: Optional[str] = None):
        self.area_id, self.column_system = area_id, system
        self.name = name or f"Area{area_id}"
        self.current_output: Optional[ConsensusResult] = None


@dataclass(frozen=True)
class AreaOutput:
    area_id: int
    consensus: ConsensusResult
    round: int
    incoming_message_count: int


class HeterarchicalGraph:
    """Cortical areas (each a multi-column system) joined by weighted long-range connections of any
    direction (HeterarchicalGraph.cs)."""

    def __init__(self):
        self.areas: Dict[int, AreaNode] = {}
        self.connections: List[LongRangeConnection] = []

    def add_area(self, area_id: int, system: MultiColumnSystem, name: Optional[str] = None) -> AreaNode:
        if area_id in self.areas:
            raise ValueError(f"area {area_id} is already registered")
        node = AreaNode(area_id, system, name)
        self.areas[area_id] = node
        return node

    def connect(self, src: int, dst: int, type: ConnectionType = ConnectionType.HETERARCHICAL,
                weight: float = 1.0) -> LongRangeConnection:
        self.get_area(src), self.get_area(dst)
        if src == dst:
            raise ValueError("self-connections are not allowed")
        c = LongRangeConnection(len(self.connections), src, dst, type, weight)
        self.connections.append(c)
        return c

    def get_area(self, area_id: int) -> AreaNode:
        if area_id not in self.areas:
            raise KeyError(f"area {area_id} not found in graph")
        return self.areas[area_id]

    def outgoing(self, area_id: int) -> List[LongRangeConnection]:
        self.get_area(area_id)
        return [c for c in self.connections if c.source_area_id == area_id]

    def incoming(self, area_id: int) -> List[LongRangeConnection]:
        self.get_area(area_id)
        return [c for c in self.connections if c.target_area_id == area_id]

    def clear(self) -> None:
        self.areas.clear()
        self.connections.clear()


class HeterarchicalMessagePassing:
    """Rounds of: every area votes on its own inputs, then each area's columns are constrained by the
    candidate objects its source areas currently hold (sources whose agreement reaches
    threshold * connection weight), until no area's candidate set changes or every area has one
    candidate (HeterarchicalMessagePassing.cs)."""

    def __init__(self, max_rounds: int = 6, convergence_threshold: float = 0.0):
        if max_rounds < 1 or not 0 <= convergence_threshold <= 1:
            raise ValueError("max_rounds >= 1 and convergence_threshold in [0, 1]")
        self.max_rounds, self.threshold = max_rounds, convergence_threshold

    @staticmethod
    def _inputs(area_inputs, area: AreaNode):
        if area.area_id not in area_inputs:
            raise KeyError(f"no inputs provided for area {area.area_id}")
        x = area_inputs[area.area_id]
        if len(x) != len(area.column_system.columns):
            raise ValueError(f"area {area.area_id} has {len(area.column_system.columns)} columns but "
                             f"{len(x)} inputs were provided")
        return x

    def gather_incoming_hypotheses(self, graph: HeterarchicalGraph, target: int) -> List[int]:
        cand = set()
        for c in graph.incoming(target):
            out = graph.get_area(c.source_area_id).current_output
            if out is None:
                continue
            if out.score >= self.threshold * c.weight:
                cand.update(out.candidates)
        return sorted(cand)

    @staticmethod
    def is_all_converged(outputs: Dict[int, AreaOutput]) -> bool:
        return all(len(o.consensus.candidates) == 1 for o in outputs.values())

    def pass_messages(self, graph: HeterarchicalGraph, area_inputs, reset: bool = True) -> Dict[int, AreaOutput]:
        outputs: Dict[int, AreaOutput] = {}
        for area in graph.areas.values():
            x = self._inputs(area_inputs, area)
            if reset:
                area.column_system.reset()
            cons = area.column_system.vote_step(x)
            area.current_output = cons
            outputs[area.area_id] = AreaOutput(area.area_id, cons, 0, 0)
        for r in range(1, self.max_rounds + 1):
            changed = False
            for area in graph.areas.values():
                ext = self.gather_incoming_hypotheses(graph, area.area_id)
                msgs = 0
                if ext:
                    area.column_system.propagate_constraint(ext)
                    msgs = sum(1 for c in graph.incoming(area.area_id)
                               if (o := graph.get_area(c.source_area_id).current_output) is not None and o.candidates)
                cons = area.column_system.vote_step(self._inputs(area_inputs, area))
                changed |= set(outputs[area.area_id].consensus.candidates) != set(cons.candidates)
                area.current_output = cons
                outputs[area.area_id] = AreaOutput(area.area_id, cons, r, msgs)
            if not changed or self.is_all_converged(outputs):
                break
        return outputs


# ----------------------------------------------------------------------------- persistence
class SdrCodec:
    """'size|b0,b1,...' text form of an SDR (SdrCodec.cs)."""

    @staticmethod
    def encode(s: Sdr) -> str:
        return f"{s.size}|{','.join(str(b) for b in s.bits)}"

    @staticmethod
    def decode(text: str) -> Sdr:
        if "|" not in text:
            raise ValueError(f"malformed SDR (no '|'): {text!r}")
        size, body = text.split("|", 1)
        bits = [int(b) for b in body.split(",")] if body.strip() else []
        return Sdr(int(size), bits)


@dataclass
class SyntheticObject:
    id: int
    points: List[FeaturePoint]


class ObjectModelStore:
    """Line-oriented text file of learned objects: a header comment, then per object
    'object <id> <count>' and one '<x> <y> <sdr>' line per landmark (ObjectModelStore.cs)."""
    HEADER = "# PredictiveCoding.Brain object models v1"

    @classmethod
    def dumps(cls, objects: Sequence[SyntheticObject]) -> str:
        lines = [cls.HEADER]
        for o in objects:
            lines.append(f"object {o.id} {len(o.points)}")
            lines += [f"{_g(p.x)} {_g(p.y)} {SdrCodec.encode(p.feature)}" for p in o.points]
        return "\n".join(lines) + "\n"

    @staticmethod
    def loads(text: str) -> List[SyntheticObject]:
        lines = iter(text.splitlines())
        out = []
        for line in lines:
            line = line.strip()
            if not line or line.startswith("#"):
                continue
            head = line.split()
            if len(head) != 3 or head[0] != "object":
                raise ValueError(f"expected 'object <id> <count>', got {line!r}")
            oid, n = int(head[1]), int(head[2])
            pts = []
            for _ in range(n):
                p = next(lines, None)
                if p is None:
                    raise ValueError(f"object {oid}: expected {n} points, file ended early")
                parts = p.split(" ", 2)
                if len(parts) != 3:
                    raise ValueError(f"malformed point line: {p!r}")
                pts.append(FeaturePoint(float(parts[0]), float(parts[1]), SdrCodec.decode(parts[2])))
            out.append(SyntheticObject(oid, pts))
        return out

    @classmethod
    def save(cls, path: str, objects: Sequence[SyntheticObject]) -> None:
        with open(path, "w", encoding="utf-8") as f:
            f.write(cls.dumps(objects))

    @classmethod
    def load(cls, path: str) -> List[SyntheticObject]:
        with open(path, encoding="utf-8") as f:
            return cls.loads(f.read())


def _g(v: float) -> str:
    """Shortest round-trip text of a float32 value (as the reference writes floats)."""
    import numpy as np
    return repr(float(np.float32(v)))


# ----------------------------------------------------------------------------- visualisation
@dataclass
class VizBenchmarkRow:
    condition: str
    single_accuracy: float
    single_steps: float
    voting_accuracy: float
    voting_steps: float


@dataclass
class VizPoint:
    x: float
    y: float
    feature_id: int


@dataclass
class VizObject:
    id: int
    points: List[VizPoint]


@dataclass
class VizEpisode:
    target_id: int = 0
    object_count: int = 0
    columns_voting: int = 0
    objects: List[VizObject] = field(default_factory=list)
    single_steps: List[List[int]] = field(default_factory=list)     # candidate ids after each step
    voting_rounds: List[List[int]] = field(default_factory=list)


@dataclass
class VizPoseRow:
    id: int
    column_correct: bool
    displacement_correct: bool


@dataclass
class VizPoseInvariance:
    dx: float = 0.0
    dy: float = 0.0
    theta_deg: float = 0.0
    rows: List[VizPoseRow] = field(default_factory=list)


@dataclass
class VizFixation:
    col: int
    row: int
    category: int
    share: float
    luminance: float


@dataclass
class VizImageScan:
    width: int = 0
    height: int = 0
    pixels: List[float] = field(default_factory=list)
    grid_cols: int = 0
    grid_rows: int = 0
    patch_size: int = 0
    stride: int = 0
    orientation_bins: int = 0
    fixations: List[VizFixation] = field(default_factory=list)


@dataclass
class VizData:
    title: str = "Thousand Brains - sensorimotor recognition"
    benchmark: List[VizBenchmarkRow] = field(default_factory=list)
    episode: Optional[VizEpisode] = None
    pose_invariance: Optional[VizPoseInvariance] = None
    image_scan: Optional[VizImageScan] = None


def _camel(o):
    if isinstance(o, dict):
        return {k.split("_")[0] + "".join(w.title() for w in k.split("_")[1:]): _camel(v) for k, v in o.items()}
    if isinstance(o, list):
        return [_camel(v) for v in o]
    return o


_PAGE = """<!DOCTYPE html>
<html lang="en"><head><meta charset="utf-8"><title>Thousand Brains</title>
<style>
body{font:14px/1.45 system-ui,sans-serif;margin:24px auto;max-width:1000px;color:#222}
section{border:1px solid #ccd;border-radius:8px;padding:14px 18px;margin:14px 0;background:#fafbfc}
h1{font-size:22px}h2{font-size:16px;margin:0 0 10px}table{border-collapse:collapse}
td,th{padding:4px 12px;border-bottom:1px solid #ddd;text-align:left}.ok{color:#17803a}.bad{color:#c0282d}
canvas{border:1px solid #ccd;background:#fff}.chip{display:inline-block;border:1px solid #99a;border-radius:9px;
padding:0 7px;margin:1px}
</style></head><body>
<h1 id="t"></h1><div>generated GENERATED_AT</div>
<section id="ep" hidden><h2>Episode</h2><canvas id="cv" width="360" height="360"></canvas>
<div><b>single column</b> <span id="sc"></span></div><div><b>voting columns</b> <span id="vc"></span></div>
<input id="sl" type="range" min="0" value="0"></section>
<section id="bm" hidden><h2>Benchmark</h2><table id="bt"><tr><th>condition</th><th>single acc</th>
<th>single steps</th><th>voting acc</th><th>voting steps</th></tr></table></section>
<section id="pi" hidden><h2>Pose invariance</h2><div id="pd"></div><table id="pt"><tr><th>object</th>
<th>column</th><th>displacement</th></tr></table></section>
<section id="is" hidden><h2>Image scan</h2><canvas id="ic"></canvas><div id="fx"></div></section>
<script>
const D = JSON.parse(document.getElementById('data').textContent);
</script>
</body></html>
"""


class HtmlVisualizer:
    """One self-contained HTML page (inline CSS and script, data as embedded JSON, no external
    resources) with the sections whose data is present: episode player, benchmark table, pose
    invariance and image scan (HtmlVisualizer.cs:27-60)."""

    SCRIPT = """
(function(){
const $=id=>document.getElementById(id);$('t').textContent=D.title;
function chips(ids){return ids.map(i=>'<span class="chip">'+Number(i)+'</span>').join('');}
if(D.episode){const e=D.episode;$('ep').hidden=false;const n=Math.max(e.singleSteps.length,e.votingRounds.length);
$('sl').max=Math.max(0,n-1);const cv=$('cv').getContext('2d');const tgt=e.objects.find(o=>o.id===e.targetId);
function draw(k){cv.clearRect(0,0,360,360);if(tgt){const xs=tgt.points.map(p=>p.x),ys=tgt.points.map(p=>p.y);
const x0=Math.min(...xs),x1=Math.max(...xs),y0=Math.min(...ys),y1=Math.max(...ys);
for(const p of tgt.points){const u=20+320*(p.x-x0)/Math.max(1e-6,x1-x0),v=20+320*(p.y-y0)/Math.max(1e-6,y1-y0);
cv.fillStyle='hsl('+(p.featureId*47%360)+',60%,45%)';cv.fillRect(u-4,v-4,8,8);}}
$('sc').innerHTML=chips(e.singleSteps[Math.min(k,e.singleSteps.length-1)]||[]);
$('vc').innerHTML=chips(e.votingRounds[Math.min(k,e.votingRounds.length-1)]||[]);}
$('sl').oninput=ev=>draw(+ev.target.value);draw(0);}
if(D.benchmark&&D.benchmark.length){$('bm').hidden=false;for(const r of D.benchmark){const tr=document.createElement('tr');
for(const v of [r.condition,r.singleAccuracy.toFixed(3),r.singleSteps.toFixed(2),r.votingAccuracy.toFixed(3),
r.votingSteps.toFixed(2)]){const td=document.createElement('td');td.textContent=v;tr.appendChild(td);}$('bt').appendChild(tr);}}
if(D.poseInvariance){const p=D.poseInvariance;$('pi').hidden=false;
$('pd').textContent='moved by ('+p.dx+', '+p.dy+') and '+p.thetaDeg+' deg';
for(const r of p.rows){const tr=document.createElement('tr');tr.innerHTML='<td>'+Number(r.id)+'</td><td class="'+
(r.columnCorrect?'ok">yes':'bad">no')+'</td><td class="'+(r.displacementCorrect?'ok">yes':'bad">no')+'</td>';
$('pt').appendChild(tr);}}
if(D.imageScan){const s=D.imageScan;$('is').hidden=false;const c=$('ic');c.width=s.width;c.height=s.height;
const g=c.getContext('2d'),img=g.createImageData(s.width,s.height);
for(let i=0;i<s.pixels.length;i++){const v=Math.max(0,Math.min(255,s.pixels[i]*255));img.data[4*i]=img.data[4*i+1]=
img.data[4*i+2]=v;img.data[4*i+3]=255;}g.putImageData(img,0,0);g.strokeStyle='#d33';
for(const f of s.fixations){g.strokeRect(f.col*s.stride,f.row*s.stride,s.patchSize,s.patchSize);}
$('fx').textContent=s.fixations.length+' fixations, '+s.orientationBins+' orientation bins';}
})();
"""

    @classmethod
    def render(cls, data: VizData) -> str:
        payload = json.dumps(_camel(asdict(data))).replace("<", "\\u003c")
        page = _PAGE.replace("GENERATED_AT", time.strftime("%Y-%m-%d %H:%M UTC", time.gmtime()))
        page = page.replace("const D = JSON.parse(document.getElementById('data').textContent);",
                            "const D = JSON.parse(document.getElementById('data').textContent);" + cls.SCRIPT)
        return page.replace("<script>", f'<script id="data" type="application/json">{payload}</script>\n<script>', 1)

    @classmethod
    def save(cls, path: str, data: VizData) -> None:
        with open(path, "w", encoding="utf-8") as f:
            f.write(cls.render(data))
