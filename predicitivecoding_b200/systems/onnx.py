"""A self-contained ONNX subset: protobuf wire reader, ModelProto parser, graph executor on torch
(CPU or GPU), save-time optimizer and the PCNX compact graph format.

Reference: PredictiveCoding.Onnx/Proto/ProtoReader.cs:1-171 (varint / length-delimited / fixed
fields), OnnxParser.cs:1-474 (ModelProto -> graph; TensorProto float / int32 / int64 from raw_data
or the typed repeated fields), OnnxGraph.cs:1-101 (nodes, initializers, value infos, attributes),
Executor.cs:1-246 (topological execution with a per-op kernel table), Ops.*.cs (Conv, Gemm/MatMul,
pools, elementwise, reductions, shape ops, Gather, Resize, logical ops),
Optimize/GraphOptimizer.cs:1-263 (Constant nodes -> initializers, constant folding with the runtime's
own kernels, Identity/Dropout elision, dead-node and unused-initializer removal) and
Format/PcnxFormat.cs:1-313.  The PCNX layout is kept byte-compatible with the reference's
(little-endian, .NET BinaryWriter strings: 7-bit-encoded length prefix + UTF-8) so models move
between the two.
"""
from __future__ import annotations

import io
import struct
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.nn.functional as F

FLOAT, INT32, INT64 = 1, 6, 7
A_FLOAT, A_INT, A_STRING, A_TENSOR, A_FLOATS, A_INTS, A_STRINGS = 1, 2, 3, 4, 6, 7, 8


# ---------------------------------------------------------------- protobuf wire format
class ProtoReader:
    def __init__(self, data: bytes):
        self.b, self.p = memoryview(data), 0

    def eof(self) -> bool:
        return self.p >= len(self.b)

    def varint(self) -> int:
        shift = result = 0
        while True:
            c = self.b[self.p]
            self.p += 1
            result |= (c & 0x7F) << shift
            if c < 0x80:
                return result
            shift += 7
            if shift > 63:
                raise ValueError("malformed varint")

    def tag(self) -> Tuple[int, int]:
        t = self.varint()
        return t >> 3, t & 7

    def bytes_(self) -> bytes:
        n = self.varint()
        v = bytes(self.b[self.p:self.p + n])
        self.p += n
        return v

    def fixed32(self) -> bytes:
        v = bytes(self.b[self.p:self.p + 4])
        self.p += 4
        return v

    def fixed64(self) -> bytes:
        v = bytes(self.b[self.p:self.p + 8])
        self.p += 8
        return v

    def skip(self, wire: int) -> None:
        if wire == 0:
            self.varint()
        elif wire == 1:
            self.p += 8
        elif wire == 2:
            self.p += self.varint()
        elif wire == 5:
            self.p += 4
        else:
            raise ValueError(f"unsupported wire type {wire}")

    def fields(self):
        while not self.eof():
            f, w = self.tag()
            yield f, w


def _signed64(v: int) -> int:
    return v - (1 << 64) if v >= 1 << 63 else v


def _packed_varints(data: bytes) -> List[int]:
    r = ProtoReader(data)
    out = []
    while not r.eof():
        out.append(_signed64(r.varint()))
    return out


# ---------------------------------------------------------------- graph model
@dataclass
class TensorData:
    name: str = ""
    data_type: int = FLOAT
    dims: List[int] = field(default_factory=list)
    floats: Optional[np.ndarray] = None
    longs: Optional[np.ndarray] = None

    def to_torch(self) -> torch.Tensor:
        if self.floats is not None:
            return torch.from_numpy(self.floats.astype(np.float32).reshape(self.dims))
        if self.longs is not None:
            return torch.from_numpy(self.longs.astype(np.int64).reshape(self.dims))
        raise NotImplementedError(f"tensor '{self.name}' has unsupported data type {self.data_type}")

    @staticmethod
    def from_torch(name: str, t: torch.Tensor) -> "TensorData":
        t = t.detach().cpu()
        if t.is_floating_point():
            return TensorData(name, FLOAT, list(t.shape), floats=t.float().numpy().reshape(-1))
        return TensorData(name, INT64, list(t.shape), longs=t.long().numpy().reshape(-1))


@dataclass
class Attribute:
    name: str = ""
    type: int = 0
    f: float = 0.0
    i: int = 0
    s: Optional[str] = None
    floats: Optional[List[float]] = None
    ints: Optional[List[int]] = None
    strings: Optional[List[str]] = None
    t: Optional[TensorData] = None


@dataclass
class Node:
    name: str = ""
    op_type: str = ""
    inputs: List[str] = field(default_factory=list)
    outputs: List[str] = field(default_factory=list)
    attrs: Dict[str, Attribute] = field(default_factory=dict)

    def get_int(self, k, d=0):
        return self.attrs[k].i if k in self.attrs else d

    def get_ints(self, k, d=None):
        a = self.attrs.get(k)
        return list(a.ints) if a is not None and a.ints is not None else (d or [])

    def get_float(self, k, d=0.0):
        return self.attrs[k].f if k in self.attrs else d

    def get_string(self, k, d=""):
        a = self.attrs.get(k)
        return a.s if a is not None and a.s is not None else d


@dataclass
class ValueInfo:
    name: str = ""
    shape: List[int] = field(default_factory=list)


@dataclass
class Graph:
    name: str = ""
    opset: int = 0
    nodes: List[Node] = field(default_factory=list)
    initializers: Dict[str, TensorData] = field(default_factory=dict)
    inputs: List[ValueInfo] = field(default_factory=list)
    outputs: List[ValueInfo] = field(default_factory=list)


# ---------------------------------------------------------------- ONNX parser
def _parse_tensor(data: bytes) -> TensorData:
    t = TensorData()
    raw = None
    f32: List[float] = []
    i64: List[int] = []
    i32: List[int] = []
    r = ProtoReader(data)
    for f, w in r.fields():
        if f == 1:
            t.dims += _packed_varints(r.bytes_()) if w == 2 else [_signed64(r.varint())]
        elif f == 2:
            t.data_type = r.varint()
        elif f == 4:
            if w == 2:
                f32 += list(np.frombuffer(r.bytes_(), "<f4"))
            else:
                f32.append(struct.unpack("<f", r.fixed32())[0])
        elif f == 5:
            i32 += _packed_varints(r.bytes_()) if w == 2 else [_signed64(r.varint())]
        elif f == 7:
            i64 += _packed_varints(r.bytes_()) if w == 2 else [_signed64(r.varint())]
        elif f == 8:
            t.name = r.bytes_().decode()
        elif f == 9:
            raw = r.bytes_()
        else:
            r.skip(w)
    if t.data_type == FLOAT:
        t.floats = np.frombuffer(raw, "<f4").copy() if raw is not None else np.array(f32, np.float32)
    elif t.data_type == INT64:
        t.longs = np.frombuffer(raw, "<i8").copy() if raw is not None else np.array(i64, np.int64)
    elif t.data_type == INT32:
        t.longs = (np.frombuffer(raw, "<i4").astype(np.int64) if raw is not None else np.array(i32, np.int64))
    return t


def _parse_attr(data: bytes) -> Attribute:
    a = Attribute()
    r = ProtoReader(data)
    for f, w in r.fields():
        if f == 1:
            a.name = r.bytes_().decode()
        elif f == 2:
            a.f = struct.unpack("<f", r.fixed32())[0]
        elif f == 3:
            a.i = _signed64(r.varint())
        elif f == 4:
            a.s = r.bytes_().decode("utf-8", "replace")
        elif f == 5:
            a.t = _parse_tensor(r.bytes_())
        elif f == 7:
            a.floats = (a.floats or []) + (list(np.frombuffer(r.bytes_(), "<f4")) if w == 2
                                           else [struct.unpack("<f", r.fixed32())[0]])
        elif f == 8:
            a.ints = (a.ints or []) + (_packed_varints(r.bytes_()) if w == 2 else [_signed64(r.varint())])
        elif f == 9:
            a.strings = (a.strings or []) + [r.bytes_().decode("utf-8", "replace")]
        elif f == 20:
            a.type = r.varint()
        else:
            r.skip(w)
    if a.type == 0:
        a.type = (A_TENSOR if a.t is not None else A_FLOATS if a.floats is not None else A_INTS if a.ints is not None
                  else A_STRING if a.s is not None else A_FLOAT if a.f else A_INT)
    return a


def _parse_node(data: bytes) -> Node:
    n = Node()
    r = ProtoReader(data)
    for f, w in r.fields():
        if f == 1:
            n.inputs.append(r.bytes_().decode())
        elif f == 2:
            n.outputs.append(r.bytes_().decode())
        elif f == 3:
            n.name = r.bytes_().decode()
        elif f == 4:
            n.op_type = r.bytes_().decode()
        elif f == 5:
            a = _parse_attr(r.bytes_())
            n.attrs[a.name] = a
        else:
            r.skip(w)
    return n


def _parse_value_info(data: bytes) -> ValueInfo:
    v = ValueInfo()
    r = ProtoReader(data)
    for f, w in r.fields():
        if f == 1:
            v.name = r.bytes_().decode()
        elif f == 2:                                  # TypeProto -> tensor_type -> shape -> dims
            tr = ProtoReader(r.bytes_())
            for f2, w2 in tr.fields():
                if f2 == 1:
                    tt = ProtoReader(tr.bytes_())
                    for f3, w3 in tt.fields():
                        if f3 == 2:
                            sh = ProtoReader(tt.bytes_())
                            for f4, w4 in sh.fields():
                                if f4 == 1:
                                    dim = ProtoReader(sh.bytes_())
                                    val = -1
                                    for f5, w5 in dim.fields():
                                        if f5 == 1:
                                            val = _signed64(dim.varint())
                                        else:
                                            dim.skip(w5)
                                    v.shape.append(val)
                                else:
                                    sh.skip(w4)
                        else:
                            tt.skip(w3)
                else:
                    tr.skip(w2)
        else:
            r.skip(w)
    return v


def parse_model(data: bytes) -> Graph:
    g = Graph()
    r = ProtoReader(data)
    graph_bytes = None
    for f, w in r.fields():
        if f == 7:
            graph_bytes = r.bytes_()
        elif f == 8:                                  # opset_import
            o = ProtoReader(r.bytes_())
            domain, ver = "", 0
            for f2, w2 in o.fields():
                if f2 == 1:
                    domain = o.bytes_().decode()
                elif f2 == 2:
                    ver = o.varint()
                else:
                    o.skip(w2)
            if domain in ("", "ai.onnx"):
                g.opset = ver
        else:
            r.skip(w)
    if graph_bytes is None:
        raise ValueError("ModelProto has no graph")
    gr = ProtoReader(graph_bytes)
    for f, w in gr.fields():
        if f == 1:
            g.nodes.append(_parse_node(gr.bytes_()))
        elif f == 2:
            g.name = gr.bytes_().decode()
        elif f == 5:
            t = _parse_tensor(gr.bytes_())
            g.initializers[t.name] = t
        elif f == 11:
            g.inputs.append(_parse_value_info(gr.bytes_()))
        elif f == 12:
            g.outputs.append(_parse_value_info(gr.bytes_()))
        else:
            gr.skip(w)
    g.inputs = [v for v in g.inputs if v.name not in g.initializers]
    return g


# ---------------------------------------------------------------- protobuf writer (for building test models)
def _vi(v: int) -> bytes:
    v &= (1 << 64) - 1
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        out.append(b | (0x80 if v else 0))
        if not v:
            return bytes(out)


def _fld(num: int, wire: int, payload: bytes) -> bytes:
    return _vi((num << 3) | wire) + (_vi(len(payload)) + payload if wire == 2 else payload)


def encode_model(g: Graph) -> bytes:
    """ModelProto bytes for a Graph (ir_version 8, one ai.onnx opset)."""
    def tensor(t: TensorData) -> bytes:
        b = b"".join(_fld(1, 0, _vi(d)) for d in t.dims) + _fld(2, 0, _vi(t.data_type)) + _fld(8, 2, t.name.encode())
        raw = t.floats.astype("<f4").tobytes() if t.floats is not None else t.longs.astype("<i8").tobytes()
        return b + _fld(9, 2, raw)

    def attr(a: Attribute) -> bytes:
        b = _fld(1, 2, a.name.encode()) + _fld(20, 0, _vi(a.type))
        if a.type == A_FLOAT:
            b += _fld(2, 5, struct.pack("<f", a.f))
        elif a.type == A_INT:
            b += _fld(3, 0, _vi(a.i))
        elif a.type == A_STRING:
            b += _fld(4, 2, (a.s or "").encode())
        elif a.type == A_TENSOR:
            b += _fld(5, 2, tensor(a.t))
        elif a.type == A_FLOATS:
            b += _fld(7, 2, np.asarray(a.floats, "<f4").tobytes())
        elif a.type == A_INTS:
            b += _fld(8, 2, b"".join(_vi(i) for i in a.ints))
        return b

    def vinfo(v: ValueInfo) -> bytes:
        dims = b"".join(_fld(1, 2, _fld(1, 0, _vi(d))) for d in v.shape)
        return _fld(1, 2, v.name.encode()) + _fld(2, 2, _fld(1, 2, _fld(1, 0, _vi(1)) + _fld(2, 2, dims)))

    gb = b"".join(_fld(1, 2, b"".join(_fld(1, 2, i.encode()) for i in n.inputs)
                       + b"".join(_fld(2, 2, o.encode()) for o in n.outputs)
                       + _fld(3, 2, n.name.encode()) + _fld(4, 2, n.op_type.encode())
                       + b"".join(_fld(5, 2, attr(a)) for a in n.attrs.values())) for n in g.nodes)
    gb += _fld(2, 2, g.name.encode())
    gb += b"".join(_fld(5, 2, tensor(t)) for t in g.initializers.values())
    gb += b"".join(_fld(11, 2, vinfo(v)) for v in g.inputs) + b"".join(_fld(12, 2, vinfo(v)) for v in g.outputs)
    return _fld(1, 0, _vi(8)) + _fld(7, 2, gb) + _fld(8, 2, _fld(2, 0, _vi(g.opset or 13)))


# ---------------------------------------------------------------- kernels
def _pads(n: Node, spatial: int) -> List[int]:
    p = n.get_ints("pads", [0] * (2 * spatial))
    return p


def _conv(n, x, w, b=None):
    k = w.shape[2:]
    s = n.get_ints("strides", [1] * len(k))
    d = n.get_ints("dilations", [1] * len(k))
    p = _pads(n, len(k))
    if n.get_string("auto_pad", "NOTSET") in ("SAME_UPPER", "SAME_LOWER"):
        tot = [max(0, (-(-x.shape[2 + i] // s[i]) - 1) * s[i] + (k[i] - 1) * d[i] + 1 - x.shape[2 + i])
               for i in range(len(k))]
        p = [t // 2 for t in tot] + [t - t // 2 for t in tot]
    if len(k) == 2:
        x = F.pad(x, (p[1], p[3], p[0], p[2]))
        return F.conv2d(x, w, b, s, 0, d, n.get_int("group", 1))
    x = F.pad(x, (p[0], p[1]))
    return F.conv1d(x, w, b, s, 0, d, n.get_int("group", 1))


def _pool(n, x, kind):
    k = n.get_ints("kernel_shape")
    s = n.get_ints("strides", [1] * len(k))
    p = _pads(n, len(k))
    if kind == "max":
        x = F.pad(x, (p[1], p[3], p[0], p[2]), value=float("-inf"))
        return F.max_pool2d(x, k, s, ceil_mode=bool(n.get_int("ceil_mode", 0)))
    cip = bool(n.get_int("count_include_pad", 0))
    if cip or not any(p):
        return F.avg_pool2d(F.pad(x, (p[1], p[3], p[0], p[2])), k, s, ceil_mode=bool(n.get_int("ceil_mode", 0)))
    num = F.avg_pool2d(F.pad(x, (p[1], p[3], p[0], p[2])), k, s, divisor_override=1)
    den = F.avg_pool2d(F.pad(torch.ones_like(x[:, :1]), (p[1], p[3], p[0], p[2])), k, s, divisor_override=1)
    return num / den


def _gemm(n, a, b, c=None):
    if n.get_int("transA", 0):
        a = a.T
    if n.get_int("transB", 0):
        b = b.T
    y = n.get_float("alpha", 1.0) * (a @ b)
    if c is not None:
        y = y + n.get_float("beta", 1.0) * c
    return y


def _axes(n, inputs, default=None):
    if len(inputs) > 1 and inputs[1] is not None:
        return [int(v) for v in inputs[1].reshape(-1).tolist()]
    return n.get_ints("axes", default)


def _reduce(fn):
    def k(n, *inp):
        x = inp[0]
        ax = _axes(n, inp, list(range(x.dim())))
        keep = bool(n.get_int("keepdims", 1))
        if not ax:
            return x.clone() if n.get_int("noop_with_empty_axes", 0) else fn(x, list(range(x.dim())), keep)
        return fn(x, ax, keep)
    return k


def _slice(n, x, starts=None, ends=None, axes=None, steps=None):
    st = starts.tolist() if starts is not None else n.get_ints("starts")
    en = ends.tolist() if ends is not None else n.get_ints("ends")
    ax = axes.tolist() if axes is not None else n.get_ints("axes", list(range(len(st))))
    sp = steps.tolist() if steps is not None else [1] * len(st)
    idx = [slice(None)] * x.dim()
    for s, e, a, k in zip(st, en, ax, sp):
        dim = x.shape[a]
        if k < 0:
            raise NotImplementedError("negative Slice steps")
        s = max(0, min(dim, s + dim if s < 0 else s))
        e = max(0, min(dim, e + dim if e < 0 else e))
        idx[a] = slice(s, e, k)
    return x[tuple(idx)]


def _resize(n, x, roi=None, scales=None, sizes=None):
    mode = n.get_string("mode", "nearest")
    if sizes is not None and sizes.numel():
        size = [int(v) for v in sizes.tolist()[2:]]
    else:
        size = [int(x.shape[2 + i] * scales.tolist()[2 + i]) for i in range(x.dim() - 2)]
    if mode == "nearest":
        return F.interpolate(x, size=size, mode="nearest")
    ac = n.get_string("coordinate_transformation_mode", "half_pixel") == "align_corners"
    return F.interpolate(x, size=size, mode="bilinear" if x.dim() == 4 else "linear", align_corners=ac)


def _batchnorm(n, x, scale, bias, mean, var):
    eps = n.get_float("epsilon", 1e-5)
    shape = [1, -1] + [1] * (x.dim() - 2)
    return (x - mean.view(shape)) / torch.sqrt(var.view(shape) + eps) * scale.view(shape) + bias.view(shape)


def _reshape(n, x, shape):
    s = [int(v) for v in shape.tolist()]
    if not n.get_int("allowzero", 0):
        s = [x.shape[i] if v == 0 else v for i, v in enumerate(s)]
    return x.reshape(s)


def _unsqueeze(n, x, axes=None):
    ax = axes.tolist() if axes is not None else n.get_ints("axes")
    for a in sorted(int(v) + (x.dim() + len(ax) if v < 0 else 0) for v in ax):
        x = x.unsqueeze(a)
    return x


def _squeeze(n, x, axes=None):
    ax = axes.tolist() if axes is not None else n.get_ints("axes")
    if not ax:
        return x.squeeze()
    for a in sorted((int(v) % x.dim() for v in ax), reverse=True):
        x = x.squeeze(a)
    return x


def _softmax(n, x):
    return torch.softmax(x, n.get_int("axis", -1))


KERNELS: Dict[str, Callable] = {
    "Conv": _conv, "Gemm": _gemm, "MatMul": lambda n, a, b: a @ b,
    "Add": lambda n, a, b: a + b, "Sub": lambda n, a, b: a - b, "Mul": lambda n, a, b: a * b,
    "Div": lambda n, a, b: a / b if a.is_floating_point() or b.is_floating_point() else torch.div(a, b, rounding_mode="trunc"),
    "Pow": lambda n, a, b: torch.pow(a, b), "Sqrt": lambda n, x: torch.sqrt(x), "Exp": lambda n, x: torch.exp(x),
    "Log": lambda n, x: torch.log(x), "Neg": lambda n, x: -x, "Abs": lambda n, x: x.abs(),
    "Reciprocal": lambda n, x: 1.0 / x, "Floor": lambda n, x: torch.floor(x), "Ceil": lambda n, x: torch.ceil(x),
    "Relu": lambda n, x: F.relu(x), "Sigmoid": lambda n, x: torch.sigmoid(x), "Tanh": lambda n, x: torch.tanh(x),
    "LeakyRelu": lambda n, x: F.leaky_relu(x, n.get_float("alpha", 0.01)),
    "HardSigmoid": lambda n, x: torch.clamp(n.get_float("alpha", 0.2) * x + n.get_float("beta", 0.5), 0, 1),
    "Erf": lambda n, x: torch.erf(x), "Softmax": _softmax,
    "Clip": lambda n, x, lo=None, hi=None: torch.clamp(
        x, lo.item() if lo is not None else n.get_float("min", -3.4e38), hi.item() if hi is not None else n.get_float("max", 3.4e38)),
    "MaxPool": lambda n, x: _pool(n, x, "max"), "AveragePool": lambda n, x: _pool(n, x, "avg"),
    "GlobalAveragePool": lambda n, x: x.mean(dim=tuple(range(2, x.dim())), keepdim=True),
    "GlobalMaxPool": lambda n, x: x.amax(dim=tuple(range(2, x.dim())), keepdim=True),
    "BatchNormalization": _batchnorm,
    "Flatten": lambda n, x: x.reshape(int(np.prod(x.shape[:n.get_int("axis", 1)])), -1),
    "Reshape": _reshape, "Transpose": lambda n, x: x.permute(n.get_ints("perm", list(range(x.dim()))[::-1])),
    "Concat": lambda n, *xs: torch.cat([x for x in xs if x is not None and x.numel() > 0] or [xs[0]], n.get_int("axis", 0)),
    "Gather": lambda n, x, i: torch.index_select(x, n.get_int("axis", 0), i.reshape(-1).long() % x.shape[n.get_int("axis", 0)])
        .reshape(list(x.shape[:n.get_int("axis", 0)]) + list(i.shape) + list(x.shape[n.get_int("axis", 0) + 1:])),
    "Unsqueeze": _unsqueeze, "Squeeze": _squeeze, "Shape": lambda n, x: torch.tensor(list(x.shape), dtype=torch.int64),
    "Identity": lambda n, x: x, "Dropout": lambda n, x, *r: x, "Slice": _slice, "Resize": _resize,
    "Cast": lambda n, x: x.float() if n.get_int("to", 1) == FLOAT else x.long(),
    "ReduceMean": _reduce(lambda x, a, k: x.mean(a, keepdim=k)), "ReduceSum": _reduce(lambda x, a, k: x.sum(a, keepdim=k)),
    "ReduceMax": _reduce(lambda x, a, k: x.amax(a, keepdim=k)), "ReduceMin": _reduce(lambda x, a, k: x.amin(a, keepdim=k)),
    "Equal": lambda n, a, b: a == b, "Greater": lambda n, a, b: a > b, "Less": lambda n, a, b: a < b,
    "Not": lambda n, x: ~x.bool(), "And": lambda n, a, b: a.bool() & b.bool(), "Or": lambda n, a, b: a.bool() | b.bool(),
    "Where": lambda n, c, a, b: torch.where(c.bool(), a, b),
    "ConstantOfShape": lambda n, s: torch.full([int(v) for v in s.tolist()],
                                               float(n.attrs["value"].t.to_torch().reshape(-1)[0]) if "value" in n.attrs else 0.0),
    "Expand": lambda n, x, s: x.expand(*[int(v) if int(v) != 1 else -1 for v in s.tolist()]) if x.dim() == len(s) else x * torch.ones([int(v) for v in s.tolist()]),
    "Range": lambda n, a, b, d: torch.arange(a.item(), b.item(), d.item()),
    "ArgMax": lambda n, x: x.argmax(n.get_int("axis", 0), keepdim=bool(n.get_int("keepdims", 1))),
}


def constant_payload(n: Node) -> Optional[TensorData]:
    a = n.attrs.get("value")
    if a is not None and a.t is not None:
        return a.t
    if "value_float" in n.attrs:
        return TensorData("", FLOAT, [], floats=np.array([n.attrs["value_float"].f], np.float32))
    if "value_floats" in n.attrs:
        v = n.attrs["value_floats"].floats
        return TensorData("", FLOAT, [len(v)], floats=np.array(v, np.float32))
    if "value_int" in n.attrs:
        return TensorData("", INT64, [], longs=np.array([n.attrs["value_int"].i], np.int64))
    if "value_ints" in n.attrs:
        v = n.attrs["value_ints"].ints
        return TensorData("", INT64, [len(v)], longs=np.array(v, np.int64))
    return None


def run_node(n: Node, args: List[Optional[torch.Tensor]]) -> List[torch.Tensor]:
    if n.op_type == "Constant":
        p = constant_payload(n)
        if p is None:
            raise NotImplementedError("Constant node without a numeric payload")
        return [p.to_torch()]
    k = KERNELS.get(n.op_type)
    if k is None:
        raise NotImplementedError(f"ONNX op '{n.op_type}' is not supported")
    out = k(n, *args)
    return list(out) if isinstance(out, (tuple, list)) else [out]


# ---------------------------------------------------------------- executor
class OnnxModel:
    def __init__(self, graph: Graph, device: str = "cpu"):
        self.graph = graph
        self.device = torch.device(device)
        self.consts = {k: v.to_torch().to(self.device) for k, v in graph.initializers.items()}

    @staticmethod
    def load(path_or_bytes, device: str = "cpu") -> "OnnxModel":
        data = path_or_bytes if isinstance(path_or_bytes, (bytes, bytearray)) else open(path_or_bytes, "rb").read()
        g = read_pcnx(data) if looks_like_pcnx(data) else parse_model(bytes(data))
        return OnnxModel(g, device)

    def save(self, path: str, optimize: bool = True) -> None:
        write_pcnx(path, optimize_graph(self.graph) if optimize else self.graph)

    @property
    def input_names(self) -> List[str]:
        return [v.name for v in self.graph.inputs]

    @property
    def output_names(self) -> List[str]:
        return [v.name for v in self.graph.outputs]

    @torch.no_grad()
    def run(self, inputs: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        env: Dict[str, torch.Tensor] = dict(self.consts)
        for k, v in inputs.items():
            env[k] = torch.as_tensor(v).to(self.device)
        missing = [n for n in self.input_names if n not in env]
        if missing:
            raise ValueError(f"missing inputs {missing}")
        for n in self.graph.nodes:
            args = [env[i] if i else None for i in n.inputs]
            for name, val in zip(n.outputs, run_node(n, args)):
                env[name] = val
        return {o: env[o] for o in self.output_names}


# ---------------------------------------------------------------- optimizer
FOLD_CAP = 16_000_000


def optimize_graph(g: Graph) -> Graph:
    """Constant nodes -> initializers, constant folding, Identity/Dropout elision, dead-code removal."""
    import copy
    g = copy.deepcopy(g)
    keep = []
    for n in g.nodes:
        p = constant_payload(n) if n.op_type == "Constant" else None
        if p is not None:
            p = TensorData(n.outputs[0], p.data_type, list(p.dims), p.floats, p.longs)
            g.initializers[n.outputs[0]] = p
        else:
            keep.append(n)
    g.nodes = keep
    folded = []
    for n in g.nodes:
        if n.inputs and all((not i) or i in g.initializers for i in n.inputs) and n.op_type in KERNELS \
                and n.op_type not in ("Dropout",):
            outs = run_node(n, [g.initializers[i].to_torch() if i else None for i in n.inputs])
            if sum(o.numel() for o in outs) <= FOLD_CAP:
                for name, o in zip(n.outputs, outs):
                    g.initializers[name] = TensorData.from_torch(name, o)
                continue
        folded.append(n)
    g.nodes = folded
    rename: Dict[str, str] = {}
    outs = {v.name for v in g.outputs}
    kept = []
    for n in g.nodes:
        n.inputs = [rename.get(i, i) for i in n.inputs]
        if n.op_type in ("Identity", "Dropout") and n.outputs[0] not in outs:
            rename[n.outputs[0]] = n.inputs[0]
            continue
        kept.append(n)
    needed = set(outs)
    live = []
    for n in reversed(kept):
        if any(o in needed for o in n.outputs):
            live.append(n)
            needed.update(i for i in n.inputs if i)
    g.nodes = live[::-1]
    g.initializers = {k: v for k, v in g.initializers.items() if k in needed}
    return g


# ---------------------------------------------------------------- PCNX
_MAGIC, _VERSION = b"PCNX", 1


def looks_like_pcnx(b: bytes) -> bool:
    return bytes(b[:4]) == _MAGIC


def _wstr(w: io.BytesIO, s: str) -> None:
    b = s.encode("utf-8")
    n = len(b)
    while True:
        c = n & 0x7F
        n >>= 7
        w.write(bytes([c | (0x80 if n else 0)]))
        if not n:
            break
    w.write(b)


def _rstr(r: io.BytesIO) -> str:
    n = shift = 0
    while True:
        c = r.read(1)[0]
        n |= (c & 0x7F) << shift
        if c < 0x80:
            break
        shift += 7
    return r.read(n).decode("utf-8")


def _wtensor(w, t: TensorData) -> None:
    _wstr(w, t.name)
    w.write(struct.pack("<ii", t.data_type, len(t.dims)))
    for d in t.dims:
        w.write(struct.pack("<q", d))
    if t.floats is not None:
        w.write(struct.pack("<Bi", 1, t.floats.size) + t.floats.astype("<f4").tobytes())
    elif t.longs is not None:
        w.write(struct.pack("<Bi", 2, t.longs.size) + t.longs.astype("<i8").tobytes())
    else:
        w.write(b"\x00")


def _rtensor(r) -> TensorData:
    t = TensorData(_rstr(r))
    t.data_type, nd = struct.unpack("<ii", r.read(8))
    t.dims = list(struct.unpack(f"<{nd}q", r.read(8 * nd)))
    kind = r.read(1)[0]
    if kind == 1:
        n = struct.unpack("<i", r.read(4))[0]
        t.floats = np.frombuffer(r.read(4 * n), "<f4").copy()
    elif kind == 2:
        n = struct.unpack("<i", r.read(4))[0]
        t.longs = np.frombuffer(r.read(8 * n), "<i8").copy()
    elif kind != 0:
        raise ValueError(f"unknown PCNX tensor payload kind {kind}")
    return t


def pcnx_bytes(g: Graph) -> bytes:
    w = io.BytesIO()
    w.write(_MAGIC + struct.pack("<iq", _VERSION, g.opset))
    _wstr(w, g.name)
    for infos in (g.inputs, g.outputs):
        w.write(struct.pack("<i", len(infos)))
        for v in infos:
            _wstr(w, v.name)
            w.write(struct.pack(f"<i{len(v.shape)}i", len(v.shape), *v.shape))
    w.write(struct.pack("<i", len(g.initializers)))
    for name, t in g.initializers.items():
        _wstr(w, name)
        _wtensor(w, t)
    w.write(struct.pack("<i", len(g.nodes)))
    for n in g.nodes:
        _wstr(w, n.name)
        _wstr(w, n.op_type)
        for names in (n.inputs, n.outputs):
            w.write(struct.pack("<i", len(names)))
            for s in names:
                _wstr(w, s)
        w.write(struct.pack("<i", len(n.attrs)))
        for a in n.attrs.values():
            _wstr(w, a.name)
            w.write(bytes([a.type]))
            if a.type == A_FLOAT:
                w.write(struct.pack("<f", a.f))
            elif a.type == A_INT:
                w.write(struct.pack("<q", a.i))
            elif a.type == A_STRING:
                w.write(b"\x01" if a.s is not None else b"\x00")
                if a.s is not None:
                    _wstr(w, a.s)
            elif a.type == A_FLOATS:
                v = np.asarray(a.floats or [], "<f4")
                w.write(struct.pack("<i", v.size) + v.tobytes())
            elif a.type == A_INTS:
                v = np.asarray(a.ints or [], "<i8")
                w.write(struct.pack("<i", v.size) + v.tobytes())
            elif a.type == A_STRINGS:
                w.write(struct.pack("<i", len(a.strings or [])))
                for s in a.strings or []:
                    _wstr(w, s)
            elif a.type == A_TENSOR:
                w.write(b"\x01" if a.t is not None else b"\x00")
                if a.t is not None:
                    _wtensor(w, a.t)
            else:
                raise ValueError(f"attribute type {a.type} cannot be stored in PCNX")
    return w.getvalue()


def write_pcnx(path: str, g: Graph) -> None:
    import os
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(pcnx_bytes(g))
    os.replace(tmp, path)


def read_pcnx(data: bytes) -> Graph:
    r = io.BytesIO(bytes(data))
    if r.read(4) != _MAGIC:
        raise ValueError("Not a PCNX model file (bad magic).")
    ver, opset = struct.unpack("<iq", r.read(12))
    if ver != _VERSION:
        raise ValueError(f"PCNX version {ver} is not supported")
    g = Graph(_rstr(r), opset)
    for lst in (g.inputs, g.outputs):
        for _ in range(struct.unpack("<i", r.read(4))[0]):
            name = _rstr(r)
            nd = struct.unpack("<i", r.read(4))[0]
            lst.append(ValueInfo(name, list(struct.unpack(f"<{nd}i", r.read(4 * nd)))))
    for _ in range(struct.unpack("<i", r.read(4))[0]):
        name = _rstr(r)
        g.initializers[name] = _rtensor(r)
    for _ in range(struct.unpack("<i", r.read(4))[0]):
        n = Node(_rstr(r), _rstr(r))
        for lst in (n.inputs, n.outputs):
            lst.extend(_rstr(r) for _ in range(struct.unpack("<i", r.read(4))[0]))
        for _ in range(struct.unpack("<i", r.read(4))[0]):
            a = Attribute(_rstr(r), r.read(1)[0])
            if a.type == A_FLOAT:
                a.f = struct.unpack("<f", r.read(4))[0]
            elif a.type == A_INT:
                a.i = struct.unpack("<q", r.read(8))[0]
            elif a.type == A_STRING:
                a.s = _rstr(r) if r.read(1)[0] else None
            elif a.type == A_FLOATS:
                k = struct.unpack("<i", r.read(4))[0]
                a.floats = list(np.frombuffer(r.read(4 * k), "<f4"))
            elif a.type == A_INTS:
                k = struct.unpack("<i", r.read(4))[0]
                a.ints = list(np.frombuffer(r.read(8 * k), "<i8").astype(int))
            elif a.type == A_STRINGS:
                a.strings = [_rstr(r) for _ in range(struct.unpack("<i", r.read(4))[0])]
            elif a.type == A_TENSOR:
                a.t = _rtensor(r) if r.read(1)[0] else None
            n.attrs[a.name] = a
        g.nodes.append(n)
    return g
