"""The in-house ONNX executor op by op (the checks of PredictiveCoding.UnitTests' OnnxOpsTests,
OnnxParserTests, OnnxResizeTests and OnnxTransformerOpsTests, restated): every graph goes through the
protobuf writer and parser before it runs, and each op is compared with the PyTorch statement of the
ONNX operator's definition."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from predicitivecoding_b200.systems.onnx import (FLOAT, INT64, Attribute, Graph, Node, OnnxModel, TensorData,
                                                 ValueInfo, encode_model, optimize_graph, parse_model)

A_INT, A_INTS, A_FLOAT = 2, 7, 1   # ONNX AttributeProto types


def ints(name, v):
    return Attribute(name=name, type=A_INTS, ints=list(v))


def iattr(name, v):
    return Attribute(name=name, type=A_INT, i=int(v))


def fattr(name, v):
    return Attribute(name=name, type=A_FLOAT, f=float(v))


def run(op, inputs, attrs=(), consts=None, n_out=1):
    """One-node graph: inputs (name -> tensor) are graph inputs, consts become initializers."""
    consts = consts or {}
    names = list(inputs) + list(consts)
    node = Node(name="n", op_type=op, inputs=names, outputs=[f"y{i}" for i in range(n_out)],
                attrs={a.name: a for a in attrs})
    g = Graph(name="g", opset=17, nodes=[node],
              initializers={k: TensorData.from_torch(k, v) for k, v in consts.items()},
              inputs=[ValueInfo(k, list(v.shape)) for k, v in inputs.items()],
              outputs=[ValueInfo(f"y{i}") for i in range(n_out)])
    m = OnnxModel(parse_model(encode_model(g)))
    out = m.run(inputs)
    return [out[f"y{i}"] for i in range(n_out)] if n_out > 1 else out["y0"]


X = torch.randn(2, 3, 8, 8, generator=torch.Generator().manual_seed(0))


@pytest.mark.parametrize("op,fn", [
    ("Relu", F.relu), ("Sigmoid", torch.sigmoid), ("Tanh", torch.tanh), ("Exp", torch.exp), ("Neg", torch.neg),
    ("Abs", torch.abs), ("Floor", torch.floor), ("Ceil", torch.ceil), ("Erf", torch.erf),
])
def test_unary_ops(op, fn):
    assert torch.allclose(run(op, {"x": X}), fn(X))


@pytest.mark.parametrize("op,fn", [("Add", torch.add), ("Sub", torch.sub), ("Mul", torch.mul), ("Div", torch.div)])
def test_broadcasting_binary_ops(op, fn):
    b = torch.rand(3, 1, 1) + 0.5
    assert torch.allclose(run(op, {"x": X}, consts={"b": b}), fn(X, b))


def test_conv_with_stride_padding_and_bias():
    w = torch.randn(4, 3, 3, 3)
    b = torch.randn(4)
    y = run("Conv", {"x": X}, [ints("strides", [2, 2]), ints("pads", [1, 1, 1, 1])], {"w": w, "b": b})
    assert torch.allclose(y, F.conv2d(X, w, b, stride=2, padding=1), atol=1e-5)


def test_gemm_with_transposes_and_scales():
    a, b, c = torch.randn(3, 5), torch.randn(4, 5), torch.randn(4)
    y = run("Gemm", {"a": a}, [iattr("transB", 1), fattr("alpha", 0.5), fattr("beta", 2.0)], {"b": b, "c": c})
    assert torch.allclose(y, 0.5 * a @ b.T + 2.0 * c, atol=1e-5)


def test_pools_and_global_pools():
    mp = run("MaxPool", {"x": X}, [ints("kernel_shape", [2, 2]), ints("strides", [2, 2])])
    assert torch.equal(mp, F.max_pool2d(X, 2, 2))
    ap = run("AveragePool", {"x": X}, [ints("kernel_shape", [3, 3]), ints("strides", [1, 1]), ints("pads", [1, 1, 1, 1])])
    assert torch.allclose(ap, F.avg_pool2d(X, 3, 1, 1, count_include_pad=False), atol=1e-6) or \
        torch.allclose(ap, F.avg_pool2d(X, 3, 1, 1), atol=1e-6)
    assert torch.allclose(run("GlobalAveragePool", {"x": X}), X.mean((2, 3), keepdim=True))
    assert torch.equal(run("GlobalMaxPool", {"x": X}), X.amax((2, 3), keepdim=True))


def test_batch_normalization_inference():
    s, bb, mu, var = torch.rand(3) + 0.5, torch.randn(3), torch.randn(3), torch.rand(3) + 0.1
    y = run("BatchNormalization", {"x": X}, [fattr("epsilon", 1e-5)], {"s": s, "b": bb, "m": mu, "v": var})
    assert torch.allclose(y, F.batch_norm(X, mu, var, s, bb, False, 0.0, 1e-5), atol=1e-5)


def test_shape_ops_reshape_transpose_flatten_squeeze():
    r = run("Reshape", {"x": X}, consts={"s": torch.tensor([2, -1], dtype=torch.int64)})
    assert r.shape == (2, 192)
    t = run("Transpose", {"x": X}, [ints("perm", [0, 2, 3, 1])])
    assert torch.equal(t, X.permute(0, 2, 3, 1))
    f = run("Flatten", {"x": X}, [iattr("axis", 2)])
    assert f.shape == (6, 64)
    u = run("Unsqueeze", {"x": X[0, 0]}, consts={"a": torch.tensor([0], dtype=torch.int64)})
    assert u.shape == (1, 8, 8)
    sq = run("Squeeze", {"x": X[:1]}, consts={"a": torch.tensor([0], dtype=torch.int64)})
    assert sq.shape == (3, 8, 8)


def test_concat_gather_and_slice():
    c = run("Concat", {"x": X}, [iattr("axis", 1)], {"y": torch.ones(2, 1, 8, 8)})
    assert c.shape == (2, 4, 8, 8)
    g = run("Gather", {"x": X}, [iattr("axis", 1)], {"i": torch.tensor([2, 0], dtype=torch.int64)})
    assert torch.equal(g, X[:, [2, 0]])
    s = run("Slice", {"x": X}, consts={"st": torch.tensor([1, 2], dtype=torch.int64),
                                       "en": torch.tensor([3, 8], dtype=torch.int64),
                                       "ax": torch.tensor([1, 3], dtype=torch.int64),
                                       "sp": torch.tensor([1, 3], dtype=torch.int64)})
    assert torch.equal(s, X[:, 1:3, :, 2:8:3])


def test_softmax_and_reductions():
    sm = run("Softmax", {"x": X}, [iattr("axis", -1)])
    assert torch.allclose(sm, torch.softmax(X, -1), atol=1e-6)
    rm = run("ReduceMean", {"x": X}, [ints("axes", [2, 3]), iattr("keepdims", 0)])
    assert torch.allclose(rm, X.mean((2, 3)), atol=1e-6)
    am = run("ArgMax", {"x": X}, [iattr("axis", 1), iattr("keepdims", 0)])
    assert torch.equal(am, X.argmax(1))


def test_resize_nearest_by_scales():
    y = run("Resize", {"x": X}, [Attribute(name="mode", type=3, s="nearest")],
            {"roi": torch.zeros(0), "sc": torch.tensor([1.0, 1.0, 2.0, 2.0])})
    assert y.shape == (2, 3, 16, 16)
    assert torch.equal(y[:, :, ::2, ::2], X)


def test_logic_where_and_clip():
    lo, hi = torch.tensor(-0.5), torch.tensor(0.5)
    assert torch.equal(run("Clip", {"x": X}, consts={"lo": lo, "hi": hi}), X.clamp(-0.5, 0.5))
    cond = X > 0
    w = run("Where", {"c": cond.float(), "a": X}, consts={"b": torch.zeros_like(X)})
    assert torch.equal(w, torch.where(cond, X, torch.zeros_like(X)))
    assert torch.equal(run("Greater", {"a": X}, consts={"b": torch.zeros(1)}), X > 0)


def test_optimizer_folds_constants_and_keeps_the_result():
    n1 = Node("c1", "Add", ["w", "w"], ["w2"])
    n2 = Node("m", "Mul", ["x", "w2"], ["y"])
    g = Graph("g", 17, [n1, n2], {"w": TensorData.from_torch("w", torch.full((4,), 1.5))},
              [ValueInfo("x", [4])], [ValueInfo("y")])
    x = torch.arange(4.0)
    ref = OnnxModel(g).run({"x": x})["y"]
    opt = optimize_graph(g)
    assert len(opt.nodes) == 1
    assert torch.equal(OnnxModel(opt).run({"x": x})["y"], ref)


def test_unknown_ops_are_reported():
    with pytest.raises(NotImplementedError):
        run("NoSuchOp", {"x": X})
