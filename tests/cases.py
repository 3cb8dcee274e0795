"""Seeded test graphs shared by the golden-fixture generator and the tests.

Each case builds a graph in the reference IR (O0) plus its feeds. The operator matrix follows the
reference's C backend tests (``tests/test_codegen.py:95-389``: unary, broadcast binary, data
movement and reductions, MatMul shapes, Gemm alpha/beta/trans/bias shapes, Conv pads / strides /
dilation / groups / depthwise / SAME_UPPER, pooling) and its fusion tests
(``tests/test_passes.py``: epilogue fusion, LayerNorm and GELU patterns, loop fusion), built
without onnx.
"""

from __future__ import annotations

import math
import sys
import zlib
from collections.abc import Callable
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT / "ml-graph-compiler_b200") not in sys.path:
    sys.path.insert(0, str(ROOT / "ml-graph-compiler_b200"))

from mgc_cuda import zoo  # noqa: E402
from ml_graph_compiler.ir import Graph, TensorType  # noqa: E402
from ml_graph_compiler.shape_inference import infer_shapes  # noqa: E402

Spec = tuple[str, Any]  # ("in", array) | ("const", array) | ("none", None)


def op_graph(op: str, inputs: list[Spec], attrs: dict[str, Any] | None = None, n_outputs: int = 1,
             name: str = "g") -> tuple[Graph, dict[str, np.ndarray]]:
    """A one-node graph: dynamic inputs become graph inputs, the rest constants."""
    g = Graph(name)
    values: list[Any] = []
    feeds: dict[str, np.ndarray] = {}
    for k, (kind, arr) in enumerate(inputs):
        if kind == "none":
            values.append(None)
        elif kind == "in":
            a = np.asarray(arr)
            v = g.add_input(f"x{k}", TensorType(str(a.dtype) if a.dtype != np.bool_ else "bool", a.shape))
            feeds[v.name] = a
            values.append(v)
        else:
            values.append(g.constant(np.asarray(arr), f"c{k}"))
    node = g.add_node(op, values, n_outputs=n_outputs, attrs=attrs or {})
    for k, out in enumerate(node.outputs):
        g.add_output(out, f"y{k}")
    infer_shapes(g)
    return g, feeds


def _seed(name: str) -> int:
    """A seed derived from a case name, stable across processes (unlike ``hash``)."""
    return zlib.crc32(name.encode()) % 10_000


def _rng(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)


def f32(rng: np.random.Generator, *shape: int, scale: float = 1.0) -> np.ndarray:
    return (rng.standard_normal(shape) * scale).astype(np.float32)


def pos(rng: np.random.Generator, *shape: int) -> np.ndarray:
    return (rng.random(shape) + 0.5).astype(np.float32)


@dataclass
class Case:
    name: str
    build: Callable[[], tuple[Graph, dict[str, np.ndarray]]]
    opt: str = "O0"
    big: bool = False           # a whole model: golden stores summaries, tests run it less often
    rtol: float = 1e-4
    atol: float = 1e-5


def _unary(op: str, positive: bool = False) -> Case:
    def build() -> tuple[Graph, dict[str, np.ndarray]]:
        r = _rng(_seed(op))
        x = pos(r, 3, 70) if positive else f32(r, 3, 70, scale=3.0)
        return op_graph(op, [("in", x)])
    return Case(f"unary_{op}", build, atol=2e-6, rtol=2e-5)


def _binary(op: str, a_shape: tuple[int, ...], b_shape: tuple[int, ...], positive: bool = False) -> Case:
    def build() -> tuple[Graph, dict[str, np.ndarray]]:
        r = _rng(7)
        a = pos(r, *a_shape) if positive else f32(r, *a_shape)
        b = pos(r, *b_shape) if positive or op == "Div" else f32(r, *b_shape)
        return op_graph(op, [("in", a), ("in", b)])
    return Case(f"binary_{op}_{'x'.join(map(str, a_shape))}_{'x'.join(map(str, b_shape))}", build)


def _simple(name: str, fn: Callable[[np.random.Generator], tuple[Graph, dict[str, np.ndarray]]], **kw: Any) -> Case:
    return Case(name, lambda: fn(_rng(_seed(name))), **kw)


def op_cases() -> list[Case]:
    cases: list[Case] = []
    for op in ("Relu", "Sigmoid", "Tanh", "Erf", "Exp", "Neg", "Abs", "Floor", "Ceil", "Sin", "Cos",
               "Softplus", "Identity"):
        cases.append(_unary(op))
    for op in ("Sqrt", "Log", "Reciprocal"):
        cases.append(_unary(op, positive=True))
    for op in ("Add", "Sub", "Mul", "Div", "Max", "Min"):
        cases.append(_binary(op, (4, 1, 6), (3, 1)))
    cases.append(_binary("Pow", (5, 7), (7,), positive=True))
    cases.append(_binary("Add", (2, 3, 4, 5), (2, 3, 4, 5)))
    C = cases.append
    C(_simple("compare_all", lambda r: _chain(r, "compare")))
    C(_simple("logic_all", lambda r: _chain(r, "logic")))
    C(_simple("where", lambda r: op_graph("Where", [("in", r.random((3, 4)) > 0.5), ("in", f32(r, 3, 4)), ("in", f32(r, 1, 4))])))
    # innermost extents that are multiples of 4: the four-wide elementwise forms (all-fp32, and
    # mixed dtypes), with leaves broadcast along the innermost and along outer dimensions
    C(_simple("add_inner_bcast", lambda r: op_graph("Add", [("in", f32(r, 2, 3, 8, 12)), ("in", f32(r, 2, 1, 8, 1))])))
    C(_simple("mul_outer_bcast", lambda r: op_graph("Mul", [("in", f32(r, 3, 1, 16)), ("const", f32(r, 5, 16))])))
    C(_simple("where_mask", lambda r: op_graph("Where", [("in", r.random((1, 1, 8, 8)) > 0.5), ("in", f32(r, 2, 3, 8, 8)), ("const", np.float32(-1e9))])))
    C(_simple("clip_inputs_quad", lambda r: op_graph("Clip", [("in", f32(r, 6, 8, scale=5)), ("in", np.float32(-1.5)), ("const", np.float32(2))])))
    C(_simple("cast_f2i", lambda r: op_graph("Cast", [("in", f32(r, 4, 5, scale=10))], {"to": 7})))
    C(_simple("cast_i2f", lambda r: op_graph("Cast", [("in", r.integers(-50, 50, (4, 5)))], {"to": 1})))
    C(_simple("cast_f2b", lambda r: op_graph("Cast", [("in", np.round(f32(r, 4, 5)))], {"to": 9})))
    C(_simple("clip_inputs", lambda r: op_graph("Clip", [("in", f32(r, 6, 7, scale=5)), ("const", np.float32(0)), ("const", np.float32(6))])))
    C(_simple("clip_attrs", lambda r: op_graph("Clip", [("in", f32(r, 6, 7, scale=5))], {"min": -1.0, "max": 2.0})))
    C(_simple("gelu_erf", lambda r: op_graph("Gelu", [("in", f32(r, 5, 9, scale=3))])))
    C(_simple("gelu_tanh", lambda r: op_graph("Gelu", [("in", f32(r, 5, 9, scale=3))], {"approximate": "tanh"})))
    C(_simple("leaky_relu", lambda r: op_graph("LeakyRelu", [("in", f32(r, 5, 9))], {"alpha": 0.2})))
    C(_simple("hard_sigmoid", lambda r: op_graph("HardSigmoid", [("in", f32(r, 5, 9, scale=4))])))
    C(_simple("int_add_bcast", lambda r: op_graph("Add", [("in", r.integers(-9, 9, (3, 4))), ("in", r.integers(-9, 9, (4,)))])))
    C(_simple("int_div", lambda r: op_graph("Div", [("in", r.integers(-90, 90, (3, 4))), ("const", np.asarray([3, -4, 5, 7]))])))
    C(_simple("int_relu", lambda r: op_graph("Relu", [("in", r.integers(-9, 9, (3, 4)))])))
    # data movement
    C(_simple("transpose_nchw_nhwc", lambda r: op_graph("Transpose", [("in", f32(r, 2, 3, 5, 7))], {"perm": [0, 2, 3, 1]})))
    C(_simple("transpose_2d", lambda r: op_graph("Transpose", [("in", f32(r, 33, 17))])))
    C(_simple("transpose_heads", lambda r: op_graph("Transpose", [("in", f32(r, 2, 8, 4, 16))], {"perm": [0, 2, 1, 3]})))
    # the tiled-transpose copy: batch dimensions, ragged 32 x 32 tiles on both transposed axes
    C(_simple("transpose_tiles", lambda r: op_graph("Transpose", [("in", f32(r, 2, 3, 40, 24))], {"perm": [0, 1, 3, 2]})))
    C(_simple("expand", lambda r: op_graph("Expand", [("in", f32(r, 3, 1)), ("const", np.asarray([2, 3, 4]))])))
    C(_simple("slice_steps", lambda r: op_graph("Slice", [("in", f32(r, 6, 9, 5)), ("const", np.asarray([1, -1])), ("const", np.asarray([5, 0])), ("const", np.asarray([0, 1])), ("const", np.asarray([2, -2]))])))
    C(_simple("slice_clamp", lambda r: op_graph("Slice", [("in", f32(r, 6, 9)), ("const", np.asarray([-100])), ("const", np.asarray([1 << 40])), ("const", np.asarray([1]))])))
    C(_simple("concat", lambda r: op_graph("Concat", [("in", f32(r, 2, 3, 4)), ("in", f32(r, 2, 1, 4)), ("const", f32(r, 2, 2, 4))], {"axis": 1})))
    C(_simple("split_sizes", lambda r: op_graph("Split", [("in", f32(r, 4, 9)), ("const", np.asarray([2, 3, 4]))], {"axis": 1}, n_outputs=3)))
    C(_simple("split_equal", lambda r: op_graph("Split", [("in", f32(r, 6, 4))], {"axis": 0}, n_outputs=3)))
    C(_simple("pad_value", lambda r: op_graph("Pad", [("in", f32(r, 2, 3, 4)), ("const", np.asarray([0, 1, 2, 1, 0, 3])), ("const", np.float32(1.5))])))
    C(_simple("tile", lambda r: op_graph("Tile", [("in", f32(r, 2, 3)), ("const", np.asarray([2, 3]))])))
    C(_simple("gather_rows", lambda r: op_graph("Gather", [("const", f32(r, 50, 8)), ("in", np.asarray([[3, -1, 0], [49, 7, 7]]))], {"axis": 0})))
    C(_simple("gather_axis1_scalar", lambda r: op_graph("Gather", [("in", f32(r, 3, 5, 4)), ("const", np.asarray(0))], {"axis": 1})))
    C(_simple("shape_size", lambda r: _shape_chain(r)))
    C(_simple("constant_of_shape", lambda r: op_graph("ConstantOfShape", [("const", np.asarray([2, 3]))], {"value": np.asarray([2.5], np.float32)})))
    C(_simple("range_f", lambda r: op_graph("Range", [("const", np.float32(1.0)), ("const", np.float32(7.0)), ("const", np.float32(0.5))])))
    # reductions and normalisation
    C(_simple("reduce_mean_last", lambda r: op_graph("ReduceMean", [("in", f32(r, 3, 4, 10))], {"axes": [-1], "keepdims": 1})))
    C(_simple("reduce_sum_mid", lambda r: op_graph("ReduceSum", [("in", f32(r, 3, 4, 10)), ("const", np.asarray([1]))], {"keepdims": 0})))
    C(_simple("reduce_max", lambda r: op_graph("ReduceMax", [("in", f32(r, 3, 4, 10))], {"axes": [0, 1], "keepdims": 1})))
    C(_simple("reduce_min", lambda r: op_graph("ReduceMin", [("in", f32(r, 3, 4, 10))], {"axes": [2], "keepdims": 0})))
    C(_simple("reduce_prod", lambda r: op_graph("ReduceProd", [("in", pos(r, 3, 6))], {"axes": [1], "keepdims": 1})))
    C(_simple("reduce_int_sum", lambda r: op_graph("ReduceSum", [("in", r.integers(-9, 9, (3, 5)))], {"axes": [1], "keepdims": 0})))
    C(_simple("argmax", lambda r: op_graph("ArgMax", [("in", f32(r, 4, 7, 3))], {"axis": 1, "keepdims": 0})))
    C(_simple("argmax_keep", lambda r: op_graph("ArgMax", [("in", f32(r, 4, 7))], {"axis": -1, "keepdims": 1})))
    C(_simple("softmax_last", lambda r: op_graph("Softmax", [("in", f32(r, 2, 3, 130, scale=4))], {"axis": -1})))
    C(_simple("softmax_mid", lambda r: op_graph("Softmax", [("in", f32(r, 2, 9, 5, scale=4))], {"axis": 1})))
    C(_simple("log_softmax", lambda r: op_graph("LogSoftmax", [("in", f32(r, 4, 37, scale=4))], {"axis": -1})))
    C(_simple("layer_norm", lambda r: op_graph("LayerNormalization", [("in", f32(r, 6, 96, scale=2)), ("const", pos(r, 96)), ("const", f32(r, 96))], {"axis": -1, "epsilon": 1e-5})))
    C(_simple("layer_norm_odd", lambda r: op_graph("LayerNormalization", [("in", f32(r, 5, 3, 7)), ("const", pos(r, 3, 7)), ("none", None)], {"axis": -2, "epsilon": 1e-3})))
    C(_simple("batch_norm", lambda r: op_graph("BatchNormalization", [("in", f32(r, 2, 5, 4, 3)), ("const", pos(r, 5)), ("const", f32(r, 5)), ("const", f32(r, 5)), ("const", pos(r, 5))], {"epsilon": 1e-5})))
    # matrix products
    C(_simple("matmul_2d", lambda r: op_graph("MatMul", [("in", f32(r, 37, 29)), ("in", f32(r, 29, 41))])))
    C(_simple("matmul_batched_bcast", lambda r: op_graph("MatMul", [("in", f32(r, 2, 1, 4, 5)), ("in", f32(r, 3, 5, 6))])))
    C(_simple("matmul_vec_left", lambda r: op_graph("MatMul", [("in", f32(r, 7)), ("in", f32(r, 3, 7, 5))])))
    C(_simple("matmul_vec_right", lambda r: op_graph("MatMul", [("in", f32(r, 4, 7)), ("in", f32(r, 7))])))
    C(_simple("matmul_const_b", lambda r: op_graph("MatMul", [("in", f32(r, 3, 10, 16)), ("const", f32(r, 16, 24))])))
    C(_simple("gemm_trans", lambda r: op_graph("Gemm", [("in", f32(r, 9, 6)), ("in", f32(r, 11, 9))], {"transA": 1, "transB": 1, "alpha": 0.5})))
    C(_simple("gemm_bias_vec", lambda r: op_graph("Gemm", [("in", f32(r, 6, 9)), ("const", f32(r, 9, 11)), ("const", f32(r, 11))], {"beta": 2.0})))
    C(_simple("gemm_bias_col", lambda r: op_graph("Gemm", [("in", f32(r, 6, 9)), ("const", f32(r, 9, 11)), ("const", f32(r, 6, 1))])))
    C(_simple("gemm_full_c", lambda r: op_graph("Gemm", [("in", f32(r, 6, 9)), ("const", f32(r, 9, 11)), ("in", f32(r, 6, 11))], {"alpha": 1.5, "beta": 0.5})))
    # convolution and pooling
    def conv(r: np.random.Generator, x: tuple[int, ...], w: tuple[int, ...], bias: bool = True, **attrs: Any) -> tuple[Graph, dict[str, np.ndarray]]:
        ins: list[Spec] = [("in", f32(r, *x)), ("const", f32(r, *w, scale=0.3))]
        if bias:
            ins.append(("const", f32(r, w[0])))
        return op_graph("Conv", ins, attrs)
    C(_simple("conv3x3_p1", lambda r: conv(r, (2, 5, 9, 11), (7, 5, 3, 3), kernel_shape=[3, 3], pads=[1, 1, 1, 1])))
    C(_simple("conv3x3_s2", lambda r: conv(r, (1, 4, 12, 10), (6, 4, 3, 3), kernel_shape=[3, 3], strides=[2, 2], pads=[1, 1, 1, 1])))
    C(_simple("conv_dilated", lambda r: conv(r, (1, 3, 13, 13), (4, 3, 3, 3), kernel_shape=[3, 3], dilations=[2, 2], pads=[2, 2, 2, 2])))
    C(_simple("conv_groups", lambda r: conv(r, (2, 6, 8, 8), (4, 3, 3, 3), kernel_shape=[3, 3], group=2, pads=[1, 1, 1, 1])))
    C(_simple("conv_depthwise", lambda r: conv(r, (2, 8, 9, 9), (8, 1, 3, 3), kernel_shape=[3, 3], group=8, strides=[2, 2], pads=[1, 1, 1, 1])))
    # stride-1 depthwise with a ragged last group of four output columns (the four-column form)
    C(_simple("conv_depthwise_s1", lambda r: conv(r, (2, 12, 7, 10), (12, 1, 3, 3), kernel_shape=[3, 3], group=12, pads=[1, 1, 1, 1])))
    C(_simple("conv_same_upper", lambda r: conv(r, (1, 3, 10, 7), (5, 3, 4, 4), kernel_shape=[4, 4], strides=[2, 2], auto_pad="SAME_UPPER")))
    C(_simple("conv_1x1", lambda r: conv(r, (2, 16, 6, 6), (24, 16, 1, 1), bias=False, kernel_shape=[1, 1])))
    C(_simple("conv_stem7x7", lambda r: conv(r, (1, 3, 32, 32), (16, 3, 7, 7), kernel_shape=[7, 7], strides=[2, 2], pads=[3, 3, 3, 3])))
    C(_simple("maxpool", lambda r: op_graph("MaxPool", [("in", f32(r, 2, 3, 11, 11))], {"kernel_shape": [3, 3], "strides": [2, 2], "pads": [1, 1, 1, 1]})))
    C(_simple("maxpool_ceil", lambda r: op_graph("MaxPool", [("in", f32(r, 1, 2, 10, 10))], {"kernel_shape": [3, 3], "strides": [2, 2], "ceil_mode": 1})))
    C(_simple("avgpool_pad", lambda r: op_graph("AveragePool", [("in", f32(r, 1, 3, 9, 9))], {"kernel_shape": [3, 3], "strides": [2, 2], "pads": [1, 1, 1, 1]})))
    C(_simple("avgpool_include", lambda r: op_graph("AveragePool", [("in", f32(r, 1, 3, 9, 9))], {"kernel_shape": [3, 3], "strides": [2, 2], "pads": [1, 1, 1, 1], "count_include_pad": 1, "ceil_mode": 1})))
    C(_simple("global_avg", lambda r: op_graph("GlobalAveragePool", [("in", f32(r, 2, 5, 7, 7))])))
    C(_simple("global_max", lambda r: op_graph("GlobalMaxPool", [("in", f32(r, 2, 5, 4, 3))])))
    return cases


def _chain(r: np.random.Generator, kind: str) -> tuple[Graph, dict[str, np.ndarray]]:
    g = Graph(kind)
    if kind == "compare":
        a = g.add_input("a", TensorType("float32", (4, 5)))
        b = g.add_input("b", TensorType("float32", (5,)))
        feeds = {"a": np.round(f32(r, 4, 5)), "b": np.round(f32(r, 5))}
        for op in ("Equal", "Less", "Greater", "LessOrEqual", "GreaterOrEqual"):
            g.add_output(g.add_node(op, [a, b]).output, op)
    else:
        a = g.add_input("a", TensorType("bool", (3, 4)))
        b = g.add_input("b", TensorType("bool", (3, 4)))
        feeds = {"a": r.random((3, 4)) > 0.5, "b": r.random((3, 4)) > 0.5}
        for op in ("And", "Or", "Xor"):
            g.add_output(g.add_node(op, [a, b]).output, op)
        g.add_output(g.add_node("Not", [a]).output, "Not")
    infer_shapes(g)
    return g, feeds


def _shape_chain(r: np.random.Generator) -> tuple[Graph, dict[str, np.ndarray]]:
    g = Graph("shape")
    x = g.add_input("x", TensorType("float32", (2, 3, 5)))
    g.add_output(g.add_node("Shape", [x]).output, "shape")
    g.add_output(g.add_node("Size", [x]).output, "size")
    g.add_output(g.add_node("Shape", [x], attrs={"start": 1}).output, "shape_tail")
    infer_shapes(g)
    return g, {"x": f32(r, 2, 3, 5)}


# -- fused patterns (each exercised after the reference O3 pipeline) -------------------------------
def _pattern(name: str, builder: Callable[[np.random.Generator], tuple[Graph, dict[str, np.ndarray]]]) -> Case:
    return Case(f"pattern_{name}", lambda: builder(_rng(_seed(name))), opt="O3")


def _p_conv_block(r: np.random.Generator) -> tuple[Graph, dict[str, np.ndarray]]:
    """Conv+BN+ReLU, Conv+BN, residual Add, ReLU -> FusedConv NHWC with residual and relu."""
    g = Graph("conv_block")
    x = g.add_input("x", TensorType("float32", (2, 8, 10, 10)))

    def cbn(v: Any, cin: int, cout: int, k: int) -> Any:
        w = g.constant(f32(r, cout, cin, k, k, scale=0.3))
        y = g.add_node("Conv", [v, w], attrs={"kernel_shape": [k, k], "pads": [k // 2] * 4}).output
        ps = [g.constant(a) for a in (pos(r, cout), f32(r, cout), f32(r, cout, scale=0.1), pos(r, cout))]
        return g.add_node("BatchNormalization", [y, *ps], attrs={"epsilon": 1e-5}).output

    h = g.add_node("Relu", [cbn(x, 8, 8, 3)]).output
    h = cbn(h, 8, 8, 3)
    y = g.add_node("Relu", [g.add_node("Add", [h, x]).output]).output
    e = g.add_node("Clip", [cbn(y, 8, 16, 1), g.constant(np.float32(0)), g.constant(np.float32(6))]).output
    g.add_output(e, "y")
    infer_shapes(g)
    return g, {"x": f32(r, 2, 8, 10, 10)}


def _p_narrow_convs(r: np.random.Generator) -> tuple[Graph, dict[str, np.ndarray]]:
    """A chain of NHWC convolutions with fewer than 32 input channels (3, 8, 12, 6, 16, 28):
    7x7 stride 2 stem, SAME_UPPER 4x4 (asymmetric padding), dilation 2, stride 2, with BN/ReLU
    epilogues and a residual add, so every tap-packing arrangement of the K axis is exercised
    (one to seven 4-channel groups per filter tap, a channel count that needs padding both at the
    graph input and in the middle of the network)."""
    g = Graph("narrow_convs")
    x = g.add_input("x", TensorType("float32", (2, 3, 22, 18)))

    def conv(v: Any, cin: int, cout: int, k: int, bn: bool = True, **attrs: Any) -> Any:
        w = g.constant(f32(r, cout, cin, k, k, scale=0.5 / math.sqrt(cin * k * k) * 3))
        y = g.add_node("Conv", [v, w, g.constant(f32(r, cout, scale=0.1))],
                       attrs={"kernel_shape": [k, k], **attrs}).output
        if bn:
            ps = [g.constant(a) for a in (pos(r, cout), f32(r, cout, scale=0.1), f32(r, cout, scale=0.1), pos(r, cout))]
            y = g.add_node("BatchNormalization", [y, *ps], attrs={"epsilon": 1e-5}).output
        return y

    h = g.add_node("Relu", [conv(x, 3, 8, 7, strides=[2, 2], pads=[3, 3, 3, 3])]).output
    h2 = conv(h, 8, 12, 3, pads=[1, 1, 1, 1])
    h3 = g.add_node("Relu", [conv(h2, 12, 6, 4, auto_pad="SAME_UPPER")]).output
    h4 = conv(h3, 6, 8, 3, dilations=[2, 2], pads=[2, 2, 2, 2])
    h5 = g.add_node("Relu", [g.add_node("Add", [h4, h]).output]).output
    h6 = g.add_node("Relu", [conv(h5, 8, 16, 3, strides=[2, 2], pads=[1, 1, 1, 1])]).output
    h7 = conv(h6, 16, 28, 3, pads=[1, 1, 1, 1])
    y = conv(h7, 28, 5, 5, bn=False, pads=[2, 2, 2, 2])
    g.add_output(y, "y")
    infer_shapes(g)
    return g, {"x": f32(r, 2, 3, 22, 18)}


def narrow_window_chain(r: np.random.Generator, batch: int = 2, h: int = 32, w: int = 48) -> tuple[Graph, dict[str, np.ndarray]]:
    """Narrow-channel convolutions whose output width is a multiple of 8 (the window-row form):
    a 7x7 stride-2 stem on 3 channels, 8 / 12 / 16 / 28 input channels with window rows of one
    or two K blocks, height dilation 2 with width dilation 1, a residual add, and a final stride-2
    layer whose output width (12 at the default size) falls back to tap-packed boxes."""
    g = Graph("narrow_window")
    x = g.add_input("x", TensorType("float32", (batch, 3, h, w)))

    def conv(v: Any, cin: int, cout: int, k: tuple[int, int], **attrs: Any) -> Any:
        wt = g.constant(f32(r, cout, cin, *k, scale=1.5 / math.sqrt(cin * k[0] * k[1])))
        return g.add_node("Conv", [v, wt, g.constant(f32(r, cout, scale=0.1))],
                          attrs={"kernel_shape": list(k), **attrs}).output

    ps = [g.constant(a) for a in (pos(r, 8), f32(r, 8, scale=0.1), f32(r, 8, scale=0.1), pos(r, 8))]
    h1 = conv(x, 3, 8, (7, 7), strides=[2, 2], pads=[3, 3, 3, 3])
    h1 = g.add_node("Relu", [g.add_node("BatchNormalization", [h1, *ps], attrs={"epsilon": 1e-5}).output]).output
    h2 = conv(h1, 8, 12, (3, 3), pads=[1, 1, 1, 1])
    h3 = g.add_node("Relu", [conv(h2, 12, 16, (5, 5), pads=[2, 2, 2, 2])]).output
    h4 = conv(h3, 16, 16, (3, 3), dilations=[2, 1], pads=[2, 1, 2, 1])
    h4 = g.add_node("Relu", [g.add_node("Add", [h4, h3]).output]).output
    h5 = g.add_node("Relu", [conv(h4, 16, 28, (3, 3), pads=[1, 1, 1, 1])]).output
    y = conv(h5, 28, 8, (3, 3), strides=[2, 2], pads=[1, 1, 1, 1])
    g.add_output(y, "y")
    infer_shapes(g)
    return g, {"x": f32(r, batch, 3, h, w)}


def _p_dense_gelu(r: np.random.Generator) -> tuple[Graph, dict[str, np.ndarray]]:
    """MatMul + bias + erf GELU subgraph, MatMul(x, Transpose(W)), residual Add, tanh GELU."""
    g = Graph("dense_gelu")
    x = g.add_input("x", TensorType("float32", (2, 5, 16)))
    w = g.constant(f32(r, 16, 32, scale=0.3))
    h = g.add_node("Add", [g.add_node("MatMul", [x, w]).output, g.constant(f32(r, 32))]).output
    e = g.add_node("Erf", [g.add_node("Div", [h, g.constant(np.float32(math.sqrt(2.0)))]).output]).output
    h = g.add_node("Mul", [g.add_node("Mul", [h, g.add_node("Add", [e, g.constant(np.float32(1.0))]).output]).output,
                            g.constant(np.float32(0.5))]).output
    wt = g.constant(f32(r, 16, 32, scale=0.3))
    o = g.add_node("MatMul", [h, g.add_node("Transpose", [wt], attrs={"perm": [1, 0]}).output]).output
    o = g.add_node("Add", [o, x]).output
    g.add_output(o, "y")
    infer_shapes(g)
    return g, {"x": f32(r, 2, 5, 16)}


def _p_layer_norm(r: np.random.Generator) -> tuple[Graph, dict[str, np.ndarray]]:
    """Decomposed LayerNorm (the below-opset-17 export) -> LayerNormalization."""
    n = zoo._Net("ln", 0)
    x = n.g.add_input("x", TensorType("float32", (3, 7, 24)))
    y = n.layer_norm(x, 24, decomposed=True)
    g = n.done((y, "y"))
    return g, {"x": f32(r, 3, 7, 24, scale=2)}


def _p_loopfuse(r: np.random.Generator) -> tuple[Graph, dict[str, np.ndarray]]:
    """An elementwise chain with broadcasts -> one FusedElementwise."""
    g = Graph("chain")
    x = g.add_input("x", TensorType("float32", (2, 3, 8, 8)))
    m = g.add_input("m", TensorType("float32", (2, 1, 1, 8)))
    t = g.add_node("Div", [x, g.constant(np.float32(8.0))]).output
    t = g.add_node("Add", [t, m]).output
    t = g.add_node("Mul", [t, g.constant(f32(r, 8))]).output
    t = g.add_node("Tanh", [t]).output
    t = g.add_node("Sub", [t, g.constant(np.float32(0.25))]).output
    g.add_output(t, "y")
    infer_shapes(g)
    return g, {"x": f32(r, 2, 3, 8, 8), "m": f32(r, 2, 1, 1, 8)}


def _p_masked_softmax(r: np.random.Generator) -> tuple[Graph, dict[str, np.ndarray]]:
    """Attention-score scale and mask feeding a softmax over the last axis: a causal bool mask
    through Where (GPT-2), an additive fp32 mask broadcast over heads and queries (BERT) into
    LogSoftmax, and a row too short for groups of four."""
    g = Graph("masked_softmax")
    x = g.add_input("x", TensorType("float32", (2, 3, 8, 16)))
    m = g.add_input("m", TensorType("float32", (2, 1, 1, 16)))
    z = g.add_input("z", TensorType("float32", (4, 6)))
    causal = g.constant(np.tril(np.ones((8, 16), dtype=bool)).reshape(1, 1, 8, 16))
    t = g.add_node("Mul", [x, g.constant(np.float32(0.125))]).output
    t = g.add_node("Where", [causal, t, g.constant(np.float32(-1e9))]).output
    g.add_output(g.add_node("Softmax", [t], attrs={"axis": -1}).output, "p")
    u = g.add_node("Div", [x, g.constant(np.float32(4.0))]).output
    u = g.add_node("Add", [u, m]).output
    g.add_output(g.add_node("LogSoftmax", [u], attrs={"axis": 3}).output, "lp")
    w = g.add_node("Mul", [z, g.constant(np.float32(2.0))]).output
    g.add_output(g.add_node("Softmax", [w], attrs={"axis": -1}).output, "q")
    infer_shapes(g)
    mask = np.where(r.random((2, 1, 1, 16)) > 0.25, 0.0, -10000.0).astype(np.float32)
    return g, {"x": f32(r, 2, 3, 8, 16, scale=3), "m": mask, "z": f32(r, 4, 6)}


def _p_softmax_programs(r: np.random.Generator) -> tuple[Graph, dict[str, np.ndarray]]:
    """Softmax over elementwise programs of other shapes: a chain with a tensor operand
    (x * w + 1), a program that reuses an earlier result ((x + 1) * (x - 1), no chain), and rows
    of 256 (two groups of four per lane)."""
    g = Graph("softmax_programs")
    x = g.add_input("x", TensorType("float32", (3, 5, 32)))
    w = g.add_input("w", TensorType("float32", (5, 1)))
    z = g.add_input("z", TensorType("float32", (2, 256)))
    t = g.add_node("Mul", [x, w]).output
    t = g.add_node("Add", [t, g.constant(np.float32(1.0))]).output
    g.add_output(g.add_node("Softmax", [t], attrs={"axis": -1}).output, "chain")
    a = g.add_node("Add", [x, g.constant(np.float32(1.0))]).output
    b = g.add_node("Sub", [x, g.constant(np.float32(1.0))]).output
    g.add_output(g.add_node("LogSoftmax", [g.add_node("Mul", [a, b]).output], attrs={"axis": -1}).output, "general")
    u = g.add_node("Mul", [z, g.constant(np.float32(0.5))]).output
    g.add_output(g.add_node("Softmax", [u], attrs={"axis": 1}).output, "wide")
    infer_shapes(g)
    return g, {"x": f32(r, 3, 5, 32), "w": f32(r, 5, 1), "z": f32(r, 2, 256, scale=4)}


def _p_attention(r: np.random.Generator) -> tuple[Graph, dict[str, np.ndarray]]:
    """Attention scores: Q Kᵀ (Kᵀ read through its Transpose) scaled, an additive mask over keys,
    Softmax, then P V (the BERT form); and V Kᵀ divided, a causal Where, LogSoftmax (the GPT-2
    form), the softmax evaluating the scale-and-mask program as it reads the scores."""
    g = Graph("attention")
    q = g.add_input("q", TensorType("float32", (2, 3, 16, 8)))
    k = g.add_input("k", TensorType("float32", (2, 3, 16, 8)))
    v = g.add_input("v", TensorType("float32", (2, 3, 16, 8)))
    m = g.add_input("m", TensorType("float32", (2, 1, 1, 16)))
    kt = g.add_node("Transpose", [k], attrs={"perm": [0, 1, 3, 2]}).output
    s = g.add_node("MatMul", [q, kt]).output
    t = g.add_node("Mul", [s, g.constant(np.float32(0.35))]).output
    t = g.add_node("Add", [t, m]).output
    pr = g.add_node("Softmax", [t], attrs={"axis": -1}).output
    g.add_output(g.add_node("MatMul", [pr, v]).output, "o")
    kt2 = g.add_node("Transpose", [k], attrs={"perm": [0, 1, 3, 2]}).output
    s2 = g.add_node("MatMul", [v, kt2]).output
    u = g.add_node("Div", [s2, g.constant(np.float32(2.5))]).output
    causal = g.constant(np.tril(np.ones((16, 16), dtype=bool)).reshape(1, 1, 16, 16))
    u = g.add_node("Where", [causal, u, g.constant(np.float32(-1e9))]).output
    g.add_output(g.add_node("LogSoftmax", [u], attrs={"axis": -1}).output, "lp")
    infer_shapes(g)
    mask = np.where(r.random((2, 1, 1, 16)) > 0.25, 0.0, -10000.0).astype(np.float32)
    return g, {"q": f32(r, 2, 3, 16, 8), "k": f32(r, 2, 3, 16, 8), "v": f32(r, 2, 3, 16, 8), "m": mask}


def _p_conv_maxpool(r: np.random.Generator) -> tuple[Graph, dict[str, np.ndarray]]:
    """Conv + ReLU then max pooling in NHWC (the O3 layout): 3x3 stride 2 pad 1 (the ResNet stem
    pool) and 3x3 stride 1 pad 1, output widths 7 and 13 (ragged groups of four columns), eight
    channels (two groups of four), negative values kept by a second, unrectified branch."""
    g = Graph("conv_maxpool")
    x = g.add_input("x", TensorType("float32", (2, 8, 13, 13)))
    w = g.constant(f32(r, 8, 8, 3, 3, scale=0.3))
    h = g.add_node("Conv", [x, w], attrs={"kernel_shape": [3, 3], "pads": [1, 1, 1, 1]}).output
    a = g.add_node("Relu", [h]).output
    p1 = g.add_node("MaxPool", [a], attrs={"kernel_shape": [3, 3], "strides": [2, 2], "pads": [1, 1, 1, 1]}).output
    p2 = g.add_node("MaxPool", [h], attrs={"kernel_shape": [3, 3], "strides": [1, 1], "pads": [1, 1, 1, 1]}).output
    w2 = g.constant(f32(r, 4, 8, 1, 1, scale=0.3))
    g.add_output(g.add_node("Conv", [p1, w2], attrs={"kernel_shape": [1, 1]}).output, "a")
    g.add_output(g.add_node("Conv", [p2, w2], attrs={"kernel_shape": [1, 1]}).output, "b")
    infer_shapes(g)
    return g, {"x": f32(r, 2, 8, 13, 13)}


def pattern_cases() -> list[Case]:
    return [
        _pattern("conv_block", _p_conv_block),
        _pattern("narrow_convs", _p_narrow_convs),
        _pattern("narrow_window", narrow_window_chain),
        _pattern("dense_gelu", _p_dense_gelu),
        _pattern("layer_norm", _p_layer_norm),
        _pattern("loopfuse", _p_loopfuse),
        _pattern("masked_softmax", _p_masked_softmax),
        _pattern("softmax_programs", _p_softmax_programs),
        _pattern("attention", _p_attention),
        _pattern("conv_maxpool", _p_conv_maxpool),
    ]


# -- whole models ------------------------------------------------------------------------------------
def _model(name: str, fn: Callable[[], Graph], seed: int, opt: str, big: bool = False, **kw: Any) -> Case:
    def build() -> tuple[Graph, dict[str, np.ndarray]]:
        g = fn()
        return g, zoo.feeds(g, seed)
    return Case(f"model_{name}_{opt}", build, opt=opt, big=big, **kw)


def model_cases() -> list[Case]:
    out = []
    for opt in ("O0", "O3"):
        out.append(_model("mlp", lambda: zoo.mlp(), 0, opt))
        out.append(_model("tiny_cnn", lambda: zoo.tiny_cnn(batch=2), 0, opt))
        out.append(_model("tiny_gpt", lambda: zoo.tiny_transformer(kind="gpt", batch=2), 0, opt))
        out.append(_model("tiny_bert", lambda: zoo.tiny_transformer(kind="bert", batch=2), 0, opt))
    out.append(_model("tiny_cnn", lambda: zoo.tiny_cnn(batch=2), 0, "O2"))
    return out


def big_model_cases() -> list[Case]:
    """The benchmark configurations at their batch-1 sizes."""
    return [
        _model("resnet50_b1", lambda: zoo.resnet50(batch=1, seed=0), 0, "O3", big=True),
        _model("mobilenet_v2_b1", lambda: zoo.mobilenet_v2(batch=1, seed=1), 1, "O3", big=True),
        _model("bert_b1", lambda: zoo.bert(batch=1, seq=128, seed=2), 2, "O3", big=True),
        _model("gpt2_b1", lambda: zoo.gpt2(batch=1, seq=128, seed=3), 3, "O3", big=True),
    ]


def all_cases() -> list[Case]:
    return op_cases() + pattern_cases() + model_cases()


def prepare(case: Case) -> tuple[Graph, dict[str, np.ndarray]]:
    """Build the case graph and run the reference pipeline at the case's level."""
    from ml_graph_compiler.passes import optimize
    from ml_graph_compiler.schedule import schedule

    g, feeds = case.build()
    if case.opt != "O0":
        optimize(g, case.opt)
        schedule(g)
    return g, feeds
