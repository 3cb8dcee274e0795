"""numpy restatement of the reference operator semantics on the cuda target's path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``). Every function cites the reference
definition it restates (paths relative to ``src/ml_graph_compiler/``). The code is independent of
the reference's implementation: window geometry, slicing, padding and broadcasting are derived
here from the ONNX attributes, and floating point arithmetic runs in float64 before rounding to
the output dtype.
"""

from __future__ import annotations

import math
from collections.abc import Callable, Sequence
from typing import Any

import numpy as np
from scipy import special

Array = np.ndarray


class OracleError(Exception):
    """The oracle cannot evaluate a node (unsupported attribute or an out-of-range index)."""


def _f64(x: Array) -> Array:
    return np.asarray(x, dtype=np.float64)


def _as(y: Any, like: Array) -> Array:
    """Round to the dtype of ``like`` (the reference keeps the first operand's dtype, ops.py:125)."""
    return np.asarray(np.asarray(y).astype(like.dtype, copy=False), order="C")


def _ints(v: Any) -> list[int]:
    return [int(x) for x in np.asarray(v).reshape(-1)]


def _norm_axis(axis: int, rank: int) -> int:
    a = axis + rank if axis < 0 else axis
    if not 0 <= a < max(rank, 1):
        raise OracleError(f"axis {axis} out of range for rank {rank}")
    return a


# ---------------------------------------------------------------------------------------------
# elementwise (ops.py:132-341)
# ---------------------------------------------------------------------------------------------
def gelu(x: Array, approximate: str = "none") -> Array:
    """GELU: erf form, or the tanh approximation (ops.py:233-237)."""
    v = _f64(x)
    if approximate == "tanh":
        y = 0.5 * v * (1.0 + np.tanh(math.sqrt(2.0 / math.pi) * (v + 0.044715 * v**3)))
    else:
        y = 0.5 * v * (1.0 + special.erf(v / math.sqrt(2.0)))
    return _as(y, x)


def _float_unary(fn: Callable[[Array], Array]) -> Callable[[Array], Array]:
    def run(x: Array) -> Array:
        if np.issubdtype(x.dtype, np.floating):
            with np.errstate(all="ignore"):
                return _as(fn(_f64(x)), x)
        with np.errstate(all="ignore"):
            return _as(fn(_f64(x)), x)

    return run


UNARY: dict[str, Callable[[Array], Array]] = {
    "Relu": lambda x: _as(np.maximum(x, 0), x),
    "Sigmoid": _float_unary(lambda v: 1.0 / (1.0 + np.exp(-v))),
    "Tanh": _float_unary(np.tanh),
    "Erf": _float_unary(special.erf),
    "Sqrt": _float_unary(np.sqrt),
    "Exp": _float_unary(np.exp),
    "Log": _float_unary(np.log),
    "Neg": lambda x: _as(np.negative(x), x),
    "Abs": lambda x: _as(np.abs(x), x),
    "Reciprocal": _float_unary(lambda v: 1.0 / v),
    "Floor": _float_unary(np.floor),
    "Ceil": _float_unary(np.ceil),
    "Sin": _float_unary(np.sin),
    "Cos": _float_unary(np.cos),
    "Softplus": _float_unary(lambda v: np.logaddexp(0.0, v)),
    "Identity": lambda x: x.copy(),
}


def _binary_arith(op: str, a: Array, b: Array) -> Array:
    """Add/Sub/Mul/Div/Pow/Max/Min with the result in a's dtype (ops.py:136-167)."""
    if np.issubdtype(a.dtype, np.integer) or a.dtype == np.bool_:
        ai, bi = a.astype(np.int64), b.astype(np.int64)
        if op == "Div":
            with np.errstate(all="ignore"):
                return _as(np.trunc(ai / np.where(bi == 0, 1, bi)), a)
        fn = {"Add": np.add, "Sub": np.subtract, "Mul": np.multiply, "Max": np.maximum,
              "Min": np.minimum, "Pow": np.power}[op]
        return _as(fn(ai, bi), a)
    av, bv = _f64(a), _f64(b)
    with np.errstate(all="ignore"):
        y = {"Add": np.add, "Sub": np.subtract, "Mul": np.multiply, "Div": np.divide,
             "Pow": np.power, "Max": np.maximum, "Min": np.minimum}[op](av, bv)
    return _as(y, a)


COMPARE = {
    "Equal": np.equal, "Less": np.less, "Greater": np.greater, "LessOrEqual": np.less_equal,
    "GreaterOrEqual": np.greater_equal,
}
LOGICAL = {"And": np.logical_and, "Or": np.logical_or, "Xor": np.logical_xor}

CAST_CODES = {1: "float32", 6: "int32", 7: "int64", 9: "bool", 11: "float64", 2: "uint8", 3: "int8"}


def elementwise(op: str, attrs: dict[str, Any], xs: Sequence[Array | None]) -> Array:
    """One elementwise operator (ops.py:132-341)."""
    x = xs[0]
    assert x is not None
    if op in UNARY:
        return UNARY[op](x)
    if op in ("Add", "Sub", "Mul", "Div", "Pow", "Max", "Min"):
        assert xs[1] is not None
        return _binary_arith(op, x, xs[1])
    if op in COMPARE:
        assert xs[1] is not None
        return np.asarray(COMPARE[op](x, xs[1]), dtype=np.bool_)
    if op in LOGICAL:
        assert xs[1] is not None
        return np.asarray(LOGICAL[op](x, xs[1]), dtype=np.bool_)
    if op == "Not":
        return np.logical_not(x)
    if op == "Where":
        assert xs[1] is not None and xs[2] is not None
        return _as(np.where(x, xs[1], xs[2]), xs[1])
    if op == "Gelu":
        return gelu(x, str(attrs.get("approximate", "none")))
    if op == "LeakyRelu":
        alpha = float(attrs.get("alpha", 0.01))
        return _as(np.where(_f64(x) >= 0, _f64(x), alpha * _f64(x)), x)
    if op == "HardSigmoid":
        a, b = float(attrs.get("alpha", 0.2)), float(attrs.get("beta", 0.5))
        return _as(np.clip(a * _f64(x) + b, 0.0, 1.0), x)
    if op == "Clip":
        lo = attrs.get("min", -np.inf)
        hi = attrs.get("max", np.inf)
        if len(xs) > 1 and xs[1] is not None:
            lo = np.asarray(xs[1]).reshape(()).item()
        if len(xs) > 2 and xs[2] is not None:
            hi = np.asarray(xs[2]).reshape(()).item()
        return _as(np.minimum(np.maximum(x, lo), hi), x)
    if op == "Cast":
        to = attrs.get("to", 1)
        dtype = to if isinstance(to, str) else CAST_CODES[int(to)]
        return np.asarray(x.astype(dtype), order="C")
    raise OracleError(f"elementwise {op} is not in the oracle")


def fused_elementwise(program: Sequence[Any], xs: Sequence[Array | None]) -> Array:
    """Replay a FusedElementwise program: argument a < len(inputs) is input a, otherwise the
    result of instruction a - len(inputs); -1 is an omitted input (ops.py:1165-1202)."""
    regs: list[Array | None] = list(xs)
    for op, attrs, args in program:
        regs.append(elementwise(str(op), dict(attrs), [regs[int(a)] if int(a) >= 0 else None for a in args]))
    out = regs[-1]
    assert out is not None
    return out


def batch_norm(x: Array, scale: Array, bias: Array, mean: Array, var: Array, eps: float, nhwc: bool) -> Array:
    """(x - mean) * scale / sqrt(var + eps) + bias per channel (ops.py:832-840)."""
    shape = [1] * x.ndim
    shape[x.ndim - 1 if nhwc else 1] = -1
    inv = _f64(scale) / np.sqrt(_f64(var) + eps)
    y = (_f64(x) - _f64(mean).reshape(shape)) * inv.reshape(shape) + _f64(bias).reshape(shape)
    return _as(y, x)


# ---------------------------------------------------------------------------------------------
# activations of fused epilogues (ops.py:894-911)
# ---------------------------------------------------------------------------------------------
def activation(y: Array, attrs: dict[str, Any]) -> Array:
    act = str(attrs.get("activation", "none"))
    if act == "none":
        return y
    if act == "relu":
        return np.maximum(y, 0.0)
    if act == "clip":
        return np.clip(y, float(attrs.get("clip_min", 0.0)), float(attrs.get("clip_max", 6.0)))
    if act == "gelu":
        return 0.5 * y * (1.0 + special.erf(y / math.sqrt(2.0)))
    if act == "gelu_tanh":
        return 0.5 * y * (1.0 + np.tanh(math.sqrt(2.0 / math.pi) * (y + 0.044715 * y**3)))
    if act == "tanh":
        return np.tanh(y)
    if act == "sigmoid":
        return 1.0 / (1.0 + np.exp(-y))
    raise OracleError(f"activation {act!r}")


# ---------------------------------------------------------------------------------------------
# windows: convolution and pooling (ops.py:940-1159)
# ---------------------------------------------------------------------------------------------
def window(attrs: dict[str, Any], in_hw: tuple[int, int], kernel: tuple[int, int], ceil_mode: bool = False
           ) -> tuple[tuple[int, int], tuple[int, int], tuple[int, int, int, int], tuple[int, int]]:
    """(strides, dilations, pads top/left/bottom/right, output hw) for a 2-D window, following the
    ONNX rules for explicit pads and auto_pad SAME_UPPER / SAME_LOWER / VALID (ops.py:951-987)."""
    sh, sw = (int(s) for s in attrs.get("strides", (1, 1)))
    dh, dw = (int(d) for d in attrs.get("dilations", (1, 1)))
    pads = [int(p) for p in attrs.get("pads", (0, 0, 0, 0))]
    stride, dil = (sh, sw), (dh, dw)
    span = [(kernel[i] - 1) * dil[i] + 1 for i in range(2)]
    auto = attrs.get("auto_pad", "NOTSET")
    if auto in ("SAME_UPPER", "SAME_LOWER"):
        out = [(in_hw[i] + stride[i] - 1) // stride[i] for i in range(2)]
        total = [max((out[i] - 1) * stride[i] + span[i] - in_hw[i], 0) for i in range(2)]
        first = [t // 2 if auto == "SAME_UPPER" else t - t // 2 for t in total]
        pads = [first[0], first[1], total[0] - first[0], total[1] - first[1]]
    elif auto == "VALID":
        pads = [0, 0, 0, 0]
    out_hw = []
    for i in range(2):
        room = in_hw[i] + pads[i] + pads[i + 2] - span[i]
        if room < 0:
            raise OracleError("window larger than the padded input")
        o = (room + stride[i] - 1) // stride[i] + 1 if ceil_mode else room // stride[i] + 1
        if ceil_mode and (o - 1) * stride[i] >= in_hw[i] + pads[i]:
            o -= 1  # the last window must start inside the input or its leading pad
        out_hw.append(o)
    return stride, dil, (pads[0], pads[1], pads[2], pads[3]), (out_hw[0], out_hw[1])


def _patches(xp: Array, kernel: tuple[int, int], stride: tuple[int, int], dil: tuple[int, int],
             out_hw: tuple[int, int]) -> Array:
    """View [N, C, OH, OW, KH, KW] of a padded NCHW array."""
    n, c, _, _ = xp.shape
    s = xp.strides
    return np.lib.stride_tricks.as_strided(
        xp,
        shape=(n, c, out_hw[0], out_hw[1], kernel[0], kernel[1]),
        strides=(s[0], s[1], s[2] * stride[0], s[3] * stride[1], s[2] * dil[0], s[3] * dil[1]),
        writeable=False,
    )


def conv(x: Array, w: Array, b: Array | None, res: Array | None, attrs: dict[str, Any]) -> Array:
    """act(conv(x, w) + b + res), grouped, NCHW with OIHW weights or NHWC with HWIO weights
    (ops.py:997-1069). Computed in float64."""
    nhwc = attrs.get("layout", "NCHW") == "NHWC"
    group = int(attrs.get("group", 1))
    xn = _f64(x.transpose(0, 3, 1, 2) if nhwc else x)
    wn = _f64(w.transpose(3, 2, 0, 1) if nhwc else w)  # -> [K, C/g, KH, KW]
    n, c, h, wd = xn.shape
    k, cg, kh, kw = wn.shape
    if cg * group != c or k % group:
        raise OracleError("conv channels do not match the weights and group")
    stride, dil, pads, out_hw = window(attrs, (h, wd), (kh, kw))
    xp = np.pad(xn, ((0, 0), (0, 0), (pads[0], pads[2]), (pads[1], pads[3])))
    patches = _patches(np.asarray(xp, order="C"), (kh, kw), stride, dil, out_hw)
    kg = k // group
    outs = []
    for gi in range(group):
        pg = patches[:, gi * cg : (gi + 1) * cg]           # [N, cg, OH, OW, KH, KW]
        cols = pg.transpose(0, 2, 3, 1, 4, 5).reshape(n * out_hw[0] * out_hw[1], cg * kh * kw)
        wg = wn[gi * kg : (gi + 1) * kg].reshape(kg, cg * kh * kw)
        outs.append((cols @ wg.T).reshape(n, out_hw[0], out_hw[1], kg))
    y = np.concatenate(outs, axis=3)  # NHWC float64
    if b is not None:
        y = y + _f64(b).reshape(1, 1, 1, -1)
    if not nhwc:
        y = y.transpose(0, 3, 1, 2)
    if res is not None:
        y = y + _f64(res)
    return _as(activation(y, attrs), x)


def pool(x: Array, attrs: dict[str, Any], kind: str) -> Array:
    """Max / average pooling with pads, ceil_mode and count_include_pad (ops.py:1072-1134)."""
    nhwc = attrs.get("layout", "NCHW") == "NHWC"
    xn = _f64(x.transpose(0, 3, 1, 2) if nhwc else x)
    kernel = tuple(int(k) for k in attrs["kernel_shape"])
    stride, dil, pads, out_hw = window(attrs, (xn.shape[2], xn.shape[3]), (kernel[0], kernel[1]),
                                       bool(attrs.get("ceil_mode", 0)))
    h, wd = xn.shape[2], xn.shape[3]
    # extra room at the bottom/right for ceil-mode windows that run past the explicit pads
    need_h = (out_hw[0] - 1) * stride[0] + (kernel[0] - 1) * dil[0] + 1
    need_w = (out_hw[1] - 1) * stride[1] + (kernel[1] - 1) * dil[1] + 1
    eb = max(need_h - (h + pads[0] + pads[2]), 0)
    er = max(need_w - (wd + pads[1] + pads[3]), 0)
    widths = ((0, 0), (0, 0), (pads[0], pads[2] + eb), (pads[1], pads[3] + er))
    if kind == "max":
        xp = np.pad(xn, widths, constant_values=-np.inf)
        y = _patches(np.asarray(xp, order="C"), kernel, stride, dil, out_hw).max(axis=(4, 5))
    else:
        xp = np.pad(xn, widths)
        total = _patches(np.asarray(xp, order="C"), kernel, stride, dil, out_hw).sum(axis=(4, 5))
        ones = np.zeros((1, 1, h + pads[0] + pads[2] + eb, wd + pads[1] + pads[3] + er))
        if int(attrs.get("count_include_pad", 0)):
            ones[:, :, : h + pads[0] + pads[2], : wd + pads[1] + pads[3]] = 1.0
        else:
            ones[:, :, pads[0] : pads[0] + h, pads[1] : pads[1] + wd] = 1.0
        cnt = _patches(ones, kernel, stride, dil, out_hw).sum(axis=(4, 5))
        y = total / cnt
    y = y.transpose(0, 2, 3, 1) if nhwc else y
    return _as(y, x)


def global_pool(x: Array, attrs: dict[str, Any], kind: str) -> Array:
    """GlobalAveragePool / GlobalMaxPool over the spatial axes (ops.py:1137-1159)."""
    nhwc = attrs.get("layout", "NCHW") == "NHWC"
    axes = tuple(range(1, x.ndim - 1)) if nhwc else tuple(range(2, x.ndim))
    v = _f64(x)
    y = v.mean(axis=axes, keepdims=True) if kind == "avg" else v.max(axis=axes, keepdims=True)
    return _as(y, x)


# ---------------------------------------------------------------------------------------------
# matrix products (ops.py:846-934)
# ---------------------------------------------------------------------------------------------
def matmul(a: Array, b: Array) -> Array:
    """numpy matmul semantics with rank-1 promotion and batch broadcasting (ops.py:846-868)."""
    return _as(np.matmul(_f64(a), _f64(b)), a)


def gemm(a: Array, b: Array, c: Array | None, attrs: dict[str, Any]) -> Array:
    """alpha * op(A) @ op(B) + beta * C (ops.py:871-891)."""
    av = _f64(a).T if int(attrs.get("transA", 0)) else _f64(a)
    bv = _f64(b).T if int(attrs.get("transB", 0)) else _f64(b)
    y = float(attrs.get("alpha", 1.0)) * (av @ bv)
    if c is not None:
        y = y + float(attrs.get("beta", 1.0)) * _f64(c)
    return _as(y, a)


def fused_gemm(a: Array, b: Array, bias: Array | None, res: Array | None, attrs: dict[str, Any]) -> Array:
    """act(A @ B + bias + residual), A of any rank, B 2-D, optionally transposed (ops.py:914-934)."""
    bv = _f64(b).T if int(attrs.get("trans_b", 0)) else _f64(b)
    y = _f64(a) @ bv
    if bias is not None:
        y = y + _f64(bias)
    if res is not None:
        y = y + _f64(res)
    return _as(activation(y, attrs), a)


# ---------------------------------------------------------------------------------------------
# normalisation and reductions (ops.py:726-829)
# ---------------------------------------------------------------------------------------------
def softmax(x: Array, axis: int, log: bool = False) -> Array:
    """Softmax / LogSoftmax with max subtraction (ops.py:784-801)."""
    v = _f64(x)
    m = v.max(axis=axis, keepdims=True)
    e = np.exp(v - m)
    s = e.sum(axis=axis, keepdims=True)
    return _as(v - m - np.log(s) if log else e / s, x)


def layer_norm(x: Array, scale: Array | None, bias: Array | None, axis: int, eps: float) -> Array:
    """(x - mean) / sqrt(var + eps) * scale + bias over axes [axis, rank) (ops.py:804-829)."""
    v = _f64(x)
    axes = tuple(range(axis, x.ndim))
    mu = v.mean(axis=axes, keepdims=True)
    var = np.square(v - mu).mean(axis=axes, keepdims=True)
    y = (v - mu) / np.sqrt(var + eps)
    if scale is not None:
        y = y * _f64(scale)
    if bias is not None:
        y = y + _f64(bias)
    return _as(y, x)


def reduce(x: Array, kind: str, axes: tuple[int, ...], keepdims: bool) -> Array:
    """ReduceMean / Sum / Max / Min / Prod (ops.py:726-763)."""
    if not axes:
        return x.copy()
    if np.issubdtype(x.dtype, np.floating):
        v = _f64(x)
    else:
        v = x.astype(np.int64)
    fn = {"mean": np.mean, "sum": np.sum, "max": np.max, "min": np.min, "prod": np.prod}[kind]
    y = fn(v, axis=axes, keepdims=keepdims)
    if kind == "mean" and not np.issubdtype(x.dtype, np.floating):
        y = np.trunc(y)
    return _as(y, x)


def argmax(x: Array, axis: int, keepdims: bool) -> Array:
    """First index of the maximum along ``axis`` (ops.py:766-781)."""
    y = np.argmax(x, axis=axis)
    if keepdims:
        y = np.expand_dims(y, axis)
    return np.asarray(y.astype(np.int64), order="C")


# ---------------------------------------------------------------------------------------------
# data movement (ops.py:362-720)
# ---------------------------------------------------------------------------------------------
def gather(x: Array, idx: Array, axis: int) -> Array:
    """np.take with negative indices wrapped; an out-of-range index is an error (ops.py:590-603)."""
    dim = x.shape[axis]
    k = np.where(idx < 0, idx + dim, idx)
    if k.size and (int(k.min()) < 0 or int(k.max()) >= dim):
        raise OracleError(f"Gather index out of range for axis {axis} of size {dim}")
    return np.asarray(np.take(x, k, axis=axis), order="C")


def slice_(x: Array, starts: Sequence[int], ends: Sequence[int], axes: Sequence[int] | None,
           steps: Sequence[int] | None) -> Array:
    """ONNX Slice: clamp starts/ends per axis, any non-zero step (ops.py:545-587)."""
    rank = x.ndim
    axes = list(range(len(starts))) if axes is None else [_norm_axis(int(a), rank) for a in axes]
    steps = [1] * len(starts) if steps is None else [int(s) for s in steps]
    index: list[slice] = [slice(None)] * rank
    for s, e, a, st in zip(starts, ends, axes, steps, strict=True):
        if st == 0:
            raise OracleError("Slice step 0")
        dim = x.shape[a]
        s, e = int(s), int(e)
        if s < 0:
            s += dim
        if e < 0:
            e += dim
        if st > 0:
            s, e = min(max(s, 0), dim), min(max(e, 0), dim)
            index[a] = slice(s, e, st)
        else:
            s, e = min(max(s, -1), dim - 1), min(max(e, -1), dim - 1)
            index[a] = slice(s, e if e >= 0 else None, st)
    return np.asarray(x[tuple(index)], order="C")


def pad(x: Array, pads: Sequence[int], value: float) -> Array:
    """Constant Pad with per-axis (begin..., end...) amounts (ops.py:689-720)."""
    r = x.ndim
    return np.pad(x, [(int(pads[i]), int(pads[i + r])) for i in range(r)], constant_values=value)
