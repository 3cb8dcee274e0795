"""Run a reference IR graph node by node with the oracle semantics.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``). The walk mirrors the reference
interpreter's contract (``interpreter.py:71-93``: inputs validated, nodes in graph order, named
outputs returned) but evaluates every node with ``oracle.semantics``.
"""

from __future__ import annotations

from collections.abc import Mapping
from typing import Any

import numpy as np

from oracle import semantics as S

VIEW_OPS = {"Reshape", "Flatten", "Squeeze", "Unsqueeze", "Identity", "Dropout"}
ELEMENTWISE = set(S.UNARY) | {
    "Add", "Sub", "Mul", "Div", "Pow", "Max", "Min", *S.COMPARE, *S.LOGICAL, "Not", "Where",
    "Gelu", "LeakyRelu", "HardSigmoid", "Clip", "Cast",
}


def _axes(node: Any, xs: list[np.ndarray | None], index: int) -> list[int] | None:
    if "axes" in node.attrs:
        return [int(a) for a in node.attrs["axes"]]
    if len(xs) > index and xs[index] is not None:
        return S._ints(xs[index])
    return None


def run_node(node: Any, xs: list[np.ndarray | None]) -> list[np.ndarray]:
    """Evaluate one node; returns its outputs in order."""
    op, at = node.op, node.attrs
    outs = [o.tensor_type for o in node.outputs]
    x = xs[0] if xs else None
    if op in VIEW_OPS:
        assert x is not None
        res = [np.asarray(x, order="C").reshape(outs[0].shape).copy()]
        if op == "Dropout" and len(node.outputs) > 1:
            res.append(np.ones(outs[1].shape, np.bool_))
        return res
    if op == "FusedElementwise":
        return [S.fused_elementwise(at["program"], xs)]
    if op in ELEMENTWISE:
        return [S.elementwise(op, dict(at), xs)]
    assert x is not None
    if op == "Transpose":
        perm = at.get("perm")
        perm = list(range(x.ndim))[::-1] if perm is None else [int(p) for p in perm]
        return [np.asarray(x.transpose(perm), order="C")]
    if op == "Expand":
        return [np.asarray(np.broadcast_to(x, outs[0].shape), order="C")]
    if op == "Tile":
        assert xs[1] is not None
        return [np.tile(x, S._ints(xs[1]))]
    if op == "Slice":
        if "starts" in at:
            return [S.slice_(x, at["starts"], at["ends"], at.get("axes"), None)]
        get = lambda i: S._ints(xs[i]) if len(xs) > i and xs[i] is not None else None  # noqa: E731
        return [S.slice_(x, get(1), get(2), get(3), get(4))]
    if op == "Concat":
        arrays = [a for a in xs if a is not None]
        return [np.concatenate(arrays, axis=int(at.get("axis", 0)))]
    if op == "Split":
        axis = S._norm_axis(int(at.get("axis", 0)), x.ndim)
        sizes = [t.shape[axis] for t in outs]
        bounds = np.cumsum(sizes)[:-1]
        return [np.asarray(p, order="C") for p in np.split(x, bounds, axis=axis)]
    if op == "Pad":
        if at.get("mode", "constant") != "constant":
            raise S.OracleError("Pad mode")
        pads = [int(p) for p in at["pads"]] if "pads" in at else S._ints(xs[1])
        if len(xs) > 3 and xs[3] is not None:
            full = [0] * (2 * x.ndim)
            ax = [S._norm_axis(a, x.ndim) for a in S._ints(xs[3])]
            for i, a in enumerate(ax):
                full[a], full[a + x.ndim] = pads[i], pads[i + len(ax)]
            pads = full
        value = float(np.asarray(xs[2]).reshape(())) if len(xs) > 2 and xs[2] is not None else 0.0
        return [S.pad(x, pads, value)]
    if op == "Gather":
        assert xs[1] is not None
        return [S.gather(x, xs[1], S._norm_axis(int(at.get("axis", 0)), x.ndim))]
    if op == "Shape":
        start = int(at.get("start", 0))
        end = at.get("end")
        dims = x.shape[start:] if end is None else x.shape[start : int(end)]
        return [np.asarray(dims, np.int64)]
    if op == "Size":
        return [np.asarray(x.size, np.int64)]
    if op == "ConstantOfShape":
        value = at.get("value")
        fill = np.asarray(value).reshape(-1)[0] if value is not None else np.float32(0)
        return [np.full(outs[0].shape, fill, dtype=np.dtype(outs[0].dtype))]
    if op == "Range":
        assert xs[2] is not None
        start = np.asarray(x).reshape(())
        delta = np.asarray(xs[2]).reshape(())
        n = outs[0].shape[0]
        return [np.asarray(start + np.arange(n, dtype=start.dtype) * delta, dtype=np.dtype(outs[0].dtype))]
    if op in ("ReduceMean", "ReduceSum", "ReduceMax", "ReduceMin", "ReduceProd"):
        axes = _axes(node, xs, 1)
        if not axes:
            axes_t = () if int(at.get("noop_with_empty_axes", 0)) else tuple(range(x.ndim))
        else:
            axes_t = tuple(sorted(S._norm_axis(a, x.ndim) for a in axes))
        kind = op[len("Reduce"):].lower()
        return [S.reduce(x, kind, axes_t, bool(int(at.get("keepdims", 1))))]
    if op == "ArgMax":
        return [S.argmax(x, S._norm_axis(int(at.get("axis", 0)), x.ndim), bool(int(at.get("keepdims", 1))))]
    if op in ("Softmax", "LogSoftmax"):
        return [S.softmax(x, S._norm_axis(int(at.get("axis", -1)), x.ndim), op == "LogSoftmax")]
    if op == "LayerNormalization":
        scale = xs[1] if len(xs) > 1 else None
        bias = xs[2] if len(xs) > 2 else None
        axis = S._norm_axis(int(at.get("axis", -1)), x.ndim)
        return [S.layer_norm(x, scale, bias, axis, float(at.get("epsilon", 1e-5)))]
    if op == "BatchNormalization":
        p = [xs[i] for i in range(1, 5)]
        assert all(v is not None for v in p)
        return [S.batch_norm(x, p[0], p[1], p[2], p[3], float(at.get("epsilon", 1e-5)),  # type: ignore[arg-type]
                             at.get("layout") == "NHWC")]
    if op == "MatMul":
        assert xs[1] is not None
        return [S.matmul(x, xs[1])]
    if op == "Gemm":
        assert xs[1] is not None
        return [S.gemm(x, xs[1], xs[2] if len(xs) > 2 else None, dict(at))]
    if op == "FusedGemm":
        assert xs[1] is not None
        return [S.fused_gemm(x, xs[1], xs[2] if len(xs) > 2 else None, xs[3] if len(xs) > 3 else None, dict(at))]
    if op in ("Conv", "FusedConv"):
        assert xs[1] is not None
        attrs = dict(at) if op == "FusedConv" else {**at, "activation": "none"}
        return [S.conv(x, xs[1], xs[2] if len(xs) > 2 else None, xs[3] if len(xs) > 3 else None, attrs)]
    if op in ("MaxPool", "AveragePool"):
        return [S.pool(x, dict(at), "max" if op == "MaxPool" else "avg")]
    if op in ("GlobalAveragePool", "GlobalMaxPool"):
        return [S.global_pool(x, dict(at), "avg" if op == "GlobalAveragePool" else "max")]
    raise S.OracleError(f"the oracle has no semantics for {op}")


def run(graph: Any, feeds: Mapping[str, np.ndarray]) -> dict[str, np.ndarray]:
    """Evaluate ``graph`` on ``feeds``; returns {output name: array}."""
    env: dict[int, np.ndarray] = {}
    for v in graph.inputs:
        if v.name not in feeds:
            raise S.OracleError(f"missing input {v.name!r}")
        a = np.asarray(feeds[v.name], order="C")
        if tuple(a.shape) != tuple(v.tensor_type.shape):
            raise S.OracleError(f"input {v.name!r}: shape {a.shape} != {v.tensor_type.shape}")
        env[id(v)] = a

    def get(v: Any) -> np.ndarray | None:
        if v is None:
            return None
        if v.data is not None:
            return np.asarray(v.data)
        return env[id(v)]

    for node in graph.nodes:
        results = run_node(node, [get(v) for v in node.inputs])
        for value, arr in zip(node.outputs, results, strict=False):
            if value.type is not None and tuple(arr.shape) != tuple(value.tensor_type.shape):
                raise S.OracleError(f"{node.op} {node.name!r}: shape {arr.shape} != {value.tensor_type.shape}")
            env[id(value)] = arr
    return {name: get(v) for name, v in graph.named_outputs()}  # type: ignore[misc]
