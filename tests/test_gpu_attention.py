"""The fused attention kernel (MGC_K_ATTENTION, csrc/attention.cuh): softmax(program(Q K^T)) V in
TF32 mode, for every operand layout the lowering hands it (Q and the output with the head width
contiguous; K^T read with the head width or the keys contiguous; V with the head width or the
keys contiguous), every score program of the unfused softmax's ScaleMask form (X * s, X / s, then
+ M, - M, Where(C, t, lit), Where(C, lit, t)), ragged key counts, two query tiles and head widths
other than 64, and grids of more CTAs than fit at once; the forms the kernel compiles without runtime tests (X * s alone, + fp32 mask,
Where with a byte mask either way round) and its generic form (X / s, - M, ragged masks). Each
case is compared with a float64 emulation of the kernel's arithmetic: Q, K and
V rounded to TF32 on load (ties away from zero, what a TFLOAT32 tensor map does), the scores and
the softmax exact, P rounded to TF32 before P V; the remaining differences are fp32 accumulation
and the one-ulp TF32 rounding flips of P that they cause."""

from __future__ import annotations

import numpy as np
import pytest

from mgc_cuda.runtime import compile_graph
from ml_graph_compiler.ir import Graph, TensorType
from ml_graph_compiler.passes import optimize
from ml_graph_compiler.schedule import schedule
from ml_graph_compiler.shape_inference import infer_shapes

pytestmark = pytest.mark.gpu

FMIN = float(np.finfo(np.float32).min)


def tf32(a: np.ndarray) -> np.ndarray:
    from mgc_cuda.lowering import tf32_split

    return tf32_split(np.ascontiguousarray(a, dtype=np.float32))[0].astype(np.float64)


def build(b: int, h: int, sq: int, sk: int, dqk: int, dv: int, k_keys_contig: bool, v_keys_contig: bool, program: str,
          merge: bool, seed: int) -> tuple[Graph, dict[str, np.ndarray], dict[str, np.ndarray]]:
    """The attention chain as the reference IR writes it, with its inputs and (for the
    emulation) the program's operands. K comes as [b, h, sk, dqk] transposed to K^T (head width
    contiguous) or as K^T [b, h, dqk, sk] itself (keys contiguous); V as [b, h, sk, dv] (head width
    contiguous) or as [b, h, dv, sk] transposed (keys contiguous)."""
    rng = np.random.default_rng(seed)
    g = Graph("attention")
    feeds: dict[str, np.ndarray] = {}

    def inp(name: str, shape: tuple[int, ...]):
        feeds[name] = rng.standard_normal(shape).astype(np.float32)
        return g.add_input(name, TensorType("float32", shape))

    q = inp("q", (b, h, sq, dqk))
    if k_keys_contig:
        kt = inp("kt", (b, h, dqk, sk))
    else:
        kt = g.add_node("Transpose", [inp("k", (b, h, sk, dqk))], attrs={"perm": [0, 1, 3, 2]}).output
    if v_keys_contig:
        v = g.add_node("Transpose", [inp("vt", (b, h, dv, sk))], attrs={"perm": [0, 1, 3, 2]}).output
    else:
        v = inp("v", (b, h, sk, dv))
    s = g.add_node("MatMul", [q, kt]).output
    ops: dict[str, np.ndarray] = {}
    scale = np.float32(1.0 / np.sqrt(dqk))
    if program.startswith("div"):
        t = g.add_node("Div", [s, g.constant(np.float32(1.0 / scale), "d")]).output
    else:
        t = g.add_node("Mul", [s, g.constant(scale, "s")]).output
    if program.endswith("add") or program.endswith("sub"):
        feeds["mask"] = np.where(rng.random((b, 1, 1, sk)) < 0.2, FMIN, 0.0).astype(np.float32)
        feeds["mask"][..., 0] = 0.0  # every row keeps a key
        mask = g.add_input("mask", TensorType("float32", (b, 1, 1, sk)))
        if program.endswith("sub"):
            feeds["mask"] = -feeds["mask"]
        t = g.add_node("Add" if program.endswith("add") else "Sub", [t, mask]).output
        ops["mask"] = feeds["mask"]
    elif program.endswith("keep") or program.endswith("fill"):
        keep = np.tril(np.ones((sq, sk), dtype=bool), max(sk - sq, 0))[None, None]
        lit = g.constant(np.float32(FMIN), "mask_value")
        if program.endswith("keep"):
            t = g.add_node("Where", [g.constant(keep, "keep"), t, lit]).output
        else:
            t = g.add_node("Where", [g.constant(~keep, "upper"), lit, t]).output
        ops["keep"] = keep
    p = g.add_node("Softmax", [t], attrs={"axis": -1}).output
    o = g.add_node("MatMul", [p, v]).output
    if merge:
        o = g.add_node("Transpose", [o], attrs={"perm": [0, 2, 1, 3]}).output
        o = g.add_node("Reshape", [o, g.constant(np.asarray([b, sq, h * dv], np.int64), "shape")]).output
    g.add_output(o, "out")
    infer_shapes(g)
    return g, feeds, ops


def emulate(feeds: dict[str, np.ndarray], ops: dict[str, np.ndarray], program: str, dqk: int, merge: bool) -> np.ndarray:
    q = tf32(feeds["q"])
    kt = tf32(feeds["kt"]) if "kt" in feeds else np.swapaxes(tf32(feeds["k"]), -1, -2)
    v = np.swapaxes(tf32(feeds["vt"]), -1, -2) if "vt" in feeds else tf32(feeds["v"])
    s = (q @ kt).astype(np.float32)
    scale = np.float32(1.0 / np.sqrt(dqk))
    t = s / np.float32(1.0 / scale) if program.startswith("div") else s * scale
    if "mask" in ops:
        t = t + ops["mask"] if program.endswith("add") else t - ops["mask"]
    if "keep" in ops:
        t = np.where(ops["keep"], t, np.float32(FMIN))
    t = t.astype(np.float64)
    e = np.exp(t - t.max(-1, keepdims=True))
    pm = tf32((e / e.sum(-1, keepdims=True)).astype(np.float32))
    o = pm @ v
    if merge:
        o = np.swapaxes(o, 1, 2).reshape(o.shape[0], o.shape[2], -1)
    return o


CASES = [
    # b, h, sq, sk, dqk, dv, K keys contiguous, V keys contiguous, program, head merge
    (2, 12, 128, 128, 64, 64, False, False, "mul_add", True),     # BERT's layer
    (2, 12, 128, 128, 64, 64, False, False, "mul_fill", True),    # GPT-2's layer
    (3, 2, 200, 77, 64, 32, False, False, "div_keep", False),     # two query tiles, ragged keys
    (1, 3, 64, 256, 32, 64, True, True, "mul_sub", False),       # K^T and V with keys contiguous
    (2, 4, 8, 8, 8, 8, False, True, "mul", True),                 # tiny heads, no mask
    (1, 2, 130, 36, 96, 64, True, False, "div_add", True),
    (2, 3, 96, 64, 64, 64, False, False, "mul_keep", True),
    # more (batch, head) items than the CTAs the GPU holds at once (two waves and a tail)
    (26, 12, 128, 128, 64, 64, False, False, "mul_add", True),
    (4, 80, 64, 96, 32, 32, True, True, "div_keep", False),
]


@pytest.mark.parametrize("case", CASES, ids=[f"{c[2]}x{c[3]}_d{c[4]}-{c[5]}_{c[8]}_k{int(c[6])}v{int(c[7])}" for c in CASES])
def test_fused_attention_matches_tf32_emulation(case: tuple) -> None:
    b, h, sq, sk, dqk, dv, kc, vc, program, merge = case
    g, feeds, ops = build(b, h, sq, sk, dqk, dv, kc, vc, program, merge, seed=sq * 7 + sk)
    want = emulate(feeds, ops, program, dqk, merge)
    optimize(g, "O3")
    schedule(g)
    m = compile_graph(g, precision="tf32")
    try:
        assert m.lowered.kernels.get("attention") == 1, m.lowered.kernels
        paths = m.gemm_paths()
        assert [p for _, _, _, p in paths] == ["tcgen05"], paths
        got = m.run(feeds)["out"].astype(np.float64)
        again = m.run(feeds)["out"]
    finally:
        m.close()
    np.testing.assert_array_equal(again, got.astype(np.float32))
    scale = float(np.abs(want).max())
    err = float(np.abs(got - want).max())
    # fp32 accumulation (about 1e-6 of the scale) and one-ulp flips of P's TF32 rounding (2^-11
    # of one weight times a value of V)
    assert err <= 2e-3 * scale, f"max abs err {err:.3g} (scale {scale:.3g})"
    assert float(np.abs(got - want).mean()) <= 2e-5 * scale


def test_fused_attention_close_to_float64() -> None:
    """BERT's layer against the exact float64 attention: the TF32 budget of the product chain."""
    g, feeds, _ = build(2, 12, 128, 128, 64, 64, False, False, "mul_add", True, seed=5)
    optimize(g, "O3")
    schedule(g)
    q, k, v = (feeds[n].astype(np.float64) for n in ("q", "k", "v"))
    t = q @ np.swapaxes(k, -1, -2) / 8.0 + feeds["mask"]
    e = np.exp(t - t.max(-1, keepdims=True))
    want = np.swapaxes((e / e.sum(-1, keepdims=True)) @ v, 1, 2).reshape(2, 128, -1)
    m = compile_graph(g, precision="tf32")
    try:
        got = m.run(feeds)["out"].astype(np.float64)
    finally:
        m.close()
    assert float(np.abs(got - want).max()) <= 1e-2 * float(np.abs(want).max())
