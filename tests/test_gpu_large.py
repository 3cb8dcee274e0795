"""Convolution layers at sizes where the tensor-core kernel keeps each CTA's whole B panel in
shared memory (every CTA walks at least two M tiles: M >= 2 * 148 * 128 rows for one N tile)
and the narrow-channel window-row path runs at full width, against the float64 oracle.

The small parity cases never reach these kernel variants; the benchmark models only do at
large batch. Budgets as in the other GPU tests: 1e-4 (strict) / 2e-2 (tf32) relative to the
largest |output|."""

from __future__ import annotations

import math

import numpy as np
import pytest

import cases
from mgc_cuda.lowering import tf32_split
from mgc_cuda.runtime import compile_graph
from ml_graph_compiler.ir import Graph, TensorType
from ml_graph_compiler.passes import optimize
from ml_graph_compiler.schedule import schedule
from ml_graph_compiler.shape_inference import infer_shapes
from oracle import runner

pytestmark = pytest.mark.gpu

TOL = {"strict": 1e-4, "tf32": 2e-2}


def _bottleneck(batch: int) -> tuple[Graph, dict[str, np.ndarray]]:
    """A ResNet-50 layer1 bottleneck (1x1 64->64, 3x3 64->64, 1x1 64->256 + projection
    residual, ReLU) at 56x56: 1x1 K = 64 panels fit in shared memory for N tiles of 64 and 128."""
    r = np.random.default_rng(11)
    g = Graph("bottleneck")
    x = g.add_input("x", TensorType("float32", (batch, 64, 56, 56)))

    def conv(v, cin, cout, k):  # noqa: ANN001, ANN202
        w = g.constant((r.standard_normal((cout, cin, k, k)) * (1.4 / math.sqrt(cin * k * k))).astype(np.float32))
        b = g.constant((r.standard_normal(cout) * 0.1).astype(np.float32))
        return g.add_node("Conv", [v, w, b], attrs={"kernel_shape": [k, k], "pads": [k // 2] * 4}).output

    h = g.add_node("Relu", [conv(x, 64, 64, 1)]).output
    h = g.add_node("Relu", [conv(h, 64, 64, 3)]).output
    h = conv(h, 64, 256, 1)
    y = g.add_node("Relu", [g.add_node("Add", [h, conv(x, 64, 256, 1)]).output]).output
    g.add_output(y, "y")
    infer_shapes(g)
    optimize(g, "O3")
    schedule(g)
    return g, {"x": r.standard_normal((batch, 64, 56, 56)).astype(np.float32)}


def _window_chain() -> tuple[Graph, dict[str, np.ndarray]]:
    g, feeds = cases.narrow_window_chain(np.random.default_rng(5), batch=16, h=96, w=128)
    optimize(g, "O3")
    schedule(g)
    return g, feeds


@pytest.fixture(scope="module")
def graphs() -> dict:
    out = {}
    for name, make in (("bottleneck_b16", lambda: _bottleneck(16)), ("narrow_window_b16", _window_chain)):
        g, feeds = make()
        out[name] = (g, feeds, runner.run(g, feeds))
    return out


@pytest.mark.parametrize("precision", ["strict", "tf32"])
@pytest.mark.parametrize("name", ["bottleneck_b16", "narrow_window_b16"])
def test_resident_panel_layers_match_oracle(name: str, precision: str, graphs: dict) -> None:
    g, feeds, want = graphs[name]
    model = compile_graph(g, precision=precision)
    try:
        got = model.run(feeds)
        again = model.run(feeds)
    finally:
        model.close()
    for k, w in want.items():
        scale = max(float(np.abs(w).max()), 1.0)
        err = float(np.abs(got[k].astype(np.float64) - w).max())
        assert err <= TOL[precision] * scale, f"{name}:{k} max abs err {err:.3g} (scale {scale:.3g})"
        np.testing.assert_array_equal(got[k], again[k])


def _tf32_exact(a: np.ndarray) -> np.ndarray:
    """Truncate fp32 values to TF32 (10 explicit mantissa bits), so that rounding them to TF32
    changes nothing."""
    return (a.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)


# (M, K, N) reaching each tensor-core form: one CTA per 128-row tile; a CTA pair per 256-row
# tile with one B plane in each CTA (N tiles of 128, long K, enough pair tiles to fill the
# GPU); a wide pair (256 x 256 tiles, N > 128; N = 640 leaves a partial last tile)
# (M, K, N) that select each tile form; "wide192": 256 x 192 pair tiles, ragged in M and in N
# (704 = 3 x 192 + 128), chosen because 64 of them fill the SM pairs in one wave; "split": two
# tiles of 144 K blocks, split K into 36 runs of 4 whose partial tiles are summed in order
GEMM_FORMS = {"single": (1024, 512, 128), "pair": (20480, 512, 128), "wide": (9728, 512, 640),
              "wide192": (4000, 768, 704), "split": (100, 4608, 256)}


def _run_gemm(form: str, m: int, k: int, n: int, seed: int = 3) -> tuple[np.ndarray, ...]:
    """A one-Gemm graph (TF32 mode) on TF32-exact activations: (x, w, bias, output)."""
    r = np.random.default_rng(seed)
    x = _tf32_exact(r.standard_normal((m, k)).astype(np.float32))
    w = r.standard_normal((k, n)).astype(np.float32)
    bias = r.standard_normal(n).astype(np.float32)
    g = Graph(f"gemm_{form}")
    xi = g.add_input("x", TensorType("float32", (m, k)))
    y = g.add_node("Gemm", [xi, g.constant(w), g.constant(bias)]).output
    g.add_output(y, "y")
    infer_shapes(g)
    optimize(g, "O3")
    schedule(g)
    model = compile_graph(g, precision="tf32")
    try:
        got = model.run({"x": x})["y"].astype(np.float64)
        # the split form sums its partial tiles in a fixed order: repeated runs agree bit for bit
        again = model.run({"x": x})["y"].astype(np.float64)
    finally:
        model.close()
    assert np.array_equal(got, again), f"{form}: two runs differ"
    return x, w, bias, got


@pytest.mark.parametrize("form", sorted(GEMM_FORMS))
def test_tf32_gemm_keeps_weights_exact(form: str, monkeypatch: pytest.MonkeyPatch) -> None:
    """With TF32-exact activations and exact weights asked for (MGC_CUDA_WEIGHT_PLANES=2, what
    TF32 mode does for graphs with convolutions), the only error left is the fp32 accumulation:
    the weights enter as their TF32 part plus the residual in every kernel form (without the
    residual the error would be about 3e-4 of the largest output)."""
    monkeypatch.setenv("MGC_CUDA_WEIGHT_PLANES", "2")
    x, w, bias, got = _run_gemm(form, *GEMM_FORMS[form])
    want = x.astype(np.float64) @ w.astype(np.float64) + bias.astype(np.float64)
    err = float(np.abs(got - want).max() / np.abs(want).max())
    assert err <= 2e-5, f"{form}: max error {err:.3g} of the largest output"


@pytest.mark.parametrize("form,shape", [("wide192", GEMM_FORMS["wide192"]), ("wide256", (8192, 512, 1024)),
                                        ("pair128", GEMM_FORMS["pair"]), ("single", GEMM_FORMS["single"]),
                                        ("split", GEMM_FORMS["split"])])
def test_tf32_gemms_take_one_weight_plane(form: str, shape: tuple) -> None:
    """A graph without convolutions lets the tile forms (256 x 192, 256 x 256 and 256 x 128 CTA
    pairs chosen here by the cost model, the last in the wide layout with 64 rows of B_hi per CTA;
    one-CTA 128 x 128 tiles; split K) take the weights as their TF32 part alone, one MMA per K step:
    the result is the product with B_hi (the weights rounded to the nearest TF32 value) up to the
    fp32 accumulation, and measurably not the product with exact weights."""
    x, w, bias, got = _run_gemm(form, *shape, seed=5)
    hi, _ = tf32_split(w)
    xs = x.astype(np.float64)
    want = xs @ hi.astype(np.float64) + bias.astype(np.float64)
    exact = xs @ w.astype(np.float64) + bias.astype(np.float64)
    scale = float(np.abs(want).max())
    assert float(np.abs(got - want).max()) <= 2e-5 * scale, form
    assert float(np.abs(got - exact).max()) > 1e-4 * scale, f"{form}: the weights entered exactly"


def test_tf32_residual_gemm_takes_one_weight_plane(monkeypatch: pytest.MonkeyPatch) -> None:
    """GPT-2's output projection shape (2048 x 768 x 768 + residual, one-CTA tiles with the residual
    in its own staging): in a graph without convolutions the weights enter as their TF32 part
    alone (one N = 128 MMA per K step), so the result is the product with B_hi up to the fp32
    accumulation; with MGC_CUDA_WEIGHT_PLANES=2 it is the exact-weight product."""
    m, k, n = 2048, 768, 768
    r = np.random.default_rng(11)
    x = _tf32_exact(r.standard_normal((m, k)).astype(np.float32))
    w = r.standard_normal((k, n)).astype(np.float32)
    bias = r.standard_normal(n).astype(np.float32)
    res = r.standard_normal((m, n)).astype(np.float32)

    def run() -> np.ndarray:
        g = Graph("gemm_residual")
        xi = g.add_input("x", TensorType("float32", (m, k)))
        ri = g.add_input("r", TensorType("float32", (m, n)))
        y = g.add_node("Gemm", [xi, g.constant(w), g.constant(bias)]).output
        z = g.add_node("Add", [y, ri]).output
        g.add_output(z, "z")
        infer_shapes(g)
        optimize(g, "O3")
        schedule(g)
        assert [nd.op for nd in g.nodes] == ["FusedGemm"]
        model = compile_graph(g, precision="tf32")
        try:
            return model.run({"x": x, "r": res})["z"].astype(np.float64)
        finally:
            model.close()

    hi, _ = tf32_split(w)
    base = bias.astype(np.float64) + res.astype(np.float64)
    want1 = x.astype(np.float64) @ hi.astype(np.float64) + base
    want2 = x.astype(np.float64) @ w.astype(np.float64) + base
    scale = float(np.abs(want2).max())
    got1 = run()
    assert float(np.abs(got1 - want1).max()) <= 2e-5 * scale
    assert float(np.abs(got1 - want2).max()) > 1e-4 * scale
    monkeypatch.setenv("MGC_CUDA_WEIGHT_PLANES", "2")
    got2 = run()
    assert float(np.abs(got2 - want2).max()) <= 2e-5 * scale


def test_tf32_batched_matmul_of_activations_is_exact_for_tf32_inputs() -> None:
    """Attention-shaped batched MatMuls on the tensor cores: Q K^T with both operands read through
    their head Transposes (two batch dimensions, strided rows), and P V with V N-major (copied
    K-major into the workspace). With TF32-exact inputs the only error left is the fp32
    accumulation (within 2e-5 of the largest output)."""
    r = np.random.default_rng(13)
    b, s, h, d = 2, 128, 12, 64

    def exact(*shape: int) -> np.ndarray:
        return _tf32_exact(r.standard_normal(shape).astype(np.float32))

    g = Graph("attention_matmuls")
    q = g.add_input("q", TensorType("float32", (b, s, h, d)))
    k = g.add_input("k", TensorType("float32", (b, s, h, d)))
    v = g.add_input("v", TensorType("float32", (b, s, h, d)))
    pr = g.add_input("p", TensorType("float32", (b, h, s, s)))
    qt = g.add_node("Transpose", [q], attrs={"perm": [0, 2, 1, 3]}).output
    kt = g.add_node("Transpose", [k], attrs={"perm": [0, 2, 3, 1]}).output
    vt = g.add_node("Transpose", [v], attrs={"perm": [0, 2, 1, 3]}).output
    g.add_output(g.add_node("MatMul", [qt, kt]).output, "scores")
    g.add_output(g.add_node("MatMul", [pr, vt]).output, "context")
    infer_shapes(g)
    optimize(g, "O3")
    schedule(g)
    feeds = {"q": exact(b, s, h, d), "k": exact(b, s, h, d), "v": exact(b, s, h, d), "p": exact(b, h, s, s)}
    model = compile_graph(g, precision="tf32")
    try:
        got = model.run(feeds)
    finally:
        model.close()
    q64, k64, v64 = (feeds[n].astype(np.float64).transpose(0, 2, 1, 3) for n in ("q", "k", "v"))
    want = {"scores": q64 @ k64.transpose(0, 1, 3, 2), "context": feeds["p"].astype(np.float64) @ v64}
    for name, w in want.items():
        err = float(np.abs(got[name].astype(np.float64) - w).max() / np.abs(w).max())
        assert err <= 2e-5, f"{name}: max error {err:.3g} of the largest output"
