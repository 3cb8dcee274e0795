"""Parity at the configurations bench.py measures (3 and 4): their batch sizes,
precision, memory plans and the run() upload path, checked image by image (sequence by sequence)
against the strict batch-1 model, and, for the one image (sequence) that is the golden fixture's
input, against the reference interpreter's and C backend's outputs. Also which kernel computes
every GEMM-family record (mgc_cuda_gemm_paths): a TF32 model must not fall back to the CUDA-core
SIMT kernel anywhere, a strict one only on the batched products of two activations."""

from __future__ import annotations

import numpy as np
import pytest

from mgc_cuda import zoo
from mgc_cuda.runtime import compile_graph
from ml_graph_compiler.ir import Graph, TensorType
from ml_graph_compiler.passes import optimize
from ml_graph_compiler.schedule import schedule
from ml_graph_compiler.shape_inference import infer_shapes

pytestmark = pytest.mark.gpu

TF32 = 2e-2  # max abs logit error budget of TF32 mode


def prepared(make, **kw) -> Graph:
    g = make(**kw)
    optimize(g, "O3")
    schedule(g)
    return g


def assert_close_rows(got: np.ndarray, want: np.ndarray, scale: float, what: str) -> None:
    """Max abs error within the TF32 budget of the scale, and the argmax of every row equal
    wherever the reference's top two values are further apart than twice that budget."""
    err = float(np.abs(got.astype(np.float64) - want).max())
    assert err <= TF32 * scale, f"{what}: max abs err {err:.3g} > {TF32 * scale:.3g}"
    w2 = want.reshape(-1, want.shape[-1])
    g2 = got.reshape(-1, got.shape[-1])
    top2 = np.sort(w2, axis=1)[:, -2:]
    clear = top2[:, 1] - top2[:, 0] > 2 * TF32 * scale
    np.testing.assert_array_equal(g2.argmax(1)[clear], w2.argmax(1)[clear], err_msg=what)


def gemm_kernels(model) -> dict[str, list[str]]:
    out: dict[str, list[str]] = {"tcgen05": [], "simt": []}
    for _, op, name, path in model.gemm_paths():
        out[path].append(f"{op} {name}")
    return out


@pytest.fixture(scope="module")
def resnet50_strict_b1():
    m = compile_graph(prepared(zoo.resnet50, batch=1, seed=0), precision="strict")
    yield m
    m.close()


@pytest.mark.parametrize("strategy", ["greedy_by_size", "naive"])
def test_resnet50_b256_tf32_headline(strategy: str, resnet50_strict_b1, golden_models: dict) -> None:
    """The headline workload: ResNet-50 batch 256 in TF32 mode through run() with the input
    uploaded in four slices, on the planner's default plan and on the naive one. Image 0 is the
    golden input (compared with the reference's own logits); eight images spread over the four
    upload slices are compared with the strict batch-1 model; all 54 GEMM records run on tcgen05."""
    g = prepared(zoo.resnet50, batch=256, seed=0)
    x = np.random.default_rng(4).standard_normal((256, 3, 224, 224)).astype(np.float32)
    x[0] = zoo.feeds(prepared(zoo.resnet50, batch=1, seed=0), 0)["image"][0]
    m = compile_graph(g, precision="tf32", strategy=strategy)
    try:
        paths = gemm_kernels(m)
        assert not paths["simt"], paths["simt"]
        assert len(paths["tcgen05"]) == 54
        assert m.slices == 4
        y = m.run({"image": x})["logits"]
        again = m.run({"image": x})["logits"]
    finally:
        m.close()
    np.testing.assert_array_equal(again, y)  # deterministic replay
    for src in ("out", "c"):  # reference interpreter, reference C backend
        ref = golden_models[f"model_resnet50_b1_O3|{src}|logits|full"][0]
        assert float(np.abs(y[0].astype(np.float64) - ref).max()) <= TF32, src
    assert int(y[0].argmax()) == int(golden_models["model_resnet50_b1_O3|out|logits|argmax"][0])
    for i in (0, 37, 64, 100, 128, 170, 192, 255):  # every upload slice holds two of these
        want = resnet50_strict_b1.run({"image": x[i : i + 1]})["logits"]
        assert_close_rows(y[i : i + 1], want, 1.0, f"image {i}")


def test_mobilenet_v2_b128_tf32(golden_models: dict) -> None:
    """MobileNetV2 batch 128 (config 1) in TF32 mode. Its random-init logits are about 1e-9, so
    errors are measured relative to the largest logit; image 0 is the golden input."""
    g = prepared(zoo.mobilenet_v2, batch=128, seed=1)
    x = np.random.default_rng(1).standard_normal((128, 3, 224, 224)).astype(np.float32)
    x[0] = zoo.feeds(prepared(zoo.mobilenet_v2, batch=1, seed=1), 1)["image"][0]
    m = compile_graph(g, precision="tf32")
    try:
        paths = gemm_kernels(m)
        assert not paths["simt"], paths["simt"]
        y = m.run({"image": x})["logits"]
    finally:
        m.close()
    ref = golden_models["model_mobilenet_v2_b1_O3|out|logits|full"][0]
    assert_close_rows(y[:1], ref[None], float(np.abs(ref).max()), "golden image")
    m1 = compile_graph(prepared(zoo.mobilenet_v2, batch=1, seed=1), precision="strict")
    try:
        for i in (0, 45, 90, 127):
            want = m1.run({"image": x[i : i + 1]})["logits"]
            assert_close_rows(y[i : i + 1], want, float(np.abs(want).max()), f"image {i}")
    finally:
        m1.close()


def test_gpt2_b16_tf32(golden_models: dict) -> None:
    """GPT-2 batch 16, sequence 128 (config 3) in TF32 mode on the default plan: sequence 0 is the
    golden input (the reference's first 512 logits, row maxima and argmax), sequences 0, 7 and 15
    against the strict batch-1 model."""
    g = prepared(zoo.gpt2, batch=16, seq=128, seed=3)
    feeds = zoo.feeds(g, 11)
    feeds["input_ids"][0] = zoo.feeds(prepared(zoo.gpt2, batch=1, seq=128, seed=3), 3)["input_ids"][0]
    m = compile_graph(g, precision="tf32")
    try:
        paths = gemm_kernels(m)
        assert not paths["simt"], paths["simt"]
        y = m.run(feeds)["logits"]
    finally:
        m.close()
    key = "model_gpt2_b1_O3|out|logits"
    scale = max(float(np.abs(golden_models[f"{key}|rowmax"]).max()), 1.0)
    head = golden_models[f"{key}|head"]
    assert float(np.abs(y[0].reshape(-1)[: head.size] - head).max()) <= TF32 * scale
    assert float(np.abs(y[0].max(axis=-1) - golden_models[f"{key}|rowmax"]).max()) <= TF32 * scale
    m1 = compile_graph(prepared(zoo.gpt2, batch=1, seq=128, seed=3), precision="strict")
    try:
        for i in (0, 7, 15):
            want = m1.run({k: v[i : i + 1] for k, v in feeds.items()})["logits"]
            assert_close_rows(y[i : i + 1], want, max(float(np.abs(want).max()), 1.0), f"sequence {i}")
    finally:
        m1.close()


@pytest.mark.parametrize("name,batch,strategy", [("bert", 32, "naive"), ("bert", 1, "greedy_by_size"),
                                                  ("gpt2", 16, "greedy_by_size")])
def test_transformer_gemms_run_on_tensor_cores(name: str, batch: int, strategy: str) -> None:
    """Every GEMM-family record of BERT-base (the benchmark's batch 32 on its naive plan, and
    batch 1) and GPT-2 (batch 16) runs on tcgen05 in TF32 mode: per layer the projections and the
    FFN (BERT: Q, K, V, output, two FFN; GPT-2: QKV, output, two FFN) and one fused attention
    record (its two products)."""
    g = prepared(getattr(zoo, name), batch=batch, seq=128)
    m = compile_graph(g, precision="tf32", strategy=strategy)
    try:
        paths = gemm_kernels(m)
        kernels = dict(m.lowered.kernels)
    finally:
        m.close()
    assert not paths["simt"], paths["simt"]
    assert kernels.get("attention") == 12
    assert len(paths["tcgen05"]) >= 12 * ((6 if name == "bert" else 4) + 1)


@pytest.mark.parametrize("name", ["resnet50", "mobilenet_v2", "bert", "gpt2"])
def test_strict_gemm_paths(name: str) -> None:
    """Strict (3xTF32) mode: the convolutions and every GEMM with constant weights run on
    tcgen05; only batched products of two activations (attention's Q K^T and P V, MatMul nodes)
    may take the exact-fp32 SIMT kernel."""
    kw = {"seq": 128} if name in ("bert", "gpt2") else {}
    m = compile_graph(prepared(getattr(zoo, name), batch=1, **kw), precision="strict")
    try:
        rows = m.gemm_paths()
    finally:
        m.close()
    assert rows and all(path == "tcgen05" or op == "MatMul" for _, op, _, path in rows), \
        [r for r in rows if r[3] == "simt" and r[1] != "MatMul"]


def test_strict_step_bias_is_compensated() -> None:
    """The strict epilogue multiplies every output by (1 + STEP_BIAS), STEP_BIAS = 4.3e-8, to
    cancel the shrink toward zero of the tensor core's fp32 accumulation in one strict TMEM region
    (one K = 8 step, three products). This re-measures it: a strict GEMM with a constant B on
    positive raw fp32 data (uniform [0.5, 1.5), K = 512, the data the constant was measured on),
    where every region shrinks its partial sum by the same relative amount, must be unbiased after
    the compensation. The shrink implied by the result (STEP_BIAS minus the mean signed relative
    error) must lie within 20 % of STEP_BIAS, so that a change of the tensor core's accumulation
    (driver, firmware) shows here instead of silently shifting every strict result."""
    step_bias = 4.3e-8
    m_, k_, n_ = 4096, 512, 512
    rng = np.random.default_rng(21)
    g = Graph("strict_bias")
    x = g.add_input("x", TensorType("float32", (m_, k_)))
    w = g.constant(rng.uniform(0.5, 1.5, (k_, n_)).astype(np.float32), "w")
    g.add_output(g.add_node("MatMul", [x, w]).output, "y")
    infer_shapes(g)
    xv = rng.uniform(0.5, 1.5, (m_, k_)).astype(np.float32)
    m = compile_graph(g, precision="strict")
    try:
        assert [p for _, _, _, p in m.gemm_paths()] == ["tcgen05"]
        y = m.run({"x": xv})["y"].astype(np.float64)
    finally:
        m.close()
    exact = xv.astype(np.float64) @ w.data.astype(np.float64)
    rel = (y - exact) / exact
    implied = step_bias - float(rel.mean())
    assert 0.8 * step_bias <= implied <= 1.2 * step_bias, f"implied step shrink {implied:.3g} (mean rel err {rel.mean():.3g})"
    assert float(np.abs(rel).max()) <= 1e-6
