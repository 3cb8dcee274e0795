"""Pin the oracle to the reference: the oracle must reproduce every golden fixture that the
reference's own interpreter and C backend produced (tests/golden/make_golden.py)."""

from __future__ import annotations

import numpy as np
import pytest

import cases
from oracle import runner
from oracle.semantics import OracleError

ALL = cases.all_cases()
BIG = cases.big_model_cases()


def _close(got: np.ndarray, want: np.ndarray, rtol: float, atol: float, what: str) -> None:
    assert got.shape == want.shape, what
    assert got.dtype == want.dtype, f"{what}: dtype {got.dtype} != {want.dtype}"
    if np.issubdtype(want.dtype, np.floating):
        scale = max(float(np.abs(want).max()) if want.size else 0.0, 1.0)
        np.testing.assert_allclose(got, want, rtol=rtol, atol=atol * scale, err_msg=what)
    else:
        np.testing.assert_array_equal(got, want, err_msg=what)


@pytest.mark.parametrize("case", ALL, ids=[c.name for c in ALL])
def test_oracle_matches_reference_interpreter(case: cases.Case, golden_ops: dict) -> None:
    g, feeds = cases.prepare(case)
    for k, v in feeds.items():
        np.testing.assert_array_equal(v, golden_ops[f"{case.name}|in|{k}"], err_msg="input drift")
    out = runner.run(g, feeds)
    for name, got in out.items():
        _close(got, golden_ops[f"{case.name}|out|{name}"], 2e-5, 2e-6, f"{case.name}:{name}")


@pytest.mark.parametrize("case", BIG, ids=[c.name for c in BIG])
def test_oracle_matches_reference_on_models(case: cases.Case, golden_models: dict) -> None:
    """Whole benchmark models at batch 1: oracle vs the interpreter's and the C backend's
    summaries (head values, per-row sums and maxima, argmax)."""
    g, feeds = cases.prepare(case)
    for k, v in feeds.items():
        want = golden_models[f"{case.name}|in|{k}|checksum"]
        v64 = np.asarray(v, np.float64).reshape(-1)
        got = np.asarray([v64.sum(), np.abs(v64).sum(), v64[:64].sum(), float(v64.size)])
        np.testing.assert_allclose(got, want, rtol=1e-12, err_msg="input drift")
    out = runner.run(g, feeds)
    for name, arr in out.items():
        rows = np.asarray(arr, np.float64).reshape(-1, arr.shape[-1])
        scale = float(np.abs(rows).max())
        for src in ("out", "c"):
            head = golden_models[f"{case.name}|{src}|{name}|head"]
            np.testing.assert_allclose(arr.reshape(-1)[: head.size], head, atol=2e-6 * max(scale, 1.0), rtol=0)
            np.testing.assert_allclose(rows.max(axis=1), golden_models[f"{case.name}|{src}|{name}|rowmax"],
                                       atol=2e-6 * max(scale, 1.0), rtol=0)
            np.testing.assert_allclose(rows.sum(axis=1), golden_models[f"{case.name}|{src}|{name}|rowsum"],
                                       atol=2e-6 * max(scale, 1.0) * rows.shape[1] ** 0.5, rtol=0)
        np.testing.assert_array_equal(rows.argmax(axis=1), golden_models[f"{case.name}|out|{name}|argmax"])


def test_oracle_gather_out_of_range_raises() -> None:
    g, feeds = cases.op_graph("Gather", [("const", np.zeros((4, 2), np.float32)), ("in", np.asarray([1, 4]))])
    with pytest.raises(OracleError):
        runner.run(g, feeds)


def test_oracle_detects_a_planted_error(golden_ops: dict) -> None:
    """The comparison is live: a conv oracle with a perturbed weight no longer matches."""
    case = next(c for c in ALL if c.name == "conv3x3_p1")
    g, feeds = cases.prepare(case)
    node = g.nodes[0]
    w = node.inputs[1]
    w.data = w.data.copy()
    w.data[0, 0, 1, 1] += 0.01
    got = runner.run(g, feeds)["y0"]
    with pytest.raises(AssertionError):
        _close(got, golden_ops[f"{case.name}|out|y0"], 2e-5, 2e-6, "planted")
