"""Parity of the cuda target with the oracle on every operator, fused pattern and toy model.

Every case is lowered from the reference's own graph (after its O0/O2/O3 pipeline) and run
through the public API (``compile_graph`` -> ``CudaCompiledModel.run``, i.e. the C ABI). Integer,
boolean and index outputs must be bit-exact. Floating point tolerances, relative to the largest
|output| of the case (at least 1):

* ``strict`` (3xTF32 / exact fp32): 1e-4 max abs, the budget the benchmark configurations set
  for strict-fp32 logits;
* ``tf32``: 2e-2 max abs, the TF32-mode budget, and argmax agreement along the last axis.
"""

from __future__ import annotations

import numpy as np
import pytest

import cases
from mgc_cuda.runtime import compile_graph
from oracle import runner

pytestmark = pytest.mark.gpu

ALL = cases.all_cases()
TOL = {"strict": 1e-4, "tf32": 2e-2, "fp32": 1e-4}


def assert_parity(got: dict, want: dict, precision: str, what: str) -> None:
    assert set(got) == set(want)
    for name, w in want.items():
        g = got[name]
        assert g.shape == w.shape and g.dtype == w.dtype, f"{what}:{name}"
        if not np.issubdtype(w.dtype, np.floating):
            np.testing.assert_array_equal(g, w, err_msg=f"{what}:{name}")
            continue
        finite = np.isfinite(w)
        np.testing.assert_array_equal(np.isfinite(g), finite, err_msg=f"{what}:{name} non-finite pattern")
        scale = max(float(np.abs(w[finite]).max()) if finite.any() else 0.0, 1.0)
        err = float(np.abs(g[finite].astype(np.float64) - w[finite]).max()) if finite.any() else 0.0
        assert err <= TOL[precision] * scale, f"{what}:{name} max abs err {err:.3g} (scale {scale:.3g})"


@pytest.mark.parametrize("precision", ["strict", "tf32"])
@pytest.mark.parametrize("case", ALL, ids=[c.name for c in ALL])
def test_case_matches_oracle(case: cases.Case, precision: str) -> None:
    g, feeds = cases.prepare(case)
    want = runner.run(g, feeds)
    model = compile_graph(g, precision=precision)
    try:
        got = model.run(feeds)
        assert_parity(got, want, precision, case.name)
        # replaying the captured graph again gives bit-identical results
        again = model.run(feeds)
        for k in got:
            np.testing.assert_array_equal(got[k], again[k])
    finally:
        model.close()


def test_cases_match_reference_interpreter_fixtures(golden_ops: dict) -> None:
    """The same outputs against the reference interpreter's stored results (strict mode)."""
    for case in ALL:
        g, feeds = cases.prepare(case)
        model = compile_graph(g, precision="strict")
        got = model.run(feeds)
        want = {k.split("|")[2]: v for k, v in golden_ops.items() if k.startswith(f"{case.name}|out|")}
        assert_parity(got, want, "strict", case.name)
        model.close()


@pytest.mark.parametrize("shape,sizes", [((3, 5, 24), [8, 12, 4]), ((7, 9), [2, 3, 4]), ((4, 33, 16), [4, 12]),
                                         ((2, 6, 20), [4, 4, 4, 4, 4])])
def test_split_along_the_last_axis(shape: tuple, sizes: list) -> None:
    """A Split along the last axis whose outputs are all copied: up to four outputs in one
    split-mode copy record (four floats per thread when every width is a multiple of four and the
    buffers are 16-byte aligned, else one), more as one copy per output. Bit-exact with the
    oracle."""
    rng = np.random.default_rng(sum(shape) + len(sizes))
    g, feeds = cases.op_graph("Split", [("in", cases.f32(rng, *shape)), ("const", np.asarray(sizes))],
                              {"axis": -1}, n_outputs=len(sizes))
    want = runner.run(g, feeds)
    model = compile_graph(g, precision="tf32")
    try:
        splits = [r for r in model.lowered.launches if r.kind == 8 and r.i[28] == 2]
        assert len(splits) == (1 if len(sizes) <= 4 else 0)
        got = model.run(feeds)
        assert set(got) == set(want)
        for name, w in want.items():
            np.testing.assert_array_equal(got[name], w)
    finally:
        model.close()
