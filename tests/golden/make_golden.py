"""Generate the golden fixtures that pin the oracle to the reference.

Runs the reference compiler's own numpy interpreter (``interpreter.run_graph``) and, for whole
models, its C backend (``codegen.compile_graph``, gcc + OpenMP) on every case of
``tests/cases.py`` and stores inputs and outputs:

* ``ops.npz``: small cases, full inputs and interpreter outputs;
* ``models.npz``: whole models (inputs are regenerated from seeds by the builders; a checksum of
  each input is stored to detect drift), output summaries from the interpreter and from the C
  backend: the first 512 values, per-row sums / maxima / argmax over the last axis;
* ``manifest.json``: versions and the command line.

Run from the repository root in a checkout where the reference is importable::

    MGC_CC=/usr/bin/gcc python tests/golden/make_golden.py [--big]

It imports the reference's sources from ``$MGC_REFERENCE_SRC`` (the ``src`` directory of a
reference checkout) when that variable names an existing directory, else the installed copy in
``baseline/_ref``.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
_SRC = os.environ.get("MGC_REFERENCE_SRC", "")
if _SRC and Path(_SRC).is_dir():
    sys.path.insert(0, _SRC)
else:
    sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
sys.path.insert(0, str(ROOT / "tests"))

import cases  # noqa: E402
import ml_graph_compiler  # noqa: E402
from ml_graph_compiler.interpreter import run_graph  # noqa: E402

SUMMARY_HEAD = 512


def summarize(a: np.ndarray) -> dict[str, np.ndarray]:
    """Size-independent summaries of a (possibly large) output."""
    flat = np.asarray(a).reshape(-1)
    rows = np.asarray(a, dtype=np.float64).reshape(-1, a.shape[-1] if a.ndim else 1)
    return {
        "head": flat[:SUMMARY_HEAD].copy(),
        "rowsum": rows.sum(axis=1),
        "rowmax": rows.max(axis=1),
        "argmax": rows.argmax(axis=1).astype(np.int64),
    }


def checksum(a: np.ndarray) -> np.ndarray:
    v = np.asarray(a, dtype=np.float64).reshape(-1)
    return np.asarray([v.sum(), np.abs(v).sum(), v[: min(64, v.size)].sum(), float(v.size)])


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--big", action="store_true", help="also run the whole benchmark models")
    args = ap.parse_args()
    store: dict[str, np.ndarray] = {}
    for case in cases.all_cases():
        g, feeds = cases.prepare(case)
        out = run_graph(g, feeds)
        for k, v in feeds.items():
            store[f"{case.name}|in|{k}"] = np.asarray(v)
        for k, v in out.items():
            store[f"{case.name}|out|{k}"] = np.asarray(v)
    np.savez_compressed(HERE / "ops.npz", **store)
    print(f"ops.npz: {len(store)} arrays")
    if args.big:
        from ml_graph_compiler.codegen import compile_graph

        models: dict[str, np.ndarray] = {}
        for case in cases.big_model_cases():
            t0 = time.time()
            g, feeds = cases.prepare(case)
            for k, v in feeds.items():
                models[f"{case.name}|in|{k}|checksum"] = checksum(v)
            ref = run_graph(g, feeds)
            t1 = time.time()
            compiled = compile_graph(g, cache_dir="/tmp/mgc-golden-cache")
            cout = compiled.run(feeds)
            t2 = time.time()
            for k, v in ref.items():
                for sk, sv in summarize(v).items():
                    models[f"{case.name}|out|{k}|{sk}"] = sv
                for sk, sv in summarize(cout[k]).items():
                    models[f"{case.name}|c|{k}|{sk}"] = sv
                if v.size <= 4096:  # small outputs (classifier logits, pooler) are kept whole
                    models[f"{case.name}|out|{k}|full"] = np.asarray(v)
                    models[f"{case.name}|c|{k}|full"] = np.asarray(cout[k])
                diff = float(np.abs(np.asarray(cout[k], np.float64) - ref[k]).max())
                print(f"{case.name} {k}: interp {t1 - t0:.1f}s, C {t2 - t1:.1f}s, C vs interp max abs {diff:.3g}, "
                      f"|out| max {float(np.abs(ref[k]).max()):.4g}")
        np.savez_compressed(HERE / "models.npz", **models)
    path = HERE / "manifest.json"
    manifest = json.loads(path.read_text()) if path.exists() else {}
    manifest.pop("generator", None)
    made = {
        "reference_version": ml_graph_compiler.__version__,
        "reference_path": str(Path(ml_graph_compiler.__file__).parent),
        "numpy": np.__version__,
        "cc": os.environ.get("MGC_CC", ""),
    }
    manifest.update(made)
    manifest["ops.npz"] = {"generator": "tests/golden/make_golden.py", **made}
    if args.big:
        manifest["models.npz"] = {"generator": "tests/golden/make_golden.py --big", **made}
    path.write_text(json.dumps(manifest, indent=2) + "\n")


if __name__ == "__main__":
    main()
