"""``python -m mgc_cuda``: the reference's ``mgc`` parser with ``compile --target cuda``
(reference cli.py:193-240, 269-329). CPU tests parse and validate; the GPU test compiles a zoo
model, checks it against the reference interpreter, times it and round-trips ``-o``."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from mgc_cuda import cli

ROOT = Path(__file__).resolve().parents[1]


def test_parser_keeps_the_reference_subcommands_and_adds_the_target() -> None:
    p = cli.build_parser()
    args = p.parse_args(["compile", "zoo:tiny_cnn:batch=2", "--target", "cuda", "--precision", "strict",
                         "--device", "0", "-o", "out", "--check", "--bench", "3", "--json"])
    assert (args.target, args.precision, args.device, args.output, args.check, args.bench) == \
        ("cuda", "strict", 0, "out", True, 3)
    assert args.fn is cli.cmd_compile
    # the reference's defaults: the c target, -O3, the default planner strategy
    d = p.parse_args(["compile", "model.onnx"])
    assert (d.target, d.opt, d.precision, d.strategy) == ("c", "O3", "tf32", "greedy_by_size")
    for sub in ("inspect", "optimize", "run", "plan", "mlir"):
        assert p.parse_args([sub, "model.onnx"]).command == sub
    with pytest.raises(SystemExit):
        p.parse_args(["compile", "m.onnx", "--target", "rocm"])


def test_zoo_models_and_their_options() -> None:
    g = cli._zoo_graph("zoo:mlp:batch=3")
    assert g.inputs[0].tensor_type.shape[0] == 3
    g = cli._zoo_graph("zoo:tiny_transformer:kind=bert,batch=2")
    assert {v.name for v in g.inputs} == {"input_ids", "attention_mask"}
    with pytest.raises(cli.CompilerError):
        cli._zoo_graph("zoo:alexnet")
    with pytest.raises(cli.CompilerError):
        cli._zoo_graph("zoo:mlp:batch")


def test_target_specific_options_are_refused_before_any_device_work(capsys: pytest.CaptureFixture) -> None:
    assert cli.main(["compile", "zoo:mlp", "--target", "cuda", "--emit-c", "x.c"]) == 2
    assert "--emit-c" in capsys.readouterr().err
    assert cli.main(["compile", "zoo:mlp"]) == 2  # the c target loads ONNX files and samples
    assert "zoo models" in capsys.readouterr().err


def test_module_entry_point_prints_help() -> None:
    env = {**os.environ, "PYTHONPATH": os.pathsep.join([str(ROOT / "ml-graph-compiler_b200"), str(ROOT)])}
    out = subprocess.run([sys.executable, "-m", "mgc_cuda", "compile", "--help"], capture_output=True, text=True,
                         env=env, timeout=120)
    assert out.returncode == 0, out.stderr
    assert "--target" in out.stdout and "--precision" in out.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("model,precision,budget", [("zoo:tiny_cnn:batch=2", "strict", 1e-4),
                                                    ("zoo:tiny_transformer:kind=gpt,batch=2", "tf32", 2e-2)])
def test_compile_target_cuda_check_bench_and_save(model: str, precision: str, budget: float, tmp_path: Path,
                                                  capsys: pytest.CaptureFixture) -> None:
    from mgc_cuda.runtime import CudaCompiledModel
    from ml_graph_compiler.interpreter import random_feeds

    out_dir = tmp_path / "saved"
    rc = cli.main(["compile", model, "--target", "cuda", "--precision", precision, "--check", "--bench", "3",
                   "-o", str(out_dir), "--json"])
    assert rc == 0
    payload = json.loads(capsys.readouterr().out)
    assert payload["backend"] == "cuda" and payload["precision"] == precision
    assert payload["gemm_records"]["simt"] == 0 and payload["gemm_records"]["tcgen05"] > 0
    assert payload["max_abs_diff_vs_interpreter"] <= budget
    assert payload["latency_ms_median"] > 0
    loaded = CudaCompiledModel.load(out_dir)
    try:
        feeds = random_feeds(cli._zoo_graph(model), 0, int_high=100)
        got = loaded.run(feeds)
        assert set(got) == {n for n, _ in loaded.outputs}
        assert all(np.isfinite(v).all() for v in got.values())
    finally:
        loaded.close()
