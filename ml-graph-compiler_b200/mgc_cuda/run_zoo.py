"""Compile one of the built-in benchmark models (``mgc_cuda.zoo``) at O3 for the `cuda` target and
run it through ``CudaCompiledModel.run``: the smallest driver of a forward pass, for profiling
one model at one size with external tools.

    python ml-graph-compiler_b200/mgc_cuda/run_zoo.py bert --batch 32 --seq 128 --strategy naive
    python ml-graph-compiler_b200/mgc_cuda/run_zoo.py resnet50 --batch 1

The model is compiled once; ``--runs`` forward passes follow (the first replay of the CUDA Graph
is a run like the others). Prints the output names and shapes and exits 0.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

if __package__ in (None, ""):
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from mgc_cuda import zoo  # noqa: E402
from mgc_cuda.runtime import compile_graph  # noqa: E402
from ml_graph_compiler.passes import optimize  # noqa: E402
from ml_graph_compiler.schedule import schedule  # noqa: E402

MODELS = {
    "resnet50": lambda a: zoo.resnet50(batch=a.batch, seed=0),
    "mobilenet_v2": lambda a: zoo.mobilenet_v2(batch=a.batch, seed=1),
    "bert": lambda a: zoo.bert(batch=a.batch, seq=a.seq, seed=2),
    "gpt2": lambda a: zoo.gpt2(batch=a.batch, seq=a.seq, seed=3),
}


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("model", choices=sorted(MODELS))
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--seq", type=int, default=128, help="sequence length (bert, gpt2)")
    ap.add_argument("--runs", type=int, default=1)
    ap.add_argument("--precision", default="tf32", choices=["tf32", "strict", "fp32"])
    ap.add_argument("--strategy", default="greedy_by_size", choices=["greedy_by_size", "first_fit", "naive"],
                    help="the reference planner's memory strategy")
    args = ap.parse_args(argv)
    g = MODELS[args.model](args)
    optimize(g, "O3")
    schedule(g)
    model = compile_graph(g, precision=args.precision, strategy=args.strategy)
    try:
        feeds = zoo.feeds(g, 0)
        out = {}
        for _ in range(max(args.runs, 1)):
            out = model.run(feeds)
    finally:
        model.close()
    for name, value in out.items():
        print(f"{name}: {tuple(value.shape)}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
