"""``mgc`` with the cuda target: ``python -m mgc_cuda compile MODEL --target cuda ...``.

The parser is the reference's own (``cli.py:269-329`` ``build_parser``, every subcommand
unchanged); its ``compile`` subcommand gains

* ``--target {c,cuda}``: ``c`` (the default) runs the reference's ``cmd_compile`` untouched
  (``cli.py:193-240``); ``cuda`` lowers the optimised, scheduled graph for the B200 and loads it
  (``mgc_cuda.runtime.compile_graph``);
* ``--precision {tf32,strict,fp32}``, ``--device N`` and ``--strategy`` (the memory planner's
  strategy) for the cuda target.

With ``--target cuda`` the reference's flags keep their meaning: ``-O``, ``--seed`` and
``--int-high`` (random feeds from the reference interpreter's ``random_feeds``), ``--check``
(max abs difference against the reference interpreter on the unoptimised graph), ``--bench N``
(median and minimum latency of N runs through ``run``), ``-o DIR`` (``CudaCompiledModel.save``;
reload with ``CudaCompiledModel.load``), ``--json``. ``--emit-c``, ``--threads``, ``--no-openmp``,
``--no-neon`` and ``--cache-dir`` belong to the C build and are rejected or ignored as the reference
treats an inapplicable option: ``--emit-c`` is an error, the others have no effect.

MODEL is what the reference accepts (an ONNX file or a bundled sample; both need ``onnx``) or,
for either target of this CLI, ``zoo:NAME[:key=value,...]`` for a benchmark model built directly in
the reference IR (``mgc_cuda.zoo``: resnet50, mobilenet_v2, bert, gpt2, tiny_cnn,
tiny_transformer, mlp), e.g. ``zoo:resnet50:batch=1``.
"""

from __future__ import annotations

import argparse
import sys
from collections.abc import Sequence
from typing import Any

import numpy as np

from mgc_cuda import _reference  # noqa: F401
from ml_graph_compiler import cli as reference_cli
from ml_graph_compiler.errors import CompilerError
from ml_graph_compiler.ir import Graph

ZOO_PREFIX = "zoo:"


def _zoo_graph(spec: str) -> Graph:
    """``zoo:NAME[:key=value,...]`` -> the benchmark model built in the reference IR."""
    from mgc_cuda import zoo

    parts = spec[len(ZOO_PREFIX):].split(":", 1)
    name = parts[0]
    if name not in zoo.MODELS:
        raise CompilerError(f"unknown zoo model {name!r} (one of {', '.join(sorted(zoo.MODELS))})")
    kwargs: dict[str, Any] = {}
    if len(parts) > 1 and parts[1]:
        for item in parts[1].split(","):
            key, _, value = item.partition("=")
            if not key or not value:
                raise CompilerError(f"zoo model options are key=value, got {item!r}")
            kwargs[key] = int(value) if value.lstrip("-").isdigit() else value
    return zoo.MODELS[name](**kwargs)


def load_model(args: argparse.Namespace) -> Graph:
    if str(args.model).startswith(ZOO_PREFIX):
        if args.shape or args.dim:
            raise CompilerError("--shape / --dim apply to ONNX models; give zoo models their sizes as options")
        return _zoo_graph(args.model)
    return reference_cli.load_model(args)


def cmd_compile(args: argparse.Namespace) -> int:
    """``compile`` for both targets (the c target is the reference's own command)."""
    if args.target == "c":
        if str(args.model).startswith(ZOO_PREFIX):
            raise CompilerError("zoo models are for --target cuda; the c target loads ONNX files and samples")
        return int(reference_cli.cmd_compile(args))
    if args.emit_c:
        raise CompilerError("--emit-c applies to the c target")
    from mgc_cuda.runtime import compile_graph
    from ml_graph_compiler.interpreter import Interpreter, random_feeds
    from ml_graph_compiler.passes import optimize
    from ml_graph_compiler.schedule import schedule

    graph = load_model(args)
    feeds = random_feeds(graph, args.seed, int_high=args.int_high)
    reference = Interpreter(graph).run(feeds) if args.check else None
    optimize(graph, args.opt)
    schedule(graph)
    compiled = compile_graph(graph, strategy=args.strategy, precision=args.precision, device=args.device)
    try:
        report = compiled.report
        assert report is not None
        paths = compiled.gemm_paths()
        payload: dict[str, Any] = {
            "backend": "cuda",
            "pipeline": args.opt,
            "precision": args.precision,
            "device": args.device,
            "memory_plan": args.strategy,
            "launches": report.launches,
            "kernels": report.kernels,
            "gemm_records": {"tcgen05": sum(p[3] == "tcgen05" for p in paths),
                             "simt": sum(p[3] == "simt" for p in paths)},
            "arena_mb": round(report.arena_bytes / 2**20, 2),
            "weights_mb": round(report.weights_bytes / 2**20, 2),
            "lowering_s": report.lowering_seconds,
            "create_s": report.create_seconds,
        }
        outputs = compiled.run(feeds)
        if reference is not None:
            payload["max_abs_diff_vs_interpreter"] = max(
                float(np.max(np.abs(outputs[k].astype(np.float64) - reference[k]))) for k in reference
            )
        if args.bench:
            times = sorted(compiled.benchmark(feeds, warmup=2, repeat=args.bench))
            payload["latency_ms_median"] = round(1000 * times[len(times) // 2], 3)
            payload["latency_ms_min"] = round(1000 * times[0], 3)
        if args.output:
            payload["saved"] = str(compiled.save(args.output))
    finally:
        compiled.close()
    reference_cli._print(payload, args.json)
    return 0


def _subparser(parser: argparse.ArgumentParser, name: str) -> argparse.ArgumentParser:
    for action in parser._actions:  # argparse keeps the subcommands on its _SubParsersAction
        if isinstance(action, argparse._SubParsersAction) and name in action.choices:
            return action.choices[name]
    raise KeyError(name)


def build_parser() -> argparse.ArgumentParser:
    """The reference's parser with the target options on ``compile``."""
    parser = reference_cli.build_parser()
    p = _subparser(parser, "compile")
    p.add_argument("--target", choices=["c", "cuda"], default="c",
                   help="c: the reference's C backend; cuda: the B200 backend (this package)")
    p.add_argument("--precision", choices=["tf32", "strict", "fp32"], default="tf32",
                   help="cuda: TF32 tensor cores (default), 3xTF32 strict fp32 semantics, or exact fp32 SIMT")
    p.add_argument("--device", type=int, default=0, help="cuda: device ordinal")
    p.add_argument("--strategy", choices=["greedy_by_size", "first_fit", "naive"], default="greedy_by_size",
                   help="cuda: the memory planner's strategy")
    p.set_defaults(fn=cmd_compile)
    return parser


def main(argv: Sequence[str] | None = None) -> int:
    parser = build_parser()
    args = parser.parse_args(argv)
    try:
        return int(args.fn(args))
    except CompilerError as exc:
        print(f"error: {exc}", file=sys.stderr)
        return 2


if __name__ == "__main__":
    sys.exit(main())
