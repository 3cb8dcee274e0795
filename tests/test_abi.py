"""The C ABI library builds for sm_100a, loads without a GPU, and exports every entry point that
include/mgc_cuda.h declares (no compute calls here)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from mgc_cuda import build, lowering, runtime

HEADER = Path(__file__).resolve().parents[1] / "include" / "mgc_cuda.h"


def declared() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mgc_cuda_\w+)\s*\(", text)))


def test_header_declares_the_model_and_kernel_abi() -> None:
    names = declared()
    for required in ("mgc_cuda_create", "mgc_cuda_run", "mgc_cuda_destroy", "mgc_cuda_profile",
                     "mgc_cuda_last_error", "mgc_cuda_gemm", "mgc_cuda_softmax", "mgc_cuda_layer_norm",
                     "mgc_cuda_pool_nhwc", "mgc_cuda_depthwise_nhwc", "mgc_cuda_reduce_mid",
                     "mgc_cuda_execute"):
        assert required in names


def test_library_exports_every_declared_symbol() -> None:
    lib = runtime.library()
    for name in declared():
        assert hasattr(lib, name), name
    assert set(declared()) == set(runtime.SIGNATURES), "ctypes signatures must cover the header"


def test_library_is_built_for_sm100a() -> None:
    flags = build.nvcc_flags()
    assert any("arch=compute_100a,code=sm_100a" in f for f in flags)
    assert build.library_path().exists()


def test_abi_version_and_errors_without_gpu() -> None:
    lib = runtime.library()
    assert lib.mgc_cuda_abi_version() == 3
    # a NULL handle is rejected on the host, before any CUDA call
    assert lib.mgc_cuda_run(None, None, None) == 2
    assert "NULL" in runtime.last_error(lib)
    assert lib.mgc_cuda_launch_count(None) == -1
    paths = (ctypes.c_int32 * 4)()
    assert lib.mgc_cuda_gemm_paths(None, paths, 4) == 2


def test_launch_record_layout_matches_header() -> None:
    text = HEADER.read_text()
    for name, value in (("MGC_LAUNCH_INTS", lowering.LAUNCH_INTS), ("MGC_LAUNCH_FLOATS", lowering.LAUNCH_FLOATS),
                        ("MGC_LAUNCH_REFS", lowering.LAUNCH_REFS)):
        assert re.search(rf"#define {name} {value}\b", text), name
    assert ctypes.sizeof(lowering.Launch) == 16 + 8 * 64 + 8 * 8 + 16 * 8 + 16
    kinds = dict(re.findall(r"(MGC_K_\w+) = (\d+)", text))
    assert int(kinds["MGC_K_GEMM"]) == lowering.K_GEMM
    assert int(kinds["MGC_K_MEMCPY"]) == lowering.K_MEMCPY
    assert int(kinds["MGC_K_ELEMENTWISE"]) == lowering.K_ELEMENTWISE


def test_elementwise_opcodes_match_the_kernel() -> None:
    src = (Path(build.SRC_DIR) / "kernels_mem.cuh").read_text()
    body = src[src.index("enum EwOp"): src.index("EW_NUM_OPS")]
    names = re.findall(r"EW_(\w+)", body)
    mapping = {"ADD": "Add", "SUB": "Sub", "MUL": "Mul", "DIV": "Div", "POW": "Pow", "MAX": "Max",
               "MIN": "Min", "EQ": "Equal", "LT": "Less", "GT": "Greater", "LE": "LessOrEqual",
               "GE": "GreaterOrEqual", "AND": "And", "OR": "Or", "XOR": "Xor", "WHERE": "Where",
               "RELU": "Relu", "SIGMOID": "Sigmoid", "TANH": "Tanh", "ERF": "Erf", "SQRT": "Sqrt",
               "EXP": "Exp", "LOG": "Log", "NEG": "Neg", "ABS": "Abs", "RECIP": "Reciprocal",
               "FLOOR": "Floor", "CEIL": "Ceil", "SIN": "Sin", "COS": "Cos", "SOFTPLUS": "Softplus",
               "IDENTITY": "Identity", "NOT": "Not", "GELU": "Gelu", "LEAKYRELU": "LeakyRelu",
               "HARDSIGMOID": "HardSigmoid", "CLIP": "Clip", "CAST": "Cast"}
    assert [mapping[n] for n in names] == lowering.EW_OPS


@pytest.mark.parametrize("name", ["mgc_cuda_device_supported"])
def test_device_query_without_gpu_is_zero(name: str) -> None:
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert getattr(runtime.library(), name)(0) == 0
