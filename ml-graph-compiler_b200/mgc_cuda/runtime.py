"""Load and run a model compiled for the `cuda` target through the libmgc_cuda C ABI (ctypes).

``CudaCompiledModel`` has the surface of the reference's ``CompiledModel``
(``codegen/runtime_lib.py:44-194``): ``run(feeds)`` validates names, shapes and dtypes and returns
numpy outputs, ``benchmark``, ``profile``, ``save`` / ``load``, ``report``, ``inputs`` /
``outputs``; an out-of-range Gather index raises ``GraphError`` (runtime_lib.py:142-143). The
native handle owns the device arena, the resident weights and the CUDA Graph; calls are
serialised with a lock because they share the arena.
"""

from __future__ import annotations

import ctypes
import json
import os
import threading
import time
from collections.abc import Mapping
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import numpy as np

from mgc_cuda import _reference  # noqa: F401
from mgc_cuda import build as _build
from mgc_cuda.lowering import BLOB_ALIGN, Chunk, Launch, LoweredModel, input_slice_plan, lower_graph
from ml_graph_compiler.errors import CodegenError, GraphError
from ml_graph_compiler.ir import Graph, TensorType, numpy_dtype
from ml_graph_compiler.memory import Strategy

_LIB: ctypes.CDLL | None = None
_LIB_LOCK = threading.Lock()

# Every symbol include/mgc_cuda.h declares, with its ctypes signature.
_VP, _I, _I64, _F, _D = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_double
SIGNATURES: dict[str, tuple[Any, list[Any]]] = {
    "mgc_cuda_abi_version": (_I, []),
    "mgc_cuda_last_error": (ctypes.c_char_p, []),
    "mgc_cuda_device_supported": (_I, [_I]),
    "mgc_cuda_create": (_I, [_VP, _I, _VP, _I64, _VP, _I64, _I64, _I64, _VP, _I, _VP, _I, _I, ctypes.POINTER(_VP)]),
    "mgc_cuda_run": (_I, [_VP, _VP, _VP]),
    "mgc_cuda_run_device": (_I, [_VP, _I]),
    "mgc_cuda_set_input_chunks": (_I, [_VP, _I, _I, _I64, _VP, _I]),
    "mgc_cuda_input_ptr": (_VP, [_VP, _I]),
    "mgc_cuda_output_ptr": (_VP, [_VP, _I]),
    "mgc_cuda_stream": (_VP, [_VP]),
    "mgc_cuda_profile": (_I, [_VP, ctypes.POINTER(_D), _I]),
    "mgc_cuda_launch_count": (_I, [_VP]),
    "mgc_cuda_gemm_paths": (_I, [_VP, ctypes.POINTER(ctypes.c_int32), _I]),
    "mgc_cuda_arena_bytes": (_I64, [_VP]),
    "mgc_cuda_weights_bytes": (_I64, [_VP]),
    "mgc_cuda_destroy": (None, [_VP]),
    "mgc_cuda_execute": (_I, [_VP, _I, _VP, _I64, _VP, _VP]),
    "mgc_cuda_gemm": (
        _I,
        [_I, _I, _I, _I, _VP, _I64, _I64, _I64, _VP, _I64, _I64, _I64, _VP, _I64, _I64, _F, _VP, _I, _VP,
         _I64, _I64, _F, _I, _F, _F, _I, _VP],
    ),
    "mgc_cuda_conv_nhwc": (
        _I,
        [_I] * 15 + [_VP, _VP, _VP, _VP, _I, _F, _F, _VP, _I, _VP],
    ),
    "mgc_cuda_conv_nhwc_noalloc": (_I, [_I] * 15 + [_VP, _VP, _VP, _VP, _I, _F, _F, _VP, _VP]),
    "mgc_cuda_depthwise_nhwc": (_I, [_I] * 14 + [_VP, _VP, _VP, _VP, _I, _F, _F, _VP, _VP]),
    "mgc_cuda_pool_nhwc": (_I, [_I] * 18 + [_VP, _VP, _VP]),
    "mgc_cuda_reduce_mid": (_I, [_I, _I64, _I64, _I64, _VP, _VP, _VP]),
    "mgc_cuda_softmax": (_I, [_I64, _I64, _I64, _VP, _VP, _I, _VP]),
    "mgc_cuda_layer_norm": (_I, [_I64, _I64, _VP, _VP, _VP, _F, _VP, _VP]),
}


def library(path: str | Path | None = None) -> ctypes.CDLL:
    """Load libmgc_cuda.so (building it first if its sources changed) and declare signatures."""
    global _LIB
    with _LIB_LOCK:
        if _LIB is not None and path is None:
            return _LIB
        lib_path = Path(path) if path is not None else _build.library_path()
        if path is None and not lib_path.exists():
            lib_path = _build.build()
        lib = ctypes.CDLL(str(lib_path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _LIB = lib
        return lib


def last_error(lib: ctypes.CDLL | None = None) -> str:
    raw = (lib or library()).mgc_cuda_last_error()
    return raw.decode() if raw else ""


def check(status: int, what: str, lib: ctypes.CDLL | None = None) -> None:
    """Raise the reference's exception types for a non-zero ABI status."""
    if status == 0:
        return
    msg = last_error(lib)
    if status == 1:
        raise GraphError(msg or "compiled model reported an out-of-range Gather index")
    raise CodegenError(f"{what} failed with status {status}: {msg}")


@dataclass
class CudaCompileReport:
    """The reference's CompileReport (runtime_lib.py:31-41) for the cuda target."""

    nodes: int
    launches: int
    arena_bytes: int
    weights_bytes: int
    lowering_seconds: float
    create_seconds: float
    precision: str
    device: int
    kernels: dict[str, int] = field(default_factory=dict)
    plan: dict[str, object] = field(default_factory=dict)


class CudaCompiledModel:
    """A model lowered to the cuda target: ``run(feeds)`` returns outputs as numpy arrays."""

    def __init__(self, lowered: LoweredModel, device: int = 0, report: CudaCompileReport | None = None) -> None:
        self.lib = library()
        self.lowered = lowered
        self.device = device
        self.inputs = lowered.inputs
        self.outputs = lowered.outputs
        self.node_names = lowered.node_names
        self.report = report
        self._lock = threading.Lock()
        self._handle = ctypes.c_void_p()
        blob = lowered.weights.blob()
        launches = lowered.launch_array()
        ins = (ctypes.c_int64 * max(len(self.inputs), 1))(*[t.nbytes for _, t in self.inputs])
        outs = (ctypes.c_int64 * max(len(self.outputs), 1))(*[t.nbytes for _, t in self.outputs])
        aux = np.ascontiguousarray(lowered.aux, np.int64)
        # run(): upload the input in slices that overlap the first layers' compute
        # (MGC_CUDA_SLICES=0 turns it off, =k uses k slices; 4 by default); buffers the sliced
        # prefix moves out of shared memory live after the lowered workspace
        self.slices = 0
        slices = int(os.environ.get("MGC_CUDA_SLICES", "4") or 0)
        plan = input_slice_plan(lowered, slices) if slices >= 2 else None
        workspace = lowered.workspace_bytes
        if plan is not None and plan[3]:
            workspace = -(-workspace // BLOB_ALIGN) * BLOB_ALIGN + plan[3]
        st = self.lib.mgc_cuda_create(
            ctypes.addressof(launches), len(lowered.launches), aux.ctypes.data, aux.size,
            blob.ctypes.data, blob.nbytes, lowered.arena_bytes, workspace, ctypes.addressof(ins),
            len(self.inputs),
            ctypes.addressof(outs), len(self.outputs), device, ctypes.byref(self._handle),
        )
        check(st, "mgc_cuda_create", self.lib)
        if plan is not None:
            prefix, images, descs, _ = plan
            arr = (Chunk * len(descs))(*descs)
            st = self.lib.mgc_cuda_set_input_chunks(self._handle, slices, prefix, images, ctypes.addressof(arr),
                                                    len(descs))
            check(st, "mgc_cuda_set_input_chunks", self.lib)
            self.slices = slices

    def __del__(self) -> None:
        self.close()

    def close(self) -> None:
        handle = getattr(self, "_handle", None)
        if handle is not None and handle.value:
            self.lib.mgc_cuda_destroy(handle)
            self._handle = ctypes.c_void_p()

    @property
    def handle(self) -> int:
        return int(self._handle.value or 0)

    @property
    def launch_count(self) -> int:
        return int(self.lib.mgc_cuda_launch_count(self._handle))

    # MGC_CUDA_PATH_* of include/mgc_cuda.h
    GEMM_PATHS = {1: "tcgen05", 2: "simt"}

    def gemm_paths(self) -> list[tuple[int, str, str, str]]:
        """(node index, op, node name, "tcgen05" | "simt") for every GEMM-family launch record:
        which kernel computes it (mgc_cuda_gemm_paths)."""
        n = len(self.lowered.launches)
        buf = (ctypes.c_int32 * max(n, 1))()
        check(self.lib.mgc_cuda_gemm_paths(self._handle, buf, n), "mgc_cuda_gemm_paths", self.lib)
        out = []
        for k, rec in enumerate(self.lowered.launches):
            if buf[k] in self.GEMM_PATHS:
                op, name = self.node_names[rec.node] if 0 <= rec.node < len(self.node_names) else ("", "")
                out.append((int(rec.node), op, name, self.GEMM_PATHS[buf[k]]))
        return out

    def input_ptr(self, i: int) -> int:
        return int(self.lib.mgc_cuda_input_ptr(self._handle, i) or 0)

    def output_ptr(self, i: int) -> int:
        return int(self.lib.mgc_cuda_output_ptr(self._handle, i) or 0)

    @property
    def stream(self) -> int:
        return int(self.lib.mgc_cuda_stream(self._handle) or 0)

    def _check_feeds(self, feeds: Mapping[str, np.ndarray]) -> list[np.ndarray]:
        names = [n for n, _ in self.inputs]
        missing = set(names) - set(feeds)
        extra = set(feeds) - set(names)
        if missing or extra:
            raise GraphError(f"inputs: missing {sorted(missing)}, unexpected {sorted(extra)}")
        arrays = []
        for name, t in self.inputs:
            a = np.asarray(feeds[name], order="C")
            if a.shape != t.shape or a.dtype != numpy_dtype(t.dtype):
                raise GraphError(f"input {name!r}: expected {t}, got {a.dtype}{list(a.shape)}")
            arrays.append(np.ascontiguousarray(a))
        return arrays

    def run(self, feeds: Mapping[str, np.ndarray], out: Mapping[str, np.ndarray] | None = None) -> dict[str, np.ndarray]:
        """Copy the inputs in, replay the CUDA Graph, copy the outputs out (runtime_lib.py:117-144).
        ``out`` may supply preallocated (e.g. pinned) output arrays."""
        arrays = self._check_feeds(feeds)
        results: dict[str, np.ndarray] = {}
        for name, t in self.outputs:
            o = out[name] if out is not None and name in out else np.empty(t.shape, numpy_dtype(t.dtype))
            if o.shape != t.shape or o.dtype != numpy_dtype(t.dtype) or not o.flags.c_contiguous:
                raise GraphError(f"output buffer {name!r} must be a contiguous {t}")
            results[name] = o
        # pointer tables of this call only: concurrent calls each pass their own buffers, and the
        # lock serialises the native call that shares the arena
        in_ptrs = (ctypes.c_void_p * max(len(arrays), 1))(*[a.ctypes.data for a in arrays])
        out_ptrs = (ctypes.c_void_p * max(len(results), 1))(*[o.ctypes.data for o in results.values()])
        with self._lock:
            st = self.lib.mgc_cuda_run(self._handle, ctypes.addressof(in_ptrs), ctypes.addressof(out_ptrs))
        check(st, "mgc_cuda_run", self.lib)
        return results

    def run_device(self, sync: bool = True) -> None:
        """Replay the graph on inputs already in the device input buffers."""
        with self._lock:
            st = self.lib.mgc_cuda_run_device(self._handle, int(sync))
        check(st, "mgc_cuda_run_device", self.lib)

    def benchmark(self, feeds: Mapping[str, np.ndarray], warmup: int = 3, repeat: int = 20) -> list[float]:
        """Wall-clock seconds of ``repeat`` calls of ``run`` (runtime_lib.py:146-156)."""
        for _ in range(warmup):
            self.run(feeds)
        times = []
        for _ in range(repeat):
            start = time.perf_counter()
            self.run(feeds)
            times.append(time.perf_counter() - start)
        return times

    def profile(self) -> list[tuple[str, str, float]]:
        """(op, node name, seconds) per scheduled node from one eagerly launched pass with CUDA
        events around each launch (the cuda form of runtime_lib.py:107-115)."""
        n = len(self.node_names)
        buf = (ctypes.c_double * max(n, 1))()
        with self._lock:
            st = self.lib.mgc_cuda_profile(self._handle, buf, n)
        check(st, "mgc_cuda_profile", self.lib)
        return [(op, name, float(buf[i]) * 1e-3) for i, (op, name) in enumerate(self.node_names)]

    # -- persistence -----------------------------------------------------------------------------
    def save(self, directory: str | Path) -> Path:
        """Write the launch list, aux data, weights blob and I/O metadata (runtime_lib.py:159-181)."""
        d = Path(directory)
        d.mkdir(parents=True, exist_ok=True)
        arr = self.lowered.launch_array()
        (d / "launches.bin").write_bytes(bytes(memoryview(arr))[: ctypes.sizeof(Launch) * len(self.lowered.launches)])
        np.asarray(self.lowered.aux, np.int64).tofile(d / "aux.bin")
        self.lowered.weights.blob().tofile(d / "weights.bin")
        meta = {
            "format": "mgc-cuda-1",
            "arena_bytes": self.lowered.arena_bytes,
            "workspace_bytes": self.lowered.workspace_bytes,
            "precision": self.lowered.precision,
            "inputs": [[n, t.dtype, list(t.shape)] for n, t in self.inputs],
            "outputs": [[n, t.dtype, list(t.shape)] for n, t in self.outputs],
            "nodes": [list(p) for p in self.node_names],
            "kernels": self.lowered.kernels,
            "report": self.report.__dict__ if self.report else None,
        }
        (d / "model.json").write_text(json.dumps(meta, indent=2) + "\n")
        return d

    @classmethod
    def load(cls, directory: str | Path, device: int = 0) -> CudaCompiledModel:
        """Reload a saved model without lowering again (runtime_lib.py:183-194)."""
        from mgc_cuda.lowering import Blob

        d = Path(directory)
        meta = json.loads((d / "model.json").read_text())
        raw = (d / "launches.bin").read_bytes()
        size = ctypes.sizeof(Launch)
        launches = [Launch.from_buffer_copy(raw[k : k + size]) for k in range(0, len(raw), size)]
        blob = Blob()
        blob.add(np.fromfile(d / "weights.bin", dtype=np.uint8))
        io = {k: [(n, TensorType(dt, tuple(s))) for n, dt, s in meta[k]] for k in ("inputs", "outputs")}
        lowered = LoweredModel(
            launches=launches,
            aux=np.fromfile(d / "aux.bin", dtype=np.int64),
            weights=blob,
            arena_bytes=int(meta["arena_bytes"]),
            workspace_bytes=int(meta.get("workspace_bytes", 0)),
            inputs=io["inputs"],
            outputs=io["outputs"],
            plan=None,  # type: ignore[arg-type]
            kernels=dict(meta.get("kernels", {})),
            node_names=[(str(a), str(b)) for a, b in meta.get("nodes", [])],
            precision=str(meta.get("precision", "tf32")),
        )
        return cls(lowered, device)


def compile_graph(
    graph: Graph,
    options: Any = None,
    cache_dir: str | Path | None = None,
    strategy: Strategy = "greedy_by_size",
    inplace: bool = True,
    name: str = "model",
    profile: bool = False,
    *,
    precision: str = "tf32",
    device: int = 0,
) -> CudaCompiledModel:
    """Lower an (already optimised and scheduled) graph for the cuda target and load it on
    ``device`` (the cuda form of runtime_lib.py:197-236, with the reference's positional
    parameters in its order; ``precision`` and ``device`` are keyword-only). ``options`` (the C
    compiler's BuildOptions), ``cache_dir``, ``name`` and ``profile`` are accepted for signature
    compatibility: there is no per-model build (one shared library, built in tree) and
    per-node profiling is always available through ``CudaCompiledModel.profile``."""
    del name, profile, cache_dir, options
    start = time.perf_counter()
    lowered = lower_graph(graph, strategy, inplace, precision)
    lowering_seconds = time.perf_counter() - start
    start = time.perf_counter()
    model = CudaCompiledModel(lowered, device)
    model.report = CudaCompileReport(
        nodes=len(graph.nodes),
        launches=model.launch_count,
        arena_bytes=lowered.arena_bytes,
        weights_bytes=lowered.weights.nbytes,
        lowering_seconds=round(lowering_seconds, 4),
        create_seconds=round(time.perf_counter() - start, 4),
        precision=precision,
        device=device,
        kernels=lowered.kernels,
        plan=lowered.plan.summary(),
    )
    return model


def compile_model(
    model: Any,
    opt: str = "O3",
    input_shapes: dict[str, tuple[int, ...]] | None = None,
    dims: dict[str, int] | None = None,
    reschedule: bool = True,
    **kwargs: Any,
) -> CudaCompiledModel:
    """ONNX model (proto or path) to a loaded cuda model (runtime_lib.py:239-256): import with the
    reference frontend, optimise, schedule, lower. Needs the ``onnx`` package."""
    from ml_graph_compiler.onnx_import import from_onnx
    from ml_graph_compiler.passes import optimize
    from ml_graph_compiler.schedule import schedule

    graph = from_onnx(model, input_shapes, dims)
    optimize(graph, opt)
    if reschedule:
        schedule(graph)
    return compile_graph(graph, **kwargs)
