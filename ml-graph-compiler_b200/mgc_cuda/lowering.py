"""Lowering of a scheduled, memory-planned graph to a CUDA launch list.

This is the `cuda` target's counterpart of the reference's C emitter (``codegen/c.py``): it walks
``graph.nodes`` in scheduled order, asks the reference planner (``memory.plan_memory``) where
every value lives exactly as ``CEmitter.ptr`` does (``c.py:323-335``), and produces

* one ``mgc_cuda_launch`` record (``include/mgc_cuda.h``) per kernel launch, whose tensor
  references are (space, index, byte offset) triples: arena offsets from the plan, offsets into
  the constant blob built here, or graph input / output numbers;
* an ``aux`` int64 array with the variable-length data of elementwise programs;
* the constant blob: every constant the kernels read, in the layout the kernels want (GEMM
  right-hand sides K-major and split into a TF32-exact high part and an fp32 residual).

Views (``memory.ALIAS_OPS``) emit nothing; output copies come from ``plan.copies``; an operator
without a lowering raises ``CodegenError`` (there is no CPU fallback). The slot layout of each
launch kind is written at its ``_emit_*`` function and read by ``csrc/launch.cuh``.
"""

from __future__ import annotations

import ctypes
import math
import os
import struct
from collections.abc import Sequence
from dataclasses import dataclass, field
from typing import Any

import numpy as np

from mgc_cuda import _reference  # noqa: F401
from ml_graph_compiler import ops
from ml_graph_compiler.codegen.c import CEmitter, WeightsBuilder
from ml_graph_compiler.errors import CodegenError
from ml_graph_compiler.ir import Graph, Node, TensorType, Value
from ml_graph_compiler.memory import ALIAS_OPS, MemoryPlan, Strategy, plan_memory

# ---- constants mirrored from include/mgc_cuda.h ------------------------------------------------
SPACE_NONE, SPACE_ARENA, SPACE_WEIGHTS, SPACE_INPUT, SPACE_OUTPUT, SPACE_RAW, SPACE_WORKSPACE = range(7)
DTYPES = {"float32": 0, "float64": 1, "int64": 2, "int32": 3, "int8": 4, "uint8": 5, "bool": 6}
ACTS = {"none": 0, "relu": 1, "clip": 2, "gelu": 3, "gelu_tanh": 4, "tanh": 5, "sigmoid": 6}
STRIDED, CONV_NHWC, CONV_NCHW = 0, 2, 3
PACKED_REGION = 1  # workspace reference index of a packed image until its offset is final
PRECISIONS = {"fp32": 0, "tf32": 1, "strict": 2}
K_GEMM, K_DEPTHWISE, K_POOL, K_REDUCE_MID, K_SOFTMAX, K_LAYER_NORM = 1, 2, 3, 4, 5, 6
K_ELEMENTWISE, K_COPY, K_FILL, K_GATHER, K_REDUCE, K_ARGMAX, K_RANGE, K_MEMCPY, K_IM2COL, K_PACK = range(7, 17)
K_ATTENTION = 17
KIND_NAMES = {
    K_GEMM: "gemm", K_DEPTHWISE: "depthwise", K_POOL: "pool", K_REDUCE_MID: "reduce",
    K_SOFTMAX: "softmax", K_LAYER_NORM: "layer_norm", K_ELEMENTWISE: "elementwise",
    K_COPY: "copy", K_FILL: "fill", K_GATHER: "gather", K_REDUCE: "reduce", K_ARGMAX: "argmax",
    K_RANGE: "range", K_MEMCPY: "memcpy", K_IM2COL: "im2col", K_PACK: "pack", K_ATTENTION: "attention",
}
LAUNCH_INTS, LAUNCH_FLOATS, LAUNCH_REFS = 64, 8, 8
# Elementwise program operations, numbered as csrc/kernels_mem.cuh EwOp.
EW_OPS = [
    "Add", "Sub", "Mul", "Div", "Pow", "Max", "Min",
    "Equal", "Less", "Greater", "LessOrEqual", "GreaterOrEqual", "And", "Or", "Xor",
    "Where", "Relu", "Sigmoid", "Tanh", "Erf", "Sqrt", "Exp", "Log",
    "Neg", "Abs", "Reciprocal", "Floor", "Ceil", "Sin", "Cos", "Softplus",
    "Identity", "Not", "Gelu", "LeakyRelu", "HardSigmoid", "Clip", "Cast",
]
EW_CODE = {name: i for i, name in enumerate(EW_OPS)}
EW_MAX_RANK, EW_MAX_LEAVES, EW_MAX_INSTR, COPY_MAX_RANK = 6, 20, 40, 8
SPLIT_MAX_OUT = 4  # outputs of one split-mode copy (csrc/kernels_mem.cuh)
SOFTMAX_ROW_MAX = 1024  # longest row the register-resident softmax holds (kernels_norm.cuh)
# fused attention (csrc/attention.cuh): keys per row, head widths, shared memory per CTA
ATTN_MAX_SK, ATTN_MAX_D, ATTN_SMEM_LIMIT = 256, 128, 232448 - 1024
ATTN_NONE, ATTN_ADD, ATTN_SUB, ATTN_KEEP, ATTN_FILL = range(5)  # score program masks (attention.cuh)


def _attn_fits(sk: int, dqk: int, dv: int) -> bool:
    """Whether the fused attention kernel takes these extents (attention.cuh attn_fits)."""
    if not (1 <= sk <= ATTN_MAX_SK and 4 <= dqk <= ATTN_MAX_D and 4 <= dv <= ATTN_MAX_D) or dqk % 4 or dv % 4:
        return False
    skp, dqp, dvp = (-(-x // 32) * 32 for x in (sk, dqk, dv))
    region0 = max(skp * 512, dqp * 512 + skp * dqp * 4, dvp * 512)
    return 1024 + region0 + skp * dvp * 4 <= ATTN_SMEM_LIMIT
PHASE_TILE_ROWS = 128  # output pixels of one phase-split row tile (the tensor-core M tile)
PHASE_MAX_KH = 7  # filter rows of a phase-split tile (its packed rows fill one shared-memory stage)
HEAD_FLOP_SHARE = 0.02  # largest share of a graph's GEMM FLOPs an output head computed in 3xTF32 may have
_EW_BINARY = {"Add", "Sub", "Mul", "Div", "Pow", "Max", "Min"}
_EW_FLOAT_ONLY = {"Clip", "Relu", "Sigmoid", "Tanh", "Erf", "Sqrt", "Exp", "Log", "Neg", "Abs", "Reciprocal",
                  "Floor", "Ceil", "Sin", "Cos", "Softplus", "Gelu", "LeakyRelu", "HardSigmoid"}


def _f32x4_instr(op: str, cls: list[str]) -> bool:
    """One instruction of the four-wide fp32 form (kernels_mem.cuh ``ew_f32x4_form``): byte
    operands (class I) only where the typed program converts them to fp32 as well."""
    if op in _EW_BINARY:
        return "F" in cls[:2]
    if op == "Where":
        return cls[0] == "I"
    if op in _EW_FLOAT_ONLY:
        return cls[0] == "F"
    return op in ("Identity", "Cast")
BLOB_ALIGN = 256
TF32_MASK = np.uint32(0xFFFFE000)


class Ref(ctypes.Structure):
    _fields_ = [("space", ctypes.c_int32), ("index", ctypes.c_int32), ("offset", ctypes.c_int64)]


class Launch(ctypes.Structure):
    _fields_ = [
        ("kind", ctypes.c_int32),
        ("node", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("i", ctypes.c_int64 * LAUNCH_INTS),
        ("f", ctypes.c_double * LAUNCH_FLOATS),
        ("r", Ref * LAUNCH_REFS),
        ("aux_offset", ctypes.c_int64),
        ("aux_len", ctypes.c_int64),
    ]


assert ctypes.sizeof(Launch) == 16 + 8 * LAUNCH_INTS + 8 * LAUNCH_FLOATS + 16 * LAUNCH_REFS + 16

class Chunk(ctypes.Structure):
    """mgc_cuda_chunk: one batch-dependent field of a record of the sliced prefix."""

    _fields_ = [("launch", ctypes.c_int32), ("what", ctypes.c_int32), ("slot", ctypes.c_int32),
                ("reserved", ctypes.c_int32), ("per_image", ctypes.c_int64)]


RefT = tuple[int, int, int]
NO_REF: RefT = (SPACE_NONE, 0, 0)


def tf32_split(a: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """(hi, lo) with hi = a rounded to the nearest TF32 value (10 mantissa bits, ties away from
    zero) and lo = a - hi, exact in fp32; hi + lo == a bit for bit."""
    a = np.ascontiguousarray(a, np.float32)
    bits = a.view(np.uint32)
    hi = ((bits + np.uint32(0x1000)) & TF32_MASK).view(np.float32)
    finite = np.isfinite(a) & np.isfinite(hi)
    hi = np.where(finite, hi, a).astype(np.float32)
    lo = np.where(finite, a - hi, np.float32(0)).astype(np.float32)
    return hi, lo


class Blob(WeightsBuilder):
    """The constant blob: the reference's ``WeightsBuilder`` (c.py:166-218: chunks kept as
    references, keyed de-duplication, ``digest``, ``blob``) with every chunk starting on a
    256-byte boundary instead of 64 (TMA needs 16; whole 256-byte lines for the weight panels)."""

    def add(self, array: np.ndarray, key: Any = None) -> int:
        offset = super().add(array, key)
        self.size = -(-self.size // BLOB_ALIGN) * BLOB_ALIGN
        return offset


@dataclass
class LoweredModel:
    launches: list[Launch]
    aux: np.ndarray
    weights: Blob
    arena_bytes: int
    workspace_bytes: int
    inputs: list[tuple[str, TensorType]]
    outputs: list[tuple[str, TensorType]]
    plan: MemoryPlan
    kernels: dict[str, int]
    node_names: list[tuple[str, str]]
    precision: str

    def launch_array(self) -> ctypes.Array:
        arr = (Launch * max(len(self.launches), 1))()
        for k, rec in enumerate(self.launches):
            arr[k] = rec
        return arr


def _strides(shape: Sequence[int]) -> list[int]:
    out = [1] * len(shape)
    for i in range(len(shape) - 2, -1, -1):
        out[i] = out[i + 1] * int(shape[i + 1])
    return out


def _broadcast_strides(shape: Sequence[int], out_shape: Sequence[int]) -> list[int]:
    """Element strides of ``shape`` broadcast right-aligned to ``out_shape`` (0 on broadcast)."""
    src = _strides(shape)
    pad = len(out_shape) - len(shape)
    return [0 if d - pad < 0 or shape[d - pad] == 1 else src[d - pad] for d in range(len(out_shape))]


def _collapse(dims: list[int], strides: list[list[int]]) -> tuple[list[int], list[list[int]]]:
    """Fewest loop dimensions for a nest over ``dims`` that addresses every operand through
    ``strides``: size-1 axes are dropped, and an axis joins the group before it when, for every
    operand, stepping the group once equals stepping this axis across its whole extent (the loop
    nests of ``CEmitter.loops``, c.py:360-379, collapse the same way)."""
    out_dims: list[int] = []
    out_strides: list[list[int]] = [[] for _ in strides]
    for axis, extent in enumerate(dims):
        if extent == 1:
            continue
        joins = bool(out_dims) and all(o[-1] == s[axis] * extent for o, s in zip(out_strides, strides))
        if joins:
            out_dims[-1] *= extent
        else:
            out_dims.append(extent)
        for o, s in zip(out_strides, strides):
            if joins:
                o[-1] = s[axis]
            else:
                o.append(s[axis])
    return out_dims, out_strides


def _split_at(shape: Sequence[int], first: int, last: int | None = None) -> tuple[int, int, int]:
    """(outer, n, inner): the products of the extents before axis ``first``, of axes first..last
    and after ``last`` -- how a reduction, softmax, argmax or gather walks a row-major tensor."""
    last = first if last is None else last
    sizes = [int(d) for d in shape]
    return math.prod(sizes[:first]), math.prod(sizes[first : last + 1]), math.prod(sizes[last + 1 :])


def _axis_attr(node: Node, rank: int, default: int) -> int:
    """The node's ``axis`` attribute made non-negative."""
    axis = int(node.attrs.get("axis", default))
    return axis % rank if rank and axis < 0 else axis


@dataclass(frozen=True)
class ConvShape:
    """Geometry of a Conv / FusedConv node in its own layout: the image is x [N,H,W,C] with HWIO
    weights after the layout pass (NHWC), else x [N,C,H,W] with OIHW weights."""

    nhwc: bool
    n: int
    h: int
    w: int
    c: int
    kh: int
    kw: int
    cg: int      # input channels per group
    cout: int
    group: int
    win: Any     # ops.window_geometry: strides, dilations, pads, out_hw

    @property
    def pointwise(self) -> bool:
        return self.kh == self.kw == 1 and self.win.strides == (1, 1) and self.win.pads == (0, 0, 0, 0)

    def geo(self) -> dict[str, int]:
        """The K_GEMM / K_IM2COL convolution slots."""
        (sh, sw), (dh, dw), (pt, pl, _, _), (oh, ow) = self.win.strides, self.win.dilations, self.win.pads, self.win.out_hw
        return {"H": self.h, "W": self.w, "C": self.c, "KH": self.kh, "KW": self.kw, "SH": sh, "SW": sw, "DH": dh,
                "DW": dw, "PT": pt, "PL": pl, "OH": oh, "OW": ow}


# positions of (n, h, w, c) in the image shape and of (kh, kw, cin, cout) in the weight shape
_CONV_AXES = {True: ((0, 1, 2, 3), (0, 1, 2, 3)), False: ((0, 2, 3, 1), (2, 3, 1, 0))}


def conv_shape(node: Node) -> ConvShape:
    nhwc = ops.conv_layout(node) == "NHWC"
    x_axes, w_axes = _CONV_AXES[nhwc]
    xs, ws = node.input(0).tensor_type.shape, node.input(1).tensor_type.shape
    n, h, w, c = (int(xs[a]) for a in x_axes)
    kh, kw, cg, cout = (int(ws[a]) for a in w_axes)
    return ConvShape(nhwc, n, h, w, c, kh, kw, cg, cout, int(node.attrs.get("group", 1)),
                     ops.window_geometry(node, (h, w), (kh, kw)))


def _oriented(shape: Sequence[int], transposed: int) -> tuple[int, int]:
    """(rows, cols) of a 2-D operand as the product reads it."""
    rows, cols = int(shape[0]), int(shape[1])
    return (cols, rows) if transposed else (rows, cols)


def _bits(value: float) -> int:
    return struct.unpack("<q", struct.pack("<d", float(value)))[0]


class CudaEmitter:
    """Builds the launch list for one scheduled graph (see the module docstring)."""

    SUPPORTED = CEmitter.SUPPORTED

    def __init__(
        self,
        graph: Graph,
        strategy: Strategy = "greedy_by_size",
        inplace: bool = True,
        precision: str = "tf32",
    ) -> None:
        unsupported = sorted({n.op for n in graph.nodes} - self.SUPPORTED)
        if unsupported:
            raise CodegenError(f"the cuda backend has no kernel for: {', '.join(unsupported)}")
        for v in graph.values():
            if v.type is not None and v.type.dtype == "float16":
                raise CodegenError(f"float16 tensors are not supported ({v.name})")
        if precision not in PRECISIONS:
            raise CodegenError(f"precision must be one of {sorted(PRECISIONS)}, got {precision!r}")
        self.graph = graph
        self.precision = precision
        # TF32 mode takes the weights of a graph without convolutions (the transformer models) in
        # one TF32 plane, B rounded to the nearest TF32 value, where a tile form allows it: the
        # float64 oracle with every GEMM operand rounded so puts BERT-base's last hidden state
        # within 2.5e-3 and GPT-2's logits within 2.8e-3 (1.5e-3 / 1.8e-3 with exact weights)
        # against the 2e-2 budget, while ResNet-50's 53 stacked convolutions need exact weights
        # (3.95e-2 with rounded ones). MGC_CUDA_WEIGHT_PLANES=2 keeps exact weights everywhere.
        self._one_plane = (precision == "tf32" and os.environ.get("MGC_CUDA_WEIGHT_PLANES", "") != "2"
                           and not any(n.op in ("Conv", "FusedConv") for n in graph.nodes))
        self.plan = plan_memory(graph, strategy=strategy, inplace=inplace)
        self.weights = Blob()
        self.launches: list[Launch] = []
        self.aux: list[int] = []
        self.kernels: dict[str, int] = {}
        self._node = -1
        self._keep_alive: list[Value] = []
        self.workspace_bytes = 0  # scratch regions (im2col patch matrices, channel-packed images)
        self._im2col_bytes = 0    # the im2col region at offset 0, shared by every im2col launch
        self._packed: dict[int, RefT] = {}  # id(value) -> its channel-packed copy in the workspace
        # id(value) -> (source, element strides, first element) of a Transpose that MatMul reads
        # through (not copied)
        self._through: dict[int, tuple[Value, list[int], int]] = {}
        # id(Split output) -> (the Split's input, element strides, first element): an output that
        # only Transposes read, through strides, is never copied (see _split_view)
        self._split_src: dict[int, tuple[Value, list[int], int]] = {}
        self._pack_regions: list[tuple[int, int]] = []  # (offset, bytes) of each packed image
        # id(value) -> element strides of a Transpose output stored K-major for MatMul (see
        # _kmajor_b_only); every reader goes through _view
        self._stored: dict[int, list[int]] = {}
        # Transposes whose input MatMul wrote their output directly (see _write_through)
        self._written_through: set[int] = set()
        # id(value) -> aux words of the elementwise program that the softmax reading it evaluates
        self._row_programs: dict[int, list[int]] = {}
        self._heads = self._output_heads()  # nodes computed in 3xTF32 in TF32 mode
        # fused attention chains (_attention_plan): id(second MatMul) -> its K_ATTENTION record
        # (ints, floats, refs), and the ids of the nodes the record absorbs
        self._attn_emit: dict[int, tuple[list[int], list[float], list[RefT]]] = {}
        self._attn_skip: set[int] = set()
        # MaxPool nodes computed in the epilogue of the convolution before them (_pooled_by)
        self._pool_skip: set[int] = set()
        # GlobalAveragePool nodes that add their producer's epilogue partial sums (_gap_partials)
        self._gap_from_partials: set[int] = set()

    # -- references ----------------------------------------------------------------------------
    def _root(self, value: Value) -> Value:
        while value.data is None and value.producer is not None and value.producer.op in ALIAS_OPS:
            value = value.producer.input(0)
        return value

    def const_data(self, value: Value) -> np.ndarray:
        root = self._root(value)
        if root.data is None:
            raise CodegenError(f"constant {value.name!r} has no data")
        return root.data.reshape(value.tensor_type.shape)

    def ref(self, value: Value | None, byte_offset: int = 0) -> RefT:
        if value is None:
            return NO_REF
        loc = self.plan.location(value)
        if loc.kind == "const":
            root = self._root(value)
            if root.data is None:
                raise CodegenError(f"constant {value.name!r} has no data")
            off = self.weights.add(root.data, key=("raw", id(root)))
            return (SPACE_WEIGHTS, 0, off + byte_offset)
        if loc.kind == "input":
            return (SPACE_INPUT, loc.index, byte_offset)
        if loc.kind == "output":
            return (SPACE_OUTPUT, loc.index, byte_offset)
        return (SPACE_ARENA, 0, loc.index + byte_offset)

    def weights_ref(self, array: np.ndarray, key: Any = None) -> RefT:
        return (SPACE_WEIGHTS, 0, self.weights.add(array, key=key))

    # -- records -----------------------------------------------------------------------------------
    def emit(
        self,
        kind: int,
        ints: Sequence[int] = (),
        floats: Sequence[float] = (),
        refs: Sequence[RefT] = (),
        dtype: int = 0,
        aux: Sequence[int] | None = None,
        count: str | None = None,
    ) -> None:
        if len(ints) > LAUNCH_INTS or len(floats) > LAUNCH_FLOATS or len(refs) > LAUNCH_REFS:
            raise CodegenError("launch record overflow")
        rec = Launch()
        rec.kind = kind
        rec.node = self._node
        rec.dtype = dtype
        for k, v in enumerate(ints):
            rec.i[k] = int(v)
        for k, v in enumerate(floats):
            rec.f[k] = float(v)
        for k, (space, index, offset) in enumerate(refs):
            rec.r[k].space, rec.r[k].index, rec.r[k].offset = space, index, offset
        if aux is not None:
            rec.aux_offset = len(self.aux)
            rec.aux_len = len(aux)
            self.aux.extend(int(v) for v in aux)
        self.launches.append(rec)
        name = count or KIND_NAMES[kind]
        self.kernels[name] = self.kernels.get(name, 0) + 1

    # -- dispatch ------------------------------------------------------------------------------------
    def node(self, node: Node) -> None:
        if id(node) in self._attn_skip:
            self.kernels["fused into attention"] = self.kernels.get("fused into attention", 0) + 1
            return
        if id(node) in self._pool_skip:
            self.kernels["pool fused into convolution"] = self.kernels.get("pool fused into convolution", 0) + 1
            return
        if node.op in ALIAS_OPS:
            if node.op == "Dropout" and len(node.outputs) > 1:
                mask = node.outputs[1]
                self._fill(mask, 1)
            self.kernels["view"] = self.kernels.get("view", 0) + 1
            return
        if node.op == "FusedElementwise" or ops.is_elementwise(node.op):
            if node.op == "FusedElementwise":
                program = [(str(op), dict(a), [int(x) for x in args]) for op, a, args in node.attrs["program"]]
            else:
                program = [(node.op, dict(node.attrs), [i if node.inputs[i] is not None else -1
                                                        for i in range(len(node.inputs))])]
            if self._softmax_reads(node):
                made = self._elementwise(node.output, program, list(node.inputs), defer=True)
                if made is not None and made[1] and made[0][made[0][0]] % node.output.tensor_type.shape[-1] == 0:
                    self._row_programs[id(node.output)] = made[0]
                    self.kernels["elementwise into softmax"] = self.kernels.get("elementwise into softmax", 0) + 1
                    return
            self._elementwise(node.output, program, list(node.inputs))
            return
        if node.op in self.REDUCE_KINDS:
            self._reduce(node)
            return
        handler = getattr(self, f"op_{node.op}", None)
        if handler is None:
            raise CodegenError(f"the cuda backend has no kernel for {node.op}")
        handler(node)

    # -- elementwise programs (c.py:471-529) -------------------------------------------------------
    def _elementwise(
        self, out_value: Value, program: list[tuple[str, dict[str, Any], list[int]]], leaves: list[Value | None],
        defer: bool = False,
    ) -> tuple[list[int], bool] | None:
        """Emit a K_ELEMENTWISE record for the program; with ``defer``, return its aux words instead,
        with whether the program has the four-wide fp32 form (the kernels' ``ew_f32x4_form``)."""
        shape = list(out_value.tensor_type.shape)
        if int(np.prod(shape)) == 0:
            return None
        tensor_leaves = [
            i for i, v in enumerate(leaves)
            if v is not None and not (v.is_constant and v.data is not None and v.data.size == 1)
        ]
        all_strides = [_strides(shape)] + [
            _broadcast_strides(leaves[i].tensor_type.shape, shape) for i in tensor_leaves  # type: ignore[union-attr]
        ]
        dims, coll = _collapse(list(shape), all_strides)
        if len(dims) > EW_MAX_RANK:
            raise CodegenError(f"elementwise loop nest of rank {len(dims)} (max {EW_MAX_RANK})")
        present = [v for v in leaves if v is not None]
        if len(leaves) > EW_MAX_LEAVES or len(program) > EW_MAX_INSTR:
            raise CodegenError(f"elementwise program too large ({len(present)} leaves, {len(program)} ops)")
        aux: list[int] = [len(dims), *dims]
        aux += [DTYPES[out_value.tensor_type.dtype], *self.ref(out_value)]
        aux.append(len(leaves))
        types_all: list[TensorType | None] = []
        consts: list[np.ndarray | None] = []
        # register classes of the four-wide fp32 form: F fp32, I bytes read as fp32, X neither
        cls: list[str] = []
        for i, v in enumerate(leaves):
            if v is None:  # omitted optional input: never read
                aux += [DTYPES["float32"], 1, 0, *NO_REF, *([0] * len(dims))]
                types_all.append(None)
                consts.append(None)
                cls.append("F")
                continue
            t = v.tensor_type
            types_all.append(t)
            consts.append(v.data)
            if i in tensor_leaves:
                strides = coll[1 + tensor_leaves.index(i)]
                aux += [DTYPES[t.dtype], 0, 0, *self.ref(v), *strides]
                cls.append("F" if t.dtype == "float32" else "I" if t.dtype in ("bool", "uint8") else "X")
            else:
                scalar = self.const_data(v).reshape(()).item()
                bits = _bits(scalar) if t.dtype in ("float32", "float64") else int(scalar)
                aux += [DTYPES[t.dtype], 1, bits, *NO_REF, *([0] * len(dims))]
                cls.append("F" if t.dtype == "float32" else "X")
        f32x4 = out_value.tensor_type.dtype == "float32" and "X" not in cls
        aux.append(len(program))
        for op, attrs, args in program:
            if op not in EW_CODE:
                raise CodegenError(f"elementwise {op} has no cuda kernel")
            sub = Node(op, [], [Value("_")], dict(attrs))
            arg_types = [types_all[a] if a >= 0 else None for a in args]
            out_t = ops.spec(op).infer(sub, arg_types, [consts[a] if a >= 0 else None for a in args])[0]
            if out_t.dtype == "float16":
                raise CodegenError("float16 is not supported")
            types_all.append(out_t)
            consts.append(None)
            a = list(args) + [-1] * (3 - len(args))
            imm = [0.0, 0.0]
            if op == "Clip":
                imm = [float(attrs.get("min", -np.inf)), float(attrs.get("max", np.inf))]
            elif op == "Gelu":
                imm = [1.0 if attrs.get("approximate", "none") == "tanh" else 0.0, 0.0]
            elif op == "LeakyRelu":
                imm = [float(attrs.get("alpha", 0.01)), 0.0]
            elif op == "HardSigmoid":
                imm = [float(attrs.get("alpha", 0.2)), float(attrs.get("beta", 0.5))]
            aux += [EW_CODE[op], DTYPES[out_t.dtype], a[0], a[1], a[2], _bits(imm[0]), _bits(imm[1])]
            f32x4 = f32x4 and out_t.dtype == "float32" and _f32x4_instr(op, [cls[x] if x >= 0 else "" for x in a])
            cls.append("F" if out_t.dtype == "float32" else "X")
        if defer:
            return aux, f32x4
        self.emit(K_ELEMENTWISE, aux=aux, dtype=DTYPES[out_value.tensor_type.dtype], count="elementwise")
        return None

    def _clobbered(self, first: Node, last: Node, values: Sequence[Value]) -> bool:
        """Whether a node scheduled strictly between ``first`` and ``last`` writes memory that one
        of ``values`` occupies (the planner may reuse it once its last reader has run)."""
        ranges = [r for r in (self._arena_range(v) for v in values) if r is not None]
        if not ranges:
            return False
        order = {id(n): k for k, n in enumerate(self.graph.nodes)}
        for later in self.graph.nodes[order[id(first)] + 1 : order[id(last)]]:
            if later.op in ALIAS_OPS:
                continue
            for v in later.outputs:
                r = self._arena_range(v)
                if r is not None and any(r[0] < hi and lo < r[1] for lo, hi in ranges):
                    return True
        return False

    def _softmax_reads(self, node: Node) -> bool:
        """Whether this elementwise node's output is read only by a Softmax / LogSoftmax over its
        last axis that can evaluate the program itself as it reads each row (the scale and mask of
        attention scores; the fused output never reaches memory): rows of at most
        SOFTMAX_ROW_MAX fp32 elements in groups of four, the program's tensor leaves untouched until
        the softmax runs, and the softmax output either clear of every leaf or exactly on a leaf of
        the same shape (each row is read whole before it is written)."""
        out = node.output
        t = out.tensor_type
        if len(out.users) != 1 or any(v is out for _, v in self.graph.named_outputs()):
            return False
        user = out.users[0]
        if user.op not in ("Softmax", "LogSoftmax") or user.input(0) is not out or t.dtype != "float32":
            return False
        axis = int(user.attrs.get("axis", -1))
        axis = axis + t.rank if axis < 0 else axis
        n = t.shape[-1] if t.rank else 0
        if axis != t.rank - 1 or n == 0 or n % 4 or n > SOFTMAX_ROW_MAX or t.size >= 1 << 31:
            return False
        leaves = [v for v in node.inputs if v is not None and not v.is_constant]
        if self._clobbered(node, user, leaves):
            return False
        dst = self._arena_range(user.output)
        for v in leaves:
            r = self._arena_range(v)
            if dst is None or r is None or not (r[0] < dst[1] and dst[0] < r[1]):
                continue
            if tuple(v.tensor_type.shape) != tuple(t.shape) or r[0] != dst[0]:
                return False
        return True

    # -- copies (c.py:558-660) --------------------------------------------------------------------
    def _copy(
        self,
        shape: Sequence[int],
        src: RefT,
        src_strides: Sequence[int],
        src_base: int,
        dst: RefT,
        dst_strides: Sequence[int],
        dst_base: int,
        esize: int,
        count: str = "copy",
    ) -> None:
        """K_COPY slots: i[0] rank, i[1] element bytes, i[2..9] shape, i[10..17] source strides,
        i[18] source base, i[19..26] destination strides, i[27] destination base (elements),
        i[28] 0 (1 selects Tile, 2 the split mode of _split_copy); r[0] source, r[1] destination."""
        if int(np.prod([int(d) for d in shape])) == 0:
            return
        dims, (ss, ds) = _collapse([int(d) for d in shape], [list(src_strides), list(dst_strides)])
        if len(dims) > COPY_MAX_RANK:
            raise CodegenError(f"copy of rank {len(dims)} (max {COPY_MAX_RANK})")
        ints = [0] * 29
        ints[0], ints[1] = len(dims), esize
        for d in range(len(dims)):
            ints[2 + d], ints[10 + d], ints[19 + d] = dims[d], ss[d], ds[d]
        ints[18], ints[27] = src_base, dst_base
        self.emit(K_COPY, ints, refs=[src, dst], count=count)

    def _copy_value(self, out_shape: Sequence[int], src: Value, dst_ref: RefT, dst_strides: Sequence[int],
                    dst_base: int, count: str = "copy") -> None:
        t = src.tensor_type
        if src.is_constant and src.data is not None and src.data.size == 1:
            # broadcast a scalar constant: a fill of the destination region
            if list(dst_strides) == _strides(out_shape) and dst_base == 0:
                self._fill_ref(dst_ref, int(np.prod(out_shape)), src.data.reshape(()).item(), t.dtype)
                return
        self._copy(out_shape, self.ref(src), _broadcast_strides(t.shape, out_shape), 0, dst_ref,
                   dst_strides, dst_base, t.itemsize, count)

    def _arena_range(self, value: Value) -> tuple[int, int] | None:
        loc = self.plan.location(value)
        if loc.kind != "arena":
            return None
        root = self._root(value)
        return loc.index, loc.index + root.tensor_type.nbytes

    def _read_through(self, node: Node, x: Value, view_strides: list[int]) -> bool:
        """Whether the batched MatMul(s) using this Transpose's output can read its source through
        strides instead of a copy (TF32 mode, where the tensor-core batched GEMM takes strided
        operands): every user is a MatMul that finds k (A) or k or n (B) contiguous in the view,
        the output is no graph output, and no node scheduled before the last such MatMul writes
        memory the source occupies (the planner may reuse it once the Transpose has run). The
        MatMul's own destination is checked when it is lowered (op_MatMul)."""
        out = node.output
        if self.precision != "tf32" or out.tensor_type.rank < 3 or x.tensor_type.dtype != "float32":
            return False
        if any(v is out for _, v in self.graph.named_outputs()) or not out.users:
            return False
        for user in out.users:
            if user.op != "MatMul" or user.input(0).tensor_type.rank < 3 or user.input(1).tensor_type.rank < 3:
                return False
            if user.input(0) is out and view_strides[-1] != 1:
                return False
            if user.input(1) is out and view_strides[-1] != 1 and view_strides[-2] != 1:
                return False
        src = self.plan.location(x)
        if src.kind not in ("arena", "input"):
            return False
        own = self._arena_range(x)
        order = {id(n): k for k, n in enumerate(self.graph.nodes)}
        last = max(order[id(u)] for u in out.users)
        for later in self.graph.nodes[order[id(node)] + 1 : last]:
            if later.op in ALIAS_OPS:
                continue
            for v in later.outputs:
                r = self._arena_range(v)
                if own is not None and r is not None and r[0] < own[1] and own[0] < r[1]:
                    # a later Transpose that is itself read through its source writes nothing
                    if later.op == "Transpose" and self._transpose_reads_through(later):
                        continue
                    return False
        return True

    def _transpose_reads_through(self, node: Node) -> bool:
        """Whether op_Transpose will lower this Transpose to nothing by letting its MatMuls read its
        source through strides: the same test, on the same source and strides, that op_Transpose
        applies when it reaches the node (a Split view's source, else the Transpose's input)."""
        if id(node) in self._written_through:
            return True
        x = node.input(0)
        perm = ops.transpose_perm(node, x.tensor_type.rank)
        view = self._split_view_of(x)
        if view is not None:
            src, ss, _ = view
            return self._read_through(node, src, [ss[p] for p in perm])
        ss = _strides(x.tensor_type.shape)
        return self._read_through(node, x, [ss[p] for p in perm])

    def _kmajor_b_only(self, out: Value, view_strides: list[int]) -> bool:
        """Whether a Transpose's output is read only as the N-major B operand of batched MatMuls
        in TF32 mode (attention's values in P @ V), so that it can be stored K-major instead of
        being copied once more by the MatMul."""
        t = out.tensor_type
        if self.precision != "tf32" or t.rank < 3 or t.dtype != "float32" or not out.users:
            return False
        if any(v is out for _, v in self.graph.named_outputs()):
            return False
        if self.plan.location(out).kind != "arena":
            return False
        for user in out.users:
            if user.op != "MatMul" or user.input(1) is not out or user.input(0) is out:
                return False
            if user.input(0).tensor_type.rank < 3:
                return False
        return True

    def op_Transpose(self, node: Node) -> None:
        if id(node) in self._written_through:
            self.kernels["view"] = self.kernels.get("view", 0) + 1
            return
        x = node.input(0)
        perm = ops.transpose_perm(node, x.tensor_type.rank)
        ss = _strides(x.tensor_type.shape)
        shape = node.output.tensor_type.shape
        out = node.output
        view = self._split_view_of(x)
        if view is not None:
            # x is a view of a Split's input that was never copied: read it there
            src, ss, base = view
            vs = [ss[p] for p in perm]
            if self._read_through(node, src, vs):
                self._through[id(out)] = (src, vs, base)
                return
            if self._kmajor_b_only(out, vs):
                kshape = [*shape[:-2], shape[-1], shape[-2]]
                kst = _strides(kshape)
                self._stored[id(out)] = [*kst[:-2], kst[-1], kst[-2]]
                self._copy(kshape, self.ref(src), [*vs[:-2], vs[-1], vs[-2]], base, self.ref(out), kst, 0,
                           src.tensor_type.itemsize, count="transpose")
                return
            self._copy(shape, self.ref(src), vs, base, self.ref(out), _strides(shape), 0, src.tensor_type.itemsize,
                       count="transpose")
            return
        if self._read_through(node, x, [ss[p] for p in perm]):
            self._through[id(out)] = (x, [ss[p] for p in perm], 0)
            return
        if self._kmajor_b_only(out, [ss[p] for p in perm]):
            # every reader is a batched MatMul taking it as an N-major B: store it K-major
            # ([..., n, k]) in its own buffer, so the MatMul reads it as it is
            kshape = [*shape[:-2], shape[-1], shape[-2]]
            kst = _strides(kshape)
            stored = [*kst[:-2], kst[-1], kst[-2]]
            self._stored[id(out)] = stored
            src = [ss[p] for p in perm]
            self._copy(kshape, self.ref(x), [*src[:-2], src[-1], src[-2]], 0, self.ref(out), kst, 0,
                       x.tensor_type.itemsize, count="transpose")
            return
        users = out.users
        if (len(users) == 1 and users[0].inputs and users[0].inputs[0] is out and self._tap_packed(users[0])
                and all(v is not out for _, v in self.graph.named_outputs())):
            plan = self._narrow_plan(users[0])
            if shape[3] % 4 or plan["wrows"] or plan["phase"]:
                # the only use is a narrow-channel convolution that reads a padded copy: write
                # it straight from the source (the plain transposed copy would be unused)
                self._packed[id(out)] = self._emit_pack(self.ref(x), shape[0], shape[1], shape[2], shape[3],
                                                        [ss[p] for p in perm], plan)
                return
        self._copy(shape, self.ref(x), [ss[p] for p in perm], 0, self.ref(node.output), _strides(shape), 0,
                   x.tensor_type.itemsize, count="transpose")

    def op_Expand(self, node: Node) -> None:
        shape = node.output.tensor_type.shape
        self._copy_value(shape, node.input(0), self.ref(node.output), _strides(shape), 0)

    def op_Tile(self, node: Node) -> None:
        x = node.input(0)
        xs, os_ = x.tensor_type.shape, node.output.tensor_type.shape
        if len(os_) > COPY_MAX_RANK:
            raise CodegenError(f"Tile of rank {len(os_)}")
        if int(np.prod(os_)) == 0:
            return
        ints = [0] * 29
        ints[0], ints[1], ints[28] = len(os_), x.tensor_type.itemsize, 1
        xst = _strides(xs)
        for d in range(len(os_)):
            ints[2 + d], ints[10 + d], ints[19 + d] = os_[d], xs[d], xst[d]
        self.emit(K_COPY, ints, refs=[self.ref(x), self.ref(node.output)], count="copy")

    def _consts(self, node: Node) -> list[np.ndarray | None]:
        return [v.data if v is not None else None for v in node.inputs]

    def op_Slice(self, node: Node) -> None:
        x = node.input(0)
        xs = x.tensor_type.shape
        slices = ops.slice_params(node, xs, self._consts(node))
        ss = _strides(xs)
        base = 0
        strides = []
        for sl, st in zip(slices, ss, strict=True):
            base += int(sl.start or 0) * st
            strides.append(int(sl.step or 1) * st)
        shape = node.output.tensor_type.shape
        self._copy(shape, self.ref(x), strides, base, self.ref(node.output), _strides(shape), 0,
                   x.tensor_type.itemsize)

    def op_Concat(self, node: Node) -> None:
        out_t = node.output.tensor_type
        axis = int(node.attrs.get("axis", 0))
        axis = axis + out_t.rank if axis < 0 else axis
        ost = _strides(out_t.shape)
        offset = 0
        for v in node.inputs:
            if v is None:
                continue
            t = v.tensor_type
            if t.size:
                self._copy_value(t.shape, v, self.ref(node.output), ost, offset * ost[axis])
            offset += t.shape[axis]

    def op_Split(self, node: Node) -> None:
        x = node.input(0)
        xt = x.tensor_type
        axis = int(node.attrs.get("axis", 0))
        axis = axis + xt.rank if axis < 0 else axis
        ss = _strides(xt.shape)
        offset = 0
        views = [self._split_view(node, out_v) for out_v in node.outputs]
        wanted = [bool(out_v.users) or out_v in self.graph.outputs for out_v in node.outputs]
        if (axis == xt.rank - 1 and xt.itemsize == 4 and 2 <= len(node.outputs) <= SPLIT_MAX_OUT
                and not any(views) and all(wanted) and xt.size):
            # every output copied: one pass over the input writes them all (K_COPY split mode)
            self._split_copy(x, list(node.outputs))
            return
        for out_v, view in zip(node.outputs, views, strict=True):
            t = out_v.tensor_type
            if view:
                self._split_src[id(out_v)] = (x, list(ss), offset * ss[axis])
                self.kernels["view"] = self.kernels.get("view", 0) + 1
            elif out_v.users or out_v in self.graph.outputs:
                self._copy(t.shape, self.ref(x), ss, offset * ss[axis], self.ref(out_v), _strides(t.shape), 0,
                           xt.itemsize)
            offset += t.shape[axis]

    def _split_copy(self, x: Value, outs: list[Value]) -> None:
        """K_COPY in split mode: i[28] 2, i[0] 2 and i[2..3] (rows, row width) for the generic
        checks, i[1] element bytes, i[29] outputs, i[30..33] their widths along the last axis,
        i[34] rows; r[0] the input, r[1..] the outputs (each contiguous)."""
        xt = x.tensor_type
        width = int(xt.shape[-1])
        rows = int(xt.size) // width
        ints = [0] * 35
        ints[0], ints[1], ints[2], ints[3] = 2, xt.itemsize, rows, width
        ints[28], ints[29], ints[34] = 2, len(outs), rows
        for j, o in enumerate(outs):
            ints[30 + j] = int(o.tensor_type.shape[-1])
        self.emit(K_COPY, ints, refs=[self.ref(x)] + [self.ref(o) for o in outs], count="split")

    @staticmethod
    def _split_strides(vshape: Sequence[int], strides: list[int], shape: Sequence[int]) -> list[int] | None:
        """Element strides of a Reshape of a strided view of shape vshape, when the Reshape keeps
        every leading axis and splits only the last, contiguous one (heads out of the hidden
        axis); None otherwise."""
        vshape, shape = list(vshape), list(shape)
        if vshape == shape:
            return list(strides)
        r = len(vshape)
        if len(shape) < r or shape[: r - 1] != vshape[: r - 1] or strides[-1] != 1:
            return None
        if int(np.prod(shape[r - 1 :])) != vshape[-1]:
            return None
        return list(strides[:-1]) + _strides(shape[r - 1 :])

    def _split_view(self, node: Node, out_v: Value) -> bool:
        """Whether a Split output is read only by Transposes (directly or through one Reshape that
        splits its last axis), which then read the Split's input through strides: no copy. The
        Split's input must stay untouched until the last of those Transposes (and, when they are
        read through, until their MatMuls: _read_through checks that against the same source)."""
        if any(v is out_v for _, v in self.graph.named_outputs()) or not out_v.users:
            return False
        x = node.input(0)
        if self.plan.location(x).kind not in ("arena", "input") or x.tensor_type.dtype != "float32":
            return False
        readers: list[Node] = []
        for u in out_v.users:
            if u.op == "Transpose" and u.input(0) is out_v:
                readers.append(u)
            elif u.op == "Reshape" and u.input(0) is out_v and len(u.outputs) == 1:
                rv = u.output
                if any(v is rv for _, v in self.graph.named_outputs()) or not rv.users:
                    return False
                if self._split_strides(out_v.tensor_type.shape, [1] * (out_v.tensor_type.rank - 1) + [1],
                                       rv.tensor_type.shape) is None:
                    return False
                for w in rv.users:
                    if w.op != "Transpose" or w.input(0) is not rv:
                        return False
                    readers.append(w)
            else:
                return False
        order = {id(n): k for k, n in enumerate(self.graph.nodes)}
        last = max(readers, key=lambda n: order[id(n)])
        return not self._clobbered(node, last, [x]) and not any(
            self._overlaps(r.output, x) for r in readers)

    def _overlaps(self, a: Value, b: Value) -> bool:
        ra, rb = self._arena_range(a), self._arena_range(b)
        return ra is not None and rb is not None and ra[0] < rb[1] and rb[0] < ra[1]

    def _split_view_of(self, v: Value) -> tuple[Value, list[int], int] | None:
        """(source, element strides, first element) of a value that is a Split view or one
        Reshape of it (see _split_view), else None."""
        if id(v) in self._split_src:
            return self._split_src[id(v)]
        prod = v.producer
        if prod is not None and prod.op == "Reshape" and id(prod.input(0)) in self._split_src:
            src, strides, base = self._split_src[id(prod.input(0))]
            inner = prod.input(0).tensor_type.shape
            st = self._split_strides(inner, strides, v.tensor_type.shape)
            if st is not None:
                return src, st, base
        return None

    def op_Pad(self, node: Node) -> None:
        if node.attrs.get("mode", "constant") != "constant":
            raise CodegenError(f"Pad mode {node.attrs.get('mode')!r} has no cuda kernel")
        x = node.input(0)
        xt, ot = x.tensor_type, node.output.tensor_type
        pads = ops.pad_amounts(node, xt.rank, self._consts(node))
        if any(p < 0 for p in pads):
            raise CodegenError("negative Pad amounts have no cuda kernel")
        fill = 0.0
        value_v = node.optional_input(2)
        if value_v is not None:
            if value_v.data is None:
                raise CodegenError("Pad value must be a constant")
            fill = value_v.data.reshape(()).item()
        self._fill(node.output, fill)
        ost = _strides(ot.shape)
        base = sum(p * s for p, s in zip(pads[: xt.rank], ost, strict=True))
        if xt.size:
            self._copy_value(xt.shape, x, self.ref(node.output), ost, base)

    # -- constants (c.py:690-734) -------------------------------------------------------------------
    def _fill_ref(self, dst: RefT, count: int, value: Any, dtype: str) -> None:
        """K_FILL slots: i[0] element count, i[1] element bytes, i[2] raw value bits; r[0] dst."""
        if count == 0:
            return
        arr = np.asarray(value, dtype=np.dtype(dtype if dtype != "bool" else np.bool_))
        raw = int.from_bytes(arr.tobytes(), "little", signed=False)
        if raw >= 1 << 63:
            raw -= 1 << 64
        self.emit(K_FILL, [count, arr.itemsize, raw], refs=[dst], count="constant")

    def _fill(self, value: Value, fill: Any) -> None:
        t = value.tensor_type
        self._fill_ref(self.ref(value), t.size, fill, t.dtype)

    def _write_constant(self, value: Value, array: np.ndarray) -> None:
        t = value.tensor_type
        flat = np.asarray(array, dtype=np.dtype(t.dtype if t.dtype != "bool" else np.bool_)).reshape(-1)
        if flat.size and np.all(flat == flat[0]):
            self._fill_ref(self.ref(value), t.size, flat[0].item(), t.dtype)
            return
        src = self.weights_ref(flat)
        self.emit(K_MEMCPY, [t.nbytes], refs=[src, self.ref(value)], count="constant")

    def op_Shape(self, node: Node) -> None:
        self._write_constant(node.output, ops.shape_value(node, node.input(0).tensor_type.shape))

    def op_Size(self, node: Node) -> None:
        self._write_constant(node.output, np.asarray([node.input(0).tensor_type.size], np.int64))

    def op_ConstantOfShape(self, node: Node) -> None:
        value = node.attrs.get("value")
        fill = np.asarray(value).reshape(-1)[0].item() if value is not None else 0.0
        self._fill(node.output, fill)

    def op_Range(self, node: Node) -> None:
        """K_RANGE slots: i[0] count; dtype; r[0] out, r[1] start scalar, r[2] delta scalar."""
        t = node.output.tensor_type
        self.emit(K_RANGE, [t.size], refs=[self.ref(node.output), self.ref(node.input(0)), self.ref(node.input(2))],
                  dtype=DTYPES[t.dtype], count="constant")

    # -- gather (c.py:662-688) -----------------------------------------------------------------------
    def op_Gather(self, node: Node) -> None:
        """K_GATHER slots: i[0] outer, i[1] axis extent, i[2] inner, i[3] index count, i[4] index
        dtype, i[5] element bytes; r[0] data, r[1] indices, r[2] out."""
        x, idx = node.input(0), node.input(1)
        xt, it = x.tensor_type, idx.tensor_type
        axis = _axis_attr(node, xt.rank, 0)
        outer, extent, inner = _split_at(xt.shape, axis)
        if it.dtype not in ("int64", "int32"):
            raise CodegenError(f"Gather indices of type {it.dtype} have no cuda kernel")
        if xt.itemsize not in (1, 4, 8):
            raise CodegenError(f"Gather of {xt.dtype} has no cuda kernel")
        self.emit(K_GATHER, [outer, extent, inner, it.size, DTYPES[it.dtype], xt.itemsize],
                  refs=[self.ref(x), self.ref(idx), self.ref(node.output)], dtype=DTYPES[xt.dtype])

    # -- reductions (c.py:736-821, 1255-1273) -------------------------------------------------------
    # K_REDUCE kind codes; the fp32 kinds the row-reduction kernel (K_REDUCE_MID) serves, with its
    # is_max flag
    REDUCE_KINDS = {"ReduceSum": 0, "ReduceMean": 1, "ReduceProd": 2, "ReduceMax": 3, "ReduceMin": 4}
    REDUCE_MID = {"ReduceMean": 0, "ReduceMax": 1}

    def _reduce(self, node: Node) -> None:
        """K_REDUCE_MID slots: i[0] is_max, i[1] outer, i[2] n, i[3] inner; r[0] x, r[1] y.
        K_REDUCE slots: i[0] kind (sum, mean, prod, max, min), i[1] outer, i[2] n, i[3] inner."""
        x, out = node.input(0), node.output
        xt = x.tensor_type
        axes = list(ops.reduce_axes(node, xt.rank, self._consts(node)))
        if not axes:  # nothing reduced: a copy
            self._copy_value(xt.shape, x, self.ref(out), _strides(xt.shape), 0)
            return
        if axes != list(range(axes[0], axes[0] + len(axes))):
            raise CodegenError(f"{node.op} over non-adjacent axes {axes} has no cuda kernel")
        outer, n, inner = _split_at(xt.shape, axes[0], axes[-1])
        refs = [self.ref(x), self.ref(out)]
        if xt.dtype == "float32" and node.op in self.REDUCE_MID:
            self.emit(K_REDUCE_MID, [self.REDUCE_MID[node.op], outer, n, inner], refs=refs)
        else:
            self.emit(K_REDUCE, [self.REDUCE_KINDS[node.op], outer, n, inner], refs=refs, dtype=DTYPES[xt.dtype])

    def op_ArgMax(self, node: Node) -> None:
        """K_ARGMAX slots: i[0] outer, i[1] n, i[2] inner; dtype of x; r[0] x, r[1] y (int64)."""
        x = node.input(0)
        xt = x.tensor_type
        outer, n, inner = _split_at(xt.shape, _axis_attr(node, xt.rank, 0))
        self.emit(K_ARGMAX, [outer, n, inner], refs=[self.ref(x), self.ref(node.output)],
                  dtype=DTYPES[xt.dtype], count="reduce")

    def _global_pool(self, node: Node, is_max: int) -> None:
        """K_REDUCE_MID slots: i[0] 0 mean, 1 max, 2 mean of the producing GEMM's 32-row partial
        sums (_gap_partials), i[1] outer, i[2] n, i[3] inner; r[0] x, r[1] y."""
        x = node.input(0)
        xt = x.tensor_type
        self._require_f32(node, xt)
        if ops.conv_layout(node) == "NHWC":
            outer, n, inner = xt.shape[0], int(np.prod(xt.shape[1:-1])), xt.shape[-1]
        else:
            outer, n, inner = xt.shape[0] * xt.shape[1], int(np.prod(xt.shape[2:])), 1
        mode = 2 if id(node) in self._gap_from_partials else is_max
        self.emit(K_REDUCE_MID, [mode, outer, n, inner], refs=[self.ref(x), self.ref(node.output)])

    def _gap_partials(self, node: Node) -> Node | None:
        """The GlobalAveragePool whose mean a convolution's epilogue prepares (TF32 mode), or None:
        the convolution's output (NHWC, >= 32 pixels per image, no graph output) is read only by
        that pool, over enough tiles that the GEMM needs no split K. The epilogue then writes, in
        place of the output, the column sums of each 32-row group's rows per image into the
        output's own memory (the pool reads nothing else from it), and the pool adds them
        (reference c.py:1254-1273 reduces the whole output instead)."""
        if self.precision != "tf32" or os.environ.get("MGC_CUDA_GAP_FUSION") == "0":
            return None
        out = node.output
        if len(out.users) != 1 or any(v is out for _, v in self.graph.named_outputs()):
            return None
        gap = out.users[0]
        if gap.op != "GlobalAveragePool" or gap.input(0) is not out or ops.conv_layout(gap) != "NHWC":
            return None
        t = out.tensor_type
        if t.rank != 4 or t.dtype != "float32":
            return None
        nb, oh, ow, c = (int(d) for d in t.shape)
        if oh * ow < 32 or -(-nb * oh * ow // 128) * -(-c // 128) < 148:
            return None
        return gap

    def op_GlobalAveragePool(self, node: Node) -> None:
        self._global_pool(node, 0)

    def op_GlobalMaxPool(self, node: Node) -> None:
        self._global_pool(node, 1)

    # -- softmax, layer norm, batch norm (c.py:823-903) ----------------------------------------------
    def _require_f32(self, node: Node, t: TensorType) -> None:
        if t.dtype != "float32":
            raise CodegenError(f"{node.op} on {t.dtype} has no cuda kernel")

    def _softmax(self, node: Node, log: int) -> None:
        """K_SOFTMAX slots: i[0] outer, i[1] n, i[2] inner, i[3] log, i[4] 1 when the input is the
        elementwise program in aux (see _softmax_reads), read as the rows are; r[0] x, r[1] y."""
        x = node.input(0)
        xt = x.tensor_type
        self._require_f32(node, xt)
        outer, n, inner = _split_at(xt.shape, _axis_attr(node, xt.rank, -1))
        program = self._row_programs.pop(id(x), None)
        self.emit(K_SOFTMAX, [outer, n, inner, log, 0 if program is None else 1],
                  refs=[self.ref(x), self.ref(node.output)], aux=program)

    def op_Softmax(self, node: Node) -> None:
        self._softmax(node, 0)

    def op_LogSoftmax(self, node: Node) -> None:
        self._softmax(node, 1)

    def _vector_ref(self, value: Value | None, n: int, what: str) -> RefT:
        if value is None:
            return NO_REF
        if value.tensor_type.size != n:
            raise CodegenError(f"{what} must have {n} elements, got {value.tensor_type.shape}")
        if value.tensor_type.dtype != "float32":
            raise CodegenError(f"{what} must be float32")
        return self.ref(value)

    def op_LayerNormalization(self, node: Node) -> None:
        """K_LAYER_NORM slots: i[0] rows, i[1] cols; f[0] eps; r[0] x, r[1] scale, r[2] bias, r[3] y."""
        x = node.input(0)
        xt = x.tensor_type
        self._require_f32(node, xt)
        axis = _axis_attr(node, xt.rank, -1)
        rows, cols, _ = _split_at(xt.shape, axis, xt.rank - 1)
        scale = self._vector_ref(node.optional_input(1), cols, "LayerNormalization scale")
        bias = self._vector_ref(node.optional_input(2), cols, "LayerNormalization bias")
        self.emit(K_LAYER_NORM, [rows, cols], [float(node.attrs.get("epsilon", 1e-5))],
                  refs=[self.ref(x), scale, bias, self.ref(node.output)])

    def op_BatchNormalization(self, node: Node) -> None:
        """Inference BatchNormalization as the two-instruction program ``x * mul + add`` with
        mul = gamma / sqrt(var + eps) and add = beta - mean * mul per channel (the channel axis is
        the last one after the layout pass, else axis 1)."""
        x = node.input(0)
        xt = x.tensor_type
        self._require_f32(node, xt)
        consts = [v.data if v is not None else None for v in node.inputs[1:5]]
        if any(c is None for c in consts):
            raise CodegenError("BatchNormalization parameters must be constants")
        gamma, beta, mean, var = (np.asarray(c, np.float64).reshape(-1) for c in consts)
        inv_std = 1.0 / np.sqrt(var + float(node.attrs.get("epsilon", 1e-5)))
        mul = gamma * inv_std
        add = beta - mean * mul
        channel_shape = (mul.size,) if node.attrs.get("layout") == "NHWC" else (mul.size,) + (1,) * (xt.rank - 2)
        # free-standing constant Values (Location "const"), kept alive because blob keys use id()
        g = Graph("bn")
        operands = [g.constant(v.astype(np.float32).reshape(channel_shape), f"bn_{tag}")
                    for tag, v in (("mul", mul), ("add", add))]
        self._keep_alive += operands
        self._elementwise(node.output, [("Mul", {}, [0, 1]), ("Add", {}, [3, 2])], [x, *operands])

    # -- GEMM family (c.py:905-1226) ------------------------------------------------------------------
    def _prec(self) -> int:
        """Arithmetic of the GEMM records of the node being lowered: the model's precision, except
        for an output head in TF32 mode (see _output_heads), which gets the 3xTF32 arithmetic."""
        if self.precision == "tf32" and id(self.graph.nodes[self._node]) in self._heads:
            return PRECISIONS["strict"]
        return PRECISIONS[self.precision]

    def _output_heads(self) -> set[int]:
        """GEMM-family nodes with constant weights whose output is a graph output (directly or
        through views) and whose FLOPs are at most HEAD_FLOP_SHARE of the graph's GEMM FLOPs: a
        classifier or pooler head. TF32 mode computes them with the 3xTF32 arithmetic. The head
        reads the network's largest activations and writes the outputs directly, so the TF32
        rounding of its input dominates the output error (ResNet-50, CPU emulation against the
        float64 oracle: rounding the classifier's input alone gives about 80 % of the logit error
        variance of TF32 mode) at a negligible share of the work (0.05 % of ResNet-50's FLOPs)."""
        gemm_ops = ("FusedGemm", "Gemm", "MatMul", "FusedConv", "Conv")
        nodes = [n for n in self.graph.nodes if n.op in gemm_ops]
        total = sum(ops.flops(n) for n in nodes)
        outputs = {id(self._root(v)) for _, v in self.graph.named_outputs()}
        heads = set()
        for n in nodes:
            b = n.inputs[1] if len(n.inputs) > 1 else None
            if b is None or not (b.is_constant or self.plan.location(b).kind == "const"):
                continue
            if id(n.outputs[0]) in outputs and ops.flops(n) <= HEAD_FLOP_SHARE * total:
                heads.add(id(n))
        return heads

    def _act(self, node: Node) -> tuple[int, float, float]:
        return (
            ACTS[str(node.attrs.get("activation", "none"))],
            float(node.attrs.get("clip_min", 0.0)),
            float(node.attrs.get("clip_max", 6.0)),
        )

    def _kmajor_b(self, matrix_kn: np.ndarray, key: Any) -> tuple[RefT, RefT, int, int]:
        """Store a constant K x N right-hand side K-major ([N][K] rows) as hi + lo parts.
        Returns (hi ref, lo ref, b_rs, b_cs) for element (k, n) at b[k*b_rs + n*b_cs]."""
        k, n = matrix_kn.shape
        if key in self.weights.by_key:
            hi_off = self.weights.by_key[key]
            lo_off = self.weights.by_key[(key, "lo")]
        else:
            kmaj = np.ascontiguousarray(np.asarray(matrix_kn, np.float32).T)
            hi, lo = tf32_split(kmaj)
            hi_off = self.weights.add(hi, key=key)
            lo_off = self.weights.add(lo, key=(key, "lo"))
        return (SPACE_WEIGHTS, 0, hi_off), (SPACE_WEIGHTS, 0, lo_off), 1, k

    @staticmethod
    def _umma_b(bref: RefT, blo: RefT) -> dict[str, RefT]:
        """A constant B stored by ``_kmajor_b`` is already in the tensor-core layout."""
        return {"b_umma": bref, "b_umma_lo": blo} if blo != NO_REF else {}

    def _kmajor_conv_padded(self, w_hwio: np.ndarray, key: Any) -> tuple[RefT, RefT, int]:
        """Tensor-core layout of HWIO convolution weights for im2col loads: [CO][KH][KW][Cp] with
        the channel axis zero-padded to a multiple of 32 (one K block per filter tap and channel
        block). Returns (hi ref, lo ref, Cp)."""
        kh, kw, cg, kg = w_hwio.shape
        cp = (cg + 31) // 32 * 32
        if cp == cg:  # same bytes as the plain K-major layout
            hi, lo, _, _ = self._kmajor_b(w_hwio.reshape(kh * kw * cg, kg), key)
            return hi, lo, cp
        pkey = ("padded", key)
        if pkey not in self.weights.by_key:
            full = np.zeros((kg, kh, kw, cp), np.float32)
            full[:, :, :, :cg] = np.transpose(np.asarray(w_hwio, np.float32), (3, 0, 1, 2))
            hi, lo = tf32_split(full)
            self.weights.add(hi, key=pkey)
            self.weights.add(lo, key=(pkey, "lo"))
        return (SPACE_WEIGHTS, 0, self.weights.by_key[pkey]), (SPACE_WEIGHTS, 0, self.weights.by_key[(pkey, "lo")]), cp

    def _gemm(
        self,
        m: int,
        n: int,
        k: int,
        a: RefT,
        a_rs: int,
        a_cs: int,
        b: RefT,
        b_rs: int,
        b_cs: int,
        c: RefT,
        ldc: int,
        *,
        b_lo: RefT = NO_REF,
        batch: Sequence[int] = (),
        a_bs: Sequence[int] = (),
        b_bs: Sequence[int] = (),
        c_bs: Sequence[int] = (),
        r_bs: Sequence[int] = (),
        conv: dict[str, int] | None = None,
        a_kind: int = STRIDED,
        b_kind: int = STRIDED,
        alpha: float = 1.0,
        beta: float = 1.0,
        bias: RefT = NO_REF,
        bias_mode: int = 0,
        res: RefT = NO_REF,
        ldr: int = 0,
        act: tuple[int, float, float] = (0, 0.0, 6.0),
        b_umma: RefT = NO_REF,
        b_umma_lo: RefT = NO_REF,
        b_cpad: int = 0,
        win_rows: int = 0,
        win_L: int = 0,
        phase_w: int = 0,
        pool: tuple[int, int] = (0, 0),
        gap_hw: int = 0,
    ) -> None:
        """K_GEMM slots: i[0..2] M, N, K; i[3] batch dims; i[4..7] batch extents; i[8..11],
        i[12..15], i[16..19], i[20..23] per-dimension batch strides of A, B, C, residual;
        i[24..26] A kind, row stride, column stride; i[27..40] conv geometry H, W, C, KH, KW, SH,
        SW, DH, DW, PT, PL, OW, c_off, cg; i[41..43] B kind, row stride, column stride; i[44] ldc;
        i[45] bias mode; i[46] ldr; i[47] activation; i[48] precision; i[49] OH.
        i[50] padded channel count of the tensor-core B layout of an im2col convolution (0 when
        B is plain K-major). i[51] output pixels per window-row box and i[52] the padded window-row
        length L when the tensor-core B is laid out [N][KH][L] over a spatially padded image (0
        otherwise). i[53] pixels per phase of a phase-split packed image row (A is such an image
        and B is [N][KH][32] in phase-split tap order; 0 otherwise). i[54], i[55] the rows and
        columns of the 3x3 / stride-2 / pad-1 max pooling computed in a phase-split convolution's
        epilogue (C is then the pooled image; 0 otherwise). i[56] the pixels per image when the
        output only feeds a GlobalAveragePool: C then receives the epilogue's 32-row partial sums
        (_gap_partials; 0 otherwise). i[57] 1 when a constant B may enter as its TF32 part alone
        (one weight plane, _one_plane; the wide CTA-pair forms take it). f[0..3] alpha, beta, clip lo,
        clip hi. r[0] A, r[1] B, r[2] C,
        r[3] bias, r[4] residual, r[5] residual of a split constant B, r[6] / r[7] the
        tensor-core layout of a constant B (TF32-rounded part / residual), absent otherwise."""
        if len(batch) > 4:
            raise CodegenError(f"GEMM with {len(batch)} batch dimensions")
        ints = [0] * 58
        ints[50], ints[51], ints[52], ints[53] = b_cpad, win_rows, win_L, phase_w
        ints[54], ints[55] = pool
        ints[56] = gap_hw
        ints[57] = int(self._one_plane)
        ints[0], ints[1], ints[2], ints[3] = m, n, k, len(batch)
        for d in range(len(batch)):
            ints[4 + d] = batch[d]
            ints[8 + d], ints[12 + d], ints[16 + d] = a_bs[d], b_bs[d], c_bs[d]
            ints[20 + d] = r_bs[d] if r_bs else 0
        ints[24], ints[25], ints[26] = a_kind, a_rs, a_cs
        if conv is not None:
            for j, key in enumerate(("H", "W", "C", "KH", "KW", "SH", "SW", "DH", "DW", "PT", "PL", "OW", "c_off", "cg")):
                ints[27 + j] = conv[key]
            ints[49] = conv["OH"]
        ints[41], ints[42], ints[43] = b_kind, b_rs, b_cs
        ints[44], ints[45], ints[46] = ldc, bias_mode if bias != NO_REF else 0, ldr
        ints[47], ints[48] = act[0], self._prec()
        self.emit(K_GEMM, ints, [alpha, beta, act[1], act[2]], [a, b, c, bias, res, b_lo, b_umma, b_umma_lo],
                  count="gemm")

    def op_FusedGemm(self, node: Node) -> None:
        a, b = node.input(0), node.input(1)
        at, bt = a.tensor_type, b.tensor_type
        self._require_f32(node, at)
        trans = int(node.attrs.get("trans_b", 0))
        k, n = _oriented(bt.shape, trans)
        m = at.size // max(k, 1)  # every leading axis of A is a row (reshape lifting, fusion.py:364-387)
        if b.is_constant or self.plan.location(b).kind == "const":
            data = self.const_data(b)
            bref, blo, b_rs, b_cs = self._kmajor_b(data.T if trans else data, ("kmajor", id(self._root(b)), trans))
        else:
            bref, blo, b_rs, b_cs = self.ref(b), NO_REF, (1 if trans else n), (k if trans else 1)
        bias_v, res_v = node.optional_input(2), node.optional_input(3)
        self._gemm(
            m, n, k, self.ref(a), k, 1, bref, b_rs, b_cs, self.ref(node.output), n, b_lo=blo, **self._umma_b(bref, blo),
            bias=self._vector_ref(bias_v, n, "FusedGemm bias"), bias_mode=1,
            res=self.ref(res_v), ldr=n, act=self._act(node),
        )

    def op_Gemm(self, node: Node) -> None:
        a, b, c = node.input(0), node.input(1), node.optional_input(2)
        at, bt = a.tensor_type, b.tensor_type
        self._require_f32(node, at)
        ta, tb = int(node.attrs.get("transA", 0)), int(node.attrs.get("transB", 0))
        m, k = _oriented(at.shape, ta)
        n = _oriented(bt.shape, tb)[1]
        alpha = float(node.attrs.get("alpha", 1.0))
        beta = float(node.attrs.get("beta", 1.0))
        a_rs, a_cs = (1, m) if ta else (k, 1)
        if b.is_constant or self.plan.location(b).kind == "const":
            data = self.const_data(b)
            bref, blo, b_rs, b_cs = self._kmajor_b(data.T if tb else data, ("kmajor", id(self._root(b)), tb))
        else:
            bref, blo = self.ref(b), NO_REF
            b_rs, b_cs = (1, k) if tb else (n, 1)
        bias, mode, res, ldr = NO_REF, 0, NO_REF, 0
        if c is not None:
            ct = c.tensor_type
            full = np.broadcast_shapes(ct.shape, (m, n))
            cdata = self.const_data(c) if (c.is_constant or self.plan.location(c).kind == "const") else None
            if cdata is not None and ct.size in (1, n) and (ct.rank < 2 or ct.shape[0] == 1):
                vec = np.broadcast_to(cdata.reshape(-1) * beta, (n,)).astype(np.float32)
                bias, mode = self.weights_ref(vec), 1
            elif cdata is not None and ct.rank == 2 and tuple(ct.shape) == (m, 1):
                bias, mode = self.weights_ref((cdata.reshape(-1) * beta).astype(np.float32)), 2
            elif tuple(ct.shape) == (m, n) and full == (m, n):
                res, ldr = self.ref(c), n
            else:
                raise CodegenError(f"Gemm bias of shape {ct.shape} has no cuda lowering")
        self._gemm(m, n, k, self.ref(a), a_rs, a_cs, bref, b_rs, b_cs, self.ref(node.output), n, b_lo=blo, **self._umma_b(bref, blo),
                   alpha=alpha, beta=beta, bias=bias, bias_mode=mode, res=res, ldr=ldr)

    def _view(self, value: Value) -> tuple[RefT, list[int]]:
        """Reference and per-dimension element strides of a MatMul operand: its own contiguous
        buffer, or the source of a Transpose read through."""
        if id(value) in self._through:
            src, strides, base = self._through[id(value)]
            return self.ref(src, base * src.tensor_type.itemsize), list(strides)
        if id(value) in self._stored:
            return self.ref(value), list(self._stored[id(value)])
        return self.ref(value), _strides(value.tensor_type.shape)

    def _write_through(self, node: Node, reads: list[Value] | None = None,
                       mark: bool = True) -> tuple[RefT, int, list[int]] | None:
        """Where a batched MatMul whose only reader is a Transpose keeping the last axis in place
        (attention's (b, h, s, d) -> (b, s, h, d) before the output projection) writes its product
        straight into the Transpose's output, through strides: (reference, row stride, batch
        strides), and the Transpose emits nothing (once ``mark``ed). Only when the Transpose runs
        right after the MatMul and its output memory is clear of everything the MatMul reads
        (``reads``: by default its operands and the sources they are read through)."""
        out = node.output
        rank = out.tensor_type.rank
        if rank < 3 or len(out.users) != 1 or any(v is out for _, v in self.graph.named_outputs()):
            return None
        if node.input(0).tensor_type.rank < 2 or node.input(1).tensor_type.rank < 2:
            return None
        user = out.users[0]
        if user.op != "Transpose" or user.input(0) is not out:
            return None
        perm = ops.transpose_perm(user, rank)
        if perm[-1] != rank - 1 or list(perm) == list(range(rank)):
            return None
        dst = self._arena_range(user.output)
        if dst is None or self.plan.location(user.output).kind != "arena":
            return None
        order = {id(n): k for k, n in enumerate(self.graph.nodes)}
        if any(n.op not in ALIAS_OPS for n in self.graph.nodes[order[id(node)] + 1 : order[id(user)]]):
            return None
        if reads is None:
            reads = [node.input(0), node.input(1)]
            reads += [self._through[id(v)][0] for v in reads if id(v) in self._through]
        for v in reads:
            r = self._arena_range(v)
            if r is not None and r[0] < dst[1] and dst[0] < r[1]:
                return None
        tstrides = _strides(user.output.tensor_type.shape)
        cstrides = [0] * rank
        for j, p in enumerate(perm):
            cstrides[p] = tstrides[j]
        if mark:
            self._written_through.add(id(user))
        return self.ref(user.output), cstrides[-2], cstrides[:-2]

    # -- fused attention ------------------------------------------------------------------------------
    def _score_program(self, enode: Node, scores: Value) -> tuple[int, float, int, Value | None, float] | None:
        """The score program of ``enode`` on ``scores`` in the form the fused attention kernel
        evaluates (attention.cuh score_program; the unfused softmax's ScaleMask form,
        kernels_norm.cuh): t = X * s, s * X or X / s (s an fp32 scalar constant), then optionally
        t + M, M + t or t - M (M an fp32 tensor), Where(C, t, lit) or Where(C, lit, t) (C a bool /
        uint8 tensor, lit an fp32 scalar constant). Returns (div, s, mode, M or C, lit) or None.
        The reference's fusion pass (passes/fusion.py) builds these programs from attention's
        Div / Mul, Add and Where nodes."""
        if enode.op == "FusedElementwise":
            program = [(str(op), [int(x) for x in args]) for op, _, args in enode.attrs["program"]]
        else:
            program = [(enode.op, list(range(len(enode.inputs))))]
        leaves = list(enode.inputs)
        nl = len(leaves)
        if not 1 <= len(program) <= 2 or sum(1 for v in leaves if v is scores) != 1:
            return None

        def scalar(a: int) -> float | None:
            v = leaves[a] if 0 <= a < nl else None
            if v is None or not v.is_constant or v.tensor_type.dtype != "float32" or v.tensor_type.size != 1:
                return None
            return float(np.float32(self.const_data(v).reshape(())))

        def tensor(a: int, dtypes: tuple[str, ...]) -> Value | None:
            v = leaves[a] if 0 <= a < nl else None
            if v is None or v is scores or v.tensor_type.dtype not in dtypes or v.tensor_type.size == 0:
                return None
            if v.is_constant and v.tensor_type.size == 1:
                return None
            return v

        def is_x(a: int) -> bool:
            return 0 <= a < nl and leaves[a] is scores

        op0, a0 = program[0]
        if len(a0) != 2:
            return None
        if op0 == "Mul" and is_x(a0[0]) and scalar(a0[1]) is not None:
            div, scale = 0, scalar(a0[1])
        elif op0 == "Mul" and is_x(a0[1]) and scalar(a0[0]) is not None:
            div, scale = 0, scalar(a0[0])
        elif op0 == "Div" and is_x(a0[0]) and scalar(a0[1]) is not None:
            div, scale = 1, scalar(a0[1])
        else:
            return None
        if len(program) == 1:
            return div, float(scale), ATTN_NONE, None, 0.0  # type: ignore[arg-type]
        op1, a1 = program[1]
        t = nl  # the register of the first instruction's result
        if op1 == "Add" and len(a1) == 2 and t in a1:
            m = tensor(a1[1] if a1[0] == t else a1[0], ("float32",))
            return None if m is None else (div, float(scale), ATTN_ADD, m, 0.0)  # type: ignore[arg-type]
        if op1 == "Sub" and len(a1) == 2 and a1[0] == t:
            m = tensor(a1[1], ("float32",))
            return None if m is None else (div, float(scale), ATTN_SUB, m, 0.0)  # type: ignore[arg-type]
        if op1 == "Where" and len(a1) == 3:
            c = tensor(a1[0], ("bool", "uint8"))
            if c is not None and a1[1] == t and scalar(a1[2]) is not None:
                return div, float(scale), ATTN_KEEP, c, scalar(a1[2])  # type: ignore[return-value]
            if c is not None and a1[2] == t and scalar(a1[1]) is not None:
                return div, float(scale), ATTN_FILL, c, scalar(a1[1])  # type: ignore[return-value]
        return None

    def _attention_plan(self, m1: Node) -> bool:
        """Whether this MatMul starts an attention chain that one K_ATTENTION record computes
        (TF32 mode): MatMul(Q, K^T) -> [score program, _score_program] -> Softmax over the last
        axis -> MatMul(P, V), every intermediate read only by the next node and no graph output,
        the same batch shape throughout, Sk <= 256 and head widths <= 128 (multiples of 4), Q
        and the output with a contiguous head width, K and V with either axis contiguous. The
        record (built now, while the views of Q, K and V are known) is emitted at the second
        MatMul, where its output memory is free; it reads Q, K and the mask later than the
        unfused nodes would, so nothing scheduled in between may write their memory, and its
        output (through the head-merge Transpose when there is one) must lie clear of everything
        it reads."""
        if self.precision != "tf32":
            return False
        a, b = m1.input(0), m1.input(1)
        at, bt = a.tensor_type, b.tensor_type
        if at.rank < 3 or bt.rank != at.rank or at.dtype != "float32" or bt.dtype != "float32":
            return False
        batch = [int(d) for d in at.shape[:-2]]
        if [int(d) for d in bt.shape[:-2]] != batch:
            return False
        outs = {id(v) for _, v in self.graph.named_outputs()}

        def single(v: Value) -> bool:
            return len(v.users) == 1 and id(v) not in outs

        s = m1.output
        if not single(s):
            return False
        nxt = s.users[0]
        div, scale, mode, mask, lit = 0, 1.0, ATTN_NONE, None, 0.0
        enode = None
        if nxt.op != "Softmax":
            if nxt.op != "FusedElementwise" and not ops.is_elementwise(nxt.op):
                return False
            prog = self._score_program(nxt, s)
            e_out = nxt.output
            if prog is None or not single(e_out) or e_out.tensor_type.dtype != "float32" or \
                    tuple(e_out.tensor_type.shape) != tuple(s.tensor_type.shape):
                return False
            div, scale, mode, mask, lit = prog
            enode, nxt = nxt, e_out.users[0]
        sm = nxt
        rank = s.tensor_type.rank
        if sm.op != "Softmax" or _axis_attr(sm, rank, -1) != rank - 1:
            return False
        p = sm.output
        if not single(p):
            return False
        m2 = p.users[0]
        if m2.op != "MatMul" or m2.input(0) is not p or m2.input(1) is p:
            return False
        v = m2.input(1)
        vt = v.tensor_type
        if vt.rank != at.rank or vt.dtype != "float32" or [int(d) for d in vt.shape[:-2]] != batch:
            return False
        sq, dqk = (int(d) for d in at.shape[-2:])
        sk, dv = int(bt.shape[-1]), int(vt.shape[-1])
        if int(bt.shape[-2]) != dqk or int(vt.shape[-2]) != sk or sq < 1 or not _attn_fits(sk, dqk, dv):
            return False
        order = {id(n): k for k, n in enumerate(self.graph.nodes)}
        if v.producer is not None and order.get(id(v.producer), len(order)) > order[id(m1)]:
            return False  # V's view is not known yet
        (qref, qv), (kref, kv), (vref, vv) = self._view(a), self._view(b), self._view(v)
        if qv[-1] != 1:
            return False
        if kv[-2] == 1:
            k_mn, k_rs = 0, kv[-1]
        elif kv[-1] == 1:
            k_mn, k_rs = 1, kv[-2]
        else:
            return False
        if vv[-1] == 1:
            v_mn, v_rs = 1, vv[-2]
        elif vv[-2] == 1:
            v_mn, v_rs = 0, vv[-1]
        else:
            return False

        def source(val: Value) -> Value:
            return self._through[id(val)][0] if id(val) in self._through else val

        sources = [source(a), source(b), source(v)] + ([mask] if mask is not None else [])
        # nothing scheduled between the two MatMuls (the absorbed nodes write nothing) may write
        # what the record reads
        skip = {id(sm)} | ({id(enode)} if enode is not None else set())
        ranges = [r for r in (self._arena_range(x) for x in sources) if r is not None]
        for later in self.graph.nodes[order[id(m1)] + 1 : order[id(m2)]]:
            if later.op in ALIAS_OPS or id(later) in skip:
                continue
            for w in later.outputs:
                r = self._arena_range(w)
                if r is not None and any(r[0] < hi and lo < r[1] for lo, hi in ranges):
                    return False
        through = self._write_through(m2, reads=[], mark=False)
        if through is not None:
            oref, o_rs, o_bs = through
            o_value = m2.output.users[0].output
        else:
            ost = _strides(m2.output.tensor_type.shape)
            oref, o_rs, o_bs = self.ref(m2.output), ost[-2], ost[:-2]
            o_value = m2.output
        dst = self._arena_range(o_value)
        if dst is not None:
            # The output may lie exactly on an operand it replaces element for element (the same
            # reference and strides): each CTA reads its rows of that operand whole before it
            # writes the same bytes, and no other CTA reads them (Q always; K or V only with one
            # query tile, whose rows are then all the keys). Any other overlap is refused.
            one_tile = sq == sk and sq <= 128 and dqk == dv
            same = [(source(a), qref, qv[-2], list(qv[:-2]), dqk == dv),
                    (source(b), kref, k_rs, list(kv[:-2]), one_tile and k_mn == 0),
                    (source(v), vref, v_rs, list(vv[:-2]), one_tile and v_mn == 1)]
            if mask is not None:
                same.append((mask, NO_REF, 0, [], False))
            for val, xref, xrs, xbs, allowed in same:
                r = self._arena_range(val)
                if r is None or not (r[0] < dst[1] and dst[0] < r[1]):
                    continue
                if not (allowed and xref == oref and xrs == o_rs and xbs == list(o_bs)):
                    return False
                if sum(1 for other, *_ in same if other is val) > 1:
                    return False  # another operand read from the same buffer
        if any(ref[2] % 16 for ref in (qref, kref, vref, oref)):
            return False
        m_full = _broadcast_strides(mask.tensor_type.shape, s.tensor_type.shape) if mask is not None \
            else [0] * rank
        dims, (qb, kb, vb, ob, mb) = _collapse(batch, [list(qv[:-2]), list(kv[:-2]), list(vv[:-2]), list(o_bs),
                                                      m_full[:-2]])
        if len(dims) > 2:
            return False
        for st in (qv[-2], k_rs, v_rs, o_rs, *qb, *kb, *vb, *ob):
            if st <= 0 or st % 4:
                return False

        def inner_outer(strides: list[int]) -> tuple[int, int]:
            # (b1, b2): the kernel's inner and outer batch dimensions
            return (strides[-1], strides[0] if len(strides) == 2 else 0) if strides else (0, 0)

        nb1 = dims[-1] if dims else 1
        nb2 = dims[0] if len(dims) == 2 else 1
        ints = [nb1, nb2, sq, sk, dqk, dv,
                qv[-2], *inner_outer(qb),
                k_mn, k_rs, *inner_outer(kb),
                v_mn, v_rs, *inner_outer(vb),
                o_rs, *inner_outer(ob),
                mode, div, DTYPES[mask.tensor_type.dtype] if mask is not None else 0,
                *inner_outer(mb), m_full[-2], m_full[-1]]
        refs = [qref, kref, vref, oref, self.ref(mask) if mask is not None else NO_REF]
        if through is not None:
            self._write_through(m2, reads=[], mark=True)
        self._attn_emit[id(m2)] = (ints, [scale, lit], refs)
        self._attn_skip.update(skip)
        return True

    def _emit_attention(self, node: Node) -> None:
        """K_ATTENTION slots (csrc/launch.cuh): i[0] nb1 (inner batch extent), i[1] nb2 (outer),
        i[2] Sq, i[3] Sk, i[4] Dqk, i[5] Dv; element strides of rows and of the inner / outer
        batch dimension: Q i[6..8]; K i[9] 1 when Sk is its contiguous axis (K^T stored with
        the keys contiguous), i[10..12]; V i[13] 1 when Dv is contiguous, i[14..16]; output
        i[17..19] (Dv contiguous); score program i[20] mask mode (ATTN_*), i[21] 1 for X / s,
        i[22] mask dtype, mask strides i[23] b1, i[24] b2, i[25] query, i[26] key; f[0] s,
        f[1] the Where literal; r[0] Q, r[1] K, r[2] V, r[3] output, r[4] mask."""
        ints, floats, refs = self._attn_emit.pop(id(node))
        self.emit(K_ATTENTION, ints, floats, refs, count="attention")

    def op_MatMul(self, node: Node) -> None:
        if id(node) in self._attn_emit:
            self._emit_attention(node)
            return
        if self._attention_plan(node):
            self.kernels["fused into attention"] = self.kernels.get("fused into attention", 0) + 1
            return
        a, b = node.input(0), node.input(1)
        at, bt = a.tensor_type, b.tensor_type
        self._require_f32(node, at)
        # ONNX MatMul: a 1-D A is one row, a 1-D B one column; leading axes broadcast
        ashape = tuple(at.shape) if at.rank > 1 else (1, *at.shape)
        bshape = tuple(bt.shape) if bt.rank > 1 else (*bt.shape, 1)
        (m, k), n = ashape[-2:], bshape[-1]
        batch_shape = [int(d) for d in np.broadcast_shapes(ashape[:-2], bshape[:-2])]
        aref, av = self._view(a) if at.rank >= 2 else (self.ref(a), [k, 1])
        if bt.rank == 1:
            bref, bv = self.ref(b), [1, 1]
        else:
            bref, bv = self._view(b)
        a_rs, a_cs = av[-2], av[-1]
        b_rs, b_cs = bv[-2], bv[-1]

        def batch_strides(shape: Sequence[int], view: list[int]) -> list[int]:
            # the view's strides of the broadcast batch dimensions (0 where broadcast)
            own = list(shape[:-2])
            lead = len(batch_shape) - len(own)
            out = []
            for d, extent in enumerate(batch_shape):
                j = d - lead
                out.append(0 if j < 0 or own[j] == 1 and extent != 1 else (view[j] if j < len(view) - 2 else 0))
            return out

        a_bs = batch_strides(ashape, av if at.rank >= 2 else [0, 0])
        b_bs = batch_strides(bshape, bv if bt.rank >= 2 else [0, 0])
        c_bs = [s * m * n for s in _strides(batch_shape)]
        ws_used = 0  # workspace bytes of this MatMul's operand copies (from offset 0)
        bconst = b.is_constant or self.plan.location(b).kind == "const"
        if bconst and not any(b_bs) and id(b) not in self._through:
            data = self.const_data(b).reshape(k, n)
            bref, blo, b_rs, b_cs = self._kmajor_b(data, ("kmajor", id(self._root(b)), 0))
        else:
            blo = NO_REF
            if self.precision == "tf32" and b_cs == 1 and b_rs != 1 and bt.rank >= 2 and not (
                    batch_shape and bt.rank == 2):
                # N-major B: one transposed copy into the workspace (K-major, [batch][n][k]) for
                # the tensor-core GEMM with a dynamic B, which reads B rows along K (a rank-2 B
                # broadcast over A's batch stays on the exact-fp32 kernel)
                own = [int(d) for d in bshape[:-2]]
                tshape = [*own, n, k]
                self._copy(tshape, bref, [*bv[:-2], b_cs, b_rs], 0, (SPACE_WORKSPACE, 0, 0), _strides(tshape), 0, 4,
                           count="transpose")
                ws_used = int(np.prod(tshape)) * 4
                self._im2col_bytes = max(self._im2col_bytes, ws_used)
                self._layout_workspace()
                bref, b_rs, b_cs = (SPACE_WORKSPACE, 0, 0), 1, k
                b_bs = batch_strides(bshape, [*_strides(own + [n * k])[:-1], 0, 0] if own else [0, 0])
        cref, ldc = self.ref(node.output), n
        through = self._write_through(node)
        if through is not None:
            cref, ldc, c_bs = through
        # An operand read through a Transpose whose source lies under this GEMM's destination
        # (the planner may reuse the source's memory once the Transpose has run, and the GEMM
        # would overwrite tiles it has yet to read) is first copied into the workspace: B
        # K-major ([batch][n][k]), A row-major ([batch][m][k]).
        dst = self._arena_range(node.output.users[0].output if through is not None else node.output)

        def under_dst(v: Value) -> bool:
            if dst is None or id(v) not in self._through:
                return False
            r = self._arena_range(self._through[id(v)][0])
            return r is not None and r[0] < dst[1] and dst[0] < r[1]

        if bt.rank >= 3 and bref[0] not in (SPACE_WORKSPACE, SPACE_WEIGHTS) and under_dst(b):
            own = [int(d) for d in bshape[:-2]]
            tshape = [*own, n, k]
            off = -(-ws_used // BLOB_ALIGN) * BLOB_ALIGN
            self._copy(tshape, bref, [*bv[:-2], b_cs, b_rs], 0, (SPACE_WORKSPACE, 0, off), _strides(tshape), 0, 4,
                       count="transpose")
            ws_used = off + int(np.prod(tshape)) * 4
            bref, b_rs, b_cs = (SPACE_WORKSPACE, 0, off), 1, k
            b_bs = batch_strides(bshape, [*_strides(own + [n * k])[:-1], 0, 0] if own else [0, 0])
        if at.rank >= 3 and under_dst(a):
            own = [int(d) for d in ashape[:-2]]
            tshape = [*own, m, k]
            off = -(-ws_used // BLOB_ALIGN) * BLOB_ALIGN
            self._copy(tshape, aref, [*av[:-2], a_rs, a_cs], 0, (SPACE_WORKSPACE, 0, off), _strides(tshape), 0, 4,
                       count="transpose")
            ws_used = off + int(np.prod(tshape)) * 4
            aref, a_rs, a_cs = (SPACE_WORKSPACE, 0, off), k, 1
            a_bs = batch_strides(ashape, [*_strides(own + [m * k])[:-1], 0, 0] if own else [0, 0])
        if ws_used > self._im2col_bytes:
            self._im2col_bytes = ws_used
            self._layout_workspace()
        dims, (a_bs, b_bs, c_bs) = _collapse(batch_shape, [a_bs, b_bs, c_bs])
        self._gemm(m, n, k, aref, a_rs, a_cs, bref, b_rs, b_cs, cref, ldc, b_lo=blo,
                   **self._umma_b(bref, blo), batch=dims, a_bs=a_bs, b_bs=b_bs, c_bs=c_bs, r_bs=[0] * len(dims))

    @staticmethod
    def _depthwise(node: Node) -> bool:
        return CEmitter._depthwise(node)

    def op_Conv(self, node: Node) -> None:
        self.op_FusedConv(node)

    def op_FusedConv(self, node: Node) -> None:
        x, w = node.input(0), node.input(1)
        self._require_f32(node, x.tensor_type)
        cs = conv_shape(node)
        if not (w.is_constant or self.plan.location(w).kind == "const"):
            raise CodegenError("convolution weights must be constant for the cuda backend")
        wdata = self.const_data(w)
        bias_v, res_v = node.optional_input(2), node.optional_input(3)
        bias = self._vector_ref(bias_v, cs.cout, "Conv bias")
        res = self.ref(res_v)
        act = self._act(node) if node.op == "FusedConv" else (0, 0.0, 6.0)
        geo = cs.geo()
        nb, h, wd, c, kh, kw, cg, kout, group = cs.n, cs.h, cs.w, cs.c, cs.kh, cs.kw, cs.cg, cs.cout, cs.group
        oh, ow = geo["OH"], geo["OW"]
        nhwc = cs.nhwc
        if self._depthwise(node):
            # K_DEPTHWISE slots: i[0..13] N, H, W, C, KH, KW, SH, SW, DH, DW, PT, PL, OH, OW,
            # i[14] NHWC, i[15] activation; f[0..1] clip bounds; r[0] x, r[1] w, r[2] bias,
            # r[3] residual, r[4] y. Weights HWC (NHWC) or CHW (NCHW), as mgc_depthwise_*.
            wref = self.weights_ref(np.ascontiguousarray(wdata, np.float32), key=("raw", id(self._root(w))))
            ints = [nb, h, wd, c, kh, kw, geo["SH"], geo["SW"], geo["DH"], geo["DW"], geo["PT"], geo["PL"], oh, ow,
                    int(nhwc), act[0]]
            self.emit(K_DEPTHWISE, ints, [act[1], act[2]], [self.ref(x), wref, bias, res, self.ref(node.output)])
            return
        kg = kout // group
        pointwise = cs.pointwise
        if self._tap_packed(node):
            self._conv_tap_packed(node, wdata, geo, nb, bias, res, act)
            return
        if nhwc and group == 1 and not pointwise and cg % 4 and self.precision != "fp32":
            self._conv_via_im2col(node, wdata, geo, nb, bias, res, act)
            return
        for gi in range(group):
            bias_g = bias if bias == NO_REF else (bias[0], bias[1], bias[2] + gi * kg * 4)
            if nhwc:
                wmat = wdata[:, :, :, gi * kg : (gi + 1) * kg].reshape(kh * kw * cg, kg)
                bref, blo, b_rs, b_cs = self._kmajor_b(wmat, ("conv", id(self._root(w)), gi))
                xref = self.ref(x, gi * cg * 4) if pointwise else self.ref(x)
                out_ref = self.ref(node.output, gi * kg * 4)
                res_g = res if res == NO_REF else (res[0], res[1], res[2] + gi * kg * 4)
                if pointwise:
                    umma = self._umma_b(bref, blo)
                elif group == 1:
                    whwio = wdata[:, :, :, gi * kg : (gi + 1) * kg]
                    uhi, ulo, cp = self._kmajor_conv_padded(whwio, ("conv", id(self._root(w)), gi))
                    umma = {"b_umma": uhi, "b_umma_lo": ulo, "b_cpad": cp}
                else:
                    umma = {}
                gap = self._gap_partials(node) if group == 1 and umma else None
                if gap is not None:
                    self._gap_from_partials.add(id(gap))
                self._gemm(
                    nb * oh * ow, kg, kh * kw * cg, xref, c, 1, bref, b_rs, b_cs, out_ref, kout, b_lo=blo,
                    conv={**geo, "c_off": gi * cg, "cg": cg}, a_kind=STRIDED if pointwise else CONV_NHWC,
                    bias=bias_g, bias_mode=1, res=res_g, ldr=kout, act=act, **umma,
                    gap_hw=oh * ow if gap is not None else 0,
                )
            else:
                plane = oh * ow
                amat = np.ascontiguousarray(wdata[gi * kg : (gi + 1) * kg].reshape(kg, cg * kh * kw), np.float32)
                aref = self.weights_ref(amat, key=("convA", id(self._root(w)), gi))
                out_ref = self.ref(node.output, gi * kg * plane * 4)
                res_g = res if res == NO_REF else (res[0], res[1], res[2] + gi * kg * plane * 4)
                self._gemm(
                    kg, plane, cg * kh * kw, aref, cg * kh * kw, 1, self.ref(x), 0, 0, out_ref, plane,
                    batch=[nb], a_bs=[0], b_bs=[c * h * wd], c_bs=[kout * plane],
                    r_bs=[kout * plane], conv={**geo, "c_off": gi * cg, "cg": cg}, b_kind=CONV_NCHW,
                    bias=bias_g, bias_mode=2, res=res_g, ldr=plane, act=act,
                )

    def _conv_via_im2col(self, node: Node, w_hwio: np.ndarray, geo: dict[str, int], nb: int, bias: RefT,
                         res: RefT, act: tuple[int, float, float]) -> None:
        """NHWC convolution whose channel rows are not 16-byte multiples (the 3-channel stem):
        K_IM2COL writes the [pixels, KH*KW*C] patch matrix, zero-padded to a multiple of 32
        columns, into the workspace, and a plain GEMM consumes it.

        K_IM2COL slots: i[0..13] N, H, W, C, KH, KW, SH, SW, DH, DW, PT, PL, OH, OW, i[14] row
        length (padded K), i[15] channel offset, i[16] channels per group; r[0] x, r[1] out."""
        kh, kw, cg, kg = w_hwio.shape
        kreal = kh * kw * cg
        kp = (kreal + 31) // 32 * 32
        m = nb * geo["OH"] * geo["OW"]
        self._im2col_bytes = max(self._im2col_bytes, m * kp * 4)
        self._layout_workspace()
        ws = (SPACE_WORKSPACE, 0, 0)
        ints = [nb, geo["H"], geo["W"], geo["C"], kh, kw, geo["SH"], geo["SW"], geo["DH"], geo["DW"], geo["PT"],
                geo["PL"], geo["OH"], geo["OW"], kp, 0, cg]
        self.emit(K_IM2COL, ints, refs=[self.ref(node.input(0)), ws])
        wmat = np.zeros((kp, kg), np.float32)
        wmat[:kreal] = np.asarray(w_hwio, np.float32).reshape(kreal, kg)
        bref, blo, b_rs, b_cs = self._kmajor_b(wmat, ("im2col", id(self._root(node.input(1)))))
        self._gemm(m, kg, kp, ws, kp, 1, bref, b_rs, b_cs, self.ref(node.output), kg, b_lo=blo,
                   bias=bias, bias_mode=1, res=res, ldr=kg, act=act, **self._umma_b(bref, blo))

    def _im2col_end(self) -> int:
        return (self._im2col_bytes + 255) // 256 * 256

    def _layout_workspace(self) -> None:
        """Workspace layout: the im2col region at offset 0 (shared by every im2col launch, sized
        for the largest), then one region per packed image (each lives from its pack launch to its
        convolution, so none is shared)."""
        packed = sum((size + 255) // 256 * 256 for _, size in self._pack_regions)
        self.workspace_bytes = self._im2col_end() + packed

    def _pack_region(self, nbytes: int) -> RefT:
        """A fresh packed-image region. Its offset is relative to the end of the im2col region,
        whose final size is known only after the last node; the reference carries index
        PACKED_REGION until ``lower`` rebases it."""
        off = sum((size + 255) // 256 * 256 for _, size in self._pack_regions)
        self._pack_regions.append((off, nbytes))
        self._layout_workspace()
        return (SPACE_WORKSPACE, PACKED_REGION, off)

    def _tap_packed(self, node: Node) -> bool:
        """Whether a convolution takes the tap-packed tensor-core path: NHWC, one group, a real
        window (not 1x1 / stride 1 / no padding), fewer than 32 input channels, tensor-core
        precision."""
        if node.op not in ("FusedConv", "Conv") or self.precision == "fp32" or self._depthwise(node):
            return False
        if ops.conv_layout(node) != "NHWC" or int(node.attrs.get("group", 1)) != 1:
            return False
        xt, wt = node.input(0).tensor_type, node.input(1).tensor_type
        if xt.rank != 4 or xt.dtype != "float32":
            return False
        kh, kw, cg, _ = wt.shape
        g = ops.window_geometry(node, (xt.shape[1], xt.shape[2]), (kh, kw))
        pointwise = kh == kw == 1 and g.strides == (1, 1) and g.pads == (0, 0, 0, 0)
        return not pointwise and cg < 32

    def _narrow_plan(self, node: Node) -> dict[str, int]:
        """Input layout of a tap-packed convolution: channels padded to ``cp`` (a multiple of 4)
        and, for the window-row form (unit width dilation, OW a multiple of 8), the image padded
        spatially to Hp x Wp with the convolution's own top / left padding, so that every window
        row is KW * cp contiguous floats inside the image; ``wrows`` output pixels per TMA box,
        ``L`` the window row rounded up to whole 32-float K blocks.

        ``phase`` (TF32 mode, width stride 2, no dilation, at most 4 channels, KW <= 8,
        OW <= 128, KH <= 7, at most 64 output channels: the stems): the image is packed phase-split instead (K_PACK with phases, the
        rows padded to Hp, each row holding its even-tap and odd-tap column phases of ``Wq``
        pixels), so that a filter row's window for output pixel m is pixels m..m+3 of each phase;
        a tile is one output row and reads each filter row's packed input row with one bulk
        copy instead of one TMA row per output pixel."""
        xt, wt = node.input(0).tensor_type, node.input(1).tensor_type
        _, h, w, _ = xt.shape
        kh, kw, cg, _ = wt.shape
        g = ops.window_geometry(node, (h, w), (kh, kw))
        oh, ow = g.out_hw
        pt, pl, _, _ = g.pads
        cp = (cg + 3) // 4 * 4
        wrows = 16 if ow % 16 == 0 else 8 if ow % 8 == 0 else 0
        plan = {"cp": cp, "wrows": 0, "L": 0, "PT": 0, "PL": 0, "Hp": h, "Wp": w, "phase": 0, "Wq": 0}
        hp = max(pt + h, (oh - 1) * g.strides[0] + (kh - 1) * g.dilations[0] + 1)
        if (self.precision == "tf32" and g.strides[1] == 2 and g.dilations == (1, 1) and cp == 4 and kw <= 8
                and ow <= PHASE_TILE_ROWS and wt.shape[3] <= 64 and kh <= PHASE_MAX_KH):
            wq = (ow + 3 + 3) // 4 * 4  # output pixel m reads pixels m .. m + 3 of each phase
            plan.update(phase=1, Wq=wq, PT=pt, PL=pl, Hp=hp, Wp=2 * wq)
            return plan
        if wrows and g.dilations[1] == 1:
            sh, sw = g.strides
            plan.update(wrows=wrows, L=(kw * cp + 31) // 32 * 32, PT=pt, PL=pl, Hp=hp,
                        Wp=max(pl + w, (ow - 1) * sw + kw))
        return plan

    def _emit_pack(self, src: RefT, nb: int, h: int, w: int, c: int, strides: Sequence[int],
                   plan: dict[str, int]) -> RefT:
        """K_PACK slots: i[0..4] N, H, W, C, padded C; i[5..8] source element strides of n, h, w,
        c; i[9..12] PT, PL, padded H, padded W (both phases' pixels of a phase-split row); i[13] 2
        for the phase-split layout, else 0; r[0] source, r[1] packed NHWC destination."""
        cp, hp, wp = plan["cp"], plan["Hp"], plan["Wp"]
        dst = self._pack_region(nb * hp * wp * cp * 4)
        self.emit(K_PACK, [nb, h, w, c, cp, *strides, plan["PT"], plan["PL"], hp, wp, 2 if plan["phase"] else 0],
                  refs=[src, dst])
        return dst

    def _conv_tap_packed(self, node: Node, w_hwio: np.ndarray, geo: dict[str, int], nb: int, bias: RefT,
                         res: RefT, act: tuple[int, float, float]) -> None:
        """Narrow-channel NHWC convolution (C < 32, e.g. the 3-channel stem) on the tensor cores:
        K runs over (kh, kw, channel) with the channels padded only to a multiple of 4, so one
        32-wide K block holds 32 / Cp filter taps. A channel count that is not a multiple of 4 is
        packed first (K_PACK into the workspace; fused into the producing NCHW->NHWC transpose
        when that transpose has no other use)."""
        x = node.input(0)
        kh, kw, cg, kg = w_hwio.shape
        plan = self._narrow_plan(node)
        cp, window = plan["cp"], plan["wrows"] > 0 or plan["phase"] > 0
        if cp == cg and not window:
            xref = self.ref(x)
        elif id(x) in self._packed:
            xref = self._packed[id(x)]
        else:
            xref = self._emit_pack(self.ref(x), nb, geo["H"], geo["W"], cg,
                                   [geo["H"] * geo["W"] * cg, geo["W"] * cg, cg, 1], plan)
        wkey = id(self._root(node.input(1)))
        wpad = np.zeros((kh, kw, cp, kg), np.float32)
        wpad[:, :, :cg, :] = np.asarray(w_hwio, np.float32)
        bref, blo, b_rs, b_cs = self._kmajor_b(wpad.reshape(kh * kw * cp, kg), ("tap-packed", wkey))
        umma = {"b_umma": bref, "b_umma_lo": blo}
        conv = {**geo, "C": cp, "c_off": 0, "cg": cp}
        out_ref = self.ref(node.output)
        if plan["phase"]:
            # the packed image holds the padding; its rows are the two phases of Wq pixels each
            conv.update(H=plan["Hp"], W=plan["Wp"], PT=0, PL=0)
            # tensor-core B as [N][KH][32]: filter row kh's taps kw = 0, 2, 4, 6 (the phase read
            # at pixels m..m+3 of the first half of a packed row), then kw = 1, 3, 5, 7, four
            # channels each, absent taps zero
            rows = np.zeros((kh, 2, 4, cp, kg), np.float32)
            for k_w in range(kw):
                rows[:, k_w % 2, k_w // 2, :, :] = wpad[:, k_w, :, :]
            # one TF32-rounded plane (no residual plane): the stem's weight rounding is a small
            # share of the logit error (CPU emulation of ResNet-50 against the float64 oracle),
            # and its N = 64 MMAs then read a third less shared memory per product
            key = ("phase-rows", wkey)
            if key not in self.weights.by_key:
                self.weights.add(tf32_split(np.ascontiguousarray(rows.reshape(kh * 32, kg).T))[0], key=key)
            umma = {"b_umma": (SPACE_WEIGHTS, 0, self.weights.by_key[key]), "phase_w": plan["Wq"]}
            pool = self._pooled_by(node, res)
            if pool is not None:
                out_ref = self.ref(pool.output)
                umma["pool"] = (geo["OH"] // 2, geo["OW"] // 2)
                self._pool_skip.add(id(pool))
        elif window:
            # the image is read from its padded copy: no padding left for the kernels to apply
            conv.update(H=plan["Hp"], W=plan["Wp"], PT=0, PL=0)
            # tensor-core B as [N][KH][L]: filter row kh's KW * cp weights, zero up to L
            rows = np.zeros((kh, plan["L"], kg), np.float32)
            rows[:, : kw * cp, :] = wpad.reshape(kh, kw * cp, kg)
            uhi, ulo, _, _ = self._kmajor_b(rows.reshape(kh * plan["L"], kg), ("window-rows", wkey))
            umma = {"b_umma": uhi, "b_umma_lo": ulo, "win_rows": plan["wrows"], "win_L": plan["L"]}
        m = nb * geo["OH"] * geo["OW"]
        self._gemm(
            m, kg, kh * kw * cp, xref, cp, 1, bref, b_rs, b_cs, out_ref, kg, b_lo=blo,
            conv=conv, a_kind=CONV_NHWC, bias=bias, bias_mode=1, res=res, ldr=kg, act=act, b_cpad=cp, **umma,
        )

    def _pooled_by(self, node: Node, res: RefT) -> Node | None:
        """The MaxPool that a phase-split convolution computes in its epilogue (the stem's 3x3 /
        stride-2 / pad-1 max pooling: reference c.py:1228-1253 lowers it as its own loop), or None.
        It must be the convolution output's only reader, come next in the schedule (only views
        between), work in NHWC on even output extents, with at most 64 output channels and no
        residual; the convolution's output then never reaches memory. The pooled output's memory is
        written when the convolution runs: nothing else is live there then, since every value live
        at the convolution but not at the pool is one of its inputs, and a phase-split convolution
        reads its image from the workspace copy."""
        out = node.output
        if os.environ.get("MGC_CUDA_POOL_FUSION") == "0":  # the separate MaxPool kernel (measurements)
            return None
        if res != NO_REF or len(out.users) != 1 or any(v is out for _, v in self.graph.named_outputs()):
            return None
        pool = out.users[0]
        if pool.op != "MaxPool" or pool.input(0) is not out or ops.conv_layout(pool) != "NHWC":
            return None
        if len(pool.outputs) > 1 and any(v is not None and (v.users or any(v is o for _, o in self.graph.named_outputs()))
                                         for v in pool.outputs[1:]):
            return None
        nb, oh, ow, c = (int(d) for d in out.tensor_type.shape)
        if c > 64 or oh % 2 or ow % 2 or [int(k) for k in pool.attrs.get("kernel_shape", [])] != [3, 3]:
            return None
        g = ops.window_geometry(pool, (oh, ow), (3, 3), bool(pool.attrs.get("ceil_mode", 0)))
        if tuple(g.strides) != (2, 2) or tuple(g.dilations) != (1, 1) or tuple(g.pads) != (1, 1, 1, 1) or \
                tuple(g.out_hw) != (oh // 2, ow // 2) or int(pool.attrs.get("storage_order", 0)):
            return None
        if tuple(int(d) for d in pool.output.tensor_type.shape) != (nb, oh // 2, ow // 2, c):
            return None
        order = {id(n): k for k, n in enumerate(self.graph.nodes)}
        if any(n.op not in ALIAS_OPS for n in self.graph.nodes[order[id(node)] + 1 : order[id(pool)]]):
            return None
        return pool

    # -- pooling (c.py:1228-1253) ---------------------------------------------------------------------
    def _pool(self, node: Node, is_max: int) -> None:
        """K_POOL slots: i[0] is_max, i[1..17] N, H, W, C, KH, KW, SH, SW, DH, DW, PT, PL, PB, PR,
        OH, OW, count_include_pad, i[18] NHWC; r[0] x, r[1] y."""
        x = node.input(0)
        xt = x.tensor_type
        self._require_f32(node, xt)
        nhwc = ops.conv_layout(node) == "NHWC"
        nb, h, wd, c = xt.shape if nhwc else (xt.shape[0], xt.shape[2], xt.shape[3], xt.shape[1])
        kernel = tuple(int(k) for k in node.attrs["kernel_shape"])
        g = ops.window_geometry(node, (h, wd), (kernel[0], kernel[1]), bool(node.attrs.get("ceil_mode", 0)))
        pt, pl, pb, pr = g.pads
        oh, ow = g.out_hw
        include = int(node.attrs.get("count_include_pad", 0))
        self.emit(K_POOL, [is_max, nb, h, wd, c, kernel[0], kernel[1], g.strides[0], g.strides[1], g.dilations[0],
                           g.dilations[1], pt, pl, pb, pr, oh, ow, include, int(nhwc)],
                  refs=[self.ref(x), self.ref(node.output)])

    def op_MaxPool(self, node: Node) -> None:
        self._pool(node, 1)

    def op_AveragePool(self, node: Node) -> None:
        self._pool(node, 0)

    # -- whole program ----------------------------------------------------------------------------------
    def lower(self) -> LoweredModel:
        for k, node in enumerate(self.graph.nodes):
            self._node = k
            self.node(node)
        self._node = -1
        for value, j in self.plan.copies:
            t = value.tensor_type
            if t.nbytes:
                self.emit(K_MEMCPY, [t.nbytes], refs=[self.ref(value), (SPACE_OUTPUT, j, 0)], count="copy")
        base = self._im2col_end()
        for rec in self.launches:
            for r in rec.r:
                if r.space == SPACE_WORKSPACE and r.index == PACKED_REGION:
                    r.index, r.offset = 0, r.offset + base
        return LoweredModel(
            launches=self.launches,
            aux=np.asarray(self.aux if self.aux else [0], np.int64),
            weights=self.weights,
            arena_bytes=max(self.plan.arena_bytes, 64),
            workspace_bytes=self.workspace_bytes,
            inputs=[(v.name, v.tensor_type) for v in self.graph.inputs],
            outputs=[(name, v.tensor_type) for name, v in self.graph.named_outputs()],
            plan=self.plan,
            kernels=dict(sorted(self.kernels.items())),
            node_names=[(n.op, n.name) for n in self.graph.nodes],
            precision=self.precision,
        )


def lower_graph(
    graph: Graph, strategy: Strategy = "greedy_by_size", inplace: bool = True, precision: str = "tf32"
) -> LoweredModel:
    """Lower an optimised, scheduled graph (nodes in execution order) to a launch list."""
    return CudaEmitter(graph, strategy, inplace, precision).lower()


def algorithmic_cost(graph: Graph) -> tuple[int, int]:
    """(FLOPs, bytes) of one execution: FLOPs = sum of ``ops.flops`` (ops.py:1224-1239); bytes =
    every scheduled node's non-constant inputs and outputs (views excluded) plus each constant
    once."""
    flops = 0
    nbytes = 0
    seen: set[int] = set()
    for node in graph.nodes:
        flops += ops.flops(node)
        if node.op in ALIAS_OPS:
            continue
        for v in node.inputs:
            if v is None:
                continue
            if v.is_constant:
                if id(v) not in seen and v.data is not None:
                    seen.add(id(v))
                    nbytes += v.data.nbytes
            else:
                nbytes += v.tensor_type.nbytes
        nbytes += sum(o.tensor_type.nbytes for o in node.outputs if o.type is not None)
    return flops, nbytes


__all__ = ["CudaEmitter", "Launch", "LoweredModel", "Ref", "algorithmic_cost", "lower_graph", "tf32_split"]


# ---- input-upload overlap -------------------------------------------------------------------------
# A GEMM stays in the sliced prefix only while one slice still has rows for several waves of
# 256-row tiles over all SMs.
SLICE_MIN_ROWS = 2 * 148 * 256


def _slice_fields(rec: Launch, images: int, per: int) -> list[tuple[int, int, int]] | None:
    """(what, slot, per_image) of every batch-dependent field of a record that works image by image
    on batch-major float32 tensors, or None when the record cannot run on a slice of the batch."""
    i, r = rec.i, rec.r
    if rec.dtype != DTYPES["float32"]:
        return None
    if rec.kind == K_PACK:
        if i[0] != images:
            return None
        return [(1, 0, 1), (0, 0, i[5] * 4), (0, 1, i[11] * i[12] * i[4] * 4)]
    if rec.kind == K_POOL:
        if i[1] != images or not i[18]:
            return None
        return [(1, 1, 1), (0, 0, i[2] * i[3] * i[4] * 4), (0, 1, i[15] * i[16] * i[4] * 4)]
    if rec.kind == K_GEMM:
        h, w, c, ow, c_off, cg, oh = i[27], i[28], i[29], i[38], i[39], i[40], i[49]
        if i[3] != 0 or oh <= 0 or ow <= 0 or c_off != 0 or cg != c or i[0] != images * oh * ow:
            return None
        if per * oh * ow < SLICE_MIN_ROWS:
            return None
        if i[24] == STRIDED:  # pointwise convolution: H x W rows of a_rs floats per image
            a_img = h * w * i[25] * 4
        elif i[24] == CONV_NHWC:
            a_img = h * w * c * 4
        else:
            return None
        # C per image: the output image, or the pooled one its epilogue writes
        c_img = (i[54] * i[55] if i[54] > 0 else oh * ow) * i[44] * 4
        out = [(1, 0, oh * ow), (0, 0, a_img), (0, 2, c_img)]
        if r[4].space != SPACE_NONE:
            out.append((0, 4, oh * ow * i[46] * 4))
        return out
    return None


# reference slots each sliceable record kind writes (the others it reads)
_SLICE_WRITES = {K_PACK: (1,), K_POOL: (1,), K_GEMM: (2,)}


def input_slice_plan(lowered: LoweredModel, chunks: int = 4,
                     workspace_base: int | None = None) -> tuple[int, int, list[Chunk], int] | None:
    """(prefix records, images, descriptors, private bytes) for mgc_cuda_set_input_chunks, or None.

    The prefix is the longest run of leading nodes whose records all work image by image on
    batch-major tensors (_slice_fields), cut back until slicing it is safe. Slicing reorders the
    prefix's accesses: slice j runs the whole prefix before slice j + 1 starts. A buffer written in
    the prefix and read only inside it is consumed within its own slice's pass, so the planner's
    reuse of memory stays valid there. A buffer that the rest of the graph reads must survive the
    later slices' passes: no other prefix buffer may share its memory unless both have the same
    start and bytes per image (then every slice keeps to its own range). When the other buffer is
    read only inside the prefix, it moves instead to a private region of one slice's size after
    the workspace (``workspace_base``, the lowered workspace's bytes by default): every reference
    of the prefix to it is repointed there (descriptor ``what`` 2), the same for every slice. The
    private bytes are what the workspace must grow by."""
    if len(lowered.inputs) != 1:
        return None
    shape = lowered.inputs[0][1].shape
    if len(shape) < 2 or shape[0] < chunks or shape[0] % chunks:
        return None
    images = int(shape[0])
    per = images // chunks
    recs = lowered.launches
    base = lowered.workspace_bytes if workspace_base is None else workspace_base
    base = -(-base // BLOB_ALIGN) * BLOB_ALIGN
    # the longest sliceable run of whole nodes
    fields: list[list[tuple[int, int, int]]] = []
    end, k = 0, 0
    while k < len(recs):
        j = k
        while j < len(recs) and recs[j].node == recs[k].node:
            j += 1
        fs = [_slice_fields(recs[n], images, per) for n in range(k, j)]
        if any(f is None for f in fs):
            break
        fields += fs
        end, k = j, j
    tracked = (SPACE_ARENA, SPACE_OUTPUT, SPACE_WORKSPACE)
    moved: dict[tuple[int, int], tuple[int, int, int]] = {}  # (record, slot) -> (ws offset, lo, per image)
    while end > 0:
        moved = {}
        # buffers the prefix writes: (space, index, start, end, bytes per image, record, slot)
        writes = []
        for n in range(end):
            per_image = {slot: b for what, slot, b in fields[n] if what == 0}
            for slot in _SLICE_WRITES[recs[n].kind]:
                ref = recs[n].r[slot]
                if ref.space not in tracked:
                    return None
                writes.append((ref.space, ref.index, ref.offset, ref.offset + per_image[slot] * images,
                               per_image[slot], n, slot))
        suffix_refs = [(recs[n].r[t].space, recs[n].r[t].index, recs[n].r[t].offset)
                       for n in range(end, len(recs)) for t in range(len(recs[n].r))]

        def last_writer(sp: int, ix: int, o: int, before: int) -> tuple | None:
            """The prefix write that memory (sp, ix, o) holds before record `before`."""
            owner = None
            for w2 in writes:
                if w2[5] < before and (w2[0], w2[1]) == (sp, ix) and w2[2] <= o < w2[3]:
                    if owner is None or w2[5] > owner[5]:
                        owner = w2
            return owner

        def escapes(w: tuple) -> bool:
            """Whether the rest of the graph may read buffer w: a graph output, or memory of w's
            that no later prefix write covers and a later record refers to."""
            sp, ix, lo, hi = w[:4]
            return sp == SPACE_OUTPUT or any(s2 == sp and i2 == ix and lo <= o < hi and last_writer(sp, ix, o, end) is w
                                             for s2, i2, o in suffix_refs)

        def readers(w: tuple) -> list[tuple[int, int]] | None:
            """(record, slot) of every prefix reference to buffer w, or None when one may not be
            moved: a reference to w's memory is w's when w is its last writer before it."""
            sp, ix, lo, hi, pi, n0, _ = w
            out = []
            for r in range(n0 + 1, end):
                per_image = {slot: b for what, slot, b in fields[r] if what == 0}
                for t in range(len(recs[r].r)):
                    ref = recs[r].r[t]
                    if (ref.space, ref.index) != (sp, ix) or not lo <= ref.offset < hi or t in _SLICE_WRITES[recs[r].kind]:
                        continue
                    if last_writer(sp, ix, ref.offset, r) is not w:
                        continue
                    if t not in per_image or per_image[t] != pi or ref.offset - lo >= pi:
                        return None  # not read image by image like it was written
                    out.append((r, t))
            return out

        # conflicts: an escaping buffer and another prefix buffer over the same memory with a
        # different layout; the other moves when only the prefix reads it, else the prefix ends
        cut = None
        relocate: dict[int, tuple] = {}
        for x in writes:
            if not escapes(x):
                continue
            for y in writes:
                if y is x or (y[0], y[1]) != (x[0], x[1]) or not (y[2] < x[3] and x[2] < y[3]) or (y[2], y[4]) == (x[2], x[4]):
                    continue
                if not escapes(y) and y[0] != SPACE_OUTPUT and readers(y) is not None:
                    relocate[y[5] * 16 + y[6]] = y
                    continue
                later = max(x[5], y[5])
                cut = later if cut is None else min(cut, later)
        if cut is not None:
            node = recs[cut].node
            while cut > 0 and recs[cut - 1].node == node:
                cut -= 1
            end = cut
            fields = fields[:end]
            continue
        off = base
        for y in relocate.values():
            moved[(y[5], y[6])] = (off, y[2], y[4])
            for r, t in readers(y) or []:
                moved[(r, t)] = (off + recs[r].r[t].offset - y[2], y[2], y[4])
            off = -(-(off + y[4] * per) // BLOB_ALIGN) * BLOB_ALIGN
        break
    if end == 0 or not any(recs[n].kind == K_GEMM for n in range(end)):
        return None
    descs = []
    for n in range(end):
        for what, slot, b in fields[n]:
            if what == 0 and (n, slot) in moved:
                descs.append(Chunk(n, 2, slot, 0, moved[(n, slot)][0]))
            else:
                descs.append(Chunk(n, what, slot, 0, b))
    private = (max((o + per * pi for o, _, pi in moved.values()), default=base) - base) if moved else 0
    return end, images, descs, -(-private // BLOB_ALIGN) * BLOB_ALIGN
