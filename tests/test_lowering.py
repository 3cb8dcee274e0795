"""Host-side lowering: the launch list follows the reference planner and C emitter exactly."""

from __future__ import annotations

import numpy as np
import pytest

import cases
from mgc_cuda import lowering, zoo
from mgc_cuda.lowering import K_GEMM, K_PACK, CudaEmitter, lower_graph, tf32_split
from ml_graph_compiler.codegen.c import generate_c
from ml_graph_compiler.errors import CodegenError
from ml_graph_compiler.ir import Graph, TensorType
from ml_graph_compiler.passes import optimize
from ml_graph_compiler.schedule import schedule
from ml_graph_compiler.shape_inference import infer_shapes


def o3(g: Graph) -> Graph:
    optimize(g, "O3")
    schedule(g)
    return g


@pytest.fixture(scope="module")
def r50() -> Graph:
    return o3(zoo.resnet50(batch=1))


def test_resnet50_o3_matches_published_structure(r50: Graph) -> None:
    """58 nodes; kernels gemm 54 / pool 1 / reduce 1 / transpose 1 / view 1; arena 7,225,344 B
    (reference benchmarks/results/ablation_cnn.json, cumulative loopfuse for resnet50)."""
    assert len(r50.nodes) == 58
    low = lower_graph(r50, precision="fp32")
    assert low.kernels == {"gemm": 54, "pool": 1, "reduce": 1, "transpose": 1, "view": 1}
    assert low.arena_bytes == 7_225_344
    assert len(low.launches) == 57
    assert low.workspace_bytes == 0
    # in TF32 mode the input transpose writes the image phase-split into the workspace: 229 rows
    # (3 of top padding; the last window row ends at row 2 * 111 + 7), each holding the even-tap
    # and the odd-tap column phases of 116 four-channel pixels (output pixel m reads pixels
    # m..m+3 of each), TF32-rounded; the stem reads one packed row per filter row (B laid out
    # [64][7][32] in that tap order) and computes the 3x3 / stride-2 MaxPool in its epilogue,
    # writing the pooled 56 x 56 image where the MaxPool's output lives
    tc = lower_graph(r50, precision="tf32")
    assert tc.kernels == {"gemm": 54, "pack": 1, "pool fused into convolution": 1, "reduce": 1, "view": 1}
    assert tc.arena_bytes == 7_225_344
    assert tc.workspace_bytes == (229 * 232 * 4 * 4 + 255) // 256 * 256
    pack, stem = tc.launches[0], tc.launches[1]
    assert pack.kind == K_PACK
    assert list(pack.i[:14]) == [1, 224, 224, 3, 4, 3 * 224 * 224, 224, 1, 224 * 224, 3, 3, 229, 232, 2]
    assert stem.kind == K_GEMM and stem.i[2] == 7 * 7 * 4 and list(stem.i[50:56]) == [4, 0, 0, 116, 56, 56]
    pool = next(n for n in r50.nodes if n.op == "MaxPool")
    assert (stem.r[2].space, stem.r[2].offset) == (lowering.SPACE_ARENA, CudaEmitter(r50, "greedy_by_size", True,
                                                   "tf32").plan.location(pool.output).index)
    assert not any(r.kind == lowering.K_POOL for r in tc.launches)
    assert (stem.i[27], stem.i[28], stem.i[29], stem.i[36], stem.i[37]) == (229, 232, 4, 0, 0)
    assert (stem.r[0].space, stem.r[0].offset) == (pack.r[1].space, pack.r[1].offset)
    # strict mode keeps the window-row form: the image with its channels padded to 4 and its
    # 3-pixel border (229 x 229), window rows of 32 floats per filter row
    st = lower_graph(r50, precision="strict")
    pack, stem = st.launches[0], st.launches[1]
    assert list(pack.i[:14]) == [1, 224, 224, 3, 4, 3 * 224 * 224, 224, 1, 224 * 224, 3, 3, 229, 229, 0]
    assert list(stem.i[50:56]) == [4, 16, 32, 0, 0, 0]  # strict: MaxPool stays a kernel of its own
    assert sum(r.kind == lowering.K_POOL for r in st.launches) == 1
    assert (stem.i[27], stem.i[28], stem.i[29], stem.i[36], stem.i[37]) == (229, 229, 4, 0, 0)


def test_workspace_regions_do_not_overlap() -> None:
    """Two channel packs (one fused into the input transpose, one in the middle of the network)
    get disjoint regions inside the workspace."""
    c = [c for c in cases.all_cases() if c.name == "pattern_narrow_convs"][0]
    g, _ = cases.prepare(c)
    low = lower_graph(g, precision="tf32")
    assert low.kernels["pack"] == 2 and "im2col" not in low.kernels
    regions = sorted((r.i[0] * r.i[1] * r.i[2] * r.i[4] * 4, r.r[1].offset) for r in low.launches if r.kind == K_PACK)
    spans = sorted((off, off + size) for size, off in regions)
    assert all(a[1] <= b[0] for a, b in zip(spans, spans[1:]))
    assert spans[-1][1] <= low.workspace_bytes
    assert all(r.r[1].index == 0 for r in low.launches if r.kind == K_PACK)


def test_same_kernel_mix_and_arena_as_the_c_backend() -> None:
    """The same arena and kernel mix as the reference's C backend; in TF32 mode each fused
    attention record stands for two of its GEMMs and its softmax, and a MaxPool computed in its
    convolution's epilogue for that pool."""
    for make in (lambda: zoo.tiny_cnn(batch=2), lambda: zoo.tiny_transformer(kind="gpt"), zoo.mlp):
        g = o3(make())
        theirs = generate_c(g)
        for precision in ("strict", "tf32"):
            ours = lower_graph(g, precision=precision)
            assert ours.arena_bytes == max(theirs.arena_bytes, 64)
            fused = ours.kernels.get("attention", 0)
            assert fused == 0 or precision == "tf32"
            pooled = ours.kernels.get("pool fused into convolution", 0)
            assert pooled == 0 or precision == "tf32"
            for kind in ("gemm", "depthwise", "pool", "softmax", "layer_norm", "gather"):
                per = {"gemm": 2, "softmax": 1}.get(kind, 0)
                extra = pooled if kind == "pool" else 0
                assert ours.kernels.get(kind, 0) + per * fused + extra == theirs.kernels.get(kind, 0), kind


def test_every_arena_reference_stays_inside_the_arena(r50: Graph) -> None:
    low = lower_graph(r50)
    for rec in low.launches:
        for ref in rec.r:
            if ref.space == lowering.SPACE_ARENA:
                assert 0 <= ref.offset < low.arena_bytes
            if ref.space == lowering.SPACE_WEIGHTS:
                assert 0 <= ref.offset < low.weights.nbytes
                assert ref.offset % 4 == 0


def test_conv_launches_use_nhwc_implicit_gemm(r50: Graph) -> None:
    low = lower_graph(r50, precision="fp32")
    gemms = [r for r in low.launches if r.kind == lowering.K_GEMM]
    kinds = {int(r.i[24]) for r in gemms}
    assert kinds == {lowering.STRIDED, lowering.CONV_NHWC}
    stem = gemms[0]
    assert (stem.i[30], stem.i[31], stem.i[32]) == (7, 7, 2)  # KH, KW, SH
    assert stem.i[0] == 112 * 112 and stem.i[1] == 64 and stem.i[2] == 7 * 7 * 3
    fc = gemms[-1]
    assert (fc.i[0], fc.i[1], fc.i[2]) == (1, 1000, 2048)


def test_tf32_split_is_exact() -> None:
    rng = np.random.default_rng(0)
    a = (rng.standard_normal(10_000) * 10.0 ** rng.integers(-8, 8, 10_000)).astype(np.float32)
    a[:4] = [0.0, -0.0, np.inf, -np.inf]
    hi, lo = tf32_split(a)
    assert np.all((hi.view(np.uint32) & 0x1FFF) == 0)
    np.testing.assert_array_equal(hi + lo, a)
    finite = np.isfinite(a) & (a != 0)
    assert np.all(np.abs(lo[finite]) <= np.abs(a[finite]) * 2.0**-11)


def test_unsupported_operator_is_a_compile_error() -> None:
    g = Graph("bad")
    x = g.add_input("x", TensorType("float32", (2, 3)))
    g.add_output(g.add_node("Trilu", [x]).output, "y")
    infer_shapes(g)
    with pytest.raises(CodegenError, match="no kernel"):
        CudaEmitter(g)


def test_float16_is_rejected() -> None:
    g = Graph("half")
    x = g.add_input("x", TensorType("float16", (2, 3)))
    g.add_output(g.add_node("Relu", [x]).output, "y")
    infer_shapes(g)
    with pytest.raises(CodegenError, match="float16"):
        CudaEmitter(g)


@pytest.mark.parametrize("case", cases.all_cases(), ids=[c.name for c in cases.all_cases()])
def test_every_case_lowers(case: cases.Case) -> None:
    g, _ = cases.prepare(case)
    low = lower_graph(g, precision="strict")
    assert low.launches or all(n.op in lowering.ALIAS_OPS for n in g.nodes)
    assert all(lowering.K_GEMM <= r.kind <= lowering.K_PACK for r in low.launches)


def test_algorithmic_cost_of_resnet50(r50: Graph) -> None:
    flops, nbytes = lowering.algorithmic_cost(r50)
    assert abs(flops / 1e9 - 8.178) < 0.01
    assert 200e6 < nbytes < 230e6



def test_tensor_core_b_planes_are_ordered(r50: Graph) -> None:
    """The kernel loads B's TF32 part and residual as the two planes of one 3-D tensor map, which
    needs the residual stored after the TF32 part at a 16-byte multiple. A phase-split stem
    (i[53] > 0, TF32 mode) reads one TF32-rounded plane and has no residual."""
    for precision in ("tf32", "strict"):
        low = lower_graph(r50, precision=precision)
        single = 0
        for rec in low.launches:
            if rec.kind == lowering.K_GEMM and rec.r[6].space == lowering.SPACE_WEIGHTS:
                if rec.i[53] > 0:
                    assert precision == "tf32" and rec.r[7].space == lowering.SPACE_NONE
                    single += 1
                    continue
                gap = rec.r[7].offset - rec.r[6].offset
                assert gap > 0 and gap % 16 == 0
        assert single == (1 if precision == "tf32" else 0)


def _sliced_writes_keep_escaping_buffers(low, plan) -> int:
    """Replay the sliced order of the prefix symbolically: every buffer the rest of the graph reads
    (the last prefix write of memory a later record refers to) keeps, for every slice, what that
    slice wrote: no write after it in the sliced order (later records of its slice, or any record
    of a later slice) touches that slice's part of it. Returns how many slice parts were checked."""
    prefix, images, descs, _ = plan
    slices = 4
    per = images // slices
    by = {}
    for d in descs:
        by.setdefault((d.launch, d.slot), []).append(d)
    fields = [lowering._slice_fields(low.launches[n], images, per) for n in range(prefix)]

    def write_range(n: int, slot: int, j: int):
        ref = low.launches[n].r[slot]
        pi = next(b for what, sl, b in fields[n] if what == 0 and sl == slot)
        ds = by.get((n, slot), [])
        if any(d.what == 2 for d in ds):
            off = next(d.per_image for d in ds if d.what == 2)
            return (lowering.SPACE_WORKSPACE, 0, off, off + per * pi)
        return (ref.space, ref.index, ref.offset + j * per * pi, ref.offset + (j + 1) * per * pi)

    order = [(j, n, slot) for j in range(slices) for n in range(prefix)
             for slot in lowering._SLICE_WRITES[low.launches[n].kind]]
    unsliced = [(n, slot) for n in range(prefix) for slot in lowering._SLICE_WRITES[low.launches[n].kind]]
    moved = {key for key, ds in by.items() if any(d.what == 2 for d in ds)}

    def orig(n: int, slot: int):  # the buffer in the planner's memory (the one-pass graph)
        ref = low.launches[n].r[slot]
        pi = next(b for what, sl, b in fields[n] if what == 0 and sl == slot)
        return ref.space, ref.index, ref.offset, ref.offset + images * pi

    suffix = [(r.space, r.index, r.offset) for rec in low.launches[prefix:] for r in rec.r]
    checked = 0
    for s2, i2, o in suffix:
        covering = [w for w in unsliced if orig(*w)[:2] == (s2, i2) and orig(*w)[2] <= o < orig(*w)[3]]
        if not covering:
            continue
        n, slot = max(covering)  # the buffer the rest of the graph reads there
        assert (n, slot) not in moved, f"record {n}'s output is read after the prefix but was moved"
        for j in range(slices):
            mine = write_range(n, slot, j)
            at = order.index((j, n, slot))
            for j2, n2, slot2 in order[at + 1:]:
                other = write_range(n2, slot2, j2)
                assert not (other[:2] == mine[:2] and other[2] < mine[3] and mine[2] < other[3]), \
                    f"slice {j2} record {n2} overwrites slice {j}'s part of record {n}'s output"
            checked += 1
    return checked


@pytest.mark.parametrize("strategy,records,moved", [("greedy_by_size", 12, 4), ("naive", 13, 0)])
def test_input_slice_plan_of_resnet50(strategy: str, records: int, moved: int) -> None:
    """The sliced prefix at batch 256: pack, the stem with its pooling, layer1 and (naive) the
    first layer2 convolution, up to the first GEMM whose slice has too few rows. Under the default
    plan layer1's 64-channel buffers share memory with the 256-channel block outputs the rest of
    the graph reads; read only inside the prefix, they move to private regions of one slice each
    (4 x 64 images x 56 x 56 x 64 floats), and the symbolic replay of the sliced order finds every
    escaping buffer intact."""
    g = o3(zoo.resnet50(batch=256))
    low = lower_graph(g, strategy, True, "tf32")
    plan = lowering.input_slice_plan(low, 4)
    assert plan is not None
    prefix, images, descs, private = plan
    assert (prefix, images) == (records, 256)
    writers = {(d.launch, d.slot) for d in descs if d.what == 2 and d.slot in lowering._SLICE_WRITES[low.launches[d.launch].kind]}
    assert len(writers) == moved
    assert private == moved * 64 * 56 * 56 * 64 * 4
    assert all(d.per_image >= -(-low.workspace_bytes // 256) * 256 for d in descs if d.what == 2)
    stem = low.launches[1]
    assert stem.kind == K_GEMM and low.launches[0].kind == K_PACK
    fields = {(d.what, d.slot): d.per_image for d in descs if d.launch == 1}
    # M = images * 112 * 112; A = the phase-split image (229 rows of 2 x 116 four-channel
    # pixels); C = the pooled image, 56 * 56 * 64 floats (greedy: in a private region)
    assert fields[(1, 0)] == 112 * 112 and fields[(0, 0)] == 229 * 232 * 4 * 4
    assert fields.get((0, 2)) == (None if moved else 56 * 56 * 64 * 4)
    assert all(d.launch < prefix for d in descs)
    assert _sliced_writes_keep_escaping_buffers(low, plan) > 0
    if moved:
        # the same prefix without the moves: later slices overwrite block outputs the rest of the
        # graph reads (what the check exists to catch)
        per = images // 4
        plain = []
        for d in descs:
            if d.what == 2:
                pi = next(b for what, sl, b in lowering._slice_fields(low.launches[d.launch], images, per)
                          if what == 0 and sl == d.slot)
                d = lowering.Chunk(d.launch, 0, d.slot, 0, pi)
            plain.append(d)
        with pytest.raises(AssertionError, match="overwrites"):
            _sliced_writes_keep_escaping_buffers(low, (prefix, images, plain, 0))


@pytest.mark.parametrize("batch,precision,fused", [(256, "tf32", True), (1, "tf32", False), (256, "strict", False)])
def test_global_average_pool_from_partials(batch: int, precision: str, fused: bool) -> None:
    """TF32 ResNet-50 at a batch with enough tiles: the last convolution's record carries the
    pixels per image (49) and the pool adds its epilogue's partial sums (K_REDUCE_MID mode 2) from
    the convolution's own output memory; batch 1 (a split-K GEMM) and strict mode keep the pool."""
    low = lower_graph(o3(zoo.resnet50(batch=batch)), "greedy_by_size", True, precision)
    red = [r for r in low.launches if r.kind == lowering.K_REDUCE_MID]
    gap = [r for r in low.launches if r.kind == K_GEMM and r.i[56] > 0]
    assert len(red) == 1 and red[0].i[0] == (2 if fused else 0)
    if fused:
        assert len(gap) == 1 and gap[0].i[56] == 49 and (gap[0].i[0], gap[0].i[1]) == (batch * 49, 2048)
        assert (gap[0].r[2].space, gap[0].r[2].offset) == (red[0].r[0].space, red[0].r[0].offset)
    else:
        assert not gap


def test_input_slice_plan_needs_a_batch() -> None:
    low = lower_graph(o3(zoo.resnet50(batch=1)), "greedy_by_size", True, "tf32")
    assert lowering.input_slice_plan(low, 4) is None


@pytest.mark.parametrize("name", ["bert", "gpt2"])
def test_attention_scale_and_mask_run_inside_the_softmax(name: str) -> None:
    """Strict mode (no fused attention): every layer's score scale + mask program (BERT: additive
    fp32 mask; GPT-2: causal bool mask through Where) is evaluated by the softmax that reads it:
    no K_ELEMENTWISE record for it, and one K_SOFTMAX record per layer carrying the program."""
    g = getattr(zoo, name)(batch=2, seq=128)
    optimize(g, "O3")
    schedule(g)
    low = lower_graph(g, precision="strict")
    assert low.kernels.get("elementwise into softmax") == 12
    assert "attention" not in low.kernels
    soft = [r for r in low.launches if r.kind == lowering.K_SOFTMAX]
    assert len(soft) == 12 and all(r.i[4] == 1 and r.aux_len > 0 for r in soft)


def _attn_spans(rec) -> dict[str, tuple[int, int, tuple]]:
    """Arena byte range and layout (offset, row stride, batch strides) of each operand of a
    K_ATTENTION record (slots documented at CudaEmitter._emit_attention)."""
    i = [int(x) for x in rec.i[:27]]
    nb1, nb2, sq, sk, dqk, dv = i[:6]
    batch = [(nb1, i[7]), (nb2, i[8])]
    shapes = {
        "q": (0, [(sq, i[6]), (dqk, 1), (nb1, i[7]), (nb2, i[8])], 4),
        "k": (1, [(dqk if i[9] else sk, i[10]), (sk if i[9] else dqk, 1), (nb1, i[11]), (nb2, i[12])], 4),
        "v": (2, [(sk if i[13] else dv, i[14]), (dv if i[13] else sk, 1), (nb1, i[15]), (nb2, i[16])], 4),
        "o": (3, [(sq, i[17]), (dv, 1), (nb1, i[18]), (nb2, i[19])], 4),
        "mask": (4, [(nb1, i[23]), (nb2, i[24]), (sq, i[25]), (sk, i[26])], 1 if i[22] in (5, 6) else 4),
    }
    del batch
    out = {}
    for name, (slot, dims, esize) in shapes.items():
        if rec.r[slot].space != lowering.SPACE_ARENA:
            continue
        last = sum((e - 1) * abs(st) for e, st in dims)
        lo = rec.r[slot].offset
        out[name] = (lo, lo + (last + 1) * esize, (lo, dims[0][1], dims[2][1], dims[3][1]))
    return out


@pytest.mark.parametrize("name,batch", [("bert", 2), ("gpt2", 2), ("tiny_transformer", 3)])
@pytest.mark.parametrize("strategy", ["greedy_by_size", "naive"])
def test_attention_is_one_record_per_layer_in_tf32(name: str, batch: int, strategy: str) -> None:
    """TF32 mode: each layer's MatMul(Q, K^T) -> scale / mask -> Softmax -> MatMul(P, V) is one
    K_ATTENTION record (no softmax, no score GEMMs), and its output lies clear of every operand
    it reads, or exactly on Q, K or V with their layout (each CTA reads its rows of that operand
    before it writes the same bytes)."""
    kw = {"seq": 128} if name != "tiny_transformer" else {}
    g = getattr(zoo, name)(batch=batch, **kw)
    optimize(g, "O3")
    schedule(g)
    low = lower_graph(g, precision="tf32", strategy=strategy)
    layers = 2 if name == "tiny_transformer" else 12
    att = [r for r in low.launches if r.kind == lowering.K_ATTENTION]
    assert len(att) == layers and "softmax" not in low.kernels
    assert low.kernels.get("fused into attention") == 3 * layers  # Q K^T, score program, softmax
    for rec in att:
        spans = _attn_spans(rec)
        o = spans.get("o")
        if o is None:
            continue
        for which in ("q", "k", "v", "mask"):
            r = spans.get(which)
            if r is None or not (r[0] < o[1] and o[0] < r[1]):
                continue
            assert which != "mask" and r[2] == o[2], f"attention of node {rec.node} writes over its {which}"
            if which != "q":
                assert rec.i[2] <= 128  # one query tile


def test_attention_record_slots_of_bert_and_gpt2() -> None:
    """The record of BERT's layer (Q, K, V read through the projections' [b, s, h * d] outputs,
    the output written through the head merge, scores * 0.125 + the fp32 mask [b, 1, 1, s]) and
    of GPT-2's (Q, K, V read through the fused QKV output's [b, s, 3 * h * d] rows, the causal
    mask as Where(upper, fmin, t) over a bool [1, 1, s, s] constant)."""
    got = {}
    for name in ("bert", "gpt2"):
        g = getattr(zoo, name)(batch=2, seq=128)
        optimize(g, "O3")
        schedule(g)
        low = lower_graph(g, precision="tf32", strategy="naive")
        got[name] = next(r for r in low.launches if r.kind == lowering.K_ATTENTION)
    bert, gpt2 = got["bert"], got["gpt2"]
    seq = 128 * 768
    assert list(bert.i[:27]) == [12, 2, 128, 128, 64, 64, 768, 64, seq, 0, 768, 64, seq, 1, 768, 64, seq,
                                 768, 64, seq, lowering.ATTN_ADD, 0, 0, 0, 128, 0, 1]
    assert list(bert.f[:2]) == [0.125, 0.0]
    row = 3 * 768
    assert list(gpt2.i[:27]) == [12, 2, 128, 128, 64, 64, row, 64, 128 * row, 0, row, 64, 128 * row, 1, row, 64,
                                 128 * row, 768, 64, seq, lowering.ATTN_FILL, 0, 6, 0, 0, 128, 1]
    assert gpt2.f[0] == 0.125 and gpt2.f[1] == float(np.finfo(np.float32).min)
    # Q, K and V: column offsets 0, 768 and 1536 of the same rows
    assert gpt2.r[1].offset - gpt2.r[0].offset == 768 * 4 and gpt2.r[2].offset - gpt2.r[1].offset == 768 * 4


def test_attention_stays_unfused_where_the_kernel_does_not_apply() -> None:
    """Strict and fp32 modes keep the unfused nodes (their products are exact-fp32 or 3xTF32); so
    do rows longer than the kernel's 256 keys."""
    for precision in ("strict", "fp32"):
        g = o3(zoo.tiny_transformer(batch=2))
        assert "attention" not in lower_graph(g, precision=precision).kernels
    g = o3(zoo.tiny_transformer(batch=1, seq=320))
    low = lower_graph(g, precision="tf32")
    assert "attention" not in low.kernels and low.kernels.get("softmax") == 2


def _gemm_span(rec, which: str) -> tuple[int, int] | None:
    """Arena byte range a K_GEMM record's strided operand touches (None: not in the arena)."""
    i = rec.i
    slot = {"a": 0, "b": 1, "c": 2}[which]
    if rec.r[slot].space != lowering.SPACE_ARENA:
        return None
    nb = i[3]
    dims = [i[4 + d] for d in range(nb)]
    if which == "a":
        if i[24] != lowering.STRIDED:
            return None
        bs, extents = [i[8 + d] for d in range(nb)], [(i[0], i[25]), (i[2], i[26])]
    elif which == "b":
        if i[41] != lowering.STRIDED:
            return None
        bs, extents = [i[12 + d] for d in range(nb)], [(i[2], i[42]), (i[1], i[43])]
    else:
        bs, extents = [i[16 + d] for d in range(nb)], [(i[0], i[44]), (i[1], 1)]
    last = sum((e - 1) * abs(s) for e, s in zip(dims, bs)) + sum((e - 1) * abs(s) for e, s in extents)
    lo = rec.r[slot].offset
    return lo, lo + (last + 1) * 4


@pytest.mark.parametrize("name", ["bert", "gpt2"])
@pytest.mark.parametrize("precision", ["tf32", "strict"])
@pytest.mark.parametrize("strategy", ["greedy_by_size", "naive"])
def test_no_gemm_writes_over_an_operand_it_reads(name: str, precision: str, strategy: str) -> None:
    """A GEMM that reads an operand through strides (a Transpose read through) must not write
    over that operand's memory: the planner may reuse a Transpose's source once the Transpose
    has run, so the lowering copies such an operand into the workspace first."""
    g = getattr(zoo, name)(batch=2, seq=128)
    optimize(g, "O3")
    schedule(g)
    low = lower_graph(g, precision=precision, strategy=strategy)
    checked = 0
    for rec in low.launches:
        if rec.kind != K_GEMM:
            continue
        c = _gemm_span(rec, "c")
        for which in ("a", "b"):
            r = _gemm_span(rec, which)
            if c is None or r is None:
                continue
            checked += 1
            assert not (r[0] < c[1] and c[0] < r[1]), f"GEMM of node {rec.node} writes over its {which} operand"
    assert checked > 0


def test_gpt2_split_outputs_are_views_on_the_naive_plan() -> None:
    """GPT-2's fused QKV output is split into Q, K and V, each read only by head Transposes: with
    every buffer in its own memory the Split copies nothing (the Transposes read the QKV buffer
    through strides); with the greedy plan, whose later buffers reuse that memory, each layer's
    Split copies its three outputs in one split-mode copy record (one pass over the QKV rows), and
    every head Transpose still reads its copy through strides: K's Transpose, scheduled between
    Q's and Q's MatMul, has its planned output over Q's copy but is itself read through, so it
    writes nothing there."""
    g = zoo.gpt2(batch=2, seq=128)
    optimize(g, "O3")
    schedule(g)
    naive = lower_graph(g, strategy="naive")
    assert "copy" not in naive.kernels and "split" not in naive.kernels
    greedy = lower_graph(g)
    assert greedy.kernels.get("split") == 12 and "copy" not in greedy.kernels and "transpose" not in greedy.kernels
    splits = [r for r in greedy.launches if r.kind == lowering.K_COPY and r.i[28] == 2]
    assert len(splits) == 12
    for rec in splits:
        assert rec.i[29] == 3 and list(rec.i[30:33]) == [768, 768, 768] and rec.i[34] == 2 * 128


def test_weight_plane_policy(monkeypatch: pytest.MonkeyPatch) -> None:
    """TF32 mode marks the GEMM records of a graph without convolutions (slot i[57]) so that the
    tile forms may take the weights as their TF32 part alone; graphs with convolutions keep exact
    weights, as do strict mode and MGC_CUDA_WEIGHT_PLANES=2."""
    def flags(g: Graph, precision: str) -> set[int]:
        return {int(r.i[57]) for r in lower_graph(g, precision=precision).launches if r.kind == K_GEMM}

    gpt = o3(zoo.tiny_transformer(kind="gpt"))
    cnn = o3(zoo.tiny_cnn(batch=2))
    assert flags(gpt, "tf32") == {1}
    assert flags(gpt, "strict") == {0}
    assert flags(cnn, "tf32") == {0}
    monkeypatch.setenv("MGC_CUDA_WEIGHT_PLANES", "2")
    assert flags(gpt, "tf32") == {0}
