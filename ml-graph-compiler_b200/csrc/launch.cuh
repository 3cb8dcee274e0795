// Decoding of mgc_cuda_launch records (built by mgc_cuda/lowering.py) into kernel parameters,
// and the dispatch of one record onto a stream. The slot layout of every kind is documented at
// the matching `_emit_*` function of the lowering; the two must stay in step.
#pragma once

#include <vector>

#include "common.cuh"
#include "gemm_simt.cuh"
#include "attention.cuh"
#include "gemm_umma.cuh"
#include "kernels_mem.cuh"
#include "kernels_norm.cuh"
#include "depthwise.cuh"

namespace mgc {

// Device base addresses the references of a launch list resolve against.
struct Bases {
    char *arena = nullptr;
    char *weights = nullptr;
    char *workspace = nullptr;
    const std::vector<char *> *inputs = nullptr;
    const std::vector<char *> *outputs = nullptr;
    // split-K scratch of a model (none for raw-pointer calls)
    float *split_ws = nullptr;
    long long split_ws_floats = 0;
};

inline int resolve(const mgc_cuda_ref &r, const Bases &b, void **out) {
    switch (r.space) {
    case MGC_SPACE_NONE: *out = nullptr; return MGC_CUDA_OK;
    case MGC_SPACE_RAW: *out = (void *)(uintptr_t)r.offset; return MGC_CUDA_OK;
    case MGC_SPACE_ARENA:
        if (!b.arena) break;
        *out = b.arena + r.offset;
        return MGC_CUDA_OK;
    case MGC_SPACE_WEIGHTS:
        if (!b.weights) break;
        *out = b.weights + r.offset;
        return MGC_CUDA_OK;
    case MGC_SPACE_WORKSPACE:
        if (!b.workspace) break;
        *out = b.workspace + r.offset;
        return MGC_CUDA_OK;
    case MGC_SPACE_INPUT:
        if (!b.inputs || r.index < 0 || r.index >= (int)b.inputs->size()) break;
        *out = (*b.inputs)[r.index] + r.offset;
        return MGC_CUDA_OK;
    case MGC_SPACE_OUTPUT:
        if (!b.outputs || r.index < 0 || r.index >= (int)b.outputs->size()) break;
        *out = (*b.outputs)[r.index] + r.offset;
        return MGC_CUDA_OK;
    default: break;
    }
    return fail(MGC_CUDA_BAD_ARGUMENT, "reference space %d (index %d) cannot be resolved here",
                r.space, r.index);
}

#define MGC_RESOLVE(ref, ptr)                                                                \
    do {                                                                                     \
        void *mgc_p_ = nullptr;                                                              \
        MGC_CHECK(resolve((ref), bases, &mgc_p_));                                           \
        (ptr) = (decltype(ptr))mgc_p_;                                                       \
    } while (0)

// What one launch record did: how many kernels it launched and, for a GEMM-family record, which
// kernel computed it (MGC_CUDA_PATH_*, reported per record by mgc_cuda_gemm_paths).
struct LaunchInfo {
    int kernels = 0;
    int gemm_path = MGC_CUDA_PATH_NONE;
};

// Run every GEMM-family launch of the model ABI: the tcgen05 kernel when it accepts the problem,
// else the exact-fp32 SIMT kernel; `info` records which (and the split-K reduce's extra launch).
inline int run_gemm(const GemmParams &p, cudaStream_t stream, LaunchInfo *info = nullptr) {
    int taken = 0;
    MGC_CHECK(try_gemm_umma(p, stream, &taken));
    if (info) {
        info->kernels = taken > 0 ? taken : 1;
        info->gemm_path = taken > 0 ? MGC_CUDA_PATH_TCGEN05 : MGC_CUDA_PATH_SIMT;
    }
    if (taken) return MGC_CUDA_OK;
    if (p.phase_w > 0 || p.pool_ph > 0 || p.gap_hw > 0)  // a phase-split packed image is no NHWC
                                                         // operand for the exact-fp32 kernel, which
                                                         // has no pooling epilogues either
        return fail(MGC_CUDA_UNSUPPORTED, "gemm: the tensor-core kernel declined a phase-split convolution "
                                          "(M %d, N %d, OW %d, pooled %d x %d)", p.M, p.N, p.OW, p.pool_ph, p.pool_pw);
    return launch_gemm_simt(p, stream);
}

inline int decode_gemm(const mgc_cuda_launch &L, const Bases &bases, GemmParams &p) {
    const int64_t *i = L.i;
    p = GemmParams{};
    p.M = (int)i[0]; p.N = (int)i[1]; p.K = (int)i[2];
    p.nb = (int)i[3];
    if (p.nb < 0 || p.nb > 4) return fail(MGC_CUDA_BAD_ARGUMENT, "gemm: %d batch dims", p.nb);
    for (int d = 0; d < 4; ++d) {
        p.bdims[d] = i[4 + d];
        p.a_bs[d] = i[8 + d]; p.b_bs[d] = i[12 + d]; p.c_bs[d] = i[16 + d]; p.r_bs[d] = i[20 + d];
    }
    p.a_kind = (int)i[24]; p.a_rs = i[25]; p.a_cs = i[26];
    p.H = (int)i[27]; p.W = (int)i[28]; p.C = (int)i[29]; p.KH = (int)i[30]; p.KW = (int)i[31];
    p.SH = (int)i[32]; p.SW = (int)i[33]; p.DH = (int)i[34]; p.DW = (int)i[35];
    p.PT = (int)i[36]; p.PL = (int)i[37]; p.OW = (int)i[38]; p.c_off = (int)i[39]; p.cg = (int)i[40];
    p.b_kind = (int)i[41]; p.b_rs = i[42]; p.b_cs = i[43];
    p.ldc = i[44]; p.bias_mode = (int)i[45]; p.ldr = i[46]; p.act = (int)i[47];
    p.precision = (int)i[48]; p.OH = (int)i[49];
    p.alpha = (float)L.f[0]; p.beta = (float)L.f[1]; p.lo = (float)L.f[2]; p.hi = (float)L.f[3];
    MGC_RESOLVE(L.r[0], p.a);
    MGC_RESOLVE(L.r[1], p.b);
    MGC_RESOLVE(L.r[2], p.c);
    MGC_RESOLVE(L.r[3], p.bias);
    MGC_RESOLVE(L.r[4], p.res);
    MGC_RESOLVE(L.r[5], p.b_lo);
    MGC_RESOLVE(L.r[6], p.b_umma);
    MGC_RESOLVE(L.r[7], p.b_umma_lo);
    p.b_cpad = (int)i[50];
    p.win_rows = (int)i[51]; p.win_L = (int)i[52];
    p.phase_w = (int)i[53];
    p.pool_ph = (int)i[54]; p.pool_pw = (int)i[55];
    p.gap_hw = (int)i[56];
    p.one_plane = (int)i[57];
    if (!p.a || !p.b || !p.c) return fail(MGC_CUDA_BAD_ARGUMENT, "gemm: missing operand");
    return MGC_CUDA_OK;
}

inline int decode_elementwise(const mgc_cuda_launch &L, const int64_t *aux, int64_t aux_len,
                              const Bases &bases, EwParams &P) {
    int64_t pos = L.aux_offset, end = L.aux_offset + L.aux_len;
    if (pos < 0 || end > aux_len) return fail(MGC_CUDA_BAD_ARGUMENT, "elementwise: aux out of range");
    auto next = [&](int64_t &v) -> bool {
        if (pos >= end) return false;
        v = aux[pos++];
        return true;
    };
    int64_t v = 0;
    memset(&P, 0, sizeof P);
    if (!next(v) || v < 0 || v > EW_MAX_RANK) return fail(MGC_CUDA_UNSUPPORTED, "elementwise: rank %lld", (long long)v);
    P.rank = (int)v;
    P.total = 1;
    for (int d = 0; d < P.rank; ++d) {
        if (!next(v)) return fail(MGC_CUDA_BAD_ARGUMENT, "elementwise: truncated shape");
        P.shape[d] = v;
        P.total *= v;
    }
    int64_t sp, ix, off;
    if (!next(v)) return fail(MGC_CUDA_BAD_ARGUMENT, "elementwise: truncated");
    P.out_dt = (int)v;
    if (!next(sp) || !next(ix) || !next(off)) return fail(MGC_CUDA_BAD_ARGUMENT, "elementwise: truncated");
    mgc_cuda_ref oref{(int32_t)sp, (int32_t)ix, off};
    MGC_RESOLVE(oref, P.out);
    if (!next(v) || v < 0 || v > EW_MAX_LEAVES)
        return fail(MGC_CUDA_UNSUPPORTED, "elementwise: %lld leaves (max %d)", (long long)v, EW_MAX_LEAVES);
    P.nleaves = (int)v;
    P.contiguous = P.rank <= 1 ? 1 : 0;
    for (int l = 0; l < P.nleaves; ++l) {
        EwLeaf &lf = P.leaves[l];
        int64_t dt, lit, bits;
        if (!next(dt) || !next(lit) || !next(bits) || !next(sp) || !next(ix) || !next(off))
            return fail(MGC_CUDA_BAD_ARGUMENT, "elementwise: truncated leaf");
        lf.dtype = (int)dt;
        lf.is_lit = (int)lit;
        P.cls[l] = class_of(lf.dtype);
        if (lf.is_lit) {
            double d;
            memcpy(&d, &bits, sizeof d);
            if (lf.dtype == MGC_F32) lf.lit.f = (float)d;
            else if (lf.dtype == MGC_F64) lf.lit.d = d;
            else lf.lit.i = bits;
        } else {
            mgc_cuda_ref r{(int32_t)sp, (int32_t)ix, off};
            MGC_RESOLVE(r, lf.p);
        }
        for (int d = 0; d < P.rank; ++d) {
            if (!next(v)) return fail(MGC_CUDA_BAD_ARGUMENT, "elementwise: truncated strides");
            lf.strides[d] = v;
            if (!lf.is_lit && P.rank == 1 && v != 0 && v != 1) P.contiguous = 0;
        }
        if (P.rank == 0) lf.strides[0] = 0;
    }
    if (!next(v) || v < 1 || v > EW_MAX_INSTR)
        return fail(MGC_CUDA_UNSUPPORTED, "elementwise: %lld instructions (max %d)", (long long)v, EW_MAX_INSTR);
    P.ninstr = (int)v;
    for (int k = 0; k < P.ninstr; ++k) {
        EwInstr &in = P.ins[k];
        int64_t op, odt, a0, a1, a2, b0, b1;
        if (!next(op) || !next(odt) || !next(a0) || !next(a1) || !next(a2) || !next(b0) || !next(b1))
            return fail(MGC_CUDA_BAD_ARGUMENT, "elementwise: truncated instruction");
        if (op < 0 || op >= EW_NUM_OPS) return fail(MGC_CUDA_UNSUPPORTED, "elementwise: op %lld", (long long)op);
        const int64_t lim = P.nleaves + k;
        if (a0 < 0 || a0 >= lim || a1 >= lim || a2 >= lim)
            return fail(MGC_CUDA_BAD_ARGUMENT, "elementwise: instruction %d reads a later register", k);
        in.op = (int16_t)op; in.out_dt = (int16_t)odt;
        in.a[0] = (int16_t)a0; in.a[1] = (int16_t)a1; in.a[2] = (int16_t)a2;
        memcpy(&in.imm[0], &b0, sizeof(double));
        memcpy(&in.imm[1], &b1, sizeof(double));
        P.cls[P.nleaves + k] = class_of(in.out_dt);
    }
    if (P.rank == 0) P.shape[0] = 1;
    return MGC_CUDA_OK;
}

template <typename T>
inline int launch_copy_t(const CopyParams &P, cudaStream_t s) {
    // Vectorised, 32-bit form: the innermost dimension contiguous on both sides, its extent,
    // every stride and both bases multiples of 16 bytes, both pointers 16-byte aligned, and every
    // index (in elements) below 2^31.
    const int r = P.rank;
    const long long v = 16 / (long long)sizeof(T);
    bool vec = r >= 1 && P.sstr[r - 1] == 1 && P.dstr[r - 1] == 1 && P.shape[r - 1] % v == 0 &&
               P.sbase % v == 0 && P.dbase % v == 0 && (reinterpret_cast<uintptr_t>(P.src) & 15) == 0 &&
               (reinterpret_cast<uintptr_t>(P.dst) & 15) == 0;
    long long smax = P.sbase, dmax = P.dbase;
    for (int k = 0; k < r && vec; ++k) {
        if (k < r - 1 && (P.sstr[k] % v || P.dstr[k] % v)) vec = false;
        smax += (P.shape[k] - 1) * (P.sstr[k] < 0 ? 0 : P.sstr[k]);
        dmax += (P.shape[k] - 1) * (P.dstr[k] < 0 ? 0 : P.dstr[k]);
        if (P.sstr[k] < 0 || P.dstr[k] < 0) vec = false;
    }
    if (vec && P.total < (1ll << 31) && smax < (1ll << 31) && dmax < (1ll << 31)) {
        CopyParams Q = P;
        Q.shape[r - 1] = P.shape[r - 1] / v;
        for (int k = 0; k < r - 1; ++k) { Q.sstr[k] = P.sstr[k] / v; Q.dstr[k] = P.dstr[k] / v; }
        Q.sbase = P.sbase / v; Q.dbase = P.dbase / v;
        Q.total = P.total / v;
        copy_vec_kernel<uint4><<<grid_for(Q.total, 256), 256, 0, s>>>(Q);
        return check_launch("copy_vec_kernel");
    }
    // Tiled transpose: the destination contiguous along the last dimension, the source along
    // another one, both extents at least 16 (narrower ones waste most of a 32 x 32 tile).
    if (r >= 2 && P.dstr[r - 1] == 1 && P.sstr[r - 1] != 1 && P.shape[r - 1] >= 16) {
        int jj = -1;
        for (int k = 0; k < r - 1; ++k)
            if (P.sstr[k] == 1 && P.shape[k] >= 16) jj = k;
        bool fits = true;
        long long smax = P.sbase, dmax = P.dbase;
        for (int k = 0; k < r; ++k) {
            fits = fits && P.sstr[k] >= 0 && P.dstr[k] >= 0;
            smax += (P.shape[k] - 1) * P.sstr[k];
            dmax += (P.shape[k] - 1) * P.dstr[k];
        }
        const long long nbatch = jj >= 0 ? P.total / (P.shape[r - 1] * P.shape[jj]) : 0;
        const long long tiles = nbatch * ((P.shape[r - 1] + 31) / 32) * (jj >= 0 ? (P.shape[jj] + 31) / 32 : 0);
        if (jj >= 0 && fits && smax < (1ll << 31) && dmax < (1ll << 31) && tiles < (1ll << 31)) {
            transpose_tile_kernel<T><<<grid_for(tiles, 1), 256, 0, s>>>(P, jj, (unsigned)nbatch);
            return check_launch("transpose_tile_kernel");
        }
    }
    copy_kernel<T><<<grid_for(P.total, 256), 256, 0, s>>>(P);
    return check_launch("copy_kernel");
}

// Depthwise convolution in shared-memory tiles (depthwise_nhwc4_tile_kernel): one block per
// (image, row tile, column tile, channel chunk).
template <int S, int CG>
inline int launch_dw_tile(const DepthwiseParams &p, cudaStream_t s) {
    using T = DwTile<S, CG>;
    const unsigned row_tiles = (unsigned)ceil_div(p.OH, T::TH), col_tiles = (unsigned)ceil_div(p.OW, T::TW);
    const unsigned chunks = (unsigned)(p.C / 4 / CG);
    const long long blocks = (long long)p.N * row_tiles * col_tiles * chunks;
    if (blocks >= (1ll << 31)) return fail(MGC_CUDA_UNSUPPORTED, "depthwise: %lld tiles", blocks);
    MGC_CHECK(raise_smem_ceiling((const void *)depthwise_nhwc4_tile_kernel<S, CG>));
    depthwise_nhwc4_tile_kernel<S, CG><<<(unsigned)blocks, 256, T::SMEM, s>>>(p, row_tiles, col_tiles, chunks);
    return check_launch("depthwise_nhwc4_tile_kernel");
}

// Depthwise convolution in row bands (depthwise.cuh). The block shape: the divisor `cg` of the
// C / VEC channel vectors (at most 32) whose column tiles of at most 256 / cg columns (and at most
// `max_tw`) leave the fewest warp lanes idle (ties: the larger cg, so that a block reads longer
// pieces of each pixel); then the band height that minimises (waves of blocks) x (input rows per
// block + `fill` rows of fixed cost per block), waves counted with the kernel's occupancy at
// `smem_per_vec` bytes of shared memory per input column and channel vector plus `smem_extra`.
inline int dw_band_shape(const DepthwiseParams &p, int vec, int S, const void *kernel, int fill, int max_tw,
                         unsigned smem_per_vec, unsigned smem_extra, DwBand &t, unsigned &smem) {
    const int cv = p.C / vec;
    t = DwBand{};
    double best = -1.0;
    for (int cg = cv < 32 ? cv : 32; cg >= 1; --cg) {
        if (cv % cg) continue;
        const int wmax = 256 / cg < max_tw ? 256 / cg : max_tw;
        const int tiles = (int)ceil_div(p.OW, wmax);
        const int tw = (int)ceil_div(p.OW, tiles);
        const double eff = (double)p.OW * cg / ((double)tiles * ceil_div(tw * cg, 32) * 32);
        if (eff > best + 1e-9) {
            best = eff;
            t.cg = cg;
            t.tw = tw;
            t.tiles = (unsigned)tiles;
        }
    }
    t.chunks = (unsigned)(cv / t.cg);
    const int threads = t.tw * t.cg;
    smem = smem_per_vec * (unsigned)(((t.tw - 1) * S + 3) * t.cg) + smem_extra;
    MGC_CHECK(raise_smem_ceiling(kernel));
    int per_sm = 0;
    MGC_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem));
    int dev = 0, sms = 148;
    MGC_CHECK_CUDA(cudaGetDevice(&dev));
    MGC_CHECK_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const long long slots = (long long)sms * (per_sm > 0 ? per_sm : 1);
    const long long per_band = (long long)p.N * t.tiles * t.chunks;
    long long best_cost = -1;
    for (int bh = 1; bh <= p.OH; ++bh) {
        const long long bands = ceil_div(p.OH, bh);
        const long long waves = ceil_div(per_band * bands, slots);
        const long long cost = waves * ((long long)(bh - 1) * S + 3 + fill);
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            t.bh = bh;
            t.bands = (unsigned)bands;
        }
    }
    if (per_band * t.bands >= (1ll << 31)) return fail(MGC_CUDA_UNSUPPORTED, "depthwise: %lld bands", per_band * t.bands);
    return MGC_CUDA_OK;
}

// Ring slots of the band forms: 5 rows in flight (4 and 10 measured slower on MobileNetV2's layers).
constexpr int DW_SLOTS = 6;

template <int S, int VEC, int D = DW_SLOTS>
inline int launch_dw_ring(const DepthwiseParams &p, cudaStream_t s) {
    DwBand t;
    unsigned smem = 0;
    const void *k = (const void *)depthwise_ring_kernel<S, VEC, D>;
    MGC_CHECK(dw_band_shape(p, VEC, S, k, D, 256, D * VEC * 4, 0, t, smem));
    const long long blocks = (long long)p.N * t.tiles * t.chunks * t.bands;
    depthwise_ring_kernel<S, VEC, D><<<(unsigned)blocks, t.tw * t.cg, smem, s>>>(p, t);
    return check_launch("depthwise_ring_kernel");
}

// The TMA form: a 4-D map of the input (channels, columns, rows, images) with boxes of one band
// row (cg * 4 channels x (tw - 1) * S + 3 columns); out-of-range boxes read zeros.
template <int S, int ACT, int D = DW_SLOTS>
inline int launch_dw_tma_act(const DepthwiseParams &p, cudaStream_t s) {
    DwBand t;
    unsigned smem = 0;
    const void *k = (const void *)depthwise_tma_kernel<S, D, ACT>;
    // each slot rounded up to 128 bytes, D barriers, 128 bytes of alignment slack
    MGC_CHECK(dw_band_shape(p, 4, S, k, D, (256 - 3) / S + 1, D * 16, D * (128 + 8) + 128, t, smem));
    auto fn = umma::encode_tiled_fn();
    if (!fn) return fail(MGC_CUDA_UNSUPPORTED, "depthwise: no cuTensorMapEncodeTiled");
    CUtensorMap map;
    const cuuint64_t dims[4] = {(cuuint64_t)p.C, (cuuint64_t)p.W, (cuuint64_t)p.H, (cuuint64_t)p.N};
    const cuuint64_t strides[3] = {(cuuint64_t)p.C * 4, (cuuint64_t)p.W * p.C * 4, (cuuint64_t)p.H * p.W * p.C * 4};
    const cuuint32_t box[4] = {(cuuint32_t)(t.cg * 4), (cuuint32_t)((t.tw - 1) * S + 3), 1, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float *>(p.x), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MGC_CUDA_UNSUPPORTED, "depthwise: tensor map (%d)", (int)r);
    const long long blocks = (long long)p.N * t.tiles * t.chunks * t.bands;
    depthwise_tma_kernel<S, D, ACT><<<(unsigned)blocks, t.tw * t.cg, smem, s>>>(p, t, map);
    return check_launch("depthwise_tma_kernel");
}

// The TMA band form with the activation resolved at compile time for none, ReLU and Clip.
template <int S>
inline int launch_dw_tma(const DepthwiseParams &p, cudaStream_t s) {
    switch (p.act) {
    case MGC_ACT_NONE: return launch_dw_tma_act<S, DW_NONE>(p, s);
    case MGC_ACT_RELU: return launch_dw_tma_act<S, DW_RELU>(p, s);
    case MGC_ACT_CLIP: return launch_dw_tma_act<S, DW_CLIP>(p, s);
    default: return launch_dw_tma_act<S, DW_ANY>(p, s);
    }
}

template <typename T>
inline int launch_tile_t(const TileParams &P, cudaStream_t s) {
    tile_kernel<T><<<grid_for(P.total, 256), 256, 0, s>>>(P);
    return check_launch("tile_kernel");
}

// Launch one record. `info`, if not NULL, receives the number of kernel launches and the GEMM
// path taken.
inline int launch_record(const mgc_cuda_launch &L, const int64_t *aux, int64_t aux_len,
                         const Bases &bases, int *status_dev, cudaStream_t stream, LaunchInfo *info) {
    const int64_t *i = L.i;
    int launched = 1;
    int st = MGC_CUDA_OK;
    LaunchInfo gemm;
    switch (L.kind) {
    case MGC_K_GEMM: {
        GemmParams p;
        MGC_CHECK(decode_gemm(L, bases, p));
        p.err = status_dev;
        p.split_ws = bases.split_ws;
        p.split_ws_floats = bases.split_ws_floats;
        st = run_gemm(p, stream, &gemm);
        launched = gemm.kernels;
        break;
    }
    case MGC_K_DEPTHWISE: {
        DepthwiseParams p{};
        p.N = (int)i[0]; p.H = (int)i[1]; p.W = (int)i[2]; p.C = (int)i[3]; p.KH = (int)i[4];
        p.KW = (int)i[5]; p.SH = (int)i[6]; p.SW = (int)i[7]; p.DH = (int)i[8]; p.DW = (int)i[9];
        p.PT = (int)i[10]; p.PL = (int)i[11]; p.OH = (int)i[12]; p.OW = (int)i[13];
        p.nhwc = (int)i[14]; p.act = (int)i[15];
        p.lo = (float)L.f[0]; p.hi = (float)L.f[1];
        MGC_RESOLVE(L.r[0], p.x); MGC_RESOLVE(L.r[1], p.w); MGC_RESOLVE(L.r[2], p.bias);
        MGC_RESOLVE(L.r[3], p.res); MGC_RESOLVE(L.r[4], p.y);
        p.err = status_dev;
        const long long total = (long long)p.N * p.OH * p.OW * p.C;
        if (total == 0) { launched = 0; break; }
        const bool vec4 = p.nhwc && p.C % 4 == 0 &&
                          ((((uintptr_t)p.x) | ((uintptr_t)p.w) | ((uintptr_t)p.y) |
                            ((uintptr_t)p.bias) | ((uintptr_t)p.res)) % 16 == 0);
        const int c4 = p.C / 4;
        const bool reg = vec4 && p.KH <= 3 && p.KW <= 3 && c4 <= 256 &&
                         (long long)p.N * p.H * p.W * c4 < (1ll << 31) && total / 4 < (1ll << 31);
        const uintptr_t any_ptr = ((uintptr_t)p.x) | ((uintptr_t)p.w) | ((uintptr_t)p.y) | ((uintptr_t)p.bias) |
                                  ((uintptr_t)p.res);
        // 3x3, stride 1 or 2: row bands (depthwise.cuh), the ring filled by TMA when C % 4 == 0 and
        // the tensors are 16-byte aligned, else by cp.async. MGC_CUDA_DW selects a form for
        // comparisons: "ring" (cp.async, four channels per thread where possible), "ring2" (two),
        // "legacy" (the forms below).
        const char *form_env = getenv("MGC_CUDA_DW");
        const std::string form = form_env ? form_env : "tma";
        const bool band = form != "legacy" && p.nhwc && p.KH == 3 && p.KW == 3 && p.DH == 1 && p.DW == 1 &&
                          p.SH == p.SW && (p.SW == 1 || p.SW == 2) && p.C % 2 == 0 && any_ptr % 8 == 0;
        if (band) {
            const bool v4 = p.C % 4 == 0 && any_ptr % 16 == 0;
            if (v4 && form == "tma")
                st = p.SW == 1 ? launch_dw_tma<1>(p, stream) : launch_dw_tma<2>(p, stream);
            else if (v4 && form != "ring2")
                st = p.SW == 1 ? launch_dw_ring<1, 4>(p, stream) : launch_dw_ring<2, 4>(p, stream);
            else
                st = p.SW == 1 ? launch_dw_ring<1, 2>(p, stream) : launch_dw_ring<2, 2>(p, stream);
            break;
        }
        if (reg && p.DH == 1 && p.DW == 1 && p.SH == p.SW && (p.SW == 1 || p.SW == 2) && c4 % 4 == 0 && p.OW >= 16) {
            // shared-memory tiles: the input window of a tile crosses L2 once
            st = p.SW == 1 ? (c4 % 8 == 0 ? launch_dw_tile<1, 8>(p, stream) : launch_dw_tile<1, 4>(p, stream))
                           : (c4 % 8 == 0 ? launch_dw_tile<2, 8>(p, stream) : launch_dw_tile<2, 4>(p, stream));
            break;
        }
        if (reg && p.DW == 1 && (p.SW == 1 || p.SW == 2)) {
            // four output columns per thread
            const int block = (256 / c4) * c4;
            const long long items = (long long)p.N * p.OH * ((p.OW + 3) / 4);
            if (p.SW == 1) depthwise_nhwc4_rows_kernel<4, 1><<<grid_for(items, block / c4), block, 0, stream>>>(p);
            else depthwise_nhwc4_rows_kernel<4, 2><<<grid_for(items, block / c4), block, 0, stream>>>(p);
        } else if (reg) {
            const int block = (256 / c4) * c4;  // a multiple of C / 4: each thread keeps its channels
            const long long npix = (long long)p.N * p.OH * p.OW;
            depthwise_nhwc4_reg_kernel<<<grid_for(npix, block / c4), block, 0, stream>>>(p);
        } else if (vec4) {
            depthwise_nhwc4_kernel<<<grid_for(total / 4, 256), 256, 0, stream>>>(p);
        } else {
            depthwise_kernel<<<grid_for(total, 256), 256, 0, stream>>>(p);
        }
        st = check_launch("depthwise_kernel");
        break;
    }
    case MGC_K_POOL: {
        PoolParams p{};
        p.is_max = (int)i[0]; p.N = (int)i[1]; p.H = (int)i[2]; p.W = (int)i[3]; p.C = (int)i[4];
        p.KH = (int)i[5]; p.KW = (int)i[6]; p.SH = (int)i[7]; p.SW = (int)i[8]; p.DH = (int)i[9];
        p.DW = (int)i[10]; p.PT = (int)i[11]; p.PL = (int)i[12]; p.PB = (int)i[13]; p.PR = (int)i[14];
        p.OH = (int)i[15]; p.OW = (int)i[16]; p.include_pad = (int)i[17]; p.nhwc = (int)i[18];
        MGC_RESOLVE(L.r[0], p.x); MGC_RESOLVE(L.r[1], p.y);
        const long long total = (long long)p.N * p.OH * p.OW * p.C;
        if (total == 0) { launched = 0; break; }
        const bool vec = p.nhwc && (p.C & 3) == 0 && (reinterpret_cast<uintptr_t>(p.x) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(p.y) & 15) == 0 &&
                         (long long)p.N * p.H * p.W < (1ll << 31) && total / 4 < (1ll << 31);
        if (vec && p.is_max && p.KH <= 3 && p.KW <= 3 && p.DW == 1 && (p.SW == 1 || p.SW == 2)) {
            // four output columns per thread
            const long long items = (long long)p.N * p.OH * ((p.OW + 3) / 4) * (p.C / 4);
            if (p.SW == 1) maxpool4_nhwc_rows_kernel<1><<<grid_for(items, 256), 256, 0, stream>>>(p);
            else maxpool4_nhwc_rows_kernel<2><<<grid_for(items, 256), 256, 0, stream>>>(p);
            st = check_launch("maxpool4_nhwc_rows_kernel");
            break;
        }
        if (vec) {
            pool4_nhwc_kernel<<<grid_for(total / 4, 256), 256, 0, stream>>>(p);
            st = check_launch("pool4_nhwc_kernel");
            break;
        }
        pool_kernel<<<grid_for(total, 256), 256, 0, stream>>>(p);
        st = check_launch("pool_kernel");
        break;
    }
    case MGC_K_REDUCE_MID: {
        const float *x; float *y;
        MGC_RESOLVE(L.r[0], x); MGC_RESOLVE(L.r[1], y);
        const long long total = i[1] * i[3];
        if (total == 0) { launched = 0; break; }
        if (i[0] == 2) {  // mean from the producing GEMM's 32-row partial sums (gap_hw)
            if (i[2] < 32) return fail(MGC_CUDA_BAD_ARGUMENT, "reduce: partials need >= 32 rows per image");
            gap_partials_kernel<<<grid_for(total, 256), 256, 0, stream>>>(i[1], i[2], i[3], x, y);
            st = check_launch("gap_partials_kernel");
            break;
        }
        reduce_mid_kernel<<<grid_for(total, 256), 256, 0, stream>>>((int)i[0], i[1], i[2], i[3], x, y);
        st = check_launch("reduce_mid_kernel");
        break;
    }
    case MGC_K_ATTENTION: {
        // fused softmax(program(Q K^T)) V: slots documented at CudaEmitter._emit_attention
        attn::AttnArgs a{};
        a.nb1 = (int)i[0]; a.nb2 = (int)i[1]; a.sq = (int)i[2]; a.sk = (int)i[3]; a.dqk = (int)i[4]; a.dv = (int)i[5];
        a.q_rs = i[6]; a.q_b1 = i[7]; a.q_b2 = i[8];
        a.k_mn = (int)i[9]; a.k_rs = i[10]; a.k_b1 = i[11]; a.k_b2 = i[12];
        a.v_mn = (int)i[13]; a.v_rs = i[14]; a.v_b1 = i[15]; a.v_b2 = i[16];
        a.o_rs = i[17]; a.o_b1 = i[18]; a.o_b2 = i[19];
        a.mode = (int)i[20]; a.div = (int)i[21]; a.mask_dt = (int)i[22];
        a.m_b1 = i[23]; a.m_b2 = i[24]; a.m_q = i[25]; a.m_s = i[26];
        a.scale = (float)L.f[0]; a.lit = (float)L.f[1];
        MGC_RESOLVE(L.r[0], a.q); MGC_RESOLVE(L.r[1], a.k); MGC_RESOLVE(L.r[2], a.v);
        MGC_RESOLVE(L.r[3], a.o); MGC_RESOLVE(L.r[4], a.mask);
        a.err = status_dev;
        st = attn::launch_attention(a, stream);
        gemm.gemm_path = MGC_CUDA_PATH_TCGEN05;
        break;
    }
    case MGC_K_SOFTMAX: {
        const float *x = nullptr; float *y;
        MGC_RESOLVE(L.r[1], y);
        const long long rows = i[0] * i[2], n = i[1];
        if (rows == 0 || n == 0) { launched = 0; break; }
        EwParams P;
        unsigned vec_leaf = 0;
        if (i[4]) {
            // the rows are the output of an elementwise program (aux), evaluated as they are read
            MGC_CHECK(decode_elementwise(L, aux, aux_len, bases, P));
            if (i[2] != 1 || n % 4 || n > SOFTMAX_ROW_MAX || P.total != rows * n || !ew_vec4_form(P, vec_leaf) ||
                !ew_f32x4_form(P) || P.shape[P.rank - 1] % n)
                return fail(MGC_CUDA_UNSUPPORTED, "softmax of an elementwise program: rows of %lld", (long long)n);
        } else {
            MGC_RESOLVE(L.r[0], x);
            P.rank = 0;
        }
        if (i[2] == 1 && n % 4 == 0 && n <= SOFTMAX_ROW_MAX && rows * n < (1ll << 31)) {
            const int vec_io = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
            st = launch_softmax_rows(P, i[4] != 0, x, y, rows, (int)n, (int)i[3], vec_leaf, vec_io, stream);
        } else {
            softmax_kernel<<<grid_for(rows, 8), 256, 0, stream>>>(i[0], i[1], i[2], x, y, (int)i[3]);
            st = check_launch("softmax_kernel");
        }
        break;
    }
    case MGC_K_LAYER_NORM: {
        const float *x, *g, *b; float *y;
        MGC_RESOLVE(L.r[0], x); MGC_RESOLVE(L.r[1], g); MGC_RESOLVE(L.r[2], b); MGC_RESOLVE(L.r[3], y);
        if (i[0] == 0 || i[1] == 0) { launched = 0; break; }
        st = launch_layer_norm(i[0], i[1], x, g, b, (float)L.f[0], y, stream);
        break;
    }
    case MGC_K_ELEMENTWISE: {
        EwParams P;
        MGC_CHECK(decode_elementwise(L, aux, aux_len, bases, P));
        if (P.total == 0) { launched = 0; break; }
        // four elements per thread when the innermost dimension comes in groups of four
        unsigned vec_leaf = 0;
        const bool vec = ew_vec4_form(P, vec_leaf);
        const bool f32 = vec && ew_f32x4_form(P);
        if (vec && f32 && ew_chain_form(P)) {
            const int vec_out = (reinterpret_cast<uintptr_t>(P.out) & 15) == 0;
            ew_chain4_kernel<<<grid_for(P.total / 4, 256), 256, 0, stream>>>(P, vec_leaf, vec_out);
            st = check_launch("ew_chain4_kernel");
        } else if (vec && f32) {
            const int vec_out = (reinterpret_cast<uintptr_t>(P.out) & 15) == 0;
            ew_f32x4_kernel<<<grid_for(P.total / 4, 256), 256, 0, stream>>>(P, vec_leaf, vec_out);
            st = check_launch("ew_f32x4_kernel");
        } else if (vec) {
            ew_vec4_kernel<<<grid_for(P.total / 4, 256), 256, 0, stream>>>(P);
            st = check_launch("ew_vec4_kernel");
        } else {
            ew_kernel<<<grid_for(P.total, 256), 256, 0, stream>>>(P);
            st = check_launch("ew_kernel");
        }
        break;
    }
    case MGC_K_COPY: {
        const int rank = (int)i[0], esize = (int)i[1];
        if (rank < 0 || rank > COPY_MAX_RANK) return fail(MGC_CUDA_UNSUPPORTED, "copy: rank %d", rank);
        const char *src; char *dst;
        MGC_RESOLVE(L.r[0], src); MGC_RESOLVE(L.r[1], dst);
        long long total = 1;
        for (int d = 0; d < rank; ++d) total *= i[2 + d];
        if (total == 0) { launched = 0; break; }
        if (i[28] == 2) {  // Split along the last axis: i[29] outputs of widths i[30..33], i[34] rows
            const int k = (int)i[29];
            if (esize != 4 || k < 1 || k > SPLIT_MAX_OUT) return fail(MGC_CUDA_UNSUPPORTED, "split: %d outputs", k);
            char *outs[SPLIT_MAX_OUT] = {};
            uintptr_t any = (uintptr_t)src;
            long long width = 0;
            bool vec = true;
            for (int j = 0; j < k; ++j) {
                MGC_RESOLVE(L.r[1 + j], outs[j]);
                any |= (uintptr_t)outs[j];
                vec = vec && i[30 + j] % 4 == 0;
                width += i[30 + j];
            }
            const long long rows = i[34];
            vec = vec && any % 16 == 0;
            if (rows * width == 0) { launched = 0; break; }
            if (width >= (1ll << 31)) return fail(MGC_CUDA_UNSUPPORTED, "split: row of %lld", width);
            auto go = [&](auto unit, int per) -> int {
                using T = decltype(unit);
                SplitParams<T> P{};
                P.src = reinterpret_cast<const T *>(src);
                P.rows = rows;
                P.k = k;
                P.total = (int)(width / per);
                for (int j = 0; j < k; ++j) {
                    P.dst[j] = reinterpret_cast<T *>(outs[j]);
                    P.start[j + 1] = P.start[j] + (int)(i[30 + j] / per);
                }
                split_last_kernel<T><<<grid_for(rows * P.total, 256), 256, 0, stream>>>(P);
                return check_launch("split_last_kernel");
            };
            st = vec ? go(uint4{}, 4) : go(uint32_t{}, 1);
            break;
        }
        if (i[28] == 1) {  // Tile
            TileParams P{};
            P.rank = rank; P.esize = esize; P.total = total; P.src = src; P.dst = dst;
            for (int d = 0; d < rank; ++d) { P.oshape[d] = i[2 + d]; P.xshape[d] = i[10 + d]; P.xstr[d] = i[19 + d]; }
            switch (esize) {
            case 1: st = launch_tile_t<uint8_t>(P, stream); break;
            case 2: st = launch_tile_t<uint16_t>(P, stream); break;
            case 4: st = launch_tile_t<uint32_t>(P, stream); break;
            case 8: st = launch_tile_t<uint64_t>(P, stream); break;
            default: return fail(MGC_CUDA_UNSUPPORTED, "copy: element size %d", esize);
            }
            break;
        }
        CopyParams P{};
        P.rank = rank; P.esize = esize; P.total = total; P.src = src; P.dst = dst;
        for (int d = 0; d < rank; ++d) { P.shape[d] = i[2 + d]; P.sstr[d] = i[10 + d]; P.dstr[d] = i[19 + d]; }
        P.sbase = i[18]; P.dbase = i[27];
        switch (esize) {
        case 1: st = launch_copy_t<uint8_t>(P, stream); break;
        case 2: st = launch_copy_t<uint16_t>(P, stream); break;
        case 4: st = launch_copy_t<uint32_t>(P, stream); break;
        case 8: st = launch_copy_t<uint64_t>(P, stream); break;
        default: return fail(MGC_CUDA_UNSUPPORTED, "copy: element size %d", esize);
        }
        break;
    }
    case MGC_K_FILL: {
        char *dst;
        MGC_RESOLVE(L.r[0], dst);
        const long long n = i[0];
        const int esize = (int)i[1];
        const int64_t bits = i[2];
        if (n == 0) { launched = 0; break; }
        const unsigned g = grid_for(n, 256);
        switch (esize) {
        case 1: fill_kernel<uint8_t><<<g, 256, 0, stream>>>((uint8_t *)dst, n, (uint8_t)bits); break;
        case 2: fill_kernel<uint16_t><<<g, 256, 0, stream>>>((uint16_t *)dst, n, (uint16_t)bits); break;
        case 4: fill_kernel<uint32_t><<<g, 256, 0, stream>>>((uint32_t *)dst, n, (uint32_t)bits); break;
        case 8: fill_kernel<uint64_t><<<g, 256, 0, stream>>>((uint64_t *)dst, n, (uint64_t)bits); break;
        default: return fail(MGC_CUDA_UNSUPPORTED, "fill: element size %d", esize);
        }
        st = check_launch("fill_kernel");
        break;
    }
    case MGC_K_GATHER: {
        const char *x; const void *idx; char *out;
        MGC_RESOLVE(L.r[0], x); MGC_RESOLVE(L.r[1], idx); MGC_RESOLVE(L.r[2], out);
        const long long outer = i[0], dim = i[1], inner = i[2], n = i[3];
        const int idt = (int)i[4], esize = (int)i[5];
        const long long total = outer * n * inner;
        if (total == 0) { launched = 0; break; }
        const unsigned g = grid_for(total, 256);
        switch (esize) {
        case 1: gather_kernel<uint8_t><<<g, 256, 0, stream>>>((const uint8_t *)x, idx, idt, (uint8_t *)out, outer, dim, inner, n, status_dev); break;
        case 4: gather_kernel<uint32_t><<<g, 256, 0, stream>>>((const uint32_t *)x, idx, idt, (uint32_t *)out, outer, dim, inner, n, status_dev); break;
        case 8: gather_kernel<uint64_t><<<g, 256, 0, stream>>>((const uint64_t *)x, idx, idt, (uint64_t *)out, outer, dim, inner, n, status_dev); break;
        default: return fail(MGC_CUDA_UNSUPPORTED, "gather: element size %d", esize);
        }
        st = check_launch("gather_kernel");
        break;
    }
    case MGC_K_REDUCE: {
        const void *x; void *y;
        MGC_RESOLVE(L.r[0], x); MGC_RESOLVE(L.r[1], y);
        const long long total = i[1] * i[3];
        if (total == 0) { launched = 0; break; }
        reduce_kernel<<<grid_for(total, 256), 256, 0, stream>>>((int)i[0], L.dtype, i[1], i[2], i[3], x, y);
        st = check_launch("reduce_kernel");
        break;
    }
    case MGC_K_ARGMAX: {
        const void *x; long long *y;
        MGC_RESOLVE(L.r[0], x); MGC_RESOLVE(L.r[1], y);
        const long long total = i[0] * i[2];
        if (total == 0) { launched = 0; break; }
        argmax_kernel<<<grid_for(total, 256), 256, 0, stream>>>(L.dtype, i[0], i[1], i[2], x, y);
        st = check_launch("argmax_kernel");
        break;
    }
    case MGC_K_RANGE: {
        void *y; const void *s0; const void *dl;
        MGC_RESOLVE(L.r[0], y); MGC_RESOLVE(L.r[1], s0); MGC_RESOLVE(L.r[2], dl);
        if (i[0] == 0) { launched = 0; break; }
        range_kernel<<<grid_for(i[0], 256), 256, 0, stream>>>(y, L.dtype, i[0], s0, dl);
        st = check_launch("range_kernel");
        break;
    }
    case MGC_K_IM2COL: {
        Im2colParams p{};
        p.N = (int)i[0]; p.H = (int)i[1]; p.W = (int)i[2]; p.C = (int)i[3]; p.KH = (int)i[4];
        p.KW = (int)i[5]; p.SH = (int)i[6]; p.SW = (int)i[7]; p.DH = (int)i[8]; p.DW = (int)i[9];
        p.PT = (int)i[10]; p.PL = (int)i[11]; p.OH = (int)i[12]; p.OW = (int)i[13];
        p.kp = (int)i[14]; p.c_off = (int)i[15]; p.cg = (int)i[16];
        MGC_RESOLVE(L.r[0], p.x); MGC_RESOLVE(L.r[1], p.out);
        if (p.kp <= 0 || (p.kp & 3) || (reinterpret_cast<uintptr_t>(p.out) & 15))
            return fail(MGC_CUDA_BAD_ARGUMENT, "im2col: row length %d / output alignment", p.kp);
        const long long total = (long long)p.N * p.OH * p.OW * (p.kp / 4);
        if (total == 0) { launched = 0; break; }
        im2col_nhwc_kernel<<<grid_for(total, 256), 256, 0, stream>>>(p);
        st = check_launch("im2col_nhwc_kernel");
        break;
    }
    case MGC_K_PACK: {
        PackParams p{};
        p.N = (int)i[0]; p.H = (int)i[1]; p.W = (int)i[2]; p.C = (int)i[3]; p.cp = (int)i[4];
        p.sn = i[5]; p.sh = i[6]; p.sw = i[7]; p.sc = i[8];
        p.PT = (int)i[9]; p.PL = (int)i[10]; p.Hp = (int)i[11]; p.Wp = (int)i[12];
        p.phases = (int)i[13];
        MGC_RESOLVE(L.r[0], p.x); MGC_RESOLVE(L.r[1], p.out);
        if (p.cp <= 0 || (p.cp & 3) || p.C > p.cp || (reinterpret_cast<uintptr_t>(p.out) & 15))
            return fail(MGC_CUDA_BAD_ARGUMENT, "pack: %d of %d channels / output alignment", p.C, p.cp);
        if (p.phases) {
            const long long total = (long long)p.N * p.Hp * p.Wp;
            const long long src_last = (long long)(p.N - 1) * p.sn + (long long)(p.H - 1) * p.sh +
                                       (long long)(p.W - 1) * p.sw + (long long)(p.C - 1) * p.sc;
            if (p.phases != 2 || p.cp != 4 || (p.Wp & 1) || p.PT < 0 || p.Hp < p.PT + p.H || total >= (1ll << 31) ||
                src_last >= (1ll << 31) || p.sn < 0 || p.sh < 0 || p.sw < 0 || p.sc < 0 ||
                2ll * (p.Wp / 2) < (long long)p.W + p.PL)
                return fail(MGC_CUDA_BAD_ARGUMENT, "pack: phase-split layout %dx%d of a %dx%dx%d image", p.Hp, p.Wp,
                            p.H, p.W, p.C);
            if (total == 0) { launched = 0; break; }
            static const bool rows_env = [] {  // MGC_CUDA_PACK_ROWS=0: the one-pixel-per-thread kernel
                const char *e = getenv("MGC_CUDA_PACK_ROWS");
                return !(e && e[0] == '0');
            }();
            if (rows_env && (long long)p.N * p.Hp <= 65535) {  // one block per packed row
                pack_phase_rows_kernel<<<dim3((unsigned)((p.Wp / 2 + 127) / 128), (unsigned)(p.N * p.Hp)), 128, 0,
                                         stream>>>(p);
                st = check_launch("pack_phase_rows_kernel");
                break;
            }
            pack_phase_kernel<<<grid_for(total, 256), 256, 0, stream>>>(p);
            st = check_launch("pack_phase_kernel");
            break;
        }
        if (p.PT < 0 || p.PL < 0 || p.Hp < p.PT + p.H || p.Wp < p.PL + p.W)
            return fail(MGC_CUDA_BAD_ARGUMENT, "pack: padded %dx%d cannot hold %dx%d at (%d, %d)", p.Hp, p.Wp,
                        p.H, p.W, p.PT, p.PL);
        const long long total = (long long)p.N * p.Hp * p.Wp;
        if (total == 0) { launched = 0; break; }
        // 32-bit indices when every pixel index and source offset fits
        const long long src_last = (long long)(p.N - 1) * p.sn + (long long)(p.H - 1) * p.sh +
                                   (long long)(p.W - 1) * p.sw + (long long)(p.C - 1) * p.sc;
        const bool small = total < (1ll << 31) && src_last < (1ll << 31) && p.sn >= 0 && p.sh >= 0 && p.sw >= 0 &&
                           p.sc >= 0 && p.sn < (1ll << 31) && p.sh < (1ll << 31) && p.sw < (1ll << 31) &&
                           p.sc < (1ll << 31);
        if (small) pack_nhwc32_kernel<<<grid_for(total, 256), 256, 0, stream>>>(p);
        else pack_nhwc_kernel<<<grid_for(total, 256), 256, 0, stream>>>(p);
        st = check_launch("pack_nhwc_kernel");
        break;
    }
    case MGC_K_MEMCPY: {
        const void *src; void *dst;
        MGC_RESOLVE(L.r[0], src); MGC_RESOLVE(L.r[1], dst);
        launched = 0;
        if (i[0] > 0) MGC_CHECK_CUDA(cudaMemcpyAsync(dst, src, (size_t)i[0], cudaMemcpyDeviceToDevice, stream));
        break;
    }
    default:
        return fail(MGC_CUDA_UNSUPPORTED, "unknown launch kind %d (node %d)", L.kind, L.node);
    }
    if (st != MGC_CUDA_OK) return st;
    if (info) {
        info->kernels = launched;
        info->gemm_path = gemm.gemm_path;
    }
    return MGC_CUDA_OK;
}

}  // namespace mgc
