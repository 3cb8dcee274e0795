// Depthwise 3x3 convolution (NHWC) in row bands: the forms for a 3x3 window with the same stride
// (1 or 2) in both dimensions and no dilation, the shape of every depthwise layer of MobileNetV2.
// Other windows keep the forms of kernels_norm.cuh.
//
// A block computes a band of `bh` output rows x `tw` output columns x `cg` channel vectors (VEC =
// 2 or 4 fp32 channels each); one thread per column and vector, channel vectors fastest, so a
// warp reads whole pieces of pixels. The band's input rows pass through a ring of D row slots in
// shared memory ((tw - 1) * S + 3 input columns x cg vectors each, zeros outside the image),
// filled D - 1 rows ahead of the row in use, so a block keeps D - 1 rows of loads in flight while
// it computes; one block barrier per input row makes a row visible and frees the slot of the
// row before it. Each thread walks its column down the band and takes its three taps of every
// input row from the ring; the row's products go to every output row that uses it (at stride 1
// the rows o, o + 1 and o + 2 take its tap rows 2, 1 and 0; at stride 2 the rows o and o + 1 take
// tap rows 2 and 0, the odd rows in between tap row 1). So every output adds bias, then
// kh = 0, 1, 2 with kw = 0, 1, 2 in that order, as the other depthwise forms do, two channels
// per packed fp32x2 FMA (`__ffma2_rn`, rounded like two fmaf).
//
// depthwise_tma_kernel (C % 4 == 0, 16-byte aligned tensors): one thread fills a slot with one
// TMA load of a 4-D tile (channels, columns, row, image), completing on the slot's mbarrier;
// out-of-image columns and rows read as zeros. depthwise_ring_kernel (C % 2 == 0): every thread
// copies its share of a row with cp.async (zeros by a source size of 0).
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "common.cuh"
#include "gemm_umma.cuh"
#include "kernels_norm.cuh"

namespace mgc {

template <int VEC>
struct DwVec;
template <>
struct DwVec<4> {
    using T = float4;
    __device__ static __forceinline__ void split(const float4 v, float2 (&r)[2]) {
        r[0] = make_float2(v.x, v.y);
        r[1] = make_float2(v.z, v.w);
    }
    __device__ static __forceinline__ float4 join(const float2 (&r)[2]) { return make_float4(r[0].x, r[0].y, r[1].x, r[1].y); }
};
template <>
struct DwVec<2> {
    using T = float2;
    __device__ static __forceinline__ void split(const float2 v, float2 (&r)[1]) { r[0] = v; }
    __device__ static __forceinline__ float2 join(const float2 (&r)[1]) { return r[0]; }
};

struct DwBand {
    int tw, bh, cg;                 // columns, output rows and channel vectors of one block
    unsigned tiles, bands, chunks;  // column tiles, row bands and channel chunks of one image
};

// One block's place: image, band, column tile and channel chunk (chunk fastest, so the blocks
// running together share their input rows' halo columns in L2).
struct DwPlace {
    unsigned n, band, ct, chunk;
    __device__ __forceinline__ explicit DwPlace(const DwBand &t) {
        unsigned b = blockIdx.x;
        chunk = b % t.chunks;
        b /= t.chunks;
        ct = b % t.tiles;
        b /= t.tiles;
        band = b % t.bands;
        n = b / t.bands;
    }
};

// This thread's weights (3x3, HWC) and bias for channels [c, c + VEC).
template <int VEC>
__device__ __forceinline__ void dw_weights(const DepthwiseParams &p, int c, float2 (&wk)[9][VEC / 2],
                                           float2 (&bias)[VEC / 2]) {
    using V = typename DwVec<VEC>::T;
#pragma unroll
    for (int k = 0; k < 9; ++k) DwVec<VEC>::split(__ldg(reinterpret_cast<const V *>(p.w + (size_t)k * p.C + c)), wk[k]);
    if (p.bias) {
        DwVec<VEC>::split(__ldg(reinterpret_cast<const V *>(p.bias + c)), bias);
    } else {
#pragma unroll
        for (int j = 0; j < VEC / 2; ++j) bias[j] = make_float2(0.0f, 0.0f);
    }
}

// Activations the band forms apply in the store: compile-time cases for the common ones.
enum DwAct { DW_NONE = 0, DW_RELU = 1, DW_CLIP = 2, DW_ANY = 3 /* p.act at run time */ };

// The walk of one thread down output rows [oh0, oh1) of its column; `next_row(v)` delivers the
// next input row's three taps (false: stop, the block gave up waiting). o_off: the element
// offset of output row oh0 of this thread's column and channels; `active`: the column exists.
template <int S, int VEC, int ACT, typename NextRow>
__device__ __forceinline__ void dw_walk(const DepthwiseParams &p, const float2 (&wk)[9][VEC / 2],
                                        const float2 (&bias)[VEC / 2], int oh0, int oh1, long long o_off,
                                        bool active, NextRow &next_row) {
    constexpr int P = VEC / 2;
    using V = typename DwVec<VEC>::T;
    V *yp = reinterpret_cast<V *>(p.y + o_off);
    const long long vstride = (long long)p.OW * p.C / VEC;  // output row stride in vectors
    const long long res_delta = p.res ? p.res - p.y : 0;   // the residual's element offset from the output
    auto taps = [&](float2 (&acc)[P], const float2 (&v)[3][P], int kh, bool fresh) {
#pragma unroll
        for (int j = 0; j < P; ++j) {
            float2 a = fresh ? bias[j] : acc[j];
            a = __ffma2_rn(v[0][j], wk[kh * 3 + 0][j], a);
            a = __ffma2_rn(v[1][j], wk[kh * 3 + 1][j], a);
            a = __ffma2_rn(v[2][j], wk[kh * 3 + 2][j], a);
            acc[j] = a;
        }
    };
    // residual, activation and the store of a finished output row
    auto finish = [&](float2 (&acc)[P]) {
        if (active) {
            if (p.res) {
                float2 r[P];
                DwVec<VEC>::split(*reinterpret_cast<const V *>(reinterpret_cast<const float *>(yp) + res_delta), r);
#pragma unroll
                for (int j = 0; j < P; ++j) acc[j] = __fadd2_rn(acc[j], r[j]);
            }
#pragma unroll
            for (int j = 0; j < P; ++j) {
                float2 &a = acc[j];
                if (ACT == DW_RELU || (ACT == DW_ANY && p.act == MGC_ACT_RELU)) {
                    a.x = fmaxf(a.x, 0.0f); a.y = fmaxf(a.y, 0.0f);
                } else if (ACT == DW_CLIP || (ACT == DW_ANY && p.act == MGC_ACT_CLIP)) {
                    a.x = fminf(fmaxf(a.x, p.lo), p.hi); a.y = fminf(fmaxf(a.y, p.lo), p.hi);
                } else if (ACT == DW_ANY && p.act != MGC_ACT_NONE) {
                    a.x = apply_act(a.x, p.act, p.lo, p.hi); a.y = apply_act(a.y, p.act, p.lo, p.hi);
                }
            }
            *yp = DwVec<VEC>::join(acc);
        }
        yp += vstride;
    };
    float2 v[3][P];
    float2 a0[P], a1[P], a2[P];
    int o = oh0;
    if (S == 1) {
        if (!next_row(v)) return;
        taps(a0, v, 0, true);
        if (!next_row(v)) return;
        taps(a0, v, 1, false);
        taps(a1, v, 0, true);
        // r0 finishes with this row; r1 and r2 are the next two output rows
        auto step = [&](float2 (&r0)[P], float2 (&r1)[P], float2 (&r2)[P]) -> bool {
            if (!next_row(v)) return false;
            taps(r0, v, 2, false);
            finish(r0);
            taps(r1, v, 1, false);
            taps(r2, v, 0, true);
            return ++o < oh1;
        };
#pragma unroll 1
        while (step(a0, a1, a2) && step(a1, a2, a0) && step(a2, a0, a1)) {
        }
    } else {
        if (!next_row(v)) return;
        taps(a0, v, 0, true);
        auto step = [&](float2 (&r0)[P], float2 (&r1)[P]) -> bool {
            if (!next_row(v)) return false;
            taps(r0, v, 1, false);
            if (!next_row(v)) return false;
            taps(r0, v, 2, false);
            finish(r0);
            taps(r1, v, 0, true);
            return ++o < oh1;
        };
#pragma unroll 1
        while (step(a0, a1) && step(a1, a0)) {
        }
    }
    (void)a2;
}

template <int S, int D, int ACT>
__global__ void __launch_bounds__(256, 3) depthwise_tma_kernel(const __grid_constant__ DepthwiseParams p, const DwBand t,
                                                            const __grid_constant__ CUtensorMap map) {
    constexpr int VEC = 4;
    extern __shared__ uint8_t dw_smem_raw[];
    // [D slots, each 128-byte aligned][D full barriers]; aligned by an offset into the window
    uint8_t *smem = dw_smem_raw + ((128u - (umma::smem_addr(dw_smem_raw) & 127u)) & 127u);
    const DwPlace at(t);
    const int g = (int)threadIdx.x % t.cg, col = (int)threadIdx.x / t.cg;
    const int ow = (int)at.ct * t.tw + col;
    const int oh0 = (int)at.band * t.bh, oh1 = min(oh0 + t.bh, p.OH);
    const int slot_vecs = ((t.tw - 1) * S + 3) * t.cg;
    const uint32_t slot_bytes = (uint32_t)slot_vecs * 16u, slot_stride = (slot_bytes + 127u) & ~127u;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)D * slot_stride);
    const int rows = (oh1 - oh0 - 1) * S + 3;
    const bool leader = threadIdx.x == 0;
    if (leader) {
        umma::prefetch_tmap(&map);
        for (int s = 0; s < D; ++s) umma::mbar_init(&full[s], 1);
        umma::fence_barrier_init();
    }
    __syncthreads();
    const int cx = (int)at.chunk * t.cg * VEC, wx = (int)at.ct * t.tw * S - p.PL, hy = oh0 * S - p.PT;
    // the leader loads band row r into slot s
    auto issue = [&](int r, int s) {
        if (leader && r < rows) {
            umma::mbar_expect_tx(&full[s], slot_bytes);
            umma::tma_load_4d(smem + (size_t)s * slot_stride, &map, &full[s], cx, wx, hy + r, (int)at.n);
        }
    };
    for (int r = 0; r < D - 1; ++r) issue(r, r);
    float2 wk[9][2], bias[2];
    const int c = cx + g * VEC;
    dw_weights<VEC>(p, c, wk, bias);
    // this thread's first tap in a slot, the slot in use and its barrier's phase parity
    const uint32_t ring_s = umma::smem_addr(smem);
    const uint32_t tap0 = (uint32_t)(col * S * t.cg + g) * 16u, kw_bytes = (uint32_t)t.cg * 16u;
    int s_use = 0;
    uint32_t parity = 0, slot_addr = ring_s;
    int used = 0;  // rows taken from the ring
    bool failed = false;
    auto next_row = [&](float2 (&v)[3][2]) -> bool {
        // every thread is done with the previous row's slot, which the next load refills
        if (__syncthreads_or(failed)) return false;
        issue(used + D - 1, s_use == 0 ? D - 1 : s_use - 1);
        if (!umma::mbar_wait(&full[s_use], parity)) {
            failed = true;
            umma::set_error(p.err, MGC_CUDA_TIMEOUT);
        }
        const uint32_t a = slot_addr + tap0;
#pragma unroll
        for (int kw = 0; kw < 3; ++kw) {
            float4 x;
            asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                         : "=f"(x.x), "=f"(x.y), "=f"(x.z), "=f"(x.w)
                         : "r"(a + (uint32_t)kw * kw_bytes));
            DwVec<VEC>::split(x, v[kw]);
        }
        ++used;
        if (++s_use == D) {
            s_use = 0;
            parity ^= 1u;
            slot_addr = ring_s;
        } else {
            slot_addr += slot_stride;
        }
        return true;
    };
    const long long o_off = (((long long)at.n * p.OH + oh0) * p.OW + ow) * p.C + c;
    dw_walk<S, VEC, ACT>(p, wk, bias, oh0, oh1, o_off, ow < p.OW, next_row);
    // a block that gave up waits (bounded) for the loads it issued before its shared memory goes
    if (__syncthreads_or(failed) && leader) {
        const int issued = min(rows, used + D - 1);
        for (int r = used; r < issued; ++r) (void)umma::mbar_wait(&full[r % D], (uint32_t)((r / D) & 1));
    }
}

template <int S, int VEC, int D>
__global__ void __launch_bounds__(256, VEC == 4 ? 3 : 4) depthwise_ring_kernel(const __grid_constant__ DepthwiseParams p,
                                                             const DwBand t) {
    constexpr int P = VEC / 2;
    constexpr int MAXL = 3;  // copies per thread and row: ((tw - 1) * S + 3) * cg <= 3 * tw * cg
    using V = typename DwVec<VEC>::T;
    extern __shared__ float4 dw_ring_raw[];
    V *ring = reinterpret_cast<V *>(dw_ring_raw);
    const DwPlace at(t);
    const int threads = t.tw * t.cg;
    const int tid = (int)threadIdx.x;
    const int g = tid % t.cg, col = tid / t.cg;
    const int ow = (int)at.ct * t.tw + col;
    const int oh0 = (int)at.band * t.bh, oh1 = min(oh0 + t.bh, p.OH);
    const int slot_vecs = ((t.tw - 1) * S + 3) * t.cg;
    const int rows = (oh1 - oh0 - 1) * S + 3;
    const int ih0 = oh0 * S - p.PT;
    const int iw0 = (int)at.ct * t.tw * S - p.PL;
    const int c = ((int)at.chunk * t.cg + g) * VEC;
    // this thread's copies of every row: slot element, source offset within a row, inside the image
    const long long row_elems = (long long)p.W * p.C;
    const long long img = (long long)at.n * p.H * row_elems;
    long long src_off[MAXL];
    uint32_t dst[MAXL];
    bool in_w[MAXL];
    const uint32_t ring_s = static_cast<uint32_t>(__cvta_generic_to_shared(ring));
#pragma unroll
    for (int k = 0; k < MAXL; ++k) {
        const int e = tid + k * threads;
        const int pix = e / t.cg, gg = e % t.cg;
        const int iw = iw0 + pix;
        in_w[k] = e < slot_vecs && iw >= 0 && iw < p.W;
        src_off[k] = img + (long long)iw * p.C + ((int)at.chunk * t.cg + gg) * VEC;
        dst[k] = e < slot_vecs ? ring_s + (uint32_t)e * (uint32_t)sizeof(V) : 0xffffffffu;
    }
    // copy input row r of the band into its slot (zeros outside the image) as one commit group
    auto issue = [&](int r) {
        if (r < rows) {
            const int ih = ih0 + r;
            const bool in_h = (unsigned)ih < (unsigned)p.H;
            const uint32_t slot = (uint32_t)((r % D) * slot_vecs) * (uint32_t)sizeof(V);
#pragma unroll
            for (int k = 0; k < MAXL; ++k) {
                if (dst[k] == 0xffffffffu) continue;
                const bool inside = in_h && in_w[k];
                const float *src = inside ? p.x + src_off[k] + (long long)ih * row_elems : p.x;
                if (VEC == 4)
                    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst[k] + slot), "l"(src),
                                 "r"(inside ? 16 : 0)
                                 : "memory");
                else
                    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst[k] + slot), "l"(src),
                                 "r"(inside ? 8 : 0)
                                 : "memory");
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    float2 wk[9][P], bias[P];
    dw_weights<VEC>(p, c, wk, bias);
#pragma unroll
    for (int r = 0; r < D - 1; ++r) issue(r);
    int used = 0;
    // wait for row `used`, then refill the slot of the row before it D - 1 rows ahead
    auto next_row = [&](float2 (&v)[3][P]) -> bool {
        asm volatile("cp.async.wait_group %0;" ::"n"(D - 2) : "memory");
        __syncthreads();
        issue(used + D - 1);
        const V *row = ring + (used % D) * slot_vecs + col * S * t.cg + g;
#pragma unroll
        for (int kw = 0; kw < 3; ++kw) DwVec<VEC>::split(row[kw * t.cg], v[kw]);
        ++used;
        return true;
    };
    const long long o_off = (((long long)at.n * p.OH + oh0) * p.OW + ow) * p.C + c;
    dw_walk<S, VEC, DW_ANY>(p, wk, bias, oh0, oh1, o_off, ow < p.OW, next_row);
    asm volatile("cp.async.wait_all;" ::: "memory");
}

}  // namespace mgc
