// Fused attention for sm_100a: O = softmax(program(Q K^T)) V, one CTA per (batch, head, tile of
// 128 queries), the scores never leaving the SM.
//
// The chain it replaces is the scheduled graph's MatMul(Q, K^T) -> [the score program: X * s or
// X / s, then optionally + M, - M or Where(C, t, lit) / Where(C, lit, t)] -> Softmax(last axis)
// -> MatMul(P, V) (reference passes/fusion.py builds the FusedElementwise program; its C backend
// runs the four as separate loops, codegen/c.py:823-852 and 974-1226). Here:
// * Q [128 x Dqk], K [Sk x Dqk] and V [Sk x Dv] arrive by TMA through TFLOAT32 tensor maps (each
//   value rounded to the nearest TF32 value, as the unfused tensor-core GEMMs load them) in
//   128B-swizzled rows: Q and a K with contiguous Dqk as K-major operands, a V with contiguous Dv
//   (and a K^T with contiguous Sk) as MN-major operands in the 32-byte-atom swizzle, the only
//   swizzled MN-major form tcgen05 reads for 32-bit types; a V stored [Dv][Sk] is K-major.
// * One elected thread issues S = Q K^T (M = 128, N = Sk rounded up to 32, K = Dqk in steps of 8)
//   into TMEM columns [0, Sk).
// * Threads t, t + 128, t + 256 and t + 384 of the sixteen warps own query row t (TMEM lane t;
//   warps w, w + 4, w + 8 and w + 12 read the same lanes) and take every fourth 32-column slice of
//   it into registers: each evaluates the score program on its slices (compiled for the forms the
//   benchmark models use), the four combine their maxima and sums through shared memory, and
//   each writes P = e * (1 / sum) (e = __expf(t - max), as the unfused softmax kernel)
//   rounded to TF32 (ties away from zero, the TFLOAT32 tensor map's rounding) into shared memory
//   in the K-major 128B-swizzled layout, over Q and K (no longer read).
// * The elected thread issues O = P V (M = 128, N = Dv rounded up to 32, K = Sk) into TMEM
//   columns [0, Dv) (S is dead by then); the warps stage O's rows in shared memory and one
//   thread stores them with TMA into the output's strided view (attention's head merge
//   (b, h, s, d) -> (b, s, h, d) included), rows past Sq clipped by the tensor map.
//
// Every mbarrier wait is bounded; on timeout the CTA records MGC_CUDA_TIMEOUT in the error word,
// skips the rest of its work, frees its TMEM and returns.
#pragma once

#include "gemm_umma.cuh"

namespace mgc {
namespace attn {

using umma::fence_barrier_init;
using umma::fence_proxy_async_smem;
using umma::instr_desc_tf32;
using umma::mbar_arrive;
using umma::mbar_expect_tx;
using umma::mbar_init;
using umma::mbar_wait;
using umma::mma_commit;
using umma::mma_tf32;
using umma::prefetch_tmap;
using umma::smem_addr;
using umma::sts4;
using umma::sw128_desc;
using umma::tc_fence_after;
using umma::tc_fence_before;
using umma::tma_load_4d;
using umma::tma_store_4d;
using umma::tmem_alloc;
using umma::tmem_dealloc;
using umma::tmem_ld32;
using umma::tmem_wait_ld;

constexpr int THREADS = 512;   // sixteen warps: four threads per query row (TMEM lane)
constexpr int QROWS = 128;     // queries per CTA (the MMA's M)
constexpr int MAX_SK = 256;    // keys per row: S's TMEM columns and the MMA's N
constexpr int MAX_D = 128;     // head width of Q / K and of V
constexpr uint32_t CHUNK = 128 * 128;  // one 32-column slice of a 128-row K-major operand

// Score program (the ScaleMask form of the unfused softmax, kernels_norm.cuh).
enum { MASK_NONE = 0, MASK_ADD = 1, MASK_SUB = 2, MASK_KEEP = 3, MASK_FILL = 4 };

struct AttnParams {
    CUtensorMap tmQ;   // {Dqk, Sq, b1, b2}, boxes {32, 128}
    CUtensorMap tmK;   // k_mn 0: {Dqk, Sk, b1, b2}, boxes {32, skp}; 1: {Sk, Dqk, b1, b2}, boxes {32, dqp}
    CUtensorMap tmV;   // v_mn 1: {Dv, Sk, b1, b2}, boxes {32, skp}; 0: {Sk, Dv, b1, b2}, boxes {32, dvp}
    CUtensorMap tmO;   // {Dv, Sq, b1, b2}, boxes {32, 128}
    const void *mask;  // M (fp32) or C (bool / uint8), element strides below
    long long m_b1, m_b2, m_q, m_s;
    float scale, lit;
    int mode, div, mask_u8, mask_vec;  // mask_vec: m_s == 1, Sk % 4 == 0, rows 16 (fp32) / 4 (byte) aligned
    int sq, sk;
    int skp, dqp, dvp;  // Sk, Dqk, Dv rounded up to 32
    int k_mn, v_mn;
    int nb1, q_tiles;
    uint32_t tmem_cols;
    uint32_t region0;   // bytes of the Q + K / P / O region; V follows
    int *err;
};

// MN-major operand of 32-bit elements in the 32-byte-atom 128B swizzle: rows of 128 bytes along
// M / N (32 elements), consecutive K rows 128 bytes apart, 32-byte chunks swizzled within 4-row
// (512-byte) atoms: what a CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B box of 32 x rows lands as. `lbo`
// bytes between 32-element blocks along M / N, 512 bytes between 4-row groups along K.
__device__ __forceinline__ uint64_t mn32_desc(uint32_t saddr, uint32_t lbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu)
           | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16)
           | ((uint64_t)(512 >> 4) << 32)
           | ((uint64_t)1 << 46)                   // descriptor version (sm_100)
           | ((uint64_t)1 << 61);                  // 128-byte swizzle, 32-byte atoms
}

// Descriptor of K step `ks` (8 K values) of a B operand with `n_pad` rows along N and `k_pad`
// along K: K-major in 32-column slices of n_pad x 128 bytes, or MN-major in 32-row blocks of
// k_pad x 128 bytes.
__device__ __forceinline__ uint64_t b_desc(uint32_t base, int mn, int ks, int n_pad, int k_pad) {
    return mn ? mn32_desc(base + (uint32_t)ks * 1024u, (uint32_t)k_pad * 128u)
              : sw128_desc(base + (uint32_t)(ks >> 2) * (uint32_t)n_pad * 128u + (uint32_t)(ks & 3) * 32u);
}

// Score-program forms compiled without runtime tests (the forms of the benchmark models), and the
// generic form that reads every choice from the parameters.
enum {
    FORM_GENERIC = 0,
    FORM_MUL = 1,       // t = X * s
    FORM_MUL_ADD = 2,   // t = X * s + M, M fp32 with 16-byte aligned rows (BERT)
    FORM_MUL_FILL = 3,  // t = Where(C, lit, X * s), C bytes with 4-byte aligned rows (GPT-2)
    FORM_MUL_KEEP = 4,  // t = Where(C, X * s, lit), C bytes with 4-byte aligned rows
};

// The score program on 32 values of a row (columns s0 .. s0 + 31); columns at or past Sk become
// -inf (no weight). The mask row starts at element `mrow`. Vector mask loads need Sk % 4 == 0
// (the host's mask_vec): a load past Sk is moved back to the row's last four values (in bounds)
// and its columns are -inf anyway.
template <int FORM>
__device__ __forceinline__ void score_program(const AttnParams &p, float (&t)[32], int s0, long long mrow) {
    constexpr bool G = FORM == FORM_GENERIC;
    if (G && p.div) {
#pragma unroll
        for (int j = 0; j < 32; ++j) t[j] = t[j] / p.scale;
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) t[j] = t[j] * p.scale;
    }
    const int mode = G ? p.mode
                       : FORM == FORM_MUL_ADD ? MASK_ADD
                       : FORM == FORM_MUL_FILL ? MASK_FILL
                       : FORM == FORM_MUL_KEEP ? MASK_KEEP : MASK_NONE;
    if (mode != MASK_NONE) {
        const bool u8 = G ? p.mask_u8 != 0 : (FORM == FORM_MUL_FILL || FORM == FORM_MUL_KEEP);
        const bool vec = G ? p.mask_vec != 0 : true;
        auto apply = [&](float &x, float m) {
            if (mode == MASK_ADD) x = x + m;
            else if (mode == MASK_SUB) x = x - m;
            else if (mode == MASK_KEEP) x = m != 0.0f ? x : p.lit;
            else x = m != 0.0f ? p.lit : x;
        };
        if (vec) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int s4 = min(s0 + 4 * j, p.sk - 4);
                float4 m;
                if (u8) {
                    const uchar4 c = __ldg(reinterpret_cast<const uchar4 *>(static_cast<const unsigned char *>(p.mask) + mrow + s4));
                    m = make_float4(c.x, c.y, c.z, c.w);
                } else {
                    m = __ldg(reinterpret_cast<const float4 *>(static_cast<const float *>(p.mask) + mrow + s4));
                }
                apply(t[4 * j], m.x);
                apply(t[4 * j + 1], m.y);
                apply(t[4 * j + 2], m.z);
                apply(t[4 * j + 3], m.w);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const long long off = mrow + (long long)min(s0 + j, p.sk - 1) * p.m_s;
                apply(t[j], u8 ? (float)__ldg(static_cast<const unsigned char *>(p.mask) + off)
                               : __ldg(static_cast<const float *>(p.mask) + off));
            }
        }
    }
    if (s0 + 32 > p.sk) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (s0 + j >= p.sk) t[j] = -INFINITY;
    }
}

// P values rounded to the nearest TF32 value, ties away from zero (cvt.rna: the rounding a
// TFLOAT32 tensor map applies on load).
__device__ __forceinline__ float round_tf32_rna(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// NCH: 32-column slices of a row per thread (the four threads of a row take every fourth slice);
// FORM: the score program's form.
template <int NCH, int FORM>
__global__ void __launch_bounds__(THREADS, NCH == 1 ? 2 : 1) attention_kernel(const __grid_constant__ AttnParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t bar_qk, bar_v, bar_mma;
    __shared__ uint32_t tslot;
    __shared__ int abort_flag;
    __shared__ float red[4][QROWS];  // per row: the four threads' partial maximum, then sum
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sQ = base;                                  // dqp / 32 slices of 128 x 128 B
    uint8_t *sK = base + (uint32_t)p.dqp * 512u;         // skp x dqp fp32
    uint8_t *sP = base;                                  // skp / 32 slices of 128 x 128 B (over Q, K)
    uint8_t *sO = base;                                  // dvp / 32 slices of 128 x 128 B (over P)
    uint8_t *sV = base + p.region0;                      // skp x dvp fp32
    const int tid = threadIdx.x, warp = tid >> 5;
    const int row = tid & (QROWS - 1);   // query row = TMEM lane (warp w reads lanes 32 (w % 4) ...)
    const int part = tid >> 7;           // which of every four 32-column slices of the row
    const int qt = (int)(blockIdx.x % (unsigned)p.q_tiles);
    const int z = (int)(blockIdx.x / (unsigned)p.q_tiles);
    const int b1 = z % p.nb1, b2 = z / p.nb1;
    const int q0 = qt * QROWS;
    const int skc = p.skp >> 5, dqc = p.dqp >> 5, dvc = p.dvp >> 5;

    if (tid == 0) {
        mbar_init(&bar_qk, 1);
        mbar_init(&bar_v, 1);
        mbar_init(&bar_mma, 1);
        abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&p.tmQ);
        prefetch_tmap(&p.tmK);
        prefetch_tmap(&p.tmV);
        prefetch_tmap(&p.tmO);
    }
    if (warp == 0) tmem_alloc(&tslot, p.tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = tslot;

    // ---- loads and S = Q K^T ----
    if (tid == 0) {
        mbar_expect_tx(&bar_qk, (uint32_t)p.dqp * 512u + (uint32_t)p.skp * (uint32_t)p.dqp * 4u);
        for (int c = 0; c < dqc; ++c) tma_load_4d(sQ + c * CHUNK, &p.tmQ, &bar_qk, c * 32, q0, b1, b2);
        if (!p.k_mn)
            for (int c = 0; c < dqc; ++c) tma_load_4d(sK + c * p.skp * 128, &p.tmK, &bar_qk, c * 32, 0, b1, b2);
        else
            for (int c = 0; c < skc; ++c) tma_load_4d(sK + c * p.dqp * 128, &p.tmK, &bar_qk, c * 32, 0, b1, b2);
        mbar_expect_tx(&bar_v, (uint32_t)p.skp * (uint32_t)p.dvp * 4u);
        if (p.v_mn)
            for (int c = 0; c < dvc; ++c) tma_load_4d(sV + c * p.skp * 128, &p.tmV, &bar_v, c * 32, 0, b1, b2);
        else
            for (int c = 0; c < skc; ++c) tma_load_4d(sV + c * p.dvp * 128, &p.tmV, &bar_v, c * 32, 0, b1, b2);
        if (mbar_wait(&bar_qk, 0)) {
            tc_fence_after();
            const uint32_t idesc = instr_desc_tf32(p.skp) | ((uint32_t)p.k_mn << 16);
            const uint32_t qa = smem_addr(sQ), ka = smem_addr(sK);
            for (int ks = 0; ks < (p.dqp >> 3); ++ks)
                mma_tf32(tbase, sw128_desc(qa + (uint32_t)(ks >> 2) * CHUNK + (uint32_t)(ks & 3) * 32u),
                         b_desc(ka, p.k_mn, ks, p.skp, p.dqp), idesc, ks > 0 ? 1u : 0u);
            mma_commit(&bar_mma);
        } else {
            abort_flag = 1;
            umma::set_error(p.err, MGC_CUDA_TIMEOUT);
            mbar_arrive(&bar_mma);
        }
    }
    __syncwarp();
    // rows past Sq are TMA zero fill, never stored: they read row 0's mask (in bounds)
    const int q = q0 + row;
    const long long mrow = (long long)b1 * p.m_b1 + (long long)b2 * p.m_b2 + (long long)(q < p.sq ? q : 0) * p.m_q;
    bool ok = mbar_wait(&bar_mma, 0);
    tc_fence_after();
    ok = __syncthreads_and(ok && !*(volatile int *)&abort_flag) != 0;

    // ---- the row program and softmax, P into shared memory ----
    const uint32_t trow = tbase + ((uint32_t)((warp & 3) * 32) << 16);
    float v[NCH][32];
    float mx = -INFINITY;
    if (ok) {
#pragma unroll
        for (int j = 0; j < NCH; ++j) {
            const int c = part + 4 * j;
            if (c < skc) {  // warp-uniform
                uint32_t r[32];
                tmem_ld32(trow + (uint32_t)(c * 32), r);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) v[j][i] = __uint_as_float(r[i]);
                score_program<FORM>(p, v[j], c * 32, mrow);
#pragma unroll
                for (int i = 0; i < 32; ++i) mx = fmaxf(mx, v[j][i]);
            }
        }
    }
    red[part][row] = mx;
    __syncthreads();
    float sum = 0.0f;
    if (ok) {
        const float mr = fmaxf(fmaxf(red[0][row], red[1][row]), fmaxf(red[2][row], red[3][row]));
#pragma unroll
        for (int j = 0; j < NCH; ++j) {
            if (part + 4 * j < skc) {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    v[j][i] = __expf(v[j][i] - mr);
                    sum += v[j][i];
                }
            }
        }
    }
    __syncthreads();  // every maximum read before the sums overwrite them
    red[part][row] = sum;
    __syncthreads();
    if (ok) {
        const float inv = 1.0f / ((red[0][row] + red[1][row]) + (red[2][row] + red[3][row]));
        const uint32_t prow = smem_addr(sP) + (uint32_t)row * 128u;
#pragma unroll
        for (int j = 0; j < NCH; ++j) {
            const int c = part + 4 * j;
            if (c < skc) {
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    sts4(prow + (uint32_t)c * CHUNK + ((uint32_t)(u ^ (row & 7)) << 4),
                         make_float4(round_tf32_rna(v[j][4 * u] * inv), round_tf32_rna(v[j][4 * u + 1] * inv),
                                     round_tf32_rna(v[j][4 * u + 2] * inv), round_tf32_rna(v[j][4 * u + 3] * inv)));
            }
        }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    // ---- O = P V ----
    if (tid == 0) {
        tc_fence_after();
        if (ok && mbar_wait(&bar_v, 0)) {
            const uint32_t idesc = instr_desc_tf32(p.dvp) | ((uint32_t)p.v_mn << 16);
            const uint32_t pa = smem_addr(sP), va = smem_addr(sV);
            for (int ks = 0; ks < (p.skp >> 3); ++ks)
                mma_tf32(tbase, sw128_desc(pa + (uint32_t)(ks >> 2) * CHUNK + (uint32_t)(ks & 3) * 32u),
                         b_desc(va, p.v_mn, ks, p.dvp, p.skp), idesc, ks > 0 ? 1u : 0u);
            mma_commit(&bar_mma);
        } else {
            if (ok) {
                abort_flag = 1;
                umma::set_error(p.err, MGC_CUDA_TIMEOUT);
            }
            mbar_arrive(&bar_mma);
        }
    }
    __syncwarp();
    bool ok2 = mbar_wait(&bar_mma, 1);
    tc_fence_after();
    ok2 = __syncthreads_and(ok2 && ok && !*(volatile int *)&abort_flag) != 0;

    // ---- O rows into shared memory (over P), then TMA stores ----
    if (ok2) {
        // Dv <= 128: at most one 32-column slice of O per thread, in two halves of 16
        const int c = part;
        if (c < dvc) {  // warp-uniform
            const uint32_t orow = smem_addr(sO) + (uint32_t)c * CHUNK + (uint32_t)row * 128u;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint32_t r[16];
                umma::tmem_ld16(trow + (uint32_t)(c * 32 + h * 16), r);
                tmem_wait_ld();
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    sts4(orow + ((uint32_t)((4 * h + u) ^ (row & 7)) << 4),
                         make_float4(__uint_as_float(r[4 * u]), __uint_as_float(r[4 * u + 1]),
                                     __uint_as_float(r[4 * u + 2]), __uint_as_float(r[4 * u + 3])));
            }
        }
        fence_proxy_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && ok2) {
        for (int c = 0; c < dvc; ++c) tma_store_4d(&p.tmO, sO + c * CHUNK, c * 32, q0, b1, b2);
        umma::tma_store_commit_and_wait();
    }
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tbase, p.tmem_cols);
    }
}

// ---- host side ---------------------------------------------------------------------------------
// One decoded MGC_K_ATTENTION record: element strides of the operands' rows and of their two
// batch dimensions (b1 inner, b2 outer); the contiguous axis of each operand is implied (Q, O:
// the head width; K: Dqk when k_mn is 0, Sk when 1; V: Dv when v_mn is 1, Sk when 0).
struct AttnArgs {
    int nb1, nb2, sq, sk, dqk, dv;
    const float *q; long long q_rs, q_b1, q_b2;
    const float *k; int k_mn; long long k_rs, k_b1, k_b2;
    const float *v; int v_mn; long long v_rs, v_b1, v_b2;
    float *o; long long o_rs, o_b1, o_b2;
    int mode, div, mask_dt;
    const void *mask; long long m_b1, m_b2, m_q, m_s;
    float scale, lit;
    int *err;
};

inline long long round32(long long v) { return (v + 31) / 32 * 32; }

// Bytes of the Q + K / P / O region and the dynamic shared memory of a launch (0: too large).
inline uint32_t attn_smem(long long skp, long long dqp, long long dvp, uint32_t *region0) {
    long long r0 = skp * 512;
    if (dqp * 512 + skp * dqp * 4 > r0) r0 = dqp * 512 + skp * dqp * 4;
    if (dvp * 512 > r0) r0 = dvp * 512;
    const long long total = 1024 + r0 + skp * dvp * 4;
    if (total > (long long)umma::SMEM_LIMIT - 1024) return 0;
    *region0 = (uint32_t)r0;
    return (uint32_t)total;
}

// Whether the fused kernel takes a problem of these extents (the lowering fuses only these).
inline bool attn_fits(long long sk, long long dqk, long long dv) {
    uint32_t r0;
    return sk >= 1 && sk <= MAX_SK && dqk >= 4 && dqk <= MAX_D && dv >= 4 && dv <= MAX_D && dqk % 4 == 0 &&
           dv % 4 == 0 && attn_smem(round32(sk), round32(dqk), round32(dv), &r0) != 0;
}

// fp32 tensor {cols, rows, b1, b2} with element strides (row, b1, b2), boxes {32, box_rows, 1, 1}.
inline bool attn_map(CUtensorMap *map, const void *base, long long cols, long long rows, long long b1, long long b2,
                     long long rs, long long s1, long long s2, int box_rows, CUtensorMapSwizzle swizzle, bool tf32) {
    auto fn = umma::encode_tiled_fn();
    if (!fn) return false;
    cuuint64_t dims[4] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)b1, (cuuint64_t)b2};
    cuuint64_t strides[3] = {(cuuint64_t)(rs * 4), (cuuint64_t)(s1 * 4), (cuuint64_t)(s2 * 4)};
    cuuint32_t box[4] = {32u, (cuuint32_t)box_rows, 1u, 1u};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(map, tf32 ? CU_TENSOR_MAP_DATA_TYPE_TFLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4,
                    const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

inline int launch_attention(const AttnArgs &a, cudaStream_t stream) {
    if (a.nb1 <= 0 || a.nb2 <= 0 || a.sq <= 0 || !attn_fits(a.sk, a.dqk, a.dv))
        return fail(MGC_CUDA_UNSUPPORTED, "attention: Sq %d, Sk %d, Dqk %d, Dv %d", a.sq, a.sk, a.dqk, a.dv);
    if (!a.q || !a.k || !a.v || !a.o || (a.mode != MASK_NONE && !a.mask) || a.mode < 0 || a.mode > MASK_FILL)
        return fail(MGC_CUDA_BAD_ARGUMENT, "attention: missing operand");
    auto al = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    auto st = [](long long v) { return v > 0 && (v & 3) == 0 && v < (1ll << 36); };
    // strides of batch dimensions of extent 1 (never stepped): any valid value
    auto b1s = [&](long long s, long long rs, long long rows) { return a.nb1 > 1 ? s : rs * rows; };
    auto b2s = [&](long long s, long long s1) { return a.nb2 > 1 ? s : s1 * a.nb1; };
    const long long qs1 = b1s(a.q_b1, a.q_rs, a.sq), qs2 = b2s(a.q_b2, qs1);
    const long long krows = a.k_mn ? a.dqk : a.sk, vrows = a.v_mn ? a.sk : a.dv;
    const long long ks1 = b1s(a.k_b1, a.k_rs, krows), ks2 = b2s(a.k_b2, ks1);
    const long long vs1 = b1s(a.v_b1, a.v_rs, vrows), vs2 = b2s(a.v_b2, vs1);
    const long long os1 = b1s(a.o_b1, a.o_rs, a.sq), os2 = b2s(a.o_b2, os1);
    if (!al(a.q) || !al(a.k) || !al(a.v) || !al(a.o) || !st(a.q_rs) || !st(a.k_rs) || !st(a.v_rs) || !st(a.o_rs) ||
        !st(qs1) || !st(qs2) || !st(ks1) || !st(ks2) || !st(vs1) || !st(vs2) || !st(os1) || !st(os2))
        return fail(MGC_CUDA_UNSUPPORTED, "attention: operands need 16-byte aligned rows and batch strides");
    const long long skp = round32(a.sk), dqp = round32(a.dqk), dvp = round32(a.dv);
    AttnParams p;
    memset(&p, 0, sizeof p);
    const bool ok =
        attn_map(&p.tmQ, a.q, a.dqk, a.sq, a.nb1, a.nb2, a.q_rs, qs1, qs2, QROWS, CU_TENSOR_MAP_SWIZZLE_128B, true) &&
        (a.k_mn ? attn_map(&p.tmK, a.k, a.sk, a.dqk, a.nb1, a.nb2, a.k_rs, ks1, ks2, (int)dqp,
                           CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, true)
                : attn_map(&p.tmK, a.k, a.dqk, a.sk, a.nb1, a.nb2, a.k_rs, ks1, ks2, (int)skp,
                           CU_TENSOR_MAP_SWIZZLE_128B, true)) &&
        (a.v_mn ? attn_map(&p.tmV, a.v, a.dv, a.sk, a.nb1, a.nb2, a.v_rs, vs1, vs2, (int)skp,
                           CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, true)
                : attn_map(&p.tmV, a.v, a.sk, a.dv, a.nb1, a.nb2, a.v_rs, vs1, vs2, (int)dvp,
                           CU_TENSOR_MAP_SWIZZLE_128B, true)) &&
        attn_map(&p.tmO, a.o, a.dv, a.sq, a.nb1, a.nb2, a.o_rs, os1, os2, QROWS, CU_TENSOR_MAP_SWIZZLE_128B, false);
    if (!ok) return fail(MGC_CUDA_UNSUPPORTED, "attention: tensor map encoding failed");
    p.mask = a.mask;
    p.m_b1 = a.m_b1; p.m_b2 = a.m_b2; p.m_q = a.m_q; p.m_s = a.m_s;
    p.scale = a.scale; p.lit = a.lit;
    p.mode = a.mode; p.div = a.div;
    p.mask_u8 = a.mask_dt == MGC_U8 || a.mask_dt == MGC_BOOL;
    if (a.mode != MASK_NONE && !p.mask_u8 && a.mask_dt != MGC_F32)
        return fail(MGC_CUDA_UNSUPPORTED, "attention: mask of type %d", a.mask_dt);
    if (a.mode == MASK_ADD || a.mode == MASK_SUB) {
        if (p.mask_u8) return fail(MGC_CUDA_UNSUPPORTED, "attention: additive mask must be fp32");
    } else if (a.mode != MASK_NONE && !p.mask_u8) {
        return fail(MGC_CUDA_UNSUPPORTED, "attention: Where condition must be bool / uint8");
    }
    const uintptr_t malign = p.mask_u8 ? 3 : 15;
    p.mask_vec = a.mode != MASK_NONE && a.m_s == 1 && (reinterpret_cast<uintptr_t>(a.mask) & malign) == 0 &&
                 a.m_b1 % 4 == 0 && a.m_b2 % 4 == 0 && a.m_q % 4 == 0 && a.sk % 4 == 0;
    p.sq = a.sq; p.sk = a.sk;
    p.skp = (int)skp; p.dqp = (int)dqp; p.dvp = (int)dvp;
    p.k_mn = a.k_mn; p.v_mn = a.v_mn;
    p.nb1 = a.nb1;
    p.q_tiles = (int)ceil_div(a.sq, QROWS);
    uint32_t cols = 32;
    while (cols < (uint32_t)(skp > dvp ? skp : dvp)) cols <<= 1;
    p.tmem_cols = cols;
    const uint32_t smem = attn_smem(skp, dqp, dvp, &p.region0);
    p.err = a.err;
    const long long grid = (long long)p.q_tiles * a.nb1 * a.nb2;
    if (grid > 0x7FFFFFFF) return fail(MGC_CUDA_UNSUPPORTED, "attention: %lld tiles", grid);
    // the score program's compiled form, else the generic one
    int form = FORM_GENERIC;
    if (!a.div && a.mode == MASK_NONE) form = FORM_MUL;
    else if (!a.div && p.mask_vec && a.mode == MASK_ADD && !p.mask_u8) form = FORM_MUL_ADD;
    else if (!a.div && p.mask_vec && a.mode == MASK_FILL && p.mask_u8) form = FORM_MUL_FILL;
    else if (!a.div && p.mask_vec && a.mode == MASK_KEEP && p.mask_u8) form = FORM_MUL_KEEP;
    auto go = [&](auto kern) -> int {
        MGC_CHECK(raise_smem_ceiling((const void *)kern));
        kern<<<(unsigned)grid, THREADS, smem, stream>>>(p);
        return check_launch("attention_kernel");
    };
    const bool one = skp <= 128;  // one 32-column slice per thread
    switch (form) {
    case FORM_MUL: return one ? go(attention_kernel<1, FORM_MUL>) : go(attention_kernel<2, FORM_MUL>);
    case FORM_MUL_ADD: return one ? go(attention_kernel<1, FORM_MUL_ADD>) : go(attention_kernel<2, FORM_MUL_ADD>);
    case FORM_MUL_FILL: return one ? go(attention_kernel<1, FORM_MUL_FILL>) : go(attention_kernel<2, FORM_MUL_FILL>);
    case FORM_MUL_KEEP: return one ? go(attention_kernel<1, FORM_MUL_KEEP>) : go(attention_kernel<2, FORM_MUL_KEEP>);
    default: return one ? go(attention_kernel<1, FORM_GENERIC>) : go(attention_kernel<2, FORM_GENERIC>);
    }
}

}  // namespace attn
}  // namespace mgc
