// Exact-fp32 GEMM on the CUDA cores with the fused epilogue. It runs every GEMM-family launch
// the tensor-core kernel does not take (NCHW convolutions, grouped convolutions, operands whose
// strides TMA cannot describe, MGC_PREC_FP32 requests) and is the arithmetic baseline the
// tcgen05 path is checked against.
//
// Reference: mgc_gemm / gemm_task / pack_a / pack_b / epilogue (mgc_kernels.c:86-396) with the
// operand kinds of mgc_runtime.h:123-137: STRIDED, CONV_NHWC (A rows are output pixels, columns
// (kh*KW + kw)*cg + c) and CONV_NCHW (B rows (c*KH + kh)*KW + kw, columns output pixels).
// Unlike the CPU driver, NHWC convolutions fold the batch into M (row m = image*OH*OW + pixel)
// so small feature maps still fill the GPU.
#pragma once

#include "common.cuh"
#include "kernels_norm.cuh"

namespace mgc {

struct GemmParams {
    int M, N, K;
    int nb;                       // batch dimensions (0..4)
    long long bdims[4];
    long long a_bs[4], b_bs[4], c_bs[4], r_bs[4];  // element strides per batch dimension
    int a_kind, b_kind;
    long long a_rs, a_cs, b_rs, b_cs;
    const float *a, *b;
    // convolution geometry of the implicit operand (A for CONV_NHWC, B for CONV_NCHW)
    int H, W, C, KH, KW, SH, SW, DH, DW, PT, PL, OH, OW, c_off, cg;
    float *c;
    long long ldc;
    float alpha, beta;
    int bias_mode;                // 0 none, 1 per column, 2 per row
    const float *bias, *res;
    long long ldr;
    int act;
    float lo, hi;
    int precision;
    const float *b_lo;            // residual of a split constant B (B = b + b_lo exactly), may be NULL
    // tensor-core layout of a constant B: K-major [N][Kp] (for im2col, K = (kh, kw, channel
    // padded to b_cpad)), TF32-rounded high part and fp32 residual; NULL when not provided
    const float *b_umma, *b_umma_lo;
    int b_cpad;
    // window-row layout of an im2col convolution over a spatially padded image: output pixels per
    // TMA box (0: not used) and the padded length of one window row (B is [N][KH][win_L])
    int win_rows, win_L;
    // phase-split rows (narrow stride-2 convolutions, TF32): A is a packed image whose rows hold
    // the even-tap and the odd-tap column phases of `phase_w` 4-channel pixels each (K_PACK with
    // phases); B is [N][KH][32] in the matching tap order. 0: not used
    int phase_w;
    // phase-split convolution followed by a 3x3 / stride-2 / pad-1 max pooling computed in its
    // epilogue: the pooled output's rows and columns (c is then the pooled output); 0: no pooling
    int pool_ph, pool_pw;
    // the output only feeds a GlobalAveragePool of gap_hw pixels per image: c receives the
    // tensor-core epilogue's 32-row partial sums instead (0: the output itself)
    int gap_hw;
    // TF32 mode: B may enter as its TF32 part alone (one weight plane; the wide pair forms use it)
    int one_plane;
    int *err;                     // device word for bounded-wait timeouts (may be NULL)
    // split-K scratch of the model (NULL: no split): room for the partial tiles
    float *split_ws;
    long long split_ws_floats;
};

__device__ __forceinline__ float fetch_a(const GemmParams &p, const float *a, long long m, long long k) {
    if (p.a_kind == MGC_CONV_NHWC) {
        const long long hw = (long long)p.OH * p.OW;
        const long long img = m / hw;
        const int pix = (int)(m - img * hw);
        const int oh = pix / p.OW, ow = pix - oh * p.OW;
        const int kwcg = p.KW * p.cg;
        const int kh = (int)(k / kwcg);
        const int rem = (int)(k - (long long)kh * kwcg);
        const int kw = rem / p.cg, c = rem - kw * p.cg;
        const int ih = oh * p.SH - p.PT + kh * p.DH, iw = ow * p.SW - p.PL + kw * p.DW;
        if (ih < 0 || ih >= p.H || iw < 0 || iw >= p.W) return 0.0f;
        return a[((img * p.H + ih) * p.W + iw) * p.C + p.c_off + c];
    }
    return a[m * p.a_rs + k * p.a_cs];
}

__device__ __forceinline__ float fetch_b(const GemmParams &p, const float *b, long long k, long long n) {
    if (p.b_kind == MGC_CONV_NCHW) {
        const int kw = (int)(k % p.KW);
        const long long t = k / p.KW;
        const int kh = (int)(t % p.KH), c = (int)(t / p.KH);
        const int oh = (int)(n / p.OW), ow = (int)(n % p.OW);
        const int ih = oh * p.SH - p.PT + kh * p.DH, iw = ow * p.SW - p.PL + kw * p.DW;
        if (ih < 0 || ih >= p.H || iw < 0 || iw >= p.W) return 0.0f;
        return b[((long long)(p.c_off + c) * p.H + ih) * p.W + iw];
    }
    return b[k * p.b_rs + n * p.b_cs];
}

constexpr int SG_BM = 64, SG_BN = 64, SG_BK = 16;

// 256 threads; each computes a 4x4 block of a 64x64 tile; grid (M tiles, N tiles, batch).
__global__ void __launch_bounds__(256) gemm_simt_kernel(const __grid_constant__ GemmParams p) {
    __shared__ float As[2][SG_BK][SG_BM + 4];
    __shared__ float Bs[2][SG_BK][SG_BN + 4];
    const int tid = threadIdx.x;
    const int tx = tid % 16, ty = tid / 16;
    const long long m0 = (long long)blockIdx.x * SG_BM, n0 = (long long)blockIdx.y * SG_BN;
    // batch offsets
    long long bi = blockIdx.z, aoff = 0, boff = 0, coff = 0, roff = 0;
    for (int d = p.nb - 1; d >= 0; --d) {
        long long i = bi % p.bdims[d];
        bi /= p.bdims[d];
        aoff += i * p.a_bs[d]; boff += i * p.b_bs[d]; coff += i * p.c_bs[d]; roff += i * p.r_bs[d];
    }
    const float *a = p.a + aoff;
    const float *b = p.b + boff;
    float acc[4][4] = {};
    // tile loaders: A 64x16 and B 16x64, 4 elements per thread each
    float ra[4], rb[4];
    auto load = [&](int k0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int e = tid + j * 256;            // 0..1023
            int am = e / SG_BK, ak = e % SG_BK;  // A: m-major walk
            long long gm = m0 + am, gk = k0 + ak;
            ra[j] = (gm < p.M && gk < p.K) ? fetch_a(p, a, gm, gk) : 0.0f;
            int bk = e / SG_BN, bn = e % SG_BN;
            long long gk2 = k0 + bk, gn = n0 + bn;
            rb[j] = (gk2 < p.K && gn < p.N) ? fetch_b(p, b, gk2, gn) : 0.0f;
            if (p.b_lo && gk2 < p.K && gn < p.N) rb[j] += p.b_lo[boff + gk2 * p.b_rs + gn * p.b_cs];
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int e = tid + j * 256;
            As[buf][e % SG_BK][e / SG_BK] = ra[j];
            Bs[buf][e / SG_BN][e % SG_BN] = rb[j];
        }
    };
    const int ktiles = (p.K + SG_BK - 1) / SG_BK;
    if (ktiles > 0) {
        load(0);
        store(0);
    }
    __syncthreads();
    for (int t = 0; t < ktiles; ++t) {
        const int buf = t & 1;
        if (t + 1 < ktiles) load((t + 1) * SG_BK);
#pragma unroll
        for (int kk = 0; kk < SG_BK; ++kk) {
            float av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) av[i] = As[buf][kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) bv[j] = Bs[buf][kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        if (t + 1 < ktiles) store(buf ^ 1);
        __syncthreads();
    }
    // epilogue: act(alpha*acc + bias + beta*res)  (mgc_kernels.c:282-323)
    float *c = p.c + coff;
    const float *res = p.res ? p.res + roff : nullptr;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const long long m = m0 + ty * 4 + i;
        if (m >= p.M) continue;
        const float rowb = (p.bias && p.bias_mode == 2) ? p.bias[m] : 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const long long n = n0 + tx * 4 + j;
            if (n >= p.N) continue;
            float v = p.alpha * acc[i][j] + rowb;
            if (p.bias && p.bias_mode == 1) v += p.bias[n];
            if (res) v += p.beta * res[m * p.ldr + n];
            c[m * p.ldc + n] = apply_act(v, p.act, p.lo, p.hi);
        }
    }
}

inline int launch_gemm_simt(const GemmParams &p, cudaStream_t stream) {
    long long batch = 1;
    for (int d = 0; d < p.nb; ++d) batch *= p.bdims[d];
    if (p.M <= 0 || p.N <= 0 || batch <= 0) return MGC_CUDA_OK;
    dim3 grid((unsigned)ceil_div(p.M, SG_BM), (unsigned)ceil_div(p.N, SG_BN), (unsigned)batch);
    if (grid.y > 65535u || grid.z > 65535u)
        return fail(MGC_CUDA_UNSUPPORTED, "gemm grid too large (M=%d, batch=%lld)", p.M, batch);
    gemm_simt_kernel<<<grid, 256, 0, stream>>>(p);
    return check_launch("gemm_simt_kernel");
}

}  // namespace mgc
