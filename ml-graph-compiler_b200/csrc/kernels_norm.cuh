// Row-wise and window kernels: softmax / log-softmax, layer normalization, max / average
// pooling and depthwise convolution.
//
// Reference kernels: mgc_kernels.c:618-655 (softmax), :657-679 (layer norm), :510-591 (pooling,
// window_count for count_include_pad and ceil-mode windows), :428-504 (depthwise NHWC / NCHW
// with bias, residual and activation). Semantics: ops.py:784-816, 1072-1134, 1023-1069.
#pragma once

#include <math.h>
#include "common.cuh"

namespace mgc {

__device__ inline float warp_sum(float v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ inline float warp_max(float v) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Activation epilogue shared by the GEMM, conv and depthwise kernels (mgc_runtime.h:103-113,
// ops.py:894-911), using CUDA's float math functions.
__device__ __forceinline__ float apply_act(float v, int act, float lo, float hi) {
    switch (act) {
    case MGC_ACT_RELU: return v > 0.0f ? v : 0.0f;
    case MGC_ACT_CLIP: return fminf(fmaxf(v, lo), hi);
    case MGC_ACT_GELU: return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
    case MGC_ACT_GELU_TANH:
        return 0.5f * v * (1.0f + tanhf(0.79788456080286536f * (v + 0.044715f * v * v * v)));
    case MGC_ACT_TANH: return tanhf(v);
    case MGC_ACT_SIGMOID: return 0.5f * (1.0f + tanhf(0.5f * v));
    default: return v;
    }
}

// ---------------------------------------------------------------------------------------------
// softmax over the middle axis of [outer, n, inner]: one warp per (outer, inner) row.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) softmax_kernel(long long outer, long long n, long long inner,
                                                      const float *x, float *y, int log_softmax) {
    const int lane = threadIdx.x & 31;
    const long long rows = outer * inner;
    const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
    for (long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows;
         row += warps) {
        const long long o = row / inner, i = row % inner;
        const float *src = x + o * n * inner + i;
        float *dst = y + o * n * inner + i;
        float m = -INFINITY;
        for (long long k = lane; k < n; k += 32) m = fmaxf(m, src[k * inner]);
        m = warp_max(m);
        float s = 0.0f;
        for (long long k = lane; k < n; k += 32) s += expf(src[k * inner] - m);
        s = warp_sum(s);
        if (log_softmax) {
            const float ls = logf(s);
            for (long long k = lane; k < n; k += 32) dst[k * inner] = src[k * inner] - m - ls;
        } else {
            const float inv = 1.0f / s;
            for (long long k = lane; k < n; k += 32) dst[k * inner] = expf(src[k * inner] - m) * inv;
        }
    }
}

// ---------------------------------------------------------------------------------------------
// layer normalization of [rows, cols]: one warp per row, two passes (mean, then the sum of
// squared deviations) as mgc_layer_norm does, fp32 throughout.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) layer_norm_kernel(long long rows, long long cols, const float *x,
                                                         const float *scale, const float *bias,
                                                         float eps, float *y) {
    const int lane = threadIdx.x & 31;
    const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
    const bool vec = (cols % 4 == 0) && ((((uintptr_t)x) | ((uintptr_t)y)) % 16 == 0) &&
                     (!scale || ((uintptr_t)scale) % 16 == 0) && (!bias || ((uintptr_t)bias) % 16 == 0);
    for (long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const float *src = x + r * cols;
        float *dst = y + r * cols;
        float s = 0.0f;
        if (vec) {
            for (long long k = lane * 4; k < cols; k += 128) {
                float4 v = *(const float4 *)(src + k);
                s += (v.x + v.y) + (v.z + v.w);
            }
        } else {
            for (long long k = lane; k < cols; k += 32) s += src[k];
        }
        const float mean = warp_sum(s) / (float)cols;
        float q = 0.0f;
        if (vec) {
            for (long long k = lane * 4; k < cols; k += 128) {
                float4 v = *(const float4 *)(src + k);
                float a = v.x - mean, b = v.y - mean, c = v.z - mean, d = v.w - mean;
                q += (a * a + b * b) + (c * c + d * d);
            }
        } else {
            for (long long k = lane; k < cols; k += 32) {
                float d = src[k] - mean;
                q += d * d;
            }
        }
        const float inv = 1.0f / sqrtf(warp_sum(q) / (float)cols + eps);
        if (vec) {
            for (long long k = lane * 4; k < cols; k += 128) {
                float4 v = *(const float4 *)(src + k);
                float4 o;
                o.x = (v.x - mean) * inv; o.y = (v.y - mean) * inv;
                o.z = (v.z - mean) * inv; o.w = (v.w - mean) * inv;
                if (scale) {
                    float4 g = *(const float4 *)(scale + k);
                    o.x *= g.x; o.y *= g.y; o.z *= g.z; o.w *= g.w;
                }
                if (bias) {
                    float4 b = *(const float4 *)(bias + k);
                    o.x += b.x; o.y += b.y; o.z += b.z; o.w += b.w;
                }
                *(float4 *)(dst + k) = o;
            }
        } else {
            for (long long k = lane; k < cols; k += 32) {
                float v = (src[k] - mean) * inv;
                if (scale) v *= scale[k];
                if (bias) v += bias[k];
                dst[k] = v;
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// pooling
// ---------------------------------------------------------------------------------------------
struct PoolParams {
    int is_max, N, H, W, C, KH, KW, SH, SW, DH, DW, PT, PL, PB, PR, OH, OW, include_pad, nhwc;
    const float *x;
    float *y;
};

__device__ inline int window_count(const PoolParams &p, int oh, int ow) {
    int count = 0;
    for (int kh = 0; kh < p.KH; ++kh) {
        int ih = oh * p.SH - p.PT + kh * p.DH;
        bool in_h = p.include_pad ? (ih >= -p.PT && ih < p.H + p.PB) : (ih >= 0 && ih < p.H);
        if (!in_h) continue;
        for (int kw = 0; kw < p.KW; ++kw) {
            int iw = ow * p.SW - p.PL + kw * p.DW;
            bool in_w = p.include_pad ? (iw >= -p.PL && iw < p.W + p.PR) : (iw >= 0 && iw < p.W);
            if (in_w) ++count;
        }
    }
    return count;
}

__global__ void __launch_bounds__(256) pool_kernel(const __grid_constant__ PoolParams p) {
    const long long total = (long long)p.N * p.OH * p.OW * p.C;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
        int c, ow, oh, n;
        if (p.nhwc) {
            c = (int)(e % p.C);
            long long r = e / p.C;
            ow = (int)(r % p.OW); r /= p.OW;
            oh = (int)(r % p.OH);
            n = (int)(r / p.OH);
        } else {
            ow = (int)(e % p.OW);
            long long r = e / p.OW;
            oh = (int)(r % p.OH); r /= p.OH;
            c = (int)(r % p.C);
            n = (int)(r / p.C);
        }
        float acc = p.is_max ? -INFINITY : 0.0f;
        for (int kh = 0; kh < p.KH; ++kh) {
            int ih = oh * p.SH - p.PT + kh * p.DH;
            if (ih < 0 || ih >= p.H) continue;
            for (int kw = 0; kw < p.KW; ++kw) {
                int iw = ow * p.SW - p.PL + kw * p.DW;
                if (iw < 0 || iw >= p.W) continue;
                long long src = p.nhwc ? (((long long)n * p.H + ih) * p.W + iw) * p.C + c
                                       : (((long long)n * p.C + c) * p.H + ih) * p.W + iw;
                float v = p.x[src];
                acc = p.is_max ? (v > acc ? v : acc) : acc + v;
            }
        }
        if (!p.is_max) {
            int cnt = window_count(p, oh, ow);
            acc = cnt > 0 ? acc * (1.0f / (float)cnt) : 0.0f;
        }
        p.y[e] = acc;
    }
}

// NHWC pooling, four channels per thread (C % 4 == 0, 16-byte aligned x and y): the same window
// walk and the same comparisons as pool_kernel (a NaN never replaces the running maximum), with
// 16-byte loads and stores and 32-bit index arithmetic (the caller checks the sizes fit).
__global__ void __launch_bounds__(256) pool4_nhwc_kernel(const __grid_constant__ PoolParams p) {
    const int c4n = p.C >> 2;
    const unsigned total = (unsigned)p.N * p.OH * p.OW * c4n;
    const unsigned stride = gridDim.x * blockDim.x;
    const float4 *x4 = reinterpret_cast<const float4 *>(p.x);
    float4 *y4 = reinterpret_cast<float4 *>(p.y);
    for (unsigned e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
        const int c4 = (int)(e % c4n);
        unsigned r = e / c4n;
        const int ow = (int)(r % p.OW);
        r /= p.OW;
        const int oh = (int)(r % p.OH);
        const int n = (int)(r / p.OH);
        const float init = p.is_max ? -INFINITY : 0.0f;
        float4 acc = make_float4(init, init, init, init);
        for (int kh = 0; kh < p.KH; ++kh) {
            const int ih = oh * p.SH - p.PT + kh * p.DH;
            if (ih < 0 || ih >= p.H) continue;
            const unsigned rowbase = ((unsigned)n * p.H + ih) * p.W;
            for (int kw = 0; kw < p.KW; ++kw) {
                const int iw = ow * p.SW - p.PL + kw * p.DW;
                if (iw < 0 || iw >= p.W) continue;
                const float4 v = __ldg(x4 + (size_t)(rowbase + iw) * c4n + c4);
                if (p.is_max) {
                    acc.x = v.x > acc.x ? v.x : acc.x;
                    acc.y = v.y > acc.y ? v.y : acc.y;
                    acc.z = v.z > acc.z ? v.z : acc.z;
                    acc.w = v.w > acc.w ? v.w : acc.w;
                } else {
                    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
                }
            }
        }
        if (!p.is_max) {
            const int cnt = window_count(p, oh, ow);
            const float inv = 1.0f / (float)cnt;
            acc = cnt > 0 ? make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        y4[e] = acc;
    }
}

// ---------------------------------------------------------------------------------------------
// depthwise convolution (one input channel per group) with bias, residual and activation
// ---------------------------------------------------------------------------------------------
struct DepthwiseParams {
    int N, H, W, C, KH, KW, SH, SW, DH, DW, PT, PL, OH, OW, nhwc, act;
    float lo, hi;
    const float *x, *w, *bias, *res;
    float *y;
};

// NHWC: one thread per (pixel, 4 channels) when C % 4 == 0, channels contiguous; weights HWC.
__global__ void __launch_bounds__(256) depthwise_nhwc4_kernel(const __grid_constant__ DepthwiseParams p) {
    const int C4 = p.C / 4;
    const long long total = (long long)p.N * p.OH * p.OW * C4;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
        const int c = (int)(e % C4) * 4;
        long long r = e / C4;
        const int ow = (int)(r % p.OW); r /= p.OW;
        const int oh = (int)(r % p.OH);
        const int n = (int)(r / p.OH);
        float4 acc = p.bias ? *(const float4 *)(p.bias + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        const float *img = p.x + (long long)n * p.H * p.W * p.C;
        for (int kh = 0; kh < p.KH; ++kh) {
            const int ih = oh * p.SH - p.PT + kh * p.DH;
            if (ih < 0 || ih >= p.H) continue;
            for (int kw = 0; kw < p.KW; ++kw) {
                const int iw = ow * p.SW - p.PL + kw * p.DW;
                if (iw < 0 || iw >= p.W) continue;
                const float4 v = *(const float4 *)(img + ((long long)ih * p.W + iw) * p.C + c);
                const float4 k = *(const float4 *)(p.w + ((long long)kh * p.KW + kw) * p.C + c);
                acc.x = fmaf(v.x, k.x, acc.x); acc.y = fmaf(v.y, k.y, acc.y);
                acc.z = fmaf(v.z, k.z, acc.z); acc.w = fmaf(v.w, k.w, acc.w);
            }
        }
        const long long o = e * 4;
        if (p.res) {
            const float4 rr = *(const float4 *)(p.res + o);
            acc.x += rr.x; acc.y += rr.y; acc.z += rr.z; acc.w += rr.w;
        }
        acc.x = apply_act(acc.x, p.act, p.lo, p.hi); acc.y = apply_act(acc.y, p.act, p.lo, p.hi);
        acc.z = apply_act(acc.z, p.act, p.lo, p.hi); acc.w = apply_act(acc.w, p.act, p.lo, p.hi);
        *(float4 *)(p.y + o) = acc;
    }
}

// NHWC, C % 4 == 0, KH, KW <= 3, sizes below 2^31: each thread keeps one 4-channel group (the
// block size is a multiple of C / 4, so the group never changes along the grid-stride loop) with
// its bias and up to 3x3 weights in registers, and walks output pixels with 32-bit index
// arithmetic. Same accumulation order as depthwise_nhwc4_kernel (bias, then taps row by row).
__global__ void __launch_bounds__(256) depthwise_nhwc4_reg_kernel(const __grid_constant__ DepthwiseParams p) {
    const int C4 = p.C >> 2;
    const int c4 = (int)(threadIdx.x % (unsigned)C4);
    const unsigned pix_per_block = blockDim.x / C4;
    const unsigned npix = (unsigned)p.N * p.OH * p.OW;
    const float4 *x4 = reinterpret_cast<const float4 *>(p.x);
    const float4 *w4 = reinterpret_cast<const float4 *>(p.w);
    float4 wk[9];  // [kh][kw] of a 3x3 frame, zero outside KH x KW (static indices only)
#pragma unroll
    for (int t = 0; t < 9; ++t) {
        const int kh = t / 3, kw = t % 3;
        wk[t] = (kh < p.KH && kw < p.KW) ? __ldg(w4 + (kh * p.KW + kw) * C4 + c4) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const float4 b = p.bias ? __ldg(reinterpret_cast<const float4 *>(p.bias) + c4) : make_float4(0.f, 0.f, 0.f, 0.f);
    for (unsigned pix = blockIdx.x * pix_per_block + threadIdx.x / C4; pix < npix; pix += gridDim.x * pix_per_block) {
        const unsigned ow = pix % p.OW, r = pix / p.OW;
        const unsigned oh = r % p.OH, n = r / p.OH;
        float4 acc = b;
#pragma unroll
        for (int kh = 0; kh < 3; ++kh) {
            if (kh >= p.KH) break;
            const int ih = (int)oh * p.SH - p.PT + kh * p.DH;
            if (ih < 0 || ih >= p.H) continue;
            const unsigned rowbase = (n * p.H + ih) * p.W;
#pragma unroll
            for (int kw = 0; kw < 3; ++kw) {
                if (kw >= p.KW) break;
                const int iw = (int)ow * p.SW - p.PL + kw * p.DW;
                if (iw < 0 || iw >= p.W) continue;
                const float4 v = __ldg(x4 + (size_t)(rowbase + iw) * C4 + c4);
                const float4 k = wk[kh * 3 + kw];
                acc.x = fmaf(v.x, k.x, acc.x); acc.y = fmaf(v.y, k.y, acc.y);
                acc.z = fmaf(v.z, k.z, acc.z); acc.w = fmaf(v.w, k.w, acc.w);
            }
        }
        const size_t o = (size_t)pix * C4 + c4;
        if (p.res) {
            const float4 rr = reinterpret_cast<const float4 *>(p.res)[o];
            acc.x += rr.x; acc.y += rr.y; acc.z += rr.z; acc.w += rr.w;
        }
        if (p.act == MGC_ACT_RELU) {
            acc.x = fmaxf(acc.x, 0.0f); acc.y = fmaxf(acc.y, 0.0f); acc.z = fmaxf(acc.z, 0.0f); acc.w = fmaxf(acc.w, 0.0f);
        } else if (p.act == MGC_ACT_CLIP) {
            acc.x = fminf(fmaxf(acc.x, p.lo), p.hi); acc.y = fminf(fmaxf(acc.y, p.lo), p.hi);
            acc.z = fminf(fmaxf(acc.z, p.lo), p.hi); acc.w = fminf(fmaxf(acc.w, p.lo), p.hi);
        } else if (p.act != MGC_ACT_NONE) {
            acc.x = apply_act(acc.x, p.act, p.lo, p.hi); acc.y = apply_act(acc.y, p.act, p.lo, p.hi);
            acc.z = apply_act(acc.z, p.act, p.lo, p.hi); acc.w = apply_act(acc.w, p.act, p.lo, p.hi);
        }
        reinterpret_cast<float4 *>(p.y)[o] = acc;
    }
}

// Any C, either layout (NCHW weights CHW).
__global__ void __launch_bounds__(256) depthwise_kernel(const __grid_constant__ DepthwiseParams p) {
    const long long total = (long long)p.N * p.OH * p.OW * p.C;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
        int c, ow, oh, n;
        if (p.nhwc) {
            c = (int)(e % p.C);
            long long r = e / p.C;
            ow = (int)(r % p.OW); r /= p.OW;
            oh = (int)(r % p.OH);
            n = (int)(r / p.OH);
        } else {
            ow = (int)(e % p.OW);
            long long r = e / p.OW;
            oh = (int)(r % p.OH); r /= p.OH;
            c = (int)(r % p.C);
            n = (int)(r / p.C);
        }
        float acc = p.bias ? p.bias[c] : 0.0f;
        for (int kh = 0; kh < p.KH; ++kh) {
            const int ih = oh * p.SH - p.PT + kh * p.DH;
            if (ih < 0 || ih >= p.H) continue;
            for (int kw = 0; kw < p.KW; ++kw) {
                const int iw = ow * p.SW - p.PL + kw * p.DW;
                if (iw < 0 || iw >= p.W) continue;
                float v, k;
                if (p.nhwc) {
                    v = p.x[(((long long)n * p.H + ih) * p.W + iw) * p.C + c];
                    k = p.w[((long long)kh * p.KW + kw) * p.C + c];
                } else {
                    v = p.x[(((long long)n * p.C + c) * p.H + ih) * p.W + iw];
                    k = p.w[((long long)c * p.KH + kh) * p.KW + kw];
                }
                acc = fmaf(v, k, acc);
            }
        }
        if (p.res) acc += p.res[e];
        p.y[e] = apply_act(acc, p.act, p.lo, p.hi);
    }
}

}  // namespace mgc
