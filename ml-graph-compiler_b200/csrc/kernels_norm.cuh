// Row-wise and window kernels: softmax / log-softmax, layer normalization, max / average
// pooling and depthwise convolution.
//
// Reference kernels: mgc_kernels.c:618-655 (softmax), :657-679 (layer norm), :510-591 (pooling,
// window_count for count_include_pad and ceil-mode windows), :428-504 (depthwise NHWC / NCHW
// with bias, residual and activation). Semantics: ops.py:784-816, 1072-1134, 1023-1069.
#pragma once

#include <math.h>
#include "common.cuh"
#include "kernels_mem.cuh"

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

// Softmax / log-softmax of rows of n contiguous elements (n % 4 == 0, n <= 128 * CH): one warp
// per R rows holds them in registers (CH groups of four per lane and row), so every row is read
// once and written once, and the loads of R rows are in flight together. Exponentials use the
// fast __expf (relative error about |x| * 6e-8 for an argument x <= 0, far inside the tf32 and
// strict budgets). With PROG the rows are
// the output of the elementwise program P (the scale and mask of attention scores) evaluated as
// they are read, so that output never reaches memory: PROG 1 for chain programs (instruction by
// instruction over all R x CH groups, each leaf's offset at a row start in shared memory),
// PROG 2 for any other ew_f32x4_form program (ew_run4, register file in local memory), PROG 3
// for the scale-and-mask form of attention scores (ScaleMask: no interpretation at all).
constexpr int SOFTMAX_ROW_MAX = 1024;

// Attention's score program, recognised so that the softmax runs it without interpreting it:
// t = X * s or X / s (X fp32 laid out as the output, s an fp32 literal), then optionally
// t + M, t - M (M an fp32 tensor leaf, any broadcast), Where(C, t, lit) or Where(C, lit, t)
// (C a bool / uint8 leaf). The operations are the ones ew_f32 runs, in the same order.
struct ScaleMask {
    int x_leaf, s_leaf, div;  // t = X * s (div 0) or X / s (div 1)
    int mode;                 // 0 t, 1 t + M, 2 t - M, 3 Where(C, t, lit), 4 Where(C, lit, t)
    int m_leaf, lit_leaf;     // M or C; the Where literal
};

inline bool scale_mask_form(const EwParams &P, ScaleMask &sm) {
    if (P.ninstr < 1 || P.ninstr > 2) return false;
    auto tensor = [&](int a, bool f32) {
        return a >= 0 && a < P.nleaves && !P.leaves[a].is_lit && (f32 ? P.leaves[a].dtype == MGC_F32
                                                                       : (P.leaves[a].dtype == MGC_BOOL ||
                                                                          P.leaves[a].dtype == MGC_U8));
    };
    auto literal = [&](int a) { return a >= 0 && a < P.nleaves && P.leaves[a].is_lit && P.leaves[a].dtype == MGC_F32; };
    auto dense = [&](int a) {
        long long want = 1;
        for (int d = P.rank - 1; d >= 0; --d) {
            if (P.shape[d] != 1 && P.leaves[a].strides[d] != want) return false;
            want *= P.shape[d];
        }
        return true;
    };
    const EwInstr &i0 = P.ins[0];
    if (i0.a[2] >= 0 || i0.out_dt != MGC_F32) return false;
    if (i0.op == EW_MUL && tensor(i0.a[0], true) && literal(i0.a[1])) { sm.x_leaf = i0.a[0]; sm.s_leaf = i0.a[1]; }
    else if (i0.op == EW_MUL && literal(i0.a[0]) && tensor(i0.a[1], true)) { sm.x_leaf = i0.a[1]; sm.s_leaf = i0.a[0]; }
    else if (i0.op == EW_DIV && tensor(i0.a[0], true) && literal(i0.a[1])) { sm.x_leaf = i0.a[0]; sm.s_leaf = i0.a[1]; }
    else return false;
    sm.div = i0.op == EW_DIV;
    if (!dense(sm.x_leaf)) return false;
    sm.mode = 0;
    sm.m_leaf = sm.lit_leaf = 0;
    if (P.ninstr == 1) return true;
    const EwInstr &i1 = P.ins[1];
    const int t = P.nleaves;  // the register of the first instruction's result
    if (i1.out_dt != MGC_F32) return false;
    if (i1.op == EW_ADD && i1.a[2] < 0 && i1.a[0] == t && tensor(i1.a[1], true)) { sm.mode = 1; sm.m_leaf = i1.a[1]; }
    else if (i1.op == EW_ADD && i1.a[2] < 0 && i1.a[1] == t && tensor(i1.a[0], true)) { sm.mode = 1; sm.m_leaf = i1.a[0]; }
    else if (i1.op == EW_SUB && i1.a[2] < 0 && i1.a[0] == t && tensor(i1.a[1], true)) { sm.mode = 2; sm.m_leaf = i1.a[1]; }
    else if (i1.op == EW_WHERE && tensor(i1.a[0], false) && i1.a[1] == t && literal(i1.a[2])) {
        sm.mode = 3; sm.m_leaf = i1.a[0]; sm.lit_leaf = i1.a[2];
    } else if (i1.op == EW_WHERE && tensor(i1.a[0], false) && literal(i1.a[1]) && i1.a[2] == t) {
        sm.mode = 4; sm.m_leaf = i1.a[0]; sm.lit_leaf = i1.a[1];
    } else {
        return false;
    }
    return true;
}

template <int CH, int R, int PROG>
__global__ void __launch_bounds__(256) softmax_rows_kernel(const __grid_constant__ EwParams P, const float *x,
                                                           float *y, long long rows, int n, int log_softmax,
                                                           unsigned vec_leaf, int vec_io, const ScaleMask sm) {
    float4 regs[PROG == 2 ? EW_MAX_LEAVES + EW_MAX_INSTR : 1];
    __shared__ unsigned row_base[8][R][PROG == 1 ? EW_MAX_LEAVES : 1];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nq = n >> 2;
    const int last = P.rank - 1;
    const long long groups = (rows + R - 1) / R;
    const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
    for (long long g = (long long)blockIdx.x * (blockDim.x >> 5) + warp; g < groups; g += warps) {
        const long long row0 = g * R;
        const int nr = rows - row0 < R ? (int)(rows - row0) : R;
        float4 v[R][CH];
        if constexpr (PROG == 1) {
            __syncwarp();
            for (int t = lane; t < nr * P.nleaves; t += 32) {
                const int r = t / P.nleaves, l = t - r * P.nleaves;
                unsigned idx[EW_MAX_RANK];
                ew_coords(P, (unsigned)((row0 + r) * n), idx);
                row_base[warp][r][l] = ew_leaf_offset(P, l, idx);
            }
            __syncwarp();
            float4 acc[R * CH];
            bool live[R * CH];
#pragma unroll
            for (int g = 0; g < R * CH; ++g) {
                live[g] = g / CH < nr && lane + 32 * (g % CH) < nq;
                acc[g] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
            for (int k = 0; k < P.ninstr; ++k)
                ew_chain_step<R * CH>(P.ins[k], P.nleaves, acc, live, [&](int l, int g) {
                    const EwLeaf &lf = P.leaves[l];
                    const unsigned inner = (unsigned)lf.strides[last];
                    const unsigned q = lane + 32 * (g % CH);
                    return ew_leaf4(lf, row_base[warp][g / CH][l] + inner * 4u * q, inner == 0, (vec_leaf >> l) & 1u);
                });
#pragma unroll
            for (int g = 0; g < R * CH; ++g) v[g / CH][g % CH] = acc[g];
        } else if constexpr (PROG == 3) {
            // the mask leaf's offset at each row start: lane r computes row r's
            unsigned mb = 0;
            if (sm.mode != 0 && lane < nr) {
                unsigned idx[EW_MAX_RANK];
                ew_coords(P, (unsigned)((row0 + lane) * n), idx);
                mb = ew_leaf_offset(P, sm.m_leaf, idx);
            }
            const EwLeaf &xl = P.leaves[sm.x_leaf];
            const EwLeaf &ml = P.leaves[sm.m_leaf];
            const float sc = P.leaves[sm.s_leaf].lit.f, lit = P.leaves[sm.lit_leaf].lit.f;
            const bool xq = (vec_leaf >> sm.x_leaf) & 1u, mq = (vec_leaf >> sm.m_leaf) & 1u;
            const unsigned m_inner = (unsigned)ml.strides[last];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const unsigned mrow = __shfl_sync(0xffffffffu, mb, r);
                if (r >= nr) continue;
#pragma unroll
                for (int c = 0; c < CH; ++c) {
                    const int q = lane + 32 * c;
                    if (q >= nq) continue;
                    float4 t = ew_leaf4(xl, (unsigned)((row0 + r) * n) + 4u * q, false, xq);
                    if (sm.div) t = make_float4(t.x / sc, t.y / sc, t.z / sc, t.w / sc);
                    else t = make_float4(t.x * sc, t.y * sc, t.z * sc, t.w * sc);
                    if (sm.mode != 0) {
                        const float4 mv = ew_leaf4(ml, mrow + m_inner * 4u * q, m_inner == 0, mq);
                        if (sm.mode == 1) t = make_float4(t.x + mv.x, t.y + mv.y, t.z + mv.z, t.w + mv.w);
                        else if (sm.mode == 2) t = make_float4(t.x - mv.x, t.y - mv.y, t.z - mv.z, t.w - mv.w);
                        else if (sm.mode == 3)
                            t = make_float4(mv.x != 0.0f ? t.x : lit, mv.y != 0.0f ? t.y : lit, mv.z != 0.0f ? t.z : lit,
                                            mv.w != 0.0f ? t.w : lit);
                        else
                            t = make_float4(mv.x != 0.0f ? lit : t.x, mv.y != 0.0f ? lit : t.y, mv.z != 0.0f ? lit : t.z,
                                            mv.w != 0.0f ? lit : t.w);
                    }
                    v[r][c] = t;
                }
            }
        } else {
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (r >= nr) break;
                unsigned base[PROG == 2 ? EW_MAX_LEAVES : 1];
                if constexpr (PROG == 2) ew_offsets(P, (unsigned)((row0 + r) * n), base);
#pragma unroll
                for (int c = 0; c < CH; ++c) {
                    const int q = lane + 32 * c;
                    if (q >= nq) break;
                    if constexpr (PROG == 2) {
                        unsigned off[EW_MAX_LEAVES];
                        for (int l = 0; l < P.nleaves; ++l) off[l] = base[l] + (P.leaves[l].strides[last] ? 4u * q : 0u);
                        v[r][c] = ew_run4(P, off, vec_leaf, regs);
                    } else {
                        const float *p = x + (row0 + r) * n + 4 * q;
                        v[r][c] = vec_io ? __ldg(reinterpret_cast<const float4 *>(p)) : make_float4(p[0], p[1], p[2], p[3]);
                    }
                }
            }
        }
        float m[R], s[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            m[r] = -INFINITY;
#pragma unroll
            for (int c = 0; c < CH; ++c)
                if (r < nr && lane + 32 * c < nq)
                    m[r] = fmaxf(m[r], fmaxf(fmaxf(v[r][c].x, v[r][c].y), fmaxf(v[r][c].z, v[r][c].w)));
        }
#pragma unroll
        for (int r = 0; r < R; ++r) m[r] = warp_max(m[r]);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            s[r] = 0.0f;
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                if (r >= nr || lane + 32 * c >= nq) continue;
                const float4 e = make_float4(__expf(v[r][c].x - m[r]), __expf(v[r][c].y - m[r]),
                                             __expf(v[r][c].z - m[r]), __expf(v[r][c].w - m[r]));
                s[r] += e.x + e.y + e.z + e.w;
                if (!log_softmax) v[r][c] = e;
            }
        }
#pragma unroll
        for (int r = 0; r < R; ++r) s[r] = warp_sum(s[r]);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            if (r >= nr) break;
            const float inv = log_softmax ? 0.0f : 1.0f / s[r], ls = log_softmax ? logf(s[r]) : 0.0f, mr = m[r];
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                const int q = lane + 32 * c;
                if (q >= nq) break;
                const float4 a = v[r][c];
                const float4 o = log_softmax ? make_float4(a.x - mr - ls, a.y - mr - ls, a.z - mr - ls, a.w - mr - ls)
                                             : make_float4(a.x * inv, a.y * inv, a.z * inv, a.w * inv);
                float *d = y + (row0 + r) * n + 4 * q;
                if (vec_io) *reinterpret_cast<float4 *>(d) = o;
                else { d[0] = o.x; d[1] = o.y; d[2] = o.z; d[3] = o.w; }
            }
        }
    }
}

// One block of 8 warps per 8 row groups, as many blocks as groups need: the hardware hands out
// the blocks as SMs free up, with no grid-stride tail.
template <int PROG>
inline void launch_softmax_rows_t(const EwParams &P, const float *x, float *y, long long rows, int n, int log,
                                  unsigned vec_leaf, int vec_io, const ScaleMask &sm, cudaStream_t stream) {
    const int ch = (n + 127) / 128;
    auto grid = [&](int r) { return (unsigned)((rows + 8ll * r - 1) / (8ll * r)); };
    // two rows per warp for rows of up to 256 (measured on B200: more rows per warp cost more in
    // occupancy than they gain in loads in flight)
    constexpr int G = 2;
    constexpr int R1 = G, R2 = G / 2 > 0 ? G / 2 : 1, R4 = G / 4 > 0 ? G / 4 : 1, R8 = G / 8 > 0 ? G / 8 : 1;
    if (ch <= 1) softmax_rows_kernel<1, R1, PROG><<<grid(R1), 256, 0, stream>>>(P, x, y, rows, n, log, vec_leaf, vec_io, sm);
    else if (ch <= 2) softmax_rows_kernel<2, R2, PROG><<<grid(R2), 256, 0, stream>>>(P, x, y, rows, n, log, vec_leaf, vec_io, sm);
    else if (ch <= 4) softmax_rows_kernel<4, R4, PROG><<<grid(R4), 256, 0, stream>>>(P, x, y, rows, n, log, vec_leaf, vec_io, sm);
    else softmax_rows_kernel<8, R8, PROG><<<grid(R8), 256, 0, stream>>>(P, x, y, rows, n, log, vec_leaf, vec_io, sm);
}

// Row softmax launcher: with `prog` the rows come from the program P (x unused), else from x.
inline int launch_softmax_rows(const EwParams &P, bool prog, const float *x, float *y, long long rows, int n, int log,
                               unsigned vec_leaf, int vec_io, cudaStream_t stream) {
    ScaleMask sm{};
    if (!prog) {
        launch_softmax_rows_t<0>(P, x, y, rows, n, log, vec_leaf, vec_io, sm, stream);
        return check_launch("softmax_rows_kernel");
    }
    vec_io = (reinterpret_cast<uintptr_t>(y) & 15) == 0;
    if (scale_mask_form(P, sm)) launch_softmax_rows_t<3>(P, x, y, rows, n, log, vec_leaf, vec_io, sm, stream);
    else if (ew_chain_form(P)) launch_softmax_rows_t<1>(P, x, y, rows, n, log, vec_leaf, vec_io, sm, stream);
    else launch_softmax_rows_t<2>(P, x, y, rows, n, log, vec_leaf, vec_io, sm, stream);
    return check_launch("softmax_rows_kernel(program)");
}

// Layer normalization of rows of at most 128 * CH fp32 values in groups of four (16-byte
// aligned): one warp per row holds it in registers, so the row is read from memory once; the
// mean, the sum of squared deviations and the output use layer_norm_kernel's arithmetic in the
// same order.
template <int CH>
__global__ void __launch_bounds__(256) layer_norm_rows_kernel(long long rows, int cols, const float *x,
                                                              const float *scale, const float *bias, float eps,
                                                              float *y) {
    const int lane = threadIdx.x & 31;
    const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
    for (long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const float *src = x + r * cols;
        float *dst = y + r * cols;
        float4 v[CH];
        float s = 0.0f;
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            const int k = lane * 4 + 128 * c;
            if (k < cols) {
                v[c] = __ldg(reinterpret_cast<const float4 *>(src + k));
                s += (v[c].x + v[c].y) + (v[c].z + v[c].w);
            }
        }
        const float mean = warp_sum(s) / (float)cols;
        float q = 0.0f;
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            if (lane * 4 + 128 * c < cols) {
                const float a = v[c].x - mean, b = v[c].y - mean, cc = v[c].z - mean, d = v[c].w - mean;
                q += (a * a + b * b) + (cc * cc + d * d);
            }
        }
        const float inv = 1.0f / sqrtf(warp_sum(q) / (float)cols + eps);
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            const int k = lane * 4 + 128 * c;
            if (k >= cols) continue;
            float4 o;
            o.x = (v[c].x - mean) * inv; o.y = (v[c].y - mean) * inv;
            o.z = (v[c].z - mean) * inv; o.w = (v[c].w - mean) * inv;
            if (scale) {
                const float4 g = __ldg(reinterpret_cast<const float4 *>(scale + k));
                o.x *= g.x; o.y *= g.y; o.z *= g.z; o.w *= g.w;
            }
            if (bias) {
                const float4 b = __ldg(reinterpret_cast<const float4 *>(bias + k));
                o.x += b.x; o.y += b.y; o.z += b.z; o.w += b.w;
            }
            *reinterpret_cast<float4 *>(dst + k) = o;
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
// Max pooling, NHWC, C % 4 == 0, KH, KW <= 3, width stride S (1 or 2), width dilation 1, sizes
// below 2^31: a thread takes four consecutive output columns of one output row and one 4-channel
// group, loading each input row's (3 * S + 3) columns once for all four (6.75 loads per output
// at stride 2 instead of 9). Columns outside the image read as -inf, which the comparison
// never takes, the same as skipping them.
template <int S>
__global__ void __launch_bounds__(256) maxpool4_nhwc_rows_kernel(const __grid_constant__ PoolParams p) {
    constexpr int R = 4, SPAN = (R - 1) * S + 3;
    const int c4n = p.C >> 2;
    const unsigned groups = (unsigned)(p.OW + R - 1) / R;
    const unsigned total = (unsigned)p.N * p.OH * groups * c4n;
    const unsigned stride = gridDim.x * blockDim.x;
    const float4 *x4 = reinterpret_cast<const float4 *>(p.x);
    float4 *y4 = reinterpret_cast<float4 *>(p.y);
    const float4 ninf = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    for (unsigned e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
        const int c4 = (int)(e % c4n);
        unsigned r = e / c4n;
        const unsigned g = r % groups;
        r /= groups;
        const int oh = (int)(r % p.OH);
        const unsigned n = r / p.OH;
        const int ow0 = (int)g * R, iw0 = ow0 * S - p.PL;
        float4 acc[R];
#pragma unroll
        for (int j = 0; j < R; ++j) acc[j] = ninf;
#pragma unroll
        for (int kh = 0; kh < 3; ++kh) {
            if (kh >= p.KH) break;
            const int ih = oh * p.SH - p.PT + kh * p.DH;
            if (ih < 0 || ih >= p.H) continue;
            const unsigned rowbase = (n * p.H + ih) * p.W;
            float4 in[SPAN];
#pragma unroll
            for (int t = 0; t < SPAN; ++t) {
                const int iw = iw0 + t;
                in[t] = iw >= 0 && iw < p.W ? __ldg(x4 + (size_t)(rowbase + iw) * c4n + c4) : ninf;
            }
#pragma unroll
            for (int j = 0; j < R; ++j)
#pragma unroll
                for (int kw = 0; kw < 3; ++kw) {
                    if (kw >= p.KW) break;
                    const float4 v = in[j * S + kw];
                    acc[j].x = v.x > acc[j].x ? v.x : acc[j].x;
                    acc[j].y = v.y > acc[j].y ? v.y : acc[j].y;
                    acc[j].z = v.z > acc[j].z ? v.z : acc[j].z;
                    acc[j].w = v.w > acc[j].w ? v.w : acc[j].w;
                }
        }
        const size_t o = ((size_t)r * p.OW + ow0) * c4n + c4;
#pragma unroll
        for (int j = 0; j < R; ++j)
            if (ow0 + j < p.OW) y4[o + (size_t)j * c4n] = acc[j];
    }
}

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
    int *err;  // the handle's status word (bounded waits that give up record MGC_CUDA_TIMEOUT), or NULL
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

// NHWC, C % 4 == 0, KH, KW <= 3, width stride S (1 or 2), width dilation 1, sizes below 2^31:
// as depthwise_nhwc4_reg_kernel, but a thread computes R consecutive output columns of one output
// row, loading each input row's (R - 1) * S + 3 columns once for all R of them (4.5 loads per
// output at stride 1 instead of 9). Taps outside the image contribute a zero product.
template <int R, int S>
__global__ void __launch_bounds__(256) depthwise_nhwc4_rows_kernel(const __grid_constant__ DepthwiseParams p) {
    constexpr int SPAN = (R - 1) * S + 3;
    const int C4 = p.C >> 2;
    const int c4 = (int)(threadIdx.x % (unsigned)C4);
    const unsigned per_block = blockDim.x / C4;
    const unsigned groups = (unsigned)(p.OW + R - 1) / R;
    const unsigned items = (unsigned)p.N * p.OH * groups;
    const float4 *x4 = reinterpret_cast<const float4 *>(p.x);
    const float4 *w4 = reinterpret_cast<const float4 *>(p.w);
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 wk[9];  // [kh][kw] of a 3x3 frame, zero outside KH x KW
#pragma unroll
    for (int t = 0; t < 9; ++t) {
        const int kh = t / 3, kw = t % 3;
        wk[t] = (kh < p.KH && kw < p.KW) ? __ldg(w4 + (kh * p.KW + kw) * C4 + c4) : zero;
    }
    const float4 b = p.bias ? __ldg(reinterpret_cast<const float4 *>(p.bias) + c4) : zero;
    for (unsigned it = blockIdx.x * per_block + threadIdx.x / C4; it < items; it += gridDim.x * per_block) {
        const unsigned g = it % groups, r = it / groups;
        const unsigned oh = r % p.OH, n = r / p.OH;
        const int ow0 = (int)g * R;
        const int iw0 = ow0 * S - p.PL;
        float4 acc[R];
#pragma unroll
        for (int j = 0; j < R; ++j) acc[j] = b;
#pragma unroll
        for (int kh = 0; kh < 3; ++kh) {
            if (kh >= p.KH) break;
            const int ih = (int)oh * p.SH - p.PT + kh * p.DH;
            if (ih < 0 || ih >= p.H) continue;
            const unsigned rowbase = (n * p.H + ih) * p.W;
            float4 in[SPAN];
#pragma unroll
            for (int t = 0; t < SPAN; ++t) {
                const int iw = iw0 + t;
                in[t] = (iw >= 0 && iw < p.W) ? __ldg(x4 + (size_t)(rowbase + iw) * C4 + c4) : zero;
            }
#pragma unroll
            for (int j = 0; j < R; ++j)
#pragma unroll
                for (int kw = 0; kw < 3; ++kw) {
                    if (kw >= p.KW) break;
                    const float4 v = in[j * S + kw], k = wk[kh * 3 + kw];
                    acc[j].x = fmaf(v.x, k.x, acc[j].x); acc[j].y = fmaf(v.y, k.y, acc[j].y);
                    acc[j].z = fmaf(v.z, k.z, acc[j].z); acc[j].w = fmaf(v.w, k.w, acc[j].w);
                }
        }
#pragma unroll
        for (int j = 0; j < R; ++j) {
            if (ow0 + j >= p.OW) break;
            const size_t o = ((size_t)r * p.OW + ow0 + j) * C4 + c4;
            float4 a = acc[j];
            if (p.res) {
                const float4 rr = reinterpret_cast<const float4 *>(p.res)[o];
                a.x += rr.x; a.y += rr.y; a.z += rr.z; a.w += rr.w;
            }
            if (p.act == MGC_ACT_RELU) {
                a.x = fmaxf(a.x, 0.0f); a.y = fmaxf(a.y, 0.0f); a.z = fmaxf(a.z, 0.0f); a.w = fmaxf(a.w, 0.0f);
            } else if (p.act == MGC_ACT_CLIP) {
                a.x = fminf(fmaxf(a.x, p.lo), p.hi); a.y = fminf(fmaxf(a.y, p.lo), p.hi);
                a.z = fminf(fmaxf(a.z, p.lo), p.hi); a.w = fminf(fmaxf(a.w, p.lo), p.hi);
            } else if (p.act != MGC_ACT_NONE) {
                a.x = apply_act(a.x, p.act, p.lo, p.hi); a.y = apply_act(a.y, p.act, p.lo, p.hi);
                a.z = apply_act(a.z, p.act, p.lo, p.hi); a.w = apply_act(a.w, p.act, p.lo, p.hi);
            }
            reinterpret_cast<float4 *>(p.y)[o] = a;
        }
    }
}

// NHWC, C % (4 * CG) == 0, KH, KW <= 3, height and width stride S (1 or 2), no dilation, sizes
// below 2^31: a block computes a tile of TH output rows x TW output columns x CG 4-channel groups
// (TW * CG = 256 threads). It first copies the tile's input window ((TH - 1) * S + 3 rows x
// (TW - 1) * S + 3 columns x CG groups, zero outside the image) into shared memory with coalesced
// 16-byte loads, so every input value crosses L2 once per tile instead of once per tap; then each
// thread walks one output column's TH rows for one channel group, its 3x3 weights and bias in
// registers, and, at stride 1, slides a 3-row window of inputs down the column (three shared
// loads per output row). Same accumulation order as the other depthwise forms (bias, then taps
// row by row).
template <int S, int CG>
struct DwTile {
    static constexpr int TW = 256 / CG;
    static constexpr int TH = S == 1 ? 8 : 4;
    static constexpr int IH = (TH - 1) * S + 3, IW = (TW - 1) * S + 3;
    static constexpr unsigned SMEM = (unsigned)IH * IW * CG * 16;
};

template <int S, int CG>
__global__ void __launch_bounds__(256) depthwise_nhwc4_tile_kernel(const __grid_constant__ DepthwiseParams p,
                                                                  unsigned row_tiles, unsigned col_tiles,
                                                                  unsigned chunks) {
    using T = DwTile<S, CG>;
    extern __shared__ float4 tile[];  // [IH][IW][CG]
    const int C4 = p.C >> 2;
    // block -> (image, row tile, column tile, channel chunk)
    unsigned b = blockIdx.x;
    const unsigned chunk = b % chunks;
    b /= chunks;
    const unsigned ct = b % col_tiles;
    b /= col_tiles;
    const unsigned rt = b % row_tiles;
    const unsigned n = b / row_tiles;
    const int oh0 = (int)rt * T::TH, ow0 = (int)ct * T::TW;
    const int ih0 = oh0 * S - p.PT, iw0 = ow0 * S - p.PL;
    const int c0 = (int)chunk * CG;  // first 4-channel group of the chunk
    const float4 *x4 = reinterpret_cast<const float4 *>(p.x);
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    // 1) the input window: consecutive threads take consecutive (pixel, group) float4s, copied
    // by cp.async (all of a thread's copies in flight at once; a source size of 0 writes zeros
    // for the pixels outside the image)
    const uint32_t tile_s = static_cast<uint32_t>(__cvta_generic_to_shared(tile));
#pragma unroll 4
    for (unsigned e = threadIdx.x; e < (unsigned)(T::IH * T::IW * CG); e += 256) {
        const unsigned g = e % CG, pix = e / CG;
        const int r = (int)(pix / T::IW), c = (int)(pix % T::IW);
        const int ih = ih0 + r, iw = iw0 + c;
        const bool inside = ih >= 0 && ih < p.H && iw >= 0 && iw < p.W;
        const float4 *src = inside ? x4 + ((size_t)(n * p.H + ih) * p.W + iw) * C4 + c0 + g : x4;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(tile_s + e * 16u), "l"(src),
                     "r"(inside ? 16 : 0)
                     : "memory");
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    // this thread's column and channel group, its weights and bias
    const int g = (int)(threadIdx.x % CG), col = (int)(threadIdx.x / CG);
    const float4 *w4 = reinterpret_cast<const float4 *>(p.w);
    float4 wk[9];
#pragma unroll
    for (int t = 0; t < 9; ++t) {
        const int kh = t / 3, kw = t % 3;
        wk[t] = (kh < p.KH && kw < p.KW) ? __ldg(w4 + (kh * p.KW + kw) * C4 + c0 + g) : zero;
    }
    const float4 bias = p.bias ? __ldg(reinterpret_cast<const float4 *>(p.bias) + c0 + g) : zero;
    __syncthreads();
    const int ow = ow0 + col;
    if (ow >= p.OW) return;
    auto at = [&](int r, int c) -> float4 { return tile[(r * T::IW + c) * CG + g]; };
    auto fma4 = [](float4 &a, const float4 v, const float4 k) {
        a.x = fmaf(v.x, k.x, a.x); a.y = fmaf(v.y, k.y, a.y); a.z = fmaf(v.z, k.z, a.z); a.w = fmaf(v.w, k.w, a.w);
    };
    const int cx = col * S;  // the column's first input column in the tile
    float4 win[3][3];        // stride 1: input rows r .. r + 2 of this column's three taps
    if (S == 1) {
#pragma unroll
        for (int kh = 0; kh < 2; ++kh)
#pragma unroll
            for (int kw = 0; kw < 3; ++kw) win[kh + 1][kw] = at(kh, cx + kw);
    }
#pragma unroll 1
    for (int r = 0; r < T::TH; ++r) {
        const int oh = oh0 + r;
        if (oh >= p.OH) break;
        float4 acc = bias;
        if (S == 1) {
#pragma unroll
            for (int kw = 0; kw < 3; ++kw) {
                win[0][kw] = win[1][kw];
                win[1][kw] = win[2][kw];
                win[2][kw] = at(r + 2, cx + kw);
            }
#pragma unroll
            for (int kh = 0; kh < 3; ++kh)
#pragma unroll
                for (int kw = 0; kw < 3; ++kw) fma4(acc, win[kh][kw], wk[kh * 3 + kw]);
        } else {
#pragma unroll
            for (int kh = 0; kh < 3; ++kh)
#pragma unroll
                for (int kw = 0; kw < 3; ++kw) fma4(acc, at(r * S + kh, cx + kw), wk[kh * 3 + kw]);
        }
        const size_t o = (((size_t)n * p.OH + oh) * p.OW + ow) * C4 + c0 + g;
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

// Layer normalization launcher: the register-resident form for rows of up to 1024 values in
// aligned groups of four, else layer_norm_kernel.
inline int launch_layer_norm(long long rows, long long cols, const float *x, const float *g, const float *b, float eps,
                             float *y, cudaStream_t stream) {
    const bool vec = cols % 4 == 0 && cols <= 1024 &&
                     ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(g) |
                       reinterpret_cast<uintptr_t>(b)) & 15) == 0;
    if (!vec) {
        layer_norm_kernel<<<grid_for(rows, 8), 256, 0, stream>>>(rows, cols, x, g, b, eps, y);
        return check_launch("layer_norm_kernel");
    }
    const unsigned grid = (unsigned)((rows + 7) / 8);
    const int c = (int)cols, ch = (c + 127) / 128;
    switch (ch) {
    case 1: layer_norm_rows_kernel<1><<<grid, 256, 0, stream>>>(rows, c, x, g, b, eps, y); break;
    case 2: layer_norm_rows_kernel<2><<<grid, 256, 0, stream>>>(rows, c, x, g, b, eps, y); break;
    case 3: layer_norm_rows_kernel<3><<<grid, 256, 0, stream>>>(rows, c, x, g, b, eps, y); break;
    case 4: layer_norm_rows_kernel<4><<<grid, 256, 0, stream>>>(rows, c, x, g, b, eps, y); break;
    case 5: layer_norm_rows_kernel<5><<<grid, 256, 0, stream>>>(rows, c, x, g, b, eps, y); break;
    case 6: layer_norm_rows_kernel<6><<<grid, 256, 0, stream>>>(rows, c, x, g, b, eps, y); break;
    case 7: layer_norm_rows_kernel<7><<<grid, 256, 0, stream>>>(rows, c, x, g, b, eps, y); break;
    default: layer_norm_rows_kernel<8><<<grid, 256, 0, stream>>>(rows, c, x, g, b, eps, y); break;
    }
    return check_launch("layer_norm_rows_kernel");
}

}  // namespace mgc

