// Memory-bound kernels: the elementwise program VM (FusedElementwise and single elementwise ops),
// strided copies (Transpose / Expand / Slice / Concat / Split / Pad / Tile), fills, Gather,
// Range, generic reductions and ArgMax.
//
// Reference lowerings: c.py:360-405 (loop nests with collapsed dimensions and broadcast
// strides), c.py:471-529 (elementwise programs), c.py:558-821 (data movement, Gather with its
// out-of-range return, reductions with a double accumulator for float sum/mean/prod, ArgMax).
// Semantics: ops.py:132-341 (elementwise), ops.py:1165-1202 (program format).
#pragma once

#include <math.h>
#include "common.cuh"

namespace mgc {

// ---------------------------------------------------------------------------------------------
// elementwise program VM
// ---------------------------------------------------------------------------------------------
// Operation codes of a program instruction; the Python lowering (mgc_cuda/lowering.py, EW_OPS)
// uses the same numbering.
enum EwOp : int16_t {
    EW_ADD = 0, EW_SUB, EW_MUL, EW_DIV, EW_POW, EW_MAX, EW_MIN,
    EW_EQ, EW_LT, EW_GT, EW_LE, EW_GE, EW_AND, EW_OR, EW_XOR,
    EW_WHERE, EW_RELU, EW_SIGMOID, EW_TANH, EW_ERF, EW_SQRT, EW_EXP, EW_LOG,
    EW_NEG, EW_ABS, EW_RECIP, EW_FLOOR, EW_CEIL, EW_SIN, EW_COS, EW_SOFTPLUS,
    EW_IDENTITY, EW_NOT, EW_GELU, EW_LEAKYRELU, EW_HARDSIGMOID, EW_CLIP, EW_CAST,
    EW_NUM_OPS
};

constexpr int EW_MAX_RANK = 6;
constexpr int EW_MAX_LEAVES = 20;
constexpr int EW_MAX_INSTR = 40;

// Arithmetic class of a value: fp32, fp64 or integer (every integer type and bool).
enum : int8_t { CL_F = 0, CL_D = 1, CL_I = 2 };

__host__ __device__ inline int8_t class_of(int dt) {
    return dt == MGC_F32 ? CL_F : dt == MGC_F64 ? CL_D : CL_I;
}

union Reg {
    float f;
    double d;
    long long i;
};

struct EwLeaf {
    const void *p;
    long long strides[EW_MAX_RANK];  // element strides over the output dimensions (0: broadcast)
    Reg lit;                         // value of a scalar constant leaf
    int32_t dtype;
    int32_t is_lit;
};

struct EwInstr {
    int16_t op;
    int16_t out_dt;
    int16_t a[3];  // register numbers (leaves first, then instruction results); -1: absent
    int16_t pad;
    double imm[2]; // op attributes (Clip bounds, LeakyRelu alpha, HardSigmoid alpha/beta, Gelu kind)
};

struct EwParams {
    long long shape[EW_MAX_RANK];
    long long total;
    void *out;
    int32_t rank;
    int32_t out_dt;
    int32_t nleaves;
    int32_t ninstr;
    int32_t contiguous;  // rank 1 and every tensor leaf has stride 1 or 0
    int8_t cls[EW_MAX_LEAVES + EW_MAX_INSTR];
    EwLeaf leaves[EW_MAX_LEAVES];
    EwInstr ins[EW_MAX_INSTR];
};

__device__ inline Reg load_elem(const void *p, int dt, long long i) {
    Reg r;
    switch (dt) {
    case MGC_F32: r.f = ((const float *)p)[i]; break;
    case MGC_F64: r.d = ((const double *)p)[i]; break;
    case MGC_I64: r.i = ((const long long *)p)[i]; break;
    case MGC_I32: r.i = ((const int *)p)[i]; break;
    case MGC_I8: r.i = ((const signed char *)p)[i]; break;
    default: r.i = ((const unsigned char *)p)[i]; break;  // U8, BOOL
    }
    return r;
}

__device__ inline void store_elem(void *p, int dt, long long i, Reg r) {
    switch (dt) {
    case MGC_F32: ((float *)p)[i] = r.f; break;
    case MGC_F64: ((double *)p)[i] = r.d; break;
    case MGC_I64: ((long long *)p)[i] = r.i; break;
    case MGC_I32: ((int *)p)[i] = (int)r.i; break;
    case MGC_I8: ((signed char *)p)[i] = (signed char)r.i; break;
    case MGC_BOOL: ((unsigned char *)p)[i] = r.i != 0; break;
    default: ((unsigned char *)p)[i] = (unsigned char)r.i; break;
    }
}

__device__ inline double as_d(Reg r, int c) { return c == CL_F ? (double)r.f : c == CL_D ? r.d : (double)r.i; }
__device__ inline float as_f(Reg r, int c) { return c == CL_F ? r.f : c == CL_D ? (float)r.d : (float)r.i; }
__device__ inline long long as_i(Reg r, int c) {
    return c == CL_F ? (long long)r.f : c == CL_D ? (long long)r.d : r.i;
}

// Convert a value of class `c` to the representation of dtype `dt` (bool: nonzero test).
__device__ inline Reg convert(Reg r, int c, int dt) {
    Reg o;
    if (dt == MGC_F32) o.f = as_f(r, c);
    else if (dt == MGC_F64) o.d = as_d(r, c);
    else if (dt == MGC_BOOL) o.i = (c == CL_F ? r.f != 0.0f : c == CL_D ? r.d != 0.0 : r.i != 0);
    else o.i = as_i(r, c);
    return o;
}

__device__ inline float f_sigmoid(float x) { return 0.5f * (1.0f + tanhf(0.5f * x)); }
__device__ inline double d_sigmoid(double x) { return 0.5 * (1.0 + tanh(0.5 * x)); }
__device__ inline float f_gelu(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }
__device__ inline float f_gelu_tanh(float x) {
    return 0.5f * x * (1.0f + tanhf(0.79788456080286536f * (x + 0.044715f * x * x * x)));
}
__device__ inline double d_gelu(double x) { return 0.5 * x * (1.0 + erf(x * 0.70710678118654752)); }
__device__ inline double d_gelu_tanh(double x) {
    return 0.5 * x * (1.0 + tanh(0.79788456080286536 * (x + 0.044715 * x * x * x)));
}
// log(1 + e^x) = max(x, 0) + log1p(e^-|x|)  (np.logaddexp(0, x), ops.py:259)
__device__ inline float f_softplus(float x) { return fmaxf(x, 0.0f) + log1pf(expf(-fabsf(x))); }
__device__ inline double d_softplus(double x) { return fmax(x, 0.0) + log1p(exp(-fabs(x))); }

// Evaluate one instruction. `cls` gives the class of every register.
__device__ inline Reg ew_eval(const EwInstr &in, const Reg *regs, const int8_t *cls) {
    const int oc = class_of(in.out_dt);
    const int a0 = in.a[0], a1 = in.a[1], a2 = in.a[2];
    Reg x = regs[a0];
    const int cx = cls[a0];
    Reg y{}, r{};
    int cy = CL_I;
    if (a1 >= 0) { y = regs[a1]; cy = cls[a1]; }
    int op = in.op;
    if (op <= EW_MIN || (op >= EW_EQ && op <= EW_GE)) {
        // binary arithmetic / comparison in the promoted class
        const int pc = (cx == CL_D || cy == CL_D) ? CL_D : (cx == CL_F || cy == CL_F) ? CL_F : CL_I;
        if (pc == CL_F) {
            float u = as_f(x, cx), v = as_f(y, cy), w = 0.0f;
            switch (op) {
            case EW_ADD: w = u + v; break;
            case EW_SUB: w = u - v; break;
            case EW_MUL: w = u * v; break;
            case EW_DIV: w = u / v; break;
            case EW_POW: w = powf(u, v); break;
            case EW_MAX: w = fmaxf(u, v); break;
            case EW_MIN: w = fminf(u, v); break;
            case EW_EQ: r.i = u == v; return r;
            case EW_LT: r.i = u < v; return r;
            case EW_GT: r.i = u > v; return r;
            case EW_LE: r.i = u <= v; return r;
            default: r.i = u >= v; return r;
            }
            Reg t; t.f = w;
            return convert(t, CL_F, in.out_dt);
        } else if (pc == CL_D) {
            double u = as_d(x, cx), v = as_d(y, cy), w = 0.0;
            switch (op) {
            case EW_ADD: w = u + v; break;
            case EW_SUB: w = u - v; break;
            case EW_MUL: w = u * v; break;
            case EW_DIV: w = u / v; break;
            case EW_POW: w = pow(u, v); break;
            case EW_MAX: w = fmax(u, v); break;
            case EW_MIN: w = fmin(u, v); break;
            case EW_EQ: r.i = u == v; return r;
            case EW_LT: r.i = u < v; return r;
            case EW_GT: r.i = u > v; return r;
            case EW_LE: r.i = u <= v; return r;
            default: r.i = u >= v; return r;
            }
            Reg t; t.d = w;
            return convert(t, CL_D, in.out_dt);
        } else {
            long long u = x.i, v = y.i, w = 0;
            switch (op) {
            case EW_ADD: w = u + v; break;
            case EW_SUB: w = u - v; break;
            case EW_MUL: w = u * v; break;
            case EW_DIV: w = v != 0 ? u / v : 0; break;  // truncation, as np.trunc(a / b)
            case EW_POW: { long long acc = 1; for (long long k = 0; k < v && k < 64; ++k) acc *= u; w = v < 0 ? 0 : acc; } break;
            case EW_MAX: w = u > v ? u : v; break;
            case EW_MIN: w = u < v ? u : v; break;
            case EW_EQ: r.i = u == v; return r;
            case EW_LT: r.i = u < v; return r;
            case EW_GT: r.i = u > v; return r;
            case EW_LE: r.i = u <= v; return r;
            default: r.i = u >= v; return r;
            }
            Reg t; t.i = w;
            return convert(t, CL_I, in.out_dt);
        }
    }
    switch (op) {
    case EW_AND: r.i = (as_i(x, cx) != 0) && (as_i(y, cy) != 0); return r;
    case EW_OR: r.i = (as_i(x, cx) != 0) || (as_i(y, cy) != 0); return r;
    case EW_XOR: r.i = (as_i(x, cx) != 0) != (as_i(y, cy) != 0); return r;
    case EW_NOT: r.i = as_i(x, cx) == 0; return r;
    case EW_WHERE: {
        Reg z = regs[a2];
        return as_i(x, cx) != 0 ? convert(y, cy, in.out_dt) : convert(z, cls[a2], in.out_dt);
    }
    case EW_CAST: return convert(x, cx, in.out_dt);
    case EW_IDENTITY: return convert(x, cx, in.out_dt);
    case EW_CLIP: {
        // bounds from optional inputs (a1, a2) or from the attributes (imm)
        if (cx == CL_I) {
            long long v = x.i;
            if (a1 >= 0) { long long lo = as_i(y, cy); v = v < lo ? lo : v; }
            if (a2 >= 0) { long long hi = as_i(regs[a2], cls[a2]); v = v > hi ? hi : v; }
            Reg t; t.i = v;
            return convert(t, CL_I, in.out_dt);
        }
        double lo = a1 >= 0 ? as_d(y, cy) : in.imm[0];
        double hi = a2 >= 0 ? as_d(regs[a2], cls[a2]) : in.imm[1];
        if (cx == CL_F) {
            Reg t; t.f = fminf(fmaxf(x.f, (float)lo), (float)hi);
            return convert(t, CL_F, in.out_dt);
        }
        Reg t; t.d = fmin(fmax(x.d, lo), hi);
        return convert(t, CL_D, in.out_dt);
    }
    default: break;
    }
    // unary operators
    if (cx == CL_I && (op == EW_RELU || op == EW_NEG || op == EW_ABS)) {
        long long v = x.i;
        Reg t;
        t.i = op == EW_RELU ? (v > 0 ? v : 0) : op == EW_NEG ? -v : (v < 0 ? -v : v);
        return convert(t, CL_I, in.out_dt);
    }
    if (cx == CL_F) {
        float v = x.f, w;
        switch (op) {
        case EW_RELU: w = fmaxf(v, 0.0f); break;
        case EW_SIGMOID: w = f_sigmoid(v); break;
        case EW_TANH: w = tanhf(v); break;
        case EW_ERF: w = erff(v); break;
        case EW_SQRT: w = sqrtf(v); break;
        case EW_EXP: w = expf(v); break;
        case EW_LOG: w = logf(v); break;
        case EW_NEG: w = -v; break;
        case EW_ABS: w = fabsf(v); break;
        case EW_RECIP: w = 1.0f / v; break;
        case EW_FLOOR: w = floorf(v); break;
        case EW_CEIL: w = ceilf(v); break;
        case EW_SIN: w = sinf(v); break;
        case EW_COS: w = cosf(v); break;
        case EW_SOFTPLUS: w = f_softplus(v); break;
        case EW_GELU: w = in.imm[0] != 0.0 ? f_gelu_tanh(v) : f_gelu(v); break;
        case EW_LEAKYRELU: w = v >= 0.0f ? v : (float)in.imm[0] * v; break;
        case EW_HARDSIGMOID: w = fminf(fmaxf((float)in.imm[0] * v + (float)in.imm[1], 0.0f), 1.0f); break;
        default: w = v; break;
        }
        Reg t; t.f = w;
        return convert(t, CL_F, in.out_dt);
    }
    double v = as_d(x, cx), w;
    switch (op) {
    case EW_RELU: w = fmax(v, 0.0); break;
    case EW_SIGMOID: w = d_sigmoid(v); break;
    case EW_TANH: w = tanh(v); break;
    case EW_ERF: w = erf(v); break;
    case EW_SQRT: w = sqrt(v); break;
    case EW_EXP: w = exp(v); break;
    case EW_LOG: w = log(v); break;
    case EW_NEG: w = -v; break;
    case EW_ABS: w = fabs(v); break;
    case EW_RECIP: w = 1.0 / v; break;
    case EW_FLOOR: w = floor(v); break;
    case EW_CEIL: w = ceil(v); break;
    case EW_SIN: w = sin(v); break;
    case EW_COS: w = cos(v); break;
    case EW_SOFTPLUS: w = d_softplus(v); break;
    case EW_GELU: w = in.imm[0] != 0.0 ? d_gelu_tanh(v) : d_gelu(v); break;
    case EW_LEAKYRELU: w = v >= 0.0 ? v : in.imm[0] * v; break;
    case EW_HARDSIGMOID: w = fmin(fmax(in.imm[0] * v + in.imm[1], 0.0), 1.0); break;
    default: w = v; break;
    }
    Reg t; t.d = w;
    return convert(t, CL_D, in.out_dt);
}

__global__ void __launch_bounds__(256) ew_kernel(const __grid_constant__ EwParams P) {
    Reg regs[EW_MAX_LEAVES + EW_MAX_INSTR];
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long o = (long long)blockIdx.x * blockDim.x + threadIdx.x; o < P.total; o += stride) {
        if (P.contiguous) {
            for (int l = 0; l < P.nleaves; ++l) {
                const EwLeaf &lf = P.leaves[l];
                regs[l] = lf.is_lit ? lf.lit : load_elem(lf.p, lf.dtype, o * lf.strides[0]);
            }
        } else {
            long long idx[EW_MAX_RANK];
            long long rem = o;
            for (int d = P.rank - 1; d >= 0; --d) {
                idx[d] = rem % P.shape[d];
                rem /= P.shape[d];
            }
            for (int l = 0; l < P.nleaves; ++l) {
                const EwLeaf &lf = P.leaves[l];
                if (lf.is_lit) {
                    regs[l] = lf.lit;
                    continue;
                }
                long long off = 0;
                for (int d = 0; d < P.rank; ++d) off += idx[d] * lf.strides[d];
                regs[l] = load_elem(lf.p, lf.dtype, off);
            }
        }
        for (int k = 0; k < P.ninstr; ++k) regs[P.nleaves + k] = ew_eval(P.ins[k], regs, P.cls);
        store_elem(P.out, P.out_dt, o, regs[P.nleaves + P.ninstr - 1]);
    }
}

// One instruction of the four-wide fp32 form: the fp32 branches of ew_eval, operand for operand.
// Byte values (bool, uint8) enter as the fp32 number of their value, which is what ew_eval's fp32
// arithmetic, Cast and Where read of them (ew_f32x4_form lists the operators and operand classes
// this covers).
__device__ __forceinline__ float ew_f32(const EwInstr &in, float x, float y, float z) {
    switch (in.op) {
    case EW_ADD: return x + y;
    case EW_SUB: return x - y;
    case EW_MUL: return x * y;
    case EW_DIV: return x / y;
    case EW_POW: return powf(x, y);
    case EW_MAX: return fmaxf(x, y);
    case EW_MIN: return fminf(x, y);
    case EW_WHERE: return x != 0.0f ? y : z;
    case EW_CLIP: {
        const float lo = in.a[1] >= 0 ? y : (float)in.imm[0];
        const float hi = in.a[2] >= 0 ? z : (float)in.imm[1];
        return fminf(fmaxf(x, lo), hi);
    }
    case EW_RELU: return fmaxf(x, 0.0f);
    case EW_SIGMOID: return f_sigmoid(x);
    case EW_TANH: return tanhf(x);
    case EW_ERF: return erff(x);
    case EW_SQRT: return sqrtf(x);
    case EW_EXP: return expf(x);
    case EW_LOG: return logf(x);
    case EW_NEG: return -x;
    case EW_ABS: return fabsf(x);
    case EW_RECIP: return 1.0f / x;
    case EW_FLOOR: return floorf(x);
    case EW_CEIL: return ceilf(x);
    case EW_SIN: return sinf(x);
    case EW_COS: return cosf(x);
    case EW_SOFTPLUS: return f_softplus(x);
    case EW_GELU: return in.imm[0] != 0.0 ? f_gelu_tanh(x) : f_gelu(x);
    case EW_LEAKYRELU: return x >= 0.0f ? x : (float)in.imm[0] * x;
    case EW_HARDSIGMOID: return fminf(fmaxf((float)in.imm[0] * x + (float)in.imm[1], 0.0f), 1.0f);
    default: return x;  // EW_IDENTITY, EW_CAST
    }
}

// Whether a program runs in the four-wide fp32 form with the results of ew_eval: fp32 output and
// instruction results; fp32 or byte (bool, uint8) tensor leaves and fp32 literals; byte values
// only where ew_eval converts them to fp32 (an operand of binary fp32 arithmetic next to an fp32
// one, a Where condition or branch, a Cast or Identity, a Clip bound).
inline bool ew_f32x4_form(const EwParams &P) {
    if (P.out_dt != MGC_F32) return false;
    for (int l = 0; l < P.nleaves; ++l) {
        const EwLeaf &lf = P.leaves[l];
        if (lf.is_lit ? lf.dtype != MGC_F32 : (lf.dtype != MGC_F32 && lf.dtype != MGC_BOOL && lf.dtype != MGC_U8))
            return false;
    }
    for (int k = 0; k < P.ninstr; ++k) {
        const EwInstr &in = P.ins[k];
        if (in.out_dt != MGC_F32) return false;
        const int op = in.op;
        const bool f0 = P.cls[in.a[0]] == CL_F, f1 = in.a[1] >= 0 && P.cls[in.a[1]] == CL_F;
        if (op <= EW_MIN) {
            if (!f0 && !f1) return false;
        } else if (op == EW_WHERE) {
            if (f0) return false;  // an fp32 condition truncates to an integer in ew_eval
        } else if (op == EW_CLIP || (op >= EW_RELU && op <= EW_SOFTPLUS) || op == EW_GELU ||
                   op == EW_LEAKYRELU || op == EW_HARDSIGMOID) {
            if (!f0) return false;
        } else if (op != EW_IDENTITY && op != EW_CAST) {
            return false;
        }
    }
    return true;
}

// Whether the four-wide forms apply: the innermost dimension comes in groups of four that every
// tensor leaf reads contiguously (stride 1) or broadcasts (stride 0), strides are non-negative and
// every offset fits 32 bits. Bit l of vec_leaf: leaf l of stride 1 whose groups of four start on
// 16 bytes (aligned base, outer strides multiples of 4).
inline bool ew_vec4_form(const EwParams &P, unsigned &vec_leaf) {
    vec_leaf = 0;
    if (P.rank < 1 || P.shape[P.rank - 1] % 4 != 0 || P.total >= (1ll << 31)) return false;
    for (int l = 0; l < P.nleaves; ++l) {
        const EwLeaf &lf = P.leaves[l];
        if (lf.is_lit) continue;
        const long long inner = lf.strides[P.rank - 1];
        long long span = 0;
        bool quad = lf.dtype == MGC_F32 && (reinterpret_cast<uintptr_t>(lf.p) & 15) == 0;
        for (int d = 0; d < P.rank; ++d) {
            if (lf.strides[d] < 0) return false;
            span += (P.shape[d] - 1) * lf.strides[d];
            if (d < P.rank - 1) quad = quad && lf.strides[d] % 4 == 0;
        }
        if ((inner != 0 && inner != 1) || span >= (1ll << 31)) return false;
        if (inner == 1 && quad) vec_leaf |= 1u << l;
    }
    return true;
}

// Offsets of every leaf at output element e (32-bit arithmetic; ew_vec4_form bounds them).
__device__ __forceinline__ void ew_offsets(const EwParams &P, unsigned e, unsigned *off) {
    unsigned idx[EW_MAX_RANK];
    for (int d = P.rank - 1; d > 0; --d) {
        const unsigned n = (unsigned)P.shape[d];
        const unsigned q = e / n;
        idx[d] = e - q * n;
        e = q;
    }
    idx[0] = e;
    for (int l = 0; l < P.nleaves; ++l) {
        const EwLeaf &lf = P.leaves[l];
        unsigned o = 0;
        if (!lf.is_lit)
            for (int d = 0; d < P.rank; ++d) o += idx[d] * (unsigned)lf.strides[d];
        off[l] = o;
    }
}

// Four consecutive values of a leaf from its offset: a literal, a broadcast (innermost stride 0),
// one 16-byte load (`quad`) or four loads; byte leaves as the fp32 number of their value.
__device__ __forceinline__ float4 ew_leaf4(const EwLeaf &lf, unsigned off, bool bcast, bool quad) {
    if (lf.is_lit) return make_float4(lf.lit.f, lf.lit.f, lf.lit.f, lf.lit.f);
    if (lf.dtype == MGC_F32) {
        const float *p = (const float *)lf.p + off;
        if (bcast) { const float t = __ldg(p); return make_float4(t, t, t, t); }
        if (quad) return __ldg(reinterpret_cast<const float4 *>(p));
        return make_float4(__ldg(p), __ldg(p + 1), __ldg(p + 2), __ldg(p + 3));
    }
    const unsigned char *b = (const unsigned char *)lf.p + off;
    if (bcast) { const float t = (float)__ldg(b); return make_float4(t, t, t, t); }
    return make_float4((float)__ldg(b), (float)__ldg(b + 1), (float)__ldg(b + 2), (float)__ldg(b + 3));
}

// The program over the four elements whose leaf offsets are off[] (ew_f32x4_form programs);
// `regs` is the caller's register file of four-lane values.
__device__ __forceinline__ float4 ew_run4(const EwParams &P, const unsigned *off, unsigned vec_leaf, float4 *regs) {
    const int last = P.rank - 1;
    for (int l = 0; l < P.nleaves; ++l)
        regs[l] = ew_leaf4(P.leaves[l], off[l], P.leaves[l].strides[last] == 0, (vec_leaf >> l) & 1u);
    for (int k = 0; k < P.ninstr; ++k) {
        const EwInstr &in = P.ins[k];
        const float4 x = regs[in.a[0]];
        const float4 y = in.a[1] >= 0 ? regs[in.a[1]] : x;
        const float4 z = in.a[2] >= 0 ? regs[in.a[2]] : x;
        regs[P.nleaves + k] = make_float4(ew_f32(in, x.x, y.x, z.x), ew_f32(in, x.y, y.y, z.y),
                                          ew_f32(in, x.z, y.z, z.z), ew_f32(in, x.w, y.w, z.w));
    }
    return regs[P.nleaves + P.ninstr - 1];
}

// Whether a program is a chain: every operand is a leaf or the result of the instruction just
// before, so the four-wide form needs no register file: one accumulator, and each leaf loaded
// where an instruction uses it (the attention scale and mask, embedding sums, mask arithmetic).
inline bool ew_chain_form(const EwParams &P) {
    for (int k = 0; k < P.ninstr; ++k)
        for (int j = 0; j < 3; ++j) {
            const int a = P.ins[k].a[j];
            if (a >= P.nleaves && a != P.nleaves + k - 1) return false;
        }
    return true;
}

// Output coordinates of element e; the loops unroll over EW_MAX_RANK so idx stays in registers.
__device__ __forceinline__ void ew_coords(const EwParams &P, unsigned e, unsigned (&idx)[EW_MAX_RANK]) {
#pragma unroll
    for (int d = EW_MAX_RANK - 1; d > 0; --d) {
        if (d < P.rank) {
            const unsigned n = (unsigned)P.shape[d];
            const unsigned q = e / n;
            idx[d] = e - q * n;
            e = q;
        } else {
            idx[d] = 0;
        }
    }
    idx[0] = e;
}

__device__ __forceinline__ unsigned ew_leaf_offset(const EwParams &P, int l, const unsigned (&idx)[EW_MAX_RANK]) {
    const EwLeaf &lf = P.leaves[l];
    unsigned o = 0;
#pragma unroll
    for (int d = 0; d < EW_MAX_RANK; ++d)
        if (d < P.rank) o += idx[d] * (unsigned)lf.strides[d];
    return o;
}

__device__ __forceinline__ float4 ew_f32x4(const EwInstr &in, float4 x, float4 y, float4 z) {
    return make_float4(ew_f32(in, x.x, y.x, z.x), ew_f32(in, x.y, y.y, z.y), ew_f32(in, x.z, y.z, z.z),
                       ew_f32(in, x.w, y.w, z.w));
}

// One instruction of a chain program (ew_chain_form, ew_f32x4_form) over G groups of four
// elements: operands are fetched for every live group (fetch(l, g): the four values of leaf l
// for group g; an operand that is no leaf is the accumulator), then one switch on the operator
// runs it over all groups, so the dispatch costs once per instruction and G groups rather than
// once per element. The common operators are written out; the rest go lane by lane through
// ew_f32 with the same arithmetic.
template <int G, class Fetch>
__device__ __forceinline__ void ew_chain_step(const EwInstr &in, int nleaves, float4 (&acc)[G], const bool (&live)[G],
                                              Fetch fetch) {
    const int a0 = in.a[0], a1 = in.a[1], a2 = in.a[2];
    float4 x[G], y[G], z[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        if (!live[g]) continue;
        x[g] = a0 < nleaves ? fetch(a0, g) : acc[g];
        y[g] = a1 < 0 ? x[g] : a1 < nleaves ? fetch(a1, g) : acc[g];
        z[g] = a2 < 0 ? x[g] : a2 < nleaves ? fetch(a2, g) : acc[g];
    }
#define MGC_EW_EACH(EXPR)                                                                          \
    _Pragma("unroll") for (int g = 0; g < G; ++g) {                                                \
        const float4 X = x[g], Y = y[g], Z = z[g];                                                 \
        (void)Y; (void)Z;                                                                          \
        acc[g] = make_float4(EXPR(X.x, Y.x, Z.x), EXPR(X.y, Y.y, Z.y), EXPR(X.z, Y.z, Z.z),        \
                             EXPR(X.w, Y.w, Z.w));                                                 \
    }
#define MGC_EW_ADD(u, v, w) ((u) + (v))
#define MGC_EW_SUB(u, v, w) ((u) - (v))
#define MGC_EW_MUL(u, v, w) ((u) * (v))
#define MGC_EW_DIV(u, v, w) ((u) / (v))
#define MGC_EW_MAXF(u, v, w) fmaxf((u), (v))
#define MGC_EW_MINF(u, v, w) fminf((u), (v))
#define MGC_EW_WHERE(u, v, w) ((u) != 0.0f ? (v) : (w))
#define MGC_EW_RELU(u, v, w) fmaxf((u), 0.0f)
#define MGC_EW_COPY(u, v, w) (u)
    switch (in.op) {
    case EW_ADD: MGC_EW_EACH(MGC_EW_ADD) break;
    case EW_SUB: MGC_EW_EACH(MGC_EW_SUB) break;
    case EW_MUL: MGC_EW_EACH(MGC_EW_MUL) break;
    case EW_DIV: MGC_EW_EACH(MGC_EW_DIV) break;
    case EW_MAX: MGC_EW_EACH(MGC_EW_MAXF) break;
    case EW_MIN: MGC_EW_EACH(MGC_EW_MINF) break;
    case EW_WHERE: MGC_EW_EACH(MGC_EW_WHERE) break;
    case EW_RELU: MGC_EW_EACH(MGC_EW_RELU) break;
    case EW_IDENTITY:
    case EW_CAST: MGC_EW_EACH(MGC_EW_COPY) break;
    default:
#pragma unroll
        for (int g = 0; g < G; ++g) acc[g] = ew_f32x4(in, x[g], y[g], z[g]);
        break;
    }
#undef MGC_EW_EACH
#undef MGC_EW_ADD
#undef MGC_EW_SUB
#undef MGC_EW_MUL
#undef MGC_EW_DIV
#undef MGC_EW_MAXF
#undef MGC_EW_MINF
#undef MGC_EW_WHERE
#undef MGC_EW_RELU
#undef MGC_EW_COPY
}

// A chain program over four consecutive output elements per thread, with no register file.
__global__ void __launch_bounds__(256) ew_chain4_kernel(const __grid_constant__ EwParams P, const unsigned vec_leaf,
                                                        const int vec_out) {
    const unsigned total4 = (unsigned)(P.total >> 2);
    const unsigned step = gridDim.x * blockDim.x;
    const int last = P.rank - 1;
    for (unsigned v = blockIdx.x * blockDim.x + threadIdx.x; v < total4; v += step) {
        unsigned idx[EW_MAX_RANK];
        ew_coords(P, v << 2, idx);
        float4 acc[1] = {make_float4(0.0f, 0.0f, 0.0f, 0.0f)};
        const bool live[1] = {true};
        for (int k = 0; k < P.ninstr; ++k)
            ew_chain_step<1>(P.ins[k], P.nleaves, acc, live, [&](int l, int) {
                const EwLeaf &lf = P.leaves[l];
                return ew_leaf4(lf, ew_leaf_offset(P, l, idx), lf.strides[last] == 0, (vec_leaf >> l) & 1u);
            });
        float *o = (float *)P.out + (v << 2);
        if (vec_out) *reinterpret_cast<float4 *>(o) = acc[0];
        else { o[0] = acc[0].x; o[1] = acc[0].y; o[2] = acc[0].z; o[3] = acc[0].w; }
    }
}

// An ew_f32x4_form program over four consecutive output elements per thread (ew_vec4_form
// shapes); the output leaves as one 16-byte store when `vec_out`.
__global__ void __launch_bounds__(256) ew_f32x4_kernel(const __grid_constant__ EwParams P, const unsigned vec_leaf,
                                                       const int vec_out) {
    float4 regs[EW_MAX_LEAVES + EW_MAX_INSTR];
    const unsigned total4 = (unsigned)(P.total >> 2);
    const unsigned step = gridDim.x * blockDim.x;
    for (unsigned v = blockIdx.x * blockDim.x + threadIdx.x; v < total4; v += step) {
        unsigned off[EW_MAX_LEAVES];
        ew_offsets(P, v << 2, off);
        const float4 r = ew_run4(P, off, vec_leaf, regs);
        float *o = (float *)P.out + (v << 2);
        if (vec_out) *reinterpret_cast<float4 *>(o) = r;
        else { o[0] = r.x; o[1] = r.y; o[2] = r.z; o[3] = r.w; }
    }
}

// Any program over four consecutive output elements per thread: the index arithmetic of
// ew_f32x4_kernel, then the registers and ew_eval of ew_kernel element by element.
__global__ void __launch_bounds__(256) ew_vec4_kernel(const __grid_constant__ EwParams P) {
    Reg regs[EW_MAX_LEAVES + EW_MAX_INSTR];
    const unsigned total4 = (unsigned)(P.total >> 2);
    const unsigned step = gridDim.x * blockDim.x;
    const int last = P.rank - 1;
    for (unsigned v = blockIdx.x * blockDim.x + threadIdx.x; v < total4; v += step) {
        unsigned off[EW_MAX_LEAVES];
        ew_offsets(P, v << 2, off);
        for (int j = 0; j < 4; ++j) {
            for (int l = 0; l < P.nleaves; ++l) {
                const EwLeaf &lf = P.leaves[l];
                regs[l] = lf.is_lit ? lf.lit : load_elem(lf.p, lf.dtype, off[l] + (lf.strides[last] ? j : 0));
            }
            for (int k = 0; k < P.ninstr; ++k) regs[P.nleaves + k] = ew_eval(P.ins[k], regs, P.cls);
            store_elem(P.out, P.out_dt, (long long)(v << 2) + j, regs[P.nleaves + P.ninstr - 1]);
        }
    }
}

// ---------------------------------------------------------------------------------------------
// strided copy: dst[dbase + sum idx*dstr] = src[sbase + sum idx*sstr] over `shape`
// ---------------------------------------------------------------------------------------------
constexpr int COPY_MAX_RANK = 8;

// A Split along the last axis into up to SPLIT_MAX_OUT contiguous outputs in one pass over the
// input: source [rows][total], output j [rows][start[j + 1] - start[j]] (in units of T, one
// fp32 or four). Each thread moves one unit: reads are coalesced along the input row, writes
// along each output row.
constexpr int SPLIT_MAX_OUT = 4;

template <typename T>
struct SplitParams {
    const T *src;
    T *dst[SPLIT_MAX_OUT];
    long long rows;
    int total, k;
    int start[SPLIT_MAX_OUT + 1];
};

template <typename T>
__global__ void __launch_bounds__(256) split_last_kernel(const __grid_constant__ SplitParams<T> p) {
    const long long n = p.rows * p.total;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
        const long long r = e / p.total;
        const int c = (int)(e - r * p.total);
        int j = 0;
#pragma unroll
        for (int t = 1; t < SPLIT_MAX_OUT; ++t) j += (t < p.k && c >= p.start[t]) ? 1 : 0;
        const int w = p.start[j + 1] - p.start[j];
        p.dst[j][r * w + (c - p.start[j])] = p.src[e];
    }
}

struct CopyParams {
    long long shape[COPY_MAX_RANK];
    long long sstr[COPY_MAX_RANK];
    long long dstr[COPY_MAX_RANK];
    long long sbase, dbase, total;
    const char *src;
    char *dst;
    int32_t rank;
    int32_t esize;
};

template <typename T>
__global__ void __launch_bounds__(256) copy_kernel(const __grid_constant__ CopyParams P) {
    const T *src = (const T *)P.src;
    T *dst = (T *)P.dst;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long o = (long long)blockIdx.x * blockDim.x + threadIdx.x; o < P.total; o += stride) {
        long long rem = o, s = P.sbase, d = P.dbase;
        for (int k = P.rank - 1; k >= 0; --k) {
            long long i = rem % P.shape[k];
            rem /= P.shape[k];
            s += i * P.sstr[k];
            d += i * P.dstr[k];
        }
        dst[d] = src[s];
    }
}

// The same copy with 32-bit index arithmetic and V elements per thread along the innermost
// dimension (contiguous on both sides): the caller passes the shape and strides in units of V
// elements (innermost extent divided by V) and checks alignment and that every index fits.
template <typename VT>
__global__ void __launch_bounds__(256) copy_vec_kernel(const __grid_constant__ CopyParams P) {
    const VT *src = (const VT *)P.src;
    VT *dst = (VT *)P.dst;
    int shape[COPY_MAX_RANK], sstr[COPY_MAX_RANK], dstr[COPY_MAX_RANK];
#pragma unroll
    for (int k = 0; k < COPY_MAX_RANK; ++k) {
        shape[k] = k < P.rank ? (int)P.shape[k] : 1;
        sstr[k] = k < P.rank ? (int)P.sstr[k] : 0;
        dstr[k] = k < P.rank ? (int)P.dstr[k] : 0;
    }
    const unsigned total = (unsigned)P.total, stride = gridDim.x * blockDim.x;
    for (unsigned o = blockIdx.x * blockDim.x + threadIdx.x; o < total; o += stride) {
        unsigned rem = o;
        int s = (int)P.sbase, d = (int)P.dbase;
#pragma unroll
        for (int k = COPY_MAX_RANK - 1; k >= 0; --k) {
            if (k >= P.rank) continue;
            const unsigned i = rem % (unsigned)shape[k];
            rem /= (unsigned)shape[k];
            s += (int)i * sstr[k];
            d += (int)i * dstr[k];
        }
        dst[d] = src[s];
    }
}

// A copy whose destination is contiguous along dimension ii (the last) and whose source is
// contiguous along another dimension jj (a transpose, such as attention's (b, h, s, d) ->
// (b, h, d, s)): 32 x 32 tiles staged in shared memory, read along jj and written along ii, so
// both sides move whole 128-byte lines. The remaining dimensions index the tiles' batch; all
// index arithmetic is 32-bit (the launcher checks that every offset fits).
template <typename T>
__global__ void __launch_bounds__(256) transpose_tile_kernel(const __grid_constant__ CopyParams P, const int jj,
                                                             const unsigned nbatch) {
    __shared__ T tile[32][33];
    const T *src = (const T *)P.src;
    T *dst = (T *)P.dst;
    const int ii = P.rank - 1;
    const unsigned ni = (unsigned)P.shape[ii], nj = (unsigned)P.shape[jj];
    const unsigned ti_n = (ni + 31) / 32, tj_n = (nj + 31) / 32;
    const unsigned tiles = nbatch * ti_n * tj_n;
    const unsigned s_i = (unsigned)P.sstr[ii], s_j = (unsigned)P.sstr[jj];
    const unsigned d_i = (unsigned)P.dstr[ii], d_j = (unsigned)P.dstr[jj];
    const unsigned tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    for (unsigned t = blockIdx.x; t < tiles; t += gridDim.x) {
        const unsigned tq = t / tj_n, tj = t - tq * tj_n;
        const unsigned tb = tq / ti_n, ti = tq - tb * ti_n;
        unsigned rem = tb, sb = (unsigned)P.sbase, db = (unsigned)P.dbase;
        for (int k = P.rank - 1; k >= 0; --k) {
            if (k == ii || k == jj) continue;
            const unsigned e = (unsigned)P.shape[k], q = rem / e, i = rem - q * e;
            rem = q;
            sb += i * (unsigned)P.sstr[k];
            db += i * (unsigned)P.dstr[k];
        }
        const unsigned i0 = ti * 32, j0 = tj * 32;
#pragma unroll
        for (unsigned k = ty; k < 32; k += 8) {
            const unsigned i = i0 + k, j = j0 + tx;
            if (i < ni && j < nj) tile[k][tx] = src[sb + i * s_i + j * s_j];
        }
        __syncthreads();
#pragma unroll
        for (unsigned k = ty; k < 32; k += 8) {
            const unsigned i = i0 + tx, j = j0 + k;
            if (i < ni && j < nj) dst[db + i * d_i + j * d_j] = tile[tx][k];
        }
        __syncthreads();
    }
}

// Tile: out[o] = x[src(o)] with src dims taken modulo the input shape (c.py:571-588).
struct TileParams {
    long long oshape[COPY_MAX_RANK];
    long long xshape[COPY_MAX_RANK];
    long long xstr[COPY_MAX_RANK];
    long long total;
    const char *src;
    char *dst;
    int32_t rank;
    int32_t esize;
};

template <typename T>
__global__ void __launch_bounds__(256) tile_kernel(const __grid_constant__ TileParams P) {
    const T *src = (const T *)P.src;
    T *dst = (T *)P.dst;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long o = (long long)blockIdx.x * blockDim.x + threadIdx.x; o < P.total; o += stride) {
        long long rem = o, s = 0;
        for (int k = P.rank - 1; k >= 0; --k) {
            long long i = rem % P.oshape[k];
            rem /= P.oshape[k];
            s += (i % P.xshape[k]) * P.xstr[k];
        }
        dst[o] = src[s];
    }
}

// ---------------------------------------------------------------------------------------------
// explicit im2col of an NHWC image: out[m][k], m = (image, oh, ow), k = (kh, kw, c) for
// k < KH*KW*cg and zero up to the row length kp (a multiple of 4); rows of kp fp32
// ---------------------------------------------------------------------------------------------
struct Im2colParams {
    int N, H, W, C, KH, KW, SH, SW, DH, DW, PT, PL, OH, OW, kp, c_off, cg;
    const float *x;
    float *out;
};

__global__ void __launch_bounds__(256) im2col_nhwc_kernel(const __grid_constant__ Im2colParams p) {
    const int kq = p.kp / 4;
    const long long rows = (long long)p.N * p.OH * p.OW;
    const long long total = rows * kq;
    const int kreal = p.KH * p.KW * p.cg;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
        const long long m = e / kq;
        const int k0 = (int)(e - m * kq) * 4;
        const long long hw = (long long)p.OH * p.OW;
        const int img = (int)(m / hw);
        const int pix = (int)(m - (long long)img * hw);
        const int oh = pix / p.OW, ow = pix - oh * p.OW;
        float v[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int k = k0 + t;
            float val = 0.0f;
            if (k < kreal) {
                const int kh = k / (p.KW * p.cg);
                const int rem = k - kh * p.KW * p.cg;
                const int kw = rem / p.cg, c = rem - kw * p.cg;
                const int ih = oh * p.SH - p.PT + kh * p.DH, iw = ow * p.SW - p.PL + kw * p.DW;
                if (ih >= 0 && ih < p.H && iw >= 0 && iw < p.W)
                    val = p.x[(((long long)img * p.H + ih) * p.W + iw) * p.C + p.c_off + c];
            }
            v[t] = val;
        }
        *reinterpret_cast<float4 *>(p.out + m * p.kp + k0) = make_float4(v[0], v[1], v[2], v[3]);
    }
}

// Channel packing with optional spatial padding: out is NHWC [N][Hp][Wp][cp] (cp % 4 == 0) with
// out[n, PT + h, PL + w, c] = x at n*sn + h*sh + w*sw + c*sc for h < H, w < W, c < C, and zero
// everywhere else (padding channels and the border). One thread per output pixel; the source
// reads of neighbouring threads are neighbouring for both NCHW (sw = 1) and NHWC (sc = 1)
// sources, and every write is a 16-byte store.
struct PackParams {
    int N, H, W, C, cp, PT, PL, Hp, Wp;
    long long sn, sh, sw, sc;
    const float *x;
    float *out;
    // phase-split rows (phases = 2, cp = 4, Wp = 2 * Wq): packed row r of an image holds, for
    // phase f = 0, 1 and i < Wq, image column 2 i + f - PL of image row r - PT (zero outside the
    // image), every value rounded to the nearest TF32 value (the tensor core truncates what a
    // bulk copy brings in). phases = 0: plain NHWC pixels at (r - PT, w - PL).
    int phases;
};

// Round fp32 to the nearest TF32 value (10 explicit mantissa bits; ties away from zero), as a
// TFLOAT32 tensor map does on load; infinities and NaNs pass unchanged.
__device__ __forceinline__ float round_tf32(float x) {
    const uint32_t b = __float_as_uint(x);
    return (b & 0x7F800000u) == 0x7F800000u ? x : __uint_as_float((b + 0x1000u) & 0xFFFFE000u);
}

// Phase-split packing (PackParams.phases = 2), one packed 4-channel pixel per thread and
// iteration, 32-bit indices (the launcher checks the sizes).
__global__ void __launch_bounds__(256) pack_phase_kernel(const __grid_constant__ PackParams p) {
    const unsigned wq = (unsigned)p.Wp >> 1;
    const unsigned per_row = (unsigned)p.Wp;  // both phases
    const unsigned per_img = (unsigned)p.Hp * per_row;
    const unsigned total = (unsigned)p.N * per_img;
    const unsigned stride = gridDim.x * blockDim.x;
    for (unsigned e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
        const unsigned n = e / per_img;
        const unsigned r = e - n * per_img;
        const unsigned row = r / per_row;
        const unsigned q = r - row * per_row;
        const unsigned f = q >= wq ? 1u : 0u;
        const int h = (int)row - p.PT;
        const int w = 2 * (int)(q - f * wq) + (int)f - p.PL;
        const bool inside = h >= 0 && h < p.H && w >= 0 && w < p.W;
        const float *src =
            p.x + (inside ? n * (unsigned)p.sn + (unsigned)h * (unsigned)p.sh + (unsigned)w * (unsigned)p.sw : 0u);
        float v[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) v[t] = inside && t < p.C ? round_tf32(__ldg(src + (unsigned)t * (unsigned)p.sc)) : 0.0f;
        reinterpret_cast<float4 *>(p.out)[e] = make_float4(v[0], v[1], v[2], v[3]);
    }
}

// The same packing, one block per packed row (blockIdx.y = image * Hp + row, no divisions) and one
// thread per pixel index j of both phases: the phase-0 pixel reads input column 2 j - PL + 0 and
// the phase-1 pixel column 2 j - PL + 1 (adjacent), so a warp
// reads 64 consecutive columns of each channel plane and writes two runs of 32 packed pixels;
// the other kernel's threads each read every other column. Same values (round_tf32 of the same
// elements, zeros outside the image).
__global__ void __launch_bounds__(128) pack_phase_rows_kernel(const __grid_constant__ PackParams p) {
    const unsigned wq = (unsigned)p.Wp >> 1;
    const unsigned j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= wq) return;
    const unsigned n = blockIdx.y / (unsigned)p.Hp, row = blockIdx.y - n * (unsigned)p.Hp;
    const int h = (int)row - p.PT;
    float4 *dst = reinterpret_cast<float4 *>(p.out) + (size_t)blockIdx.y * p.Wp + j;
    if (h < 0 || h >= p.H) {
        dst[0] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        dst[wq] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        return;
    }
    const float *base = p.x + n * (unsigned)p.sn + (unsigned)h * (unsigned)p.sh;
    float v[2][4];
#pragma unroll
    for (int f = 0; f < 2; ++f) {
        const int w = 2 * (int)j + f - p.PL;
        const bool inside = w >= 0 && w < p.W;
#pragma unroll
        for (int t = 0; t < 4; ++t)
            v[f][t] = inside && t < p.C ? round_tf32(__ldg(base + (unsigned)w * (unsigned)p.sw + (unsigned)t * (unsigned)p.sc))
                                        : 0.0f;
    }
    dst[0] = make_float4(v[0][0], v[0][1], v[0][2], v[0][3]);
    dst[wq] = make_float4(v[1][0], v[1][1], v[1][2], v[1][3]);
}

// The same packing with 32-bit index arithmetic (pixel counts and source offsets below 2^31).
__global__ void __launch_bounds__(256) pack_nhwc32_kernel(const __grid_constant__ PackParams p) {
    const unsigned hw = (unsigned)p.Hp * (unsigned)p.Wp;
    const unsigned total = (unsigned)p.N * hw;
    const unsigned stride = gridDim.x * blockDim.x;
    for (unsigned e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
        const unsigned n = e / hw;
        const unsigned r = e - n * hw;
        const unsigned hq = r / (unsigned)p.Wp;
        const int h = (int)hq - p.PT, w = (int)(r - hq * (unsigned)p.Wp) - p.PL;
        const bool inside = h >= 0 && h < p.H && w >= 0 && w < p.W;
        const float *src =
            p.x + (inside ? n * (unsigned)p.sn + (unsigned)h * (unsigned)p.sh + (unsigned)w * (unsigned)p.sw : 0u);
        float4 *dst = reinterpret_cast<float4 *>(p.out) + (size_t)e * (p.cp >> 2);
        for (int c0 = 0; c0 < p.cp; c0 += 4) {
            float v[4];
#pragma unroll
            for (int t = 0; t < 4; ++t)
                v[t] = inside && c0 + t < p.C ? __ldg(src + (unsigned)(c0 + t) * (unsigned)p.sc) : 0.0f;
            dst[c0 >> 2] = make_float4(v[0], v[1], v[2], v[3]);
        }
    }
}

__global__ void __launch_bounds__(256) pack_nhwc_kernel(const __grid_constant__ PackParams p) {
    const long long hw = (long long)p.Hp * p.Wp;
    const long long total = (long long)p.N * hw;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
        const long long n = e / hw;
        const long long r = e - n * hw;
        const long long h = r / p.Wp - p.PT, w = r % p.Wp - p.PL;
        const bool inside = h >= 0 && h < p.H && w >= 0 && w < p.W;
        const float *src = p.x + n * p.sn + h * p.sh + w * p.sw;
        float4 *dst = reinterpret_cast<float4 *>(p.out + e * p.cp);
        for (int c0 = 0; c0 < p.cp; c0 += 4) {
            float v[4];
#pragma unroll
            for (int t = 0; t < 4; ++t)
                v[t] = inside && c0 + t < p.C ? __ldg(src + (long long)(c0 + t) * p.sc) : 0.0f;
            dst[c0 >> 2] = make_float4(v[0], v[1], v[2], v[3]);
        }
    }
}

// ---------------------------------------------------------------------------------------------
// fill / range / gather
// ---------------------------------------------------------------------------------------------
template <typename T>
__global__ void fill_kernel(T *dst, long long n, T value) {
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long o = (long long)blockIdx.x * blockDim.x + threadIdx.x; o < n; o += stride) dst[o] = value;
}

// y[i] = start + i * delta, start/delta read from device scalars of dtype dt (c.py:724-734).
__global__ void range_kernel(void *y, int dt, long long n, const void *start, const void *delta) {
    const long long stride = (long long)gridDim.x * blockDim.x;
    Reg s = load_elem(start, dt, 0), d = load_elem(delta, dt, 0);
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        Reg v;
        if (dt == MGC_F32) v.f = s.f + (float)i * d.f;
        else if (dt == MGC_F64) v.d = s.d + (double)i * d.d;
        else v.i = s.i + i * d.i;
        store_elem(y, dt, i, v);
    }
}

// out[(o * n + t) * inner + j] = x[(o * dim + k) * inner + j], k = idx[t] (+dim if negative).
// An out-of-range index sets *status (the C backend returns 1 from mgc_run, c.py:678-680) and
// writes zeros for that row.
template <typename T>
__global__ void __launch_bounds__(256) gather_kernel(const T *x, const void *idx, int idx_dt, T *out,
                                                     long long outer, long long dim, long long inner,
                                                     long long n, int *status) {
    const long long total = outer * n * inner;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
        long long j = e % inner;
        long long t = (e / inner) % n;
        long long o = e / (inner * n);
        long long k = idx_dt == MGC_I32 ? (long long)((const int *)idx)[t] : ((const long long *)idx)[t];
        if (k < 0) k += dim;
        if (k < 0 || k >= dim) {
            if (status) atomicExch(status, MGC_CUDA_GATHER_OOB);
            out[e] = T(0);
            continue;
        }
        out[e] = x[(o * dim + k) * inner + j];
    }
}

// ---------------------------------------------------------------------------------------------
// reductions over the middle axis of [outer, n, inner]
// ---------------------------------------------------------------------------------------------
// mgc_reduce_mid (mgc_kernels.c:593-612): float mean / max, sequential fp32 accumulation.
__global__ void __launch_bounds__(256) reduce_mid_kernel(int is_max, long long outer, long long n,
                                                         long long inner, const float *x, float *y) {
    const long long total = outer * inner;
    const long long stride = (long long)gridDim.x * blockDim.x;
    const float inv = n > 0 ? 1.0f / (float)n : 0.0f;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
        long long o = e / inner, i = e % inner;
        const float *src = x + o * n * inner + i;
        float acc = is_max ? -INFINITY : 0.0f;
        for (long long k = 0; k < n; ++k) {
            float v = src[k * inner];
            acc = is_max ? (v > acc ? v : acc) : acc + v;
        }
        y[e] = is_max ? acc : acc * inv;
    }
}

// GlobalAveragePool from the producing GEMM's partials (its epilogue's gap_hw form): y[o][c] =
// (sum over the 32-row groups g holding rows of image o, in order, of part[2 g + (o - first image
// of g)][c]) * (1 / n), n >= 32 pixels per image (a group holds rows of at most two images). The
// mean's scale as reduce_mid_kernel's; the sum's order is by groups instead of row by row.
__global__ void __launch_bounds__(256) gap_partials_kernel(long long outer, long long n, long long inner,
                                                           const float *part, float *y) {
    const long long total = outer * inner;
    const long long stride = (long long)gridDim.x * blockDim.x;
    const float inv = 1.0f / (float)n;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
        const long long o = e / inner, c = e % inner;
        const long long g0 = o * n / 32, g1 = ((o + 1) * n - 1) / 32;
        float acc = 0.0f;
        for (long long g = g0; g <= g1; ++g) acc += part[(2 * g + (o - g * 32 / n)) * inner + c];
        y[e] = acc * inv;
    }
}

// Generic ReduceSum/Mean/Prod/Max/Min (c.py:736-784): double accumulator for float sum, mean
// and prod, the element type otherwise.
enum { RED_SUM = 0, RED_MEAN = 1, RED_PROD = 2, RED_MAX = 3, RED_MIN = 4 };

__global__ void __launch_bounds__(256) reduce_kernel(int kind, int dt, long long outer, long long n,
                                                     long long inner, const void *x, void *y) {
    const long long total = outer * inner;
    const long long stride = (long long)gridDim.x * blockDim.x;
    const int c = class_of(dt);
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
        long long o = e / inner, i = e % inner;
        long long base = o * n * inner + i;
        Reg out;
        if (c != CL_I) {
            double acc = kind == RED_PROD ? 1.0 : kind == RED_MAX ? -INFINITY : kind == RED_MIN ? INFINITY : 0.0;
            for (long long k = 0; k < n; ++k) {
                double v = as_d(load_elem(x, dt, base + k * inner), c);
                if (kind == RED_SUM || kind == RED_MEAN) acc += v;
                else if (kind == RED_PROD) acc *= v;
                else if (kind == RED_MAX) acc = v > acc ? v : acc;
                else acc = v < acc ? v : acc;
            }
            if (kind == RED_MEAN) acc = acc / (double)n;
            if (c == CL_F) out.f = (float)acc; else out.d = acc;
        } else {
            long long acc = kind == RED_PROD ? 1 : kind == RED_MAX ? LLONG_MIN : kind == RED_MIN ? LLONG_MAX : 0;
            for (long long k = 0; k < n; ++k) {
                long long v = load_elem(x, dt, base + k * inner).i;
                if (kind == RED_SUM || kind == RED_MEAN) acc += v;
                else if (kind == RED_PROD) acc *= v;
                else if (kind == RED_MAX) acc = v > acc ? v : acc;
                else acc = v < acc ? v : acc;
            }
            if (kind == RED_MEAN) acc = n ? acc / n : 0;
            out.i = acc;
        }
        store_elem(y, dt, e, out);
    }
}

// ArgMax along the middle axis, first maximum wins (c.py:801-821).
__global__ void __launch_bounds__(256) argmax_kernel(int dt, long long outer, long long n, long long inner,
                                                     const void *x, long long *y) {
    const long long total = outer * inner;
    const long long stride = (long long)gridDim.x * blockDim.x;
    const int c = class_of(dt);
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
        long long o = e / inner, i = e % inner;
        long long base = o * n * inner + i;
        long long best = 0;
        if (c == CL_I) {
            long long bv = load_elem(x, dt, base).i;
            for (long long k = 1; k < n; ++k) {
                long long v = load_elem(x, dt, base + k * inner).i;
                if (v > bv) { bv = v; best = k; }
            }
        } else {
            double bv = as_d(load_elem(x, dt, base), c);
            for (long long k = 1; k < n; ++k) {
                double v = as_d(load_elem(x, dt, base + k * inner), c);
                if (v > bv) { bv = v; best = k; }
            }
        }
        y[e] = best;
    }
}

}  // namespace mgc
