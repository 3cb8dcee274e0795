/* C ABI of libmgc_cuda.so: the B200 (sm_100a) backend of ml-graph-compiler's `cuda` target.
 *
 * The reference compiler's C backend turns a scheduled, memory-planned graph into a generated
 * function `mgc_run(inputs, outputs, A, W)` plus `mgc_arena_bytes()` / `mgc_weights_bytes()`
 * (reference: src/ml_graph_compiler/codegen/c.py:1308-1312), which calls the runtime kernels
 * declared in codegen/runtime/mgc_runtime.h:161-206 and is bound with ctypes in
 * codegen/runtime_lib.py:59-68.
 *
 * This library replaces both halves without generating code per model:
 *   - the model ABI (mgc_cuda_create / _run / _destroy ...) takes the scheduled node list as a
 *     launch list (an array of mgc_cuda_launch records built by the Python lowering from the
 *     reference's graph and MemoryPlan), the constant blob and the arena size; it owns one
 *     cudaMalloc'd arena with the planner's offsets, the resident weights, the input/output
 *     buffers and a CUDA Graph of the whole schedule;
 *   - the kernel ABI (mgc_cuda_gemm, mgc_cuda_softmax, ...) mirrors the runtime kernels of
 *     mgc_runtime.h with device pointers and a stream, and mgc_cuda_execute runs any list of
 *     launch records whose references are raw device pointers.
 * All entry points return 0 on success; on failure they return a status below and
 * mgc_cuda_last_error() describes it. Nothing here uses torch types.
 */
#ifndef MGC_CUDA_H
#define MGC_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MGC_CUDA_ABI_VERSION 3

/* ---- status codes (runtime_lib.py:142-143 maps mgc_run's 1 to GraphError) ---------------- */
enum {
    MGC_CUDA_OK = 0,
    MGC_CUDA_GATHER_OOB = 1,     /* a Gather index was out of range (device flag, c.py:678-680) */
    MGC_CUDA_BAD_ARGUMENT = 2,   /* malformed launch list, size mismatch, unsupported parameter */
    MGC_CUDA_UNSUPPORTED = 3,    /* a launch kind / dtype / shape this build has no kernel for */
    MGC_CUDA_TIMEOUT = 4,        /* a bounded device wait gave up (kernel returned early) */
    MGC_CUDA_CUDA_ERROR = 100    /* >= 100: 100 + cudaError_t of the failing CUDA call */
};

/* ---- where a launch operand lives (memory.py:49-55 Location kinds, plus RAW pointers) ----- */
enum {
    MGC_SPACE_NONE = 0,      /* operand absent */
    MGC_SPACE_ARENA = 1,     /* byte offset into the planner's arena (memory.py:169-316) */
    MGC_SPACE_WEIGHTS = 2,   /* byte offset into the resident constant blob */
    MGC_SPACE_INPUT = 3,     /* graph input `index`, byte offset within it */
    MGC_SPACE_OUTPUT = 4,    /* graph output `index`, byte offset within it */
    MGC_SPACE_RAW = 5,       /* `offset` is a device address (kernel ABI / mgc_cuda_execute) */
    MGC_SPACE_WORKSPACE = 6  /* byte offset into the handle's scratch buffer (im2col of narrow
                                convolutions); not part of the planner's arena */
};

/* ---- element types (ir.py:20-29) ------------------------------------------------------------ */
enum {
    MGC_F32 = 0,
    MGC_F64 = 1,
    MGC_I64 = 2,
    MGC_I32 = 3,
    MGC_I8 = 4,
    MGC_U8 = 5,
    MGC_BOOL = 6
};

/* ---- activations fused into epilogues (mgc_runtime.h:93-101, ops.py:894-911) ---------------- */
enum {
    MGC_ACT_NONE = 0,
    MGC_ACT_RELU,
    MGC_ACT_CLIP,
    MGC_ACT_GELU,
    MGC_ACT_GELU_TANH,
    MGC_ACT_TANH,
    MGC_ACT_SIGMOID
};

/* ---- GEMM operand kinds (mgc_runtime.h:123-137) -------------------------------------------- */
enum {
    MGC_STRIDED = 0,     /* element (r, c) = p[r*rs + c*cs] */
    MGC_CONV_NHWC = 2,   /* A: implicit im2col of an NHWC image, row = output pixel */
    MGC_CONV_NCHW = 3    /* B: implicit im2col of an NCHW image, column = output pixel */
};

/* ---- arithmetic of the GEMM family ---------------------------------------------------------- */
enum {
    MGC_PREC_FP32 = 0,    /* exact fp32 FMA on the CUDA cores */
    MGC_PREC_TF32 = 1,    /* tcgen05 kind::tf32, fp32 accumulate */
    MGC_PREC_3XTF32 = 2   /* tcgen05, big/small operand split (strict fp32 semantics) */
};

/* ---- launch kinds: one record per kernel launch ---------------------------------------------
 * Integer parameters live in i[], float parameters in f[], tensor operands in r[]. The meaning
 * of each slot per kind is listed in mgc_cuda/lowering.py next to the code that fills it; the
 * C++ side reads the same slots (csrc/launch.cuh). Kinds mirror the C emitter's lowerings. */
enum {
    MGC_K_GEMM = 1,         /* op_FusedGemm / op_Gemm / op_MatMul / op_FusedConv (c.py:974-1226) */
    MGC_K_DEPTHWISE = 2,    /* mgc_depthwise_nhwc / _nchw (mgc_kernels.c:455-504) */
    MGC_K_POOL = 3,         /* mgc_pool_nhwc / _nchw (mgc_kernels.c:526-591) */
    MGC_K_REDUCE_MID = 4,   /* mgc_reduce_mid (mgc_kernels.c:593-612) */
    MGC_K_SOFTMAX = 5,      /* mgc_softmax (mgc_kernels.c:618-655) */
    MGC_K_LAYER_NORM = 6,   /* mgc_layer_norm (mgc_kernels.c:657-679) */
    MGC_K_ELEMENTWISE = 7,  /* generated loop nests for elementwise / FusedElementwise (c.py:471-529) */
    MGC_K_COPY = 8,         /* Transpose/Expand/Slice/Concat/Split/Pad/Tile loop nests (c.py:558-660) */
    MGC_K_FILL = 9,         /* constant writes: Pad fill, ConstantOfShape, Shape, Size (c.py:690-722) */
    MGC_K_GATHER = 10,      /* op_Gather with the out-of-range check (c.py:662-688) */
    MGC_K_REDUCE = 11,      /* generic reductions with a double accumulator (c.py:736-784) */
    MGC_K_ARGMAX = 12,      /* op_ArgMax (c.py:801-821) */
    MGC_K_RANGE = 13,       /* op_Range (c.py:724-734) */
    MGC_K_MEMCPY = 14,      /* output copies of plan.copies and constant stores (c.py:1283-1285) */
    MGC_K_IM2COL = 15,      /* explicit im2col of an NHWC image into the workspace, for
                               convolutions whose channel rows TMA cannot address (C % 4 != 0);
                               the packing of pack_a's MGC_CONV_NHWC branch, mgc_kernels.c:103-126 */
    MGC_K_PACK = 16,        /* copy of a 4-D image with any strides into NHWC with the channels
                               zero-padded to a multiple of 4, so that TMA can address its pixels
                               (a narrow-channel convolution input, e.g. the 3-channel stem); no
                               counterpart in the reference, whose C kernels read 3-float rows */
    MGC_K_ATTENTION = 17    /* TF32 mode: MatMul(Q, K^T) -> score program (scale, mask) ->
                               Softmax -> MatMul(P, V) as one tcgen05 kernel, the scores kept
                               on chip; the reference's C backend runs the four nodes as
                               separate loops (c.py:823-852, 974-1226) */
};

typedef struct {
    int32_t space;   /* MGC_SPACE_* */
    int32_t index;   /* graph input / output number for MGC_SPACE_INPUT / OUTPUT */
    int64_t offset;  /* byte offset (or device address for MGC_SPACE_RAW) */
} mgc_cuda_ref;

#define MGC_LAUNCH_INTS 64
#define MGC_LAUNCH_FLOATS 8
#define MGC_LAUNCH_REFS 8

typedef struct {
    int32_t kind;    /* MGC_K_* */
    int32_t node;    /* index of the scheduled node that emitted it (profiling) */
    int32_t dtype;   /* element type of the main operand */
    int32_t flags;
    int64_t i[MGC_LAUNCH_INTS];
    double f[MGC_LAUNCH_FLOATS];
    mgc_cuda_ref r[MGC_LAUNCH_REFS];
    int64_t aux_offset; /* first int64 of this record's variable-length data in the aux array */
    int64_t aux_len;
} mgc_cuda_launch;

/* Description of one graph input or output buffer. */
typedef struct {
    int64_t nbytes;
} mgc_cuda_io;

/* ---- model ABI -------------------------------------------------------------------------------
 * mgc_cuda_create replaces loading the generated library and its weights blob
 * (runtime_lib.py:44-83 CompiledModel.__init__, c.py:1308-1309 mgc_arena_bytes/mgc_weights_bytes):
 * it uploads `weights_bytes` of constants once, allocates the arena (`arena_bytes`, the
 * planner's MemoryPlan.arena_bytes) and device buffers for the graph inputs and outputs,
 * resolves every record's references to device addresses, and captures the launch list into a
 * CUDA Graph on its own stream. `workspace_bytes` sizes the scratch buffer that MGC_SPACE_WORKSPACE
 * references point into (0 when no launch uses one). `device` is the CUDA ordinal. */
int mgc_cuda_create(const mgc_cuda_launch *launches, int n_launches, const int64_t *aux,
                    int64_t aux_len, const void *weights_host, int64_t weights_bytes,
                    int64_t arena_bytes, int64_t workspace_bytes, const mgc_cuda_io *inputs,
                    int n_inputs, const mgc_cuda_io *outputs, int n_outputs, int device,
                    void **handle);

/* Replaces `int mgc_run(const void *const *inputs, void *const *outputs, A, W)` (c.py:1311-1312,
 * called at runtime_lib.py:135-140): copies each host input to the device (pinned host memory
 * makes this asynchronous), replays the CUDA Graph, copies each output back to its host buffer
 * and waits. Returns MGC_CUDA_GATHER_OOB when a Gather index was out of range. */
int mgc_cuda_run(void *handle, const void *const *inputs_host, void *const *outputs_host);

/* Input-upload overlap for mgc_cuda_run (no counterpart in the reference, whose mgc_run reads
 * host memory directly). After this call, mgc_cuda_run copies input 0 in `chunks` equal slices of
 * `images / chunks` images on a copy stream and replays a second CUDA Graph in which the first
 * `prefix` launch records run once per slice, each slice starting when its copy has landed, so
 * the copy of slice j+1 overlaps the compute of slice j; the remaining records then run once on
 * the whole batch. The caller (the lowering) guarantees that the prefix works image by image on
 * batch-major tensors whose memory is not shared between different layouts. Each descriptor
 * names one batch-dependent field of a prefix record: `what` 0, reference r[slot] advances by
 * `per_image` bytes per image of the slice's start; `what` 1, integer i[slot] becomes `per_image`
 * times the slice's images; `what` 2, reference r[slot] becomes workspace byte `per_image`, the
 * same for every slice (a buffer that only the prefix reads, moved out of memory it shares with
 * one the rest of the graph reads into a private region of one slice's size, which the caller
 * includes in the handle's workspace). mgc_cuda_run_device keeps the one-pass graph. Requires one
 * graph input; chunks 2..16 dividing `images`, which divides input 0's bytes. */
typedef struct {
    int32_t launch;    /* index of the record, below `prefix` */
    int32_t what;      /* 0 reference offset, 1 integer field, 2 reference into the workspace */
    int32_t slot;      /* r[] or i[] index */
    int32_t reserved;
    int64_t per_image; /* bytes (what 0) or count (what 1) per image; workspace offset (what 2) */
} mgc_cuda_chunk;

int mgc_cuda_set_input_chunks(void *handle, int chunks, int prefix, int64_t images,
                              const mgc_cuda_chunk *descs, int n_descs);

/* The same replay with the inputs already in the handle's device input buffers and the outputs
 * left in its device output buffers; enqueued on the handle's stream without waiting when
 * `sync` is 0 (for device-timed throughput). */
int mgc_cuda_run_device(void *handle, int sync);

/* Device addresses of the handle's graph input / output buffers and its stream (cudaStream_t). */
void *mgc_cuda_input_ptr(void *handle, int i);
void *mgc_cuda_output_ptr(void *handle, int i);
void *mgc_cuda_stream(void *handle);

/* Per-node profile (replaces the profile=True build, c.py:1278-1302 and runtime_lib.py:107-115):
 * runs the launch list once without the graph, timing each scheduled node with CUDA events,
 * and writes the milliseconds of node k into per_node_ms[k] for k < n. */
int mgc_cuda_profile(void *handle, double *per_node_ms, int n);

/* Number of kernel launches in one replay of the handle's graph. */
int mgc_cuda_launch_count(void *handle);

/* Which kernel computes each GEMM-family launch record (FusedConv, FusedGemm, Gemm, MatMul, and
 * the fused attention of MGC_K_ATTENTION, whose two products run on tcgen05) of the handle's
 * graphs: per_record[k] for record k < n is MGC_CUDA_PATH_NONE for a record of another kind, MGC_CUDA_PATH_TCGEN05 when the tcgen05 tensor-core kernel runs it, and
 * MGC_CUDA_PATH_SIMT when the exact-fp32 CUDA-core kernel does (fp32 precision, or a problem
 * the tensor-core forms cannot describe). No counterpart in the reference, whose C backend has
 * one GEMM kernel; the reference's CompileReport.kernels (runtime_lib.py:31-41) counts kernels
 * by kind only. A record that runs slice by slice (mgc_cuda_set_input_chunks) reports SIMT if
 * any of its slices does. */
enum { MGC_CUDA_PATH_NONE = 0, MGC_CUDA_PATH_TCGEN05 = 1, MGC_CUDA_PATH_SIMT = 2 };
int mgc_cuda_gemm_paths(void *handle, int32_t *per_record, int n);

int64_t mgc_cuda_arena_bytes(void *handle);
int64_t mgc_cuda_weights_bytes(void *handle);
void mgc_cuda_destroy(void *handle);

/* Text of the last error on this thread (empty when none). */
const char *mgc_cuda_last_error(void);

/* Replaces mgc_has_openmp / mgc_has_neon (mgc_runtime.h:172-173): 1 when device `device` is an
 * sm_100 part this library's tcgen05 kernels run on, 0 otherwise (or on error). */
int mgc_cuda_device_supported(int device);
int mgc_cuda_abi_version(void);

/* ---- kernel ABI ------------------------------------------------------------------------------
 * Runs `n` launch records whose references are MGC_SPACE_RAW device addresses on `stream`
 * (a cudaStream_t, 0 for the legacy default stream). `status_dev`, if not NULL, is a device int
 * that Gather kernels set to MGC_CUDA_GATHER_OOB. */
int mgc_cuda_execute(const mgc_cuda_launch *launches, int n, const int64_t *aux, int64_t aux_len,
                     int *status_dev, void *stream);

/* GEMM with fused epilogue, the device counterpart of mgc_gemm (mgc_runtime.h:139-162):
 *   C[b] = act(alpha * A[b] x B[b] + bias + beta * R[b]),  b < batch,
 * A is M x K with element (m, k) at a[m*a_rs + k*a_cs], B is K x N at b[k*b_rs + n*b_cs], C and
 * R are M x N with leading dimensions ldc / ldr. Batch item b is offset by b*stride elements
 * (mgc_gemm takes per-item offset arrays; a constant stride covers conv batches and MatMul).
 * bias_mode 1 adds bias[n], 2 adds bias[m]. precision:
 *   MGC_PREC_FP32  exact fp32 FMA on the CUDA cores (the reference's arithmetic), any strides;
 *   MGC_PREC_TF32  the tcgen05 tensor cores, A and B rounded to TF32 on load, fp32 accumulate;
 *                  needs A and B K-major (a_cs == 1, b_rs == 1) with 16-byte aligned bases and
 *                  row strides, K and N multiples of 4, no per-row bias, and for batch > 1 no
 *                  bias, residual, activation or alpha; anything else returns
 *                  MGC_CUDA_UNSUPPORTED (nothing runs);
 *   MGC_PREC_3XTF32 returns MGC_CUDA_UNSUPPORTED: the strict split needs constant weights laid
 *                  out at load time, which the model ABI (mgc_cuda_create) does. */
int mgc_cuda_gemm(int M, int N, int K, int batch, const float *a, int64_t a_rs, int64_t a_cs,
                  int64_t a_bstride, const float *b, int64_t b_rs, int64_t b_cs, int64_t b_bstride,
                  float *c, int64_t ldc, int64_t c_bstride, float alpha, const float *bias,
                  int bias_mode, const float *res, int64_t ldr, int64_t r_bstride, float beta,
                  int act, float lo, float hi, int precision, void *stream);

/* Implicit-GEMM NHWC convolution with the FusedConv epilogue (c.py:1146-1185 lowering onto
 * mgc_gemm with MGC_CONV_NHWC, mgc_kernels.c:103-126): x [N,H,W,C], w HWIO [KH,KW,C,CO],
 * y = act(conv + bias[co] + res), y and res [N,OH,OW,CO]. group must be 1. precision must be
 * MGC_PREC_FP32 (exact fp32 on the CUDA cores, the reference's arithmetic); TF32 and 3xTF32
 * return MGC_CUDA_UNSUPPORTED, because their tensor-core forms read the weights in a K-major
 * layout that the model ABI prepares at load time, not HWIO. */
int mgc_cuda_conv_nhwc(int N, int H, int W, int C, int KH, int KW, int SH, int SW, int DH, int DW,
                       int PT, int PL, int OH, int OW, int CO, const float *x, const float *w,
                       const float *bias, const float *res, int act, float lo, float hi,
                       float *y, int precision, void *stream);

/* No counterpart in the reference. The same convolution as mgc_cuda_conv_nhwc, computed as an
 * explicit im2col followed by an exact-fp32 GEMM, for callers that cannot allocate device memory:
 * code that plans every byte up front and never allocates after start-up (the discipline of the
 * reference's static arena, whose generated code allocates nothing), or code running where a
 * cudaMalloc is not allowed or would stall other work. The im2col scratch lives in a fixed,
 * file-scope device array of MGC_CUDA_NOALLOC_SCRATCH_BYTES (16 MiB) that every GPU loading the
 * library holds until exit; a convolution whose patch matrix (N*OH*OW rows of KH*KW*C floats,
 * rounded up to a multiple of 4) does not fit is rejected with MGC_CUDA_BAD_ARGUMENT. The first
 * call on a device looks the array's device address up (cudaGetSymbolAddress), so make that first
 * call before any stream capture. All calls share the array: calls that overlap on the GPU (other
 * streams, other threads) race on it; serialise them. Nothing is allocated or freed. */
#define MGC_CUDA_NOALLOC_SCRATCH_BYTES (16 * 1024 * 1024)
int mgc_cuda_conv_nhwc_noalloc(int N, int H, int W, int C, int KH, int KW, int SH, int SW, int DH,
                               int DW, int PT, int PL, int OH, int OW, int CO, const float *x,
                               const float *w, const float *bias, const float *res, int act,
                               float lo, float hi, float *y, void *stream);

/* Same signatures as mgc_runtime.h:182-207, plus the stream. */
int mgc_cuda_depthwise_nhwc(int N, int H, int W, int C, int KH, int KW, int SH, int SW, int DH,
                            int DW, int PT, int PL, int OH, int OW, const float *x, const float *w,
                            const float *bias, const float *res, int act, float lo, float hi,
                            float *y, void *stream);
int mgc_cuda_pool_nhwc(int is_max, int N, int H, int W, int C, int KH, int KW, int SH, int SW,
                       int DH, int DW, int PT, int PL, int PB, int PR, int OH, int OW,
                       int count_include_pad, const float *x, float *y, void *stream);
int mgc_cuda_reduce_mid(int is_max, int64_t outer, int64_t n, int64_t inner, const float *x,
                        float *y, void *stream);
int mgc_cuda_softmax(int64_t outer, int64_t n, int64_t inner, const float *x, float *y,
                     int log_softmax, void *stream);
int mgc_cuda_layer_norm(int64_t rows, int64_t cols, const float *x, const float *scale,
                        const float *bias, float eps, float *y, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* MGC_CUDA_H */
