// tcgen05 (UMMA) implicit-GEMM / GEMM for sm_100a with the fused FusedConv / FusedGemm epilogue.
//
// C[m, n] = act(alpha * sum_k A[m, k] * B[n, k] + bias[n] + R[m, n]), fp32 in and out.
//
// Data movement
// * A (activations) is loaded by TMA into 128B-swizzled shared memory, 128 rows x 32 fp32 per
//   K block: either a tiled 2-D box of a row-major [M, K] matrix (pointwise convolutions,
//   FusedGemm, Gemm), or an im2col box of an NHWC image (3x3 / strided / dilated convolutions:
//   128 consecutive output pixels x 32 channels at one filter tap; padding comes from the
//   tensor map's bounding box, out-of-image taps read as zero).
// * B (weights) is K-major [N][Kp] in the resident constant blob, stored by the lowering as a
//   TF32-exact high part and the fp32 residual (hi + lo == B exactly); for im2col the K axis is
//   (kh, kw, channel padded to 32).
//
// Arithmetic (measured on B200 with TF32-exact operands and TMA round trips): the tensor core reads fp32 operands by
// truncating them to TF32, and its accumulator rounds toward zero, a bias that compounds through
// deep networks. Both are handled explicitly:
// * MGC_PREC_TF32: A is loaded through a TFLOAT32 tensor map, which rounds it to the nearest
//   TF32 value; each K step issues one MMA of A against the stacked [B_hi; B_lo] tile (B exact
//   to fp32), so the only operand error is the unbiased rounding of the activations.
// * MGC_PREC_3XTF32 ("strict"): the epilogue warps split the raw A tile into hi = RN_tf32(A) and
//   lo = A - hi in shared memory; each K step issues A_lo*B_hi + A_hi*B_lo + A_hi*B_hi.
// * Accumulation: TF32 mode keeps a tile's whole K in one TMEM accumulator (double buffered
//   across tiles). Strict mode gives each of the four K=8 steps of a block its own region, which
//   the epilogue warps add into fp64 registers, so no tensor-core accumulation chain is longer
//   than one step.
//
// Roles: warp 0 issues TMA (lane 0, or the whole warp for the narrow-channel forms); warp 1
// allocates TMEM and lane 0 issues tcgen05.mma; warps 2-9 (256 threads: two per TMEM lane, each
// taking half of the tile's columns) split A (strict), drain TMEM, and run the epilogue.
//
// Every wait on an mbarrier is bounded (about a second of clock cycles); on timeout the kernel
// records MGC_CUDA_TIMEOUT in the error word, drains what it issued, frees its TMEM and returns.
// Every TMA copy lands in the shared memory of the CTA that issues it; a CTA pair shares B only
// through its cta_group::2 MMAs.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdlib.h>
#include <string.h>

#include <type_traits>

#include "common.cuh"
#include "gemm_simt.cuh"
#include "kernels_norm.cuh"

namespace mgc {
namespace umma {

constexpr int BM = 128;
constexpr int BK = 32;                       // fp32 elements per K block: one 128-byte swizzle row
constexpr uint32_t A_TILE_BYTES = BM * BK * 4;
constexpr long long WAIT_LIMIT_CYCLES = 1ll << 31;  // ~1.1 s at 1.9 GHz

// TF32 mode accumulates a tile's whole K in TMEM. Measured on ResNet-50 (batch 4 against the
// float64 oracle): promoting the accumulator to fp32 registers every 1, 2, 4 or 8 K blocks, or
// never, gives the same logit error (max 1.6-1.8e-2, mean |err| 3.6-3.7e-3, mean signed error
// within +-8e-5): the rounding of the activations to TF32 dominates, the accumulator's rounding
// toward zero over a long chain does not show.

// DYN: TF32 with a dynamic B (an activation, rounded to TF32 by its tensor map like A): one
// plane, one accumulator, tiles batched over up to two batch dimensions of 4-D tensor maps.
enum Mode { TF32 = 0, STRICT = 1, DYN = 2 };

// The tensor core's fp32 accumulation rounds toward zero. Strict mode keeps every K = 8 step in
// its own TMEM region, where three products land (A_lo*B_hi, A_hi*B_lo, A_hi*B_hi), so every
// output carries about the same relative shrink per region; below half an fp32 ulp per value, it
// compounds coherently through deep networks. Measured on B200 through this kernel with raw fp32
// operands and K = 512 (mean relative shrink of the outputs before compensation): 4.3e-8
// (uniform [0.5, 1.5)), 4.3e-8 (uniform [0, 1)), 4.1e-8 (half-normal), 5.0e-8 (uniform [1, 2));
// with TF32-exact operands (one product per region) 2.5e-8 to 3.9e-8. Batch-1 strict logits
// against the float64 oracle with this constant / with 2.5e-8 / without compensation: ResNet-50
// 1.5e-5 / 3.1e-5 / 9.2e-5, the other benchmark models unchanged at <= 2.1e-6. The strict epilogue
// forms alpha * acc * (1 + STEP_BIAS) + bias + residual in fp64 and rounds once.
constexpr double STEP_BIAS = 4.3e-8;

struct Params {
    CUtensorMap tmA;
    CUtensorMap tmB;                 // [2][N][Kp]: plane 0 B's TF32 part, plane 1 its residual
    CUtensorMap tmC;                 // output tile store (when tma_out)
    CUtensorMap tmR;                 // residual tile load (when tma_res)
    int tma_out, tma_res;
    int out2;                        // a second output staging tile (after the bias), used by
                                     // alternate epilogue passes: set by launch() when it fits
    int M, N, num_kb, n_tiles;
    int im2col;                      // 0 tiled A, 1 im2col (32-channel blocks), 2 tap-packed im2col,
                                     // 3 window rows, 4 row tiles, 5 phase-split row tiles
    int KW, DH, DW, cblocks;         // im2col: K block kb -> (kh, kw, channel block)
    int cpix, kreal;                 // tap-packed: channels per pixel (4..28), real K = KH*KW*cpix
    int wrows;                       // window rows (im2col 3): output pixels per box (divides OW)
    int rt_rows, rt_per_img;         // row tiles (im2col 4, 5): output rows per tile, tiles per image
    const char *a_rows;              // phase-split row tiles (im2col 5): the packed image's first row
    long long prow_bytes;            // bytes of one packed row (both phases)
    int prows, phase_bytes;          // packed rows per image; bytes of one phase of a row
    uint32_t a_bytes;                // bytes of one K block's A boxes (row tiles fill rt_rows*OW rows)
    uint32_t res_box_bytes;          // row tiles: bytes of one 32-column residual box (rt_rows*OW rows)
    int m_tiles;                     // ceil(M / 128) (DYN: times the batches)
    int m_per_batch, nbatch1;        // DYN: M tiles per batch; extent of the first batch dimension
    uint32_t b_res_bytes;            // B-resident kernels: bytes of this CTA's whole B panel
    int OH, OW, SH, SW, PT, PL;      // im2col: output pixel -> window origin
    float *c;
    long long ldc;
    const float *bias;
    const float *res;
    long long ldr;
    float alpha, lo, hi;
    int act;
    int *err;
    // split K (one-CTA TF32 tiles): work unit (tile, ks) runs K blocks [ks * kb_per,
    // (ks + 1) * kb_per) and leaves its raw partial tile in part ([tile][split][BM][BN]);
    // split_reduce_kernel sums the partials in split order and applies the epilogue.
    // splits <= 1: no split.
    int splits, kb_per;
    float *part;
    // phase-split row tiles with the 3x3 / stride-2 / pad-1 max pooling in the epilogue (pool_bp
    // > 0): CTA b walks bands b, b + gridDim.x, ... of pool_bp pooled rows; a band's tiles are
    // its 2 pool_bp + 1 output rows from 2 p0 - 1 (the row above the image is a dummy tile);
    // c is the pooled output [image][pool_ph][pool_pw][ldc]
    int pool_bp, pool_nbp, pool_nbands, pool_ph, pool_pw;
    // GlobalAveragePool partials (gap_hw > 0: rows per image, >= 32): instead of the output, each
    // 32-row group g of rows writes the column sums of the rows of its first image to c[2 g][.]
    // and of its second image (if any) to c[2 g + 1][.] (row stride ldc); K_REDUCE_MID mode 2
    // adds them per image
    int gap_hw;
};

// ---- PTX wrappers -----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Non-blocking test of the same (the thread never suspends); the result is read later, so the
// test's latency overlaps whatever the thread issues meanwhile.
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait for the phase with parity `parity` to complete. Returns false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > WAIT_LIMIT_CYCLES) return false;
    }
    return true;
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];"
        ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

__device__ __forceinline__ void tma_load_im2col_4d(void *dst, const CUtensorMap *map, uint64_t *bar, int c, int w,
                                                   int h, int n, uint16_t off_w, uint16_t off_h) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2], {%7, %8};"
        ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c), "r"(w), "r"(h),
        "r"(n), "h"(off_w), "h"(off_h)
        : "memory");
}

__device__ __forceinline__ void tma_load_5d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y, int z,
                                            int w, int v) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];"
        ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y), "r"(z),
        "r"(w), "r"(v)
        : "memory");
}

// ---- CTA pairs (cta_group::2) ------------------------------------------------------------------
// A pair of CTAs (a cluster of two) computes one 256-row tile: each CTA loads its own 128 rows of
// A and one plane of B (rank 0 the TF32 part, rank 1 the residual) into the same shared-memory
// offsets, and rank 0 issues MMAs with M = 256 that read both CTAs' operands and write each CTA's
// rows into its own TMEM. Every load of the pair completes on rank 0's stage barrier.
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_index() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
// Address of the same shared variable in the pair's rank-0 CTA (shared::cluster window).
__device__ __forceinline__ uint32_t leader_addr(const void *p) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(r) : "r"(smem_addr(p)));
    return r;
}
// All threads of both CTAs; orders barrier initialisation before any remote arrive, and every
// remote access before either CTA exits.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];"
        ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(void *dst, const CUtensorMap *map, uint32_t bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
        : "memory");
}
__device__ __forceinline__ void tma_load_im2col_4d_pair(void *dst, const CUtensorMap *map, uint32_t bar, int c, int w,
                                                        int h, int n, uint16_t off_w, uint16_t off_h) {
    asm volatile(
        "cp.async.bulk.tensor.4d.im2col.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2], {%7, %8};"
        ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c), "r"(w), "r"(h), "r"(n),
        "h"(off_w), "h"(off_h)
        : "memory");
}

// Plain bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned) from global to
// this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Warm the TMA unit's descriptor cache with a tensor map (kernel-parameter copies included).
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y, int z, int w) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2];"
        ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
        : "memory");
}

__device__ __forceinline__ void tma_store_4d(const CUtensorMap *map, const void *src, int x, int y, int z, int w) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(src)), "r"(x), "r"(y), "r"(z), "r"(w)
                 : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(src)), "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void tma_store_commit_and_wait() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

__device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Every committed store of this thread has finished reading shared memory.
__device__ __forceinline__ void tma_store_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Every committed store group but the most recent one has read its shared memory.
__device__ __forceinline__ void tma_store_wait_read_but_one() {
    asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

// Epilogue warps: two per TMEM lane quadrant, each taking half of the tile's columns.
constexpr int EPI_THREADS = 256;
// A TMA instruction holds its issuing thread for ~350 cycles (measured, any box size), so A and
// B of a K block are issued by different warps: warp 0 (A), warp 10 (B, one 3-D box of both
// planes).
constexpr int B_WARP = 2 + EPI_THREADS / 32;
constexpr int THREADS = 64 + EPI_THREADS + 32;  // A producer, MMA, eight epilogue warps, B producer

// Barrier among the epilogue threads only (named barrier 1).
__device__ __forceinline__ void epilogue_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)),
                 "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

// Pair forms: warp 1 of both CTAs allocates (and frees) the same columns in each CTA's TMEM.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *slot, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)),
                 "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand in 128B-swizzled rows of 128 bytes, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu)      // start address
           | ((uint64_t)1 << 16)                    // leading byte offset (unused for swizzled K-major)
           | ((uint64_t)(1024 >> 4) << 32)          // stride byte offset: 8 rows x 128 B
           | ((uint64_t)1 << 46)                    // descriptor version (sm_100)
           | ((uint64_t)2 << 61);                   // 128-byte swizzle
}

// K-major operand without swizzle, in core matrices of 8 rows x 16 bytes (rows 16 bytes apart):
// `lbo` bytes between core matrices adjacent in K, `sbo` bytes between those adjacent in M / N.
__device__ __forceinline__ uint64_t plain_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu)
           | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16)
           | ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32)
           | ((uint64_t)1 << 46);                   // descriptor version (sm_100); layout 0: no swizzle
}

// Tap-packed A tile (narrow-channel convolutions): the K block's 32 fp32 columns are eight
// 16-byte column groups, each an im2col box of 128 output pixels x 4 channels at one filter tap,
// stored box after box (128 rows x 16 bytes = 2 KB each). Core matrices: 128 bytes apart along M,
// 2 KB apart along K.
constexpr uint32_t PACKED_BOX_BYTES = BM * 16;

// kind::tf32, fp32 accumulate, both operands K-major; M = 128 (one CTA) or 256 (a CTA pair).
__host__ __device__ constexpr uint32_t instr_desc_tf32(int n, int m = BM) {
    return (1u << 4)                 // D format f32
           | (2u << 7)               // A format tf32
           | (2u << 10)              // B format tf32
           | ((uint32_t)(n >> 3) << 17)
           | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// Pair MMA (issued by rank 0): A rows 0-127 from rank 0's shared memory and 128-255 from rank 1's,
// B rows [0, N/2) from rank 0 and [N/2, N) from rank 1; D rows land in each CTA's own TMEM.
__device__ __forceinline__ void mma_tf32_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` (same offset) in both CTAs of the pair once the pair MMAs issued so far complete.
__device__ __forceinline__ void mma_commit_pair(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
                 ::"r"(smem_addr(bar)), "h"((uint16_t)3)
                 : "memory");
}

__device__ __forceinline__ void mma_commit_pair_local(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// A K block's four MMAs (K = 8 each) issued back to back from one asm block, with the test of
// the next stage's barrier between the first and the second. tcgen05.mma holds the issuing
// thread until the tensor pipe takes it, so any instruction between two MMAs adds to the
// block's time; every descriptor is computed before the first. first_acc: whether the first
// MMA accumulates. Returns the barrier test.
#define MGC_MMA4_BODY(GROUP, A0, A1, A2, A3, B0, B1, B2, B3, EXTRA)                                       \
    "{\n\t.reg .pred p, t, q;\n\t"                                                                      \
    "setp.ne.b32 p, %12, 0;\n\t"                                                                         \
    "setp.eq.b32 t, %12, %12;\n\t"                                                                       \
    "tcgen05.mma.cta_group::" GROUP ".kind::tf32 [%1], " A0 ", " B0 ", %11, p;\n\t"                      \
    "mbarrier.test_wait.parity.shared::cta.b64 q, [%13], %14;\n\t"                                      \
    EXTRA                                                                                                 \
    "tcgen05.mma.cta_group::" GROUP ".kind::tf32 [%1], " A1 ", " B1 ", %11, t;\n\t"                      \
    "tcgen05.mma.cta_group::" GROUP ".kind::tf32 [%1], " A2 ", " B2 ", %11, t;\n\t"                      \
    "tcgen05.mma.cta_group::" GROUP ".kind::tf32 [%1], " A3 ", " B3 ", %11, t;\n\t"                      \
    "selp.u32 %0, 1, 0, q;\n\t}\n"

template <int PAIR>
__device__ __forceinline__ bool mma_block4(uint32_t d, const uint64_t (&ad)[4], const uint64_t (&bd)[4], uint32_t idesc,
                                           uint32_t first_acc, uint64_t *next_bar, uint32_t next_parity) {
    uint32_t ready;
    if (PAIR)
        asm volatile(MGC_MMA4_BODY("2", "%2", "%3", "%4", "%5", "%6", "%7", "%8", "%9", "")
                     : "=r"(ready)
                     : "r"(d), "l"(ad[0]), "l"(ad[1]), "l"(ad[2]), "l"(ad[3]), "l"(bd[0]), "l"(bd[1]), "l"(bd[2]),
                       "l"(bd[3]), "r"(0), "r"(idesc), "r"(first_acc), "r"(smem_addr(next_bar)), "r"(next_parity)
                     : "memory");
    else
        asm volatile(MGC_MMA4_BODY("1", "%2", "%3", "%4", "%5", "%6", "%7", "%8", "%9", "")
                     : "=r"(ready)
                     : "r"(d), "l"(ad[0]), "l"(ad[1]), "l"(ad[2]), "l"(ad[3]), "l"(bd[0]), "l"(bd[1]), "l"(bd[2]),
                       "l"(bd[3]), "r"(0), "r"(idesc), "r"(first_acc), "r"(smem_addr(next_bar)), "r"(next_parity)
                     : "memory");
    return ready != 0;
}

// Wide pair: per K step the B_hi and the B_lo MMA into one accumulator (eight MMAs).
__device__ __forceinline__ bool mma_block4_wide(uint32_t d, const uint64_t (&ad)[4], const uint64_t (&bd)[4],
                                                const uint64_t (&bld)[4], uint32_t idesc, uint32_t first_acc,
                                                uint64_t *next_bar, uint32_t next_parity) {
    uint32_t ready;
    asm volatile(
        "{\n\t.reg .pred p, t, q;\n\t"
        "setp.ne.b32 p, %15, 0;\n\t"
        "setp.eq.b32 t, %15, %15;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%1], %2, %6, %14, p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 q, [%16], %17;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%1], %2, %10, %14, t;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%1], %3, %7, %14, t;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%1], %3, %11, %14, t;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%1], %4, %8, %14, t;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%1], %4, %12, %14, t;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%1], %5, %9, %14, t;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%1], %5, %13, %14, t;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}\n"
        : "=r"(ready)
        : "r"(d), "l"(ad[0]), "l"(ad[1]), "l"(ad[2]), "l"(ad[3]), "l"(bd[0]), "l"(bd[1]), "l"(bd[2]), "l"(bd[3]),
          "l"(bld[0]), "l"(bld[1]), "l"(bld[2]), "l"(bld[3]), "r"(idesc), "r"(first_acc), "r"(smem_addr(next_bar)),
          "r"(next_parity)
        : "memory");
    return ready != 0;
}

// 16 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ float4 lds4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}

__device__ __forceinline__ void sts4(uint32_t addr, float4 v) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ long long ceil_div_dev(long long a, long long b) { return (a + b - 1) / b; }

__device__ __forceinline__ void set_error(int *err, int code) {
    if (err) atomicExch(err, code);
}

// Round fp32 to the nearest TF32 value (10 explicit mantissa bits; ties away from zero), the
// rounding a TFLOAT32 tensor map applies on load.
__device__ __forceinline__ float tf32_hi(float x) {
    uint32_t b = __float_as_uint(x);
    uint32_t r = (b + 0x1000u) & 0xFFFFE000u;
    return ((b & 0x7F800000u) == 0x7F800000u) ? x : __uint_as_float(r);
}

// 32 consecutive fp32 columns of this thread's TMEM lane (no wait).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

// Position in a ring of N slots (shared-memory stages, TMEM buffers): the slot, the parity of
// the current lap, and whether the ring has wrapped (a slot's previous use must then be waited
// out). Advanced incrementally: no 64-bit division in the issue loops.
template <int N>
struct RingPos {
    int slot = 0;
    uint32_t phase = 0;
    bool wrapped = false;
    __device__ __forceinline__ void advance() {
        if (++slot == N) {
            slot = 0;
            phase ^= 1u;
            wrapped = true;
        }
    }
    __device__ __forceinline__ RingPos next() const {
        RingPos r = *this;
        r.advance();
        return r;
    }
};

constexpr uint32_t SMEM_LIMIT = 232448;  // dynamic shared memory per block on sm_100 (227 KB)

// RB: B-resident variant. The CTA keeps one N tile for its whole life and loads that tile's B
// panel (every K block, hi and lo) into shared memory once; the stages then carry A only.
// PAIR: CTA-pair variant (TF32 mode): 256-row tiles, each CTA holding one plane of B.
// WIDE (a pair with BN = 256): 256 x 256 tiles; each CTA holds both planes of its 128 B rows and
// the hi and lo products go to one accumulator through two N = 256 MMAs per K step. SP (wide
// pairs, or one-CTA TF32 tiles): the weights in one TF32 plane (B_hi, B rounded to the nearest
// TF32), one N = BN MMA per K step into one accumulator.
// SR (one CTA per tile, TF32, with a residual): the residual moves through its own staging
// buffer, so the next pass's residual loads while this pass's output is stored; SR = 2 runs the
// epilogue in passes of 64 columns, so that both buffers take the shared memory of one.
// PH: phase-split row tiles (im2col 5): a stage holds one tile's KH packed input rows (both
// phases each), brought in by one bulk copy; B stays resident as one TF32 plane (N = BN MMAs,
// one accumulator). Tile rows past OW read past the end of a packed row (into the next row, or
// the stage's slack): they are never stored.
constexpr uint32_t PHASE_STAGE_BYTES = 26624;  // 7 packed rows of 3,712 bytes plus slack (1024-aligned)
constexpr int POOL_PER_THREAD = 4;             // pooled bands: pooled columns per epilogue thread (PW <= 64)
template <int BN, int MODE, int RB = 0, int PAIR = 0, int SR = 0, int PH = 0, int SP = 0>
struct Cfg {
    static_assert(!SR || (!PAIR && MODE == TF32), "a separate residual buffer is a one-CTA TF32 form");
    static_assert(!PH || (!PAIR && !SR && RB && MODE == TF32 && BN == 64),
                  "phase-split tiles: one CTA, TF32, N tile 64, B resident");
    static_assert(!PAIR || MODE == TF32, "CTA pairs run TF32 mode only");
    // wide layout: each CTA of the pair holds the B rows of its half of the N tile (N tiles of
    // 192 and 256; with one weight plane, also 128)
    static constexpr bool WIDE = PAIR && (BN > 128 || SP);
    static_assert(!SP || WIDE || (!PAIR && !PH && MODE == TF32), "one weight plane: wide pairs or one-CTA TF32");
    static_assert(BN <= 128 || (WIDE && RB == 0 && BN % 64 == 0 && BN <= 256),
                  "N tiles of 192 and 256 are pair-only, without B residency");
    static_assert(MODE != DYN || (!PAIR && !RB && !SR), "dynamic-B GEMMs run one CTA per tile");
    static constexpr bool ONEACC = WIDE || MODE == DYN || PH || SP;  // one accumulator (no B_lo columns)
    static constexpr int REGIONS = MODE == STRICT ? 4 : 1;  // TMEM regions per K block
    static constexpr int BROWS = WIDE ? BN / 2 : BN;         // B rows of one plane in this CTA
    static constexpr uint32_t B_TILE_BYTES = BROWS * BK * 4;
    static constexpr int B_PLANES = (PAIR && !WIDE) || MODE == DYN || PH || SP ? 1 : 2;  // B planes in this CTA's smem
    static constexpr int TM = PAIR ? 2 * BM : BM;            // rows of one tile
    static constexpr int EN = WIDE || SR == 2 ? 64 : BN;     // columns of one epilogue pass
    static constexpr int NH = BN / EN;                       // epilogue passes per tile
    // stage: A (| A_lo) (| B_hi | B_lo), or A | this rank's B plane
    static constexpr uint32_t A_BYTES = PH ? PHASE_STAGE_BYTES : A_TILE_BYTES;
    static constexpr uint32_t STAGE_BYTES =
        A_BYTES + (MODE == STRICT ? A_TILE_BYTES : 0) + (RB ? 0 : B_PLANES * B_TILE_BYTES);
    // output staging of one epilogue pass: EN/32 slabs of [128 rows][32 fp32] in the
    // 128B-swizzled TMA layout
    static constexpr uint32_t OUT_BYTES = BM * EN * 4;
    static constexpr uint32_t BAR_BYTES = 512;                     // mbarriers and the TMEM address
    // everything else: output staging, alignment slack, barriers, the tile's bias
    static constexpr uint32_t RES_BYTES = SR ? OUT_BYTES : 0;       // the residual's own staging
    static constexpr uint32_t STAGE_BUDGET = SMEM_LIMIT - OUT_BYTES - RES_BYTES - 1024 - BAR_BYTES - BN * 4;
    static constexpr int MAX_STAGES = 8;
    static constexpr int STAGES = PH ? 3
                                  : RB ? (MODE == STRICT || SR ? 2 : 4)
                                  : (STAGE_BUDGET / STAGE_BYTES) < 2 ? 2
                                  : (int)(STAGE_BUDGET / STAGE_BYTES) > MAX_STAGES ? MAX_STAGES
                                  : (STAGE_BUDGET / STAGE_BYTES);
    // TMEM columns of one buffer: strict, four step regions of BN; TF32, the products with B_hi
    // (columns [0, BN)) and with B_lo ([BN, 2 BN)) from one N = 2 BN MMA per K step; wide, one
    // accumulator of BN columns
    static constexpr uint32_t BUF_COLS = MODE == STRICT ? REGIONS * BN : ONEACC ? BN : 2 * BN;
    static constexpr int TBUFS = (512 / BUF_COLS) > 4 ? 4 : (512 / BUF_COLS);  // TMEM buffers in the ring
    static constexpr uint32_t TMEM_COLS = TBUFS * BUF_COLS;
    // columns allocated: a power of two (two buffers of 192 take 512)
    static constexpr uint32_t TMEM_ALLOC = TMEM_COLS <= 32 ? 32 : TMEM_COLS <= 64 ? 64 : TMEM_COLS <= 128 ? 128
                                           : TMEM_COLS <= 256 ? 256 : 512;
    // fixed part; a B-resident launch adds its B panel (b_res_bytes) in front of the stages
    static constexpr uint32_t SMEM_BYTES =
        STAGES * STAGE_BYTES + OUT_BYTES + RES_BYTES + 1024 /*align*/ + BAR_BYTES + BN * 4 /*bias*/;
    static constexpr uint32_t B_RES_MAX = RB ? SMEM_LIMIT - SMEM_BYTES : 0;
    static_assert((3 * STAGES + 2 * TBUFS + 3) * 8 + 4 <= BAR_BYTES, "barrier area");
    static_assert(TMEM_COLS <= 512, "TMEM columns");
    static_assert(TBUFS >= 2, "need at least two TMEM buffers");
};

// Persistent. Default order: CTA b processes tiles b, b + gridDim.x, ... (N tile fastest, so the
// CTAs running together share A tiles in L2). B-resident order: CTA b keeps N tile b % n_tiles
// and walks the M tiles b / n_tiles, + gridDim.x / n_tiles, ... The shared-memory stage ring and
// the TMEM buffer ring run on a K-block counter that continues across tiles, so the next tile's
// loads and MMAs overlap this tile's drain and epilogue.
template <int BN, int MODE, int RB, int PAIR, int SR, int PH, int SP = 0>
__global__ void __launch_bounds__(THREADS, 1) umma_gemm_kernel(const __grid_constant__ Params p) {
    using C = Cfg<BN, MODE, RB, PAIR, SR, PH, SP>;
    constexpr int S = C::STAGES;
    constexpr int R = C::REGIONS;
    constexpr int TB = C::TBUFS;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // [B panel (B-resident only)] [stages] [output staging] [barriers] [bias]
    uint8_t *b_panel = smem;
    uint8_t *stages = smem + (RB ? p.b_res_bytes : 0u);
    auto a_tile = [&](int s) { return stages + (size_t)s * C::STAGE_BYTES; };
    auto alo_tile = [&](int s) { return stages + (size_t)s * C::STAGE_BYTES + C::A_BYTES; };
    // B_hi of K block kb (B_lo follows it directly: the stacked [B_hi; B_lo] operand)
    auto b_tile = [&](int s, int kb) {
        return RB ? b_panel + (size_t)kb * C::B_PLANES * C::B_TILE_BYTES
                  : stages + (size_t)s * C::STAGE_BYTES + C::A_BYTES + (MODE == STRICT ? A_TILE_BYTES : 0);
    };
    uint8_t *out_tile = stages + (size_t)S * C::STAGE_BYTES;  // 1024-aligned
    uint8_t *res_tile = SR ? out_tile + C::OUT_BYTES : out_tile;  // where a residual pass lands
    uint64_t *full = reinterpret_cast<uint64_t *>(out_tile + C::OUT_BYTES + C::RES_BYTES);
    uint64_t *empty = full + S;
    uint64_t *split = empty + S;
    uint64_t *tfull = split + S;       // [TB] a K block's products are in TMEM buffer b
    uint64_t *tempty = tfull + TB;     // [TB] the epilogue has drained TMEM buffer b
    uint64_t *mma_done = tempty + TB;  // every issued MMA has completed
    uint64_t *res_full = mma_done + 1; // a tile's residual has landed in the staging tile
    uint64_t *bres_full = res_full + 1; // the B panel has landed (B-resident)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bres_full + 1);
    float *bias_s = reinterpret_cast<float *>(out_tile + C::OUT_BYTES + C::RES_BYTES + C::BAR_BYTES);  // [BN] bias
    // the second staging tile (p.out2): the next 1024-byte boundary after the bias
    uint8_t *out_tile2 = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(bias_s + BN) + 1023) & ~uintptr_t(1023));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_kb = p.num_kb;
    const int total_tiles = p.n_tiles * p.m_tiles;
    // pairs: this CTA's rank (0 issues the MMAs) and the pair as the unit of the tile walk
    const uint32_t rank = PAIR ? cluster_rank() : 0u;
    const int unit = PAIR ? (int)cluster_index() : (int)blockIdx.x;
    const int units = PAIR ? (int)cluster_count() : (int)gridDim.x;
    const int row0 = (int)rank * BM;  // this CTA's first row within a tile
    // DYN: M tile mt of the flattened batch -> first row within its batch and the two batch
    // coordinates of the 4-D tensor maps
    auto dyn_rows = [&](int mt, int &m0, int &b1, int &b2) {
        const int bt = mt / p.m_per_batch;
        m0 = (mt - bt * p.m_per_batch) * BM;
        b2 = bt / p.nbatch1;
        b1 = bt - b2 * p.nbatch1;
    };
    // split K: the work units are (tile, split) pairs; K blocks [kb_lo(ks), kb_hi(ks)) per unit
    const int splits = p.splits > 1 ? p.splits : 1;
    const int kb_per = splits > 1 ? p.kb_per : num_kb;
    auto kb_lo = [&](int ks) { return ks * kb_per; };
    auto kb_hi = [&](int ks) { return (ks + 1) * kb_per < num_kb ? (ks + 1) * kb_per : num_kb; };
    // the i-th work unit of this CTA (or pair) as (M tile, N tile, split); false past the last
    auto unit_at = [&](int i, int &mt, int &nt, int &ks) -> bool {
        ks = 0;
        if (PH && p.pool_bp > 0) {  // pooled bands: mt is the band
            const int band = unit + (i / (2 * p.pool_bp + 1)) * units;
            nt = 0;
            mt = band;
            return band < p.pool_nbands;
        }
        if (RB) {
            const int per = units / p.n_tiles;
            nt = unit % p.n_tiles;
            mt = unit / p.n_tiles + i * per;
            return unit < per * p.n_tiles && mt < p.m_tiles;
        }
        const int t = unit + i * units;
        const int tt = splits > 1 ? t / splits : t;
        if (splits > 1) ks = t - tt * splits;
        nt = tt % p.n_tiles;
        mt = tt / p.n_tiles;
        return tt < total_tiles;
    };
    auto tile_at = [&](int i, int &mt, int &nt) -> bool {
        int ks;
        return unit_at(i, mt, nt, ks);
    };
    // pooled bands: tile i's image and output row (-1: the dummy row above the image), and
    // whether it is its band's first
    auto pool_row = [&](int i, int &img, int &oh, bool &first) {
        const int rows = 2 * p.pool_bp + 1;
        const int bj = i / rows, r = i - bj * rows;
        const int band = unit + bj * units;
        img = band / p.pool_nbp;
        oh = 2 * (band - img * p.pool_nbp) * p.pool_bp - 1 + r;
        first = r == 0;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            mbar_init(&split[s], EPI_THREADS);
        }
        for (int b = 0; b < TB; ++b) {
            mbar_init(&tfull[b], 1);
            // pairs: one arrival per epilogue warp of both CTAs, on rank 0's barrier
            mbar_init(&tempty[b], PAIR ? 2 * (EPI_THREADS / 32) : EPI_THREADS);
        }
        mbar_init(mma_done, 1);
        mbar_init(res_full, 1);
        mbar_init(bres_full, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        if (PAIR) tmem_alloc_pair(tmem_slot, C::TMEM_ALLOC);
        else tmem_alloc(tmem_slot, C::TMEM_ALLOC);
    }
    tc_fence_before();
    __syncthreads();
    if (PAIR) cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (PH && warp == 0) {
        // ---------------- producer, phase-split row tiles (lane 0) ----------------
        // A tile's KH packed input rows are consecutive in memory: one bulk copy per tile, into
        // a stage that holds them all (a copy holds its issuing thread for hundreds of cycles,
        // so one per K block would starve the MMAs of a 7-block tile).
        if (lane == 0) {
            long long g = 0;  // tiles issued
            RingPos<S> pos;   // stage of tile g
            int mt, nt;
            if (tile_at(0, mt, nt)) {  // the B panel, once
                mbar_expect_tx(bres_full, p.b_res_bytes);
                for (int kb = 0; kb < num_kb; ++kb) tma_load_3d(b_tile(0, kb), &p.tmB, bres_full, kb * BK, nt * BN, 0);
            }
            const uint32_t bytes = (uint32_t)num_kb * p.a_bytes;
            // the B-resident walk: M tiles unit, unit + units, ... (one N tile); (image, output
            // row) advanced without divisions
            const int step = units, img_step = step / p.rt_per_img, oh_step = step - img_step * p.rt_per_img;
            int img = unit / p.rt_per_img, oh = unit - img * p.rt_per_img;
            for (int i = 0; tile_at(i, mt, nt); ++i, ++g, pos.advance()) {
                const int s = pos.slot;
                if (pos.wrapped && !mbar_wait(&empty[s], pos.phase ^ 1u)) {
                    set_error(p.err, MGC_CUDA_TIMEOUT);
                    break;
                }
                if (p.pool_bp > 0) {  // pooled bands (the dummy row loads row 0; never stored)
                    bool first;
                    pool_row(i, img, oh, first);
                    if (oh < 0) oh = 0;
                } else if (i > 0) {
                    img += img_step;
                    oh += oh_step;
                    if (oh >= p.rt_per_img) {
                        oh -= p.rt_per_img;
                        ++img;
                    }
                }
                mbar_expect_tx(&full[s], bytes);
                bulk_load(a_tile(s), p.a_rows + ((long long)img * p.prows + (long long)oh * p.SH) * p.prow_bytes, bytes,
                          &full[s]);
            }
            // the copies of the last (up to S) issued tiles must have landed before exit
            for (long long k = g - 1; k >= 0 && k >= g - S; --k) {
                if (!mbar_wait(&full[k % S], (uint32_t)((k / S) & 1))) set_error(p.err, MGC_CUDA_TIMEOUT);
            }
            if (tile_at(0, mt, nt) && !mbar_wait(bres_full, 0)) set_error(p.err, MGC_CUDA_TIMEOUT);
        }
    } else if (warp == 0 && !PAIR && p.im2col >= 2) {
        // ---------------- TMA producer, narrow-channel forms (the whole warp) ----------------
        // A TMA instruction holds its issuing thread for a few hundred cycles. These forms need
        // eight or more A boxes per K block, so lane j issues box j, all in one instruction.
        // Lane 0 alone waits on the ring, arms the barrier and loads B; the warp reconverges
        // before the loads.
        const uint32_t bytes = p.a_bytes + (RB ? 0 : 2 * C::B_TILE_BYTES);
        long long g = 0;  // K blocks issued so far
        RingPos<S> pos;   // stage of K block g
        bool ok = true;
        int mt, nt;
        if (RB && tile_at(0, mt, nt)) {  // this CTA's B panel, once: lane j loads K blocks j, j+32, ...
            if (lane == 0) mbar_expect_tx(bres_full, p.b_res_bytes);
            __syncwarp();
            for (int kb = lane; kb < num_kb; kb += 32) tma_load_3d(b_tile(0, kb), &p.tmB, bres_full, kb * BK, nt * BN, 0);
        }
        for (int i = 0; ok && tile_at(i, mt, nt); ++i) {
            const int n0 = nt * BN, m0 = mt * BM;
            const int hw = p.OH * p.OW;
            const int nb = m0 / hw;
            const int rem0 = m0 - nb * hw;
            const int oh0 = rem0 / p.OW, ow0 = rem0 - oh0 * p.OW;
            const int wb = ow0 * p.SW - p.PL, hb = oh0 * p.SH - p.PT;
            // row tiles: the tile's image and first output row; window rows / row tiles: the K
            // block's filter row kh and first column x0, advanced per block (no division)
            const int rimg = p.im2col >= 4 ? mt / p.rt_per_img : 0;
            const int roh0 = p.im2col >= 4 ? (mt - rimg * p.rt_per_img) * p.rt_rows : 0;
            int kh_w = 0, cb_w = 0;
            for (int kb = 0; kb < num_kb; ++kb, ++g, pos.advance()) {
                const int s = pos.slot;
                const int kh = kh_w, x0 = cb_w * BK;
                if (++cb_w == p.cblocks) {
                    cb_w = 0;
                    ++kh_w;
                }
                int waited = 1;
                if (lane == 0) {
                    if (pos.wrapped && !mbar_wait(&empty[s], pos.phase ^ 1u)) waited = 0;
                    else mbar_expect_tx(&full[s], bytes);
                }
                if (!__shfl_sync(0xffffffffu, waited, 0)) {
                    if (lane == 0) set_error(p.err, MGC_CUDA_TIMEOUT);
                    ok = false;
                    break;
                }
                if (p.im2col == 5) {
                    // phase-split row tiles: the K block is filter row kh; both column phases of
                    // the packed input row it reads, one contiguous bulk copy
                    if (lane == 0)
                        bulk_load(a_tile(s), p.a_rows + ((long long)rimg * p.prows + roh0 * p.SH + kh * p.DH) * p.prow_bytes,
                                  p.a_bytes, &full[s]);
                } else if (p.im2col == 4) {
                    // row tiles: one box of rt_rows whole output rows (OW pixels each) of one
                    // image; the tile's remaining smem rows are never loaded and never stored
                    if (lane == 0) tma_load_5d(a_tile(s), &p.tmA, &full[s], x0, 0, roh0, rimg, kh);
                } else if (p.im2col == 3) {
                    // window rows: the K block is 32 consecutive floats of the padded image row
                    // (kh) starting at the window origin, for wrows output pixels per box
                    for (int r0 = lane * p.wrows; r0 < BM; r0 += 32 * p.wrows) {
                        const int m = m0 + r0;
                        const int img = m / hw, rem = m - img * hw;
                        const int oh = rem / p.OW, ow = rem - oh * p.OW;
                        tma_load_5d(a_tile(s) + r0 * 128, &p.tmA, &full[s], x0, ow, oh, img, kh);
                    }
                } else if (lane < BK / 4) {
                    // tap-packed: eight 4-channel boxes; K column k = tap * cpix + channel.
                    // Columns past the real K reload tap 0 (their weights are zero)
                    const int k0 = kb * BK + lane * 4;
                    const int tap = k0 < p.kreal ? k0 / p.cpix : 0;
                    const int ch = k0 < p.kreal ? k0 - tap * p.cpix : 0;
                    const int kw = tap % p.KW, kh = tap / p.KW;
                    tma_load_im2col_4d(a_tile(s) + lane * PACKED_BOX_BYTES, &p.tmA, &full[s], ch, wb, hb, nb,
                                       (uint16_t)(kw * p.DW), (uint16_t)(kh * p.DH));
                }
                (void)n0;  // B comes from the B producer warp
                __syncwarp();
            }
        }
        // the copies of the last (up to S) issued K blocks must have landed before exit
        if (lane == 0) {
            for (long long k = g - 1; k >= 0 && k >= g - S; --k) {
                if (!mbar_wait(&full[k % S], (uint32_t)((k / S) & 1))) set_error(p.err, MGC_CUDA_TIMEOUT);
            }
            if (RB && tile_at(0, mt, nt) && !mbar_wait(bres_full, 0)) set_error(p.err, MGC_CUDA_TIMEOUT);
        }
    } else if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer: one A box per K block (lane 0) ----------------
            // a pair's stage barrier (rank 0's) counts the bytes of both CTAs
            constexpr uint32_t bytes = (PAIR ? 2 : 1) * (A_TILE_BYTES + (RB ? 0 : C::B_PLANES * C::B_TILE_BYTES));
            const bool arms = !PAIR || rank == 0;  // this thread arms the stage barriers
            long long g = 0;  // K blocks issued so far
            RingPos<S> pos;   // stage of K block g
            bool ok = true;
            bool free_next = false;  // the slot of K block g was tested free
            int mt, nt;
            if (RB && tile_at(0, mt, nt)) {  // this CTA's B panel (its plane, for a pair), once
                if (arms) mbar_expect_tx(bres_full, PAIR ? 2 * p.b_res_bytes : p.b_res_bytes);
#pragma unroll 1
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (PAIR) tma_load_3d_pair(b_tile(0, kb), &p.tmB, leader_addr(bres_full), kb * BK, nt * BN, (int)rank);
                    else tma_load_3d(b_tile(0, kb), &p.tmB, bres_full, kb * BK, nt * BN, 0);
                }
            }
            int ks;
            for (int i = 0; ok && unit_at(i, mt, nt, ks); ++i) {
                const int n0 = nt * BN;
                int m0 = mt * C::TM + row0, db1 = 0, db2 = 0;
                if (MODE == DYN) dyn_rows(mt, m0, db1, db2);
                const int klo = kb_lo(ks), khi = kb_hi(ks);
                int wb = 0, hb = 0, nb = 0;
                if (p.im2col) {
                    const int hw = p.OH * p.OW;
                    nb = m0 / hw;
                    const int rem = m0 - nb * hw;
                    const int oh = rem / p.OW, ow = rem - oh * p.OW;
                    wb = ow * p.SW - p.PL;
                    hb = oh * p.SH - p.PT;
                }
                // im2col: K block kb -> (filter row kh, column kw, channel block cb), advanced
                // per block; the tap offsets are kept as the box's 16-bit offsets
                int cb = 0, kw = 0;
                uint16_t off_w = 0, off_h = 0;
                if (p.im2col && klo > 0) {  // a split's first K block (one division per unit)
                    const int tap = klo / p.cblocks, kh = tap / p.KW;
                    cb = klo - tap * p.cblocks;
                    kw = tap - kh * p.KW;
                    off_w = (uint16_t)(kw * p.DW);
                    off_h = (uint16_t)(kh * p.DH);
                }
                for (int kb = klo; kb < khi; ++kb, ++g, pos.advance()) {
                    const int s = pos.slot;
                    if (pos.wrapped && !free_next && !mbar_wait(&empty[s], pos.phase ^ 1u)) {
                        set_error(p.err, MGC_CUDA_TIMEOUT);
                        ok = false;
                        break;
                    }
                    // test the next K block's slot now; the test's latency overlaps this block's
                    // TMA issue, and a slot found free needs no wait
                    const RingPos<S> nx = pos.next();
                    free_next = !nx.wrapped || mbar_test_wait(&empty[nx.slot], nx.phase ^ 1u);
                    if (arms) mbar_expect_tx(&full[s], bytes);
                    if (p.im2col) {
                        if (PAIR)
                            tma_load_im2col_4d_pair(a_tile(s), &p.tmA, leader_addr(&full[s]), cb * BK, wb, hb, nb,
                                                    off_w, off_h);
                        else
                            tma_load_im2col_4d(a_tile(s), &p.tmA, &full[s], cb * BK, wb, hb, nb, off_w, off_h);
                        if (++cb == p.cblocks) {
                            cb = 0;
                            off_w = (uint16_t)(off_w + p.DW);
                            if (++kw == p.KW) {
                                kw = 0;
                                off_w = 0;
                                off_h = (uint16_t)(off_h + p.DH);
                            }
                        }
                    } else if (PAIR) {
                        tma_load_2d_pair(a_tile(s), &p.tmA, leader_addr(&full[s]), kb * BK, m0);
                    } else if (MODE == DYN) {
                        tma_load_4d(a_tile(s), &p.tmA, &full[s], kb * BK, m0, db1, db2);
                    } else {
                        tma_load_2d(a_tile(s), &p.tmA, &full[s], kb * BK, m0);
                    }
                    (void)n0;  // B comes from the B producer warp
                }
            }
            // the copies of the last (up to S) issued K blocks must have landed before exit (a
            // pair's rank 0 waits for both CTAs' copies; rank 1 leaves after the closing cluster
            // barrier, which rank 0 reaches only after these waits)
            if (arms) {
                for (long long k = g - 1; k >= 0 && k >= g - S; --k) {
                    if (!mbar_wait(&full[k % S], (uint32_t)((k / S) & 1))) set_error(p.err, MGC_CUDA_TIMEOUT);
                }
                if (RB && tile_at(0, mt, nt) && !mbar_wait(bres_full, 0)) set_error(p.err, MGC_CUDA_TIMEOUT);
            }
        }
    } else if (warp == B_WARP) {
        if (lane == 0 && !RB) {
            // ---------------- B producer: one 3-D box (TF32 part and residual) per K block ----------------
            RingPos<S> pos;  // stage of the next K block
            bool ok = true;
            bool free_next = false;  // that stage was tested free
            int mt, nt, ks;
            for (int i = 0; ok && unit_at(i, mt, nt, ks); ++i) {
                int dm0 = 0, db1 = 0, db2 = 0;
                if (MODE == DYN) dyn_rows(mt, dm0, db1, db2);
                for (int kb = kb_lo(ks); kb < kb_hi(ks); ++kb, pos.advance()) {
                    const int s = pos.slot;
                    if (pos.wrapped && !free_next && !mbar_wait(&empty[s], pos.phase ^ 1u)) {
                        set_error(p.err, MGC_CUDA_TIMEOUT);
                        ok = false;
                        break;
                    }
                    const RingPos<S> nx = pos.next();
                    free_next = !nx.wrapped || mbar_test_wait(&empty[nx.slot], nx.phase ^ 1u);
                    // a pair: this rank's plane, or (wide) both planes of this rank's 128 rows;
                    // DYN: the batch's B rows
                    if (MODE == DYN)
                        tma_load_4d(b_tile(s, kb), &p.tmB, &full[s], kb * BK, nt * BN, db1, db2);
                    else if (C::WIDE)
                        tma_load_3d_pair(b_tile(s, kb), &p.tmB, leader_addr(&full[s]), kb * BK,
                                         nt * BN + (int)rank * C::BROWS, 0);
                    else if (PAIR)
                        tma_load_3d_pair(b_tile(s, kb), &p.tmB, leader_addr(&full[s]), kb * BK, nt * BN, (int)rank);
                    else
                        tma_load_3d(b_tile(s, kb), &p.tmB, &full[s], kb * BK, nt * BN, 0);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // ---------------- MMA issuer (a pair's rank 0 issues for both CTAs) ----------------
            if (PH) {
                // phase-split row tiles: one stage per tile, the KH filter rows of the tile in
                // it (K block kh: packed row kh; steps 0-1 the even-tap phase, 2-3 the odd-tap)
                constexpr uint32_t idesc_t = instr_desc_tf32(BN);  // one TF32 plane of B
                RingPos<S> pos;
                RingPos<TB> buf;
                bool ok = true;
                int mt, nt;
                if (tile_at(0, mt, nt) && !mbar_wait(bres_full, 0)) {  // the B panel (CTAs with tiles)
                    set_error(p.err, MGC_CUDA_TIMEOUT);
                    ok = false;
                }
                // this CTA's tiles (one N tile): unit, unit + units, ... below m_tiles; pooled,
                // the rows of its bands unit, unit + units, ...
                const int my_tiles = p.pool_bp > 0
                    ? (unit < p.pool_nbands ? ((p.pool_nbands - 1 - unit) / units + 1) * (2 * p.pool_bp + 1) : 0)
                    : unit < p.m_tiles ? (p.m_tiles - 1 - unit) / units + 1 : 0;
                for (int i = 0; ok && i < my_tiles; ++i, pos.advance()) {
                    const int s = pos.slot, b = buf.slot;
                    if (!mbar_wait(&full[s], pos.phase)) {
                        set_error(p.err, MGC_CUDA_TIMEOUT);
                        break;
                    }
                    if (buf.wrapped) {  // the epilogue has drained this TMEM buffer
                        if (!mbar_wait(&tempty[b], buf.phase ^ 1u)) {
                            set_error(p.err, MGC_CUDA_TIMEOUT);
                            break;
                        }
                        tc_fence_after();
                    }
                    const uint32_t dbase = tmem_base + (uint32_t)(b * C::BUF_COLS);
                    const uint32_t a0 = smem_addr(a_tile(s));
                    for (int kb = 0; kb < num_kb; ++kb) {
                        const uint32_t a_addr = a0 + (uint32_t)(kb * p.a_bytes), b_addr = smem_addr(b_tile(s, kb));
                        uint64_t ad[BK / 8], bd[BK / 8];
#pragma unroll
                        for (int k = 0; k < BK / 8; ++k) {
                            ad[k] = plain_desc(a_addr + (k < 2 ? 32 * k : p.phase_bytes + 32 * (k - 2)), 16, 128);
                            bd[k] = sw128_desc(b_addr + k * 32);
                        }
                        (void)mma_block4<0>(dbase, ad, bd, idesc_t, kb == 0 ? 0u : 1u, &full[s], pos.phase);
                    }
                    mma_commit(&empty[s]);
                    mma_commit(&tfull[b]);
                    buf.advance();
                }
                mma_commit(mma_done);
                if (!mbar_wait(mma_done, 0)) set_error(p.err, MGC_CUDA_TIMEOUT);
            } else {
            constexpr uint32_t idesc = instr_desc_tf32(BN);
            // the stacked [B_hi; B_lo] tile, or (wide, DYN) one plane of all BN columns
            constexpr uint32_t idesc2 = instr_desc_tf32(C::ONEACC ? BN : 2 * BN, C::TM);
            RingPos<S> pos;   // stage of the next K block
            RingPos<TB> buf;  // TMEM buffer of the next K-block group
            bool ok = true;
            int mt, nt;
            if (RB && tile_at(0, mt, nt) && !mbar_wait(bres_full, 0)) {
                set_error(p.err, MGC_CUDA_TIMEOUT);
                ok = false;
            }
            uint64_t *const ready = MODE == STRICT ? split : full;  // a stage's operands are in place
            // MMA issue blocks while the tensor pipe is busy, so a barrier test between two K
            // blocks would leave the pipe idle for its whole latency (~150 cycles). Instead the
            // next K block's stage is tested right after this block's first MMA is issued, and
            // a block whose stage tested complete skips its wait.
            bool have = false;
            int ks;
            for (int i = 0; ok && unit_at(i, mt, nt, ks); ++i) {
                const int klo = kb_lo(ks), khi = kb_hi(ks);
                for (int kb = klo; kb < khi; ++kb, pos.advance()) {
                    const int s = pos.slot;
                    const int b = buf.slot;
                    // a TMEM buffer per K block (strict) or per tile (TF32)
                    const bool first = MODE == STRICT || kb == klo, last = MODE == STRICT || kb == khi - 1;
                    if (!have && !mbar_wait(&ready[s], pos.phase)) {
                        set_error(p.err, MGC_CUDA_TIMEOUT);
                        ok = false;
                        break;
                    }
                    if (first && buf.wrapped) {
                        // the epilogue has drained this TMEM buffer; order the MMAs after its loads.
                        // (The stage's operands need no tcgen05 fence: the TMA writes and the MMA
                        // reads are both async-proxy accesses ordered by the stage barrier. A fence
                        // per K block would also cost ~600 cycles: it waits for the MMA pipe.)
                        if (!mbar_wait(&tempty[b], buf.phase ^ 1u)) {
                            set_error(p.err, MGC_CUDA_TIMEOUT);
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                    }
                    const uint32_t a_addr = smem_addr(a_tile(s)), b_addr = smem_addr(b_tile(s, kb));
                    const uint32_t bl_addr = b_addr + C::B_TILE_BYTES, al_addr = smem_addr(alo_tile(s));
                    const uint32_t dbase = tmem_base + (uint32_t)(b * C::BUF_COLS);
                    const RingPos<S> nx = pos.next();
                    uint64_t *const next_ready = &ready[nx.slot];
                    const uint32_t next_parity = nx.phase;
                    const bool packed = p.im2col == 2, phased = p.im2col == 5;
                    // the block's descriptors, all before the first MMA: 8 tf32 = 32 bytes per step
                    uint64_t ad[BK / 8], bd[BK / 8], bld[BK / 8];
#pragma unroll
                    for (int k = 0; k < BK / 8; ++k) {
                        // phase-split rows: output pixel m's four taps of one phase are pixels m..m+3
                        // of that phase's buffer, so row m of the operand starts 16 bytes after row
                        // m - 1 and the K-adjacent core matrix 16 bytes after this one; steps 0-1
                        // read the even-tap phase, steps 2-3 the odd-tap phase
                        ad[k] = phased ? plain_desc(a_addr + (k < 2 ? 32 * k : p.phase_bytes + 32 * (k - 2)), 16, 128)
                              : packed ? plain_desc(a_addr + k * 2 * PACKED_BOX_BYTES, PACKED_BOX_BYTES, 128)
                                       : sw128_desc(a_addr + k * 32);
                        bd[k] = sw128_desc(b_addr + k * 32);
                        bld[k] = sw128_desc(bl_addr + k * 32);
                    }
                    if (MODE == STRICT) {
                        bool peek = false;
#pragma unroll
                        for (int k = 0; k < BK / 8; ++k) {
                            const uint32_t d = dbase + (uint32_t)(k * BN);  // own region per K step
                            const uint64_t ald = packed ? plain_desc(al_addr + k * 2 * PACKED_BOX_BYTES, PACKED_BOX_BYTES, 128)
                                                        : sw128_desc(al_addr + k * 32);
                            mma_tf32(d, ald, bd[k], idesc, 0u);    // A_lo * B_hi (fresh region)
                            mma_tf32(d, ad[k], bld[k], idesc, 1u);  // A_hi * B_lo
                            mma_tf32(d, ad[k], bd[k], idesc, 1u);   // A_hi * B_hi
                            if (k == 0) peek = mbar_test_wait(next_ready, next_parity);
                        }
                        have = peek;
                    } else if (C::WIDE && !SP) {
                        // B_hi's and B_lo's products into one accumulator
                        have = mma_block4_wide(dbase, ad, bd, bld, idesc2, first ? 0u : 1u, next_ready, next_parity);
                    } else {
                        // B_lo's tile directly follows B_hi's in the stage with the same
                        // 128B-swizzled row layout, so one descriptor spans both as 2 BN rows: one
                        // MMA, A read once per K step (a pair: the same descriptor names B_hi in
                        // rank 0, B_lo in rank 1; SP: each rank's BN / 2 rows of the one plane)
                        have = mma_block4<PAIR>(dbase, ad, bd, idesc2, first ? 0u : 1u, next_ready, next_parity);
                    }
                    // shared-memory slot free once these MMAs read it (in both CTAs of a pair)
                    if (PAIR) mma_commit_pair(&empty[s]);
                    else mma_commit(&empty[s]);
                    if (last) {
                        // TMEM buffer b holds this group's products
                        if (PAIR) mma_commit_pair(&tfull[b]);
                        else mma_commit(&tfull[b]);
                        buf.advance();
                    }
                }
            }
            if (PAIR) mma_commit_pair_local(mma_done);
            else mma_commit(mma_done);
            if (!mbar_wait(mma_done, 0)) set_error(p.err, MGC_CUDA_TIMEOUT);
            }
        }
    } else {
        // ---------------- epilogue warps (2..9): A split (strict), TMEM drain, epilogue ----------------
        // A tile's epilogue runs in NH passes of EN columns (one pass unless wide); each pass
        // stages, stores and (with a residual) prefetches EN columns.
        constexpr int EN = C::EN, NH = C::NH;
        static_assert(EN <= EPI_THREADS, "one bias column per epilogue thread");
        constexpr int HALF = EN / 2;        // columns per epilogue thread and pass
        const int et = threadIdx.x - 64;    // 0..255
        const int q = warp & 3;             // TMEM lane quadrant this warp may access
        const int hc = ((warp - 2) >> 2) * HALF;  // first column of this warp's half
        const int row = q * 32 + lane;      // this thread's tile row (its TMEM lane)
        const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)hc;
        RingPos<TB> dpos;      // TMEM buffer to drain next
        RingPos<S> spos;       // stage to split next (strict)
        bool ok = true;
        // strict mode accumulates K blocks in fp64 (each block's four step regions summed in fp32
        // first); TF32 mode accumulates in fp32
        using AccT = typename std::conditional<MODE == STRICT, double, float>::type;
        AccT acc[HALF];
        // pooled bands: this thread's running maxima of the pooled row being built
        float4 pool_acc[PH ? POOL_PER_THREAD : 1];
        // hand TMEM buffer b back to the MMA warp (a pair: one arrival per warp, on rank 0's barrier)
        auto release = [&](int b) {
            tc_fence_before();
            if (PAIR) {
                __syncwarp();
                if (lane == 0) mbar_arrive_remote(leader_addr(&tempty[b]));
            } else {
                mbar_arrive(&tempty[b]);
            }
            dpos.advance();
        };
        // TF32: this thread's HALF accumulator columns of pass h of the tile in TMEM buffer
        // dpos (B_hi's and B_lo's products summed, or, wide, the one accumulator); the first
        // pass waits for the buffer, the last hands it back
        auto load_pass = [&](int h) -> bool {
            const int b = dpos.slot;
            if (h == 0) {
                if (!mbar_wait(&tfull[b], dpos.phase)) return false;
                tc_fence_after();
            }
#pragma unroll
            for (int c0 = 0; c0 < HALF; c0 += 32) {
                uint32_t vh[32], vl[32];
                const uint32_t addr = lane_base + (uint32_t)(b * C::BUF_COLS + h * EN + c0);
                tmem_ld32(addr, vh);
                if (!C::ONEACC) tmem_ld32(addr + BN, vl);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    acc[c0 + j] = C::ONEACC ? __uint_as_float(vh[j]) : __uint_as_float(vh[j]) + __uint_as_float(vl[j]);
            }
            if (h == NH - 1) release(b);
            return true;
        };
        // strict: add K block's four step regions into the fp64 accumulators
        auto drain = [&]() -> bool {
            const int b = dpos.slot;
            if (!mbar_wait(&tfull[b], dpos.phase)) return false;
            tc_fence_after();
            {
#pragma unroll
                for (int c0 = 0; c0 < HALF; c0 += 32) {
                    float blk[32];
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        uint32_t v[32];
                        tmem_ld32(lane_base + (uint32_t)(b * C::BUF_COLS + r * BN + c0), v);
                        tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 32; ++j) blk[j] = r == 0 ? __uint_as_float(v[j]) : blk[j] + __uint_as_float(v[j]);
                    }
#pragma unroll
                    for (int j = 0; j < 32; ++j) acc[c0 + j] += (double)blk[j];
                }
            }
            release(b);
            return true;
        };
        auto split_one = [&]() -> bool {
            const int s = spos.slot;
            if (!mbar_wait(&full[s], spos.phase)) return false;
            float4 *a4 = reinterpret_cast<float4 *>(a_tile(s));
            float4 *l4 = reinterpret_cast<float4 *>(alo_tile(s));
#pragma unroll
            for (int i = 0; i < (int)(A_TILE_BYTES / 16 / EPI_THREADS); ++i) {
                const int idx = i * EPI_THREADS + et;
                const float4 v = a4[idx];
                float4 h, l;
                h.x = tf32_hi(v.x); h.y = tf32_hi(v.y); h.z = tf32_hi(v.z); h.w = tf32_hi(v.w);
                l.x = v.x - h.x; l.y = v.y - h.y; l.z = v.z - h.z; l.w = v.w - h.w;
                a4[idx] = h;
                l4[idx] = l;
            }
            fence_proxy_async_smem();
            mbar_arrive(&split[s]);
            spos.advance();
            return true;
        };
        // byte offset of columns c0..c0+3 of row r in the staging tile: EN / 32 slabs of 128 rows
        // x 128 bytes, 16-byte chunks XOR-swizzled by the row (the TMA 128-byte swizzle)
        auto stage_offset = [](int r, int c0) -> uint32_t {
            const int sl = c0 >> 5, j = (c0 & 31) >> 2;
            return (uint32_t)(sl * (BM * 128) + r * 128 + ((j ^ (r & 7)) << 4));
        };
        // the staging tile of the current pass: with p.out2 the passes alternate between two, so
        // that a pass stages while the previous pass's TMA store still reads its tile
        uint8_t *stg = out_tile;
        auto stage_slot = [&](int r, int c0) { return reinterpret_cast<float4 *>(stg + stage_offset(r, c0)); };
        // Output path. Step 1 (unrolled over the accumulator registers, no calls): alpha * acc +
        // bias (+ the residual, TMA-prefetched into the staging tile) and a ReLU / Clip, into the
        // 128B-swizzled staging tile. Step 2 (compact, own row): GELU / tanh / sigmoid. Then one
        // thread TMA-stores the tile and prefetches the next tile's residual into it; without a
        // TMA-able C the warps store their rows with coalesced 128-byte writes instead.
        const bool direct = !p.tma_out;
        const bool res_tma = p.tma_res != 0;
        const bool res_direct = p.res != nullptr && !res_tma;
        const bool cheap = p.act == MGC_ACT_NONE || p.act == MGC_ACT_RELU || p.act == MGC_ACT_CLIP;
        const bool act_in_step1 = cheap && !res_direct;
        const bool issuer = warp == 2 && lane == 0;
        if (issuer && p.tma_out) prefetch_tmap(&p.tmC);
        if (issuer && p.tma_res) prefetch_tmap(&p.tmR);
        const bool rows = p.im2col >= 4;
        // the residual of pass h_ of tile (mt_, nt_) into its staging (the output staging tile,
        // or with SR its own)
        auto issue_residual = [&](int mt_, int nt_, int h_) {
            const int tn0 = nt_ * BN + h_ * EN, tm0 = mt_ * C::TM + row0;
            if (rows) {
                const int img = mt_ / p.rt_per_img, oh0 = (mt_ - img * p.rt_per_img) * p.rt_rows;
                mbar_expect_tx(res_full, (uint32_t)(EN / 32) * p.res_box_bytes);
#pragma unroll 1
                for (int sl = 0; sl < EN / 32; ++sl)
                    tma_load_4d(res_tile + sl * (BM * 128), &p.tmR, res_full, tn0 + sl * 32, 0, oh0, img);
                return;
            }
            mbar_expect_tx(res_full, C::OUT_BYTES);
#pragma unroll 1
            for (int sl = 0; sl < EN / 32; ++sl)
                tma_load_2d(res_tile + sl * (BM * 128), &p.tmR, res_full, tn0 + sl * 32, tm0);
        };
        int mt, nt, ks;
        if (res_tma && issuer && tile_at(0, mt, nt)) issue_residual(mt, nt, 0);
        int local = 0;  // epilogue passes this CTA has finished
        for (int i = 0; ok && unit_at(i, mt, nt, ks); ++i) {
          int m0 = mt * C::TM + row0, db1 = 0, db2 = 0;
          if (MODE == DYN) dyn_rows(mt, m0, db1, db2);
          if (MODE == STRICT) {
#pragma unroll
            for (int j = 0; j < HALF; ++j) acc[j] = AccT(0);
            // this unit's K blocks (all of them unless split K)
            const int klo = kb_lo(ks), khi = kb_hi(ks);
            for (int kb = klo; kb < khi && ok; ++kb) {
                if (!split_one()) ok = false;
                else if (kb > klo && !drain()) ok = false;  // one block behind the split
            }
            if (ok && khi > klo && !drain()) ok = false;
          }
          for (int h = 0; ok && h < NH; ++h, ++local) {
            const int n0 = nt * BN + h * EN;
            // this pass's bias column, loaded before the TMEM wait so that its latency overlaps it
            // (EN <= EPI_THREADS: one column per thread)
            const float bias_v = p.bias && et < EN && n0 + et < p.N ? __ldg(p.bias + n0 + et) : 0.0f;
            if (MODE != STRICT && !load_pass(h)) {
                ok = false;
                break;
            }
            if ((MODE == TF32 || MODE == STRICT) && !PAIR && !RB && NH == 1 && splits > 1) {
                // split K: this unit's raw partial tile (its row, this thread's columns); the
                // reduce kernel that follows on the stream applies the epilogue. Strict partials are
                // the fp64 sums themselves (the reduce finishes in fp64, as the tile epilogue does).
                const size_t at = ((size_t)(mt * p.n_tiles + nt) * splits + ks) * (BM * BN) + (size_t)row * BN + hc;
                if (MODE == STRICT) {
                    double *mine = reinterpret_cast<double *>(p.part) + at;
#pragma unroll
                    for (int j = 0; j < HALF; j += 2)
                        *reinterpret_cast<double2 *>(mine + j) = make_double2((double)acc[j], (double)acc[j + 1]);
                } else {
                    float *mine = p.part + at;
#pragma unroll
                    for (int j = 0; j < HALF; j += 4)
                        *reinterpret_cast<float4 *>(mine + j) =
                            make_float4((float)acc[j], (float)acc[j + 1], (float)acc[j + 2], (float)acc[j + 3]);
                }
                continue;
            }
            // this pass's bias columns into shared memory (the previous pass's readers have all
            // passed its second barrier)
            if (p.bias && et < EN) bias_s[et] = bias_v;
            // the staging tile is free (the previous TMA store was read out: SR, and every form
            // without a residual, waits for it here rather than right after issuing it) and the
            // residual staging holds this pass's residual
            stg = p.out2 && (local & 1) ? out_tile2 : out_tile;
            if ((SR || !res_tma) && issuer) {
                // with two staging tiles only the store that read this pass's tile (two passes
                // back; one commit group per pass) must be done
                if (p.out2) tma_store_wait_read_but_one();
                else tma_store_wait_read();
            }
            epilogue_sync();
            if (res_tma && !mbar_wait(res_full, (uint32_t)(local & 1))) {
                ok = false;
                break;
            }
            // 32 columns at a time: the residual and bias loads of a chunk are all issued before
            // its stores, so no load waits behind a store to the same staging tile
            const uint32_t out_s = smem_addr(stg), res_s = smem_addr(res_tile);
            const uint32_t bias_addr = smem_addr(bias_s);
#pragma unroll
            for (int a0 = 0; a0 < HALF; a0 += 32) {  // a0: accumulator index; column hc + a0
                float4 rv[8], bvs[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    rv[j] = res_tma ? lds4(res_s + stage_offset(row, hc + a0 + 4 * j)) : make_float4(0.f, 0.f, 0.f, 0.f);
                    bvs[j] = p.bias ? lds4(bias_addr + 4 * (hc + a0 + 4 * j)) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int c = a0 + 4 * j;  // accumulator index
                    const float4 bv = bvs[j];
                    float4 o;
                    if (MODE == STRICT) {  // the same sum in fp64 with the step-bias compensation
                        const double sa = (double)p.alpha * (1.0 + STEP_BIAS);
                        double d0 = sa * (double)acc[c + 0] + (double)bv.x, d1 = sa * (double)acc[c + 1] + (double)bv.y;
                        double d2 = sa * (double)acc[c + 2] + (double)bv.z, d3 = sa * (double)acc[c + 3] + (double)bv.w;
                        if (res_tma) {
                            d0 += rv[j].x; d1 += rv[j].y; d2 += rv[j].z; d3 += rv[j].w;
                        }
                        o = make_float4((float)d0, (float)d1, (float)d2, (float)d3);
                    } else {
                        o.x = p.alpha * (float)acc[c + 0] + bv.x;
                        o.y = p.alpha * (float)acc[c + 1] + bv.y;
                        o.z = p.alpha * (float)acc[c + 2] + bv.z;
                        o.w = p.alpha * (float)acc[c + 3] + bv.w;
                        if (res_tma) {
                            o.x += rv[j].x; o.y += rv[j].y; o.z += rv[j].z; o.w += rv[j].w;
                        }
                    }
                    if (act_in_step1 && p.act == MGC_ACT_RELU) {
                        o.x = fmaxf(o.x, 0.0f); o.y = fmaxf(o.y, 0.0f); o.z = fmaxf(o.z, 0.0f); o.w = fmaxf(o.w, 0.0f);
                    } else if (act_in_step1 && p.act == MGC_ACT_CLIP) {
                        o.x = fminf(fmaxf(o.x, p.lo), p.hi); o.y = fminf(fmaxf(o.y, p.lo), p.hi);
                        o.z = fminf(fmaxf(o.z, p.lo), p.hi); o.w = fminf(fmaxf(o.w, p.lo), p.hi);
                    }
                    sts4(out_s + stage_offset(row, hc + c), o);
                }
            }
            if (!act_in_step1 && !res_direct) {  // transcendental activation on this thread's row
#pragma unroll 1
                for (int c0 = hc; c0 < hc + HALF; c0 += 4) {
                    float4 *slot = stage_slot(row, c0);
                    float4 o = *slot;
                    o.x = apply_act(o.x, p.act, p.lo, p.hi);
                    o.y = apply_act(o.y, p.act, p.lo, p.hi);
                    o.z = apply_act(o.z, p.act, p.lo, p.hi);
                    o.w = apply_act(o.w, p.act, p.lo, p.hi);
                    *slot = o;
                }
            }
            if (!PH && p.gap_hw > 0) {
                // GlobalAveragePool partials from the staged pass (thread et: column et % EN of the
                // 32-row groups of row part et / EN), in place of the output stores
                static_assert(EPI_THREADS % EN == 0 && (BM / 32) % (EPI_THREADS / EN) == 0, "GAP row groups");
                constexpr int RG = EPI_THREADS / EN, PER = (BM / 32) / RG;  // threads per column, groups each
                epilogue_sync();
                const int gc = et % EN, rg = et / EN;
                if (n0 + gc < p.N) {
#pragma unroll 1
                    for (int g = rg * PER; g < (rg + 1) * PER; ++g) {
                        const long long mg = (long long)m0 + g * 32;
                        if (mg >= p.M) break;
                        // rows of the group that exist, and the first of them in the next image
                        const int lim = p.M - mg < 32 ? (int)(p.M - mg) : 32;
                        const int split = (int)((mg / p.gap_hw + 1) * p.gap_hw - mg);
                        float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
                        for (int r = 0; r < 32; ++r) {
                            const float x = reinterpret_cast<const float *>(stg + stage_offset(g * 32 + r, gc & ~3))[gc & 3];
                            if (r < lim) {
                                if (r < split) s0 += x;
                                else s1 += x;
                            }
                        }
                        float *dst = p.c + (mg / 32) * 2 * p.ldc + n0 + gc;
                        dst[0] = s0;
                        dst[p.ldc] = s1;
                    }
                }
                fence_proxy_async_smem();
                epilogue_sync();  // the staged pass is read out
                if (issuer && res_tma) {  // the next pass's residual: this tile's, or the next tile's first
                    int mt2, nt2;
                    if (h + 1 < NH) issue_residual(mt, nt, h + 1);
                    else if (tile_at(i + 1, mt2, nt2)) issue_residual(mt2, nt2, 0);
                }
            } else if (PH && p.pool_bp > 0) {
                // 3x3 / stride-2 / pad-1 max pooling of the output rows, in order: thread et keeps
                // channels 4 (et % 16) .. + 3 of pooled columns et / 16, + 16, ... (PW <= 64); a
                // pooled row ph is complete at output row 2 ph + 1 (padding: -inf, never the
                // maximum)
                epilogue_sync();
                int img, oh;
                bool first;
                pool_row(i, img, oh, first);
                const int c4 = (et & 15) * 4, pw0 = et >> 4;
                const bool live_c = c4 < p.N;
                if (oh < 0) {
#pragma unroll
                    for (int k = 0; k < POOL_PER_THREAD; ++k)
                        pool_acc[k] = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
                } else {
                    const int mode = first ? 0 : (oh & 1) ? 2 : 1;  // 0 start, 1 accumulate, 2 complete
                    float *orow = p.c + ((long long)img * p.pool_ph + (oh >> 1)) * p.pool_pw * p.ldc + c4;
                    auto mx4 = [](float4 a, float4 b) {
                        return make_float4(fmaxf(a.x, b.x), fmaxf(a.y, b.y), fmaxf(a.z, b.z), fmaxf(a.w, b.w));
                    };
#pragma unroll
                    for (int k = 0; k < POOL_PER_THREAD; ++k) {
                        const int pw = pw0 + 16 * k;
                        if (pw >= p.pool_pw || !live_c) continue;
                        float4 h = mx4(*stage_slot(2 * pw, c4), *stage_slot(2 * pw + 1, c4));
                        if (pw > 0) h = mx4(h, *stage_slot(2 * pw - 1, c4));
                        if (mode == 0) {
                            pool_acc[k] = h;
                        } else if (mode == 1) {
                            pool_acc[k] = mx4(pool_acc[k], h);
                        } else {
                            *reinterpret_cast<float4 *>(orow + (long long)pw * p.ldc) = mx4(pool_acc[k], h);
                            pool_acc[k] = h;
                        }
                    }
                }
                epilogue_sync();  // the next tile may overwrite the staging tile
            } else if (direct) {
                epilogue_sync();
#pragma unroll 1
                for (int rr = 0; rr < 32; ++rr) {
                    const int r = q * 32 + rr;
                    const long long m = (long long)m0 + r;
                    if (m >= p.M) continue;
#pragma unroll
                    for (int sl = hc / 32; sl < (hc + HALF) / 32; ++sl) {
                        const int c = sl * 32 + lane;
                        const int n = n0 + c;
                        if (n >= p.N) continue;
                        float x = reinterpret_cast<const float *>(stage_slot(r, c & ~3))[c & 3];
                        if (res_direct) x = apply_act(x + p.res[m * p.ldr + n], p.act, p.lo, p.hi);
                        p.c[m * p.ldc + n] = x;
                    }
                }
                epilogue_sync();  // the next tile may overwrite the staging tile
            } else {
                fence_proxy_async_smem();
                epilogue_sync();
                if (issuer) {
                    int mt2, nt2;
                    if (SR) {  // the residual staging is read out: the next pass's residual now
                        if (res_tma && h + 1 < NH) issue_residual(mt, nt, h + 1);
                        else if (res_tma && tile_at(i + 1, mt2, nt2)) issue_residual(mt2, nt2, 0);
                    }
                    if (rows) {  // the tile's rt_rows output rows; staging rows past them are dropped
                        const int img = mt / p.rt_per_img, oh0 = (mt - img * p.rt_per_img) * p.rt_rows;
#pragma unroll 1
                        for (int sl = 0; sl < EN / 32; ++sl)
                            tma_store_4d(&p.tmC, stg + sl * (BM * 128), n0 + sl * 32, 0, oh0, img);
                    } else if (m0 < p.M && n0 < p.N) {  // (a pair's second half, or a wide tile's last
                                                         // passes, may lie wholly past the edge)
#pragma unroll 1
                        for (int sl = 0; sl < EN / 32; ++sl) {
                            if (MODE == DYN) tma_store_4d(&p.tmC, stg + sl * (BM * 128), n0 + sl * 32, m0, db1, db2);
                            else tma_store_2d(&p.tmC, stg + sl * (BM * 128), n0 + sl * 32, m0);
                        }
                    }
                    if (SR || !res_tma) {
                        tma_store_commit();  // read out before the next pass writes the staging tile
                    } else {
                        tma_store_commit_and_wait();
                        // the next pass's residual: this tile's, or the next tile's first
                        if (res_tma && h + 1 < NH) issue_residual(mt, nt, h + 1);
                        else if (res_tma && tile_at(i + 1, mt2, nt2)) issue_residual(mt2, nt2, 0);
                    }
                }
            }
          }
        }
        if (!ok) set_error(p.err, MGC_CUDA_TIMEOUT);
        // a residual prefetch that no tile consumed must land, and the last store must have read
        // the staging tile, before the CTA exits
        if (res_tma && issuer && !ok) mbar_wait(res_full, (uint32_t)(local & 1));
        if ((SR || !res_tma) && issuer) tma_store_wait_read();
        (void)et;
    }
    tc_fence_before();
    __syncthreads();
    if (PAIR) cluster_sync_all();  // no CTA of a pair leaves while its peer may still signal it
    if (warp == 1) {
        tc_fence_after();
        if (PAIR) tmem_dealloc_pair(tmem_base, C::TMEM_ALLOC);
        else tmem_dealloc(tmem_base, C::TMEM_ALLOC);
    }
}

// Split-K epilogue: out[m][n] = act(alpha * sum_ks part[tile][ks][m % 128][n % BN] + bias[n]
// (+ res[m][n])), the partials summed in split order (the same result on every run), one
// output per thread; the same arithmetic as the tile epilogue's direct path.
__global__ void __launch_bounds__(256) split_reduce_kernel(const float *part, int splits, int n_tiles, int bn, int M,
                                                           int N, float *c, long long ldc, const float *bias,
                                                           const float *res, long long ldr, float alpha, int act,
                                                           float lo, float hi) {
    const long long total = (long long)M * N;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const int m = (int)(e / N), n = (int)(e - (long long)m * N);
        const int mt = m / BM, nt = n / bn;
        const float *src = part + ((size_t)(mt * n_tiles + nt) * splits) * (BM * bn) + (size_t)(m - mt * BM) * bn + (n - nt * bn);
        // eight partials in flight at a time, added in split order
        const size_t step = (size_t)BM * bn;
        float acc = 0.0f;
        int ks = 0;
        for (; ks + 8 <= splits; ks += 8) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __ldcg(src + (size_t)(ks + j) * step);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc += v[j];
        }
        for (; ks < splits; ++ks) acc += __ldcg(src + (size_t)ks * step);
        float x = alpha * acc + (bias ? bias[n] : 0.0f);
        if (res) x += res[(long long)m * ldr + n];
        c[(long long)m * ldc + n] = apply_act(x, act, lo, hi);
    }
}

// Strict split K: the fp64 partials summed in split order in fp64, then the strict tile epilogue's
// arithmetic: alpha * (1 + STEP_BIAS) * acc + bias (+ res) in fp64, rounded once, activation.
__global__ void __launch_bounds__(256) split_reduce_f64_kernel(const double *part, int splits, int n_tiles, int bn,
                                                               int M, int N, float *c, long long ldc, const float *bias,
                                                               const float *res, long long ldr, float alpha, int act,
                                                               float lo, float hi) {
    const long long total = (long long)M * N;
    const double sa = (double)alpha * (1.0 + STEP_BIAS);
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const int m = (int)(e / N), n = (int)(e - (long long)m * N);
        const int mt = m / BM, nt = n / bn;
        const double *src = part + ((size_t)(mt * n_tiles + nt) * splits) * (BM * bn) + (size_t)(m - mt * BM) * bn + (n - nt * bn);
        const size_t step = (size_t)BM * bn;
        double acc = 0.0;
        for (int ks = 0; ks < splits; ++ks) acc += __ldcg(src + (size_t)ks * step);
        double x = sa * acc + (bias ? (double)bias[n] : 0.0);
        if (res) x += (double)res[(long long)m * ldr + n];
        c[(long long)m * ldc + n] = apply_act((float)x, act, lo, hi);
    }
}

// ---- host side ---------------------------------------------------------------------------------
inline PFN_cuTensorMapEncodeTiled_v12000 encode_tiled_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void *ptr = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
        else
            cudaGetLastError();
    }
    return fn;
}

inline PFN_cuTensorMapEncodeIm2col_v12000 encode_im2col_fn() {
    static PFN_cuTensorMapEncodeIm2col_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void *ptr = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(ptr);
        else
            cudaGetLastError();
    }
    return fn;
}

// Row-major fp32 matrix [rows, cols] with row stride `ld` elements, boxes of 32 x box_rows.
// `tf32` selects the TFLOAT32 element type, which rounds to the nearest TF32 value on load.
inline bool make_map_2d(CUtensorMap *map, const void *base, long long rows, long long cols, long long ld,
                        int box_rows, bool tf32 = false) {
    auto fn = encode_tiled_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * 4)};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, tf32 ? CU_TENSOR_MAP_DATA_TYPE_TFLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                    const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// The two K-major planes of a constant B ([N][Kp] TF32 part at `hi`, residual at `lo`, lo > hi)
// as one tensor [2][N][Kp]; a box {32, box_rows, 2} lands as the hi tile followed by the lo tile,
// a box {32, box_rows, 1} (planes = 1, CTA pairs) as the tile of one plane.
inline bool make_map_b(CUtensorMap *map, const float *hi, const float *lo, long long rows, long long kp, int box_rows,
                       int planes = 2) {
    auto fn = encode_tiled_fn();
    if (!fn) return false;
    const long long gap = reinterpret_cast<const char *>(lo) - reinterpret_cast<const char *>(hi);
    if (gap <= 0 || (gap & 15) || gap >= (1ll << 40)) return false;
    cuuint64_t dims[3] = {(cuuint64_t)kp, (cuuint64_t)rows, 2};
    cuuint64_t strides[2] = {(cuuint64_t)(kp * 4), (cuuint64_t)gap};
    cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)box_rows, (cuuint32_t)planes};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(hi), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// One K-major plane of a constant B ([N][Kp], TF32-exact) as a 3-D tensor [1][N][Kp], boxes {32,
// box_rows, 1}: the coordinates the two-plane map takes, with plane 0 only.
inline bool make_map_b1(CUtensorMap *map, const float *plane, long long rows, long long kp, int box_rows) {
    auto fn = encode_tiled_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)kp, (cuuint64_t)rows, 1};
    cuuint64_t strides[2] = {(cuuint64_t)(kp * 4), (cuuint64_t)(rows * kp * 4)};
    cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(plane), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// NHWC fp32 image, im2col boxes of `chans` channels x 128 output pixels: 32 channels in 128-byte
// swizzled rows, or 4 channels in plain 16-byte rows (tap-packed).
inline bool make_map_im2col(CUtensorMap *map, const GemmParams &g, bool tf32, int chans = BK) {
    auto fn = encode_im2col_fn();
    if (!fn) return false;
    const long long nimg = (long long)g.M / ((long long)g.OH * g.OW);
    cuuint64_t dims[4] = {(cuuint64_t)g.C, (cuuint64_t)g.W, (cuuint64_t)g.H, (cuuint64_t)nimg};
    cuuint64_t strides[3] = {(cuuint64_t)g.C * 4, (cuuint64_t)g.W * g.C * 4, (cuuint64_t)g.H * g.W * g.C * 4};
    // bounding box of window origins: from -pad to the last output's origin, W then H
    int lower[2] = {-g.PL, -g.PT};
    int upper[2] = {(g.OW - 1) * g.SW - g.PL - (g.W - 1), (g.OH - 1) * g.SH - g.PT - (g.H - 1)};
    cuuint32_t estr[4] = {1, (cuuint32_t)g.SW, (cuuint32_t)g.SH, 1};
    CUresult r = fn(map, tf32 ? CU_TENSOR_MAP_DATA_TYPE_TFLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4,
                    const_cast<float *>(g.a), dims, strides, lower, upper, (cuuint32_t)chans, BM, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, chans == BK ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Window rows of a spatially padded NHWC image (C channels, Hp x Wp, no further padding needed):
// element (x, ow, oh, n, kh) = image[n][oh*SH + kh*DH][ow*SW + x / C][x % C] for x < KW * C, the
// contiguous run that one filter row of a window covers. Consecutive output pixels overlap (their
// stride SW*C*4 bytes is below the 128-byte box row), so a TMA tile box {32, wrows, 1, 1, 1}
// reads 128-byte rows with no gather; x past KW * C is outside the tensor and reads as zero.
inline bool make_map_window(CUtensorMap *map, const GemmParams &g, int wrows, bool tf32, int box_oh = 1) {
    auto fn = encode_tiled_fn();
    if (!fn) return false;
    const long long nimg = (long long)g.M / ((long long)g.OH * g.OW);
    const long long px = (long long)g.C * 4;  // bytes per pixel
    cuuint64_t dims[5] = {(cuuint64_t)g.KW * g.C, (cuuint64_t)g.OW, (cuuint64_t)g.OH, (cuuint64_t)nimg, (cuuint64_t)g.KH};
    cuuint64_t strides[4] = {(cuuint64_t)(g.SW * px), (cuuint64_t)(g.SH * g.W * px), (cuuint64_t)((long long)g.H * g.W * px),
                             (cuuint64_t)(g.DH * g.W * px)};
    cuuint32_t box[5] = {(cuuint32_t)BK, (cuuint32_t)wrows, (cuuint32_t)box_oh, 1, 1};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = fn(map, tf32 ? CU_TENSOR_MAP_DATA_TYPE_TFLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 5,
                    const_cast<float *>(g.a), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// An NHWC output (or residual) [nimg][OH][OW][N] with row stride ld as a 4-D tensor {N, OW, OH,
// nimg}; a box {32, OW, rows, 1} covers whole output rows (row tiles), clipped at OH.
inline bool make_map_rows(CUtensorMap *map, const void *base, long long n, long long ld, int ow, int oh, long long nimg,
                          int rows) {
    auto fn = encode_tiled_fn();
    if (!fn) return false;
    cuuint64_t dims[4] = {(cuuint64_t)n, (cuuint64_t)ow, (cuuint64_t)oh, (cuuint64_t)nimg};
    cuuint64_t strides[3] = {(cuuint64_t)(ld * 4), (cuuint64_t)(ow * ld * 4), (cuuint64_t)((long long)oh * ow * ld * 4)};
    cuuint32_t box[4] = {(cuuint32_t)BK, (cuuint32_t)ow, (cuuint32_t)rows, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Dynamic shared memory of a launch. Pair launches ask for more than half an SM's shared memory,
// so no two CTAs (and no two TMEM allocations) ever share an SM.
// fp32 tensor [b2][b1][rows][cols] with element strides (row, b1, b2) as a 4-D map {cols, rows, b1,
// b2}, boxes {32, box_rows, 1, 1}; TFLOAT32 rounds to the nearest TF32 value on load.
inline bool make_map_4d(CUtensorMap *map, const void *base, long long cols, long long rows, long long b1, long long b2,
                        long long row_stride, long long b1_stride, long long b2_stride, int box_rows, bool tf32) {
    auto fn = encode_tiled_fn();
    if (!fn) return false;
    cuuint64_t dims[4] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)b1, (cuuint64_t)b2};
    cuuint64_t strides[3] = {(cuuint64_t)(row_stride * 4), (cuuint64_t)(b1_stride * 4), (cuuint64_t)(b2_stride * 4)};
    cuuint32_t box[4] = {(cuuint32_t)BK, (cuuint32_t)box_rows, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(map, tf32 ? CU_TENSOR_MAP_DATA_TYPE_TFLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4,
                    const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int BN, int MODE, int RB, int PAIR, int SR = 0, int PH = 0, int SP = 0>
inline uint32_t launch_smem(const Params &p) {
    using C = Cfg<BN, MODE, RB, PAIR, SR, PH, SP>;
    const uint32_t smem = C::SMEM_BYTES + (RB ? p.b_res_bytes : 0u);
    return PAIR && smem < SMEM_LIMIT / 2 + 1024 ? SMEM_LIMIT / 2 + 1024 : smem;
}

template <int BN, int MODE, int RB, int PAIR, int SR = 0, int PH = 0, int SP = 0>
inline int launch(const Params &p_in, int grid, cudaStream_t stream) {
    using C = Cfg<BN, MODE, RB, PAIR, SR, PH, SP>;
    Params p = p_in;
    uint32_t smem = launch_smem<BN, MODE, RB, PAIR, SR, PH, SP>(p);
    // a second output staging tile where shared memory has room for it and the epilogue stores
    // by TMA without a residual staged in the output tile (MGC_CUDA_OUT2=0 keeps one, for
    // comparisons)
    p.out2 = 0;
    if (MODE != STRICT && !SR && p.tma_out && !p.tma_res && p.splits <= 1 &&
        C::SMEM_BYTES + (RB ? p.b_res_bytes : 0u) + C::OUT_BYTES + 1024 <= SMEM_LIMIT &&
        !(getenv("MGC_CUDA_OUT2") && getenv("MGC_CUDA_OUT2")[0] == '0')) {
        p.out2 = 1;
        const uint32_t need = C::SMEM_BYTES + (RB ? p.b_res_bytes : 0u) + C::OUT_BYTES + 1024;
        if (need > smem) smem = need;
    }
    // per device (the attribute belongs to the current context); allowed under capture
    MGC_CHECK(raise_smem_ceiling((const void *)umma_gemm_kernel<BN, MODE, RB, PAIR, SR, PH, SP>));
    if (!PAIR) {
        umma_gemm_kernel<BN, MODE, RB, PAIR, SR, PH, SP><<<grid, THREADS, smem, stream>>>(p);
        return check_launch("umma_gemm_kernel");
    }
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1] = {};
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    MGC_CHECK_CUDA(cudaLaunchKernelEx(&cfg, umma_gemm_kernel<BN, MODE, RB, PAIR, SR, PH, SP>, p));
    return check_launch("umma_gemm_kernel (pair)");
}

// The B-resident variant when this CTA's B panel fits beside its stages and every CTA walks at
// least two M tiles (else loading the panel per tile costs the same).
template <int BN, int MODE>
inline int launch_best(Params &p, long long m_tiles, cudaStream_t stream) {
    const int sms = sm_count();
    const uint32_t panel = (uint32_t)p.num_kb * 2u * Cfg<BN, MODE, 1>::B_TILE_BYTES;
    const int per = p.n_tiles <= sms ? sms / p.n_tiles : 0;
    if (per > 0 && panel <= Cfg<BN, MODE, 1>::B_RES_MAX && m_tiles >= 2LL * per) {
        p.b_res_bytes = panel;
        return launch<BN, MODE, 1, 0>(p, per * p.n_tiles, stream);
    }
    p.b_res_bytes = 0;
    const long long tiles = (long long)p.n_tiles * m_tiles;
    return launch<BN, MODE, 0, 0>(p, (int)(tiles < sms ? tiles : sms), stream);
}

// Phase-split row tiles (one N tile of 64, TF32, B resident; the caller checked that the panel
// and a tile's rows fit): one CTA per SM, or one per tile when there are fewer tiles.
inline int launch_phase(Params &p, long long m_tiles, cudaStream_t stream) {
    using C1 = Cfg<64, TF32, 1, 0, 0, 1>;
    p.b_res_bytes = (uint32_t)p.num_kb * C1::B_PLANES * C1::B_TILE_BYTES;
    const int sms = sm_count();
    return launch<64, TF32, 1, 0, 0, 1>(p, (int)(m_tiles < sms ? m_tiles : sms), stream);
}

// Whether a phase-split launch fits: the B panel beside the stages, and every byte the MMAs read
// inside a stage (the last K block's odd-tap phase, read at pixel offsets up to BM - 1 + 3).
inline bool phase_fits(int num_kb, uint32_t row_bytes, uint32_t phase_bytes) {
    using C1 = Cfg<64, TF32, 1, 0, 0, 1>;
    const uint32_t last = (uint32_t)(num_kb - 1) * row_bytes + phase_bytes + 32 + (BM - 1) * 16 + 32;
    return (uint32_t)num_kb * C1::B_PLANES * C1::B_TILE_BYTES <= C1::B_RES_MAX && last <= PHASE_STAGE_BYTES;
}

// One CTA per tile with a residual through its own staging buffer (N tiles of 128, TF32), when
// the B panel fits beside a two-stage A ring (B-resident; measured on ResNet-50 batch 256: the
// 1x1 C64->256 + residual layers 16 % faster). With B streamed, two stages starve the MMAs
// (+33 % on 1x1 C256->1024 + residual), so the output staging is shared as before.
inline int launch_best_sr(Params &p, long long m_tiles, cudaStream_t stream) {
    using C1 = Cfg<128, TF32, 1, 0, 1>;
    const int sms = sm_count();
    const uint32_t panel = (uint32_t)p.num_kb * 2u * C1::B_TILE_BYTES;
    const int per = p.n_tiles <= sms ? sms / p.n_tiles : 0;
    if (per > 0 && panel <= C1::B_RES_MAX && m_tiles >= 2LL * per) {
        p.b_res_bytes = panel;
        return launch<128, TF32, 1, 0, 1>(p, per * p.n_tiles, stream);
    }
    // 64-column passes leave room for a B panel of up to 128 KB (1x1 C128->512)
    if (per > 0 && panel <= Cfg<128, TF32, 1, 0, 2>::B_RES_MAX && m_tiles >= 2LL * per) {
        p.b_res_bytes = panel;
        return launch<128, TF32, 1, 0, 2>(p, per * p.n_tiles, stream);
    }
    p.b_res_bytes = 0;
    const long long tiles = (long long)p.n_tiles * m_tiles;
    return launch<128, TF32, 0, 0, 2>(p, (int)(tiles < sms ? tiles : sms), stream);
}

// Clusters of two that fit on the device at once (one CTA per SM), per kernel variant; 0 if
// the query fails. Cached per device.
template <int BN, int RB>
inline int pair_clusters() {
    static int cached[64];
    static bool known[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return 0;
    }
    if (known[dev]) return cached[dev];
    Params dummy;
    memset(&dummy, 0, sizeof dummy);
    const uint32_t smem = launch_smem<BN, TF32, RB, 1>(dummy);
    int n = 0;
    if (cudaFuncSetAttribute(umma_gemm_kernel<BN, TF32, RB, 1, 0, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)SMEM_LIMIT) == cudaSuccess) {
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1] = {};
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(2);
        cfg.blockDim = dim3(THREADS);
        cfg.dynamicSmemBytes = smem;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, umma_gemm_kernel<BN, TF32, RB, 1, 0, 0>, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();
    cached[dev] = n;
    known[dev] = true;
    return n;
}

// Wide CTA-pair launch: 256 x BN tiles, BN 192 or 256, or 128 with SP (p.m_tiles and p.n_tiles
// count them; p.tmB boxes both planes of BN / 2 rows, or with SP the TF32 plane only).
template <int BN, int SP = 0>
inline int launch_wide(Params &p, int clusters, cudaStream_t stream) {
    p.b_res_bytes = 0;
    const long long tiles = (long long)p.n_tiles * p.m_tiles;
    return launch<BN, TF32, 0, 1, 0, 0, SP>(p, 2 * (int)(tiles < clusters ? tiles : clusters), stream);
}

// CTA-pair launch (TF32 mode, tiled or 32-channel im2col A): p.m_tiles counts 256-row tiles and
// p.tmB boxes one plane. B-resident when this CTA's plane of the panel fits.
template <int BN>
inline int launch_pair(Params &p, int clusters, cudaStream_t stream) {
    using C1 = Cfg<BN, TF32, 1, 1>;
    const uint32_t panel = (uint32_t)p.num_kb * C1::B_TILE_BYTES;
    const int per = p.n_tiles <= clusters ? clusters / p.n_tiles : 0;
    if (per > 0 && panel <= C1::B_RES_MAX && p.m_tiles >= 2LL * per) {
        p.b_res_bytes = panel;
        return launch<BN, TF32, 1, 1>(p, 2 * per * p.n_tiles, stream);
    }
    p.b_res_bytes = 0;
    const long long tiles = (long long)p.n_tiles * p.m_tiles;
    return launch<BN, TF32, 0, 1>(p, 2 * (int)(tiles < clusters ? tiles : clusters), stream);
}

}  // namespace umma

// GEMM with a dynamic B (an activation, rounded to TF32 by its tensor map like A) on the tensor
// cores: attention's Q K^T and P V, any MatMul of two activations, and the kernel ABI's TF32
// GEMM. TF32 mode, both operands K-major (k contiguous), no, one or two batch dimensions with
// strides TMA can address (no broadcast). Without batch dimensions the FusedGemm epilogue applies
// (alpha, bias per column, residual, activation); batched products take none. Each tile lies
// inside one batch, so rows past M are clipped per batch. *taken: kernels launched (0 or 1).
inline int try_gemm_umma_dyn(const GemmParams &p, cudaStream_t stream, int *taken) {
    *taken = 0;
    if (p.precision != MGC_PREC_TF32 || p.nb < 0 || p.nb > 2 || p.b_umma || p.b_lo) return MGC_CUDA_OK;
    if (p.a_kind != MGC_STRIDED || p.b_kind != MGC_STRIDED || p.a_cs != 1 || p.b_rs != 1) return MGC_CUDA_OK;
    if (p.M <= 0 || p.N <= 0 || p.K <= 0) return MGC_CUDA_OK;
    const bool epilogue = p.bias || p.res || p.act != MGC_ACT_NONE || p.alpha != 1.0f;
    if ((epilogue && p.nb != 0) || (p.bias && p.bias_mode != 1)) return MGC_CUDA_OK;
    auto al = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    auto st = [](long long v) { return v > 0 && (v & 3) == 0; };  // a 16-byte multiple, not a broadcast
    if (!al(p.a) || !al(p.b) || !al(p.c) || !st(p.a_rs) || !st(p.b_cs) || !st(p.ldc) || (p.K & 3) || (p.N & 3))
        return MGC_CUDA_OK;
    if (p.res && (!al(p.res) || !st(p.ldr))) return MGC_CUDA_OK;
    const long long b1 = p.nb >= 1 ? p.bdims[0] : 1, b2 = p.nb == 2 ? p.bdims[1] : 1;
    if (b1 <= 0 || b2 <= 0) return MGC_CUDA_OK;
    for (int d = 0; d < p.nb; ++d)
        if (!st(p.a_bs[d]) || !st(p.b_bs[d]) || !st(p.c_bs[d])) return MGC_CUDA_OK;
    // strides of batch dimensions of extent 1 (unused): any valid value
    const long long a1 = p.nb >= 1 ? p.a_bs[0] : p.a_rs * p.M, bb1 = p.nb >= 1 ? p.b_bs[0] : p.b_cs * p.N;
    const long long c1 = p.nb >= 1 ? p.c_bs[0] : p.ldc * p.M;
    const long long a2 = p.nb == 2 ? p.a_bs[1] : a1 * b1, bb2 = p.nb == 2 ? p.b_bs[1] : bb1 * b1;
    const long long c2 = p.nb == 2 ? p.c_bs[1] : c1 * b1;
    const int bn = p.N <= 64 ? 64 : 128;
    umma::Params u;
    memset(&u, 0, sizeof u);
    if (!umma::make_map_4d(&u.tmA, p.a, p.K, p.M, b1, b2, p.a_rs, a1, a2, umma::BM, true) ||
        !umma::make_map_4d(&u.tmB, p.b, p.K, p.N, b1, b2, p.b_cs, bb1, bb2, bn, true) ||
        !umma::make_map_4d(&u.tmC, p.c, p.N, p.M, b1, b2, p.ldc, c1, c2, umma::BM, false))
        return MGC_CUDA_OK;
    if (p.res) {
        // the residual tile is TMA-loaded into the output staging tile (rows m0.. of the one batch)
        if (!umma::make_map_2d(&u.tmR, p.res, p.M, p.N, p.ldr, umma::BM)) return MGC_CUDA_OK;
        u.tma_res = 1;
        u.res = p.res;
        u.ldr = p.ldr;
    }
    const long long m_per = ceil_div(p.M, umma::BM), tiles_m = m_per * b1 * b2;
    const long long n_tiles = ceil_div(p.N, bn);
    if (tiles_m * n_tiles > 0x7FFFFFFF) return MGC_CUDA_OK;
    u.M = p.M;
    u.N = p.N;
    u.num_kb = (int)ceil_div(p.K, umma::BK);
    u.n_tiles = (int)n_tiles;
    u.m_tiles = (int)tiles_m;
    u.m_per_batch = (int)m_per;
    u.nbatch1 = (int)b1;
    u.a_bytes = umma::A_TILE_BYTES;
    u.tma_out = 1;
    u.c = p.c; u.ldc = p.ldc;
    u.bias = p.bias;
    u.alpha = p.alpha; u.lo = p.lo; u.hi = p.hi; u.act = p.act;
    u.err = p.err;
    const int sms = sm_count();
    const long long tiles = tiles_m * n_tiles;
    const int grid = (int)(tiles < sms ? tiles : sms);
    const int rc = bn == 64 ? umma::launch<64, umma::DYN, 0, 0>(u, grid, stream)
                            : umma::launch<128, umma::DYN, 0, 0>(u, grid, stream);
    if (rc != MGC_CUDA_OK) return rc;
    *taken = 1;
    return MGC_CUDA_OK;
}

// Whether the tensor-core kernel takes this GEMM, and its launch; *taken is the number of kernels
// launched (0: not taken, the caller runs the SIMT kernel). Requirements: tf32 or 3xtf32
// precision, no batch dimensions, a constant K-major B in the layout the lowering provides
// (b_umma + b_umma_lo), A as a unit-stride row-major matrix or an NHWC im2col operand with
// 16-byte aligned rows, bias per column (or none), fp32 output.
inline int try_gemm_umma(const GemmParams &p, cudaStream_t stream, int *taken) {
    *taken = 0;
    if (!p.b_umma) return try_gemm_umma_dyn(p, stream, taken);
    // a constant B in two planes (TF32 part + residual), or one TF32 plane for phase-split tiles
    if (p.precision == MGC_PREC_FP32 || p.nb != 0 || !p.b_umma || (!p.b_umma_lo && p.phase_w <= 0) || p.M <= 0 ||
        p.N <= 0 || p.K <= 0)
        return MGC_CUDA_OK;
    if (p.bias && p.bias_mode != 1) return MGC_CUDA_OK;
    const bool strict = p.precision == MGC_PREC_3XTF32;
    if ((reinterpret_cast<uintptr_t>(p.a) & 15) || (reinterpret_cast<uintptr_t>(p.b_umma) & 15) ||
        (reinterpret_cast<uintptr_t>(p.b_umma_lo) & 15))
        return MGC_CUDA_OK;
    if (p.phase_w > 0 && p.b_umma_lo) return MGC_CUDA_OK;  // phase-split tiles read one TF32 plane
    umma::Params u;
    memset(&u, 0, sizeof u);
    u.M = p.M;
    u.N = p.N;
    // TF32 mode rounds A to nearest while loading; strict mode loads raw fp32 and splits it
    const bool a_tf32 = !strict;
    int kp;  // K extent of the B operand (padded)
    if (p.a_kind == MGC_STRIDED) {
        if (p.a_cs != 1 || (p.a_rs & 3) || p.a_rs < p.K || (p.K & 3)) return MGC_CUDA_OK;
        kp = p.K;
        if (!umma::make_map_2d(&u.tmA, p.a, p.M, p.K, p.a_rs, umma::BM, a_tf32)) return MGC_CUDA_OK;
        u.im2col = 0;
        u.num_kb = (int)ceil_div(p.K, umma::BK);
    } else if (p.a_kind == MGC_CONV_NHWC) {
        if (p.cg != p.C || p.c_off != 0 || (p.C & 3) || p.b_cpad <= 0) return MGC_CUDA_OK;
        if (p.M % (p.OH * p.OW)) return MGC_CUDA_OK;
        // phase-split row tiles when the lowering packed the image by column phase (phase_w);
        // window rows when it laid B out as [N][KH][L] over a padded image (win_rows);
        // tap-packed when B is K-major over (kh, kw, channel) without channel padding (b_cpad ==
        // C < 32); otherwise one K block per filter tap and 32-channel block
        const bool phase = p.phase_w > 0;
        const bool window = !phase && p.win_rows > 0;
        const bool packed = !phase && !window && p.b_cpad == p.C && p.C < umma::BK;
        if (!window && !phase) {  // limits of the im2col tensor map: corner offsets, traversal strides
            const int lw = -p.PL, lh = -p.PT;
            const int uw = (p.OW - 1) * p.SW - p.PL - (p.W - 1), uh = (p.OH - 1) * p.SH - p.PT - (p.H - 1);
            if (lw < -128 || lh < -128 || uw > 127 || uh > 127 || uw < -128 || uh < -128) return MGC_CUDA_OK;
            if (p.SW > 8 || p.SH > 8 || (p.KW - 1) * p.DW > 65535 || (p.KH - 1) * p.DH > 65535) return MGC_CUDA_OK;
        }
        if (phase) {
            // the packed rows hold both phases of phase_w pixels of 4 channels (the image's padding
            // included); output pixel m reads pixels m .. m + 3 of each phase (tile rows past OW
            // read on into the stage and are never stored); a tile's KH rows are consecutive
            // (unit height dilation) and arrive in one copy
            const long long row_bytes = 2ll * p.phase_w * 16;
            if (strict || p.C != 4 || p.W != 2 * p.phase_w || p.PT || p.PL || p.SW != 2 || p.DW != 1 || p.DH != 1 || p.KW > 8 ||
                p.OW > umma::BM || p.phase_w < p.OW + 3 || p.b_cpad != 4 || p.N > 64 ||
                (long long)(p.OH - 1) * p.SH + (long long)(p.KH - 1) * p.DH >= p.H ||
                (reinterpret_cast<uintptr_t>(p.a) & 15) ||
                !umma::phase_fits(p.KH, (uint32_t)row_bytes, (uint32_t)p.phase_w * 16))
                return MGC_CUDA_OK;
            u.im2col = 5;
            u.cblocks = 1;
            u.num_kb = p.KH;
            kp = p.KH * umma::BK;
            u.a_rows = reinterpret_cast<const char *>(p.a);
            u.prow_bytes = row_bytes;
            u.prows = p.H;
            u.phase_bytes = p.phase_w * 16;
            u.a_bytes = (uint32_t)row_bytes;
        } else if (window) {
            if (p.PT || p.PL || p.DW != 1 || p.OW % p.win_rows || umma::BM % p.win_rows ||
                p.win_L != (int)ceil_div(p.KW * p.C, umma::BK) * umma::BK ||
                (long long)(p.OW - 1) * p.SW + p.KW > p.W ||
                (long long)(p.OH - 1) * p.SH + (long long)(p.KH - 1) * p.DH >= p.H)
                return MGC_CUDA_OK;
            if (!umma::make_map_window(&u.tmA, p, p.win_rows, a_tf32)) return MGC_CUDA_OK;
            u.im2col = 3;
            u.wrows = p.win_rows;
            u.cblocks = p.win_L / umma::BK;
            u.num_kb = p.KH * u.cblocks;
            kp = p.KH * p.win_L;
        } else if (!packed && (p.b_cpad & (umma::BK - 1))) {
            return MGC_CUDA_OK;
        } else if (!umma::make_map_im2col(&u.tmA, p, a_tf32, packed ? 4 : umma::BK)) {
            return MGC_CUDA_OK;
        } else if (packed) {
            u.im2col = 2;
            u.cpix = p.C;
            u.kreal = p.KH * p.KW * p.C;
            kp = u.kreal;
            u.num_kb = (int)ceil_div(kp, umma::BK);
        } else {
            u.im2col = 1;
            u.cblocks = p.b_cpad / umma::BK;
            u.num_kb = p.KH * p.KW * u.cblocks;
            kp = p.KH * p.KW * p.b_cpad;
        }
        u.KW = p.KW; u.DH = p.DH; u.DW = p.DW;
        u.OH = p.OH; u.OW = p.OW; u.SH = p.SH; u.SW = p.SW; u.PT = p.PT; u.PL = p.PL;
    } else {
        return MGC_CUDA_OK;
    }
    // strict mode keeps four TMEM regions per K block, which fits only N tiles of 64
    const int bn = (strict || p.N <= 64) ? 64 : 128;
    if (u.im2col == 5 ? !umma::make_map_b1(&u.tmB, p.b_umma, p.N, kp, bn)
                      : !umma::make_map_b(&u.tmB, p.b_umma, p.b_umma_lo, p.N, kp, bn))
        return MGC_CUDA_OK;
    u.n_tiles = (int)ceil_div(p.N, bn);
    long long m_tiles = ceil_div(p.M, umma::BM);
    if (u.im2col != 5) u.a_bytes = umma::A_TILE_BYTES;
    const long long tiles = (long long)u.n_tiles * m_tiles;
    if (tiles > 0x7FFFFFFF) return MGC_CUDA_OK;
    u.c = p.c; u.ldc = p.ldc; u.bias = p.bias; u.res = p.res; u.ldr = p.ldr;
    u.alpha = p.alpha; u.lo = p.lo; u.hi = p.hi; u.act = p.act;
    u.err = p.err;
    u.gap_hw = p.gap_hw;  // the pixels of one image, when the output is only pooled
    // output through a TMA store of the staged tile when C's rows are 16-byte aligned, with the
    // residual tile TMA-loaded into the staging buffer (both, or neither)
    u.tma_out = ((reinterpret_cast<uintptr_t>(p.c) & 15) == 0 && (p.ldc & 3) == 0 &&
                 umma::make_map_2d(&u.tmC, p.c, p.M, p.N, p.ldc, umma::BM)) ? 1 : 0;
    u.tma_res = (u.tma_out && p.res && (reinterpret_cast<uintptr_t>(p.res) & 15) == 0 && (p.ldr & 3) == 0 &&
                 umma::make_map_2d(&u.tmR, p.res, p.M, p.N, p.ldr, umma::BM)) ? 1 : 0;
    if (p.res && !u.tma_res) u.tma_out = 0;
    // Window rows with OW <= 128: M tiles of whole output rows (rt_rows of them, one image), so a
    // K block's A is one TMA box; output and residual move through 4-D maps that clip the rows
    // past the tile's last output row.
    if (u.im2col == 3 && u.tma_out && p.OW <= umma::BM) {
        const long long nimg = (long long)p.M / ((long long)p.OH * p.OW);
        const int rows = umma::BM / p.OW < p.OH ? umma::BM / p.OW : p.OH;
        CUtensorMap a4, c4, r4;
        bool okr = umma::make_map_window(&a4, p, p.OW, a_tf32, rows) &&
                   umma::make_map_rows(&c4, p.c, p.N, p.ldc, p.OW, p.OH, nimg, rows);
        if (okr && u.tma_res) okr = umma::make_map_rows(&r4, p.res, p.N, p.ldr, p.OW, p.OH, nimg, rows);
        if (okr) {
            u.tmA = a4;
            u.tmC = c4;
            if (u.tma_res) u.tmR = r4;
            u.im2col = 4;
            u.rt_rows = rows;
            u.rt_per_img = (int)ceil_div(p.OH, rows);
            m_tiles = nimg * u.rt_per_img;
            u.a_bytes = (uint32_t)rows * p.OW * 128;
            u.res_box_bytes = u.a_bytes;
        }
    }
    // Phase-split row tiles: one output row per tile (its output and residual through 4-D maps
    // that clip the tile's rows past OW), A read by bulk copies of packed rows.
    if (p.gap_hw > 0 && (u.im2col == 5 || p.gap_hw < 32)) return MGC_CUDA_OK;  // partials: not these forms
    if (u.im2col == 5 && p.pool_ph > 0) {
        // with the 3x3 / stride-2 / pad-1 max pooling in the epilogue: one N tile, even output
        // extents, the pooled image stored by the epilogue threads (no output map, no residual).
        // Bands of bp pooled rows cost 2 bp + 1 tiles each (one output row shared with the band
        // above, recomputed); bp is the divisor of the pooled height with the fewest tiles on the
        // busiest CTA (batch 256 at 56 pooled rows: bp 14, 7 bands per CTA, 203 tiles).
        const long long nimg = (long long)p.M / ((long long)p.OH * p.OW);
        if (p.N > 64 || (p.N & 3) || p.res || p.OH != 2 * p.pool_ph || p.OW != 2 * p.pool_pw ||
            p.pool_pw > 16 * umma::POOL_PER_THREAD || p.ldc < p.N || (p.ldc & 3) ||
            (reinterpret_cast<uintptr_t>(p.c) & 15) || nimg * p.pool_ph > 0x7FFFFFFF)
            return MGC_CUDA_OK;
        const long long sms = sm_count();
        int best = 0;
        long long best_cost = 0;
        for (int bp = 1; bp <= p.pool_ph; ++bp) {
            if (p.pool_ph % bp) continue;
            const long long cost = ceil_div(nimg * (p.pool_ph / bp), sms) * (2 * bp + 1);
            if (best == 0 || cost <= best_cost) { best = bp; best_cost = cost; }
        }
        u.tma_out = 0;
        u.tma_res = 0;
        u.rt_rows = 1;
        u.rt_per_img = p.OH;
        u.pool_bp = best;
        u.pool_nbp = p.pool_ph / best;
        u.pool_nbands = (int)(nimg * u.pool_nbp);
        u.pool_ph = p.pool_ph;
        u.pool_pw = p.pool_pw;
        m_tiles = u.pool_nbands;  // the launch's grid: one CTA per band at most
    } else if (u.im2col == 5) {
        const long long nimg = (long long)p.M / ((long long)p.OH * p.OW);
        CUtensorMap c4, r4;
        if (!u.tma_out || !umma::make_map_rows(&c4, p.c, p.N, p.ldc, p.OW, p.OH, nimg, 1) ||
            (u.tma_res && !umma::make_map_rows(&r4, p.res, p.N, p.ldr, p.OW, p.OH, nimg, 1)))
            return MGC_CUDA_OK;
        u.tmC = c4;
        if (u.tma_res) u.tmR = r4;
        u.rt_rows = 1;
        u.rt_per_img = p.OH;
        m_tiles = nimg * p.OH;
        u.res_box_bytes = (uint32_t)p.OW * 128;
    } else if (p.pool_ph > 0) {
        return MGC_CUDA_OK;  // pooling runs only in the phase-split epilogue
    }
    u.m_tiles = (int)m_tiles;
    // CTA pairs (256-row tiles, B planes split between the two CTAs: a third less shared-memory
    // fill per K block) for long-K GEMMs with N tiles of 128 and enough pair tiles to occupy
    // every pair of SMs. Measured on ResNet-50 (batch 256): 8-15 % faster from K = 256 up
    // (without a residual; from K = 512 with one), slower below, no gain for N tiles of 64.
    // MGC_CUDA_PAIR=0 never uses them, =1 whenever the form allows (any size: tests).
    static const int pair_env = [] {
        const char *e = getenv("MGC_CUDA_PAIR");
        return e && e[0] == '0' ? 0 : e && e[0] == '1' ? 1 : 2;
    }();
    // Wide pairs (256 x 256 tiles: per K block a CTA loads 16 KB of A and 32 KB of B for 128 x
    // 256 outputs, a quarter less than the 256 x 128 pair tile) for N >= 256 and long K.
    // MGC_CUDA_WIDE=0 never uses them, =1 the 256 form whenever it is allowed (tests).
    static const int wide_env = [] {
        const char *e = getenv("MGC_CUDA_WIDE");
        return e && e[0] == '0' ? 0 : e && strcmp(e, "192") == 0 ? 3 : e && e[0] == '1' ? 1 : 2;
    }();
    // A wide tile does the work of two 256 x 128 pair tiles in about 0.88 of their time
    // (measured, ResNet-50 3x3 layers), so it is taken when its waves of tiles over the pairs of
    // SMs cost less than the pair form's. Tiles of 256 x 192 (one and a half pair tiles, costed
    // at 1.38) fill the pairs better where N is a multiple of 192 but not of 256 (the 768-wide
    // projections of BERT and GPT-2: 64 tiles in one wave instead of 96 pair tiles in two).
    // MGC_CUDA_WIDE=192 takes the 192 form whenever the form allows.
    if (!strict && pair_env != 0 && wide_env != 0 && (u.im2col == 0 || u.im2col == 1) && bn == 128 && p.N > 128) {
        const long long pair_m = ceil_div(p.M, 2 * umma::BM), wide_n = ceil_div(p.N, 256), w3_n = ceil_div(p.N, 192);
        const bool worth = u.num_kb >= (p.res ? 16 : 8);
        const int clusters = umma::pair_clusters<256, 0>(), clusters3 = umma::pair_clusters<192, 0>();
        const long long waves_w = clusters > 0 ? ceil_div(pair_m * wide_n, clusters) : 0;
        const long long waves_p = clusters > 0 ? ceil_div(pair_m * u.n_tiles, clusters) : 0;
        const long long waves_3 = clusters3 > 0 ? ceil_div(pair_m * w3_n, clusters3) : 0;
        const bool w256 = clusters > 0 && (wide_env == 1 || (worth && pair_m * wide_n >= clusters && 176 * waves_w < 100 * waves_p));
        const bool w192 = !w256 && clusters3 > 0 && clusters3 == clusters &&
                          (wide_env == 3 || (wide_env == 2 && worth && 138 * waves_3 < 100 * waves_p));
        // one weight plane (p.one_plane): boxes of the TF32 part only, one MMA per K step
        const int planes = p.one_plane ? 1 : 2;
        CUtensorMap map3, map1;
        if (w192 && umma::make_map_b(&map3, p.b_umma, p.b_umma_lo, p.N, kp, 96, planes)) {
            u.tmB = map3;
            u.m_tiles = (int)pair_m;
            u.n_tiles = (int)w3_n;
            const int st = p.one_plane ? umma::launch_wide<192, 1>(u, clusters3, stream)
                                       : umma::launch_wide<192>(u, clusters3, stream);
            if (st != MGC_CUDA_OK) return st;
            *taken = 1;
            return MGC_CUDA_OK;
        }
        if (w256 && (!p.one_plane || umma::make_map_b(&map1, p.b_umma, p.b_umma_lo, p.N, kp, 128, 1))) {
            if (p.one_plane) u.tmB = map1;
            u.m_tiles = (int)pair_m;
            u.n_tiles = (int)wide_n;
            const int st = p.one_plane ? umma::launch_wide<256, 1>(u, clusters, stream)
                                       : umma::launch_wide<256>(u, clusters, stream);
            if (st != MGC_CUDA_OK) return st;
            *taken = 1;
            return MGC_CUDA_OK;
        }
    }
    if (!strict && pair_env != 0 && (u.im2col == 0 || u.im2col == 1)) {
        const long long pair_m = ceil_div(p.M, 2 * umma::BM);
        const bool worth = bn == 128 && u.num_kb >= (p.res ? 16 : 8);
        const int clusters = bn == 64 ? umma::pair_clusters<64, 0>() : umma::pair_clusters<128, 0>();
        CUtensorMap plane_map;
        // one weight plane (N tiles of 128): the wide layout, each CTA with 64 rows of B_hi
        const bool sp = p.one_plane && bn == 128;
        if (clusters > 0 && (pair_env == 1 || (worth && pair_m * u.n_tiles >= clusters)) &&
            umma::make_map_b(&plane_map, p.b_umma, p.b_umma_lo, p.N, kp, sp ? 64 : bn, 1)) {
            u.tmB = plane_map;
            u.m_tiles = (int)pair_m;
            const int st = sp ? umma::launch_wide<128, 1>(u, clusters, stream)
                         : bn == 64 ? umma::launch_pair<64>(u, clusters, stream) : umma::launch_pair<128>(u, clusters, stream);
            if (st != MGC_CUDA_OK) return st;
            *taken = 1;
            return MGC_CUDA_OK;
        }
    }
    // Split K when the tiles cover at most half the SMs and K is long (the late layers at batch
    // 1: a 3x3 C512 convolution is 4 tiles of 144 K blocks): K blocks in runs of at least 4, as
    // many runs as fill the SMs; the units leave raw partial tiles in the model's split scratch
    // and split_reduce_kernel sums them and runs the epilogue. Strict mode splits the same way with
    // fp64 partials and an fp64 reduce (split_reduce_f64_kernel). MGC_CUDA_SPLIT=0 never splits.
    static const bool split_env = [] {
        const char *e = getenv("MGC_CUDA_SPLIT");
        return !(e && e[0] == '0');
    }();
    // shortest run of K blocks per unit (MGC_CUDA_SPLIT_KB, default 4)
    static const int split_min_kb = [] {
        const char *e = getenv("MGC_CUDA_SPLIT_KB");
        const int v = e ? atoi(e) : 4;
        return v >= 1 ? v : 4;
    }();
    if (split_env && p.split_ws && (u.im2col == 0 || u.im2col == 1) && u.num_kb >= 2 * split_min_kb && p.gap_hw == 0) {
        const long long tiles = (long long)u.n_tiles * m_tiles;
        const int sms = sm_count();
        if (tiles * 2 <= sms) {
            const long long want = sms / tiles;
            long long kb_per = ceil_div(u.num_kb, want);
            if (kb_per < split_min_kb) kb_per = split_min_kb;
            const long long splits = ceil_div(u.num_kb, kb_per);
            // strict partials are fp64: twice the scratch
            if (splits > 1 && (strict ? 2 : 1) * tiles * splits * umma::BM * bn <= p.split_ws_floats) {
                u.splits = (int)splits;
                u.kb_per = (int)kb_per;
                u.part = p.split_ws;
                u.tma_out = 0;
                u.tma_res = 0;
                u.b_res_bytes = 0;
                const long long units = tiles * splits;
                const int grid = (int)(units < sms ? units : sms);
                // one weight plane: boxes of the TF32 part, one N = BN MMA per K step
                CUtensorMap map1;
                const bool sp = !strict && p.one_plane && umma::make_map_b(&map1, p.b_umma, p.b_umma_lo, p.N, kp, bn, 1);
                if (sp) u.tmB = map1;
                int st = strict ? umma::launch<64, umma::STRICT, 0, 0, 0>(u, grid, stream)
                         : bn == 64 ? (sp ? umma::launch<64, umma::TF32, 0, 0, 0, 0, 1>(u, grid, stream)
                                          : umma::launch<64, umma::TF32, 0, 0, 0>(u, grid, stream))
                                    : (sp ? umma::launch<128, umma::TF32, 0, 0, 0, 0, 1>(u, grid, stream)
                                          : umma::launch<128, umma::TF32, 0, 0, 0>(u, grid, stream));
                if (st != MGC_CUDA_OK) return st;
                const long long outs = (long long)p.M * p.N;
                if (strict)
                    umma::split_reduce_f64_kernel<<<grid_for(outs, 256), 256, 0, stream>>>(
                        reinterpret_cast<const double *>(p.split_ws), (int)splits, u.n_tiles, bn, p.M, p.N, p.c, p.ldc,
                        p.bias, p.res, p.ldr, p.alpha, p.act, p.lo, p.hi);
                else
                    umma::split_reduce_kernel<<<grid_for(outs, 256), 256, 0, stream>>>(
                        p.split_ws, (int)splits, u.n_tiles, bn, p.M, p.N, p.c, p.ldc, p.bias, p.res, p.ldr, p.alpha,
                        p.act, p.lo, p.hi);
                st = check_launch("split_reduce_kernel");
                if (st != MGC_CUDA_OK) return st;
                *taken = 2;  // the split GEMM and its reduce
                return MGC_CUDA_OK;
            }
        }
    }
    // persistent grid: one CTA per SM (the shared-memory footprint allows no more). With a
    // residual, its own staging buffer (MGC_CUDA_SR=0 shares the output's)
    static const bool sr_env = [] {
        const char *e = getenv("MGC_CUDA_SR");
        return !(e && e[0] == '0');
    }();
    int st;
    if (u.im2col == 5) st = umma::launch_phase(u, m_tiles, stream);
    else if (strict) st = umma::launch_best<64, umma::STRICT>(u, m_tiles, stream);
    else if (bn == 64) st = umma::launch_best<64, umma::TF32>(u, m_tiles, stream);
    else if (u.tma_res && sr_env && p.one_plane) {
        // one weight plane: the streamed form with 64-column passes, B boxes of the TF32 part
        CUtensorMap map1;
        if (!umma::make_map_b(&map1, p.b_umma, p.b_umma_lo, p.N, kp, bn, 1)) return MGC_CUDA_OK;
        u.tmB = map1;
        u.b_res_bytes = 0;
        const long long tiles = (long long)u.n_tiles * m_tiles;
        const int sms = sm_count();
        st = umma::launch<128, umma::TF32, 0, 0, 2, 0, 1>(u, (int)(tiles < sms ? tiles : sms), stream);
    } else if (u.tma_res && sr_env) st = umma::launch_best_sr(u, m_tiles, stream);
    else if (p.one_plane && !u.tma_res) {
        // one weight plane without a residual: streamed one-CTA tiles on boxes of the TF32 part
        CUtensorMap map1;
        if (umma::make_map_b(&map1, p.b_umma, p.b_umma_lo, p.N, kp, bn, 1)) {
            u.tmB = map1;
            const long long tiles = (long long)u.n_tiles * m_tiles;
            const int sms = sm_count();
            st = umma::launch<128, umma::TF32, 0, 0, 0, 0, 1>(u, (int)(tiles < sms ? tiles : sms), stream);
        } else {
            st = umma::launch_best<128, umma::TF32>(u, m_tiles, stream);
        }
    } else st = umma::launch_best<128, umma::TF32>(u, m_tiles, stream);
    if (st != MGC_CUDA_OK) return st;
    *taken = 1;
    return MGC_CUDA_OK;
}

}  // namespace mgc
