// Shared helpers of libmgc_cuda: error reporting, status codes, element types.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>
#include <mutex>
#include <set>
#include <string>
#include <utility>

#include "mgc_cuda.h"

namespace mgc {

// Text of the last error, per host thread (mgc_cuda_last_error).
inline std::string &last_error() {
    static thread_local std::string text;
    return text;
}

inline int fail(int status, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    last_error() = buf;
    return status;
}

inline int cuda_fail(cudaError_t err, const char *what) {
    return fail(MGC_CUDA_CUDA_ERROR + (int)err, "%s: %s (%s)", what, cudaGetErrorString(err),
                cudaGetErrorName(err));
}

#define MGC_CHECK_CUDA(call)                                                                 \
    do {                                                                                     \
        cudaError_t mgc_err_ = (call);                                                       \
        if (mgc_err_ != cudaSuccess) return ::mgc::cuda_fail(mgc_err_, #call);               \
    } while (0)

#define MGC_CHECK(call)                                                                      \
    do {                                                                                     \
        int mgc_st_ = (call);                                                                \
        if (mgc_st_ != MGC_CUDA_OK) return mgc_st_;                                          \
    } while (0)

// After a kernel launch: report a launch configuration error.
inline int check_launch(const char *what) {
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return cuda_fail(err, what);
    return MGC_CUDA_OK;
}

inline int dtype_size(int dt) {
    switch (dt) {
    case MGC_F32: return 4;
    case MGC_F64: return 8;
    case MGC_I64: return 8;
    case MGC_I32: return 4;
    case MGC_I8: return 1;
    case MGC_U8: return 1;
    case MGC_BOOL: return 1;
    default: return 0;
    }
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Number of SMs of the current device (cached per device ordinal).
inline int sm_count() {
    static int counts[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return 148;
    }
    if (!counts[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = 148;
        }
        counts[dev] = n;
    }
    return counts[dev];
}

// Grid size for a grid-stride loop over `n` items: a multiple of the SM count (148 on B200),
// capped, never zero.
// Let `kernel` launch with up to the device's opt-in maximum of dynamic shared memory, once per
// device. The ceiling goes to the maximum rather than to each launch's own size: a kernel whose
// launches need different sizes (a B panel, a second output staging tile) would otherwise be
// left with the last launch's ceiling, below what an earlier launch captured into a CUDA Graph
// needs when that node is launched again on its own (as a profiler replays graph nodes).
inline int raise_smem_ceiling(const void *kernel) {
    static std::mutex mu;
    static std::set<std::pair<const void *, int>> done;
    int dev = 0;
    MGC_CHECK_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> guard(mu);
    if (done.count({kernel, dev})) return MGC_CUDA_OK;
    int optin = 0;
    MGC_CHECK_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    cudaFuncAttributes fa;
    MGC_CHECK_CUDA(cudaFuncGetAttributes(&fa, kernel));
    MGC_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        optin - (int)fa.sharedSizeBytes));
    done.insert({kernel, dev});
    return MGC_CUDA_OK;
}

inline unsigned grid_for(int64_t n, int threads, int sms = 148, int per_sm = 8) {
    int64_t blocks = ceil_div(n, threads);
    int64_t cap = (int64_t)sms * per_sm;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (unsigned)blocks;
}

}  // namespace mgc
