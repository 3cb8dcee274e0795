// libmgc_cuda: the C ABI declared in include/mgc_cuda.h.
//
// A handle (Model) owns, on one device: the planner's arena (one cudaMalloc of
// MemoryPlan.arena_bytes, so every value keeps the offset the reference planner gave it), the
// resident constant blob, one device buffer per graph input and output, a status word for
// Gather range errors, a non-blocking stream and a CUDA Graph holding the whole launch list.
// mgc_cuda_run replays that graph between the host<->device copies; nothing is allocated after
// mgc_cuda_create returns.
#include <cuda_runtime.h>
#include <string.h>

#include <atomic>
#include <memory>
#include <mutex>
#include <vector>

#include "launch.cuh"
#include "mgc_cuda.h"

using namespace mgc;

namespace {

// split-K scratch per model: 32 MiB of partial tiles (GEMMs with fewer tiles than SMs)
constexpr long long SPLIT_WS_FLOATS = 8ll << 20;

struct Model {
    int device = 0;
    cudaStream_t stream = nullptr;
    char *arena = nullptr;
    int64_t arena_bytes = 0;
    char *weights = nullptr;
    int64_t weights_bytes = 0;
    char *workspace = nullptr;
    int64_t workspace_bytes = 0;
    std::vector<char *> inputs, outputs;
    std::vector<int64_t> in_bytes, out_bytes;
    std::vector<mgc_cuda_launch> launches;
    std::vector<int64_t> aux;
    int *status_dev = nullptr;
    int *status_host = nullptr;
    float *split_ws = nullptr;  // split-K partial tiles
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    int kernel_launches = 0;
    std::vector<int32_t> gemm_paths;  // MGC_CUDA_PATH_* per launch record
    // input-upload overlap (mgc_cuda_set_input_chunks): a copy stream, one event per slice and
    // the graph whose prefix runs slice by slice
    int chunks = 0, prefix = 0;
    int64_t images = 0;
    std::vector<mgc_cuda_chunk> chunk_descs;
    cudaStream_t copy_stream = nullptr;
    std::vector<cudaEvent_t> slice_ready;
    cudaEvent_t stream_done = nullptr;  // the copy stream starts after the stream's earlier work
    cudaGraph_t graph_host = nullptr;
    cudaGraphExec_t exec_host = nullptr;

    Bases bases() const {
        Bases b;
        b.arena = arena;
        b.weights = weights;
        b.workspace = workspace;
        b.inputs = &inputs;
        b.outputs = &outputs;
        b.split_ws = split_ws;
        b.split_ws_floats = split_ws ? SPLIT_WS_FLOATS : 0;
        return b;
    }

    // Record k's kernel count and GEMM path (the worst path seen, when it runs more than once).
    void note(size_t k, const LaunchInfo &info, int *kernels) {
        *kernels += info.kernels;
        if (gemm_paths.size() < launches.size()) gemm_paths.assign(launches.size(), MGC_CUDA_PATH_NONE);
        if (info.gemm_path > gemm_paths[k]) gemm_paths[k] = info.gemm_path;
    }

    // Enqueue the whole launch list on `stream` (also used under graph capture).
    int enqueue(int *kernels) {
        MGC_CHECK_CUDA(cudaMemsetAsync(status_dev, 0, sizeof(int), stream));
        Bases b = bases();
        for (size_t k = 0; k < launches.size(); ++k) {
            LaunchInfo info;
            MGC_CHECK(launch_record(launches[k], aux.data(), (int64_t)aux.size(), b, status_dev, stream, &info));
            note(k, info, kernels);
        }
        return MGC_CUDA_OK;
    }

    // The prefix once per input slice (each after its slice's copy), then the rest once.
    int enqueue_sliced(int *kernels) {
        MGC_CHECK_CUDA(cudaMemsetAsync(status_dev, 0, sizeof(int), stream));
        Bases b = bases();
        const int64_t per = images / chunks;
        for (int j = 0; j < chunks; ++j) {
            MGC_CHECK_CUDA(cudaStreamWaitEvent(stream, slice_ready[(size_t)j], cudaEventWaitExternal));
            for (int r = 0; r < prefix; ++r) {
                mgc_cuda_launch L = launches[(size_t)r];
                for (const mgc_cuda_chunk &d : chunk_descs) {
                    if (d.launch != r) continue;
                    if (d.what == 0) {
                        L.r[d.slot].offset += (int64_t)j * per * d.per_image;
                    } else if (d.what == 2) {  // a buffer only the prefix reads, in one slice's
                                               // private region (the same for every slice)
                        L.r[d.slot].space = MGC_SPACE_WORKSPACE;
                        L.r[d.slot].index = 0;
                        L.r[d.slot].offset = d.per_image;
                    } else {
                        L.i[d.slot] = d.per_image * per;
                    }
                }
                LaunchInfo info;
                MGC_CHECK(launch_record(L, aux.data(), (int64_t)aux.size(), b, status_dev, stream, &info));
                note((size_t)r, info, kernels);
            }
        }
        for (size_t r = (size_t)prefix; r < launches.size(); ++r) {
            LaunchInfo info;
            MGC_CHECK(launch_record(launches[r], aux.data(), (int64_t)aux.size(), b, status_dev, stream, &info));
            note(r, info, kernels);
        }
        return MGC_CUDA_OK;
    }

    void release_chunks() {
        if (exec_host) cudaGraphExecDestroy(exec_host);
        if (graph_host) cudaGraphDestroy(graph_host);
        if (copy_stream) cudaStreamSynchronize(copy_stream);
        for (cudaEvent_t e : slice_ready) cudaEventDestroy(e);
        if (stream_done) cudaEventDestroy(stream_done);
        if (copy_stream) cudaStreamDestroy(copy_stream);
        exec_host = nullptr; graph_host = nullptr; copy_stream = nullptr; stream_done = nullptr;
        slice_ready.clear();
        chunks = 0; prefix = 0;
    }

    void release() {
        if (device >= 0) cudaSetDevice(device);
        release_chunks();
        if (exec) cudaGraphExecDestroy(exec);
        if (graph) cudaGraphDestroy(graph);
        if (stream) cudaStreamSynchronize(stream);
        for (char *p : inputs) cudaFree(p);
        for (char *p : outputs) cudaFree(p);
        if (arena) cudaFree(arena);
        if (weights) cudaFree(weights);
        if (workspace) cudaFree(workspace);
        if (status_dev) cudaFree(status_dev);
        if (status_host) cudaFreeHost(status_host);
        if (split_ws) cudaFree(split_ws);
        if (stream) cudaStreamDestroy(stream);
        exec = nullptr; graph = nullptr; stream = nullptr; arena = nullptr; weights = nullptr; workspace = nullptr;
        status_dev = nullptr; status_host = nullptr; split_ws = nullptr;
        inputs.clear(); outputs.clear();
    }
};

int alloc_bytes(char **p, int64_t n) {
    // at least 256 bytes so every buffer is a valid, aligned device address
    size_t bytes = (size_t)(n > 256 ? n : 256);
    cudaError_t err = cudaMalloc((void **)p, bytes);
    if (err != cudaSuccess) return cuda_fail(err, "cudaMalloc");
    return MGC_CUDA_OK;
}

int create(Model &m, const mgc_cuda_launch *launches, int n_launches, const int64_t *aux,
           int64_t aux_len, const void *weights_host, int64_t weights_bytes, int64_t arena_bytes,
           int64_t workspace_bytes, const mgc_cuda_io *inputs, int n_inputs, const mgc_cuda_io *outputs,
           int n_outputs, int device) {
    if (n_launches < 0 || aux_len < 0 || weights_bytes < 0 || arena_bytes < 0 || workspace_bytes < 0 || n_inputs < 0 ||
        n_outputs < 0 || (n_launches && !launches) || (aux_len && !aux) ||
        (weights_bytes && !weights_host))
        return fail(MGC_CUDA_BAD_ARGUMENT, "mgc_cuda_create: invalid arguments");
    m.device = device;
    MGC_CHECK_CUDA(cudaSetDevice(device));
    MGC_CHECK_CUDA(cudaStreamCreateWithFlags(&m.stream, cudaStreamNonBlocking));
    m.launches.assign(launches, launches + n_launches);
    m.aux.assign(aux, aux + aux_len);
    m.arena_bytes = arena_bytes;
    m.weights_bytes = weights_bytes;
    MGC_CHECK(alloc_bytes(&m.arena, arena_bytes));
    MGC_CHECK(alloc_bytes(&m.weights, weights_bytes));
    if (workspace_bytes > 0) {
        MGC_CHECK(alloc_bytes(&m.workspace, workspace_bytes));
        m.workspace_bytes = workspace_bytes;
    }
    if (weights_bytes)
        MGC_CHECK_CUDA(cudaMemcpy(m.weights, weights_host, (size_t)weights_bytes, cudaMemcpyHostToDevice));
    for (int k = 0; k < n_inputs; ++k) {
        char *p = nullptr;
        MGC_CHECK(alloc_bytes(&p, inputs[k].nbytes));
        m.inputs.push_back(p);
        m.in_bytes.push_back(inputs[k].nbytes);
    }
    for (int k = 0; k < n_outputs; ++k) {
        char *p = nullptr;
        MGC_CHECK(alloc_bytes(&p, outputs[k].nbytes));
        m.outputs.push_back(p);
        m.out_bytes.push_back(outputs[k].nbytes);
    }
    MGC_CHECK_CUDA(cudaMalloc((void **)&m.status_dev, sizeof(int)));
    MGC_CHECK_CUDA(cudaMallocHost((void **)&m.status_host, sizeof(int)));
    MGC_CHECK_CUDA(cudaMalloc((void **)&m.split_ws, (size_t)SPLIT_WS_FLOATS * sizeof(float)));
    // capture the schedule into one CUDA Graph
    MGC_CHECK_CUDA(cudaStreamBeginCapture(m.stream, cudaStreamCaptureModeThreadLocal));
    int kernels = 0;
    int st = m.enqueue(&kernels);
    cudaGraph_t graph = nullptr;
    cudaError_t err = cudaStreamEndCapture(m.stream, &graph);
    if (st != MGC_CUDA_OK) {
        if (graph) cudaGraphDestroy(graph);
        return st;
    }
    if (err != cudaSuccess) return cuda_fail(err, "cudaStreamEndCapture");
    m.graph = graph;
    m.kernel_launches = kernels;
    MGC_CHECK_CUDA(cudaGraphInstantiate(&m.exec, m.graph, 0));
    MGC_CHECK_CUDA(cudaGraphUpload(m.exec, m.stream));
    MGC_CHECK_CUDA(cudaStreamSynchronize(m.stream));
    return MGC_CUDA_OK;
}

int finish(Model &m) {
    MGC_CHECK_CUDA(cudaMemcpyAsync(m.status_host, m.status_dev, sizeof(int), cudaMemcpyDeviceToHost, m.stream));
    MGC_CHECK_CUDA(cudaStreamSynchronize(m.stream));
    const int status = *m.status_host;
    if (status == MGC_CUDA_GATHER_OOB)
        return fail(MGC_CUDA_GATHER_OOB, "compiled model reported an out-of-range Gather index");
    if (status == MGC_CUDA_TIMEOUT)
        return fail(MGC_CUDA_TIMEOUT, "a tensor-core kernel gave up on a bounded wait (results invalid)");
    if (status != 0) return fail(status, "device status %d", status);
    return MGC_CUDA_OK;
}

}  // namespace

extern "C" {

int mgc_cuda_abi_version(void) { return MGC_CUDA_ABI_VERSION; }

const char *mgc_cuda_last_error(void) { return last_error().c_str(); }

int mgc_cuda_device_supported(int device) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return prop.major == 10 ? 1 : 0;
}

int mgc_cuda_create(const mgc_cuda_launch *launches, int n_launches, const int64_t *aux,
                    int64_t aux_len, const void *weights_host, int64_t weights_bytes,
                    int64_t arena_bytes, int64_t workspace_bytes, const mgc_cuda_io *inputs,
                    int n_inputs, const mgc_cuda_io *outputs, int n_outputs, int device,
                    void **handle) {
    last_error().clear();
    if (!handle) return fail(MGC_CUDA_BAD_ARGUMENT, "mgc_cuda_create: handle is NULL");
    *handle = nullptr;
    std::unique_ptr<Model> m(new Model());
    int st = create(*m, launches, n_launches, aux, aux_len, weights_host, weights_bytes, arena_bytes,
                    workspace_bytes, inputs, n_inputs, outputs, n_outputs, device);
    if (st != MGC_CUDA_OK) {
        std::string msg = last_error();
        m->release();
        last_error() = msg;
        return st;
    }
    *handle = m.release();
    return MGC_CUDA_OK;
}

int mgc_cuda_set_input_chunks(void *handle, int chunks, int prefix, int64_t images, const mgc_cuda_chunk *descs,
                              int n_descs) {
    last_error().clear();
    Model *m = (Model *)handle;
    if (!m) return fail(MGC_CUDA_BAD_ARGUMENT, "mgc_cuda_set_input_chunks: handle is NULL");
    if (chunks < 2 || chunks > 16 || images <= 0 || images % chunks || prefix < 0 ||
        prefix > (int)m->launches.size() || n_descs < 0 || (n_descs && !descs) || m->inputs.size() != 1 ||
        m->in_bytes[0] % images)
        return fail(MGC_CUDA_BAD_ARGUMENT, "mgc_cuda_set_input_chunks: invalid arguments");
    for (int k = 0; k < n_descs; ++k) {
        const mgc_cuda_chunk &d = descs[k];
        if (d.launch < 0 || d.launch >= prefix || d.what < 0 || d.what > 2 || d.slot < 0 ||
            d.slot >= (d.what == 1 ? MGC_LAUNCH_INTS : MGC_LAUNCH_REFS) || d.per_image < 0 ||
            (d.what == 2 && d.per_image >= m->workspace_bytes))
            return fail(MGC_CUDA_BAD_ARGUMENT, "mgc_cuda_set_input_chunks: descriptor %d is invalid", k);
    }
    MGC_CHECK_CUDA(cudaSetDevice(m->device));
    MGC_CHECK_CUDA(cudaStreamSynchronize(m->stream));
    m->release_chunks();
    m->chunks = chunks;
    m->prefix = prefix;
    m->images = images;
    m->chunk_descs.assign(descs, descs + n_descs);
    MGC_CHECK_CUDA(cudaStreamCreateWithFlags(&m->copy_stream, cudaStreamNonBlocking));
    MGC_CHECK_CUDA(cudaEventCreateWithFlags(&m->stream_done, cudaEventDisableTiming));
    for (int j = 0; j < chunks; ++j) {
        cudaEvent_t e = nullptr;
        MGC_CHECK_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        m->slice_ready.push_back(e);
    }
    MGC_CHECK_CUDA(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    int kernels = 0;  // the sliced graph's launches (mgc_cuda_launch_count reports the one-pass graph's)
    const int st = m->enqueue_sliced(&kernels);
    cudaGraph_t graph = nullptr;
    const cudaError_t err = cudaStreamEndCapture(m->stream, &graph);
    if (st != MGC_CUDA_OK || err != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        const std::string msg = last_error();
        m->release_chunks();
        if (st != MGC_CUDA_OK) return fail(st, "%s", msg.c_str());
        return cuda_fail(err, "cudaStreamEndCapture");
    }
    m->graph_host = graph;
    if (cudaGraphInstantiate(&m->exec_host, m->graph_host, 0) != cudaSuccess ||
        cudaGraphUpload(m->exec_host, m->stream) != cudaSuccess || cudaStreamSynchronize(m->stream) != cudaSuccess) {
        const cudaError_t e = cudaGetLastError();
        m->release_chunks();
        return cuda_fail(e, "instantiating the sliced graph");
    }
    return MGC_CUDA_OK;
}

int mgc_cuda_run(void *handle, const void *const *inputs_host, void *const *outputs_host) {
    last_error().clear();
    Model *m = (Model *)handle;
    if (!m) return fail(MGC_CUDA_BAD_ARGUMENT, "mgc_cuda_run: handle is NULL");
    MGC_CHECK_CUDA(cudaSetDevice(m->device));
    for (size_t k = 0; k < m->inputs.size(); ++k)
        if (!inputs_host || !inputs_host[k]) return fail(MGC_CUDA_BAD_ARGUMENT, "input %zu is NULL", k);
    if (m->exec_host) {
        // slice by slice on the copy stream; the sliced graph's prefix waits for each slice
        const size_t slice = (size_t)(m->in_bytes[0] / m->chunks);
        // no slice may land while work queued earlier on the stream still reads the input
        MGC_CHECK_CUDA(cudaEventRecord(m->stream_done, m->stream));
        MGC_CHECK_CUDA(cudaStreamWaitEvent(m->copy_stream, m->stream_done, 0));
        for (int j = 0; j < m->chunks; ++j) {
            MGC_CHECK_CUDA(cudaMemcpyAsync(m->inputs[0] + (size_t)j * slice,
                                           (const char *)inputs_host[0] + (size_t)j * slice, slice,
                                           cudaMemcpyHostToDevice, m->copy_stream));
            MGC_CHECK_CUDA(cudaEventRecord(m->slice_ready[(size_t)j], m->copy_stream));
        }
        MGC_CHECK_CUDA(cudaGraphLaunch(m->exec_host, m->stream));
    } else {
        for (size_t k = 0; k < m->inputs.size(); ++k) {
            if (m->in_bytes[k])
                MGC_CHECK_CUDA(cudaMemcpyAsync(m->inputs[k], inputs_host[k], (size_t)m->in_bytes[k],
                                               cudaMemcpyHostToDevice, m->stream));
        }
        MGC_CHECK_CUDA(cudaGraphLaunch(m->exec, m->stream));
    }
    for (size_t k = 0; k < m->outputs.size(); ++k) {
        if (!outputs_host || !outputs_host[k]) return fail(MGC_CUDA_BAD_ARGUMENT, "output %zu is NULL", k);
        if (m->out_bytes[k])
            MGC_CHECK_CUDA(cudaMemcpyAsync(outputs_host[k], m->outputs[k], (size_t)m->out_bytes[k],
                                           cudaMemcpyDeviceToHost, m->stream));
    }
    return finish(*m);
}

int mgc_cuda_run_device(void *handle, int sync) {
    last_error().clear();
    Model *m = (Model *)handle;
    if (!m) return fail(MGC_CUDA_BAD_ARGUMENT, "mgc_cuda_run_device: handle is NULL");
    MGC_CHECK_CUDA(cudaSetDevice(m->device));
    MGC_CHECK_CUDA(cudaGraphLaunch(m->exec, m->stream));
    if (!sync) return MGC_CUDA_OK;
    return finish(*m);
}

void *mgc_cuda_input_ptr(void *handle, int i) {
    Model *m = (Model *)handle;
    if (!m || i < 0 || i >= (int)m->inputs.size()) return nullptr;
    return m->inputs[i];
}

void *mgc_cuda_output_ptr(void *handle, int i) {
    Model *m = (Model *)handle;
    if (!m || i < 0 || i >= (int)m->outputs.size()) return nullptr;
    return m->outputs[i];
}

void *mgc_cuda_stream(void *handle) {
    Model *m = (Model *)handle;
    return m ? (void *)m->stream : nullptr;
}

int mgc_cuda_launch_count(void *handle) {
    Model *m = (Model *)handle;
    return m ? m->kernel_launches : -1;
}

int mgc_cuda_gemm_paths(void *handle, int32_t *per_record, int n) {
    last_error().clear();
    Model *m = (Model *)handle;
    if (!m || n < 0 || (n > 0 && !per_record)) return fail(MGC_CUDA_BAD_ARGUMENT, "mgc_cuda_gemm_paths: bad arguments");
    for (int k = 0; k < n; ++k)
        per_record[k] = (size_t)k < m->gemm_paths.size() ? m->gemm_paths[(size_t)k] : MGC_CUDA_PATH_NONE;
    return MGC_CUDA_OK;
}

int64_t mgc_cuda_arena_bytes(void *handle) {
    Model *m = (Model *)handle;
    return m ? m->arena_bytes : -1;
}

int64_t mgc_cuda_weights_bytes(void *handle) {
    Model *m = (Model *)handle;
    return m ? m->weights_bytes : -1;
}

int mgc_cuda_profile(void *handle, double *per_node_ms, int n) {
    last_error().clear();
    Model *m = (Model *)handle;
    if (!m || (n > 0 && !per_node_ms)) return fail(MGC_CUDA_BAD_ARGUMENT, "mgc_cuda_profile: bad arguments");
    MGC_CHECK_CUDA(cudaSetDevice(m->device));
    for (int k = 0; k < n; ++k) per_node_ms[k] = 0.0;
    const size_t L = m->launches.size();
    std::vector<cudaEvent_t> ev(2 * L, nullptr);
    int st = MGC_CUDA_OK;
    for (auto &e : ev) {
        if (cudaEventCreate(&e) != cudaSuccess) { st = cuda_fail(cudaGetLastError(), "cudaEventCreate"); break; }
    }
    if (st == MGC_CUDA_OK) st = cudaMemsetAsync(m->status_dev, 0, sizeof(int), m->stream) == cudaSuccess
                                    ? MGC_CUDA_OK : cuda_fail(cudaGetLastError(), "cudaMemsetAsync");
    Bases b = m->bases();
    for (size_t k = 0; k < L && st == MGC_CUDA_OK; ++k) {
        cudaEventRecord(ev[2 * k], m->stream);
        st = launch_record(m->launches[k], m->aux.data(), (int64_t)m->aux.size(), b, m->status_dev, m->stream,
                           nullptr);
        cudaEventRecord(ev[2 * k + 1], m->stream);
    }
    if (st == MGC_CUDA_OK) st = finish(*m);
    if (st == MGC_CUDA_OK) {
        for (size_t k = 0; k < L; ++k) {
            float ms = 0.0f;
            cudaEventElapsedTime(&ms, ev[2 * k], ev[2 * k + 1]);
            int node = m->launches[k].node;
            if (node >= 0 && node < n) per_node_ms[node] += ms;
        }
    }
    for (auto &e : ev)
        if (e) cudaEventDestroy(e);
    return st;
}

void mgc_cuda_destroy(void *handle) {
    Model *m = (Model *)handle;
    if (!m) return;
    m->release();
    delete m;
}

int mgc_cuda_execute(const mgc_cuda_launch *launches, int n, const int64_t *aux, int64_t aux_len,
                     int *status_dev, void *stream) {
    last_error().clear();
    if (n < 0 || (n && !launches)) return fail(MGC_CUDA_BAD_ARGUMENT, "mgc_cuda_execute: bad arguments");
    Bases b;  // raw device pointers only
    for (int k = 0; k < n; ++k)
        MGC_CHECK(launch_record(launches[k], aux, aux_len, b, status_dev, (cudaStream_t)stream, nullptr));
    return MGC_CUDA_OK;
}

int mgc_cuda_gemm(int M, int N, int K, int batch, const float *a, int64_t a_rs, int64_t a_cs,
                  int64_t a_bstride, const float *b, int64_t b_rs, int64_t b_cs, int64_t b_bstride,
                  float *c, int64_t ldc, int64_t c_bstride, float alpha, const float *bias,
                  int bias_mode, const float *res, int64_t ldr, int64_t r_bstride, float beta,
                  int act, float lo, float hi, int precision, void *stream) {
    last_error().clear();
    if (M < 0 || N < 0 || K < 0 || batch < 0 || !a || !b || !c)
        return fail(MGC_CUDA_BAD_ARGUMENT, "mgc_cuda_gemm: bad arguments");
    GemmParams p{};
    p.M = M; p.N = N; p.K = K;
    p.nb = 1; p.bdims[0] = batch;
    p.a_bs[0] = a_bstride; p.b_bs[0] = b_bstride; p.c_bs[0] = c_bstride; p.r_bs[0] = r_bstride;
    p.a_kind = MGC_STRIDED; p.a_rs = a_rs; p.a_cs = a_cs; p.a = a;
    p.b_kind = MGC_STRIDED; p.b_rs = b_rs; p.b_cs = b_cs; p.b = b;
    p.c = c; p.ldc = ldc;
    p.alpha = alpha; p.beta = beta; p.bias = bias; p.bias_mode = bias ? bias_mode : 0;
    p.res = res; p.ldr = ldr; p.act = act; p.lo = lo; p.hi = hi; p.precision = precision;
    if (batch == 1) p.nb = 0;
    if (precision == MGC_PREC_FP32) return launch_gemm_simt(p, (cudaStream_t)stream);
    if (precision == MGC_PREC_3XTF32)
        return fail(MGC_CUDA_UNSUPPORTED, "mgc_cuda_gemm: 3xTF32 needs constant weights prepared by "
                                          "mgc_cuda_create; use MGC_PREC_FP32 for exact fp32");
    if (precision != MGC_PREC_TF32) return fail(MGC_CUDA_BAD_ARGUMENT, "mgc_cuda_gemm: precision %d", precision);
    if (M == 0 || N == 0 || batch == 0) return MGC_CUDA_OK;
    int taken = 0;
    MGC_CHECK(try_gemm_umma_dyn(p, (cudaStream_t)stream, &taken));
    if (!taken)
        return fail(MGC_CUDA_UNSUPPORTED,
                    "mgc_cuda_gemm: TF32 runs on the tensor cores only with K-major A and B (a_cs == 1, b_rs == 1), "
                    "16-byte aligned bases and strides, K and N multiples of 4, bias per column, and no epilogue "
                    "on batched products; use MGC_PREC_FP32 for exact fp32 on the CUDA cores");
    return MGC_CUDA_OK;
}

int mgc_cuda_conv_nhwc(int N, int H, int W, int C, int KH, int KW, int SH, int SW, int DH, int DW,
                       int PT, int PL, int OH, int OW, int CO, const float *x, const float *w,
                       const float *bias, const float *res, int act, float lo, float hi,
                       float *y, int precision, void *stream) {
    last_error().clear();
    if (!x || !w || !y || N < 0 || OH < 0 || OW < 0 || CO < 0)
        return fail(MGC_CUDA_BAD_ARGUMENT, "mgc_cuda_conv_nhwc: bad arguments");
    if (precision == MGC_PREC_TF32 || precision == MGC_PREC_3XTF32)
        return fail(MGC_CUDA_UNSUPPORTED, "mgc_cuda_conv_nhwc: TF32 / 3xTF32 need the K-major weight layout that "
                                          "mgc_cuda_create prepares; HWIO weights run with MGC_PREC_FP32");
    if (precision != MGC_PREC_FP32) return fail(MGC_CUDA_BAD_ARGUMENT, "mgc_cuda_conv_nhwc: precision %d", precision);
    GemmParams p{};
    p.M = N * OH * OW; p.N = CO; p.K = KH * KW * C;
    p.nb = 0;
    p.a_kind = MGC_CONV_NHWC; p.a = x;
    p.H = H; p.W = W; p.C = C; p.KH = KH; p.KW = KW; p.SH = SH; p.SW = SW; p.DH = DH; p.DW = DW;
    p.PT = PT; p.PL = PL; p.OH = OH; p.OW = OW; p.c_off = 0; p.cg = C;
    // HWIO weights are row-major [KH*KW*C, CO]: element (k, n) at w[k*CO + n]
    p.b_kind = MGC_STRIDED; p.b = w; p.b_rs = CO; p.b_cs = 1;
    p.c = y; p.ldc = CO;
    p.alpha = 1.0f; p.beta = 1.0f; p.bias = bias; p.bias_mode = bias ? 1 : 0;
    p.res = res; p.ldr = CO; p.act = act; p.lo = lo; p.hi = hi; p.precision = precision;
    return launch_gemm_simt(p, (cudaStream_t)stream);
}

int mgc_cuda_depthwise_nhwc(int N, int H, int W, int C, int KH, int KW, int SH, int SW, int DH,
                            int DW, int PT, int PL, int OH, int OW, const float *x, const float *w,
                            const float *bias, const float *res, int act, float lo, float hi,
                            float *y, void *stream) {
    last_error().clear();
    mgc_cuda_launch L;
    memset(&L, 0, sizeof L);
    L.kind = MGC_K_DEPTHWISE;
    int64_t v[16] = {N, H, W, C, KH, KW, SH, SW, DH, DW, PT, PL, OH, OW, 1, act};
    for (int k = 0; k < 16; ++k) L.i[k] = v[k];
    L.f[0] = lo; L.f[1] = hi;
    const void *ptrs[5] = {x, w, bias, res, y};
    for (int k = 0; k < 5; ++k) {
        L.r[k].space = ptrs[k] ? MGC_SPACE_RAW : MGC_SPACE_NONE;
        L.r[k].offset = (int64_t)(uintptr_t)ptrs[k];
    }
    return mgc_cuda_execute(&L, 1, nullptr, 0, nullptr, stream);
}

int mgc_cuda_pool_nhwc(int is_max, int N, int H, int W, int C, int KH, int KW, int SH, int SW,
                       int DH, int DW, int PT, int PL, int PB, int PR, int OH, int OW,
                       int count_include_pad, const float *x, float *y, void *stream) {
    last_error().clear();
    mgc_cuda_launch L;
    memset(&L, 0, sizeof L);
    L.kind = MGC_K_POOL;
    int64_t v[19] = {is_max, N, H, W, C, KH, KW, SH, SW, DH, DW, PT, PL, PB, PR, OH, OW, count_include_pad, 1};
    for (int k = 0; k < 19; ++k) L.i[k] = v[k];
    L.r[0] = {MGC_SPACE_RAW, 0, (int64_t)(uintptr_t)x};
    L.r[1] = {MGC_SPACE_RAW, 0, (int64_t)(uintptr_t)y};
    return mgc_cuda_execute(&L, 1, nullptr, 0, nullptr, stream);
}

int mgc_cuda_reduce_mid(int is_max, int64_t outer, int64_t n, int64_t inner, const float *x,
                        float *y, void *stream) {
    last_error().clear();
    mgc_cuda_launch L;
    memset(&L, 0, sizeof L);
    L.kind = MGC_K_REDUCE_MID;
    L.i[0] = is_max; L.i[1] = outer; L.i[2] = n; L.i[3] = inner;
    L.r[0] = {MGC_SPACE_RAW, 0, (int64_t)(uintptr_t)x};
    L.r[1] = {MGC_SPACE_RAW, 0, (int64_t)(uintptr_t)y};
    return mgc_cuda_execute(&L, 1, nullptr, 0, nullptr, stream);
}

int mgc_cuda_softmax(int64_t outer, int64_t n, int64_t inner, const float *x, float *y,
                     int log_softmax, void *stream) {
    last_error().clear();
    mgc_cuda_launch L;
    memset(&L, 0, sizeof L);
    L.kind = MGC_K_SOFTMAX;
    L.i[0] = outer; L.i[1] = n; L.i[2] = inner; L.i[3] = log_softmax;
    L.r[0] = {MGC_SPACE_RAW, 0, (int64_t)(uintptr_t)x};
    L.r[1] = {MGC_SPACE_RAW, 0, (int64_t)(uintptr_t)y};
    return mgc_cuda_execute(&L, 1, nullptr, 0, nullptr, stream);
}

int mgc_cuda_layer_norm(int64_t rows, int64_t cols, const float *x, const float *scale,
                        const float *bias, float eps, float *y, void *stream) {
    last_error().clear();
    mgc_cuda_launch L;
    memset(&L, 0, sizeof L);
    L.kind = MGC_K_LAYER_NORM;
    L.i[0] = rows; L.i[1] = cols;
    L.f[0] = eps;
    const void *ptrs[4] = {x, scale, bias, y};
    for (int k = 0; k < 4; ++k) {
        L.r[k].space = ptrs[k] ? MGC_SPACE_RAW : MGC_SPACE_NONE;
        L.r[k].offset = (int64_t)(uintptr_t)ptrs[k];
    }
    return mgc_cuda_execute(&L, 1, nullptr, 0, nullptr, stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Convolution without allocation: its im2col scratch is this fixed device array, shared by every
// call (see mgc_cuda_conv_nhwc_noalloc in mgc_cuda.h for who needs it and the limits).
// ---------------------------------------------------------------------------------------------
static __device__ __align__(256) float g_noalloc_scratch[MGC_CUDA_NOALLOC_SCRATCH_BYTES / sizeof(float)];

namespace {

// Device address of g_noalloc_scratch on the current device, looked up once per device (with that
// device current) and published atomically, so host threads making their first call at once
// agree on it; a failed lookup is retried by the next call. In host code the array's name is only
// a stand-in for the symbol, never a usable device pointer.
int noalloc_scratch(float **out) {
    static std::atomic<float *> addr[64];
    static std::mutex lookup;
    int dev = 0;
    MGC_CHECK_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(MGC_CUDA_UNSUPPORTED, "device ordinal %d out of range", dev);
    float *known = addr[dev].load(std::memory_order_acquire);
    if (!known) {
        std::lock_guard<std::mutex> guard(lookup);
        known = addr[dev].load(std::memory_order_acquire);
        if (!known) {
            void *p = nullptr;
            MGC_CHECK_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
            known = static_cast<float *>(p);
            addr[dev].store(known, std::memory_order_release);
        }
    }
    *out = known;
    return MGC_CUDA_OK;
}

}  // namespace

extern "C" int mgc_cuda_conv_nhwc_noalloc(int N, int H, int W, int C, int KH, int KW, int SH, int SW,
                                          int DH, int DW, int PT, int PL, int OH, int OW, int CO,
                                          const float *x, const float *w, const float *bias,
                                          const float *res, int act, float lo, float hi, float *y,
                                          void *stream) {
    last_error().clear();
    if (!x || !w || !y || N < 0 || H <= 0 || W <= 0 || C <= 0 || KH <= 0 || KW <= 0 || SH <= 0 || SW <= 0 ||
        DH <= 0 || DW <= 0 || OH < 0 || OW < 0 || CO < 0)
        return fail(MGC_CUDA_BAD_ARGUMENT, "mgc_cuda_conv_nhwc_noalloc: bad arguments");
    const long long rows = (long long)N * OH * OW;
    const long long kreal = (long long)KH * KW * C;
    const long long kp = (kreal + 3) / 4 * 4;
    const long long bytes = rows * kp * (long long)sizeof(float);
    if (bytes > MGC_CUDA_NOALLOC_SCRATCH_BYTES)
        return fail(MGC_CUDA_BAD_ARGUMENT,
                    "mgc_cuda_conv_nhwc_noalloc: the patch matrix needs %lld bytes, more than the %d-byte "
                    "static scratch (N*OH*OW=%lld rows of %lld floats)",
                    bytes, MGC_CUDA_NOALLOC_SCRATCH_BYTES, rows, kp);
    if (rows == 0 || CO == 0) return MGC_CUDA_OK;
    float *scratch = nullptr;
    MGC_CHECK(noalloc_scratch(&scratch));
    const cudaStream_t s = (cudaStream_t)stream;
    // 1) patch matrix [rows][kp] into the scratch: every element written, padding columns zero
    Im2colParams ip{};
    ip.N = N; ip.H = H; ip.W = W; ip.C = C; ip.KH = KH; ip.KW = KW; ip.SH = SH; ip.SW = SW; ip.DH = DH; ip.DW = DW;
    ip.PT = PT; ip.PL = PL; ip.OH = OH; ip.OW = OW; ip.kp = (int)kp; ip.c_off = 0; ip.cg = C;
    ip.x = x;
    ip.out = scratch;
    im2col_nhwc_kernel<<<grid_for(rows * (kp / 4), 256), 256, 0, s>>>(ip);
    MGC_CHECK(check_launch("im2col_nhwc_kernel"));
    // 2) exact-fp32 GEMM: [rows, K] x HWIO weights [K, CO] with the FusedConv epilogue
    GemmParams p{};
    p.M = (int)rows; p.N = CO; p.K = (int)kreal;
    p.nb = 0;
    p.a_kind = MGC_STRIDED; p.a = scratch; p.a_rs = kp; p.a_cs = 1;
    p.b_kind = MGC_STRIDED; p.b = w; p.b_rs = CO; p.b_cs = 1;
    p.c = y; p.ldc = CO;
    p.alpha = 1.0f; p.beta = 1.0f; p.bias = bias; p.bias_mode = bias ? 1 : 0;
    p.res = res; p.ldr = CO; p.act = act; p.lo = lo; p.hi = hi; p.precision = MGC_PREC_FP32;
    return launch_gemm_simt(p, s);
}
