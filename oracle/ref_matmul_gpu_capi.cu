// TEST/BENCH INFRASTRUCTURE ONLY: C entry points to the reference's own GPU matmul
// (src/cuda_matmul.cu, compiled from the reference's sources for sm_100a), so the benchmark
// can time the reference's kernels beside the library's on the same B200 and the same inputs,
// and tests can use it as a second oracle for the GPU path.
#include <cstddef>
#include <cstdint>
#include <exception>
#include <stdexcept>
#include <string>

#include "cuda_matmul.h"

namespace {

thread_local std::string g_msg;

// 0 on success, 1 for std::invalid_argument, 2 for any other error; the message is kept for
// ref_gpu_error().
template <typename F>
int guarded(F&& f) {
    g_msg.clear();
    try {
        f();
        return 0;
    } catch (const std::invalid_argument& e) {
        g_msg = e.what();
        return 1;
    } catch (const std::exception& e) {
        g_msg = e.what();
        return 2;
    }
}

}  // namespace

extern "C" {

const char* ref_gpu_error(void) { return g_msg.c_str(); }

// kernel: the reference's GpuKernel in declaration order (cuda_matmul.h:66-72): 0 automatic,
// 1 naive, 2 tiled, 3 tiled_split, 4 skinny. rms: device pointer to k weights or NULL.
int ref_gpu_matmul_f32(size_t m, size_t n, size_t k, const float* A, const float* B, float* C,
                       int kernel, int accumulate, const float* rms) {
    return guarded([&] {
        MatmulFusion f;
        f.accumulate = accumulate != 0;
        f.rms_weight = rms;
        matmul_cuda(m, n, k, A, B, C, static_cast<GpuKernel>(kernel), f);
    });
}

int ref_gpu_matmul_q8(size_t m, size_t n, size_t k, const float* A, const int8_t* B,
                      const float* scale, float* C, int kernel, int accumulate, const float* rms) {
    return guarded([&] {
        MatmulFusion f;
        f.accumulate = accumulate != 0;
        f.rms_weight = rms;
        matmul_cuda(m, n, k, A, B, scale, C, static_cast<GpuKernel>(kernel), f);
    });
}

int ref_gpu_synchronize(void) {
    return guarded([] { cuda_synchronize(); });
}

size_t ref_gpu_scratch_generation(void) { return cuda_scratch_generation(); }

// Graph capture of the reference's own calls on the stream they launch on (the calling
// thread's per-thread default stream), as its CudaTransformer captures its decode step
// (src/cuda_model.cu:206-228); run the calls once eagerly first so its scratch has grown.
int ref_gpu_capture_begin(void) {
    const cudaError_t e = cudaStreamBeginCapture(cudaStreamPerThread,
                                                 cudaStreamCaptureModeThreadLocal);
    g_msg = e == cudaSuccess ? "" : cudaGetErrorString(e);
    return e == cudaSuccess ? 0 : 2;
}

// Ends the capture and instantiates it; *exec receives the executable graph.
int ref_gpu_capture_end(void** exec) {
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamEndCapture(cudaStreamPerThread, &graph);
    cudaGraphExec_t x = nullptr;
    if (e == cudaSuccess) e = cudaGraphInstantiate(&x, graph, 0);
    if (graph) cudaGraphDestroy(graph);
    *exec = x;
    g_msg = e == cudaSuccess ? "" : cudaGetErrorString(e);
    return e == cudaSuccess ? 0 : 2;
}

// `warmup` untimed replays, then `steps` replays timed with CUDA events on the same stream,
// synchronised on both sides; *ms receives the timed span.
int ref_gpu_time_graph(void* exec, int steps, int warmup, float* ms) {
    const auto x = static_cast<cudaGraphExec_t>(exec);
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    cudaError_t e = cudaEventCreate(&e0);
    if (e == cudaSuccess) e = cudaEventCreate(&e1);
    for (int i = 0; e == cudaSuccess && i < warmup; ++i) e = cudaGraphLaunch(x, cudaStreamPerThread);
    if (e == cudaSuccess) e = cudaStreamSynchronize(cudaStreamPerThread);
    if (e == cudaSuccess) e = cudaEventRecord(e0, cudaStreamPerThread);
    for (int i = 0; e == cudaSuccess && i < steps; ++i) e = cudaGraphLaunch(x, cudaStreamPerThread);
    if (e == cudaSuccess) e = cudaEventRecord(e1, cudaStreamPerThread);
    if (e == cudaSuccess) e = cudaEventSynchronize(e1);
    if (e == cudaSuccess) e = cudaEventElapsedTime(ms, e0, e1);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    g_msg = e == cudaSuccess ? "" : cudaGetErrorString(e);
    return e == cudaSuccess ? 0 : 2;
}

int ref_gpu_graph_destroy(void* exec) {
    return exec && cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(exec)) != cudaSuccess ? 2 : 0;
}

}  // extern "C"
