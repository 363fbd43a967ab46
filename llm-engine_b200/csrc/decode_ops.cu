// The elementwise steps of a decoder layer around the matmuls and the attention, for the
// tensor-parallel transformer (one rank's heads and hidden slice) and its single-GPU case.
// They restate the reference's CudaTransformer kernels (src/cuda_model.cu:22-75: embed,
// rope_and_cache, swiglu) and its host RoPE tables (src/model.cpp:171-184), with the layout
// generalised to a rank's local heads: a qkv row is [q: nq heads | k: nkv heads | v: nkv
// heads] of head_size each. Positions and token ids are read from device memory (feed[0] =
// the first position, feed[1..n] = the tokens), so one captured CUDA graph serves every
// position. The rotation is computed without contraction (explicit round-to-nearest products)
// as the reference's CPU model computes it (src/model.cpp:93-104). The kernels are small (one
// wave), so they release their dependents at entry (programmatic dependent launch): the next
// product starts streaming its weights while they run; they wait for their own inputs first.
#include <cmath>

#include "common.cuh"
#include "kernels.h"

namespace llme {
namespace {

constexpr int kOpThreads = 256;

// x[i][:] = table[feed[1 + i]][:], one block per row; token ids are checked by the host.
__global__ void embed_rows_kernel(int dim, const int* __restrict__ feed,
                                  const float* __restrict__ table, float* __restrict__ x) {
    pdl_launch_dependents();
    pdl_wait();
    const float* src = table + static_cast<size_t>(feed[1 + blockIdx.x]) * dim;
    float* dst = x + static_cast<size_t>(blockIdx.x) * dim;
    for (int j = threadIdx.x; j < dim; j += blockDim.x) dst[j] = src[j];
}

// Row blockIdx.y at position feed[0] + blockIdx.y: a thread rotates one (even, odd) pair of
// q or k by the position's angle for the pair's frequency (its index within the head), and
// writes rotated k pairs and v elements into the caches (row stride kv = nkv * head_size).
__global__ void rope_cache_kernel(int nq, int nkv, int head_size, const int* __restrict__ feed,
                                  const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                  float* __restrict__ qkv, float* __restrict__ key_cache,
                                  float* __restrict__ value_cache) {
    pdl_launch_dependents();
    pdl_wait();
    const int i = blockIdx.y, pos = feed[0] + i, half = head_size / 2;
    const int qd = nq * head_size, kv = nkv * head_size;
    float* q = qkv + static_cast<size_t>(i) * (qd + 2 * kv);
    float* k = q + qd;
    const float* v = k + kv;
    const int pq = qd / 2, pk = kv / 2;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j < pq + pk) {
        const bool is_k = j >= pq;
        const int pair = is_k ? j - pq : j;
        float* p = (is_k ? k : q) + 2 * pair;
        const float c = cos_t[static_cast<size_t>(pos) * half + pair % half];
        const float s = sin_t[static_cast<size_t>(pos) * half + pair % half];
        const float a = p[0], b = p[1];
        const float r0 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        const float r1 = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
        p[0] = r0;
        p[1] = r1;
        if (is_k) {
            float* dst = key_cache + static_cast<size_t>(pos) * kv + 2 * pair;
            dst[0] = r0;
            dst[1] = r1;
        }
    } else if (j < pq + pk + kv) {
        const int t = j - pq - pk;
        value_cache[static_cast<size_t>(pos) * kv + t] = v[t];
    }
}

// hb[r][c] = silu(gu[r][c]) * gu[r][hidden + c] (SwiGLU; gate | up in one row).
__global__ void swiglu_kernel(size_t total, int hidden, const float* __restrict__ gu,
                              float* __restrict__ hb) {
    pdl_launch_dependents();
    pdl_wait();
    const size_t idx = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= total) return;
    const size_t r = idx / hidden, c = idx % hidden;
    const float g = gu[r * 2 * hidden + c];
    hb[idx] = g / (1.0f + expf(-g)) * gu[r * 2 * hidden + hidden + c];
}

// Launch with programmatic stream serialization: the kernel may start while the previous
// one finishes and waits for it with griddepcontrol.wait.
template <typename... K, typename... Args>
cudaError_t launch_pdl(void (*kernel)(K...), dim3 grid, cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kOpThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace

cudaError_t launch_embed_rows(int n, int dim, const int* feed, const float* table, float* x,
                              cudaStream_t stream) {
    return launch_pdl(embed_rows_kernel, dim3(n), stream, dim, feed, table, x);
}

cudaError_t launch_rope_cache(int n, int nq, int nkv, int head_size, const int* feed,
                              const float* cos_t, const float* sin_t, float* qkv, float* key_cache,
                              float* value_cache, cudaStream_t stream) {
    const int work = (nq + nkv) * head_size / 2 + nkv * head_size;
    const dim3 grid((work + kOpThreads - 1) / kOpThreads, n);
    return launch_pdl(rope_cache_kernel, grid, stream, nq, nkv, head_size, feed, cos_t, sin_t, qkv,
                      key_cache, value_cache);
}

cudaError_t launch_swiglu(int n, int hidden, const float* gu, float* hb, cudaStream_t stream) {
    const size_t total = static_cast<size_t>(n) * hidden;
    const unsigned blocks = static_cast<unsigned>((total + kOpThreads - 1) / kOpThreads);
    return launch_pdl(swiglu_kernel, dim3(blocks), stream, total, hidden, gu, hb);
}

void rope_tables(size_t seq_len, size_t head_size, float* cos_out, float* sin_out) {
    // The reference's float expressions (src/model.cpp:171-184), evaluated with the same
    // <cmath> float overloads, so the tables agree with its host-computed ones bit for bit.
    const size_t half = head_size / 2;
    for (size_t pos = 0; pos < seq_len; ++pos) {
        for (size_t j = 0; j < half; ++j) {
            const float freq =
                1.0f / std::pow(10000.0f, static_cast<float>(2 * j) / static_cast<float>(head_size));
            const float angle = static_cast<float>(pos) * freq;
            cos_out[pos * half + j] = std::cos(angle);
            sin_out[pos * half + j] = std::sin(angle);
        }
    }
}

}  // namespace llme
