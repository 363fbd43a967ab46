// The steps of a decoder layer around the matmuls and the attention, for the transformer
// engine (model.cu): one rank's heads and hidden slice, or the whole model on one GPU.
//
// For decode-shaped products (m <= 8) RoPE with the KV-cache write and SwiGLU run inside the
// GEMV's epilogue (gemv.cu); the kernels here serve the wide (prefill) products and the steps
// that are not products:
//  * gather_rows: the token embedding row of each fed token, copied by the bulk-copy engine
//    (cp.async.bulk global -> shared -> global), one CTA per row;
//  * rope_rows: one warp per (row, head) of a qkv row [q heads | k heads | v heads]: q and k
//    heads are rotated pair by pair (float2) by the angle of the pair's index within its head,
//    k heads and v heads are also written into the caches at the row's position;
//  * swiglu_pairs: SwiGLU over the interleaved layout the engine gives w13's output, gate and
//    up of hidden unit c at columns 2c and 2c + 1, two units per thread (float4 in, float2 out);
//  * rank_sum: the in-process reduction of emulated tensor-parallel ranks (sum in rank order,
//    written back to every rank), the arithmetic of the NVLink all-reduce;
//  * fill_normal / fill_uniform: a counter-based generator (a 64-bit mix of seed and index,
//    Box-Muller for the normal draws) for synthetic models drawn on the device.
// Positions and token ids are read from device memory (feed[0] = first position, feed[1..n] =
// tokens), so one captured CUDA graph serves every position. The kernels release their
// dependents at entry (programmatic dependent launch) and wait for their own inputs.
#include <cmath>

#include "common.cuh"
#include "kernels.h"

namespace llme {
namespace {

__device__ unsigned int g_ops_error;

constexpr int kGatherChunk = 16384;  // bytes per bulk copy step (one 4096-float row)

// x[i] = table[feed[1 + i]] (rows of `dim` floats). Rows of a multiple of 16 bytes with
// 16-byte aligned bases move as bulk copies through shared memory; others float by float.
__global__ void gather_rows_kernel(int dim, const int* __restrict__ feed,
                                   const float* __restrict__ table, float* __restrict__ x,
                                   bool bulk) {
    __shared__ __align__(128) uint8_t buf[kGatherChunk];
    __shared__ uint64_t bar;
    pdl_launch_dependents();
    pdl_wait();
    const int row = blockIdx.x;
    const int token = feed[1 + row];
    const float* src = table + static_cast<size_t>(token) * dim;
    float* dst = x + static_cast<size_t>(row) * dim;
    if (!bulk) {
        for (int j = threadIdx.x; j < dim; j += blockDim.x) dst[j] = src[j];
        return;
    }
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    fence_mbar_init();
    const size_t bytes = static_cast<size_t>(dim) * 4;
    uint32_t phase = 0;
    for (size_t off = 0; off < bytes; off += kGatherChunk, phase ^= 1) {
        const uint32_t len = static_cast<uint32_t>(bytes - off < kGatherChunk ? bytes - off : kGatherChunk);
        mbar_arrive_expect_tx(&bar, len);
        bulk_load_g2s(buf, reinterpret_cast<const uint8_t*>(src) + off, len, &bar);
        if (!mbar_wait(&bar, phase, &g_ops_error)) return;
        asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(
                         reinterpret_cast<uint64_t>(reinterpret_cast<uint8_t*>(dst) + off)),
                     "r"(smem_u32(buf)), "r"(len)
                     : "memory");
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        // The buffer is refilled by the next step: its bytes must have been read out first.
        asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    }
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// The rotation of one (even, odd) pair, rounded as the reference's CPU model rounds it (each
// product rounded, no fused multiply-add).
__device__ __forceinline__ float2 rotate(float2 p, float c, float s) {
    return make_float2(__fsub_rn(__fmul_rn(p.x, c), __fmul_rn(p.y, s)),
                       __fadd_rn(__fmul_rn(p.x, s), __fmul_rn(p.y, c)));
}

// One warp per (row blockIdx.y, head): heads [0, nq) are query heads, [nq, nq + nkv) key heads,
// [nq + nkv, nq + 2 nkv) value heads of the row's qkv vector.
__global__ void rope_rows_kernel(int nq, int nkv, int head_size, const int* __restrict__ feed,
                                 const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                 float* __restrict__ qkv, float* __restrict__ key_cache,
                                 float* __restrict__ value_cache) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int head = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (head >= nq + 2 * nkv) return;
    const int row = blockIdx.y, pos = feed[0] + row, half = head_size / 2;
    const size_t kv = static_cast<size_t>(nkv) * head_size;
    float* vec = qkv + static_cast<size_t>(row) * (static_cast<size_t>(nq) * head_size + 2 * kv) +
                 static_cast<size_t>(head) * head_size;
    if (head >= nq + nkv) {  // value head: into the cache unchanged
        float* dst = value_cache + static_cast<size_t>(pos) * kv +
                     static_cast<size_t>(head - nq - nkv) * head_size;
        for (int j = lane; j < head_size; j += 32) dst[j] = vec[j];
        return;
    }
    const float* c = cos_t + static_cast<size_t>(pos) * half;
    const float* s = sin_t + static_cast<size_t>(pos) * half;
    float2* pairs = reinterpret_cast<float2*>(vec);
    float2* kdst = head >= nq ? reinterpret_cast<float2*>(key_cache + static_cast<size_t>(pos) * kv +
                                                          static_cast<size_t>(head - nq) * head_size)
                              : nullptr;
    for (int j = lane; j < half; j += 32) {
        const float2 r = rotate(pairs[j], c[j], s[j]);
        pairs[j] = r;
        if (kdst) kdst[j] = r;
    }
}

// hb[r][c] = silu(g) * u with (g, u) = gu[r][2c], gu[r][2c + 1]; two hidden units per thread.
__global__ void swiglu_pairs_kernel(size_t units, const float* __restrict__ gu, float* __restrict__ hb) {
    pdl_launch_dependents();
    pdl_wait();
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t u0 = 2 * t;
    if (u0 >= units) return;
    if (u0 + 1 < units) {
        const float4 v = reinterpret_cast<const float4*>(gu)[t];
        const float s0 = 1.0f / (1.0f + expf(-v.x)), s1 = 1.0f / (1.0f + expf(-v.z));
        reinterpret_cast<float2*>(hb)[t] = make_float2(v.x * s0 * v.y, v.z * s1 * v.w);
    } else {
        const float g = gu[2 * u0], up = gu[2 * u0 + 1];
        hb[u0] = g * (1.0f / (1.0f + expf(-g))) * up;
    }
}

// bufs[r][i] = sum over r' in rank order of bufs[r'][i], for every rank r (count floats each).
__global__ void rank_sum_kernel(float* const* __restrict__ bufs, int ranks, size_t count) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= count) return;
    float v = bufs[0][i];
    for (int r = 1; r < ranks; ++r) v += bufs[r][i];
    for (int r = 0; r < ranks; ++r) bufs[r][i] = v;
}

// A 64-bit mix (the finaliser of the SplitMix64 generator) of seed and element index.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}
// Uniform in (0, 1]: the top 24 bits of a mixed word.
__device__ __forceinline__ float unit_float(uint64_t w) {
    return (static_cast<float>(w >> 40) + 1.0f) * (1.0f / 16777216.0f);
}

__global__ void fill_normal_kernel(float* __restrict__ out, size_t count, uint64_t seed, float stddev) {
    const size_t pair = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (2 * pair >= count) return;
    const uint64_t w = mix64(seed * 0x9e3779b97f4a7c15ull + pair);
    const float u1 = unit_float(w), u2 = unit_float(mix64(w ^ 0x632be59bd9b4e019ull));
    // Box-Muller: two independent normals from two uniforms.
    const float r = sqrtf(-2.0f * logf(u1)) * stddev;
    float sn, cs;
    sincospif(2.0f * u2, &sn, &cs);
    out[2 * pair] = r * cs;
    if (2 * pair + 1 < count) out[2 * pair + 1] = r * sn;
}

__global__ void fill_uniform_kernel(float* __restrict__ out, size_t count, uint64_t seed, float lo,
                                    float hi) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= count) return;
    out[i] = lo + (hi - lo) * (unit_float(mix64(seed * 0x9e3779b97f4a7c15ull + i)) - 0.5f / 16777216.0f);
}

// Launch with programmatic stream serialization: the kernel may start while the previous
// one finishes and waits for it with griddepcontrol.wait.
template <typename... K, typename... Args>
cudaError_t launch_pdl(void (*kernel)(K...), dim3 grid, int threads, cudaStream_t stream,
                       Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
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
    const bool bulk = dim % 4 == 0 && reinterpret_cast<uintptr_t>(table) % 16 == 0 &&
                      reinterpret_cast<uintptr_t>(x) % 16 == 0;
    return launch_pdl(gather_rows_kernel, dim3(n), bulk ? 32 : 256, stream, dim, feed, table, x, bulk);
}

cudaError_t launch_rope_cache(int n, int nq, int nkv, int head_size, const int* feed,
                              const float* cos_t, const float* sin_t, float* qkv, float* key_cache,
                              float* value_cache, cudaStream_t stream) {
    constexpr int kWarps = 4;
    const dim3 grid((nq + 2 * nkv + kWarps - 1) / kWarps, n);
    return launch_pdl(rope_rows_kernel, grid, kWarps * 32, stream, nq, nkv, head_size, feed, cos_t,
                      sin_t, qkv, key_cache, value_cache);
}

cudaError_t launch_swiglu(int n, int hidden, const float* gu, float* hb, cudaStream_t stream) {
    const size_t units = static_cast<size_t>(n) * hidden;
    const size_t threads = (units + 1) / 2;
    return launch_pdl(swiglu_pairs_kernel, dim3(static_cast<unsigned>((threads + 255) / 256)), 256,
                      stream, units, gu, hb);
}

cudaError_t launch_rank_sum(float* const* bufs_dev, int ranks, size_t count, cudaStream_t stream) {
    rank_sum_kernel<<<static_cast<unsigned>((count + 255) / 256), 256, 0, stream>>>(bufs_dev, ranks, count);
    return cudaGetLastError();
}

cudaError_t launch_fill_normal(float* out, size_t count, uint64_t seed, float stddev,
                               cudaStream_t stream) {
    const size_t pairs = (count + 1) / 2;
    fill_normal_kernel<<<static_cast<unsigned>((pairs + 255) / 256), 256, 0, stream>>>(out, count, seed, stddev);
    return cudaGetLastError();
}

cudaError_t launch_fill_uniform(float* out, size_t count, uint64_t seed, float lo, float hi,
                                cudaStream_t stream) {
    fill_uniform_kernel<<<static_cast<unsigned>((count + 255) / 256), 256, 0, stream>>>(out, count, seed, lo, hi);
    return cudaGetLastError();
}

unsigned read_and_clear_ops_error() {
    unsigned v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_ops_error, sizeof(v)) != cudaSuccess) return 0;
    if (v) cudaMemcpyToSymbol(g_ops_error, &zero, sizeof(zero));
    return v;
}

void rope_tables(size_t seq_len, size_t head_size, float* cos_out, float* sin_out) {
    // The angles are the model's definition: theta_j = 10000^(-2j / head_size), evaluated in
    // float with <cmath>'s float overloads in the order the reference's CPU model uses
    // (src/model.cpp:171-184), so its host-computed tables and these agree bit for bit.
    const size_t half = head_size / 2;
    for (size_t j = 0; j < half; ++j) {
        const float freq =
            1.0f / std::pow(10000.0f, static_cast<float>(2 * j) / static_cast<float>(head_size));
        for (size_t pos = 0; pos < seq_len; ++pos) {
            const float angle = static_cast<float>(pos) * freq;
            cos_out[pos * half + j] = std::cos(angle);
            sin_out[pos * half + j] = std::sin(angle);
        }
    }
}

}  // namespace llme
