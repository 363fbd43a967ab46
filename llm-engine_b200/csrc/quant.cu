// int8 weight quantisation on the GPU: the reference's quantize_q8 (src/quant.cpp:6-28),
// bit for bit, for weights already in device memory.
//
// The reference computes, per column c of the k x n fp32 matrix B:
//   scale[c] = max_r |B[r][c]|   (std::max: the running value is kept unless it is less, so
//                                  NaNs never enter), then scale[c] /= 127,
//   inv[c]   = scale[c] > 0 ? 1 / scale[c] : 0,
//   q[r][c]  = clamp(lround(B[r][c] * inv[c]), -127, 127).
// Every step is one IEEE operation, so the GPU gets the same bits: the column maximum is
// exact in any order (an atomic max on the bit patterns of non-negative floats), the
// divisions are IEEE divisions (no fast-math in this build), the product is one rounded
// multiply and lround's round-half-away-from-zero is roundf.
//
// Three launches, all HBM-bound: column maxima (B read once; scale is zeroed first), the
// division of the n scales, then the quantisation (B read again, q written).
#include "kernels.h"

namespace llme {
namespace {

constexpr int kQuantThreads = 256;
constexpr int kQuantCols = 128;  // columns per CTA in the maximum pass (32 lanes x float4)
constexpr int kQuantRowsPerCta = 64;

// Column maxima of |B| into scale (as the bit patterns of non-negative floats, which order
// like unsigned integers). CTA (x, y): columns [128x, 128x + 128), rows [64y, 64y + 64).
__global__ void __launch_bounds__(kQuantThreads)
    colmax_kernel(int k, int n, const float* __restrict__ B, unsigned* __restrict__ maxbits) {
    __shared__ float part[kQuantThreads / 32][kQuantCols];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int c0 = blockIdx.x * kQuantCols + lane * 4;
    const int r0 = blockIdx.y * kQuantRowsPerCta;
    const int r1 = min(k, r0 + kQuantRowsPerCta);
    float m[4] = {0.f, 0.f, 0.f, 0.f};
    const bool vec = (n & 3) == 0 && (reinterpret_cast<uintptr_t>(B) & 15) == 0;
    for (int r = r0 + w; r < r1; r += kQuantThreads / 32) {
        const float* row = B + static_cast<size_t>(r) * n;
        if (vec && c0 + 3 < n) {
            const float4 v = *reinterpret_cast<const float4*>(row + c0);
            const float a[4] = {fabsf(v.x), fabsf(v.y), fabsf(v.z), fabsf(v.w)};
#pragma unroll
            for (int j = 0; j < 4; ++j) m[j] = m[j] < a[j] ? a[j] : m[j];
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (c0 + j < n) {
                    const float a = fabsf(row[c0 + j]);
                    m[j] = m[j] < a ? a : m[j];
                }
        }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) part[w][lane * 4 + j] = m[j];
    __syncthreads();
    if (threadIdx.x < kQuantCols) {
        float v = 0.0f;
#pragma unroll
        for (int i = 0; i < kQuantThreads / 32; ++i) {
            const float a = part[i][threadIdx.x];
            v = v < a ? a : v;
        }
        const int c = blockIdx.x * kQuantCols + threadIdx.x;
        if (c < n && v > 0.0f) atomicMax(maxbits + c, __float_as_uint(v));
    }
}

__global__ void scale_kernel(int n, float* __restrict__ scale) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c < n) scale[c] = scale[c] / 127.0f;
}

__device__ __forceinline__ int8_t quantize_one(float x, float inv) {
    const float v = fminf(fmaxf(roundf(__fmul_rn(x, inv)), -127.0f), 127.0f);
    return static_cast<int8_t>(static_cast<int>(v));
}

// q = clamp(round(B * inv)), 4 columns per thread, grid-stride over rows.
__global__ void __launch_bounds__(kQuantThreads)
    quantize_kernel(int k, int n, const float* __restrict__ B, const float* __restrict__ scale,
                    int8_t* __restrict__ q) {
    const int c0 = (blockIdx.x * kQuantThreads + threadIdx.x) * 4;
    if (c0 >= n) return;
    float inv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float s = c0 + j < n ? scale[c0 + j] : 0.0f;
        inv[j] = s > 0.0f ? 1.0f / s : 0.0f;
    }
    const bool vec = (n & 3) == 0 && (reinterpret_cast<uintptr_t>(B) & 15) == 0 && c0 + 3 < n;
    for (int r = blockIdx.y; r < k; r += gridDim.y) {
        const float* row = B + static_cast<size_t>(r) * n;
        int8_t* out = q + static_cast<size_t>(r) * n;
        if (vec) {
            const float4 v = *reinterpret_cast<const float4*>(row + c0);
            char4 o;
            o.x = quantize_one(v.x, inv[0]);
            o.y = quantize_one(v.y, inv[1]);
            o.z = quantize_one(v.z, inv[2]);
            o.w = quantize_one(v.w, inv[3]);
            *reinterpret_cast<char4*>(out + c0) = o;  // n % 4 == 0: 4-byte aligned
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (c0 + j < n) out[c0 + j] = quantize_one(row[c0 + j], inv[j]);
        }
    }
}

}  // namespace

cudaError_t launch_quantize_q8(int k, int n, const float* B, int8_t* q, float* scale,
                               cudaStream_t stream) {
    cudaError_t e = cudaMemsetAsync(scale, 0, static_cast<size_t>(n) * sizeof(float), stream);
    if (e != cudaSuccess) return e;
    const dim3 g1((n + kQuantCols - 1) / kQuantCols, (k + kQuantRowsPerCta - 1) / kQuantRowsPerCta);
    colmax_kernel<<<g1, kQuantThreads, 0, stream>>>(k, n, B, reinterpret_cast<unsigned*>(scale));
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    scale_kernel<<<(n + 255) / 256, 256, 0, stream>>>(n, scale);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    // Enough row slices to fill the GPU several times over, each a grid-stride loop over rows.
    const int col_ctas = (n + kQuantThreads * 4 - 1) / (kQuantThreads * 4);
    const int row_slices = std::max(1, std::min(k, (148 * 16 + col_ctas - 1) / col_ctas));
    quantize_kernel<<<dim3(col_ctas, row_slices), kQuantThreads, 0, stream>>>(k, n, B, scale, q);
    return cudaGetLastError();
}

}  // namespace llme
