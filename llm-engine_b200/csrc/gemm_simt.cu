// Exact-fp32 SIMT kernels: the naive reference-order kernel, split-K tiles for
// the mid-size m where the weight-streaming GEMV no longer applies, and the
// RMSNorm pre-pass for kernels that take A already normalised.
//
// Reference counterparts: sgemm_naive (src/cuda_matmul.cu:36-47),
// sgemm_tiled / run_tiled_split + sum_slices (:71-125, :333-363, :247-254),
// rmsnorm_rows (:258-266). The split-K reduction here is folded into the
// product (last CTA per tile adds the slices in order), so a split product is
// one launch, and repeats stay bit-identical.
#include "common.cuh"
#include "kernels.h"

namespace llme {
namespace {

__device__ unsigned int g_tiled_error;

constexpr int BM = kTiledBM, BN = kTiledBN, BK = kTiledBK;
constexpr int kThreads = 256;
constexpr int kTileElems = BM * BN;

template <bool Q8>
__device__ __forceinline__ float load_b_raw(const void* B, size_t idx) {
    if constexpr (Q8) {
        return static_cast<float>(static_cast<const int8_t*>(B)[idx]);
    } else {
        return static_cast<const float*>(B)[idx];
    }
}

// C tile BM x BN; thread (tx, ty) owns rows ty*4.. and columns tx*4.., four by
// four, reading float4s of the staged slabs. int8 B is summed raw and scaled
// per column at the store (the column scale is constant over k).
template <bool Q8>
__global__ void __launch_bounds__(kThreads) tiled_simt_kernel(const TiledArgs a) {
    __shared__ __align__(16) float As[BK][BM + 4];
    __shared__ __align__(16) float Bs[BK][BN];
    __shared__ int flag;
    const int tid = threadIdx.x;
    const int tx = tid % 16, ty = tid / 16;
    const int row0 = blockIdx.y * BM, col0 = blockIdx.x * BN;
    const int slice = blockIdx.z;
    const int p_begin = slice * a.span, p_end = min(a.k, p_begin + a.span);

    float acc[4][4] = {};
    const int ar = tid / 4, ac = (tid % 4) * 4;     // A slab: row, first k
    const int br = tid / 16, bc = (tid % 16) * 4;   // B slab: k row, first column
    for (int p0 = p_begin; p0 < p_end; p0 += BK) {
        {
            const int gr = row0 + ar;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int gp = p0 + ac + i;
                As[ac + i][ar] =
                    gr < a.m && gp < p_end ? a.A[static_cast<size_t>(gr) * a.k + gp] : 0.0f;
            }
        }
        {
            const int gp = p0 + br;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int gc = col0 + bc + i;
                Bs[br][bc + i] = gp < p_end && gc < a.n
                                     ? load_b_raw<Q8>(a.B, static_cast<size_t>(gp) * a.n + gc)
                                     : 0.0f;
            }
        }
        __syncthreads();
#pragma unroll
        for (int p = 0; p < BK; ++p) {
            const float4 av = *reinterpret_cast<const float4*>(&As[p][ty * 4]);
            const float4 bv = *reinterpret_cast<const float4*>(&Bs[p][tx * 4]);
            const float ar4[4] = {av.x, av.y, av.z, av.w};
            const float br4[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(ar4[i], br4[j], acc[i][j]);
        }
        __syncthreads();
    }

    if (a.slices > 1) {
        const int tile = blockIdx.y * gridDim.x + blockIdx.x;
        float* part = a.split.partial +
                      (static_cast<size_t>(tile) * a.slices + slice) * kTileElems + tid * 16;
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) __stcg(part + i * 4 + j, acc[i][j]);
        __threadfence();
        __syncthreads();
        if (tid == 0)
            flag = atomicAdd(a.split.counters + tile, 1u) == static_cast<unsigned>(a.slices - 1);
        __syncthreads();
        if (!flag) return;
        __threadfence();
        const float* base =
            a.split.partial + static_cast<size_t>(tile) * a.slices * kTileElems + tid * 16;
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float v = 0.0f;
                for (int s = 0; s < a.slices; ++s)
                    v += __ldcg(base + static_cast<size_t>(s) * kTileElems + i * 4 + j);
                acc[i][j] = v;
            }
        if (tid == 0) atomicExch(a.split.counters + tile, 0u);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = row0 + ty * 4 + i;
        if (r >= a.m) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int c = col0 + tx * 4 + j;
            if (c >= a.n) continue;
            float v = acc[i][j];
            if constexpr (Q8) v *= __ldg(a.scale + c);
            float* out = a.C + static_cast<size_t>(r) * a.n + c;
            *out = a.accumulate ? *out + v : v;
        }
    }
}

// One thread per element of C, p ascending: the reference's naive order, with
// int8 B dequantised per element as the reference's load_b does.
template <bool Q8>
__global__ void naive_kernel(const TiledArgs a) {
    const int col = blockIdx.x * blockDim.x + threadIdx.x;
    const int row = blockIdx.y * blockDim.y + threadIdx.y;
    if (row >= a.m || col >= a.n) return;
    float acc = 0.0f;
    for (int p = 0; p < a.k; ++p) {
        float b = load_b_raw<Q8>(a.B, static_cast<size_t>(p) * a.n + col);
        if constexpr (Q8) b *= a.scale[col];
        acc += a.A[static_cast<size_t>(row) * a.k + p] * b;
    }
    float* c = a.C + static_cast<size_t>(row) * a.n + col;
    *c = a.accumulate ? *c + acc : acc;
}

// out = A * (1 / sqrt(mean(A^2) + eps)) * w for one row per block.
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(int k, const float* __restrict__ A,
                                                           const float* __restrict__ w,
                                                           float* __restrict__ out) {
    __shared__ float part[8];
    const float* in = A + static_cast<size_t>(blockIdx.x) * k;
    float* o = out + static_cast<size_t>(blockIdx.x) * k;
    float ss = 0.0f;
    for (int j = threadIdx.x; j < k; j += 256) ss = fmaf(in[j], in[j], ss);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float total = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) total += part[i];
    const float s = 1.0f / sqrtf(total / static_cast<float>(k) + kRmsEps);
    for (int j = threadIdx.x; j < k; j += 256) o[j] = in[j] * s * w[j];
}

}  // namespace

cudaError_t launch_tiled_simt(const TiledArgs& a) {
    const dim3 grid((a.n + BN - 1) / BN, (a.m + BM - 1) / BM, a.slices);
    if (a.q8) {
        tiled_simt_kernel<true><<<grid, kThreads, 0, a.stream>>>(a);
    } else {
        tiled_simt_kernel<false><<<grid, kThreads, 0, a.stream>>>(a);
    }
    return cudaGetLastError();
}

cudaError_t launch_naive(const TiledArgs& a) {
    const dim3 block(16, 16);
    const dim3 grid((a.n + 15) / 16, (a.m + 15) / 16);
    if (a.q8) {
        naive_kernel<true><<<grid, block, 0, a.stream>>>(a);
    } else {
        naive_kernel<false><<<grid, block, 0, a.stream>>>(a);
    }
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm_rows(int m, int k, const float* A, const float* w, float* out,
                                cudaStream_t stream) {
    rmsnorm_rows_kernel<<<m, 256, 0, stream>>>(k, A, w, out);
    return cudaGetLastError();
}

unsigned read_and_clear_tiled_error() {
    unsigned v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_tiled_error, sizeof(v)) != cudaSuccess) return 0;
    if (v) cudaMemcpyToSymbol(g_tiled_error, &zero, sizeof(zero));
    return v;
}

}  // namespace llme
