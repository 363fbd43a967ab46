// Weight-streaming GEMV / skinny GEMM for decode-shaped products (m <= 8):
// C (+)= [rmsnorm(A)] x B, B fp32 or int8 k x n row-major with column scales.
//
// The reference's counterpart is sgemm_skinny + sum_slices
// (src/cuda_matmul.cu:189-254, launched by run_skinny :365-397). This design
// is B200-first rather than a translation:
//
//  * B is streamed by TMA (cp.async.bulk.tensor.2d) in 64-row x 256-byte
//    boxes into a 5-stage shared-memory ring per CTA; one producer thread
//    keeps every stage in flight, so with two CTAs per SM ~160 KB of weights
//    are outstanding per SM from the first cycle. A (and the RMSNorm weight)
//    ride in the same stage as small boxes, so the consumers never touch
//    global memory in the hot loop. Weights use an L2 evict-first policy.
//  * With programmatic dependent launch the producer issues the first stages
//    of weights before griddepcontrol.wait, overlapping the previous kernel's
//    tail; A and C are touched only after the wait.
//  * int8 is widened without I2F: a PRMT builds 2^23 + (q + 128) as a float
//    and one FADD removes the bias (exact), then the raw int8 values are
//    summed and each column scaled once at the end, as the reference does.
//  * RMSNorm is applied as an epilogue scale: each CTA sums a*a over its own
//    k rows while it streams, multiplies A by the norm weight in the loop, and
//    the final per-row 1/sqrt(mean + eps) multiplies the reduced sums -- no
//    pre-pass and no second read of A.
//  * k is split across CTAs (grid.y) when the columns alone cannot fill 148
//    SMs. Slices are reduced deterministically: partials to scratch, a ticket
//    per column strip, and the last CTA to arrive adds the slices in index
//    order. Repeats are bit-identical (no float atomics).
#include "common.cuh"
#include "kernels.h"

namespace llme {
namespace {

__device__ unsigned int g_gemv_error;

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kTmaThreads = kConsumers + 32;  // + one producer warp
constexpr int kStages = 5;
constexpr int kBoxBytesB = kGemvRowBytes * kGemvBoxRows;  // 16 KB

// Per-thread work split of one 256-byte row segment of B.
template <int M, bool Q8>
struct Shape {
    static constexpr int ESZ = Q8 ? 1 : 4;
    static constexpr int V = Q8 ? (M <= 4 ? 16 : 8) : 4;  // columns per thread
    static constexpr int NT = kGemvRowBytes / ESZ;         // columns per CTA
    static constexpr int TPR = NT / V;                     // threads per row
    static constexpr int RG = kConsumers / TPR;            // row groups
    static constexpr int RPT = kGemvBoxRows / RG;          // rows per thread per box
    static_assert(TPR == 16 || TPR == 32, "row split");
};

template <int M, bool Q8, bool Norm>
struct Layout {
    static constexpr int kB = kStages * kBoxBytesB;
    static constexpr int kABox = M * kGemvBoxRows * 4;
    static constexpr int kWBox = kGemvBoxRows * 4;
    static constexpr int kOffA = kB;
    static constexpr int kOffW = kOffA + kStages * kABox;
    static constexpr int kOffBar = kOffW + (Norm ? kStages * kWBox : 0);
    static constexpr int kBytes = kOffBar + 2 * kStages * 8 + 16;
    static constexpr uint32_t kTx = kBoxBytesB + kABox + (Norm ? kWBox : 0);
    // Reduction buffers reuse the drained ring.
    static constexpr int kRedFloats = kConsumerWarps * M * Shape<M, Q8>::NT;
    static_assert((kRedFloats + M * Shape<M, Q8>::NT) * 4 <= kB, "reduction fits in the ring");
    static_assert((kConsumerWarps + 1) * M * 4 <= kStages * kABox, "ss reduction fits");
};

template <bool Q8, int V>
__device__ __forceinline__ void load_cols(const uint8_t* p, float (&x)[V]) {
    if constexpr (Q8) {
        if constexpr (V == 16) {
            const uint4 q = *reinterpret_cast<const uint4*>(p);
            float t[4];
            s8x4_to_f32(q.x, t);
            x[0] = t[0]; x[1] = t[1]; x[2] = t[2]; x[3] = t[3];
            s8x4_to_f32(q.y, t);
            x[4] = t[0]; x[5] = t[1]; x[6] = t[2]; x[7] = t[3];
            s8x4_to_f32(q.z, t);
            x[8] = t[0]; x[9] = t[1]; x[10] = t[2]; x[11] = t[3];
            s8x4_to_f32(q.w, t);
            x[12] = t[0]; x[13] = t[1]; x[14] = t[2]; x[15] = t[3];
        } else {
            static_assert(V == 8, "int8 columns per thread");
            const uint2 q = *reinterpret_cast<const uint2*>(p);
            float t[4];
            s8x4_to_f32(q.x, t);
            x[0] = t[0]; x[1] = t[1]; x[2] = t[2]; x[3] = t[3];
            s8x4_to_f32(q.y, t);
            x[4] = t[0]; x[5] = t[1]; x[6] = t[2]; x[7] = t[3];
        }
    } else {
        static_assert(V == 4, "fp32 columns per thread");
        const float4 f = *reinterpret_cast<const float4*>(p);
        x[0] = f.x; x[1] = f.y; x[2] = f.z; x[3] = f.w;
    }
}

// Writes the CTA's M x NT sums (tot, in shared memory) to C, through the
// deterministic cross-CTA slice reduction when k is split. Called by the
// kConsumers consumer threads only (named barrier 1).
template <int M, int NT, bool Q8, bool Norm>
__device__ void finish_strip(const float* tot, const float* tot_ss, const GemvArgs& a, int strip,
                             int slice, int tid, int* flag) {
    constexpr int E = M * NT;
    const int col0 = strip * NT;
    const bool split = a.slices > 1;
    if (split) {
        float* part = a.split.partial + (static_cast<size_t>(strip) * a.slices + slice) * E;
        for (int e = tid; e < E; e += kConsumers) __stcg(part + e, tot[e]);
        if (Norm && tid < M)
            __stcg(a.split.partial_ss + (static_cast<size_t>(strip) * a.slices + slice) * M + tid,
                   tot_ss[tid]);
        __threadfence();
        named_barrier(1, kConsumers);
        if (tid == 0)
            *flag = atomicAdd(a.split.counters + strip, 1u) == static_cast<unsigned>(a.slices - 1);
        named_barrier(1, kConsumers);
        if (!*flag) return;
        __threadfence();
    }
    float rs[M];
    if constexpr (Norm) {
#pragma unroll
        for (int r = 0; r < M; ++r) {
            float s2 = 0.0f;
            if (split) {
                const float* ps = a.split.partial_ss + static_cast<size_t>(strip) * a.slices * M + r;
                for (int s = 0; s < a.slices; ++s) s2 += __ldcg(ps + static_cast<size_t>(s) * M);
            } else {
                s2 = tot_ss[r];
            }
            rs[r] = 1.0f / sqrtf(s2 / static_cast<float>(a.k) + kRmsEps);
        }
    }
    const float* base = a.split.partial + static_cast<size_t>(strip) * a.slices * E;
    for (int e = tid; e < E; e += kConsumers) {
        const int r = e / NT, col = col0 + e % NT;
        if (col >= a.n) continue;
        float v;
        if (split) {
            v = 0.0f;
            for (int s = 0; s < a.slices; ++s) v += __ldcg(base + static_cast<size_t>(s) * E + e);
        } else {
            v = tot[e];
        }
        if constexpr (Q8) v *= __ldg(a.scale + col);
        if constexpr (Norm) v *= rs[r];
        float* out = a.C + static_cast<size_t>(r) * a.n + col;
        *out = a.accumulate ? *out + v : v;
    }
    if (split && tid == 0) atomicExch(a.split.counters + strip, 0u);
}

template <int M, bool Q8, bool Norm>
__global__ void __launch_bounds__(kTmaThreads, 2)
    gemv_tma_kernel(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmA,
                    const __grid_constant__ CUtensorMap tmW, const GemvArgs a) {
    using S = Shape<M, Q8>;
    using L = Layout<M, Q8, Norm>;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
    uint64_t* empty = full + kStages;
    int* flag = reinterpret_cast<int*>(empty + kStages);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int strip = blockIdx.x, slice = blockIdx.y;
    const int col0 = strip * S::NT;
    const int k0 = slice * a.span;
    const int k1 = min(a.k, k0 + a.span);
    const int nb = (k1 - k0 + kGemvBoxRows - 1) / kGemvBoxRows;

    if (tid == kConsumers) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_mbar_init();
        prefetch_tensormap(&tmB);
        prefetch_tensormap(&tmA);
        if (Norm) prefetch_tensormap(&tmW);
    }
    __syncthreads();
    if (tid == 0) pdl_launch_dependents();

    if (warp == kConsumerWarps) {
        // Producer. Weights first (they do not depend on the previous launch),
        // then wait for it before loading activations.
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            const int pro = min(nb, kStages);
            for (int b = 0; b < pro; ++b) {
                mbar_arrive_expect_tx(&full[b], L::kTx);
                tma_load_2d(smem + b * kBoxBytesB, &tmB, col0, k0 + b * kGemvBoxRows, &full[b], pol);
            }
            pdl_wait();
            for (int b = 0; b < pro; ++b) {
                tma_load_2d_nohint(smem + L::kOffA + b * L::kABox, &tmA, k0 + b * kGemvBoxRows, 0,
                                   &full[b]);
                if (Norm)
                    tma_load_1d(smem + L::kOffW + b * L::kWBox, &tmW, k0 + b * kGemvBoxRows,
                                &full[b]);
            }
            for (int b = pro; b < nb; ++b) {
                const int s = b % kStages;
                if (!mbar_wait(&empty[s], ((b / kStages) - 1) & 1, &g_gemv_error)) break;
                mbar_arrive_expect_tx(&full[s], L::kTx);
                const int y = k0 + b * kGemvBoxRows;
                tma_load_2d(smem + s * kBoxBytesB, &tmB, col0, y, &full[s], pol);
                tma_load_2d_nohint(smem + L::kOffA + s * L::kABox, &tmA, y, 0, &full[s]);
                if (Norm) tma_load_1d(smem + L::kOffW + s * L::kWBox, &tmW, y, &full[s]);
            }
        }
        return;
    }

    // Consumers: C and the split scratch are touched after this.
    pdl_wait();
    const int cg = tid % S::TPR, rg = tid / S::TPR;
    float acc[M][S::V];
    float ss[M];
#pragma unroll
    for (int r = 0; r < M; ++r) {
        ss[r] = 0.0f;
#pragma unroll
        for (int j = 0; j < S::V; ++j) acc[r][j] = 0.0f;
    }
    for (int b = 0; b < nb; ++b) {
        const int s = b % kStages;
        if (!mbar_wait(&full[s], (b / kStages) & 1, &g_gemv_error)) break;
        const uint8_t* sb = smem + s * kBoxBytesB + cg * (S::V * S::ESZ);
        const float* sa = reinterpret_cast<const float*>(smem + L::kOffA + s * L::kABox);
        const float* sw = reinterpret_cast<const float*>(smem + L::kOffW + s * L::kWBox);
#pragma unroll
        for (int i = 0; i < S::RPT; ++i) {
            const int row = rg + i * S::RG;
            float av[M];
#pragma unroll
            for (int r = 0; r < M; ++r) av[r] = sa[r * kGemvBoxRows + row];
            if constexpr (Norm) {
                const float w = sw[row];
#pragma unroll
                for (int r = 0; r < M; ++r) {
                    ss[r] = fmaf(av[r], av[r], ss[r]);
                    av[r] *= w;
                }
            }
            float x[S::V];
            load_cols<Q8, S::V>(sb + row * kGemvRowBytes, x);
#pragma unroll
            for (int r = 0; r < M; ++r)
#pragma unroll
                for (int j = 0; j < S::V; ++j) acc[r][j] = fmaf(av[r], x[j], acc[r][j]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }

    // Reduce the row groups: pairs inside a warp by shuffle, then the 8 warps
    // through shared memory (the drained ring), always in the same order.
    named_barrier(1, kConsumers);
    float* red = reinterpret_cast<float*>(smem);
    float* tot = red + L::kRedFloats;
    float* red_ss = reinterpret_cast<float*>(smem + L::kOffA);
    float* tot_ss = red_ss + kConsumerWarps * M;
    if constexpr (S::TPR == 16) {
#pragma unroll
        for (int r = 0; r < M; ++r) {
            ss[r] += __shfl_xor_sync(0xffffffffu, ss[r], 16);
#pragma unroll
            for (int j = 0; j < S::V; ++j) acc[r][j] += __shfl_xor_sync(0xffffffffu, acc[r][j], 16);
        }
    }
    if (S::TPR == 32 || lane < 16) {
#pragma unroll
        for (int r = 0; r < M; ++r) {
            float4* dst = reinterpret_cast<float4*>(red + (warp * M + r) * S::NT + cg * S::V);
#pragma unroll
            for (int j = 0; j < S::V / 4; ++j)
                dst[j] = make_float4(acc[r][4 * j], acc[r][4 * j + 1], acc[r][4 * j + 2],
                                     acc[r][4 * j + 3]);
        }
        if (Norm && cg == 0) {
#pragma unroll
            for (int r = 0; r < M; ++r) red_ss[warp * M + r] = ss[r];
        }
    }
    named_barrier(1, kConsumers);
    for (int e = tid; e < M * S::NT; e += kConsumers) {
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) v += red[w * M * S::NT + e];
        tot[e] = v;
    }
    if (Norm && tid < M) {
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) v += red_ss[w * M + tid];
        tot_ss[tid] = v;
    }
    named_barrier(1, kConsumers);
    finish_strip<M, S::NT, Q8, Norm>(tot, tot_ss, a, strip, slice, tid, flag);
}

// Fallback for B rows that are not 16-byte multiples or pointers TMA cannot
// take: one column per lane, the 8 warps split the CTA's k slice, plain
// cached loads. Same reduction and epilogue as the TMA kernel.
template <int M, bool Q8, bool Norm>
__global__ void __launch_bounds__(kConsumers) gemv_ldg_kernel(const GemvArgs a) {
    constexpr int NT = kGemvLdgCols;
    __shared__ float red[kConsumerWarps * M * NT];
    __shared__ float tot[M * NT];
    __shared__ float red_ss[kConsumerWarps * M];
    __shared__ float tot_ss[M];
    __shared__ int flag;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) pdl_launch_dependents();
    pdl_wait();
    const int strip = blockIdx.x, slice = blockIdx.y;
    const int col = strip * NT + lane;
    const int k0 = slice * a.span, k1 = min(a.k, k0 + a.span);
    const int wspan = (k1 - k0 + kConsumerWarps - 1) / kConsumerWarps;
    const int p0 = k0 + warp * wspan, p1 = min(k1, p0 + wspan);
    float acc[M], ss[M];
#pragma unroll
    for (int r = 0; r < M; ++r) acc[r] = ss[r] = 0.0f;
    if (col < a.n) {
#pragma unroll 4
        for (int p = p0; p < p1; ++p) {
            const size_t idx = static_cast<size_t>(p) * a.n + col;
            const float b = Q8 ? static_cast<float>(static_cast<const int8_t*>(a.B)[idx])
                               : static_cast<const float*>(a.B)[idx];
            const float w = Norm ? __ldg(a.rms + p) : 1.0f;
#pragma unroll
            for (int r = 0; r < M; ++r) {
                float av = __ldg(a.A + static_cast<size_t>(r) * a.k + p);
                if constexpr (Norm) {
                    ss[r] = fmaf(av, av, ss[r]);
                    av *= w;
                }
                acc[r] = fmaf(av, b, acc[r]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < M; ++r) red[(warp * M + r) * NT + lane] = acc[r];
    if (Norm && lane == 0) {
#pragma unroll
        for (int r = 0; r < M; ++r) red_ss[warp * M + r] = ss[r];
    }
    __syncthreads();
    for (int e = tid; e < M * NT; e += kConsumers) {
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) v += red[w * M * NT + e];
        tot[e] = v;
    }
    if (Norm && tid < M) {
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) v += red_ss[w * M + tid];
        tot_ss[tid] = v;
    }
    __syncthreads();
    finish_strip<M, NT, Q8, Norm>(tot, tot_ss, a, strip, slice, tid, &flag);
}

cudaLaunchConfig_t make_config(dim3 grid, int threads, size_t smem, cudaStream_t stream, bool pdl,
                               cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.numAttrs = 0;
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cfg;
}

template <int M, bool Q8, bool Norm>
cudaError_t launch_tma_m(const GemvArgs& a, const CUtensorMap& tmB, const CUtensorMap& tmA,
                         const CUtensorMap& tmW) {
    using L = Layout<M, Q8, Norm>;
    auto kern = gemv_tma_kernel<M, Q8, Norm>;
    // Opting in to > 48 KB of dynamic shared memory is per function and device.
    static unsigned configured = 0;  // bit per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 32 && !(configured & (1u << dev))) {
        cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
        if (e != cudaSuccess) return e;
        configured |= 1u << dev;
    }
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg =
        make_config(dim3(a.strips, a.slices), kTmaThreads, L::kBytes, a.stream, a.pdl, attr);
    return cudaLaunchKernelEx(&cfg, kern, tmB, tmA, tmW, a);
}

template <bool Q8, bool Norm>
cudaError_t launch_tma_rows(const GemvArgs& a, const CUtensorMap& tmB, const CUtensorMap& tmA,
                            const CUtensorMap& tmW) {
    switch (a.m) {
        case 1: return launch_tma_m<1, Q8, Norm>(a, tmB, tmA, tmW);
        case 2: return launch_tma_m<2, Q8, Norm>(a, tmB, tmA, tmW);
        case 3: return launch_tma_m<3, Q8, Norm>(a, tmB, tmA, tmW);
        case 4: return launch_tma_m<4, Q8, Norm>(a, tmB, tmA, tmW);
        case 5: return launch_tma_m<5, Q8, Norm>(a, tmB, tmA, tmW);
        case 6: return launch_tma_m<6, Q8, Norm>(a, tmB, tmA, tmW);
        case 7: return launch_tma_m<7, Q8, Norm>(a, tmB, tmA, tmW);
        case 8: return launch_tma_m<8, Q8, Norm>(a, tmB, tmA, tmW);
        default: return cudaErrorInvalidValue;
    }
}

template <int M, bool Q8, bool Norm>
cudaError_t launch_ldg_m(const GemvArgs& a) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg =
        make_config(dim3(a.strips, a.slices), kConsumers, 0, a.stream, a.pdl, attr);
    return cudaLaunchKernelEx(&cfg, gemv_ldg_kernel<M, Q8, Norm>, a);
}

template <bool Q8, bool Norm>
cudaError_t launch_ldg_rows(const GemvArgs& a) {
    switch (a.m) {
        case 1: return launch_ldg_m<1, Q8, Norm>(a);
        case 2: return launch_ldg_m<2, Q8, Norm>(a);
        case 3: return launch_ldg_m<3, Q8, Norm>(a);
        case 4: return launch_ldg_m<4, Q8, Norm>(a);
        case 5: return launch_ldg_m<5, Q8, Norm>(a);
        case 6: return launch_ldg_m<6, Q8, Norm>(a);
        case 7: return launch_ldg_m<7, Q8, Norm>(a);
        case 8: return launch_ldg_m<8, Q8, Norm>(a);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t launch_gemv_tma(const GemvArgs& a, const CUtensorMap& tmB, const CUtensorMap& tmA,
                            const CUtensorMap& tmW) {
    const bool norm = a.rms != nullptr;
    if (a.q8) {
        return norm ? launch_tma_rows<true, true>(a, tmB, tmA, tmW)
                    : launch_tma_rows<true, false>(a, tmB, tmA, tmW);
    }
    return norm ? launch_tma_rows<false, true>(a, tmB, tmA, tmW)
                : launch_tma_rows<false, false>(a, tmB, tmA, tmW);
}

cudaError_t launch_gemv_ldg(const GemvArgs& a) {
    const bool norm = a.rms != nullptr;
    if (a.q8) return norm ? launch_ldg_rows<true, true>(a) : launch_ldg_rows<true, false>(a);
    return norm ? launch_ldg_rows<false, true>(a) : launch_ldg_rows<false, false>(a);
}

unsigned read_and_clear_gemv_error() {
    unsigned v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_gemv_error, sizeof(v)) != cudaSuccess) return 0;
    if (v) cudaMemcpyToSymbol(g_gemv_error, &zero, sizeof(zero));
    return v;
}

}  // namespace llme
