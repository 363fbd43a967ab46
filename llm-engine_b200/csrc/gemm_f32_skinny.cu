// Decode-shaped fp32-weight products (a few to ~a hundred activation rows) on the
// 5th-generation tensor cores, at the fp32 decode path's accuracy.
//
// The reference runs these shapes on sgemm_tiled<64,4,Split,float> (tiled_split,
// src/cuda_matmul.cu:71-125, 352-363) with fp32 FMA; past ~16 rows a CUDA-core product
// cannot keep up with the weight bytes. Here the product runs on tcgen05.mma.kind::tf32 in
// three TF32 terms (the hi / lo split of both operands, the lo x lo term dropped):
//
//     C = W_hi A_hi + W_hi A_lo + W_lo A_hi,   x_hi = tf32(x) (the low 13 mantissa bits
//                                              cleared), x_lo = x - x_hi (exact in fp32),
//
// which keeps about 22 bits of every product -- inside the decode path's bound of 1e-5 of
// the row's L2 norm. There is no pre-pass: per 32-deep stage TMA brings the raw W panel
// (W as stored, k x n with n contiguous: the MN-major operand, 128-byte swizzle with 32-byte
// atoms, the only layout the tensor cores take for 32-bit MN-major operands) and the raw
// activation rows (K-major, 128-byte swizzle). The MMA reads fp32 words as TF32 by ignoring
// the low 13 bits, so the raw tiles are the hi terms; the four epilogue warps, idle during
// the main loop, write the lo terms x - x_hi next to them (element by element, so the
// swizzled layout carries over) and release them to the tensor cores. Each 8-deep K step:
//     MMA 1: M=128 (the W panel's columns), N=2T ([A_hi; A_lo] rows),   W_hi
//     MMA 2: M=128,                        N=T  (A_hi rows),           W_lo
// into 3T TMEM columns; the epilogue adds the three blocks in that order.
//
// k is split across a thread-block cluster of up to 8 CTAs (grid z); each CTA parks its
// 128 x T partial in its drained shared memory and the cluster adds the partials in rank
// order through distributed shared memory -- deterministic, no scratch, no second launch.
// Every mbarrier wait is bounded (common.cuh).
#include "kernels.h"
#include "tc_common.cuh"

namespace llme {
namespace {

__device__ unsigned int g_f32sk_error;

constexpr int FW = 128;   // output columns per CTA (MMA M, TMEM lanes)
constexpr int FK = 32;    // k per stage: 32 fp32 = one 128-byte row of the activations
constexpr int kFThreads = 192;
constexpr int kConvThreads = 128;  // warps 2-5: lo terms, then the epilogue

template <int T>
struct FGeo {
    static constexpr int kWBytes = FK * FW * 4;              // 16 KB: 4 boxes of 32 x 32
    static constexpr int kRowBytes = T * FK * 4;             // T rows of 128 bytes
    // W_hi, W_lo, A_hi, A_lo
    static constexpr int kStageBytes = 2 * kWBytes + 2 * kRowBytes;  // 36 / 40 / 48 KB
    // T = 16: three stages, two CTAs per SM; T = 32 / 64: four stages, one CTA per SM.
    static constexpr int kBudget = T <= 16 ? 110592 : 196608;
    static constexpr int kStages = kBudget / kStageBytes;     // 3 / 4 / 4
    static constexpr int kSmemBytes = kStages * kStageBytes + 512 + 1024;
    static constexpr int kN = 3 * T;
    static constexpr uint32_t kTmemCols = kN <= 64 ? 64 : kN <= 128 ? 128 : 256;
};

// Shared-memory descriptor with an explicit layout type: 2 = 128-byte swizzle, 1 = 128-byte
// swizzle with 32-byte atoms (32-bit MN-major operands).
__device__ __forceinline__ uint64_t desc_layout(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                                uint64_t layout) {
    return (tc::smem_desc_sw128(saddr, lbo, sbo) & ~(7ull << 61)) | (layout << 61);
}

// tf32 x tf32 -> f32, A (the W panel) MN-major, B (activation rows) K-major.
constexpr uint32_t idesc_tf32_mn(int M, int N) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (1u << 15) |
           (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ float lo_term(float x) {
    return x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}

__device__ __forceinline__ float ld_cluster_f32(const float* local, uint32_t rank) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(tc::map_to_cta(smem_u32(local), rank)) : "memory");
    return v;
}

template <int T>
__global__ void __launch_bounds__(kFThreads)
    gemm_f32_skinny_kernel(const __grid_constant__ CUtensorMap tmW,
                           const __grid_constant__ CUtensorMap tmA, const F32SkinnyArgs a) {
    using Gm = FGeo<T>;
    constexpr int kStages = Gm::kStages;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * Gm::kStageBytes);
    uint64_t* conv = full + kStages;    // lo terms written (4 converter warps)
    uint64_t* empty = conv + kStages;   // stage free again (MMA commit)
    uint64_t* done = empty + kStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c0 = blockIdx.x * FW;
    const int r0 = blockIdx.y * T;
    const int kb0 = blockIdx.z * a.span_blocks;
    const int kb1 = min((a.k + FK - 1) / FK, kb0 + a.span_blocks);
    const int nk = max(0, kb1 - kb0);
    const int slices = gridDim.z;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&conv[s], kConvThreads / 32);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
        prefetch_tensormap(&tmW);
        prefetch_tensormap(&tmA);
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, Gm::kTmemCols);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // Weights of the first stages before the wait when they are static.
            const int pre = a.weights_static ? min(nk, kStages) : 0;
            for (int i = 0; i < pre; ++i) {
                uint8_t* st = smem + i * Gm::kStageBytes;
                mbar_arrive_expect_tx(&full[i], Gm::kWBytes + Gm::kRowBytes);
#pragma unroll
                for (int j = 0; j < FW / 32; ++j)
                    tma_load_2d_nohint(st + j * (Gm::kWBytes / 4), &tmW, c0 + j * 32,
                                       (kb0 + i) * FK, &full[i]);
            }
            pdl_wait();  // the activations come from the kernels before this one
            for (int i = 0; i < nk; ++i) {
                const int s = i % kStages;
                uint8_t* st = smem + s * Gm::kStageBytes;
                if (i >= pre) {
                    if (i >= kStages &&
                        !mbar_wait(&empty[s], ((i / kStages) - 1) & 1, &g_f32sk_error))
                        break;
                    mbar_arrive_expect_tx(&full[s], Gm::kWBytes + Gm::kRowBytes);
#pragma unroll
                    for (int j = 0; j < FW / 32; ++j)
                        tma_load_2d_nohint(st + j * (Gm::kWBytes / 4), &tmW, c0 + j * 32,
                                           (kb0 + i) * FK, &full[s]);
                }
                tma_load_2d_nohint(st + 2 * Gm::kWBytes, &tmA, (kb0 + i) * FK, r0, &full[s]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_hi = idesc_tf32_mn(FW, 2 * T);
            constexpr uint32_t idesc_lo = idesc_tf32_mn(FW, T);
            for (int i = 0; i < nk; ++i) {
                const int s = i % kStages;
                // The converters' arrival implies the stage's copies landed; waiting on both
                // keeps the tensor cores' view of the TMA writes explicit.
                if (!mbar_wait(&full[s], (i / kStages) & 1, &g_f32sk_error) ||
                    !mbar_wait(&conv[s], (i / kStages) & 1, &g_f32sk_error))
                    break;
                tc::fence_after_sync();
                const uint32_t whi = smem_u32(smem + s * Gm::kStageBytes);
                const uint32_t wlo = whi + Gm::kWBytes;
                const uint32_t ahi = wlo + Gm::kWBytes;  // [A_hi; A_lo] rows, then A_lo
#pragma unroll
                for (int kk = 0; kk < FK / 8; ++kk) {
                    // W: 4 boxes of 32 columns, 4 KB apart (LBO); 4-row atoms of 512 B (SBO);
                    // an 8-deep K step is 8 rows = 1 KB. Rows: K-major, 32 bytes per K step.
                    const uint64_t bd = tc::smem_desc_sw128(ahi + kk * 32, 16, 1024);
                    const uint32_t acc = (i | kk) != 0 ? 1u : 0u;
                    tc::mma_tf32(tmem, desc_layout(whi + kk * 1024, Gm::kWBytes / 4, 512, 1), bd,
                                 idesc_hi, acc);
                    tc::mma_tf32(tmem + 2 * T, desc_layout(wlo + kk * 1024, Gm::kWBytes / 4, 512, 1),
                                 bd, idesc_lo, acc);
                }
                tc::commit(&empty[s]);
            }
            tc::commit(done);
        }
    } else {
        // Converters: lo terms of the stage's W panel and activation rows.
        const int ct = threadIdx.x - 64;  // 0 .. 127
        pdl_wait();
        for (int i = 0; i < nk; ++i) {
            const int s = i % kStages;
            if (!mbar_wait(&full[s], (i / kStages) & 1, &g_f32sk_error)) break;
            uint8_t* st = smem + s * Gm::kStageBytes;
            const float4* whi = reinterpret_cast<const float4*>(st);
            float4* wlo = reinterpret_cast<float4*>(st + Gm::kWBytes);
            for (int e = ct; e < Gm::kWBytes / 16; e += kConvThreads) {
                const float4 v = whi[e];
                wlo[e] = make_float4(lo_term(v.x), lo_term(v.y), lo_term(v.z), lo_term(v.w));
            }
            const float4* ahi = reinterpret_cast<const float4*>(st + 2 * Gm::kWBytes);
            float4* alo = reinterpret_cast<float4*>(st + 2 * Gm::kWBytes + Gm::kRowBytes);
            for (int e = ct; e < Gm::kRowBytes / 16; e += kConvThreads) {
                const float4 v = ahi[e];
                alo[e] = make_float4(lo_term(v.x), lo_term(v.y), lo_term(v.z), lo_term(v.w));
            }
            fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor cores
            __syncwarp();
            if (lane == 0) mbar_arrive(&conv[s]);
        }

        // Epilogue: C = (D0 + D1) + D2 for this warp's 32 columns, T rows.
        const int q = warp & 3;
        const int col = c0 + q * 32 + lane;
        const bool ok = mbar_wait(done, 0, &g_f32sk_error);
        tc::fence_after_sync();
        const uint32_t base = tmem + (static_cast<uint32_t>(q * 32) << 16);
        // The partial tile (T x 128 floats) in the drained ring, [row][column].
        float* part = reinterpret_cast<float*>(smem);
#pragma unroll 1
        for (int c = 0; c < T / 16; ++c) {
            __syncwarp();
            uint32_t d0[16], d1[16], d2[16];
            tc::tmem_ld_32x32b_x16(base + c * 16, d0);
            tc::tmem_ld_32x32b_x16(base + T + c * 16, d1);
            tc::tmem_ld_32x32b_x16(base + 2 * T + c * 16, d2);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                float v = 0.0f;
                if (ok && nk > 0)
                    v = (__uint_as_float(d0[j]) + __uint_as_float(d1[j])) + __uint_as_float(d2[j]);
                part[(c * 16 + j) * FW + q * 32 + lane] = v;
            }
        }
        if (slices == 1) {
            // 16 old values in flight before their stores when accumulating (they may alias).
            for (int j0 = 0; j0 < T; j0 += 16) {
                float old[16];
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    old[j] = a.accumulate && r0 + j0 + j < a.m && col < a.n
                                 ? a.C[static_cast<size_t>(r0 + j0 + j) * a.n + col]
                                 : 0.0f;
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (r0 + j0 + j < a.m && col < a.n) {
                        const float v = part[(j0 + j) * FW + q * 32 + lane];
                        a.C[static_cast<size_t>(r0 + j0 + j) * a.n + col] =
                            a.accumulate ? old[j] + v : v;
                    }
            }
        }
    }
    if (slices > 1) {
        // The cluster's k slices: every CTA's partial is parked; CTA r of the cluster adds
        // rows r, r + slices, ... of all partials in rank order.
        __syncwarp();
        tc::pair_sync();
        if (warp >= 2) {
            const int ct = threadIdx.x - 64;
            const float* part = reinterpret_cast<const float*>(smem);
            const uint32_t me = tc::cluster_rank();
            for (int row = static_cast<int>(me); row < T; row += slices) {
                const int col = c0 + ct;
                float v[8];
#pragma unroll
                for (int r = 0; r < 8; ++r)
                    v[r] = r < slices ? ld_cluster_f32(part + row * FW + ct, r) : 0.0f;
                float sum = v[0];
#pragma unroll
                for (int r = 1; r < 8; ++r)
                    if (r < slices) sum += v[r];
                if (r0 + row < a.m && col < a.n) {
                    float* o = a.C + static_cast<size_t>(r0 + row) * a.n + col;
                    *o = a.accumulate ? *o + sum : sum;
                }
            }
        }
        __syncwarp();
        tc::pair_sync();  // no CTA leaves while another may still read its partial
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, Gm::kTmemCols);
    }
}

template <int T>
cudaError_t launch_t(const F32SkinnyArgs& a, const CUtensorMap& tmW, const CUtensorMap& tmA) {
    static unsigned configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 32 && !(configured & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(gemm_f32_skinny_kernel<T>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             FGeo<T>::kSmemBytes);
        if (e != cudaSuccess) return e;
        configured |= 1u << dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.n + FW - 1) / FW, (a.m + T - 1) / T, a.slices);
    cfg.blockDim = dim3(kFThreads);
    cfg.dynamicSmemBytes = FGeo<T>::kSmemBytes;
    cfg.stream = a.stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = a.slices;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, gemm_f32_skinny_kernel<T>, tmW, tmA, a);
}

}  // namespace

int f32_skinny_stage_k() { return FK; }

cudaError_t launch_gemm_f32_skinny(const F32SkinnyArgs& a, const CUtensorMap& tmW,
                                   const CUtensorMap& tmA) {
    switch (a.rows_per_tile) {
        case 16: return launch_t<16>(a, tmW, tmA);
        case 32: return launch_t<32>(a, tmW, tmA);
        case 64: return launch_t<64>(a, tmW, tmA);
        default: return cudaErrorInvalidValue;
    }
}

unsigned read_and_clear_f32sk_error() {
    unsigned v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_f32sk_error, sizeof(v)) != cudaSuccess) return 0;
    if (v) cudaMemcpyToSymbol(g_f32sk_error, &zero, sizeof(zero));
    return v;
}

}  // namespace llme
