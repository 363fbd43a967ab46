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
// the row's L2 norm. There is no pre-pass. Per 32-deep k block, TMA brings the raw W panel
// (32 rows x 128 columns, W as stored) and the raw activation rows (K-major, 128-byte
// swizzle). Four converter warps, one per TMEM lane quarter, read a panel from shared
// memory -- thread c of a quarter reads column c of its 32 rows -- and store the values (the hi
// term: the MMA reads an fp32 word as TF32 by ignoring its low 13 bits) and their lo terms
// into a TMEM slot, lane c: the A operand of kind::tf32 straight from tensor memory, so W
// crosses shared memory once. They also write the activation rows' lo terms next to the rows
// (element by element, so the swizzled layout carries over). Each 8-deep K step:
//     MMA 1: M=128 (the panel's columns, from TMEM), N=2T ([A_hi; A_lo] rows),  W_hi
//     MMA 2: M=128,                                  N=T  (A_hi rows),          W_lo
// into 3T TMEM columns; the epilogue adds the three blocks in that order.
//
// A tcgen05.mma occupies the tensor pipe for ~46 cycles however small N is (8 x 46 cycles a
// block at T = 16), and a barrier wait between MMA batches costs the issuing thread ~225
// cycles more, so that thread waits and commits once per group of two blocks: W panels have
// their own ring (a stage is free once the converters have read it); a stage of the other
// ring holds a block's activation rows and its TMEM W slot, released by the commit of the
// MMAs of its group. Warp 0 loads W, warp 1 issues the MMAs, warps 2-5 convert the first
// block of each group and warps 6-9 the second (warps 2-5 then run the epilogue), warp 10
// loads the activation rows.
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
constexpr int kConvWarps = 8;       // warps 2-9: two blocks of a group, four warps each
constexpr int kBlockThreads = 128;  // the converters of one block
constexpr int kGroup = 2;           // blocks per MMA wait / commit
constexpr int kRowWarp = 10;        // activation rows
constexpr int kFThreads = 11 * 32;
constexpr int kWPanelBytes = FK * FW * 4;  // 16 KB: 32 k-rows of 128 columns, 512 B each

template <int T>
struct FGeo {
    static constexpr int kRowBytes = T * FK * 4;              // T rows of 128 bytes
    static constexpr int kAStageBytes = 2 * kRowBytes;         // A_hi, A_lo
    // TMEM: 3T accumulator columns (rounded to 32), then 64 per stage (W_hi, W_lo).
    static constexpr int kAccCols = (3 * T + 31) / 32 * 32;
    static constexpr uint32_t kTmemCols = 512;                 // one CTA per SM
    static constexpr int kStages =   // 6 / 6 / 4, whole groups
        (static_cast<int>(kTmemCols) - kAccCols) / 64 / kGroup * kGroup;
    static constexpr int kGroups = kStages / kGroup;
    static constexpr int kWStages = 8;
    static constexpr int kWBytes = kWStages * kWPanelBytes;
    static constexpr int kSmemBytes = kWBytes + kStages * kAStageBytes + 512 + 1024;
    static_assert(kGroups >= 2, "rings");
    static_assert(kSmemBytes <= 232448 && kSmemBytes > 232448 / 2, "one CTA per SM");
    static_assert(T * FW * 4 <= kWBytes, "partial tile in the drained W ring");
    static_assert(kRowBytes / 16 % kBlockThreads == 0, "A_lo: whole float4 rounds");
};

// Bounded wait by every lane of a warp; the outcome is the same for all of them, so a warp
// that gives up leaves its loop as a whole.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, &g_f32sk_error));
}

__device__ __forceinline__ float lo_term(float x) {
    return x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}

__device__ __forceinline__ float4 ld_cluster_f32x4(const float* local, uint32_t rank) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(tc::map_to_cta(smem_u32(local), rank))
                 : "memory");
    return v;
}

// tf32 x tf32 -> f32, A (the W panel, in TMEM) and B (activation rows) K-major.
constexpr uint32_t idesc_tf32(int M, int N) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

// C[row][col .. col + 3] (= or +=) v, for the columns below n.
__device__ __forceinline__ void store4(const F32SkinnyArgs& a, int row, int col, float4 v) {
    float* o = a.C + static_cast<size_t>(row) * a.n + col;
    const float w[4] = {v.x, v.y, v.z, v.w};
    float old[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) old[e] = a.accumulate && col + e < a.n ? o[e] : 0.0f;
#pragma unroll
    for (int e = 0; e < 4; ++e)
        if (col + e < a.n) o[e] = a.accumulate ? old[e] + w[e] : w[e];
}

template <int T>
__global__ void __launch_bounds__(kFThreads)
    gemm_f32_skinny_kernel(const __grid_constant__ CUtensorMap tmW,
                           const __grid_constant__ CUtensorMap tmA, const F32SkinnyArgs a) {
    using Gm = FGeo<T>;
    constexpr int SW = Gm::kWStages, S = Gm::kStages, NG = Gm::kGroups;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint8_t* aring = smem + Gm::kWBytes;
    uint64_t* w_full = reinterpret_cast<uint64_t*>(aring + S * Gm::kAStageBytes);
    uint64_t* w_empty = w_full + SW;   // converters have read the panel (4 warps)
    uint64_t* a_full = w_empty + SW;   // activation rows landed (TMA)
    uint64_t* conv = a_full + S;       // a group's TMEM slots and A_lo written (8 warps)
    uint64_t* s_free = conv + NG;      // MMAs reading a group's stages complete (commit)
    uint64_t* done = s_free + NG;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c0 = blockIdx.x * FW;
    const int r0 = blockIdx.y * T;
    const int kb0 = blockIdx.z * a.span_blocks;
    const int kb1 = min((a.k + FK - 1) / FK, kb0 + a.span_blocks);
    const int nk = max(0, kb1 - kb0);
    const int slices = gridDim.z;

    if (threadIdx.x == 0) {
        for (int s = 0; s < SW; ++s) {
            mbar_init(&w_full[s], 1);
            mbar_init(&w_empty[s], kBlockThreads / 32);
        }
        for (int s = 0; s < S; ++s) mbar_init(&a_full[s], 1);
        for (int g = 0; g < NG; ++g) {
            mbar_init(&conv[g], kConvWarps);
            mbar_init(&s_free[g], 1);
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
            const int pre = a.weights_static ? min(nk, SW) : 0;
            for (int i = 0; i < pre; ++i) {
                mbar_arrive_expect_tx(&w_full[i], kWPanelBytes);
                tma_load_2d_nohint(smem + i * kWPanelBytes, &tmW, c0, (kb0 + i) * FK, &w_full[i]);
            }
            pdl_wait();
            for (int i = pre; i < nk; ++i) {
                const int s = i % SW;
                if (i >= SW && !mbar_wait(&w_empty[s], ((i / SW) - 1) & 1, &g_f32sk_error)) break;
                mbar_arrive_expect_tx(&w_full[s], kWPanelBytes);
                tma_load_2d_nohint(smem + s * kWPanelBytes, &tmW, c0, (kb0 + i) * FK, &w_full[s]);
            }
        }
    } else if (warp == kRowWarp) {
        if (lane == 0) {
            pdl_wait();  // the activations come from the kernels before this one
            for (int i = 0; i < nk; ++i) {
                const int s = i % S, g = i / kGroup;
                if (i >= S && !mbar_wait(&s_free[g % NG], ((g / NG) - 1) & 1, &g_f32sk_error))
                    break;
                mbar_arrive_expect_tx(&a_full[s], Gm::kRowBytes);
                tma_load_2d_nohint(aring + s * Gm::kAStageBytes, &tmA, (kb0 + i) * FK, r0,
                                   &a_full[s]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_hi = idesc_tf32(FW, 2 * T);
            constexpr uint32_t idesc_lo = idesc_tf32(FW, T);
            const int ngroups = (nk + kGroup - 1) / kGroup;
            for (int g = 0; g < ngroups; ++g) {
                // The converters waited for the rows' TMA before arriving: one wait covers
                // the group's stages.
                if (!mbar_wait(&conv[g % NG], (g / NG) & 1, &g_f32sk_error)) break;
                tc::fence_after_sync();
                for (int i = g * kGroup; i < min(nk, (g + 1) * kGroup); ++i) {
                    const int s = i % S;
                    const uint32_t rows = smem_u32(aring + s * Gm::kAStageBytes);  // [A_hi; A_lo]
                    const uint32_t whi = tmem + Gm::kAccCols + s * 64;
#pragma unroll
                    for (int kk = 0; kk < FK / 8; ++kk) {
                        // Rows: K-major, 32 bytes per 8-deep K step; W: 8 TMEM columns a step.
                        const uint64_t bd = tc::smem_desc_sw128(rows + kk * 32, 16, 1024);
                        const uint32_t acc = (i | kk) != 0 ? 1u : 0u;
                        tc::mma_tf32_tmem_a(tmem, whi + kk * 8, bd, idesc_hi, acc);
                        tc::mma_tf32_tmem_a(tmem + 2 * T, whi + 32 + kk * 8, bd, idesc_lo, acc);
                    }
                }
                tc::commit(&s_free[g % NG]);
            }
            tc::commit(done);
        }
    } else {
        // Converters: warp w owns TMEM lanes / panel columns 32q .. 32q + 31 (q = w % 4, the
        // lane quarter a warp may access) of block h = (w - 2) / 4 of every group.
        const int q = warp & 3, h = (warp - 2) >> 2;
        const int ct = (threadIdx.x - 64) & (kBlockThreads - 1);  // 0 .. 127 within the block
        const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
        const int ngroups = (nk + kGroup - 1) / kGroup;
        for (int g = 0; g < ngroups; ++g) {
            const int i = g * kGroup + h;
            if (i < nk) {  // the last group may hold one block: its other warps just arrive
                const int sw = i % SW, s = i % S;
                if (!warp_wait(&w_full[sw], (i / SW) & 1)) break;
                const float* panel =
                    reinterpret_cast<const float*>(smem + sw * kWPanelBytes) + q * 32 + lane;
                uint32_t hi[32], lo[32];
#pragma unroll
                for (int r = 0; r < 32; ++r) {
                    const float v = panel[r * FW];
                    hi[r] = __float_as_uint(v);
                    lo[r] = __float_as_uint(lo_term(v));
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&w_empty[sw]);
                // The stage is free once the MMAs of group g - NG completed (its rows were
                // loaded after that); then its rows land.
                if ((g >= NG && !warp_wait(&s_free[g % NG], ((g / NG) - 1) & 1)) ||
                    !warp_wait(&a_full[s], (i / S) & 1))
                    break;
                tc::fence_after_sync();
                const uint32_t slot = tmem + lane_base + Gm::kAccCols + s * 64;
                tc::tmem_st_32x32b_x32(slot, hi);
                tc::tmem_st_32x32b_x32(slot + 32, lo);
                const float4* ahi =
                    reinterpret_cast<const float4*>(aring + s * Gm::kAStageBytes);
                float4* alo =
                    reinterpret_cast<float4*>(aring + s * Gm::kAStageBytes + Gm::kRowBytes);
#pragma unroll
                for (int e0 = 0; e0 < Gm::kRowBytes / 16; e0 += kBlockThreads) {
                    const float4 v = ahi[e0 + ct];
                    alo[e0 + ct] =
                        make_float4(lo_term(v.x), lo_term(v.y), lo_term(v.z), lo_term(v.w));
                }
                fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor cores
                tc::fence_before_sync();
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&conv[g % NG]);
        }

        if (warp < 6) {
            // Epilogue: C = (D0 + D1) + D2 for this warp's 32 columns, T rows.
            const int col = c0 + q * 32 + lane;
            pdl_wait();  // C may be read or written by the kernels before this one
            const bool ok = mbar_wait(done, 0, &g_f32sk_error);
            tc::fence_after_sync();
            // The partial tile (T x 128 floats) in the drained W ring, [row][column].
            float* part = reinterpret_cast<float*>(smem);
#pragma unroll 1
            for (int c = 0; c < T / 16; ++c) {
                __syncwarp();
                uint32_t d0[16], d1[16], d2[16];
                tc::tmem_ld_32x32b_x16(tmem + lane_base + c * 16, d0);
                tc::tmem_ld_32x32b_x16(tmem + lane_base + T + c * 16, d1);
                tc::tmem_ld_32x32b_x16(tmem + lane_base + 2 * T + c * 16, d2);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    float v = 0.0f;
                    if (ok && nk > 0)
                        v = (__uint_as_float(d0[j]) + __uint_as_float(d1[j])) +
                            __uint_as_float(d2[j]);
                    part[(c * 16 + j) * FW + q * 32 + lane] = v;
                }
            }
            if (slices == 1) {
                // 16 old values in flight before their stores when accumulating (they may
                // alias).
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
    }
    if (slices > 1) {
        // The cluster's k slices: every CTA's partial is parked; CTA r of the cluster adds
        // rows r, r + slices, ... of all partials in rank order. Thread t of warps 2-5 takes
        // columns 4 (t % 32) .. + 3 of every fourth such row, two rows' loads in flight.
        __syncwarp();
        tc::pair_sync();
        if (warp >= 2 && warp < 6) {
            const int t = threadIdx.x - 64;
            const int cg = (t & 31) * 4, rg = t >> 5;
            const float* part = reinterpret_cast<const float*>(smem);
            const int me = static_cast<int>(tc::cluster_rank());
            const int nrows = (T - me + slices - 1) / slices;
            for (int j0 = rg; j0 < nrows; j0 += 8) {
                float4 v[2][8];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int row = me + slices * (j0 + 4 * u);
#pragma unroll
                    for (int r = 0; r < 8; ++r)
                        v[u][r] = j0 + 4 * u < nrows && r < slices
                                      ? ld_cluster_f32x4(part + row * FW + cg, r)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int row = me + slices * (j0 + 4 * u);
                    if (j0 + 4 * u >= nrows || r0 + row >= a.m || c0 + cg >= a.n) continue;
                    float4 sum = v[u][0];
#pragma unroll
                    for (int r = 1; r < 8; ++r)
                        if (r < slices) {
                            sum.x += v[u][r].x;
                            sum.y += v[u][r].y;
                            sum.z += v[u][r].z;
                            sum.w += v[u][r].w;
                        }
                    store4(a, r0 + row, c0 + cg, sum);
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
