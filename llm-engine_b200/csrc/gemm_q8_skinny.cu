// Decode-shaped int8-weight products (a few to ~a hundred activation rows) on the
// 5th-generation tensor cores, at the decode path's accuracy.
//
// The reference runs these shapes on sgemm_tiled<64,4,Split,int8_t> (tiled_split,
// src/cuda_matmul.cu:71-125, 352-363), fp32 FMA. The weight bytes are the whole cost of
// a decode product; at m = 16..64 a CUDA-core product cannot keep up with HBM (2·m FMAs per
// weight byte), so here the multiply runs on tcgen05.mma.kind::i8:
//
//   * the split pass writes each activation row as THREE int8 terms and a row scale,
//         x = s * (t0 + t1 / 256 + t2 / 65536),  s = max|x| / 127,
//     24 significant bits, within 1/(127 * 2^17) of the row's largest magnitude, so the
//     product stays inside the 1e-5 (of the row's L2 norm) bound of the fp32 decode path;
//   * one CTA computes a 128-column x T-row output tile over its slice of k: the MMA's
//     M operand is the 128-column W panel (MN-major, as stored), its N operand the T rows of
//     t0, t1 and t2 stacked (N = 3T, K-major), so each 32-deep K step is one
//     M=128 N=3T K=32 MMA with exact s32 sums in TMEM;
//   * the epilogue combines the three sums of an output exactly in 64 bits,
//         S = (S0 << 16) + (S1 << 8) + S2,
//     and, when k is split over several CTAs, adds S into an int64 accumulator in global
//     memory (red.global.add.u64). Integer addition is exact and associative, so the result
//     does not depend on the order in which slices arrive: bit-for-bit repeatable with no
//     fixed-order reduction. The CTA that brings the tile's ticket to the slice count writes
//     C = fl(fl(S * 2^-16) * fl(s_row * scale_col)) (+ C) and clears the accumulators and the
//     ticket for the next launch.
//
// With LLME_FLAG_WEIGHTS_STATIC the producer issues the weight loads of its first stages
// before griddepcontrol.wait, so they stream while the split pass (the previous launch) runs.
// Every mbarrier wait is bounded (common.cuh).
#include "kernels.h"
#include "tc_common.cuh"

namespace llme {
namespace {

__device__ unsigned int g_skinny_error;

constexpr int SW = 128;   // output columns per CTA (MMA M, TMEM lanes)
constexpr int SK = 128;   // k per stage
constexpr int kSkThreads = 192;
constexpr int kTerms = 3;

template <int T>
struct SkGeo {
    static constexpr int kWBytes = SK * SW;                   // 16 KB
    static constexpr int kRowsBytes = kTerms * T * SK;        // 6 / 12 / 24 KB
    static constexpr int kStageBytes = kWBytes + kRowsBytes;  // multiples of 1 KB
    static constexpr int kBudget = T >= 64 ? 163840 : 98304;  // one / two CTAs per SM
    static constexpr int kStages = kBudget / kStageBytes;     // 4 / 3 / 4
    static constexpr int kSmemBytes = kStages * kStageBytes + 256 + 1024;
    static constexpr int kN = kTerms * T;                     // 48 / 96 / 192
    static constexpr uint32_t kTmemCols = kN <= 64 ? 64 : kN <= 128 ? 128 : 256;
};

__device__ __forceinline__ void mma_i8_skinny(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// s32 accumulator, signed int8 A and B, A (the W panel) MN-major, B (term rows) K-major.
constexpr uint32_t idesc_skinny(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | (1u << 15) |
           (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ float finish64(long long s, float rs, float sc) {
    const float t = __ll2float_rn(s) * (1.0f / 65536.0f);  // power of two: exact
    return __fmul_rn(t, __fmul_rn(rs, sc));
}

// C rows row0 .. row0 + 15 of column `col` from their exact sums (one warp: lane = column).
// Row scales come one per lane and are passed around by shuffles; with accumulate, all 16 old
// values are loaded before the first store.
__device__ __forceinline__ void store_rows(const SkinnyArgs& a, int row0, int col, bool col_ok,
                                           float sc, const long long (&S)[16]) {
    const int lane = threadIdx.x & 31;
    const float rs_lane = lane < 16 && row0 + lane < a.m ? a.row_scale[row0 + lane] : 0.0f;
    float old[16];
#pragma unroll
    for (int j = 0; j < 16; ++j)
        old[j] = a.accumulate && row0 + j < a.m && col_ok
                     ? a.C[static_cast<size_t>(row0 + j) * a.n + col]
                     : 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const float rs = __shfl_sync(0xffffffffu, rs_lane, j);
        if (row0 + j < a.m && col_ok) {
            const float v = finish64(S[j], rs, sc);
            a.C[static_cast<size_t>(row0 + j) * a.n + col] = a.accumulate ? __fadd_rn(old[j], v) : v;
        }
    }
}

template <int T>
__global__ void __launch_bounds__(kSkThreads)
    gemm_q8_skinny_kernel(const __grid_constant__ CUtensorMap tmW,
                          const __grid_constant__ CUtensorMap tm0,
                          const __grid_constant__ CUtensorMap tm1,
                          const __grid_constant__ CUtensorMap tm2, const SkinnyArgs a) {
    using Gm = SkGeo<T>;
    constexpr int kStages = Gm::kStages;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * Gm::kStageBytes);
    uint64_t* empty = full + kStages;
    uint64_t* done = empty + kStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c0 = blockIdx.x * SW;      // first output column
    const int r0 = blockIdx.y * T;       // first output row
    const int kb0 = blockIdx.z * a.span_blocks;
    const int kb1 = min((a.k + SK - 1) / SK, kb0 + a.span_blocks);
    const int nk = max(0, kb1 - kb0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
        prefetch_tensormap(&tmW);
        prefetch_tensormap(&tm0);
        prefetch_tensormap(&tm1);
        prefetch_tensormap(&tm2);
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, Gm::kTmemCols);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // Weights of the first stages before the wait (they do not depend on the split).
            const int pre = a.weights_static ? min(nk, kStages) : 0;
            for (int i = 0; i < pre; ++i) {
                uint8_t* st = smem + i * Gm::kStageBytes;
                mbar_arrive_expect_tx(&full[i], Gm::kStageBytes);
                tma_load_2d_nohint(st, &tmW, c0, (kb0 + i) * SK, &full[i]);
            }
            pdl_wait();  // the term rows come from the split pass
            for (int i = 0; i < nk; ++i) {
                const int s = i % kStages;
                uint8_t* st = smem + s * Gm::kStageBytes;
                if (i >= pre) {
                    if (i >= kStages &&
                        !mbar_wait(&empty[s], ((i / kStages) - 1) & 1, &g_skinny_error))
                        break;
                    mbar_arrive_expect_tx(&full[s], Gm::kStageBytes);
                    tma_load_2d_nohint(st, &tmW, c0, (kb0 + i) * SK, &full[s]);
                }
                uint8_t* rows = st + Gm::kWBytes;
                const int x = (kb0 + i) * SK;
                tma_load_2d_nohint(rows, &tm0, x, r0, &full[s]);
                tma_load_2d_nohint(rows + T * SK, &tm1, x, r0, &full[s]);
                tma_load_2d_nohint(rows + 2 * T * SK, &tm2, x, r0, &full[s]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_skinny(SW, Gm::kN);
            for (int i = 0; i < nk; ++i) {
                const int s = i % kStages;
                if (!mbar_wait(&full[s], (i / kStages) & 1, &g_skinny_error)) break;
                tc::fence_after_sync();
                const uint32_t wp = smem_u32(smem + s * Gm::kStageBytes);
                const uint32_t rows = wp + Gm::kWBytes;
#pragma unroll
                for (int kk = 0; kk < SK / 32; ++kk) {
                    mma_i8_skinny(tmem, tc::smem_desc_sw128(wp + kk * 32 * 128, Gm::kWBytes, 1024),
                                  tc::smem_desc_sw128(rows + kk * 32, 16, 1024), idesc,
                                  (i | kk) != 0 ? 1u : 0u);
                }
                tc::commit(&empty[s]);
            }
            tc::commit(done);
        }
    } else {
        const int q = warp & 3;  // TMEM lane quadrant
        const int col = c0 + q * 32 + lane;
        const bool col_ok = col < a.n;
        pdl_wait();              // C and the row scales come after the kernels before this one
        const bool ok = mbar_wait(done, 0, &g_skinny_error);
        tc::fence_after_sync();
        const float sc = col_ok ? a.scale[col] : 0.0f;
        const uint32_t base = tmem + (static_cast<uint32_t>(q * 32) << 16);
        const bool split = a.slices > 1;
#pragma unroll 1
        for (int c = 0; c < T / 16; ++c) {
            __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp, converged
            uint32_t s0[16], s1[16], s2[16];
            tc::tmem_ld_32x32b_x16(base + c * 16, s0);
            tc::tmem_ld_32x32b_x16(base + T + c * 16, s1);
            tc::tmem_ld_32x32b_x16(base + 2 * T + c * 16, s2);
            if (!ok || nk == 0) continue;
            const int row0 = r0 + c * 16;
            long long S[16];
#pragma unroll
            for (int j = 0; j < 16; ++j)
                S[j] = (static_cast<long long>(static_cast<int>(s0[j])) << 16) +
                       (static_cast<long long>(static_cast<int>(s1[j])) << 8) +
                       static_cast<long long>(static_cast<int>(s2[j]));
            if (split) {
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (row0 + j < a.m && col_ok)
                        atomicAdd(reinterpret_cast<unsigned long long*>(a.accum) +
                                      static_cast<size_t>(row0 + j) * a.n + col,
                                  static_cast<unsigned long long>(S[j]));
            } else {
                store_rows(a, row0, col, col_ok, sc, S);
            }
        }
        if (split) {
            // Ticket: the CTA that completes the tile's count converts its sums.
            __threadfence();
            named_barrier(1, 128);
            if (threadIdx.x == 64) {
                const unsigned tile = blockIdx.y * gridDim.x + blockIdx.x;
                const unsigned t = atomicAdd(a.counters + tile, 1u);
                *last_flag = (t == static_cast<unsigned>(a.slices) - 1) ? 1 : 0;
            }
            named_barrier(1, 128);
            if (*last_flag) {
                __threadfence();
                unsigned long long* acc = reinterpret_cast<unsigned long long*>(a.accum);
#pragma unroll 1
                for (int row0 = r0; row0 < r0 + T; row0 += 16) {
                    // All 16 sums in flight before any store (loads and stores may alias).
                    long long S[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        S[j] = row0 + j < a.m && col_ok
                                   ? static_cast<long long>(
                                         __ldcg(acc + static_cast<size_t>(row0 + j) * a.n + col))
                                   : 0;
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (row0 + j < a.m && col_ok)
                            acc[static_cast<size_t>(row0 + j) * a.n + col] = 0ull;
                    store_rows(a, row0, col, col_ok, sc, S);
                }
                if (threadIdx.x == 64) a.counters[blockIdx.y * gridDim.x + blockIdx.x] = 0u;
            }
        }
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
cudaError_t launch_t(const SkinnyArgs& a, const CUtensorMap& tmW, const CUtensorMap& t0,
                     const CUtensorMap& t1, const CUtensorMap& t2) {
    static unsigned configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 32 && !(configured & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(gemm_q8_skinny_kernel<T>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             SkGeo<T>::kSmemBytes);
        if (e != cudaSuccess) return e;
        configured |= 1u << dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.n + SW - 1) / SW, (a.m + T - 1) / T, a.slices);
    cfg.blockDim = dim3(kSkThreads);
    cfg.dynamicSmemBytes = SkGeo<T>::kSmemBytes;
    cfg.stream = a.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemm_q8_skinny_kernel<T>, tmW, t0, t1, t2, a);
}

}  // namespace

int skinny_rows_per_tile(int m) { return m <= 16 ? 16 : m <= 32 ? 32 : 64; }
int skinny_ctas_per_sm(int t) { return t >= 64 ? 1 : 2; }

cudaError_t launch_gemm_q8_skinny(const SkinnyArgs& a, const CUtensorMap& tmW,
                                  const CUtensorMap& t0, const CUtensorMap& t1,
                                  const CUtensorMap& t2) {
    switch (a.rows_per_tile) {
        case 16: return launch_t<16>(a, tmW, t0, t1, t2);
        case 32: return launch_t<32>(a, tmW, t0, t1, t2);
        case 64: return launch_t<64>(a, tmW, t0, t1, t2);
        default: return cudaErrorInvalidValue;
    }
}

unsigned read_and_clear_skinny_error() {
    unsigned v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_skinny_error, sizeof(v)) != cudaSuccess) return 0;
    if (v) cudaMemcpyToSymbol(g_skinny_error, &zero, sizeof(zero));
    return v;
}

}  // namespace llme
