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
//     and writes C = fl(fl(S * 2^-16) * fl(s_row * scale_col)) (+ C);
//   * when k is split, the k slices of a column tile form one thread-block cluster (grid z,
//     at most 8 CTAs): each CTA parks its T x 128 int64 sums in its drained stage ring and,
//     after a cluster barrier, CTA r adds rows r, r + slices, ... of every slice's sums
//     through distributed shared memory and writes those rows of C. Integer addition is
//     exact, so C is the same bits whatever the slice count; there is no global scratch, no
//     atomic and no ticket, and every CTA of the cluster converts its share of the tile.
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
    static_assert(T * SW * 8 <= kStages * kStageBytes, "int64 partial tile in the drained ring");
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

__device__ __forceinline__ longlong2 ld_cluster_s64x2(const long long* local, uint32_t rank) {
    longlong2 v;
    asm volatile("ld.shared::cluster.v2.s64 {%0, %1}, [%2];"
                 : "=l"(v.x), "=l"(v.y)
                 : "r"(tc::map_to_cta(smem_u32(local), rank))
                 : "memory");
    return v;
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
        const int lc = q * 32 + lane;  // column within the tile
        const int col = c0 + lc;
        const bool col_ok = col < a.n;
        pdl_wait();              // C and the row scales come after the kernels before this one
        const bool ok = mbar_wait(done, 0, &g_skinny_error) && nk > 0;
        tc::fence_after_sync();
        const float sc = col_ok ? a.scale[col] : 0.0f;
        const uint32_t base = tmem + (static_cast<uint32_t>(q * 32) << 16);
        long long* part = reinterpret_cast<long long*>(smem);  // the ring, drained by `done`
#pragma unroll 1
        for (int c = 0; c < T / 16; ++c) {
            __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp, converged
            uint32_t s0[16], s1[16], s2[16];
            tc::tmem_ld_32x32b_x16(base + c * 16, s0);
            tc::tmem_ld_32x32b_x16(base + T + c * 16, s1);
            tc::tmem_ld_32x32b_x16(base + 2 * T + c * 16, s2);
            long long S[16];
#pragma unroll
            for (int j = 0; j < 16; ++j)
                S[j] = ok ? (static_cast<long long>(static_cast<int>(s0[j])) << 16) +
                                (static_cast<long long>(static_cast<int>(s1[j])) << 8) +
                                static_cast<long long>(static_cast<int>(s2[j]))
                          : 0;
            if (a.slices > 1) {
#pragma unroll
                for (int j = 0; j < 16; ++j) part[(c * 16 + j) * SW + lc] = S[j];
            } else if (ok) {
                store_rows(a, r0 + c * 16, col, col_ok, sc, S);
            }
        }
    }
    if (a.slices > 1) {
        // Every CTA's sums are parked; CTA `me` of the cluster adds rows me, me + slices, ... of
        // all of them. Thread t of warps 2-5 takes the column pair 2 (t % 64) of every second
        // such row, two rows' loads from every slice in flight.
        __syncwarp();
        tc::pair_sync();
        if (warp >= 2) {
            const int t = threadIdx.x - 64;
            const int cp = (t & 63) * 2;
            const int col = c0 + cp;
            const bool col_ok = col < a.n;  // n % 16 == 0: both columns of the pair or neither
            const float sc0 = col_ok ? a.scale[col] : 0.0f;
            const float sc1 = col_ok ? a.scale[col + 1] : 0.0f;
            const long long* part = reinterpret_cast<const long long*>(smem);
            const int slices = a.slices;
            const int me = static_cast<int>(tc::cluster_rank());
            const int nrows = (T - me + slices - 1) / slices;
#pragma unroll 1
            for (int j0 = t >> 6; j0 < nrows; j0 += 4) {
                longlong2 v[2][8];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int row = me + slices * (j0 + 2 * u);
#pragma unroll
                    for (int r = 0; r < 8; ++r)
                        v[u][r] = j0 + 2 * u < nrows && r < slices
                                      ? ld_cluster_s64x2(part + row * SW + cp, r)
                                      : make_longlong2(0, 0);
                }
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int grow = r0 + me + slices * (j0 + 2 * u);
                    if (j0 + 2 * u >= nrows || grow >= a.m || !col_ok) continue;
                    long long s0 = v[u][0].x, s1 = v[u][0].y;
#pragma unroll
                    for (int r = 1; r < 8; ++r) {
                        s0 += v[u][r].x;  // zero beyond the slice count
                        s1 += v[u][r].y;
                    }
                    const float rs = a.row_scale[grow];
                    float* dst = a.C + static_cast<size_t>(grow) * a.n + col;
                    const float o0 = a.accumulate ? dst[0] : 0.0f;
                    const float o1 = a.accumulate ? dst[1] : 0.0f;
                    const float v0 = finish64(s0, rs, sc0), v1 = finish64(s1, rs, sc1);
                    dst[0] = a.accumulate ? __fadd_rn(o0, v0) : v0;
                    dst[1] = a.accumulate ? __fadd_rn(o1, v1) : v1;
                }
            }
        }
        __syncwarp();
        tc::pair_sync();  // no CTA leaves while another may still read its sums
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
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = a.slices;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, gemm_q8_skinny_kernel<T>, tmW, t0, t1, t2, a);
}

}  // namespace

int skinny_rows_per_tile(int m) { return m <= 16 ? 16 : m <= 32 ? 32 : 64; }
int skinny_ctas_per_sm(int t) { return t >= 64 ? 1 : 2; }

cudaError_t launch_gemm_q8_skinny(const SkinnyArgs& a, const CUtensorMap& tmW,
                                  const CUtensorMap& t0, const CUtensorMap& t1,
                                  const CUtensorMap& t2) {
    if (a.slices < 1 || a.slices > 8) return cudaErrorInvalidValue;  // one portable cluster
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
