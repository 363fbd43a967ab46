// Prefill-shaped int8-weight products (m >= 128) on the 5th-generation tensor cores.
//
// The reference runs these on its SIMT sgemm_tiled<BM,TM,Split,BT=int8_t>
// (src/cuda_matmul.cu:71-125), widening each weight to fp32 and multiplying by
// scale[col] as the tile is stored to shared memory (:99), with fp32 FMA
// accumulation. Here the weights stay int8 all the way into the MMA:
//
//   1. split_rows_kernel turns each fp32 activation row (RMS-normalised first
//      when MatmulFusion::rms_weight is set, in the same operation order as
//      src/cuda_matmul.cu:258-266) into two int8 rows and one fp32 row scale:
//          x = s * (hi + lo / 256),  s = max|x| / 127,
//          hi = rint(x / s) in [-127, 127],  lo = rint((x / s - hi) * 256),
//      so each element is represented to within s / 512 (1/65024 of the
//      row's largest magnitude; the clamp of lo at +-127 only moves it by
//      s / 256 when the residual is exactly one half);
//   2. gemm_q8_tc_kernel computes, with tcgen05.mma.kind::i8 (s8 x s8 -> s32,
//      exact integer sums in TMEM),
//          Hi = hi . W,  Lo = lo . W,
//      and the epilogue writes C (+)= s[row] * scale[col] * (Hi + Lo / 256).
//
// The integer sums are exact (|Hi| <= 127 * 127 * k < 2^31 for k <= 131072),
// so the only rounding is the activation split and the fp32 epilogue; the
// result differs from the reference's fp32 FMA order by about 3e-5 of the
// row's magnitude, inside the 5e-3 tensor-core tolerance, and is bit-for-bit
// repeatable (every CTA computes its own tile with a fixed instruction order).
//
// Orientation: the MMA computes C^T tiles. Its M operand is a 128-column panel of
// W (W as stored, k x n with n contiguous, read MN-major), its N operand is 128
// token rows of hi followed by the same 128 rows of lo (K-major), so one
// M=128, N=256, K=32 MMA produces both integer sums for 128 columns x 128 rows:
// TMEM lane = output column, TMEM columns [0,128) = Hi per row, [128,256) = Lo.
// A tile's accumulator takes 256 of the 512 TMEM columns, so there are two and
// the epilogue of one tile overlaps the MMAs of the next.
//
// Shared memory, per pipeline stage (128 k per stage, 48 KB, 4 stages):
//   W panel: 128 k-rows x 128 columns, 128-byte swizzle (TMA box 128 x 128); the
//            MN-major descriptor steps 1 KB per 8 k-rows (SBO);
//   hi rows: 128 rows x 128 bytes of k, K-major, 128-byte swizzle;
//   lo rows: the same, directly after, so hi and lo form one 256-row operand.
// Warp roles (192 threads, one CTA per SM, persistent over output tiles):
//   warp 0     TMA producer (one thread);
//   warp 1     TMEM allocation (512 columns) and MMA issue (one thread), one
//              commit per stage to free it and one per tile to hand the
//              accumulator to the epilogue;
//   warps 2-5  epilogue: each warp owns a TMEM lane quadrant = 32 output
//              columns; per 32 rows it loads Hi and Lo with tcgen05.ld and
//              writes each row's 32 columns as one coalesced 128-byte store.
// Every mbarrier wait is bounded (common.cuh): a wait that runs out sets the
// file's error word and the kernel winds down instead of hanging.
#include <atomic>
#include <cstring>

#include "kernels.h"
#include "tc_common.cuh"

namespace llme {
namespace {

__device__ unsigned int g_q8tc_error;

constexpr int TBW = 128;   // output columns per tile (MMA M, TMEM lanes)
constexpr int TBT = 128;   // output rows per tile (MMA N = 2 * TBT: hi and lo)
constexpr int TBK = 128;   // k per stage: 128 int8 = one 128-byte swizzle row
constexpr int kThreads = 192;
constexpr int kWBytes = TBK * TBW;      // 16 KB
constexpr int kRowBytes = TBT * TBK;    // 16 KB each for hi and lo
constexpr int kAccCols = 2 * TBT;       // 256
constexpr int kAccBufs = 2;
constexpr int kRingBudget = 196608;
constexpr int kGroupT = 8;              // row tiles that share each W panel (L2 reuse)

// One CTA: a stage holds the W panel, the hi rows and the lo rows (48 KB, 4 stages).
// A CTA pair (Pair): each CTA holds its 128-column half of a 256-column W panel and one of
// hi (even CTA) / lo (odd CTA) (32 KB, 6 stages); one M=256 N=256 MMA over both.
template <bool Pair>
struct Geo {
    static constexpr int kStageBytes = Pair ? kWBytes + kRowBytes : kWBytes + 2 * kRowBytes;
    static constexpr int kStages = kRingBudget / kStageBytes;
    static constexpr int kSmemBytes = kStages * kStageBytes + 256 + 1024;
    static constexpr int kTileW = Pair ? 2 * TBW : TBW;  // output columns per unit
};

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Instruction descriptor: s32 accumulator (D format 2), signed int8 A and B (format 1),
// A (the W panel) MN-major, B (the hi / lo rows) K-major.
constexpr uint32_t idesc_i8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | (1u << 15) |
           (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// One output from the exact integer sums: (Hi + Lo / 256) rounded once, times the rounded
// product of the row and column scales. Explicit roundings, so no contraction can change the
// result: C = fl(fl(Hi + Lo * 2^-8) * fl(s_row * scale_col)) (+ C, rounded).
__device__ __forceinline__ float finish(uint32_t hi, uint32_t lo, float rs, float sc) {
    const float t = fmaf(static_cast<float>(static_cast<int>(lo)), 1.0f / 256.0f,
                         static_cast<float>(static_cast<int>(hi)));
    return __fmul_rn(t, __fmul_rn(rs, sc));
}

// Tile t -> (row tile, column tile): kGroupT row tiles run next to each other on one W panel.
__device__ __forceinline__ void tile_coords(int t, int tiles_t, int tiles_w, int* tt, int* tw) {
    const int group = kGroupT * tiles_w;
    const int first = (t / group) * kGroupT;
    const int g = min(tiles_t - first, kGroupT);
    *tt = first + (t % group) % g;
    *tw = (t % group) / g;
}

// One output tile of one product, as every role of the GEMM sees it.
struct Unit {
    const CUtensorMap *w, *hi, *lo;
    const float* scale;
    const float* row_scale;
    float* C;
    int m, n, nk, tt, tw;
    bool accumulate;
};

// The i-th unit of this CTA. Single product: tiles blockIdx.x + i * gridDim.x. Grouped: the
// CTA's own list from the batch's unit table.
template <bool G, bool Pair>
__device__ __forceinline__ bool fetch_unit(int i, const CUtensorMap* tmHi, const CUtensorMap* tmLo,
                                           const CUtensorMap* tmB, const Q8TcArgs& a,
                                           const Q8TcBatchArgs& b, Unit& u) {
    // Scheduling slot: the CTA, or the CTA pair (both CTAs of a pair walk the same units).
    const int slot = Pair ? blockIdx.x >> 1 : blockIdx.x;
    const int slots = Pair ? gridDim.x >> 1 : gridDim.x;
    constexpr int kTileW = Geo<Pair>::kTileW;
    int t, m, n, k;
    if constexpr (G) {
        const int idx = b.cta_begin[slot] + i;
        if (idx >= b.cta_begin[slot + 1]) return false;
        const uint2 e = b.unit_table[idx];
        const Q8TcItem& it = b.items[e.x];
        t = static_cast<int>(e.y);
        m = it.m;
        n = it.n;
        k = it.k;
        u.w = b.tmW + e.x;
        u.hi = b.tmHi + e.x;
        u.lo = b.tmLo + e.x;
        u.scale = it.scale;
        u.row_scale = it.row_scale;
        u.C = it.C;
        u.accumulate = it.accumulate != 0;
    } else {
        m = a.m;
        n = a.n;
        k = a.k;
        t = slot + i * slots;
        if (t >= ((m + TBT - 1) / TBT) * ((n + kTileW - 1) / kTileW)) return false;
        u.w = tmB;
        u.hi = tmHi;
        u.lo = tmLo;
        u.scale = a.scale;
        u.row_scale = a.row_scale;
        u.C = a.C;
        u.accumulate = a.accumulate;
    }
    u.m = m;
    u.n = n;
    u.nk = (k + TBK - 1) / TBK;
    tile_coords(t, (m + TBT - 1) / TBT, (n + kTileW - 1) / kTileW, &u.tt, &u.tw);
    return true;
}

__device__ __forceinline__ void mma_i8_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

template <bool G, bool Pair>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_q8_tc_kernel(const __grid_constant__ CUtensorMap tmHi,
                      const __grid_constant__ CUtensorMap tmLo,
                      const __grid_constant__ CUtensorMap tmB, const Q8TcArgs a,
                      const Q8TcBatchArgs b) {
    using Gm = Geo<Pair>;
    constexpr int kStages = Gm::kStages;
    constexpr int kStageBytes = Gm::kStageBytes;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
    uint64_t* empty = full + kStages;
    uint64_t* acc_full = empty + kStages;
    uint64_t* acc_empty = acc_full + kAccBufs;
    uint64_t* drain = acc_empty + kAccBufs;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Pair: rank 0 issues the MMAs and holds the full barriers (its loads and the peer's are
    // counted there); each CTA's empty / accumulator-full barriers are signalled by rank 0's
    // commits; rank 0's accumulator-empty barriers count the epilogue warps of both CTAs.
    const uint32_t rank = Pair ? tc::cluster_rank() : 0;
    auto in_cta = [](const void* p, uint32_t r) { return tc::map_to_cta(smem_u32(p), r); };

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int bf = 0; bf < kAccBufs; ++bf) {
            mbar_init(&acc_full[bf], 1);
            mbar_init(&acc_empty[bf], Pair ? 8 : 4);  // one arrival per epilogue warp
        }
        mbar_init(drain, 1);
        fence_mbar_init();
        if (!G) {
            prefetch_tensormap(&tmHi);
            prefetch_tensormap(&tmLo);
            prefetch_tensormap(&tmB);
        }
    }
    if (warp == 1) {
        if constexpr (Pair) tc::tmem_alloc_pair(tmem_slot, 512);
        else tc::tmem_alloc(tmem_slot, 512);
    }
    tc::fence_before_sync();
    __syncthreads();
    if constexpr (Pair) tc::pair_sync();  // both CTAs' barriers and TMEM exist
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            pdl_wait();  // the split rows come from the kernel before this one
            int it = 0;
            bool ok = true;
            Unit u;
            for (int i = 0; ok && fetch_unit<G, Pair>(i, &tmHi, &tmLo, &tmB, a, b, u); ++i) {
                for (int kb = 0; kb < u.nk; ++kb, ++it) {
                    const int s = it % kStages;
                    if (it >= kStages &&
                        !mbar_wait(&empty[s], ((it / kStages) - 1) & 1, &g_q8tc_error)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = smem + s * kStageBytes;
                    if constexpr (Pair) {
                        const uint32_t fb = in_cta(&full[s], 0);
                        if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * kStageBytes);
                        tc::tma_load_2d_pair(st, u.w, u.tw * Gm::kTileW + rank * TBW, kb * TBK, fb);
                        tc::tma_load_2d_pair(st + kWBytes, rank == 0 ? u.hi : u.lo, kb * TBK,
                                             u.tt * TBT, fb);
                    } else {
                        mbar_arrive_expect_tx(&full[s], kStageBytes);
                        tma_load_2d_nohint(st, u.w, u.tw * TBW, kb * TBK, &full[s]);
                        tma_load_2d_nohint(st + kWBytes, u.hi, kb * TBK, u.tt * TBT, &full[s]);
                        tma_load_2d_nohint(st + kWBytes + kRowBytes, u.lo, kb * TBK, u.tt * TBT,
                                           &full[s]);
                    }
                }
            }
            // Before the CTA (pair) may exit, every copy issued into its shared memory has
            // landed (already true unless a wait above gave up). A pair's copies are all
            // counted on rank 0's full barriers; the final pair_sync keeps rank 1 until then.
            if (rank == 0) {
                for (int j = it - 1; j >= 0 && j >= it - kStages; --j)
                    mbar_wait(&full[j % kStages], (j / kStages) & 1, &g_q8tc_error);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = idesc_i8(Pair ? 2 * TBW : TBW, 2 * TBT);
            int it = 0, use = 0;
            bool ok = true;
            Unit u;
            for (; ok && fetch_unit<G, Pair>(use, &tmHi, &tmLo, &tmB, a, b, u); ++use) {
                const int buf = use % kAccBufs;
                const int round = use / kAccBufs;
                if (round > 0) {
                    const bool freed = Pair ? mbar_wait_cluster(&acc_empty[buf], (round - 1) & 1,
                                                                &g_q8tc_error)
                                            : mbar_wait(&acc_empty[buf], (round - 1) & 1,
                                                        &g_q8tc_error);
                    if (!freed) break;
                }
                tc::fence_after_sync();
                const uint32_t d = tmem + buf * kAccCols;
                for (int kb = 0; kb < u.nk; ++kb, ++it) {
                    const int s = it % kStages;
                    if (!mbar_wait(&full[s], (it / kStages) & 1, &g_q8tc_error)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint32_t wp = smem_u32(smem + s * kStageBytes);
                    const uint32_t rows = wp + kWBytes;
#pragma unroll
                    for (int kk = 0; kk < TBK / 32; ++kk) {
                        // W: MN-major, 32 k-rows of 128 bytes per K step. Rows: K-major,
                        // the 32-deep K step is 32 bytes into each 128-byte row. A pair's
                        // descriptors name this CTA's halves; the peer's sit at the same
                        // offsets in its own shared memory.
                        const uint64_t ad = tc::smem_desc_sw128(wp + kk * 32 * 128, kWBytes, 1024);
                        const uint64_t bd = tc::smem_desc_sw128(rows + kk * 32, 16, 1024);
                        const uint32_t acc = (kb | kk) != 0 ? 1u : 0u;
                        if constexpr (Pair) mma_i8_pair(d, ad, bd, idesc, acc);
                        else mma_i8(d, ad, bd, idesc, acc);
                    }
                    if constexpr (Pair) {
                        tc::commit_pair(in_cta(&empty[s], 0));
                        tc::commit_pair(in_cta(&empty[s], 1));
                    } else {
                        tc::commit(&empty[s]);
                    }
                }
                if constexpr (Pair) {
                    tc::commit_pair(in_cta(&acc_full[buf], 0));
                    tc::commit_pair(in_cta(&acc_full[buf], 1));
                } else {
                    tc::commit(&acc_full[buf]);
                }
            }
            // No MMA may still be writing TMEM when it is released.
            if constexpr (Pair) tc::commit_pair(in_cta(drain, 0));
            else tc::commit(drain);
            mbar_wait(drain, 0, &g_q8tc_error);
        }
    } else {
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        pdl_wait();              // C may be read by the kernel before this one
        Unit u;
        for (int use = 0; fetch_unit<G, Pair>(use, &tmHi, &tmLo, &tmB, a, b, u); ++use) {
            const int buf = use % kAccBufs;
            const int round = use / kAccBufs;
            const bool ready = Pair ? mbar_wait_cluster(&acc_full[buf], round & 1, &g_q8tc_error)
                                    : mbar_wait(&acc_full[buf], round & 1, &g_q8tc_error);
            if (!ready) break;
            tc::fence_after_sync();
            const int col = u.tw * Gm::kTileW + static_cast<int>(rank) * TBW + q * 32 + lane;
            const bool col_ok = col < u.n;
            const float sc = col_ok ? u.scale[col] : 0.0f;
            const uint32_t base = tmem + (static_cast<uint32_t>(q * 32) << 16) + buf * kAccCols;
#pragma unroll 1
            for (int c = 0; c < TBT / 32; ++c) {
                __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp, converged
                uint32_t h[32], l[32];
                tc::tmem_ld_32x32b_x32(base + c * 32, h);
                tc::tmem_ld_32x32b_x32(base + TBT + c * 32, l);
                const int row0 = u.tt * TBT + c * 32;
                if (row0 >= u.m) continue;
                // Row scales of these 32 rows, one per lane, passed around by shuffles.
                const float rs_lane = row0 + lane < u.m ? u.row_scale[row0 + lane] : 0.0f;
                if (u.accumulate) {
                    // 16 old values in flight before the first of their stores (they may alias).
#pragma unroll
                    for (int j0 = 0; j0 < 32; j0 += 16) {
                        float old[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            old[j] = row0 + j0 + j < u.m && col_ok
                                         ? u.C[static_cast<size_t>(row0 + j0 + j) * u.n + col]
                                         : 0.0f;
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const float rs = __shfl_sync(0xffffffffu, rs_lane, j0 + j);
                            if (row0 + j0 + j < u.m && col_ok)
                                u.C[static_cast<size_t>(row0 + j0 + j) * u.n + col] =
                                    __fadd_rn(old[j], finish(h[j0 + j], l[j0 + j], rs, sc));
                        }
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float rs = __shfl_sync(0xffffffffu, rs_lane, j);
                        if (row0 + j < u.m && col_ok)
                            u.C[static_cast<size_t>(row0 + j) * u.n + col] =
                                finish(h[j], l[j], rs, sc);
                    }
                }
            }
            // This warp's reads of the buffer are complete (tcgen05.ld waits inside the helper).
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) {
                if constexpr (Pair) tc::mbar_arrive_cluster(in_cta(&acc_empty[buf], 0));
                else mbar_arrive(&acc_empty[buf]);
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if constexpr (Pair) tc::pair_sync();  // rank 0's MMAs drained, both epilogues done
    if (warp == 1) {
        __syncwarp();
        tc::fence_after_sync();
        if constexpr (Pair) tc::tmem_dealloc_pair(tmem, 512);
        else tc::tmem_dealloc(tmem, 512);
    }
}

// One CTA per row of A: the row (RMS-normalised when w is set: x = a * inv_rms * w) is split
// into hi / lo int8 rows of pitch kp and a row scale (see the file comment). Rows whose
// largest magnitude is not finite get a NaN row scale, so their outputs are NaN, as an fp32
// product with that row would be.
// Aligned rows (k % 4 == 0, 16-byte aligned A and w) that fit the launch's dynamic shared
// memory arrive with one bulk copy (cp.async.bulk) and both passes read shared memory: one
// instruction per row keeps the whole row in flight. Other aligned rows keep the first
// kSplitRegs * 4 * kSplitThreads elements in registers between the passes (a longer row's
// remainder is read twice); unaligned rows take plain scalar loads.
constexpr int kSplitThreads = 256;
constexpr int kSplitRegs = 12;      // float4 per thread in the register path
constexpr int kSplitSmemMax = kQ8TcSplitSmemMax;  // rows up to 49152 elements by bulk copy
__device__ unsigned int g_split_error;

// The split of one row. Two terms: x = s * (t0 + t1 / 256). Three terms (the skinny GEMM,
// held to the decode path's 1e-5 bound): x = s * (t0 + t1 / 256 + t2 / 65536), each residual
// scaled by 256 exactly (y - rint(y) and its multiples by 256 are exact in fp32).
struct SplitRow {
    float inv_rms, q, pre;
    bool norm;
    bool three;
    // The terms of one element (the kernel's whole arithmetic for an element).
    __device__ __forceinline__ void split(float a, float g, int8_t* o0, int8_t* o1,
                                          int8_t* o2) const {
        const float x = norm ? a * inv_rms * g : a;
        float y = pre == 1.0f ? x * q : (x * pre) * q;
        if (!(fabsf(y) <= 128.0f)) y = 0.0f;  // non-finite rows: the row scale is NaN
        int t0, t1, t2;
        int8_digits(y, t0, t1, t2);  // two terms: the first two digits
        *o0 = static_cast<int8_t>(t0);
        *o1 = static_cast<int8_t>(t1);
        if (three) *o2 = static_cast<int8_t>(t2);
    }
    __device__ __forceinline__ void split4(float4 v, float4 g, int8_t* p0, int8_t* p1,
                                           int8_t* p2) const {
        char4 a, b, c;
        split(v.x, g.x, &a.x, &b.x, &c.x);
        split(v.y, g.y, &a.y, &b.y, &c.y);
        split(v.z, g.z, &a.z, &b.z, &c.z);
        split(v.w, g.w, &a.w, &b.w, &c.w);
        *reinterpret_cast<char4*>(p0) = a;
        *reinterpret_cast<char4*>(p1) = b;
        if (three) *reinterpret_cast<char4*>(p2) = c;
    }
};

__device__ __forceinline__ void split_accumulate(float4 v, float4 g, bool norm, float* ss, float* mx) {
    float4 u = v;
    if (norm) {
        *ss = fmaf(v.x, v.x, *ss);
        *ss = fmaf(v.y, v.y, *ss);
        *ss = fmaf(v.z, v.z, *ss);
        *ss = fmaf(v.w, v.w, *ss);
        u = make_float4(v.x * g.x, v.y * g.y, v.z * g.z, v.w * g.w);
    }
    *mx = fmaxf(*mx, fmaxf(fmaxf(fabsf(u.x), fabsf(u.y)), fmaxf(fabsf(u.z), fabsf(u.w))));
    // fmaxf drops NaN; keep it visible.
    if (u.x != u.x || u.y != u.y || u.z != u.z || u.w != u.w) *mx = __int_as_float(0x7f800000);
}

// Splits one row `in` (k floats) into the term rows o0, o1 (and o2 when not null: three
// terms) and writes its scale to *rs_out. Whole CTA.
// Bulk: the launch guarantees every row is aligned and fits `srow` (the dynamic shared
// memory); the generic form takes any row. Two instantiations, so the bulk kernel does not
// carry the register path's registers.
template <bool Bulk>
__device__ __forceinline__ void split_row(int k, const float* __restrict__ in,
                                          const float* __restrict__ w, int8_t* __restrict__ oh,
                                          int8_t* __restrict__ ol, int8_t* __restrict__ o2,
                                          float* __restrict__ rs_out, float* srow) {
    __shared__ float red_ss[kSplitThreads / 32], red_mx[kSplitThreads / 32];
    __shared__ uint64_t row_bar;
    const bool norm = w != nullptr;
    const bool vec = Bulk || ((k & 3) == 0 && (reinterpret_cast<uintptr_t>(in) & 15) == 0 &&
                              (!norm || (reinterpret_cast<uintptr_t>(w) & 15) == 0));
    constexpr bool bulk = Bulk;
    constexpr int kStride = kSplitThreads * 4;
    const float4 one = make_float4(1.f, 1.f, 1.f, 1.f);
    // The norm weights are shared by every row (cached), so they are loaded where used rather
    // than held in registers.
    auto wload = [&](int j) { return norm ? *reinterpret_cast<const float4*>(w + j) : one; };
    float4 v[Bulk ? 1 : kSplitRegs];
    // Pass 1: sum of squares (for the norm) and the largest |a * w| (or |a|).
    float ss = 0.0f, mx = 0.0f;
    bool landed = true;
    if constexpr (bulk) {
        if (threadIdx.x == 0) {
            mbar_init(&row_bar, 1);
            fence_mbar_init();
            mbar_arrive_expect_tx(&row_bar, static_cast<uint32_t>(k) * 4);
            bulk_load_g2s(srow, in, static_cast<uint32_t>(k) * 4, &row_bar);
        }
        __syncthreads();  // the barrier is initialised before anyone waits on it
        landed = mbar_wait(&row_bar, 0, &g_split_error);
        if (landed) {
            for (int j = threadIdx.x * 4; j < k; j += kStride)
                split_accumulate(*reinterpret_cast<const float4*>(srow + j), wload(j), norm, &ss, &mx);
        }
    } else if (vec) {
#pragma unroll
        for (int r = 0; r < (Bulk ? 0 : kSplitRegs); ++r) {
            const int j = r * kStride + threadIdx.x * 4;
            v[r] = j < k ? *reinterpret_cast<const float4*>(in + j) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int r = 0; r < (Bulk ? 0 : kSplitRegs); ++r) {
            const int j = r * kStride + threadIdx.x * 4;
            if (j < k) split_accumulate(v[r], wload(j), norm, &ss, &mx);
        }
        for (int j = kSplitRegs * kStride + threadIdx.x * 4; j < k; j += kStride)
            split_accumulate(*reinterpret_cast<const float4*>(in + j), wload(j), norm, &ss, &mx);
    } else {
        for (int j = threadIdx.x; j < k; j += kSplitThreads) {
            const float a = in[j];
            float u = a;
            if (norm) {
                ss = fmaf(a, a, ss);
                u = a * w[j];
            }
            mx = fmaxf(mx, fabsf(u));
            if (u != u) mx = __int_as_float(0x7f800000);
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        ss += __shfl_xor_sync(0xffffffffu, ss, off);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    }
    if ((threadIdx.x & 31) == 0) {
        red_ss[threadIdx.x >> 5] = ss;
        red_mx[threadIdx.x >> 5] = mx;
    }
    __syncthreads();
    float total = 0.0f, amax = 0.0f;
#pragma unroll
    for (int i = 0; i < kSplitThreads / 32; ++i) {
        total += red_ss[i];
        amax = fmaxf(amax, red_mx[i]);
    }
    SplitRow sr;
    sr.norm = norm;
    sr.three = o2 != nullptr;
    sr.inv_rms = norm ? 1.0f / sqrtf(total / static_cast<float>(k) + kRmsEps) : 1.0f;
    amax *= sr.inv_rms;
    // Multiplier to the hi grid (127 at the row's largest magnitude). Rows so small that
    // 127 / amax would overflow are first brought up by 2^64 (exact).
    sr.pre = amax > 0.0f && amax < 1e-30f ? 18446744073709551616.0f : 1.0f;  // 2^64
    sr.q = amax > 0.0f ? 127.0f / (amax * sr.pre) : 0.0f;
    if (threadIdx.x == 0) {
        float s = amax / 127.0f;
        if (!(amax <= 3.402823466e38f)) s = __int_as_float(0x7fc00000);  // inf / NaN rows
        *rs_out = s;
    }
    // Pass 2: hi / lo.
    if constexpr (bulk) {
        if (landed) {
            for (int j = threadIdx.x * 4; j < k; j += kStride)
                sr.split4(*reinterpret_cast<const float4*>(srow + j), wload(j), oh + j, ol + j,
                          o2 + j);
        }
    } else if (vec) {
#pragma unroll
        for (int r = 0; r < (Bulk ? 0 : kSplitRegs); ++r) {
            const int j = r * kStride + threadIdx.x * 4;
            if (j < k) sr.split4(v[r], wload(j), oh + j, ol + j, o2 + j);
        }
        for (int j = kSplitRegs * kStride + threadIdx.x * 4; j < k; j += kStride)
            sr.split4(*reinterpret_cast<const float4*>(in + j), wload(j), oh + j, ol + j, o2 + j);
    } else {
        for (int j = threadIdx.x; j < k; j += kSplitThreads) {
            int8_t a8, b8, c8;
            sr.split(in[j], norm ? w[j] : 1.0f, &a8, &b8, &c8);
            oh[j] = a8;
            ol[j] = b8;
            if (o2) o2[j] = c8;
        }
    }
}

template <bool Bulk>
__global__ void __launch_bounds__(kSplitThreads)
    split_rows_kernel(int k, int kp, const float* __restrict__ A, const float* __restrict__ w,
                      int8_t* __restrict__ hi, int8_t* __restrict__ lo, int8_t* __restrict__ t2,
                      float* __restrict__ row_scale) {
    extern __shared__ __align__(16) float split_smem[];
    // A grid of one wave (decode-sized m) lets the next launch be placed at once: all its own
    // CTAs are already resident, so the early arrivals cannot crowd them out.
    if (gridDim.x <= 256) pdl_launch_dependents();
    pdl_wait();
    const size_t r = blockIdx.x;
    split_row<Bulk>(k, A + r * k, w, hi + r * kp, lo + r * kp, t2 ? t2 + r * kp : nullptr,
                    row_scale + r, split_smem);
    // Only now may the GEMM's CTAs (197 KB of shared memory each, waiting for this grid) be
    // placed: placed earlier they would take SMs that this grid's remaining rows still need.
    pdl_launch_dependents();
}

// Grouped: CTA r splits global row r, row r - row_begin[p] of product p.
template <bool Bulk>
__global__ void __launch_bounds__(kSplitThreads) split_rows_batch_kernel(const Q8TcBatchArgs b) {
    extern __shared__ __align__(16) float split_smem[];
    pdl_wait();
    const int r = blockIdx.x;
    int lo_p = 0, hi_p = b.count - 1;  // the last p with row_begin[p] <= r
    while (lo_p < hi_p) {
        const int mid = (lo_p + hi_p + 1) >> 1;
        if (b.row_begin[mid] <= r) lo_p = mid;
        else hi_p = mid - 1;
    }
    const Q8TcItem& it = b.items[lo_p];
    const size_t row = static_cast<size_t>(r - b.row_begin[lo_p]);
    split_row<Bulk>(it.k, it.A + row * it.k, nullptr, it.hi + row * it.kp, it.lo + row * it.kp,
                    nullptr, it.row_scale + row, split_smem);
    pdl_launch_dependents();  // as in split_rows_kernel: the GEMM's CTAs only after this row
}

}  // namespace

namespace {
// Both GEMM instantiations may use kSmemBytes of dynamic shared memory (once per device).
cudaError_t configure_smem() {
    static std::atomic<unsigned long long> configured{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && (configured.load() >> dev & 1ull)) return cudaSuccess;
    e = cudaFuncSetAttribute(gemm_q8_tc_kernel<false, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, Geo<false>::kSmemBytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemm_q8_tc_kernel<true, false>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, Geo<false>::kSmemBytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemm_q8_tc_kernel<false, true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, Geo<true>::kSmemBytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemm_q8_tc_kernel<true, true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, Geo<true>::kSmemBytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(split_rows_kernel<true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, kSplitSmemMax);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(split_rows_batch_kernel<true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, kSplitSmemMax);
    if (e == cudaSuccess && dev < 64) configured.fetch_or(1ull << dev);
    return e;
}
}  // namespace

int q8tc_tile_m() { return TBT; }
int q8tc_tile_n(bool pair) { return pair ? 2 * TBW : TBW; }

namespace {
// The GEMM launch (G: grouped): `slots` scheduling slots, each one CTA or (pair) a cluster of
// two CTAs; PDL after the split launch.
template <bool G>
cudaError_t launch_gemm(int slots, bool pair, cudaStream_t stream, const CUtensorMap& tmHi,
                        const CUtensorMap& tmLo, const CUtensorMap& tmB, const Q8TcArgs& a,
                        const Q8TcBatchArgs& b) {
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = pair ? 2 : 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(slots * (pair ? 2 : 1));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = pair ? Geo<true>::kSmemBytes : Geo<false>::kSmemBytes;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = pair ? 2 : 1;
    return pair ? cudaLaunchKernelEx(&cfg, gemm_q8_tc_kernel<G, true>, tmHi, tmLo, tmB, a, b)
                : cudaLaunchKernelEx(&cfg, gemm_q8_tc_kernel<G, false>, tmHi, tmLo, tmB, a, b);
}
}  // namespace

cudaError_t launch_split_rows(int m, int k, int kp, const float* A, const float* w, int8_t* hi,
                              int8_t* lo, int8_t* t2, float* row_scale, cudaStream_t stream,
                              bool pdl) {
    cudaError_t e = configure_smem();
    if (e != cudaSuccess) return e;
    // Bulk copies need 16-byte aligned rows (and norm weights) and a row that fits.
    const bool bulk = k % 4 == 0 && reinterpret_cast<uintptr_t>(A) % 16 == 0 &&
                      (w == nullptr || reinterpret_cast<uintptr_t>(w) % 16 == 0) &&
                      static_cast<size_t>(k) * 4 <= static_cast<size_t>(kSplitSmemMax);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(m);
    cfg.blockDim = dim3(kSplitThreads);
    cfg.dynamicSmemBytes = bulk ? static_cast<size_t>(k) * 4 : 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return bulk ? cudaLaunchKernelEx(&cfg, split_rows_kernel<true>, k, kp, A, w, hi, lo, t2,
                                     row_scale)
                : cudaLaunchKernelEx(&cfg, split_rows_kernel<false>, k, kp, A, w, hi, lo, t2,
                                     row_scale);
}

cudaError_t launch_gemm_q8_tc(const Q8TcArgs& a, const CUtensorMap& tmHi, const CUtensorMap& tmLo,
                              const CUtensorMap& tmB) {
    cudaError_t e = configure_smem();
    if (e != cudaSuccess) return e;
    const int tile_w = q8tc_tile_n(a.pair);
    const int tiles = ((a.m + TBT - 1) / TBT) * ((a.n + tile_w - 1) / tile_w);
    return launch_gemm<false>(std::max(1, std::min(tiles, a.slots)), a.pair, a.stream, tmHi, tmLo,
                              tmB, a, Q8TcBatchArgs{});
}

cudaError_t launch_q8tc_batch(const Q8TcBatchArgs& b) {
    cudaError_t e = configure_smem();
    if (e != cudaSuccess) return e;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(b.rows);
    cfg.blockDim = dim3(kSplitThreads);
    cfg.dynamicSmemBytes = b.bulk ? static_cast<size_t>(b.max_k) * 4 : 0;
    cfg.stream = b.stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = b.bulk ? cudaLaunchKernelEx(&cfg, split_rows_batch_kernel<true>, b)
               : cudaLaunchKernelEx(&cfg, split_rows_batch_kernel<false>, b);
    if (e != cudaSuccess) return e;
    // The tensor maps are read from the batch's device memory; these are placeholders.
    CUtensorMap none;
    memset(&none, 0, sizeof(none));
    return launch_gemm<true>(b.slots, b.pair, b.stream, none, none, none, Q8TcArgs{}, b);
}

unsigned read_and_clear_q8tc_error() {
    unsigned v = 0, w = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_q8tc_error, sizeof(v)) != cudaSuccess) return 0;
    if (v) cudaMemcpyToSymbol(g_q8tc_error, &zero, sizeof(zero));
    if (cudaMemcpyFromSymbol(&w, g_split_error, sizeof(w)) != cudaSuccess) return v;
    if (w) cudaMemcpyToSymbol(g_split_error, &zero, sizeof(zero));
    return v | w;
}

}  // namespace llme
