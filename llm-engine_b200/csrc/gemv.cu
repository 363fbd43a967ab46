// Weight-streaming GEMV / skinny GEMM for decode-shaped products (m <= 8, and fp32 B up to
// 16 rows): C (+)= [rmsnorm(A)] x B, B fp32 or int8 k x n row-major with column scales.
//
// The reference's counterpart is sgemm_skinny + sum_slices
// (src/cuda_matmul.cu:189-254, launched by run_skinny :365-397). This design
// is B200-first rather than a translation:
//
//  * B is streamed by TMA (cp.async.bulk.tensor.2d) in 128-row x 128-byte
//    boxes into a 4-stage shared-memory ring per CTA; one producer thread
//    keeps every stage in flight (a 512-row slice is requested whole at
//    launch). A (and the RMSNorm weight) ride in the same stage as small
//    boxes, so the consumers never touch global memory in the hot loop.
//    Weights use an L2 evict-first policy.
//  * k is split across the CTAs of a thread-block cluster (up to 8, grid.y):
//    each CTA reduces its slice in shared memory, then cluster rank 0 adds
//    the slices through distributed shared memory in rank order. No global
//    scratch, fence or atomic sits on the critical path, and repeats are
//    bit-identical.
//  * With programmatic dependent launch the producer issues the first stages
//    of weights before griddepcontrol.wait, overlapping the previous kernel's
//    tail; A and C are touched only after the wait.
//  * int8 is widened without I2F: a PRMT builds 2^23 + (q + 128) as a float
//    and a packed f32x2 add removes the bias (exact); products accumulate with
//    packed fma.rn.f32x2 (bitwise the same as two fmaf). Raw int8 values are
//    summed and each column scaled once at the end, as the reference does.
//  * RMSNorm is applied as an epilogue scale: each CTA sums a*a over its own
//    k rows while it streams, multiplies A by the norm weight in the loop, and
//    the final per-row 1/sqrt(mean + eps) multiplies the reduced sums -- no
//    pre-pass and no second read of A.
//  * fp32 B with 9..16 rows (one M = 16 instantiation; A rows past m arrive as the
//    TMA's zero fill and their outputs are not stored) keeps 16 x 2 outputs per
//    thread and pairs each output's accumulator over even and odd k instead of
//    over columns: a 16-byte load of A gives two k pairs of one row, used as they
//    are by fma.rn.f32x2 against the column's k pairs of B, so A needs no
//    repacking and each A load feeds four packed FMAs. It has no fused RMSNorm
//    (the caller's row pass normalises A first).
#include "common.cuh"
#include "kernels.h"

namespace llme {
namespace {

__device__ unsigned int g_gemv_error;

#ifdef LLME_GEMV_TRACE
#define GEMV_TRACE(a, point) \
    (a).trace[(static_cast<size_t>(blockIdx.y) * gridDim.x + blockIdx.x) * 16 + (point)] = global_timer_ns()
#else
#define GEMV_TRACE(a, point) ((void)0)
#endif

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kTmaThreads = kConsumers + 32;  // + one producer warp
constexpr int kStages = 4;
constexpr int kBoxBytesB = kGemvRowBytes * kGemvBoxRows;  // 16 KB

// Per-thread work split of one 128-byte row segment of B over `Warps` consumer warps.
template <int M, bool Q8, int Warps = kConsumerWarps>
struct Shape {
    static constexpr int ESZ = Q8 ? 1 : 4;
    // fp32 B past 8 rows: accumulators paired over k (two columns per thread, four
    // consecutive k rows at a time) instead of over columns.
    static constexpr bool KQ = !Q8 && M > 8;
    // Columns per thread: fewer as M grows, so M x V accumulators fit 2 CTAs per SM.
    static constexpr int V = Q8 ? (M <= 2 ? 16 : (M <= 4 ? 8 : 4)) : (KQ ? 2 : 4);
    static constexpr int ACC = KQ ? V : V / 2;              // 64-bit accumulators per row
    static constexpr int NT = kGemvRowBytes / ESZ;         // columns per CTA
    static constexpr int TPR = NT / V;                     // threads per row
    static constexpr int RG = Warps * 32 / TPR;            // row groups
    static constexpr int RPT = kGemvBoxRows / RG;          // rows per thread per box
    static constexpr int QPT = RPT / 4;                    // k-quad form: quads per thread
    static_assert(TPR == 8 || TPR == 16 || TPR == 32, "row split");
    static_assert(KQ ? (V == 2 && M <= 16 && RPT % 4 == 0) : V % 4 == 0, "packed pairs");
    static_assert(RPT * RG == kGemvBoxRows, "rows split evenly");
};

// The per-call kernel runs two CTAs per SM, each with a ring deep enough to hold the whole
// k-slice of the chain's 4096-deep products (6 boxes for m <= 2), requested before
// griddepcontrol.wait; CTAs of the next call that find room start early and stage their weights
// while this call computes, and the earliest one prefetches the next call's whole weight matrix
// into L2 so the CTAs that start later read it from there.
template <int M>
constexpr int call_warps() { return kConsumerWarps; }
template <int M>
constexpr int call_threads() { return call_warps<M>() * 32 + 32; }
constexpr int kCallResidentCtas = 2;
constexpr int kCallSmemBudget = 110 * 1024;
// Boxes a CTA prefetches into L2 beyond its ring (a sliding window).
constexpr int kPrefetchBoxes = 8;
// Weight matrices up to this size are prefetched into L2 whole by the first CTA of the call.
constexpr size_t kWholePrefetchMaxBytes = size_t{48} << 20;
constexpr uint32_t kWholePrefetchChunk = 1u << 20;

template <int M, bool Q8, bool Norm>
struct Layout {
    using Sh = Shape<M, Q8, call_warps<M>()>;
    static constexpr int CW = call_warps<M>();
    static constexpr int kABox = M * kGemvBoxRows * 4;
    static constexpr int kWBox = kGemvBoxRows * 4;
    static constexpr int kStageBytes = kBoxBytesB + kABox + (Norm ? kWBox : 0);
    // The cluster reduction's receive area: every slice's share of the strip's sums (at most
    // M x NT + 4 x slices floats over all senders), then their RMSNorm sums of squares.
    static constexpr int kRecvFloats = M * Sh::NT + 4 * kGemvMaxCluster + kGemvMaxCluster * M;
    static constexpr int kFixedBytes =
        (Q8 ? Sh::NT * 4 : 0) + 2 * 8 * 8 + 16 + 16 + kRecvFloats * 4;
    static constexpr int kBudget = kCallSmemBudget;
    // Ring depth: as many stages as the budget holds (6 for m <= 2, 5 for m = 8), at most 8.
    static constexpr int kRing = (kBudget - kFixedBytes) / kStageBytes < 8
                                 ? (kBudget - kFixedBytes) / kStageBytes
                                 : 8;
    static constexpr int kB = kRing * kBoxBytesB;
    static constexpr int kOffA = kB;
    static constexpr int kOffW = kOffA + kRing * kABox;
    static constexpr int kOffScale = kOffW + (Norm ? kRing * kWBox : 0);  // NT floats (int8)
    static constexpr int kOffBar = kOffScale + (Q8 ? Sh::NT * 4 : 0);
    static constexpr int kOffRedBar = kOffBar + 2 * kRing * 8;
    static constexpr int kOffRecv = kOffRedBar + 16;
    static constexpr int kBytes = kOffRecv + kRecvFloats * 4;
    static constexpr uint32_t kTx = kBoxBytesB + kABox + (Norm ? kWBox : 0);
    // Reduction buffers reuse the drained ring.
    static constexpr int kRedFloats = CW * M * Sh::NT;
    static_assert(kRing >= 3, "ring depth");
    static_assert(kBytes <= kBudget, "the CTA's share of the SM");
    static_assert((kRedFloats + M * Sh::NT) * 4 <= kB, "reduction fits in the ring");
    static_assert((CW + 2) * M * 4 <= kRing * kABox, "ss reduction fits");
};

// ---- packed f32x2 arithmetic (sm_100) ---------------------------------------------------
__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void unpack2(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// Four signed bytes -> two exact f32x2 pairs (see s8x4_to_f32 in common.cuh).
__device__ __forceinline__ void s8x4_to_f32x2(uint32_t w, uint64_t& p01, uint64_t& p23) {
    const uint32_t u = w ^ 0x80808080u;
    constexpr float kBias = -8388736.0f;  // -(2^23 + 128)
    const uint64_t bias = pack2(kBias, kBias);
    p01 = add2(pack2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)),
                     __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541))),
               bias);
    p23 = add2(pack2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)),
                     __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543))),
               bias);
}

// V columns of one row of B (at p, shared memory) as V/2 f32x2 pairs.
template <bool Q8, int V>
__device__ __forceinline__ void load_pairs(const uint8_t* p, uint64_t (&x)[V / 2]) {
    if constexpr (Q8) {
        if constexpr (V == 16) {
            const uint4 q = *reinterpret_cast<const uint4*>(p);
            s8x4_to_f32x2(q.x, x[0], x[1]);
            s8x4_to_f32x2(q.y, x[2], x[3]);
            s8x4_to_f32x2(q.z, x[4], x[5]);
            s8x4_to_f32x2(q.w, x[6], x[7]);
        } else if constexpr (V == 8) {
            const uint2 q = *reinterpret_cast<const uint2*>(p);
            s8x4_to_f32x2(q.x, x[0], x[1]);
            s8x4_to_f32x2(q.y, x[2], x[3]);
        } else {
            static_assert(V == 4, "int8 columns per thread");
            s8x4_to_f32x2(*reinterpret_cast<const uint32_t*>(p), x[0], x[1]);
        }
    } else {
        static_assert(V == 4, "fp32 columns per thread");
        const ulonglong2 f = *reinterpret_cast<const ulonglong2*>(p);
        x[0] = f.x;
        x[1] = f.y;
    }
}

// ---- thread-block cluster helpers ---------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// A cluster-wide rendezvous with no memory ordering: only "nobody leaves yet". A release arrive
// would first wait for this CTA's global stores to be acknowledged (~1 us here).
__device__ __forceinline__ void cluster_sync_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::
                     : "memory");
}
// A rendezvous split in two: arrive early (after initialising the barriers other CTAs
// will signal), wait late (before signalling them).
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}
// The shared::cluster address of this CTA's shared `local` in cluster CTA `rank`.
__device__ __forceinline__ uint32_t cluster_addr(const void* local, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
    return remote;
}
// Asynchronous stores into another cluster CTA's shared memory, counted in bytes on that CTA's
// mbarrier `bar` (both shared::cluster addresses).
__device__ __forceinline__ void st_async_f4(uint32_t dst, float4 v, uint32_t bar) {
    asm volatile(
        "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
            dst),
        "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void st_async_f(uint32_t dst, float v, uint32_t bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(dst),
                 "f"(v), "r"(bar)
                 : "memory");
}
// Brings `bytes` (a multiple of 16, 16-byte aligned start) of global memory into L2.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(p)),
                 "r"(bytes)
                 : "memory");
}
// The fused epilogues (GemvEpilogue): a finished pair of adjacent output columns (col even)
// of row r, already scaled.
__device__ __forceinline__ void epilogue_pair(const GemvArgs& a, int r, int col, float v0, float v1) {
    const GemvEpilogue& e = a.epi;
    if (e.kind == kEpiSwiglu) {
        const float sig = 1.0f / (1.0f + expf(-v0));
        e.out[static_cast<size_t>(r) * (a.n / 2) + col / 2] = v0 * sig * v1;
        return;
    }
    // kEpiRopeCache
    const int hs = e.head_size, head = col / hs;
    const int pos = e.feed[0] + r;
    const size_t kvd = static_cast<size_t>(e.nkv) * hs;
    const int qd = e.nq * hs;
    if (head < e.nq + e.nkv) {
        const int j = (col % hs) / 2;
        const float c = e.cos[static_cast<size_t>(pos) * (hs / 2) + j];
        const float sn = e.sin[static_cast<size_t>(pos) * (hs / 2) + j];
        const float r0 = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, sn));
        const float r1 = __fadd_rn(__fmul_rn(v0, sn), __fmul_rn(v1, c));
        v0 = r0;
        v1 = r1;
        if (head >= e.nq)
            *reinterpret_cast<float2*>(e.key_cache + static_cast<size_t>(pos) * kvd + (col - qd)) =
                make_float2(v0, v1);
    } else {
        *reinterpret_cast<float2*>(e.value_cache + static_cast<size_t>(pos) * kvd +
                                   (col - qd - static_cast<int>(kvd))) = make_float2(v0, v1);
    }
    *reinterpret_cast<float2*>(a.C + static_cast<size_t>(r) * a.n + col) = make_float2(v0, v1);
}

// ---- kEpiPeerSum: the row-parallel sum over the ranks, inside the GEMV ----------------------

__device__ __forceinline__ unsigned long long* peer_region(const PeerSum& p, int q, unsigned slot,
                                                           int unit, int src) {
    return p.base[q] + ((static_cast<size_t>(slot) * p.units + unit) * p.world + src) * p.unit_words;
}

// The `count` values this CTA owns, exchanged with the same CTA of every rank and summed in
// rank order into C. value(e) is owned element e's finished value (partial, scaled), where(e,
// r, col) its place in C (col >= n: padding, skipped). Every one of the nthreads consumer
// threads calls this; `state` is a word of this CTA's shared memory. A thread reads back only
// the elements it wrote, so after the epoch is known no barrier is needed.
template <typename Value, typename Where>
__device__ __forceinline__ void peer_sum_store(const GemvArgs& a, int count, Value value, Where where,
                                               unsigned* state, int tid, int nthreads) {
    const PeerSum& p = a.epi.peer;
    const int unit = blockIdx.y * gridDim.x + blockIdx.x;
    if (tid == 0) {
        const unsigned e = __ldcg(p.epoch + unit) + 1;
        p.epoch[unit] = e;
        state[0] = e;
    }
    named_barrier(1, nthreads);
    const unsigned epoch = state[0];
    const unsigned slot = epoch & 1u;
    for (int e = tid; e < count; e += nthreads) {
        int r, col;
        where(e, r, col);
        if (col >= a.n || r >= a.m) continue;  // past n, or a zero-filled row past m
        float v = value(e);
        float* o = a.C + static_cast<size_t>(r) * a.n + col;
        if (a.accumulate) v += *o;
        const unsigned long long w = tagged(v, epoch);
        for (int q = 0; q < p.world; ++q) st_relaxed_sys_u64(peer_region(p, q, slot, unit, p.rank) + e, w);
    }
    for (int e = tid; e < count; e += nthreads) {
        int r, col;
        where(e, r, col);
        if (col >= a.n || r >= a.m) continue;  // past n, or a zero-filled row past m
        float v = wait_tagged(peer_region(p, p.rank, slot, unit, 0) + e, epoch, p.err);
        for (int src = 1; src < p.world; ++src)
            v += wait_tagged(peer_region(p, p.rank, slot, unit, src) + e, epoch, p.err);
        a.C[static_cast<size_t>(r) * a.n + col] = v;
    }
}

// Writes C for a CTA's column strip from M x NT sums that are already complete
// (tot, shared memory) -- the kernels' common epilogue.
// sscale: the strip's column scales already in shared memory (int8 TMA kernel), or null to
// read them from global memory.
template <int M, int NT, bool Q8, bool Norm>
__device__ __forceinline__ void store_strip(const float* tot, const float* tot_ss, const GemvArgs& a,
                                            int col0, int tid, int nthreads,
                                            const float* sscale = nullptr,
                                            unsigned* peer_state = nullptr) {
    if (a.epi.kind == kEpiPeerSum && peer_state) {
        auto value = [&](int e) {
            float v = tot[e];
            if constexpr (Q8) v *= sscale ? sscale[e % NT] : __ldg(a.scale + col0 + e % NT);
            if constexpr (Norm) v *= 1.0f / sqrtf(tot_ss[e / NT] / static_cast<float>(a.k) + kRmsEps);
            return v;
        };
        auto where = [&](int e, int& r, int& col) {
            r = e / NT;
            col = col0 + e % NT;
        };
        peer_sum_store(a, M * NT, value, where, peer_state, tid, nthreads);
        return;
    }
    if (a.epi.kind != kEpiStore) {
        for (int e = 2 * tid; e < M * NT; e += 2 * nthreads) {
            const int r = e / NT, col = col0 + e % NT;
            if (col >= a.n || r >= a.m) continue;  // past n, or a zero-filled row past m
            float v0 = tot[e], v1 = tot[e + 1];
            if constexpr (Q8) {
                v0 *= sscale ? sscale[e % NT] : __ldg(a.scale + col);
                v1 *= sscale ? sscale[e % NT + 1] : __ldg(a.scale + col + 1);
            }
            if constexpr (Norm) {
                const float inv = 1.0f / sqrtf(tot_ss[r] / static_cast<float>(a.k) + kRmsEps);
                v0 *= inv;
                v1 *= inv;
            }
            epilogue_pair(a, r, col, v0, v1);
        }
        return;
    }
    for (int e = tid; e < M * NT; e += nthreads) {
        const int r = e / NT, col = col0 + e % NT;
        if (col >= a.n || r >= a.m) continue;  // past n, or a zero-filled row past m
        float v = tot[e];
        if constexpr (Q8) v *= sscale ? sscale[e % NT] : __ldg(a.scale + col);
        if constexpr (Norm) v *= 1.0f / sqrtf(tot_ss[r] / static_cast<float>(a.k) + kRmsEps);
        float* out = a.C + static_cast<size_t>(r) * a.n + col;
        *out = a.accumulate ? *out + v : v;
    }
}

template <int M, bool Q8, bool Norm>
__global__ void __launch_bounds__(call_threads<M>(), kCallResidentCtas)
    gemv_tma_kernel(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmA,
                    const __grid_constant__ CUtensorMap tmW, const GemvArgs a) {
    using L = Layout<M, Q8, Norm>;
    using S = typename L::Sh;
    constexpr int CW = L::CW;        // consumer warps
    constexpr int CT = L::CW * 32;   // consumer threads
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
    uint64_t* empty = full + L::kRing;
    constexpr int R = L::kRing;  // ring depth

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int strip = blockIdx.x, slice = blockIdx.y;  // grid.y = slices = cluster size
    const int col0 = strip * S::NT;
    const int k0 = slice * a.span;
    const int k1 = min(a.k, k0 + a.span);
    const int nb = (k1 - k0 + kGemvBoxRows - 1) / kGemvBoxRows;

    if (tid == 0) GEMV_TRACE(a, 0);
    uint64_t* rbar = reinterpret_cast<uint64_t*>(smem + L::kOffRedBar);
    if (tid == CT) {
        for (int s = 0; s < R; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CW);
        }
        mbar_init(rbar, 1);
        fence_mbar_init();
        prefetch_tensormap(&tmB);
        prefetch_tensormap(&tmA);
        if (Norm) prefetch_tensormap(&tmW);
    }
    __syncthreads();
    // The slices of a strip push their sums into each other's shared memory at the end; the
    // rendezvous that makes every CTA's reduction barrier visible is opened here and closed
    // only just before the first push.
    if (a.slices > 1) cluster_arrive_relaxed();
    if (tid == 0) {
        pdl_launch_dependents();
        GEMV_TRACE(a, 1);
    }

    float* red = reinterpret_cast<float*>(smem);
    float* tot = red + L::kRedFloats;
    float* red_ss = reinterpret_cast<float*>(smem + L::kOffA);
    float* tot_ss = red_ss + CW * M;

    if (warp == CW) {
        // Producer. Everything before griddepcontrol.wait touches weights only: with static
        // weights the first R boxes go straight into the ring, and in every case the next
        // kPrefetchBoxes boxes are prefetched into L2 (a hint, safe whatever wrote them), so
        // this CTA's weights stream from HBM while the previous launch still computes. A and
        // the RMSNorm weight are loaded only after the wait.
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            const int pro = min(nb, R);
            const int pf_end = min(nb, pro + kPrefetchBoxes);
            if (a.weights_static)
                for (int b = 0; b < pro; ++b) {
                    mbar_arrive_expect_tx(&full[b], L::kTx);
                    tma_load_2d(smem + b * kBoxBytesB, &tmB, col0, k0 + b * kGemvBoxRows, &full[b], pol);
                }
            for (int b = a.weights_static ? pro : 0; b < pf_end; ++b)
                tma_prefetch_l2_2d(&tmB, col0, k0 + b * kGemvBoxRows);
            // The first CTA to start brings the whole weight matrix into L2 (when it is not too
            // large for it), so CTAs that become resident only after the previous call ends
            // find their boxes in L2 instead of waiting on HBM.
            const size_t wbytes = static_cast<size_t>(a.k) * a.n * S::ESZ;
            if (blockIdx.x == 0 && blockIdx.y == 0 && wbytes <= kWholePrefetchMaxBytes)
                for (size_t off = 0; off < wbytes; off += kWholePrefetchChunk)
                    prefetch_l2_bulk(static_cast<const uint8_t*>(a.B) + off,
                                     wbytes - off < kWholePrefetchChunk
                                         ? static_cast<uint32_t>(wbytes - off)
                                         : kWholePrefetchChunk);
            GEMV_TRACE(a, 2);
            pdl_wait();
            for (int b = 0; b < pro; ++b) {
                if (!a.weights_static) {
                    mbar_arrive_expect_tx(&full[b], L::kTx);
                    tma_load_2d(smem + b * kBoxBytesB, &tmB, col0, k0 + b * kGemvBoxRows, &full[b], pol);
                }
                tma_load_2d_nohint(smem + L::kOffA + b * L::kABox, &tmA, k0 + b * kGemvBoxRows, 0,
                                   &full[b]);
                if (Norm)
                    tma_load_1d(smem + L::kOffW + b * L::kWBox, &tmW, k0 + b * kGemvBoxRows,
                                &full[b]);
            }
            GEMV_TRACE(a, 3);
            for (int b = pro; b < nb; ++b) {
                const int s = b % R;
                if (!mbar_wait(&empty[s], ((b / R) - 1) & 1, &g_gemv_error)) break;
                mbar_arrive_expect_tx(&full[s], L::kTx);
                const int y = k0 + b * kGemvBoxRows;
                tma_load_2d(smem + s * kBoxBytesB, &tmB, col0, y, &full[s], pol);
                tma_load_2d_nohint(smem + L::kOffA + s * L::kABox, &tmA, y, 0, &full[s]);
                if (Norm) tma_load_1d(smem + L::kOffW + s * L::kWBox, &tmW, y, &full[s]);
                if (b + kPrefetchBoxes < nb)
                    tma_prefetch_l2_2d(&tmB, col0, k0 + (b + kPrefetchBoxes) * kGemvBoxRows);
            }
        }
        __syncwarp();
    } else {
        // The strip's column scales are weights too: with static weights they are fetched
        // before waiting for the previous launch, so the epilogue never waits on DRAM for them.
        float* sscale = reinterpret_cast<float*>(smem + L::kOffScale);
        if constexpr (Q8)
            if (a.weights_static && tid < S::NT)
                sscale[tid] = col0 + tid < a.n ? __ldg(a.scale + col0 + tid) : 0.0f;
        // Consumers: C is touched only after this.
        pdl_wait();
        if constexpr (Q8)
            if (!a.weights_static && tid < S::NT)
                sscale[tid] = col0 + tid < a.n ? __ldg(a.scale + col0 + tid) : 0.0f;
        const int cg = tid % S::TPR, rg = tid / S::TPR;
        uint64_t acc[M][S::ACC];
        float ss[M];
        static_assert(!(S::KQ && Norm), "the k-quad form has no fused RMSNorm");
#pragma unroll
        for (int r = 0; r < M; ++r) {
            ss[r] = 0.0f;
#pragma unroll
            for (int j = 0; j < S::ACC; ++j) acc[r][j] = 0ull;
        }
        for (int b = 0; b < nb; ++b) {
            const int s = b % R;
            if (!mbar_wait(&full[s], (b / R) & 1, &g_gemv_error)) break;
            if (tid == 0 && b == 0) GEMV_TRACE(a, 4);
            const uint8_t* sb = smem + s * kBoxBytesB + cg * (S::V * S::ESZ);
            const float* sa = reinterpret_cast<const float*>(smem + L::kOffA + s * L::kABox);
            const float* sw = reinterpret_cast<const float*>(smem + L::kOffW + s * L::kWBox);
            if constexpr (S::KQ) {
                // Quads q = rg, rg + RG, ...: k rows 4q .. 4q + 3, columns 2 cg, 2 cg + 1.
#pragma unroll 1
                for (int i = 0; i < S::QPT; ++i) {
                    const int k4 = 4 * (rg + i * S::RG);
                    float2 bv[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        bv[j] = *reinterpret_cast<const float2*>(sb + (k4 + j) * kGemvRowBytes);
                    // One column's (k, k + 1) and (k + 2, k + 3) pairs of B.
                    const uint64_t c0lo = pack2(bv[0].x, bv[1].x), c0hi = pack2(bv[2].x, bv[3].x);
                    const uint64_t c1lo = pack2(bv[0].y, bv[1].y), c1hi = pack2(bv[2].y, bv[3].y);
#pragma unroll
                    for (int r = 0; r < M; ++r) {
                        const ulonglong2 aq =
                            *reinterpret_cast<const ulonglong2*>(sa + r * kGemvBoxRows + k4);
                        const uint64_t alo = aq.x, ahi = aq.y;
                        acc[r][0] = fma2(alo, c0lo, acc[r][0]);
                        acc[r][1] = fma2(alo, c1lo, acc[r][1]);
                        acc[r][0] = fma2(ahi, c0hi, acc[r][0]);
                        acc[r][1] = fma2(ahi, c1hi, acc[r][1]);
                    }
                }
            } else {
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
                    uint64_t x[S::V / 2];
                    load_pairs<Q8, S::V>(sb + row * kGemvRowBytes, x);
#pragma unroll
                    for (int r = 0; r < M; ++r) {
                        const uint64_t a2 = pack2(av[r], av[r]);
#pragma unroll
                        for (int j = 0; j < S::V / 2; ++j) acc[r][j] = fma2(a2, x[j], acc[r][j]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }

        // Reduce the row groups: inside a warp by shuffle, then the 8 warps
        // through shared memory (the drained ring), always in the same order.
        if (tid == 0) GEMV_TRACE(a, 5);
        named_barrier(1, CT);
        float accf[M][S::V];
#pragma unroll
        for (int r = 0; r < M; ++r) {
            if constexpr (S::KQ) {
                // Even-k and odd-k sums of each output.
#pragma unroll
                for (int j = 0; j < S::V; ++j) {
                    float lo, hi;
                    unpack2(acc[r][j], lo, hi);
                    accf[r][j] = lo + hi;
                }
            } else {
#pragma unroll
                for (int j = 0; j < S::V / 2; ++j)
                    unpack2(acc[r][j], accf[r][2 * j], accf[r][2 * j + 1]);
            }
        }
#pragma unroll
        for (int off = S::TPR; off < 32; off <<= 1) {
#pragma unroll
            for (int r = 0; r < M; ++r) {
                if constexpr (Norm) ss[r] += __shfl_xor_sync(0xffffffffu, ss[r], off);
#pragma unroll
                for (int j = 0; j < S::V; ++j) accf[r][j] += __shfl_xor_sync(0xffffffffu, accf[r][j], off);
            }
        }
        if (lane < S::TPR) {
#pragma unroll
            for (int r = 0; r < M; ++r) {
                float* dst = red + (warp * M + r) * S::NT + cg * S::V;
                if constexpr (S::V % 4 == 0) {
#pragma unroll
                    for (int j = 0; j < S::V / 4; ++j)
                        reinterpret_cast<float4*>(dst)[j] =
                            make_float4(accf[r][4 * j], accf[r][4 * j + 1], accf[r][4 * j + 2],
                                        accf[r][4 * j + 3]);
                } else {
                    *reinterpret_cast<float2*>(dst) = make_float2(accf[r][0], accf[r][1]);
                }
            }
            if (Norm && cg == 0) {
#pragma unroll
                for (int r = 0; r < M; ++r) red_ss[warp * M + r] = ss[r];
            }
        }
        named_barrier(1, CT);
        for (int e = tid; e < M * S::NT; e += CT) {
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < CW; ++w) v += red[w * M * S::NT + e];
            tot[e] = v;
        }
        if (Norm && tid < M) {
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < CW; ++w) v += red_ss[w * M + tid];
            tot_ss[tid] = v;
        }
        if (tid == 0) GEMV_TRACE(a, 6);
        if (a.slices == 1) {
            named_barrier(1, CT);
            store_strip<M, S::NT, Q8, Norm>(tot, tot_ss, a, col0, tid, CT,
                                            reinterpret_cast<const float*>(smem + L::kOffScale),
                                            reinterpret_cast<unsigned*>(smem + L::kOffRedBar + 8));
            if (tid == 0) GEMV_TRACE(a, 7);
        }
    }
    if (a.slices == 1) return;
    __syncwarp();

    // k split across the cluster: every CTA finishes 1/slices of the strip's columns. Each
    // slice pushes its sums for a column chunk into the owning CTA's receive area with
    // st.async, counted on the owner's reduction barrier; the owner adds the slices in rank
    // order. The closing rendezvous keeps every CTA alive until all pushes have landed.
    cluster_wait();
    if (tid == 0) GEMV_TRACE(a, 8);
    if (tid < CT) {
        const uint32_t me = cluster_rank();
        constexpr int E4 = M * S::NT / 4;  // float4 chunks of the strip's sums
        const int per = (E4 + a.slices - 1) / a.slices;
        const int my_begin = static_cast<int>(me) * per;
        const int my_cnt = max(0, min(E4, my_begin + per) - my_begin);
        float* recv = reinterpret_cast<float*>(smem + L::kOffRecv);         // [slice][per * 4]
        float* recv_ss = recv + M * S::NT + 4 * kGemvMaxCluster;             // [slice][M]
        if (tid == 0)
            mbar_arrive_expect_tx(rbar, static_cast<uint32_t>((a.slices - 1) *
                                                              (my_cnt * 16 + (Norm ? M * 4 : 0))));
        // tot was written by other consumer threads (element e by thread e % CT); the cluster
        // wait above orders nothing inside this CTA.
        named_barrier(1, CT);
        for (int e4 = tid; e4 < E4; e4 += CT) {
            const int owner = e4 / per;
            const float4 v = *reinterpret_cast<const float4*>(tot + 4 * e4);
            float* dst = recv + (static_cast<int>(me) * per + (e4 - owner * per)) * 4;
            if (owner == static_cast<int>(me))
                *reinterpret_cast<float4*>(dst) = v;
            else
                st_async_f4(cluster_addr(dst, owner), v, cluster_addr(rbar, owner));
        }
        if (Norm && tid < M) {
            float* dst = recv_ss + me * M + tid;
            for (int r = 0; r < a.slices; ++r) {
                if (r == static_cast<int>(me))
                    *dst = tot_ss[tid];
                else
                    st_async_f(cluster_addr(dst, r), tot_ss[tid], cluster_addr(rbar, r));
            }
        }
        named_barrier(1, CT);
        const bool ok = mbar_wait_cluster(rbar, 0, &g_gemv_error);
        if (tid == 0) GEMV_TRACE(a, 9);
        const float* sc = reinterpret_cast<const float*>(smem + L::kOffScale);
        if (a.epi.kind == kEpiPeerSum) {
            // Every consumer thread takes part (the exchange has barriers), also when the
            // cluster reduction gave up (the error word is set; the values are then not used).
            auto value = [&](int e) {
                const int eg = 4 * my_begin + e;
                float v = recv[e];
                for (int src = 1; src < a.slices; ++src) v += recv[src * per * 4 + e];
                if constexpr (Q8) v *= sc[eg % S::NT];
                if constexpr (Norm) {
                    const int r = eg / S::NT;
                    float ssum = recv_ss[r];
                    for (int src = 1; src < a.slices; ++src) ssum += recv_ss[src * M + r];
                    v *= 1.0f / sqrtf(ssum / static_cast<float>(a.k) + kRmsEps);
                }
                return ok ? v : 0.0f;
            };
            auto where = [&](int e, int& r, int& col) {
                const int eg = 4 * my_begin + e;
                r = eg / S::NT;
                col = col0 + eg % S::NT;
            };
            peer_sum_store(a, 4 * my_cnt, value, where,
                           reinterpret_cast<unsigned*>(smem + L::kOffRedBar + 8), tid, CT);
        }
        // Fused epilogues work on pairs of columns; chunks start at multiples of four
        // elements, so a pair never straddles two owners.
        for (int e = 2 * tid; a.epi.kind != kEpiStore && a.epi.kind != kEpiPeerSum && ok &&
                              e < 4 * my_cnt; e += 2 * CT) {
            const int eg = 4 * my_begin + e;
            const int r = eg / S::NT, col = col0 + eg % S::NT;
            if (col >= a.n || r >= a.m) continue;  // past n, or a zero-filled row past m
            float v0 = recv[e], v1 = recv[e + 1];
            for (int src = 1; src < a.slices; ++src) {
                v0 += recv[src * per * 4 + e];
                v1 += recv[src * per * 4 + e + 1];
            }
            if constexpr (Q8) {
                v0 *= sc[eg % S::NT];
                v1 *= sc[eg % S::NT + 1];
            }
            if constexpr (Norm) {
                float ssum = recv_ss[r];
                for (int src = 1; src < a.slices; ++src) ssum += recv_ss[src * M + r];
                const float inv = 1.0f / sqrtf(ssum / static_cast<float>(a.k) + kRmsEps);
                v0 *= inv;
                v1 *= inv;
            }
            epilogue_pair(a, r, col, v0, v1);
        }
        for (int e = tid; a.epi.kind == kEpiStore && ok && e < 4 * my_cnt; e += CT) {
            const int eg = 4 * my_begin + e;  // element of the strip's M x NT sums
            const int r = eg / S::NT, col = col0 + eg % S::NT;
            if (col >= a.n || r >= a.m) continue;  // past n, or a zero-filled row past m
            float v = recv[e];
            for (int src = 1; src < a.slices; ++src) v += recv[src * per * 4 + e];
            if constexpr (Q8) v *= sc[eg % S::NT];
            if constexpr (Norm) {
                float ssum = recv_ss[r];
                for (int src = 1; src < a.slices; ++src) ssum += recv_ss[src * M + r];
                v *= 1.0f / sqrtf(ssum / static_cast<float>(a.k) + kRmsEps);
            }
            float* o = a.C + static_cast<size_t>(r) * a.n + col;
            *o = a.accumulate ? *o + v : v;
        }
        if (tid == 0) GEMV_TRACE(a, 10);
    }
    __syncwarp();
    cluster_sync_relaxed();
    if (tid == 0) GEMV_TRACE(a, 7);
}

// The plain-load kernel's k split: partials to scratch, a ticket per column
// strip, and the CTA that brings the count to `slices` adds the slices in index
// order (loads issued eight at a time so their latencies overlap), writes C and
// resets the ticket.
template <int M, int NT, bool Q8, bool Norm>
__device__ void finish_strip(const float* tot, const float* tot_ss, const GemvArgs& a, int strip,
                             int slice, int tid, int* flag, float* red, float* red_ss) {
    constexpr int E = M * NT;
    const int col0 = strip * NT;
    if (a.slices == 1) {
        store_strip<M, NT, Q8, Norm>(tot, tot_ss, a, col0, tid, kConsumers);
        return;
    }
    float* part = a.split.partial + (static_cast<size_t>(strip) * a.slices + slice) * E;
    for (int e = tid; e < E; e += kConsumers) __stcg(part + e, tot[e]);
    if (Norm && tid < M)
        __stcg(a.split.partial_ss + (static_cast<size_t>(strip) * a.slices + slice) * M + tid,
               tot_ss[tid]);
    __threadfence();
    __syncthreads();
    if (tid == 0)
        *flag = atomicAdd(a.split.counters + strip, 1u) == static_cast<unsigned>(a.slices - 1);
    __syncthreads();
    if (!*flag) return;
    __threadfence();
    const float* base = a.split.partial + static_cast<size_t>(strip) * a.slices * E;
    for (int e = tid; e < E; e += kConsumers) {
        float v = 0.0f;
        for (int s0 = 0; s0 < a.slices; s0 += 8) {
            float t[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
                t[i] = s0 + i < a.slices ? __ldcg(base + static_cast<size_t>(s0 + i) * E + e) : 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (s0 + i < a.slices) v += t[i];
        }
        red[e] = v;
    }
    if (Norm && tid < M) {
        float v = 0.0f;
        const float* ps = a.split.partial_ss + static_cast<size_t>(strip) * a.slices * M + tid;
        for (int s = 0; s < a.slices; ++s) v += __ldcg(ps + static_cast<size_t>(s) * M);
        red_ss[tid] = v;
    }
    __syncthreads();
    store_strip<M, NT, Q8, Norm>(red, red_ss, a, col0, tid, kConsumers);
    if (tid == 0) atomicExch(a.split.counters + strip, 0u);
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
    finish_strip<M, NT, Q8, Norm>(tot, tot_ss, a, strip, slice, tid, &flag, red, red_ss);
}

// ---- grouped GEMV: independent products in one persistent launch ---------------------------
//
// Every CTA walks its own list of (product, 128-column strip) units -- balanced by bytes
// when the batch is created -- over the whole k of each product, so there is no cross-CTA
// reduction at all; its producer thread streams the boxes of
// one unit after another through the same ring, so the ring never drains between products
// (the per-call kernel pays launch, griddepcontrol release and a cluster rendezvous per
// product). The reduction buffers therefore get their own shared memory. Used for products
// that do not read each other's outputs (a decode layer's independent projections; the
// benchmark's chain of fresh activations).
template <int M>
struct BatchLayout {
    using S = Shape<M, true>;
    static constexpr int kB = kStages * kBoxBytesB;
    static constexpr int kABox = M * kGemvBoxRows * 4;
    static constexpr int kOffA = kB;
    static constexpr int kOffRed = kOffA + kStages * kABox;
    static constexpr int kRedFloats = kConsumerWarps * M * S::NT;
    static constexpr int kOffTot = kOffRed + kRedFloats * 4;
    static constexpr int kOffBar = kOffTot + M * S::NT * 4;
    static constexpr int kOffPeer = kOffBar + 2 * kStages * 8 + 16;  // the rank sum's epoch, ok
    static constexpr int kBytes = kOffPeer + 16;
    static constexpr uint32_t kTx = kBoxBytesB + kABox;
};

template <int M>
__global__ void __launch_bounds__(kTmaThreads, 2) gemv_batch_kernel(const BatchArgs a) {
    using S = Shape<M, true>;
    using L = BatchLayout<M>;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
    uint64_t* empty = full + kStages;
    float* red = reinterpret_cast<float*>(smem + L::kOffRed);
    float* tot = reinterpret_cast<float*>(smem + L::kOffTot);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid == kConsumers) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) pdl_launch_dependents();

    if (warp == kConsumerWarps) {
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            // Box cursor over this CTA's units; the first kStages weight boxes are requested
            // before griddepcontrol.wait, their activation boxes after it.
            const int u_end = __ldg(a.cta_begin + blockIdx.x + 1);
            int u = __ldg(a.cta_begin + blockIdx.x), item = 0, strip = 0, j = 0, nb = 0;
            auto load_unit = [&]() {
                const unsigned code = __ldg(a.unit_table + u);
                item = static_cast<int>(code >> 16);
                strip = static_cast<int>(code & 0xFFFFu);
                nb = (__ldg(&a.items[item].k) + kGemvBoxRows - 1) / kGemvBoxRows;
                j = 0;
            };
            if (u < u_end) load_unit();
            int pend_item[kStages], pend_j[kStages];
            int b = 0;
            bool waited = false;
            while (u < u_end) {
                const int s = b % kStages;
                if (b >= kStages) {
                    if (!waited) {
                        pdl_wait();
                        for (int t = 0; t < kStages; ++t)
                            tma_load_2d_nohint(smem + L::kOffA + t * L::kABox, &a.tmA[pend_item[t]],
                                               pend_j[t] * kGemvBoxRows, 0, &full[t]);
                        waited = true;
                    }
                    if (!mbar_wait(&empty[s], ((b / kStages) - 1) & 1, &g_gemv_error)) break;
                }
                mbar_arrive_expect_tx(&full[s], L::kTx);
                tma_load_2d(smem + s * kBoxBytesB, &a.tmB[item], strip * S::NT, j * kGemvBoxRows,
                            &full[s], pol);
                if (waited) {
                    tma_load_2d_nohint(smem + L::kOffA + s * L::kABox, &a.tmA[item],
                                       j * kGemvBoxRows, 0, &full[s]);
                } else {
                    pend_item[s] = item;
                    pend_j[s] = j;
                }
                ++b;
                if (++j == nb) {
                    ++u;
                    if (u < u_end) load_unit();
                }
            }
            if (!waited) {  // fewer boxes than stages in total
                pdl_wait();
                for (int t = 0; t < min(b, kStages); ++t)
                    tma_load_2d_nohint(smem + L::kOffA + t * L::kABox, &a.tmA[pend_item[t]],
                                       pend_j[t] * kGemvBoxRows, 0, &full[t]);
            }
        }
        return;
    }

    pdl_wait();
    const int cg = tid % S::TPR, rg = tid / S::TPR;
    int b = 0;
    const int u_begin = __ldg(a.cta_begin + blockIdx.x);
    const int u_end = __ldg(a.cta_begin + blockIdx.x + 1);
    unsigned* peer_state = reinterpret_cast<unsigned*>(smem + L::kOffPeer);
    const int c = blockIdx.x;
    if (a.peer_sum && u_begin < u_end) {
        if (tid == 0) {
            const unsigned e = __ldcg(a.peer.epoch + c) + 1;
            a.peer.epoch[c] = e;
            peer_state[0] = e;
        }
        named_barrier(1, kConsumers);
    }
    for (int u = u_begin; u < u_end; ++u) {
        const unsigned code = __ldg(a.unit_table + u);
        const int item = static_cast<int>(code >> 16), strip = static_cast<int>(code & 0xFFFFu);
        const BatchItem it = a.items[item];
        const int col0 = strip * S::NT;
        const int nb = (it.k + kGemvBoxRows - 1) / kGemvBoxRows;
        // This thread's output column (the same for all M rows) and its scale, fetched now so
        // the store at the end of the unit does not wait on memory.
        const int my_col = col0 + tid % S::NT;
        const float sc = my_col < it.n ? __ldg(it.scale + my_col) : 0.0f;
        uint64_t acc[M][S::V / 2];
#pragma unroll
        for (int r = 0; r < M; ++r)
#pragma unroll
            for (int jj = 0; jj < S::V / 2; ++jj) acc[r][jj] = 0ull;
        bool ok = true;
        for (int j = 0; j < nb; ++j, ++b) {
            const int s = b % kStages;
            if (!mbar_wait(&full[s], (b / kStages) & 1, &g_gemv_error)) {
                ok = false;
                break;
            }
            const uint8_t* sb = smem + s * kBoxBytesB + cg * S::V;
            const float* sa = reinterpret_cast<const float*>(smem + L::kOffA + s * L::kABox);
#pragma unroll
            for (int i = 0; i < S::RPT; ++i) {
                const int row = rg + i * S::RG;
                uint64_t x[S::V / 2];
                load_pairs<true, S::V>(sb + row * kGemvRowBytes, x);
#pragma unroll
                for (int r = 0; r < M; ++r) {
                    const float av = sa[r * kGemvBoxRows + row];
                    const uint64_t a2 = pack2(av, av);
#pragma unroll
                    for (int jj = 0; jj < S::V / 2; ++jj) acc[r][jj] = fma2(a2, x[jj], acc[r][jj]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        if (!ok) break;
        // Reduce the row groups (shuffle, then the 8 warps in order) and store.
        float accf[M][S::V];
#pragma unroll
        for (int r = 0; r < M; ++r)
#pragma unroll
            for (int jj = 0; jj < S::V / 2; ++jj) unpack2(acc[r][jj], accf[r][2 * jj], accf[r][2 * jj + 1]);
#pragma unroll
        for (int off = S::TPR; off < 32; off <<= 1) {
#pragma unroll
            for (int r = 0; r < M; ++r)
#pragma unroll
                for (int jj = 0; jj < S::V; ++jj)
                    accf[r][jj] += __shfl_xor_sync(0xffffffffu, accf[r][jj], off);
        }
        if (lane < S::TPR) {
#pragma unroll
            for (int r = 0; r < M; ++r) {
                float4* dst = reinterpret_cast<float4*>(red + (warp * M + r) * S::NT + cg * S::V);
#pragma unroll
                for (int jj = 0; jj < S::V / 4; ++jj)
                    dst[jj] = make_float4(accf[r][4 * jj], accf[r][4 * jj + 1], accf[r][4 * jj + 2],
                                          accf[r][4 * jj + 3]);
            }
        }
        named_barrier(1, kConsumers);
        for (int e = tid; e < M * S::NT; e += kConsumers) {
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) v += red[w * M * S::NT + e];
            const int r = e / S::NT, col = col0 + e % S::NT;
            if (col < it.n) {
                v *= sc;
                float* o = it.C + static_cast<size_t>(r) * it.n + col;
                if (a.peer_sum) {
                    if (it.accumulate) v += *o;
                    const size_t at = static_cast<size_t>(u - u_begin) * M * S::NT + e;
                    const unsigned epoch = peer_state[0];
                    const unsigned long long w = tagged(v, epoch);
                    for (int q = 0; q < a.peer.world; ++q)
                        st_relaxed_sys_u64(peer_region(a.peer, q, epoch & 1u, c, a.peer.rank) + at, w);
                } else {
                    *o = it.accumulate ? *o + v : v;
                }
            }
        }
        named_barrier(1, kConsumers);  // red is rewritten by the next unit
    }
    if (!a.peer_sum || u_begin >= u_end) return;

    // Every unit written: each thread reads back the ranks' words of the elements it wrote, in
    // rank order, and writes the sums.
    const PeerSum& p = a.peer;
    const unsigned epoch = peer_state[0], slot = epoch & 1u;
    for (int u = u_begin; u < u_end; ++u) {
        const unsigned code = __ldg(a.unit_table + u);
        const BatchItem& it = a.items[code >> 16];
        const int col0 = static_cast<int>(code & 0xFFFFu) * S::NT;
        const int n = it.n;
        float* C = it.C;
        for (int e = tid; e < M * S::NT; e += kConsumers) {
            const int r = e / S::NT, col = col0 + e % S::NT;
            if (col >= n) continue;
            const size_t at = static_cast<size_t>(u - u_begin) * M * S::NT + e;
            float v = wait_tagged(peer_region(p, p.rank, slot, c, 0) + at, epoch, p.err);
            for (int src = 1; src < p.world; ++src)
                v += wait_tagged(peer_region(p, p.rank, slot, c, src) + at, epoch, p.err);
            C[static_cast<size_t>(r) * n + col] = v;
        }
    }
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
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = make_config(dim3(a.strips, a.slices), call_threads<M>(), L::kBytes,
                                         a.stream, a.pdl, attr);
    if (a.slices > 1) {
        // The k slices of a column strip form one cluster (reduced through DSMEM).
        attr[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
        attr[cfg.numAttrs].val.clusterDim.x = 1;
        attr[cfg.numAttrs].val.clusterDim.y = static_cast<unsigned>(a.slices);
        attr[cfg.numAttrs].val.clusterDim.z = 1;
        cfg.attrs = attr;
        ++cfg.numAttrs;
    }
    return cudaLaunchKernelEx(&cfg, kern, tmB, tmA, tmW, a);
}

}  // namespace

// Clusters of `cluster` CTAs of the per-call TMA GEMV the current device holds at once. Every
// per-call instantiation has the same launch shape (call_threads, at most kCallSmemBudget of
// shared memory, two CTAs per SM), so the largest stands for all.
int gemv_max_active_clusters(int cluster) {
    auto kern = gemv_tma_kernel<1, true, false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kCallSmemBudget);
    if (e != cudaSuccess) return -1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, static_cast<unsigned>(cluster));
    cfg.blockDim = dim3(call_threads<1>());
    cfg.dynamicSmemBytes = kCallSmemBudget;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = static_cast<unsigned>(cluster);
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    return e == cudaSuccess ? n : -1;
}

namespace {

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
        default:
            // fp32 B, 9..16 rows, no fused RMSNorm: one 16-row instantiation (its A map's box
            // is 16 rows).
            if constexpr (!Q8 && !Norm)
                if (a.m > 8 && a.m <= kGemvWideRows) return launch_tma_m<kGemvWideRows, false, false>(a, tmB, tmA, tmW);
            return cudaErrorInvalidValue;
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

template <int M>
cudaError_t launch_batch_m(const BatchArgs& a) {
    using L = BatchLayout<M>;
    auto kern = gemv_batch_kernel<M>;
    static unsigned configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 32 && !(configured & (1u << dev))) {
        cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
        if (e != cudaSuccess) return e;
        configured |= 1u << dev;
    }
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_config(dim3(a.grid), kTmaThreads, L::kBytes, a.stream, a.pdl, attr);
    return cudaLaunchKernelEx(&cfg, kern, a);
}

}  // namespace

int gemv_batch_ctas_per_sm() { return 2; }

cudaError_t launch_gemv_batch(const BatchArgs& a) {
    switch (a.m) {
        case 1: return launch_batch_m<1>(a);
        case 2: return launch_batch_m<2>(a);
        case 3: return launch_batch_m<3>(a);
        case 4: return launch_batch_m<4>(a);
        case 5: return launch_batch_m<5>(a);
        case 6: return launch_batch_m<6>(a);
        case 7: return launch_batch_m<7>(a);
        case 8: return launch_batch_m<8>(a);
        default: return cudaErrorInvalidValue;
    }
}

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
