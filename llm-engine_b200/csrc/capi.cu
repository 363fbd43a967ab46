// The C ABI (include/llme_b200.h): argument checks and kernel choice, device
// scratch, the TMA descriptor cache, and the launches. Mirrors the reference's
// matmul_impl (src/cuda_matmul.cu:399-448) for validation, error text and the
// empty/k == 0 cases; the plan itself (llme_plan) is a pure function so the
// dispatch logic can be tested without a GPU.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <queue>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace {

using namespace llme;

thread_local std::string g_error;

int fail(int code, std::string msg) {
    g_error = std::move(msg);
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(LLME_E_CUDA, std::string("cuda: ") + what + ": " + cudaGetErrorString(e));
}

std::string shapes(size_t m, size_t n, size_t k) {
    return "(A is " + std::to_string(m) + "x" + std::to_string(k) + ", B is " + std::to_string(k) +
           "x" + std::to_string(n) + ")";
}

size_t ceil_div(size_t x, size_t d) { return (x + d - 1) / d; }
size_t round_up(size_t x, size_t to) { return ceil_div(x, to) * to; }

// ---- math mode -------------------------------------------------------------------------

std::atomic<int> g_math{-1};

int math_mode() {
    int v = g_math.load(std::memory_order_relaxed);
    if (v < 0) {
        const char* env = std::getenv("LLME_B200_MATH");
        v = (env && std::strcmp(env, "fp32") == 0) ? LLME_MATH_FP32 : LLME_MATH_TENSOR;
        int expected = -1;
        g_math.compare_exchange_strong(expected, v);
        v = g_math.load();
    }
    return v;
}

// ---- planning ----------------------------------------------------------------------------

constexpr size_t kMaxElems = size_t{1} << 31;  // kernels index with int
constexpr int kSkinnyMaxRows = 8;
constexpr int kSplitMaxRows = 127;             // automatic: tiled_split below 128 rows
constexpr size_t kMaxGridY = 65535;            // CUDA's limit on gridDim.y

struct PlanIn {
    size_t m, n, k;
    bool q8;
    int kernel;
    bool accumulate;
    uintptr_t a_addr, b_addr, rms_addr;
    int sms;
    int math;
    // The device's capacity for per-call GEMV clusters of 1..kGemvMaxCluster CTAs (entry c - 1),
    // or null: host-only plans then take 2 x SMs / c.
    const int* gemv_clusters = nullptr;
};

// The int8 tcgen05 GEMM on CTA pairs (one M=256 MMA over two SMs, 256-column tiles) only when
// LLME_B200_CTA_PAIRS=1 and the SM count is even. Measured on B200 under the 1 kW power cap:
// pairs do ~3% more work per clock but draw more power per unit of work, so the sustained
// clock settles ~15% lower (7B prefill: 910 TFLOP/s at 1.16 GHz with pairs, 1030 at 1.37 GHz
// without); short bursts below the cap run faster on pairs (4096x8192x8192: 1384 vs 1336).
bool q8tc_use_pairs(int sms) {
    const char* v = getenv("LLME_B200_CTA_PAIRS");
    return v && v[0] == '1' && sms >= 2 && sms % 2 == 0;
}

// int8 tcgen05 GEMM scratch: hi rows, lo rows (pitch round_up(k, 16), each region 256-byte
// aligned), then the m row scales.
size_t q8tc_pitch(size_t k) { return round_up(k, 16); }
size_t q8tc_rows_bytes(size_t m, size_t k) { return round_up(m * q8tc_pitch(k), 256); }
size_t q8tc_operand_bytes(size_t m, size_t k) { return 2 * q8tc_rows_bytes(m, k) + m * sizeof(float); }
// The skinny GEMM's three term planes, then the row scales.
size_t skinny_operand_bytes(size_t m, size_t k) { return 3 * q8tc_rows_bytes(m, k) + m * sizeof(float); }

int plan_path(const PlanIn& in, llme_plan_t* p) {
    std::memset(p, 0, sizeof(*p));
    const size_t m = in.m, n = in.n, k = in.k;
    int kernel = in.kernel;
    if (kernel < LLME_KERNEL_AUTOMATIC || kernel > LLME_KERNEL_SKINNY)
        return fail(LLME_E_INVALID, "matmul_cuda: unknown kernel " + std::to_string(kernel));
    if (kernel == LLME_KERNEL_AUTOMATIC) {
        kernel = m <= kSkinnyMaxRows ? LLME_KERNEL_SKINNY
                 : m <= kSplitMaxRows ? LLME_KERNEL_TILED_SPLIT
                                      : LLME_KERNEL_TILED;
    }
    p->kernel = kernel;
    if (kernel == LLME_KERNEL_SKINNY && m > kSkinnyMaxRows)
        return fail(LLME_E_INVALID,
                    "matmul_cuda: skinny kernel takes at most 8 rows " + shapes(m, n, k));
    if (m * k >= kMaxElems || k * n >= kMaxElems || m * n >= kMaxElems)
        return fail(LLME_E_INVALID, "matmul_cuda: more than 2^31 elements " + shapes(m, n, k));
    if (m == 0 || n == 0) {
        p->path = LLME_PATH_NONE;
        return LLME_OK;
    }
    if (k == 0) {
        p->path = in.accumulate ? LLME_PATH_NONE : LLME_PATH_ZERO;
        return LLME_OK;
    }
    const bool has_rms = in.rms_addr != 0;
    const int sms = in.sms > 0 ? in.sms : 148;

    // Operands the TMA GEMV can stream: 16-byte aligned rows and starts.
    const bool gemv_tma = in.b_addr % 16 == 0 && (n * (in.q8 ? 1 : 4)) % 16 == 0 &&
                          in.a_addr % 16 == 0 && k % 4 == 0 && (!has_rms || in.rms_addr % 16 == 0);
    // The TMA GEMV's grid: two CTAs per SM; the k slices of a column strip form one cluster (at
    // most 8), each at least two boxes deep, and every cluster must be resident at once: the
    // device holds fewer clusters than 2 x SMs / c when they do not pack every GPC (B200, c = 1..8:
    // 296, 148, 93, 71, 56, 45, 37, 33), and a cluster that waits for a second wave doubles the
    // call (the 7B wqkv, 96 strips: 18.08 us at 3 slices, 13.95 at 2; the 86-strip w1 fits at 3).
    auto plan_gemv_tma = [&](int rows) {
        p->path = LLME_PATH_GEMV_TMA;
        p->tile_m = rows;
        p->tile_n = gemv_tma_cols(in.q8);
        const size_t strips = ceil_div(n, p->tile_n);
        const size_t target = static_cast<size_t>(gemv_call_ctas_per_sm(rows)) * sms;
        size_t slices = std::max<size_t>(
            1, std::min({target / strips, ceil_div(k, 2 * kGemvBoxRows),
                         static_cast<size_t>(kGemvMaxCluster)}));
        auto capacity = [&](size_t c) {
            return in.gemv_clusters && in.gemv_clusters[c - 1] > 0
                       ? static_cast<size_t>(in.gemv_clusters[c - 1])
                       : target / c;
        };
        while (slices > 1 && strips > capacity(slices)) --slices;
        const size_t span = round_up(ceil_div(k, slices), kGemvBoxRows);
        slices = ceil_div(k, span);
        p->grid_x = static_cast<int>(strips);
        p->grid_y = static_cast<int>(slices);
        p->slices = static_cast<int>(slices);
        p->span = static_cast<int>(span);
        p->cluster = static_cast<int>(slices);
        return LLME_OK;
    };

    if (kernel == LLME_KERNEL_SKINNY && gemv_tma) return plan_gemv_tma(static_cast<int>(m));
    // fp32 B with 9..16 rows (tiled_split, or tiled) in LLME_MATH_FP32: the TMA GEMV at 16
    // rows, exact fp32 arithmetic (33 us for 16 x 4096^2 against 126 on the SIMT tiles). In
    // tensor math the three-term TF32 kernel below is faster (19 us).
    // RMSNorm runs as the separate row pass here (the 16-row kernel has no fused norm).
    if (!in.q8 && in.math == LLME_MATH_FP32 && m > kSkinnyMaxRows &&
        m <= static_cast<size_t>(kGemvWideRows) && gemv_tma &&
        (kernel == LLME_KERNEL_TILED_SPLIT || kernel == LLME_KERNEL_TILED)) {
        plan_gemv_tma(kGemvWideRows);
        p->rms_prepass = has_rms ? 1 : 0;
        if (has_rms) p->norm_bytes = m * k * sizeof(float);
        return LLME_OK;
    }

    if (kernel == LLME_KERNEL_SKINNY) {
        // Ragged rows or unaligned pointers: the plain-load GEMV.
        p->path = LLME_PATH_GEMV_LDG;
        p->tile_m = static_cast<int>(m);
        p->tile_n = kGemvLdgCols;
        const size_t strips = ceil_div(n, p->tile_n);
        const size_t target = 8 * static_cast<size_t>(sms);
        size_t slices = std::max<size_t>(1, std::min(target / strips, ceil_div(k, 256)));
        const size_t span = ceil_div(k, slices);
        slices = ceil_div(k, span);
        p->grid_x = static_cast<int>(strips);
        p->grid_y = static_cast<int>(slices);
        p->slices = static_cast<int>(slices);
        p->span = static_cast<int>(span);
        p->cluster = 1;
        if (slices > 1) {
            // The plain-load kernel reduces its slices through global scratch.
            p->counter_slots = strips;
            p->split_bytes = strips * slices * (m * p->tile_n + m) * sizeof(float);
        }
        return LLME_OK;
    }

    // naive / tiled / tiled_split: A is normalised by a separate pass first.
    p->rms_prepass = has_rms ? 1 : 0;
    if (has_rms) p->norm_bytes = m * k * sizeof(float);
    if (kernel == LLME_KERNEL_NAIVE) {
        p->path = LLME_PATH_NAIVE;
        p->tile_m = p->tile_n = 16;
        p->grid_x = static_cast<int>(ceil_div(n, 16));
        p->grid_y = static_cast<int>(ceil_div(m, 16));
        p->slices = 1;
        p->span = static_cast<int>(k);
        return LLME_OK;
    }
    // The tcgen05 GEMM: TF32 multiplies, so only in LLME_MATH_TENSOR; rows of A and B must
    // be TMA-addressable (16-byte aligned starts and pitches).
    const bool a_ok = has_rms || in.a_addr % 16 == 0;
    if (kernel == LLME_KERNEL_TILED && in.math == LLME_MATH_TENSOR && !in.q8 && m >= 128 &&
        k % 4 == 0 && n % 4 == 0 && a_ok && in.b_addr % 16 == 0) {
        p->path = LLME_PATH_TCGEN05;
        p->tile_m = tc_tile_m();
        p->tile_n = tc_tile_n();
        // B^T for the K-major operand only where the pass repays itself.
        if (m >= kTcTransposeMinRows) p->operand_bytes = k * n * sizeof(float);
        p->grid_x = static_cast<int>(ceil_div(m, p->tile_m) * ceil_div(n, p->tile_n));
        p->grid_y = 1;
        p->slices = 1;
        p->span = static_cast<int>(k);
        return LLME_OK;
    }
    // Decode-shaped int8 products on tcgen05 (three-term split: the fp32 decode path's
    // accuracy): tiled_split, or tiled below 128 rows, in LLME_MATH_TENSOR.
    const bool skinny_kernel =
        kernel == LLME_KERNEL_TILED_SPLIT || (kernel == LLME_KERNEL_TILED && m < 128);
    if (skinny_kernel && in.math == LLME_MATH_TENSOR && in.q8 && n % 16 == 0 &&
        in.b_addr % 16 == 0 && k <= static_cast<size_t>(kQ8TcMaxK)) {
        p->path = LLME_PATH_TCGEN05_SKINNY;
        p->rms_prepass = 0;
        p->norm_bytes = 0;
        const int t = skinny_rows_per_tile(static_cast<int>(std::min<size_t>(m, 64)));
        p->tile_m = t;
        p->tile_n = 128;
        p->grid_x = static_cast<int>(ceil_div(n, size_t{128}));
        p->grid_y = static_cast<int>(ceil_div(m, static_cast<size_t>(t)));
        const size_t units = static_cast<size_t>(p->grid_x) * p->grid_y;
        const size_t nkb = ceil_div(k, size_t{128});
        const size_t target = static_cast<size_t>(skinny_ctas_per_sm(t)) * sms;
        // k slices (one cluster, at most 8): as many as keep every CTA resident in one wave,
        // each at least 4 blocks deep.
        size_t slices = std::max<size_t>(
            1, std::min({target / units, ceil_div(nkb, size_t{4}), size_t{8}}));
        const size_t span_blocks = ceil_div(nkb, slices);
        slices = ceil_div(nkb, span_blocks);
        p->slices = static_cast<int>(slices);
        p->cluster = static_cast<int>(slices);
        p->span = static_cast<int>(span_blocks * 128);
        p->operand_bytes = skinny_operand_bytes(m, k);
        return LLME_OK;
    }
    // Decode-shaped fp32 products on tcgen05 in three TF32 terms (the fp32 decode path's
    // accuracy); A rows come from the RMSNorm pass when there is one.
    if (skinny_kernel && in.math == LLME_MATH_TENSOR && !in.q8 && n % 4 == 0 && k % 4 == 0 &&
        in.b_addr % 16 == 0 && (has_rms || in.a_addr % 16 == 0)) {
        p->path = LLME_PATH_TCGEN05_F32_SKINNY;
        const int t = skinny_rows_per_tile(static_cast<int>(std::min<size_t>(m, 64)));
        p->tile_m = t;
        p->tile_n = 128;
        p->grid_x = static_cast<int>(ceil_div(n, size_t{128}));
        p->grid_y = static_cast<int>(ceil_div(m, static_cast<size_t>(t)));
        const size_t units = static_cast<size_t>(p->grid_x) * p->grid_y;
        const size_t fk = static_cast<size_t>(f32_skinny_stage_k());
        const size_t nkb = ceil_div(k, fk);
        const size_t target = static_cast<size_t>(sms);  // one CTA per SM
        // k slices (one cluster, at most 8): fill the GPU once, each at least 8 blocks deep.
        size_t slices = std::max<size_t>(1, std::min({target / units, ceil_div(nkb, size_t{8}),
                                                      size_t{8}}));
        const size_t span_blocks = ceil_div(nkb, slices);
        slices = ceil_div(nkb, span_blocks);
        p->slices = static_cast<int>(slices);
        p->cluster = static_cast<int>(slices);
        p->span = static_cast<int>(span_blocks * fk);
        return LLME_OK;
    }
    // The int8 tcgen05 GEMM: also LLME_MATH_TENSOR only (the activations are split into two
    // int8 terms); W rows must be TMA-addressable and k small enough for exact s32 sums.
    // The RMSNorm of A is applied by the split pass, not by a separate one.
    if (kernel == LLME_KERNEL_TILED && in.math == LLME_MATH_TENSOR && in.q8 && m >= 128 &&
        n % 16 == 0 && in.b_addr % 16 == 0 && k <= static_cast<size_t>(kQ8TcMaxK)) {
        p->path = LLME_PATH_TCGEN05_Q8;
        p->rms_prepass = 0;
        p->norm_bytes = 0;
        // CTA pairs (cta_group::2) whenever the SMs pair up; grid_x counts CTAs, cluster 2.
        const bool pair = q8tc_use_pairs(sms);
        p->tile_m = q8tc_tile_m();
        p->tile_n = q8tc_tile_n(pair);
        const size_t tiles = ceil_div(m, p->tile_m) * ceil_div(n, p->tile_n);
        const size_t slots = std::min<size_t>(tiles, static_cast<size_t>(pair ? sms / 2 : sms));
        p->grid_x = static_cast<int>(slots * (pair ? 2 : 1));
        p->cluster = pair ? 2 : 1;
        p->grid_y = 1;
        p->slices = 1;
        p->span = static_cast<int>(k);
        p->operand_bytes = q8tc_operand_bytes(m, k);
        return LLME_OK;
    }
    p->path = LLME_PATH_TILED_SIMT;
    p->tile_m = kTiledBM;
    p->tile_n = kTiledBN;
    const size_t tiles = ceil_div(n, kTiledBN) * ceil_div(m, kTiledBM);
    size_t slices = 1;
    if (kernel == LLME_KERNEL_TILED_SPLIT) {
        // Split k until about 4 CTAs per SM, each slice at least 256 deep.
        const size_t target = 4 * static_cast<size_t>(sms);
        slices = std::max<size_t>(1, std::min(ceil_div(target, tiles), ceil_div(k, 256)));
    }
    const size_t span = round_up(ceil_div(k, slices), kTiledBK);
    slices = ceil_div(k, span);
    p->grid_x = static_cast<int>(ceil_div(n, kTiledBN));
    p->grid_y = static_cast<int>(ceil_div(m, kTiledBM));
    p->slices = static_cast<int>(slices);
    p->span = static_cast<int>(span);
    if (slices > 1) {
        p->counter_slots = tiles;
        p->split_bytes = tiles * slices * kTiledBM * kTiledBN * sizeof(float);
    }
    return LLME_OK;
}

// The SIMT and decode-shaped tensor-core paths put row tiles on grid y, whose limit is 65535
// (the prefill GEMMs put every tile on x): the planner refuses more row tiles than that
// rather than let the launch fail.
int make_plan(const PlanIn& in, llme_plan_t* p) {
    const int st = plan_path(in, p);
    if (st != LLME_OK) return st;
    if (static_cast<size_t>(p->grid_y) > kMaxGridY) {
        const llme_plan_t planned = *p;
        std::memset(p, 0, sizeof(*p));
        return fail(LLME_E_INVALID, "matmul_cuda: " + std::to_string(planned.grid_y) +
                                        " row tiles of " + std::to_string(planned.tile_m) +
                                        " exceed the grid's 65535 " + shapes(in.m, in.n, in.k));
    }
    return LLME_OK;
}

// ---- per-device state ------------------------------------------------------------------

constexpr int kMaxDevices = 64;
std::atomic<size_t> g_generation{0};

struct Scratch {
    void* ptr = nullptr;
    size_t cap = 0;
};

struct DeviceState {
    int sms = 0;
    // Split-K buffer: [counters: counter_cap x u32, zeroed][partial sums: partial_cap bytes].
    // The two regions grow independently to the largest size seen, so a fixed sequence of
    // calls stops reallocating after its first pass.
    Scratch split;
    size_t counter_cap = 0;
    size_t partial_cap = 0;
    Scratch norm;
    Scratch operand;  // split activation rows (int8 tensor-core GEMMs) or B^T (TF32 GEMM)
    // Per-call GEMV cluster capacity by cluster size (0: not queried yet).
    int gemv_clusters[kGemvMaxCluster] = {};
};

std::mutex g_dev_mu;
DeviceState g_dev[kMaxDevices];

int current_device(int* dev) {
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return cuda_fail(e, "get device");
    if (*dev < 0 || *dev >= kMaxDevices) return fail(LLME_E_UNSUPPORTED, "device index too large");
    return LLME_OK;
}

// The device's capacity for per-call GEMV clusters of 1..kGemvMaxCluster CTAs, queried once
// (the current device must be `dev`); null when the driver does not answer.
const int* device_gemv_clusters(int dev) {
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    DeviceState& d = g_dev[dev];
    if (d.gemv_clusters[0] == 0) {
        int t[kGemvMaxCluster];
        for (int c = 1; c <= kGemvMaxCluster; ++c) {
            t[c - 1] = gemv_max_active_clusters(c);
            if (t[c - 1] <= 0) {
                cudaGetLastError();  // a refused query leaves no sticky error
                return nullptr;
            }
        }
        std::copy(t, t + kGemvMaxCluster, d.gemv_clusters);
    }
    return d.gemv_clusters;
}

int device_sms(int dev, int* sms) {
    DeviceState& d = g_dev[dev];
    if (d.sms == 0) {
        int n = 0;
        cudaError_t e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return cuda_fail(e, "get SMs");
        d.sms = n;
    }
    *sms = d.sms;
    return LLME_OK;
}

// Grow-only; every growth bumps the generation (a captured graph must be re-captured).
int ensure_split(int dev, size_t counters, size_t bytes, cudaStream_t stream, SplitScratch* out,
                 size_t partial_floats) {
    DeviceState& d = g_dev[dev];
    const size_t want_counters =
        round_up(std::max<size_t>(counters, d.counter_cap) * sizeof(unsigned), 256) /
        sizeof(unsigned);
    const size_t want_partial = std::max(round_up(bytes, 256), d.partial_cap);
    if (want_counters > d.counter_cap || want_partial > d.partial_cap) {
        const size_t counter_bytes = want_counters * sizeof(unsigned);
        if (d.split.ptr) {
            cudaError_t e = cudaFree(d.split.ptr);
            if (e != cudaSuccess) return cuda_fail(e, "free scratch");
            d.split.ptr = nullptr;
            d.split.cap = d.counter_cap = d.partial_cap = 0;
        }
        cudaError_t e = cudaMalloc(&d.split.ptr, counter_bytes + want_partial);
        if (e != cudaSuccess) return cuda_fail(e, "alloc scratch");
        d.split.cap = counter_bytes + want_partial;
        d.counter_cap = want_counters;
        d.partial_cap = want_partial;
        e = cudaMemsetAsync(d.split.ptr, 0, counter_bytes, stream);
        if (e != cudaSuccess) return cuda_fail(e, "zero scratch");
        g_generation.fetch_add(1);
    }
    const size_t cbytes = round_up(d.counter_cap * sizeof(unsigned), 256);
    out->counters = static_cast<unsigned*>(d.split.ptr);
    out->partial = reinterpret_cast<float*>(static_cast<char*>(d.split.ptr) + cbytes);
    out->partial_ss = out->partial + partial_floats;
    return LLME_OK;
}

// Grow-only buffer; growth bumps the generation.
int ensure_buffer(Scratch& b, size_t bytes, float** out) {
    if (bytes > b.cap) {
        if (b.ptr) {
            cudaError_t e = cudaFree(b.ptr);
            if (e != cudaSuccess) return cuda_fail(e, "free scratch");
            b.ptr = nullptr;
            b.cap = 0;
        }
        cudaError_t e = cudaMalloc(&b.ptr, bytes);
        if (e != cudaSuccess) return cuda_fail(e, "alloc scratch");
        b.cap = bytes;
        g_generation.fetch_add(1);
    }
    *out = static_cast<float*>(b.ptr);
    return LLME_OK;
}

int ensure_norm(int dev, size_t bytes, float** out) { return ensure_buffer(g_dev[dev].norm, bytes, out); }

// ---- TMA descriptors -------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

// The driver's cuTensorMapEncodeTiled, resolved once through the runtime (no link against
// libcuda); null where the driver does not offer it.
PFN_cuTensorMapEncodeTiled_v12000 encoder() {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault,
                                             &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    return g_encode;
}

struct MapKey {
    uintptr_t ptr;
    int dtype, rank;
    uint64_t d0, d1;
    uint32_t b0, b1;
    uint64_t pitch;
    bool operator==(const MapKey& o) const {
        return ptr == o.ptr && dtype == o.dtype && rank == o.rank && d0 == o.d0 && d1 == o.d1 &&
               b0 == o.b0 && b1 == o.b1 && pitch == o.pitch;
    }
};
struct MapKeyHash {
    size_t operator()(const MapKey& k) const {
        size_t h = std::hash<uintptr_t>()(k.ptr);
        auto mix = [&h](uint64_t v) { h ^= std::hash<uint64_t>()(v) + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2); };
        mix(static_cast<uint64_t>(k.dtype) << 8 | static_cast<uint64_t>(k.rank));
        mix(k.d0);
        mix(k.d1);
        mix(static_cast<uint64_t>(k.b0) << 32 | k.b1);
        mix(k.pitch);
        return h;
    }
};
std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

// Encodes without the cache (rank 2, or rank 1 when rows == 0). pitch_bytes 0: rows are
// packed (cols * esz apart).
int encode_map(const void* ptr, CUtensorMapDataType dtype, size_t esz, uint64_t rows, uint64_t cols,
               uint32_t box_cols, uint32_t box_rows, CUtensorMap* out,
               CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE, uint64_t pitch_bytes = 0);

// Row-major matrix of `rows` x `cols` elements (rank 2), or a vector (rows == 0, rank 1),
// tiled into boxes of box_cols x box_rows.
int tensor_map(const void* ptr, CUtensorMapDataType dtype, size_t esz, uint64_t rows, uint64_t cols,
               uint32_t box_cols, uint32_t box_rows, CUtensorMap* out,
               CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE, uint64_t pitch_bytes = 0) {
    if (!encoder()) return fail(LLME_E_UNSUPPORTED, "cuda: cuTensorMapEncodeTiled is unavailable");
    const int rank = rows ? 2 : 1;
    const MapKey key{reinterpret_cast<uintptr_t>(ptr), static_cast<int>(dtype) | (static_cast<int>(swizzle) << 8),
                     rank, cols, rows, box_cols, box_rows, pitch_bytes};
    {
        std::lock_guard<std::mutex> lk(g_map_mu);
        auto it = g_maps.find(key);
        if (it != g_maps.end()) {
            *out = it->second;
            return LLME_OK;
        }
    }
    const int st = encode_map(ptr, dtype, esz, rows, cols, box_cols, box_rows, out, swizzle,
                              pitch_bytes);
    if (st) return st;
    std::lock_guard<std::mutex> lk(g_map_mu);
    if (g_maps.size() > 8192) g_maps.clear();
    g_maps.emplace(key, *out);
    return LLME_OK;
}

int encode_map(const void* ptr, CUtensorMapDataType dtype, size_t esz, uint64_t rows, uint64_t cols,
               uint32_t box_cols, uint32_t box_rows, CUtensorMap* out, CUtensorMapSwizzle swizzle,
               uint64_t pitch_bytes) {
    if (!encoder()) return fail(LLME_E_UNSUPPORTED, "cuda: cuTensorMapEncodeTiled is unavailable");
    const int rank = rows ? 2 : 1;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {pitch_bytes ? pitch_bytes : cols * esz};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(out, dtype, rank, const_cast<void*>(ptr), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(LLME_E_CUDA, "cuda: encode tensor map: CUresult " + std::to_string(int(r)));
    return LLME_OK;
}

// ---- the call --------------------------------------------------------------------------

// The pointers a product reads or writes must be set: none for an empty product, only C when
// k == 0 zeroes it, all of A, B, C (and the int8 scales) otherwise.
bool missing_pointer(size_t m, size_t n, size_t k, const float* A, const void* B,
                     const float* scale, const float* C, bool q8, bool accumulate) {
    if (m == 0 || n == 0) return false;
    if (k == 0) return !accumulate && !C;
    return !A || !B || !C || (q8 && !scale);
}

int run(size_t m, size_t n, size_t k, const float* A, const void* B, const float* scale, float* C,
        bool q8, int kernel, bool accumulate, const float* rms, unsigned flags, void* stream_ptr,
        const GemvEpilogue* epi = nullptr) {
    g_error.clear();
    if (missing_pointer(m, n, k, A, B, scale, C, q8, accumulate))
        return fail(LLME_E_INVALID, "matmul_cuda: null pointer " + shapes(m, n, k));
    cudaStream_t stream = stream_ptr ? static_cast<cudaStream_t>(stream_ptr) : cudaStreamPerThread;
    int dev = 0, sms = 0;
    int st = current_device(&dev);
    if (st) return st;
    st = device_sms(dev, &sms);
    if (st) return st;
    const int* gemv_clusters = device_gemv_clusters(dev);
    PlanIn in{m,
              n,
              k,
              q8,
              kernel,
              accumulate,
              reinterpret_cast<uintptr_t>(A),
              reinterpret_cast<uintptr_t>(B),
              reinterpret_cast<uintptr_t>(rms),
              sms,
              math_mode()};
    in.gemv_clusters = gemv_clusters;
    llme_plan_t p;
    st = make_plan(in, &p);
    if (st) return st;
    // A fused epilogue exists only in the TMA GEMV. The elementwise ones work on column pairs
    // and write plainly; the peer sum needs every CTA of the grid resident at once (each waits
    // for the same CTA of every rank) and a flag slot per CTA.
    if (epi && epi->kind == kEpiPeerSum) {
        if (p.path != LLME_PATH_GEMV_TMA ||
            static_cast<long>(p.grid_x) * p.grid_y > std::min(epi->peer.units, 2 * sms))
            return fail(LLME_E_UNSUPPORTED, "matmul: the in-kernel rank sum needs the TMA GEMV path "
                                            "with one resident grid " + shapes(m, n, k));
    } else if (epi && epi->kind != kEpiStore &&
               (p.path != LLME_PATH_GEMV_TMA || n % 2 != 0 || accumulate)) {
        return fail(LLME_E_UNSUPPORTED, "matmul: fused epilogue needs the TMA GEMV path, an even n "
                                        "and no accumulation " + shapes(m, n, k));
    }
    if (p.path == LLME_PATH_NONE) return LLME_OK;
    if (p.path == LLME_PATH_ZERO) {
        cudaError_t e = cudaMemsetAsync(C, 0, m * n * sizeof(float), stream);
        return e == cudaSuccess ? LLME_OK : cuda_fail(e, "memset");
    }

    std::lock_guard<std::mutex> lk(g_dev_mu);  // scratch is shared per device
    SplitScratch split;
    if (p.split_bytes > 0 && p.path != LLME_PATH_TCGEN05_SKINNY) {
        // Partial sums first, then (GEMV with RMSNorm) the per-slice sums of squares.
        const size_t partial_floats =
            p.path == LLME_PATH_TILED_SIMT
                ? static_cast<size_t>(p.counter_slots) * p.slices * kTiledBM * kTiledBN
                : static_cast<size_t>(p.grid_x) * p.slices * m * p.tile_n;
        st = ensure_split(dev, p.counter_slots, p.split_bytes, stream, &split, partial_floats);
        if (st) return st;
    }
    const float* a_in = A;
    if (p.rms_prepass) {
        float* normed = nullptr;
        st = ensure_norm(dev, p.norm_bytes, &normed);
        if (st) return st;
        cudaError_t e = launch_rmsnorm_rows(static_cast<int>(m), static_cast<int>(k), A, rms,
                                            normed, stream);
        if (e != cudaSuccess) return cuda_fail(e, "launch");
        a_in = normed;
    }

    cudaError_t e = cudaSuccess;
    if (p.path == LLME_PATH_GEMV_TMA || p.path == LLME_PATH_GEMV_LDG) {
        GemvArgs g;
        g.m = static_cast<int>(m);
        g.n = static_cast<int>(n);
        g.k = static_cast<int>(k);
        // RMSNorm fused in the kernel, or (16-row fp32 GEMV) already applied by the row pass.
        g.A = a_in;
        g.B = B;
        g.scale = scale;
        g.rms = p.rms_prepass ? nullptr : rms;
        g.C = C;
        g.q8 = q8;
        g.accumulate = accumulate;
        g.slices = p.slices;
        g.span = p.span;
        g.strips = p.grid_x;
        g.split = split;
        g.stream = stream;
        // The TMA kernel always launches with programmatic dependent launch: before
        // griddepcontrol.wait it reads nothing but its weights (and only with
        // LLME_FLAG_WEIGHTS_STATIC; otherwise it merely prefetches them into L2).
        g.weights_static = (flags & LLME_FLAG_WEIGHTS_STATIC) != 0;
        if (epi) g.epi = *epi;
        g.pdl = p.path == LLME_PATH_GEMV_TMA || g.weights_static;
        if (p.path == LLME_PATH_GEMV_TMA) {
            CUtensorMap tmB, tmA, tmW;
            st = q8 ? tensor_map(B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, k, n, kGemvRowBytes,
                                 kGemvBoxRows, &tmB)
                    : tensor_map(B, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, k, n, kGemvRowBytes / 4,
                                 kGemvBoxRows, &tmB);
            if (st) return st;
            // The box is the kernel's row count (16 for 9..16 fp32 rows: zero fill past m).
            st = tensor_map(g.A, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, m, k, kGemvBoxRows,
                            static_cast<uint32_t>(p.tile_m), &tmA);
            if (st) return st;
            if (g.rms) {
                st = tensor_map(g.rms, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, 0, k, kGemvBoxRows, 1,
                                &tmW);
                if (st) return st;
            } else {
                tmW = tmA;  // unused
            }
            e = launch_gemv_tma(g, tmB, tmA, tmW);
        } else {
            e = launch_gemv_ldg(g);
        }
    } else if (p.path == LLME_PATH_TCGEN05) {
        CUtensorMap tmA, tmB;
        st = tensor_map(a_in, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, m, k, 32, 128, &tmA,
                        CU_TENSOR_MAP_SWIZZLE_128B);
        if (st) return st;
        const bool transposed = p.operand_bytes > 0;
        if (transposed) {
            float* bt = nullptr;
            st = ensure_buffer(g_dev[dev].operand, p.operand_bytes, &bt);
            if (st) return st;
            e = launch_transpose(static_cast<const float*>(B), bt, static_cast<int>(k),
                                 static_cast<int>(n), stream);
            if (e != cudaSuccess) return cuda_fail(e, "launch");
            st = tensor_map(bt, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, n, k, 32, 256, &tmB,
                            CU_TENSOR_MAP_SWIZZLE_128B);
        } else {
            st = tensor_map(B, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, k, n, 32, 32, &tmB,
                            CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
        }
        if (st) return st;
        TcArgs t;
        t.m = static_cast<int>(m);
        t.n = static_cast<int>(n);
        t.k = static_cast<int>(k);
        t.C = C;
        t.accumulate = accumulate;
        t.b_transposed = transposed;
        t.tiles_m = static_cast<int>(ceil_div(m, p.tile_m));
        t.tiles_n = static_cast<int>(ceil_div(n, p.tile_n));
        t.stream = stream;
        t.pdl = (flags & LLME_FLAG_WEIGHTS_STATIC) != 0;
        e = launch_gemm_tf32(t, tmA, tmB);
    } else if (p.path == LLME_PATH_TCGEN05_F32_SKINNY) {
        CUtensorMap tmW, tmA;
        st = tensor_map(B, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, k, n, 128, 32, &tmW);
        if (!st)
            st = tensor_map(a_in, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, m, k, 32, p.tile_m, &tmA,
                            CU_TENSOR_MAP_SWIZZLE_128B);
        if (st) return st;
        F32SkinnyArgs t;
        t.m = static_cast<int>(m);
        t.n = static_cast<int>(n);
        t.k = static_cast<int>(k);
        t.C = C;
        t.accumulate = accumulate;
        t.weights_static = (flags & LLME_FLAG_WEIGHTS_STATIC) != 0;
        t.rows_per_tile = p.tile_m;
        t.slices = p.slices;
        t.span_blocks = p.span / f32_skinny_stage_k();
        t.stream = stream;
        e = launch_gemm_f32_skinny(t, tmW, tmA);
    } else if (p.path == LLME_PATH_TCGEN05_SKINNY) {
        float* ops = nullptr;
        st = ensure_buffer(g_dev[dev].operand, p.operand_bytes, &ops);
        if (st) return st;
        const size_t plane = q8tc_rows_bytes(m, k);
        int8_t* t0 = reinterpret_cast<int8_t*>(ops);
        int8_t* t1 = t0 + plane;
        int8_t* t2 = t1 + plane;
        float* rs = reinterpret_cast<float*>(t2 + plane);
        const size_t kp = q8tc_pitch(k);
        SkinnyArgs t;
        e = launch_split_rows(static_cast<int>(m), static_cast<int>(k), static_cast<int>(kp), A,
                              rms, t0, t1, t2, rs, stream, true);
        if (e != cudaSuccess) return cuda_fail(e, "launch");
        CUtensorMap tmW, tm0, tm1, tm2;
        st = tensor_map(B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, k, n, 128, 128, &tmW,
                        CU_TENSOR_MAP_SWIZZLE_128B);
        if (!st)
            st = tensor_map(t0, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, m, k, 128, p.tile_m, &tm0,
                            CU_TENSOR_MAP_SWIZZLE_128B, kp);
        if (!st)
            st = tensor_map(t1, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, m, k, 128, p.tile_m, &tm1,
                            CU_TENSOR_MAP_SWIZZLE_128B, kp);
        if (!st)
            st = tensor_map(t2, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, m, k, 128, p.tile_m, &tm2,
                            CU_TENSOR_MAP_SWIZZLE_128B, kp);
        if (st) return st;
        t.m = static_cast<int>(m);
        t.n = static_cast<int>(n);
        t.k = static_cast<int>(k);
        t.scale = scale;
        t.row_scale = rs;
        t.C = C;
        t.accumulate = accumulate;
        t.weights_static = (flags & LLME_FLAG_WEIGHTS_STATIC) != 0;
        t.rows_per_tile = p.tile_m;
        t.slices = p.slices;
        t.span_blocks = p.span / 128;
        t.stream = stream;
        e = launch_gemm_q8_skinny(t, tmW, tm0, tm1, tm2);
    } else if (p.path == LLME_PATH_TCGEN05_Q8) {
        float* ops = nullptr;
        st = ensure_buffer(g_dev[dev].operand, p.operand_bytes, &ops);
        if (st) return st;
        int8_t* hi = reinterpret_cast<int8_t*>(ops);
        int8_t* lo = hi + q8tc_rows_bytes(m, k);
        float* rs = reinterpret_cast<float*>(lo + q8tc_rows_bytes(m, k));
        const size_t kp = q8tc_pitch(k);
        e = launch_split_rows(static_cast<int>(m), static_cast<int>(k), static_cast<int>(kp), A,
                              rms, hi, lo, nullptr, rs, stream, true);
        if (e != cudaSuccess) return cuda_fail(e, "launch");
        CUtensorMap tmHi, tmLo, tmB;
        st = tensor_map(hi, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, m, k, 128, 128, &tmHi,
                        CU_TENSOR_MAP_SWIZZLE_128B, kp);
        if (st) return st;
        st = tensor_map(lo, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, m, k, 128, 128, &tmLo,
                        CU_TENSOR_MAP_SWIZZLE_128B, kp);
        if (st) return st;
        st = tensor_map(B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, k, n, 128, 128, &tmB,
                        CU_TENSOR_MAP_SWIZZLE_128B);
        if (st) return st;
        Q8TcArgs t;
        t.m = static_cast<int>(m);
        t.n = static_cast<int>(n);
        t.k = static_cast<int>(k);
        t.scale = scale;
        t.row_scale = rs;
        t.C = C;
        t.accumulate = accumulate;
        t.pair = p.cluster == 2;
        t.slots = p.grid_x / p.cluster;
        t.stream = stream;
        e = launch_gemm_q8_tc(t, tmHi, tmLo, tmB);
    } else {
        TiledArgs t;
        t.m = static_cast<int>(m);
        t.n = static_cast<int>(n);
        t.k = static_cast<int>(k);
        t.A = a_in;
        t.B = B;
        t.scale = scale;
        t.C = C;
        t.q8 = q8;
        t.accumulate = accumulate;
        t.slices = p.slices;
        t.span = p.span;
        t.split = split;
        t.stream = stream;
        e = p.path == LLME_PATH_NAIVE ? launch_naive(t) : launch_tiled_simt(t);
    }
    if (e != cudaSuccess) return cuda_fail(e, "launch");
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "launch");
    return LLME_OK;
}

// ---- allocation-free entry point ------------------------------------------------------------
//
// llme_matmul_q8_noalloc runs the split-K tile kernel (the tiled_split plan) with its
// partial sums and tickets in one fixed device array defined here, instead of the grow-only
// scratch the other entry points cudaMalloc. Layout: [tickets: kNoAllocTickets x u32]
// [partial sums: the rest]. The tickets must be zero when a launch starts; set-up clears them
// once and every launch leaves them at zero again (the last CTA of a tile resets its ticket).
// Partial sums are always written before they are read. Every call on a device shares this
// one array, so two calls that overlap on the GPU (different streams or host threads) race on
// it.
constexpr size_t kNoAllocBytes = LLME_NOALLOC_SCRATCH_BYTES;
constexpr size_t kNoAllocTickets = 4096;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

std::mutex g_noalloc_mu;
unsigned char* g_noalloc_base[kMaxDevices] = {};

// Once per device, with that device current: the array's device address (the host-side
// symbol is only a stand-in, never a device pointer) and cleared tickets. The address is kept
// for the life of the process; a cudaDeviceReset would make it stale, which the header rules
// out for callers.
int noalloc_setup(int dev, cudaStream_t stream, unsigned char** base) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_base[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "scratch symbol address");
        e = cudaMemsetAsync(p, 0, kNoAllocTickets * sizeof(unsigned), stream);
        if (e != cudaSuccess) return cuda_fail(e, "clear scratch tickets");
        g_noalloc_base[dev] = static_cast<unsigned char*>(p);
    }
    *base = g_noalloc_base[dev];
    return LLME_OK;
}

int run_noalloc(size_t m, size_t n, size_t k, const float* A, const int8_t* B, const float* scale,
                float* C, bool accumulate, void* stream_ptr) {
    g_error.clear();
    if (missing_pointer(m, n, k, A, B, scale, C, true, accumulate))
        return fail(LLME_E_INVALID, "llme_matmul_q8_noalloc: null pointer " + shapes(m, n, k));
    cudaStream_t stream = stream_ptr ? static_cast<cudaStream_t>(stream_ptr) : cudaStreamPerThread;
    int dev = 0, sms = 0;
    int st = current_device(&dev);
    if (st) return st;
    st = device_sms(dev, &sms);
    if (st) return st;
    // The plan of the kernel this entry point launches (the SIMT tiles with split k), whatever
    // the process-wide arithmetic would pick for tiled_split.
    PlanIn in{m, n, k, true, LLME_KERNEL_TILED_SPLIT, accumulate, reinterpret_cast<uintptr_t>(A),
              reinterpret_cast<uintptr_t>(B), 0, sms, LLME_MATH_FP32};
    llme_plan_t p;
    st = make_plan(in, &p);
    if (st) return st;
    if (p.path != LLME_PATH_TILED_SIMT && p.path != LLME_PATH_NONE && p.path != LLME_PATH_ZERO)
        return fail(LLME_E_UNSUPPORTED, "llme_matmul_q8_noalloc: no split-K tile plan " + shapes(m, n, k));
    if (p.path == LLME_PATH_NONE) return LLME_OK;
    if (p.path == LLME_PATH_ZERO) {
        cudaError_t e = cudaMemsetAsync(C, 0, m * n * sizeof(float), stream);
        return e == cudaSuccess ? LLME_OK : cuda_fail(e, "memset");
    }
    const size_t ticket_bytes = kNoAllocTickets * sizeof(unsigned);
    if (p.counter_slots > kNoAllocTickets || p.split_bytes > kNoAllocBytes - ticket_bytes)
        return fail(LLME_E_INVALID,
                    "llme_matmul_q8_noalloc: this product needs " + std::to_string(p.split_bytes) +
                        " bytes of split-K scratch and " + std::to_string(p.counter_slots) +
                        " tickets; the fixed scratch holds " +
                        std::to_string(kNoAllocBytes - ticket_bytes) + " bytes and " +
                        std::to_string(kNoAllocTickets) + " tickets " + shapes(m, n, k));
    unsigned char* base = nullptr;
    st = noalloc_setup(dev, stream, &base);
    if (st) return st;
    TiledArgs t;
    t.m = static_cast<int>(m);
    t.n = static_cast<int>(n);
    t.k = static_cast<int>(k);
    t.A = A;
    t.B = B;
    t.scale = scale;
    t.C = C;
    t.q8 = true;
    t.accumulate = accumulate;
    t.slices = p.slices;
    t.span = p.span;
    t.split.counters = reinterpret_cast<unsigned*>(base);
    t.split.partial = reinterpret_cast<float*>(base + ticket_bytes);
    t.stream = stream;
    cudaError_t e = launch_tiled_simt(t);
    return e == cudaSuccess ? LLME_OK : cuda_fail(e, "launch");
}

}  // namespace

struct llme_batch {
    int dev = 0;
    void* dmem = nullptr;
    llme::BatchArgs args;
    size_t max_cta_units = 0;  // units of the busiest CTA (the rank sum's per-CTA area)
    // Tensor-core batches (m >= 128): the grouped tcgen05 launch and its split-row scratch.
    bool tc = false;
    llme::Q8TcBatchArgs targs;
    void* scratch = nullptr;
};

namespace {

// Longest-processing-time-first: units by decreasing work, each to the CTA with the least work
// so far (ties to the lower index). Deterministic, and within a few percent of the best
// possible makespan; each CTA then runs its units in their original order. Returns the units
// of CTA c as per_cta[c].
std::vector<std::vector<size_t>> lpt_assign(const std::vector<size_t>& work, int grid) {
    std::vector<size_t> order(work.size());
    for (size_t u = 0; u < order.size(); ++u) order[u] = u;
    std::stable_sort(order.begin(), order.end(),
                     [&](size_t x, size_t y) { return work[x] > work[y]; });
    std::vector<std::vector<size_t>> per_cta(grid);
    using Load = std::pair<size_t, int>;  // (work, cta)
    std::priority_queue<Load, std::vector<Load>, std::greater<Load>> heap;
    for (int c = 0; c < grid; ++c) heap.push({0, c});
    for (size_t u : order) {
        Load l = heap.top();
        heap.pop();
        per_cta[l.second].push_back(u);
        heap.push({l.first + work[u], l.second});
    }
    for (auto& v : per_cta) std::sort(v.begin(), v.end());
    return per_cta;
}

// Grouped int8 products with m >= 128 on the tensor cores (gemm_q8_tc.cu).
int batch_create_tc(llme_batch_t** out, size_t m, size_t count, const llme_q8_product* p) {
    if (math_mode() != LLME_MATH_TENSOR)
        return fail(LLME_E_UNSUPPORTED,
                    "llme_batch_q8_create: m >= 128 runs on the tensor cores (LLME_MATH_TENSOR)");
    if (m * count > (size_t{1} << 30))
        return fail(LLME_E_INVALID, "llme_batch_q8_create: more than 2^30 rows in all");
    int dev = 0, sms = 0;
    int st = current_device(&dev);
    if (st) return st;
    st = device_sms(dev, &sms);
    if (st) return st;
    const bool pair = q8tc_use_pairs(sms);
    const size_t tm = ceil_div(m, static_cast<size_t>(q8tc_tile_m()));
    std::vector<Q8TcItem> items(count);
    std::vector<size_t> scratch_off(count);
    size_t scratch_bytes = 0;
    std::vector<int> row_begin(count + 1, 0);
    std::vector<uint2> units;
    std::vector<size_t> work;
    for (size_t i = 0; i < count; ++i) {
        const llme_q8_product& q = p[i];
        const std::string where = "llme_batch_q8_create: product " + std::to_string(i) + " " +
                                  shapes(m, q.n, q.k);
        if (q.n == 0 || q.k == 0 || q.n % 16)
            return fail(LLME_E_INVALID, where + ": needs n % 16 == 0 and nonzero n, k");
        if (q.k > static_cast<size_t>(kQ8TcMaxK))
            return fail(LLME_E_INVALID, where + ": k above " + std::to_string(kQ8TcMaxK));
        if (m * q.k >= kMaxElems || q.k * q.n >= kMaxElems || m * q.n >= kMaxElems)
            return fail(LLME_E_INVALID, where + ": more than 2^31 elements");
        if (reinterpret_cast<uintptr_t>(q.B) % 16)
            return fail(LLME_E_INVALID, where + ": B must be 16-byte aligned");
        scratch_off[i] = scratch_bytes;
        scratch_bytes += q8tc_operand_bytes(m, q.k);
        scratch_bytes = round_up(scratch_bytes, 256);
        row_begin[i + 1] = row_begin[i] + static_cast<int>(m);
        const size_t tiles = tm * ceil_div(q.n, static_cast<size_t>(q8tc_tile_n(pair)));
        for (size_t t = 0; t < tiles; ++t) {
            units.push_back(make_uint2(static_cast<unsigned>(i), static_cast<unsigned>(t)));
            // Work of a tile: its k-blocks plus about two for the epilogue.
            work.push_back(ceil_div(q.k, size_t{128}) + 2);
        }
    }
    const int grid = static_cast<int>(std::min<size_t>(units.size(), pair ? sms / 2 : sms));
    const auto per_cta = lpt_assign(work, grid);
    std::vector<uint2> table;
    std::vector<int> cta_begin(grid + 1, 0);
    size_t max_cta_units = 0;
    for (int c = 0; c < grid; ++c) {
        cta_begin[c] = static_cast<int>(table.size());
        for (size_t u : per_cta[c]) table.push_back(units[u]);
        max_cta_units = std::max(max_cta_units, per_cta[c].size());
    }
    cta_begin[grid] = static_cast<int>(table.size());

    auto* b = new llme_batch;
    b->dev = dev;
    b->tc = true;
    cudaError_t e = cudaMalloc(&b->scratch, std::max<size_t>(scratch_bytes, 256));
    if (e != cudaSuccess) {
        delete b;
        return cuda_fail(e, "alloc batch scratch");
    }
    std::vector<CUtensorMap> mw(count), mh(count), ml(count);
    for (size_t i = 0; i < count; ++i) {
        const llme_q8_product& q = p[i];
        const size_t kp = q8tc_pitch(q.k);
        int8_t* hi = static_cast<int8_t*>(b->scratch) + scratch_off[i];
        int8_t* lo = hi + q8tc_rows_bytes(m, q.k);
        float* rs = reinterpret_cast<float*>(lo + q8tc_rows_bytes(m, q.k));
        items[i] = Q8TcItem{q.A, q.C, q.scale, hi, lo, rs, static_cast<int>(m),
                            static_cast<int>(q.n), static_cast<int>(q.k), static_cast<int>(kp),
                            q.accumulate ? 1 : 0, 0};
        st = encode_map(q.B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, q.k, q.n, 128, 128, &mw[i],
                        CU_TENSOR_MAP_SWIZZLE_128B);
        if (!st)
            st = encode_map(hi, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, m, q.k, 128, 128, &mh[i],
                            CU_TENSOR_MAP_SWIZZLE_128B, kp);
        if (!st)
            st = encode_map(lo, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, m, q.k, 128, 128, &ml[i],
                            CU_TENSOR_MAP_SWIZZLE_128B, kp);
        if (st) {
            cudaFree(b->scratch);
            delete b;
            return st;
        }
    }
    // [maps W][maps hi][maps lo][items][row_begin][unit table][cta_begin], 128-byte aligned parts.
    const size_t maps_bytes = count * sizeof(CUtensorMap);
    const size_t items_off = 3 * maps_bytes;
    const size_t rows_off = round_up(items_off + count * sizeof(Q8TcItem), 128);
    const size_t table_off = round_up(rows_off + row_begin.size() * sizeof(int), 128);
    const size_t begin_off = round_up(table_off + table.size() * sizeof(uint2), 128);
    const size_t bytes = begin_off + cta_begin.size() * sizeof(int);
    e = cudaMalloc(&b->dmem, bytes);
    if (e != cudaSuccess) {
        cudaFree(b->scratch);
        delete b;
        return cuda_fail(e, "alloc batch");
    }
    char* base = static_cast<char*>(b->dmem);
    e = cudaMemcpy(base, mw.data(), maps_bytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(base + maps_bytes, mh.data(), maps_bytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(base + 2 * maps_bytes, ml.data(), maps_bytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(base + items_off, items.data(), count * sizeof(Q8TcItem), cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(base + rows_off, row_begin.data(), row_begin.size() * sizeof(int),
                       cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(base + table_off, table.data(), table.size() * sizeof(uint2),
                       cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(base + begin_off, cta_begin.data(), cta_begin.size() * sizeof(int),
                       cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(b->dmem);
        cudaFree(b->scratch);
        delete b;
        return cuda_fail(e, "upload batch");
    }
    Q8TcBatchArgs& a = b->targs;
    a.count = static_cast<int>(count);
    a.rows = row_begin[count];
    a.bulk = true;
    for (size_t i = 0; i < count; ++i) {
        a.max_k = std::max(a.max_k, static_cast<int>(p[i].k));
        a.bulk = a.bulk && p[i].k % 4 == 0 && reinterpret_cast<uintptr_t>(p[i].A) % 16 == 0;
    }
    a.bulk = a.bulk && static_cast<size_t>(a.max_k) * 4 <= static_cast<size_t>(kQ8TcSplitSmemMax);
    a.items = reinterpret_cast<const Q8TcItem*>(base + items_off);
    a.row_begin = reinterpret_cast<const int*>(base + rows_off);
    a.tmW = reinterpret_cast<const CUtensorMap*>(base);
    a.tmHi = reinterpret_cast<const CUtensorMap*>(base + maps_bytes);
    a.tmLo = reinterpret_cast<const CUtensorMap*>(base + 2 * maps_bytes);
    a.unit_table = reinterpret_cast<const uint2*>(base + table_off);
    a.cta_begin = reinterpret_cast<const int*>(base + begin_off);
    a.pair = pair;
    a.slots = grid;
    *out = b;
    return LLME_OK;
}

int batch_create(llme_batch_t** out, size_t m, size_t count, const llme_q8_product* p) {
    g_error.clear();
    if (!out) return fail(LLME_E_INVALID, "llme_batch_q8_create: null result pointer");
    *out = nullptr;
    if (count < 1 || count > 65535)
        return fail(LLME_E_INVALID, "llme_batch_q8_create: 1..65535 products, got " +
                                        std::to_string(count));
    if (!p) return fail(LLME_E_INVALID, "llme_batch_q8_create: null products");
    for (size_t i = 0; i < count; ++i)
        if (!p[i].A || !p[i].B || !p[i].scale || !p[i].C)
            return fail(LLME_E_INVALID, "llme_batch_q8_create: product " + std::to_string(i) +
                                            ": null pointer");
    if (m >= 128) return batch_create_tc(out, m, count, p);
    if (m < 1 || m > 8)
        return fail(LLME_E_INVALID,
                    "llme_batch_q8_create: m must be 1..8 or at least 128, got " + std::to_string(m));
    std::vector<BatchItem> items(count);
    std::vector<CUtensorMap> mb(count), ma(count);
    std::vector<unsigned> units;
    std::vector<size_t> unit_bytes;
    for (size_t i = 0; i < count; ++i) {
        const llme_q8_product& q = p[i];
        const std::string where = "llme_batch_q8_create: product " + std::to_string(i) + " " +
                                  shapes(m, q.n, q.k);
        if (q.n == 0 || q.k == 0 || q.n % 16 || q.k % 4)
            return fail(LLME_E_INVALID, where + ": needs n % 16 == 0, k % 4 == 0, both nonzero");
        if (m * q.k >= kMaxElems || q.k * q.n >= kMaxElems || m * q.n >= kMaxElems)
            return fail(LLME_E_INVALID, where + ": more than 2^31 elements");
        if (reinterpret_cast<uintptr_t>(q.A) % 16 || reinterpret_cast<uintptr_t>(q.B) % 16)
            return fail(LLME_E_INVALID, where + ": A and B must be 16-byte aligned");
        const size_t strips = ceil_div(q.n, gemv_tma_cols(true));
        if (strips > 65535) return fail(LLME_E_INVALID, where + ": too many columns");
        items[i] = BatchItem{q.A, q.C, q.scale, static_cast<int>(q.n), static_cast<int>(q.k),
                             q.accumulate ? 1 : 0, 0};
        int st = encode_map(q.B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, q.k, q.n, kGemvRowBytes,
                            kGemvBoxRows, &mb[i]);
        if (st) return st;
        st = encode_map(q.A, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, m, q.k, kGemvBoxRows,
                        static_cast<uint32_t>(m), &ma[i]);
        if (st) return st;
        for (size_t sidx = 0; sidx < strips; ++sidx) {
            units.push_back(static_cast<unsigned>(i << 16 | sidx));
            // Work of a unit: its weight bytes plus a fixed cost for the per-unit reduction.
            unit_bytes.push_back(q.k * static_cast<size_t>(gemv_tma_cols(true)) + 16384);
        }
    }
    int dev = 0, sms = 0;
    int st = current_device(&dev);
    if (st) return st;
    st = device_sms(dev, &sms);
    if (st) return st;
    // Longest-processing-time-first: units by decreasing work, each to the CTA with the least
    // work so far (ties to the lower index). Deterministic, and within a few percent of the
    // best possible makespan; each CTA then runs its units in their original order.
    const int grid = static_cast<int>(std::min<size_t>(units.size(), gemv_batch_ctas_per_sm() * sms));
    const auto per_cta = lpt_assign(unit_bytes, grid);
    std::vector<unsigned> table;
    std::vector<int> cta_begin(grid + 1, 0);
    size_t max_cta_units = 0;
    for (int c = 0; c < grid; ++c) {
        cta_begin[c] = static_cast<int>(table.size());
        for (size_t u : per_cta[c]) table.push_back(units[u]);
        max_cta_units = std::max(max_cta_units, per_cta[c].size());
    }
    cta_begin[grid] = static_cast<int>(table.size());
    // [maps B][maps A][items][unit table], each part 128-byte aligned.
    const size_t maps_bytes = count * sizeof(CUtensorMap);
    const size_t items_off = 2 * maps_bytes;
    const size_t table_off = round_up(items_off + count * sizeof(BatchItem), 128);
    const size_t begin_off = round_up(table_off + table.size() * sizeof(unsigned), 128);
    const size_t bytes = begin_off + cta_begin.size() * sizeof(int);
    auto* b = new llme_batch;
    b->dev = dev;
    cudaError_t e = cudaMalloc(&b->dmem, bytes);
    if (e != cudaSuccess) {
        delete b;
        return cuda_fail(e, "alloc batch");
    }
    char* base = static_cast<char*>(b->dmem);
    e = cudaMemcpy(base, mb.data(), maps_bytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(base + maps_bytes, ma.data(), maps_bytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(base + items_off, items.data(), count * sizeof(BatchItem), cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(base + table_off, table.data(), table.size() * sizeof(unsigned),
                       cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(base + begin_off, cta_begin.data(), cta_begin.size() * sizeof(int),
                       cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(b->dmem);
        delete b;
        return cuda_fail(e, "upload batch");
    }
    b->max_cta_units = max_cta_units;
    BatchArgs& a = b->args;
    a.m = static_cast<int>(m);
    a.units = static_cast<int>(table.size());
    a.tmB = reinterpret_cast<const CUtensorMap*>(base);
    a.tmA = reinterpret_cast<const CUtensorMap*>(base + maps_bytes);
    a.items = reinterpret_cast<const BatchItem*>(base + items_off);
    a.unit_table = reinterpret_cast<const unsigned*>(base + table_off);
    a.cta_begin = reinterpret_cast<const int*>(base + begin_off);
    a.grid = grid;
    *out = b;
    return LLME_OK;
}

}  // namespace

namespace llme {
int tensor_map_2d(const void* ptr, CUtensorMapDataType dtype, size_t esz, uint64_t rows,
                  uint64_t cols, uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows,
                  CUtensorMap* out) {
    return tensor_map(ptr, dtype, esz, rows, cols, box_cols, box_rows, out,
                      CU_TENSOR_MAP_SWIZZLE_NONE, pitch_bytes);
}
int set_error(int code, const std::string& msg) { return fail(code, msg); }
int host_failure(bool out_of_memory) noexcept {
    g_error.clear();
    try {
        g_error = out_of_memory ? "host: out of memory" : "host: internal error";
    } catch (...) {
    }
    return LLME_E_HOST;
}
int set_cuda_error(cudaError_t e, const char* what) { return cuda_fail(e, what); }
int run_product(size_t m, size_t n, size_t k, const float* A, const void* B, const float* scale,
                float* C, bool q8, int kernel, bool accumulate, const float* rms, unsigned flags,
                void* stream) {
    return run(m, n, k, A, B, scale, C, q8, kernel, accumulate, rms, flags, stream);
}
int run_product_epilogue(size_t m, size_t n, size_t k, const float* A, const void* B,
                         const float* scale, float* C, bool q8, const float* rms, unsigned flags,
                         void* stream, const GemvEpilogue& epi, bool accumulate) {
    return run(m, n, k, A, B, scale, C, q8, LLME_KERNEL_AUTOMATIC, accumulate, rms, flags, stream,
               &epi);
}
int plan_product(size_t m, size_t n, size_t k, bool q8, const void* A, const void* B,
                 const float* rms, llme_plan_t* p) {
    int dev = 0, sms = 0;
    int st = current_device(&dev);
    if (!st) st = device_sms(dev, &sms);
    if (st) return st;
    PlanIn in{m, n, k, q8, LLME_KERNEL_AUTOMATIC, false, reinterpret_cast<uintptr_t>(A),
              reinterpret_cast<uintptr_t>(B), reinterpret_cast<uintptr_t>(rms), sms, math_mode()};
    in.gemv_clusters = device_gemv_clusters(dev);
    return make_plan(in, p);
}
}  // namespace llme

extern "C" {

int llme_matmul_q8_noalloc(size_t m, size_t n, size_t k, const float* A, const int8_t* B,
                           const float* scale, float* C, int accumulate, void* stream) {
    return llme::guarded([&]() -> int {
        return run_noalloc(m, n, k, A, B, scale, C, accumulate != 0, stream);
    });
}

int llme_quantize_q8(size_t k, size_t n, const float* W, int8_t* q, float* scale, void* stream) {
    return llme::guarded([&]() -> int {
        g_error.clear();
        if (k == 0 || n == 0) return LLME_OK;
        if (!W || !q || !scale) return fail(LLME_E_INVALID, "llme_quantize_q8: null pointer");
        if (k * n >= kMaxElems)
            return fail(LLME_E_INVALID, "llme_quantize_q8: more than 2^31 elements (" +
                                            std::to_string(k) + "x" + std::to_string(n) + ")");
        cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : cudaStreamPerThread;
        cudaError_t e = launch_quantize_q8(static_cast<int>(k), static_cast<int>(n), W, q, scale, s);
        return e == cudaSuccess ? LLME_OK : cuda_fail(e, "quantize");
    });
}

int llme_embed_rows(size_t n, size_t dim, const int* feed, const float* table, float* x,
                    void* stream) {
    return llme::guarded([&]() -> int {
        g_error.clear();
        if (n == 0 || dim == 0) return LLME_OK;
        if (!feed || !table || !x) return fail(LLME_E_INVALID, "llme_embed_rows: null pointer");
        if (n >= 65536 || n * dim >= kMaxElems)
            return fail(LLME_E_INVALID, "llme_embed_rows: too many rows or elements");
        cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : cudaStreamPerThread;
        cudaError_t e = launch_embed_rows(static_cast<int>(n), static_cast<int>(dim), feed, table, x, s);
        return e == cudaSuccess ? LLME_OK : cuda_fail(e, "embed");
    });
}

int llme_rope_cache(size_t n, int nq, int nkv, int head_size, const int* feed, const float* cos,
                    const float* sin, float* qkv, float* key_cache, float* value_cache,
                    void* stream) {
    return llme::guarded([&]() -> int {
        g_error.clear();
        if (n == 0) return LLME_OK;
        if (!feed || !cos || !sin || !qkv || !key_cache || !value_cache)
            return fail(LLME_E_INVALID, "llme_rope_cache: null pointer");
        if (nq < 0 || nkv <= 0 || head_size <= 0 || head_size % 2 != 0 || n >= 65536 ||
            static_cast<size_t>(nq + 2 * nkv) * head_size * n >= kMaxElems)
            return fail(LLME_E_INVALID, "llme_rope_cache: head_size must be even and positive, nkv "
                                        "positive, n below 65536");
        cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : cudaStreamPerThread;
        cudaError_t e = launch_rope_cache(static_cast<int>(n), nq, nkv, head_size, feed, cos, sin, qkv,
                                          key_cache, value_cache, s);
        return e == cudaSuccess ? LLME_OK : cuda_fail(e, "rope");
    });
}

int llme_swiglu(size_t n, size_t hidden, const float* gu, float* hb, void* stream) {
    return llme::guarded([&]() -> int {
        g_error.clear();
        if (n == 0 || hidden == 0) return LLME_OK;
        if (!gu || !hb) return fail(LLME_E_INVALID, "llme_swiglu: null pointer");
        if (2 * n * hidden >= kMaxElems) return fail(LLME_E_INVALID, "llme_swiglu: too many elements");
        cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : cudaStreamPerThread;
        cudaError_t e = launch_swiglu(static_cast<int>(n), static_cast<int>(hidden), gu, hb, s);
        return e == cudaSuccess ? LLME_OK : cuda_fail(e, "swiglu");
    });
}

int llme_rope_tables(size_t seq_len, size_t head_size, float* cos, float* sin) {
    return llme::guarded([&]() -> int {
        g_error.clear();
        if (seq_len == 0) return LLME_OK;
        if (!cos || !sin) return fail(LLME_E_INVALID, "llme_rope_tables: null pointer");
        if (head_size == 0 || head_size % 2 != 0)
            return fail(LLME_E_INVALID, "llme_rope_tables: head_size must be even and positive");
        rope_tables(seq_len, head_size, cos, sin);
        return LLME_OK;
    });
}

int llme_batch_q8_create(llme_batch_t** batch, size_t m, size_t count,
                         const llme_q8_product* products) {
    return llme::guarded([&]() -> int {
        return batch_create(batch, m, count, products);
    });
}

int llme_batch_run(llme_batch_t* b, unsigned flags, void* stream) {
    return llme::guarded([&]() -> int {
        g_error.clear();
        if (!b) return fail(LLME_E_INVALID, "llme_batch_run: null batch");
        int dev = 0;
        int st = current_device(&dev);
        if (st) return st;
        if (dev != b->dev) return fail(LLME_E_INVALID, "llme_batch_run: batch belongs to another device");
        if (b->tc) {
            Q8TcBatchArgs t = b->targs;
            t.stream = stream ? static_cast<cudaStream_t>(stream) : cudaStreamPerThread;
            cudaError_t e = launch_q8tc_batch(t);
            return e == cudaSuccess ? LLME_OK : cuda_fail(e, "launch");
        }
        BatchArgs a = b->args;
        a.stream = stream ? static_cast<cudaStream_t>(stream) : cudaStreamPerThread;
        a.pdl = (flags & LLME_FLAG_WEIGHTS_STATIC) != 0;
        cudaError_t e = launch_gemv_batch(a);
        return e == cudaSuccess ? LLME_OK : cuda_fail(e, "launch");
    });
}

int llme_batch_run_rowpar(llme_batch_t* b, llme_comm_t* comm, unsigned flags, void* stream) {
    return llme::guarded([&]() -> int {
        g_error.clear();
        if (!b) return fail(LLME_E_INVALID, "llme_batch_run_rowpar: null batch");
        int dev = 0;
        int st = current_device(&dev);
        if (st) return st;
        if (dev != b->dev)
            return fail(LLME_E_INVALID, "llme_batch_run_rowpar: batch belongs to another device");
        if (b->tc) return fail(LLME_E_UNSUPPORTED, "llme_batch_run_rowpar: m >= 128 batch");
        GemvEpilogue epi;
        st = comm_peer_sum(comm, &epi);
        if (st) return st;
        BatchArgs a = b->args;
        const size_t floats = b->max_cta_units * static_cast<size_t>(a.m) * gemv_tma_cols(true);
        if (a.grid > epi.peer.units || floats > static_cast<size_t>(epi.peer.unit_words))
            return fail(LLME_E_UNSUPPORTED, "llme_batch_run_rowpar: a CTA's " + std::to_string(floats) +
                                                " values exceed the receive area's " +
                                                std::to_string(epi.peer.unit_words));
        a.stream = stream ? static_cast<cudaStream_t>(stream) : cudaStreamPerThread;
        a.pdl = (flags & LLME_FLAG_WEIGHTS_STATIC) != 0;
        a.peer_sum = true;
        a.peer = epi.peer;
        cudaError_t e = launch_gemv_batch(a);
        return e == cudaSuccess ? LLME_OK : cuda_fail(e, "launch");
    });
}

int llme_batch_destroy(llme_batch_t* b) {
    return llme::guarded([&]() -> int {
        if (!b) return LLME_OK;
        cudaError_t e = cudaFree(b->dmem);
        if (b->scratch) {
            cudaError_t e2 = cudaFree(b->scratch);
            if (e == cudaSuccess) e = e2;
        }
        delete b;
        return e == cudaSuccess ? LLME_OK : cuda_fail(e, "free batch");
    });
}


int llme_matmul_f32(size_t m, size_t n, size_t k, const float* A, const float* B, float* C,
                    int kernel, int accumulate, const float* rms_weight, unsigned flags,
                    void* stream) {
    return llme::guarded([&]() -> int {
        return run(m, n, k, A, B, nullptr, C, false, kernel, accumulate != 0, rms_weight, flags,
                   stream);
    });
}

int llme_matmul_q8(size_t m, size_t n, size_t k, const float* A, const int8_t* B,
                   const float* scale, float* C, int kernel, int accumulate,
                   const float* rms_weight, unsigned flags, void* stream) {
    return llme::guarded([&]() -> int {
        return run(m, n, k, A, B, scale, C, true, kernel, accumulate != 0, rms_weight, flags, stream);
    });
}

const char* llme_last_error(void) { return g_error.c_str(); }

size_t llme_scratch_generation(void) { return g_generation.load(); }

int llme_synchronize(void) {
    return llme::guarded([&]() -> int {
        g_error.clear();
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return cuda_fail(e, "synchronize");
        const unsigned dev_err =
            read_and_clear_gemv_error() | read_and_clear_tiled_error() | read_and_clear_tc_error() |
            read_and_clear_q8tc_error() | read_and_clear_skinny_error() | read_and_clear_attn_error() |
            read_and_clear_f32sk_error() | read_and_clear_ops_error();
        if (dev_err) return fail(LLME_E_TIMEOUT, "device: a bounded wait in a kernel gave up");
        return LLME_OK;
    });
}

int llme_device_available(void) {
    int count = 0;
    return cudaGetDeviceCount(&count) == cudaSuccess && count > 0;
}

int llme_device_supported(void) {
    int dev = 0, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
        return 0;
    return major == 10;
}

int llme_device_status(void) {
    return llme::guarded([&]() -> int {
        g_error.clear();
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return cuda_fail(e, "synchronize");
        const unsigned dev_err =
            read_and_clear_gemv_error() | read_and_clear_tiled_error() | read_and_clear_tc_error() |
            read_and_clear_q8tc_error() | read_and_clear_skinny_error() | read_and_clear_attn_error() |
            read_and_clear_f32sk_error() | read_and_clear_ops_error();
        return dev_err ? fail(LLME_E_TIMEOUT, "device: a bounded wait in a kernel gave up") : LLME_OK;
    });
}

int llme_set_math(int math) {
    const int prev = math_mode();
    if (math != LLME_MATH_TENSOR && math != LLME_MATH_FP32) {
        llme::guarded([&] { return fail(LLME_E_INVALID, "llme_set_math: unknown mode " +
                                                           std::to_string(math)); });
        return -1;
    }
    g_math.store(math);
    return prev;
}

int llme_get_math(void) { return math_mode(); }

int llme_alloc(void** ptr, size_t bytes) {
    return llme::guarded([&]() -> int {
        if (!ptr) return fail(LLME_E_INVALID, "llme_alloc: null result pointer");
        *ptr = nullptr;
        if (bytes == 0) return LLME_OK;
        cudaError_t e = cudaMalloc(ptr, bytes);
        return e == cudaSuccess ? LLME_OK : cuda_fail(e, "alloc");
    });
}

int llme_free(void* ptr) {
    return llme::guarded([&]() -> int {
        if (!ptr) return LLME_OK;
        cudaError_t e = cudaFree(ptr);
        return e == cudaSuccess ? LLME_OK : cuda_fail(e, "free");
    });
}

int llme_copy_to_device(void* dst, const void* src, size_t bytes) {
    return llme::guarded([&]() -> int {
        if (!bytes) return LLME_OK;
        cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, cudaStreamPerThread);
        if (e == cudaSuccess) e = cudaStreamSynchronize(cudaStreamPerThread);
        return e == cudaSuccess ? LLME_OK : cuda_fail(e, "upload");
    });
}

int llme_copy_to_host(void* dst, const void* src, size_t bytes) {
    return llme::guarded([&]() -> int {
        if (!bytes) return LLME_OK;
        cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, cudaStreamPerThread);
        if (e == cudaSuccess) e = cudaStreamSynchronize(cudaStreamPerThread);
        return e == cudaSuccess ? LLME_OK : cuda_fail(e, "download");
    });
}

int llme_plan(size_t m, size_t n, size_t k, int is_q8, int kernel, int accumulate,
              uintptr_t a_addr, uintptr_t b_addr, uintptr_t rms_addr, int sm_count, int math,
              llme_plan_t* out) {
    return llme::guarded([&]() -> int {
        return llme_plan_clusters(m, n, k, is_q8, kernel, accumulate, a_addr, b_addr, rms_addr,
                                  sm_count, math, nullptr, out);
    });
}

int llme_plan_clusters(size_t m, size_t n, size_t k, int is_q8, int kernel, int accumulate,
                       uintptr_t a_addr, uintptr_t b_addr, uintptr_t rms_addr, int sm_count,
                       int math, const int* gemv_clusters, llme_plan_t* out) {
    return llme::guarded([&]() -> int {
        g_error.clear();
        if (!out) return fail(LLME_E_INVALID, "llme_plan: null result pointer");
        PlanIn in{m, n, k, is_q8 != 0, kernel, accumulate != 0, a_addr, b_addr, rms_addr, sm_count, math};
        in.gemv_clusters = gemv_clusters;
        return make_plan(in, out);
    });
}

int llme_gemv_cluster_capacity(int* out) {
    return llme::guarded([&]() -> int {
        g_error.clear();
        if (!out) return fail(LLME_E_INVALID, "llme_gemv_cluster_capacity: null result pointer");
        int dev = 0;
        int st = current_device(&dev);
        if (st) return st;
        const int* t = device_gemv_clusters(dev);
        if (!t) return fail(LLME_E_UNSUPPORTED, "llme_gemv_cluster_capacity: the driver gave no answer");
        std::copy(t, t + kGemvMaxCluster, out);
        return LLME_OK;
    });
}

}  // extern "C"
