// Host-side launchers of the sm_100a kernels, shared between the .cu files
// and the C ABI (capi.cu). Internal to the library.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include <exception>
#include <new>
#include <string>

#include "llme_b200.h"

namespace llme {

// The calling thread's llme_last_error message (defined in capi.cu); return `code`.
int set_error(int code, const std::string& msg);
int set_cuda_error(cudaError_t e, const char* what);
// LLME_E_HOST with a fixed message, allocating nothing (capi.cu).
int host_failure(bool out_of_memory) noexcept;

// The body of a C entry point: an exception thrown on the host (std::bad_alloc from a
// message or a table, or anything else) becomes LLME_E_HOST instead of crossing the C
// boundary, where it would end the calling process.
template <typename F>
int guarded(F&& body) noexcept {
    try {
        return body();
    } catch (const std::bad_alloc&) {
        return host_failure(true);
    } catch (...) {
        return host_failure(false);
    }
}
// A cached 2D tensor map (no swizzle) over `rows` x `cols` elements of esz bytes, rows
// pitch_bytes apart (capi.cu).
int tensor_map_2d(const void* ptr, CUtensorMapDataType dtype, size_t esz, uint64_t rows,
                  uint64_t cols, uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows,
                  CUtensorMap* out);
// The C ABI's products without the public wrapper (capi.cu), for the sharded entry points.
int run_product(size_t m, size_t n, size_t k, const float* A, const void* B, const float* scale,
                float* C, bool q8, int kernel, bool accumulate, const float* rms, unsigned flags,
                void* stream);

// Deterministic split-K across CTAs: a CTA that owns slice s of a tile writes
// its partial sums to partial[(tile * slices + s) * tile_elems + e], bumps
// counters[tile], and the CTA that brings the count to `slices` adds the
// slices in order s = 0, 1, ... and writes C, then resets the counter to 0
// (so counters are all zero between launches).
struct SplitScratch {
    float* partial = nullptr;     // tiles * slices * tile_elems floats
    float* partial_ss = nullptr;  // tiles * slices * rows floats (RMSNorm sums of squares)
    unsigned* counters = nullptr; // one per tile, zero between launches
};

// What the per-call TMA GEMV (m <= 8, or 16) does with a finished pair of adjacent output columns
// (2c, 2c + 1) of row r instead of writing C as is; the decode step of the transformer engine
// fuses its elementwise work here.
enum GemvEpilogueKind { kEpiStore = 0, kEpiRopeCache = 1, kEpiSwiglu = 2, kEpiPeerSum = 3 };

// kEpiPeerSum: the tensor-parallel sum of a row-parallel product taken inside the GEMV. Every
// rank runs the same plan, so CTA u owns the same output elements on every rank. CTA u writes
// each finished value (its partial, plus C on the rank that accumulates) into region
// (slot, u, this rank) of every rank's receive area as one 64-bit word, the value's bits
// tagged with the call's epoch (a single relaxed system-scope store, so the value and its
// tag land together: no fence and no separate flag). The thread that owns an element then
// polls (bounded) region (slot, u, src) of its own area until src's word carries the epoch,
// for src = 0, 1, ..., and writes the sum in that order to C -- the same bits on every rank.
// A per-CTA epoch in device memory picks the slot (epoch & 1), so back-to-back calls and
// CUDA-graph replays never overwrite a word a peer has not read yet: a rank writes epoch
// e + 2 of CTA u only after reading every peer's e + 1 there, written after that peer's
// kernel of epoch e (which read e) had finished.
constexpr int kPeerSumMaxRanks = 8;
struct PeerSum {
    unsigned long long* base[kPeerSumMaxRanks] = {};  // every rank's receive area (own too)
    int units = 0;                       // CTAs a call may have (grid x * grid y)
    int unit_words = 0;                  // values a CTA owns at most
    unsigned* epoch = nullptr;           // `units` counters, this rank's memory
    unsigned* err = nullptr;             // device error word (LLME_E_TIMEOUT)
    int world = 0, rank = 0;
};

struct GemvEpilogue {
    int kind = kEpiStore;
    // kEpiRopeCache: C's columns are [q: nq heads | k: nkv heads | v: nkv heads] of head_size
    // floats. q and k pairs are rotated by the angle of the pair's index within its head at
    // row r's position feed[0] + r (cos / sin: rows of head_size / 2 per position) and written
    // to C; k and v pairs are also written to the caches (rows of nkv * head_size floats) at
    // that position.
    int nq = 0, nkv = 0, head_size = 0;
    const int* feed = nullptr;
    const float* cos = nullptr;
    const float* sin = nullptr;
    float* key_cache = nullptr;
    float* value_cache = nullptr;
    // kEpiSwiglu: C's columns hold (gate, up) of hidden unit c at 2c and 2c + 1; instead of C,
    // out[r][c] = silu(gate) * up (rows of n / 2 floats).
    float* out = nullptr;
    PeerSum peer;  // kEpiPeerSum
};

struct GemvArgs {
    GemvEpilogue epi;
    int m = 0, n = 0, k = 0;
    const float* A = nullptr;
    const void* B = nullptr;        // int8 or fp32, k x n
    const float* scale = nullptr;   // int8 only
    const float* rms = nullptr;     // k floats or null
    float* C = nullptr;
    bool q8 = false;
    bool accumulate = false;
    int slices = 1;                 // k slices per column strip (grid y)
    int span = 0;                   // rows of k per slice (multiple of the box depth)
    int strips = 0;                 // column strips (grid x)
    SplitScratch split;
    cudaStream_t stream = nullptr;
    bool pdl = false;               // launch with programmatic stream serialization
    // B and scale are not written by the launch before this one on the stream
    // (LLME_FLAG_WEIGHTS_STATIC): the TMA kernel may then copy weights into shared memory
    // before griddepcontrol.wait, not only prefetch them into L2.
    bool weights_static = false;
    // Timeline tracing, used only when gemv.cu is compiled with LLME_GEMV_TRACE: 16 global
    // timer slots per CTA (entry, init, weights issued, activations issued, first data, loop
    // done, CTA sums ready, end, then the cluster reduction's steps). Null and unused in
    // normal builds.
    unsigned long long* trace = nullptr;
};

// TMA GEMV: each CTA streams 128-byte row segments of B (128 int8 or 32 fp32 columns) in
// boxes of 128 rows; k is split across at most kGemvMaxCluster CTAs of one cluster.
constexpr int kGemvRowBytes = 128;
constexpr int kGemvBoxRows = 128;
constexpr int kGemvMaxCluster = 8;
// fp32 B: the TMA GEMV also takes 9..16 rows, as one 16-row instantiation whose A box is
// 16 rows (the rows past m arrive as zero fill and are not stored).
constexpr int kGemvWideRows = 16;
inline int gemv_tma_cols(bool q8) { return q8 ? kGemvRowBytes : kGemvRowBytes / 4; }
// CTAs per SM of one per-call TMA GEMV grid.
constexpr int gemv_call_ctas_per_sm(int) { return 2; }
// Clusters of `cluster` per-call TMA GEMV CTAs the current device holds at once (the driver's
// occupancy answer; below 2 x SMs / cluster when clusters do not pack every GPC); -1 on error.
int gemv_max_active_clusters(int cluster);
constexpr int kGemvLdgCols = 32;

// Grouped GEMV: many independent int8 products of the same m (<= 8) in one persistent
// launch. Work unit = (product, 128-column strip) over the product's whole k; each CTA runs
// its own list of units, balanced by bytes when the batch is created. Everything below lives
// in device memory, written once by llme_batch_q8_create.
struct BatchItem {
    const float* A;      // m x k, 16-byte aligned, k % 4 == 0
    float* C;            // m x n
    const float* scale;  // n
    int n, k;
    int accumulate;
    int pad;
};
struct BatchArgs {
    int m = 0;
    int units = 0;
    const BatchItem* items = nullptr;
    const CUtensorMap* tmB = nullptr;  // per product: B (k x n int8), box 128 x 128
    const CUtensorMap* tmA = nullptr;  // per product: A (m x k fp32), box 128 x m
    const unsigned* unit_table = nullptr;  // units, grouped by CTA: (product << 16) | strip
    const int* cta_begin = nullptr;        // CTA c runs unit_table[cta_begin[c], cta_begin[c+1])
    int grid = 0;
    cudaStream_t stream = nullptr;
    bool pdl = false;
    // The row-parallel sum over the ranks inside the launch (llme_batch_run_rowpar): every
    // rank runs the same batch, so CTA c owns the same units everywhere. CTA c writes each
    // unit's finished strip, epoch-tagged, into its region of every rank's receive area as it
    // goes (unit j of the CTA at j x m x 128 words), and after its last unit reads the ranks'
    // words back in rank order and writes the sums -- the same slots, tags and epochs as the
    // per-call GEMV's kEpiPeerSum, indexed by CTA.
    bool peer_sum = false;
    PeerSum peer;
};
cudaError_t launch_gemv_batch(const BatchArgs& a);
int gemv_batch_ctas_per_sm();

// TMA GEMV: B, A (and rms weight) read through the given tensor maps.
cudaError_t launch_gemv_tma(const GemvArgs& a, const CUtensorMap& tmB, const CUtensorMap& tmA,
                            const CUtensorMap& tmW);
// Plain-load GEMV for shapes the TMA path cannot take (ragged rows, unaligned pointers).
cudaError_t launch_gemv_ldg(const GemvArgs& a);

struct TiledArgs {
    int m = 0, n = 0, k = 0;
    const float* A = nullptr;
    const void* B = nullptr;
    const float* scale = nullptr;
    float* C = nullptr;
    bool q8 = false;
    bool accumulate = false;
    int slices = 1, span = 0;
    SplitScratch split;
    cudaStream_t stream = nullptr;
};
constexpr int kTiledBM = 64, kTiledBN = 64, kTiledBK = 16;
cudaError_t launch_tiled_simt(const TiledArgs& a);
cudaError_t launch_naive(const TiledArgs& a);

// tcgen05 tensor-core GEMM (gemm_tc.cu): 128 x 256 output tiles, TF32 operands read by
// TMA: A K-major (box 32 x 128, 128-byte swizzle); B as stored, MN-major (8 boxes of 32 x 32,
// 128-byte swizzle with 32-byte atoms), or with b_transposed from B^T written by
// launch_transpose, K-major (box 32 x 256, 128-byte swizzle).
struct TcArgs {
    int m = 0, n = 0, k = 0;
    float* C = nullptr;
    bool accumulate = false;
    bool b_transposed = false;
    int tiles_m = 0, tiles_n = 0;
    cudaStream_t stream = nullptr;
    bool pdl = false;
};
int tc_tile_m();
int tc_tile_n();
// Rows of A from which a B^T pass pays for itself (the MN-major MMAs run ~9% slower).
constexpr size_t kTcTransposeMinRows = 6144;
cudaError_t launch_gemm_tf32(const TcArgs& a, const CUtensorMap& tmA, const CUtensorMap& tmB);
// out (n x k) = B^T for fp32 B (k x n).
cudaError_t launch_transpose(const float* B, float* out, int k, int n, cudaStream_t stream);
unsigned read_and_clear_tc_error();

// int8-weight tcgen05 GEMM (gemm_q8_tc.cu). split_rows writes each fp32 activation row
// (RMS-normalised when w is set) as int8 hi / lo rows of pitch kp plus a row scale; the GEMM
// multiplies both by the int8 weights (kind::i8, s32 in TMEM) in persistent CTAs over
// output tiles of q8tc_tile_m() rows x q8tc_tile_n() columns. Requirements: n % 16 == 0,
// B 16-byte aligned, k <= kQ8TcMaxK.
struct Q8TcArgs {
    int m = 0, n = 0, k = 0;
    const float* scale = nullptr;      // n column scales
    const float* row_scale = nullptr;  // m row scales from split_rows
    float* C = nullptr;
    bool accumulate = false;
    bool pair = false;                 // CTA pairs (cta_group::2 MMAs, 256-column tiles)
    int slots = 0;                     // persistent CTAs or pairs (at most the tile count)
    cudaStream_t stream = nullptr;
};
constexpr int kQ8TcMaxK = 131072;  // 127 * 127 * k < 2^31

// Grouped int8 tcgen05 products (llme_batch_* with m >= 128): one split launch over every
// product's rows, then one persistent GEMM launch whose CTAs walk their own lists of
// (product, output tile) units, balanced by work when the batch is created. Everything the
// kernels read lives in device memory, written once at creation.
struct Q8TcItem {
    const float* A;          // m x k fp32
    float* C;                // m x n fp32
    const float* scale;      // n
    int8_t* hi;              // m x kp split rows (batch scratch)
    int8_t* lo;
    float* row_scale;        // m
    int m, n, k, kp;
    int accumulate;
    int pad;
};
struct Q8TcBatchArgs {
    int count = 0;
    int rows = 0;                          // sum of m over the products (split grid)
    int max_k = 0;                         // longest activation row (split shared memory)
    bool bulk = false;                     // every row aligned and short enough for bulk copies
    const Q8TcItem* items = nullptr;
    const int* row_begin = nullptr;        // count + 1 prefix sums of m
    const CUtensorMap* tmW = nullptr;      // per product: W, box 128 x 128, 128B swizzle
    const CUtensorMap* tmHi = nullptr;     // per product: hi rows, box 128 x 128, 128B swizzle
    const CUtensorMap* tmLo = nullptr;
    const uint2* unit_table = nullptr;     // (product, tile) grouped by CTA
    const int* cta_begin = nullptr;        // slot c runs unit_table[cta_begin[c], cta_begin[c+1])
    bool pair = false;                     // slots are CTA pairs (cta_group::2)
    int slots = 0;                         // CTAs, or CTA pairs
    cudaStream_t stream = nullptr;
};
constexpr int kQ8TcSplitSmemMax = 196608;  // bytes of a row the split pass stages in smem
cudaError_t launch_q8tc_batch(const Q8TcBatchArgs& b);
int q8tc_tile_m();
int q8tc_tile_n(bool pair);          // output columns per tile: 128, or 256 for CTA pairs
// Rows of A into int8 term rows of pitch kp: (hi, lo) for two terms, (hi, lo = the middle
// term, t2) for three (t2 null: two terms).
cudaError_t launch_split_rows(int m, int k, int kp, const float* A, const float* w, int8_t* hi,
                              int8_t* lo, int8_t* t2, float* row_scale, cudaStream_t stream,
                              bool pdl);
cudaError_t launch_gemm_q8_tc(const Q8TcArgs& a, const CUtensorMap& tmHi, const CUtensorMap& tmLo,
                              const CUtensorMap& tmB);
unsigned read_and_clear_q8tc_error();

// Decode-shaped int8 products on tcgen05 (gemm_q8_skinny.cu): three-term split rows, one CTA
// per (128-column, rows_per_tile-row) tile and k-slice; the k slices of a tile form one
// thread-block cluster (at most 8) and add their exact int64 sums through DSMEM.
struct SkinnyArgs {
    int m = 0, n = 0, k = 0;
    const float* scale = nullptr;
    const float* row_scale = nullptr;
    float* C = nullptr;
    bool accumulate = false;
    bool weights_static = false;  // weight loads may start before the previous launch ends
    int rows_per_tile = 16;       // 16, 32 or 64
    int slices = 1;               // grid z = cluster size, at most 8
    int span_blocks = 0;          // 128-deep k blocks per slice
    cudaStream_t stream = nullptr;
};
int skinny_rows_per_tile(int m);
int skinny_ctas_per_sm(int rows_per_tile);
cudaError_t launch_gemm_q8_skinny(const SkinnyArgs& a, const CUtensorMap& tmW,
                                  const CUtensorMap& t0, const CUtensorMap& t1,
                                  const CUtensorMap& t2);
unsigned read_and_clear_skinny_error();

// Causal decode attention (attention.cu). The split kernel's scratch: partial o (rows x
// heads x splits x head_size) and (m, l) pairs, merged by a second launch.
struct AttnArgs {
    int n_heads = 0, head_size = 0, group = 1, chunk_cap = 0;
    bool boxes = false;  // keys and values by 2D TMA boxes (head_size <= 256), else row copies
    size_t q_stride = 0, kv_stride = 0, out_stride = 0;
    const int* pos = nullptr;
    const float* q = nullptr;
    const float* k = nullptr;
    const float* v = nullptr;
    float* out = nullptr;
    float* part_o = nullptr;
    float2* part_ml = nullptr;
    size_t scratch_row = 0;       // floats between rows' scratch blocks (the pointers: row 0)
};
unsigned read_and_clear_attn_error();

// Decode-shaped fp32-weight products on tcgen05 in three TF32 terms (gemm_f32_skinny.cu):
// one CTA per (128 columns, rows_per_tile rows, k slice); the k slices of a tile form one
// thread-block cluster (at most 8) and add their partials through DSMEM in rank order.
// Requirements: A and B rows 16-byte aligned (k % 4 == 0, n % 4 == 0).
struct F32SkinnyArgs {
    int m = 0, n = 0, k = 0;
    float* C = nullptr;
    bool accumulate = false;
    bool weights_static = false;
    int rows_per_tile = 16;   // 16, 32 or 64
    int slices = 1;           // grid z = cluster size, at most 8
    int span_blocks = 0;      // 32-deep k blocks per slice
    cudaStream_t stream = nullptr;
};
int f32_skinny_stage_k();
cudaError_t launch_gemm_f32_skinny(const F32SkinnyArgs& a, const CUtensorMap& tmW,
                                   const CUtensorMap& tmA);
unsigned read_and_clear_f32sk_error();

// The reference's quantize_q8 (src/quant.cpp:6-28) on device memory, bit for bit (quant.cu):
// per-column scale = max|B[:,c]| / 127 and q = clamp(lround(B * (1 / scale)), -127, 127).
cudaError_t launch_quantize_q8(int k, int n, const float* B, int8_t* q, float* scale,
                               cudaStream_t stream);

// Decode-step helpers (decode_ops.cu): the transformer's elementwise steps for one rank's
// heads; feed[0] = first position, feed[1..n] = token ids, in device memory.
cudaError_t launch_embed_rows(int n, int dim, const int* feed, const float* table, float* x,
                              cudaStream_t stream);
cudaError_t launch_rope_cache(int n, int nq, int nkv, int head_size, const int* feed,
                              const float* cos_t, const float* sin_t, float* qkv, float* key_cache,
                              float* value_cache, cudaStream_t stream);
// SwiGLU over interleaved (gate, up) column pairs: hb[r][c] = silu(gu[r][2c]) * gu[r][2c + 1].
cudaError_t launch_swiglu(int n, int hidden, const float* gu, float* hb, cudaStream_t stream);
void rope_tables(size_t seq_len, size_t head_size, float* cos_out, float* sin_out);
// bufs_dev: a device array of `ranks` buffer pointers; every buffer becomes the rank-order sum.
cudaError_t launch_rank_sum(float* const* bufs_dev, int ranks, size_t count, cudaStream_t stream);
// Synthetic weights drawn on the device from (seed, element index): N(0, stddev^2), U(lo, hi).
cudaError_t launch_fill_normal(float* out, size_t count, uint64_t seed, float stddev,
                               cudaStream_t stream);
cudaError_t launch_fill_uniform(float* out, size_t count, uint64_t seed, float lo, float hi,
                                cudaStream_t stream);
unsigned read_and_clear_ops_error();

// A product with a fused GEMV epilogue (the TMA GEMV path only; LLME_E_UNSUPPORTED
// before any launch otherwise), and the plan llme_matmul_* would follow for a product.
int run_product_epilogue(size_t m, size_t n, size_t k, const float* A, const void* B,
                         const float* scale, float* C, bool q8, const float* rms, unsigned flags,
                         void* stream, const GemvEpilogue& epi, bool accumulate = false);
// Fills epi with kEpiPeerSum over the communicator's receive areas (comm.cu); LLME_E_UNSUPPORTED
// without a peer-enabled communicator of at most kPeerSumMaxRanks ranks.
int comm_peer_sum(llme_comm_t* comm, GemvEpilogue* epi);
int plan_product(size_t m, size_t n, size_t k, bool q8, const void* A, const void* B,
                 const float* rms, llme_plan_t* p);

// out = rmsnorm(A) * w per row (eps 1e-5), m rows of k.
cudaError_t launch_rmsnorm_rows(int m, int k, const float* A, const float* w, float* out,
                                cudaStream_t stream);

// Reads and clears the device error words of the kernels in each file.
unsigned read_and_clear_gemv_error();
unsigned read_and_clear_tiled_error();

}  // namespace llme
