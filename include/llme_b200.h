/*
 * llme_b200.h -- the C ABI of the B200 (sm_100a) matmul library.
 *
 * This is the thin extern "C" layer under the drop-in C++ API
 * (include/cuda_matmul.h, the same surface as the reference engine's
 * src/cuda_matmul.h). Plain pointers, sizes and int status codes only: a C
 * caller, a ctypes/cffi binding, or the C++ shim call these directly.
 *
 * Layouts (as the reference, cuda_matmul.h:94-107): A is m x k fp32 row-major
 * activations, B is k x n row-major weights ("in x out"), fp32 or int8 with one
 * fp32 scale per column (quant.h:4-9), C is m x n fp32 row-major. Every
 * pointer is device memory unless said otherwise.
 *
 * Streams: `stream` is a cudaStream_t. NULL means the calling thread's
 * per-thread default stream, which is where the reference launches (it is
 * built with --default-stream=per-thread, cuda_matmul.h:7-12). Calls are
 * asynchronous: they return before the GPU finishes. The matmul calls share
 * one scratch per device (split-K partial sums and tickets, the RMSNorm'd copy
 * of A, the split int8 activation rows, B^T); paths that use it are those
 * whose plan has split_bytes, norm_bytes or operand_bytes nonzero. Two such
 * calls whose kernels may overlap on the GPU (different streams with no
 * event between them, concurrent graphs) race on it, as the reference's
 * calls from several host threads do: order them on one stream. Plans with
 * all three zero (the TMA weight-streaming GEMV; the fp32 decode-shaped
 * kernel without RMSNorm) reduce in distributed shared memory and touch no
 * scratch; the grouped batch and the attention take their buffers from the
 * caller.
 *
 * Errors: a nonzero status; llme_last_error() then holds a message for the
 * calling thread (the text the reference puts in its exceptions). A NULL
 * pointer that a call would read or write is LLME_E_INVALID, decided before
 * any device work; pointers a call does not touch (all of them for an empty
 * product, A and B when k == 0) may be NULL.
 */
#ifndef LLME_B200_H
#define LLME_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LLME_ABI_VERSION 1

/* ---- status codes ------------------------------------------------------------------- */
enum {
    LLME_OK = 0,
    LLME_E_INVALID = 1,     /* bad shape/argument: std::invalid_argument in the reference */
    LLME_E_CUDA = 2,        /* CUDA error: std::runtime_error("cuda: <what>: <msg>") */
    LLME_E_TIMEOUT = 3,     /* a bounded device-side wait gave up (see llme_device_status) */
    LLME_E_UNSUPPORTED = 4, /* no usable sm_100 device, or a feature this build lacks */
    LLME_E_NCCL = 5,        /* NCCL error in a sharded call */
    LLME_E_HOST = 6,        /* host side: memory exhausted or an internal error; no
                               exception ever crosses this interface */
    LLME_E_RANGE = 7        /* a token or position outside the model's range:
                               std::out_of_range in the reference (its check_feed) */
};

/* ---- kernel choice: GpuKernel, cuda_matmul.h:66-72 ---------------------------------- */
enum {
    LLME_KERNEL_AUTOMATIC = 0,   /* weight-streaming GEMV for m <= 8, split-K tiles up to m = 127,
                                    tcgen05 tensor-core GEMM from m = 128 */
    LLME_KERNEL_NAIVE = 1,       /* one thread per element of C, the reference's summation order */
    LLME_KERNEL_TILED = 2,       /* whole-k tiles (tcgen05 GEMM where the shape allows it) */
    LLME_KERNEL_TILED_SPLIT = 3, /* tiles with k split across CTAs, deterministic reduction */
    LLME_KERNEL_SKINNY = 4       /* m <= 8 only: the weight-streaming GEMV */
};

/* ---- arithmetic of the tensor-core path ------------------------------------------------ */
enum {
    /* Tensor cores (tcgen05) where they pay. m >= 128: fp32 B multiplies in TF32, int8 B
       in kind::i8 against the activations split into two int8 terms (16 bits), both
       accumulating in fp32 / s32; error bound 5e-3 of the row's L2 norm. 9 <= m <= 127
       (and tiled_split): three TF32 terms (fp32 B) or three int8 activation terms (int8 B),
       the fp32 decode path's bound of 1e-5. m <= 8: the fp32-FMA GEMV. Default. */
    LLME_MATH_TENSOR = 0,
    /* fp32-faithful: every product with m >= 9 runs in fp32 FMA, as the reference's kernels
       do: fp32 B with 9..16 rows on the 16-row GEMV, the rest on the SIMT tiles (the GEMV is
       fp32 FMA in both modes). Selected at load time by LLME_B200_MATH=fp32 in the
       environment. */
    LLME_MATH_FP32 = 1
};

/* ---- call flags ------------------------------------------------------------------------ */
enum {
    /* B and scale are not written by the launch that precedes this one on the stream, so the
       kernel may start streaming them before that launch finishes (programmatic dependent
       launch). True for model weights; not assumed by default. */
    LLME_FLAG_WEIGHTS_STATIC = 1u << 0,
    /* Row-parallel products (llme_matmul_*_rowpar): every rank calls with the same m, n and
       k_local and with equally aligned pointers, so every rank's product follows the same
       plan. With a peer-enabled communicator (llme_comm_enable_peer) of 2 to 8 ranks, m <= 8
       and the automatic kernel, the sum over the ranks is then taken inside the product's
       GEMV: each CTA sends its finished columns to the same CTA of every rank over NVLink and
       writes the rank-ordered sum, with no separate all-reduce launch. Ranks that break the
       promise get LLME_E_TIMEOUT from llme_comm_status (bounded waits), not a hang. */
    LLME_FLAG_SAME_SHARDS = 1u << 1
};

/* matmul_cuda(m, n, k, A, const float* B, C, kernel, fusion): cuda_matmul.h:97-99.
 * C (+)= [rmsnorm(A) * rms_weight] x B. accumulate != 0 adds into C (MatmulFusion::accumulate,
 * cuda_matmul.h:85-92); rms_weight != NULL (k floats, device) normalises each row of A first,
 * eps 1e-5. m == 0 or n == 0 does nothing; k == 0 zeroes C unless accumulating. */
int llme_matmul_f32(size_t m, size_t n, size_t k, const float* A, const float* B, float* C,
                    int kernel, int accumulate, const float* rms_weight, unsigned flags,
                    void* stream);

/* matmul_cuda(m, n, k, A, const int8_t* B, scale, C, kernel, fusion): cuda_matmul.h:105-107.
 * C (+)= [rmsnorm(A) * rms_weight] x (B * scale), B int8 k x n, scale n floats. */
int llme_matmul_q8(size_t m, size_t n, size_t k, const float* A, const int8_t* B,
                   const float* scale, float* C, int kernel, int accumulate,
                   const float* rms_weight, unsigned flags, void* stream);

/* Allocation-free variant of llme_matmul_q8 with LLME_KERNEL_TILED_SPLIT. It has no
 * counterpart in the reference, whose matmul_cuda grows its split-K scratch with cudaMalloc.
 *
 * For callers that cannot allocate device memory once they are running: a serving process
 * whose memory pool reserved nearly all of the GPU's HBM at start-up (a cudaMalloc from inside
 * the library would fail, or take memory the pool meant to own), a latency-bound loop that may
 * not take cudaMalloc's device-wide synchronisation after start-up, and a plug-in inside a host
 * runtime that owns all device memory. The split-K partial sums and tickets live in one fixed
 * device array of LLME_NOALLOC_SCRATCH_BYTES inside the library, which every GPU that loads
 * the library holds until the process exits; the call itself makes no cudaMalloc, cudaFree or
 * other allocating call. The caller still passes A, B, scale and C (same layouts and
 * accumulate meaning as llme_matmul_q8; no RMSNorm fusion). It always runs the SIMT split-K
 * tiles (fp32 FMA arithmetic), whatever llme_set_math selects for the other entry points.
 *
 * Limits and contract:
 *  - a product whose split-K plan needs more than the fixed array (partial sums of the k
 *    slices, one 64 x 64 fp32 tile per slice per output tile, plus one ticket per tile; up to
 *    4096 tickets) is rejected with LLME_E_INVALID and a message giving both sizes;
 *  - the first call on each device looks up the array's device address (with that device
 *    current) and clears its tickets; make that first call before any stream capture begins.
 *    The address is kept for the life of the process: after cudaDeviceReset on a device, do
 *    not call the library on that device again (its grow-only scratch is lost the same way);
 *  - all calls on a device share the array and it keeps the last call's contents: calls
 *    whose kernels overlap on the GPU (other streams, other host threads) race on it, so keep
 *    them ordered on one stream. */
#define LLME_NOALLOC_SCRATCH_BYTES (16u << 20)
int llme_matmul_q8_noalloc(size_t m, size_t n, size_t k, const float* A, const int8_t* B,
                           const float* scale, float* C, int accumulate, void* stream);

/* Message for the last failed call on this thread ("" if none). Never NULL. */
const char* llme_last_error(void);

/* cuda_scratch_generation(), cuda_matmul.h:109-112: bumped whenever an internal scratch buffer
 * is reallocated; a CUDA graph captured before the bump must be captured again. */
size_t llme_scratch_generation(void);

/* cuda_synchronize(), cuda_matmul.h:118-119: waits for all queued work on the device, then
 * reports a failed launch (LLME_E_CUDA) or a device-side wait that gave up (LLME_E_TIMEOUT). */
int llme_synchronize(void);

/* cuda_available(), cuda_matmul.h:121-122: 1 if a CUDA device is usable, else 0. */
int llme_device_available(void);

/* 1 if device 0 (or the current device) is sm_100 (B200 class) and this build's kernels can run. */
int llme_device_supported(void);

/* Reads and clears the device-side error word (LLME_OK or LLME_E_TIMEOUT) of the current device.
 * Synchronises the device. */
int llme_device_status(void);

/* Process-wide arithmetic of the tensor-core path (LLME_MATH_*). Returns the previous value,
 * or -1 (message in llme_last_error) for an unknown mode. */
int llme_set_math(int math);
int llme_get_math(void);

/* ---- memory helpers for callers without a CUDA runtime of their own (the C++ shim) ------- */
int llme_alloc(void** ptr, size_t bytes);      /* cudaMalloc */
int llme_free(void* ptr);                      /* cudaFree; NULL is fine */
int llme_copy_to_device(void* dst, const void* src, size_t bytes);   /* waits */
int llme_copy_to_host(void* dst, const void* src, size_t bytes);     /* waits */

/* ---- int8 weight quantisation on the GPU --------------------------------------------------- *
 * Replaces the reference's CPU quantize_q8 (src/quant.h:6, src/quant.cpp:6-28) for weights
 * already in device memory, with the same result bit for bit: W is k x n fp32 row-major;
 * scale[c] = max_r |W[r][c]| / 127 (n floats), q[r][c] = clamp(lround(W[r][c] * (1 / scale[c])),
 * -127, 127) (k x n int8; columns of zeros give scale 0 and q 0). Asynchronous on `stream`
 * (NULL: the per-thread default stream); allocates nothing; k == 0 or n == 0 is a no-op. */
int llme_quantize_q8(size_t k, size_t n, const float* W, int8_t* q, float* scale, void* stream);

/* ---- causal decode attention over a KV cache -------------------------------------------------- *
 * The C form of the reference's cuda_attention.h (src/cuda_attention.h:8-45), which
 * include/cuda_attention.h restates for C++ callers over these three functions. */
typedef struct {
    int n_heads, n_kv_heads, head_size, seq_len;
    size_t q_stride;   /* floats between rows of q; head h starts at h * head_size */
    size_t kv_stride;  /* floats between positions of the caches */
    size_t out_stride; /* floats between rows of out */
} llme_attention_shape;

enum { LLME_ATTN_AUTOMATIC = 0, LLME_ATTN_SINGLE_BLOCK = 1, LLME_ATTN_SPLIT = 2 };

/* LLME_E_INVALID (message in llme_last_error) when `kernel` cannot run shape s: non-positive
 * sizes, n_heads % n_kv_heads, a cache past 32-bit indexing; split: head_size or a stride not
 * divisible by 4, head_size > 512; single_block: head_size + seq_len floats over 48 KB. */
int llme_attention_check(const llme_attention_shape* s, int kernel);
/* Floats of scratch llme_attention needs for up to `rows` rows (0 for single_block). */
size_t llme_attention_scratch_floats(const llme_attention_shape* s, size_t rows, int kernel);
/* Kernels one llme_attention call with these arguments enqueues on its stream: 1, or 2 when the
 * split path may divide a context into chunks (their partials are then merged by a second
 * launch); 0 when the arguments are invalid. Host only. */
size_t llme_attention_launches(const llme_attention_shape* s, size_t rows, int kernel);
/* out[i][h * head_size + d] = sum over t <= *pos_dev + i of softmax_t(q_i,h . k_t / sqrt(hs))
 * v_t[d], kv head h / (n_heads / n_kv_heads); the position is read from device memory.
 * scratch: needs no initial contents (every chunk partial is written before it is read).
 * Asynchronous on `stream` (NULL: per-thread default stream); deterministic bit for bit. */
int llme_attention(const llme_attention_shape* s, size_t rows, const int* pos_dev,
                   const float* q, const float* key_cache, const float* value_cache, float* out,
                   float* scratch, int kernel, void* stream);

/* ---- decode-step helpers (the transformer's elementwise steps, one rank's heads) ------------ *
 * The steps of a decoder layer around the matmuls and the attention for the transformer
 * engine below (what the reference's CudaTransformer computes between its matmuls,
 * src/cuda_model.cu:22-75, and its RoPE tables, src/model.cpp:171-184), used for steps wider
 * than the GEMV's fused epilogues: a rank holds nq query heads and nkv kv heads, and a qkv row is
 * [q: nq * head_size | k: nkv * head_size | v: nkv * head_size]. Positions and token ids are
 * read from device memory, feed[0] = the first position, feed[1 .. n] = the tokens, so one
 * captured graph serves every position. All asynchronous on `stream` (NULL: per-thread
 * default stream). */
/* x[i] = table[feed[1 + i]] (rows of dim floats), i < n; token ids must lie in the table. */
int llme_embed_rows(size_t n, size_t dim, const int* feed, const float* table, float* x,
                    void* stream);
/* For row i at position feed[0] + i: rotates each (even, odd) pair of q and k by the angle of
 * the pair's index within its head (cos / sin: seq_len x head_size / 2, llme_rope_tables), and
 * writes the rotated k and the v row into the caches (rows of nkv * head_size floats) at that
 * position. head_size even. */
int llme_rope_cache(size_t n, int nq, int nkv, int head_size, const int* feed, const float* cos,
                    const float* sin, float* qkv, float* key_cache, float* value_cache,
                    void* stream);
/* hb[r][c] = silu(gu[r][2c]) * gu[r][2c + 1] for r < n, c < hidden (SwiGLU over interleaved
 * (gate, up) pairs, the layout the transformer engine keeps w13's columns in). */
int llme_swiglu(size_t n, size_t hidden, const float* gu, float* hb, void* stream);
/* Host: the RoPE angle tables (seq_len x head_size / 2 each) with the reference's float
 * expressions, cos[p][j] = cos(p / 10000^(2j / head_size)). */
int llme_rope_tables(size_t seq_len, size_t head_size, float* cos, float* sin);

/* ---- grouped products ------------------------------------------------------------------------ *
 * Many independent int8 products of the same m in ONE persistent launch. The reference issues
 * one matmul_cuda per projection; products that do not read each other's outputs (a layer's
 * q/k/v, w1/w3, or the benchmark's chains of fresh activations) can instead be grouped.
 *   m = 1..8 (decode): every CTA walks a list of (product, 128-column strip) units over the
 *     product's whole k, streaming weights by TMA without a pause between products, and
 *     writes C directly (no cross-CTA reduction). Per product: n % 16 == 0, k % 4 == 0,
 *     A and B 16-byte aligned.
 *   m >= 128 (prefill; LLME_MATH_TENSOR): one launch splits every product's activation rows
 *     into int8 hi / lo terms (scratch owned by the batch), then one persistent tcgen05 launch
 *     runs every product's 128 x 128 output tiles, each CTA its own list balanced by work.
 *     Per product: n % 16 == 0, B 16-byte aligned, k <= 131072. Results are those of
 *     llme_matmul_q8 on the same product, bit for bit.
 * No product's C may overlap another product's A. */
typedef struct {
    size_t n, k;          /* B is k x n int8, C is m x n */
    const float* A;       /* m x k */
    const int8_t* B;
    const float* scale;   /* n */
    float* C;
    int accumulate;       /* C += instead of C = */
} llme_q8_product;
typedef struct llme_batch llme_batch_t;

/* Validates the products and uploads their descriptors (TMA maps, a unit table) to device
 * memory once; the pointers are captured, so the buffers must stay valid while the batch
 * lives. Allocates (cudaMalloc) -- call before capturing graphs. */
int llme_batch_q8_create(llme_batch_t** batch, size_t m, size_t count,
                         const llme_q8_product* products);
/* Runs every product of the batch in one launch on `stream` (no allocation; capturable).
 * flags: LLME_FLAG_WEIGHTS_STATIC as for llme_matmul_q8. */
int llme_batch_run(llme_batch_t* batch, unsigned flags, void* stream);
int llme_batch_destroy(llme_batch_t* batch);

/* ---- multi-GPU: tensor-parallel products over NCCL --------------------------------------- *
 * One process per GPU. The reference has no multi-GPU code (single CudaTransformer); these
 * entry points are additive. Column-parallel weights (wq, wk, wv, w1, w3, classifier) need no
 * new call: each rank runs llme_matmul_* on its contiguous k x (n/ranks) slice of B (and the
 * matching slice of scale) and owns those columns of C. Row-parallel weights (wo, w2) are
 * split along k: each rank holds rows [r*k/ranks, (r+1)*k/ranks) of B, the matching columns
 * of A, and the whole scale vector (the column scale is linear, so it applies to each partial
 * sum), and the m x n partial products are summed with an NCCL all-reduce over NVLink. NCCL
 * (libnccl.so.2) is loaded on first use. */
#define LLME_COMM_ID_BYTES 128
typedef struct llme_comm llme_comm_t;

/* A fresh communicator id (LLME_COMM_ID_BYTES bytes) on one rank, to be shared with all ranks. */
int llme_comm_unique_id(void* id);

/* Joins the communicator of `nranks` ranks with the shared id, on the current device.
 * Initialisation is non-blocking and polled: if it has not finished after timeout_s seconds
 * (a rank that never joins), it is aborted and LLME_E_TIMEOUT returned. */
int llme_comm_init(llme_comm_t** comm, int nranks, int rank, const void* id, double timeout_s);
int llme_comm_destroy(llme_comm_t* comm);   /* after all work on it has finished */
int llme_comm_abort(llme_comm_t* comm);     /* from an error path: frees without waiting */
int llme_comm_size(const llme_comm_t* comm);
int llme_comm_rank(const llme_comm_t* comm);

/* Switches llme_allreduce_sum_f32 (up to max_floats values) from NCCL to the library's own
 * one-shot all-reduce over NVLink peer memory: a symmetric buffer per rank shared through CUDA
 * IPC (handles exchanged once over this communicator; collective: every rank calls it); every
 * rank writes its values into every rank's buffer as epoch-tagged 64-bit words and sums the
 * words it receives in rank order once their tags match (bounded waits), so every rank gets
 * the same bits. Plain peer stores and local loads only. Also sets up the receive areas of the
 * in-kernel rank sums (LLME_FLAG_SAME_SHARDS, llme_batch_run_rowpar). Call before capturing
 * graphs. */
int llme_comm_enable_peer(llme_comm_t* comm, size_t max_floats);

/* Reads and clears the peer all-reduce's device error word: LLME_E_TIMEOUT if a peer did not
 * arrive within the wait limit (its result is then not valid). */
int llme_comm_status(void);

/* In-place sum all-reduce of `count` fp32 values on `stream` (capturable in a CUDA graph). */
int llme_allreduce_sum_f32(float* buf, size_t count, llme_comm_t* comm, void* stream);

/* Row-parallel product: C = A_local x (B_local * scale) summed over ranks (C += ... with
 * accumulate, the residual add: only rank 0 adds its C, so the sum counts it once). A_local
 * is m x k_local (this rank's columns of A), B_local k_local x n, scale n (the full vector).
 * Same kernels as llme_matmul_q8 on the shard, then llme_allreduce_sum_f32 on C, both on
 * `stream`. No RMSNorm fusion here: a row norm needs the whole row of A. */
int llme_matmul_q8_rowpar(size_t m, size_t n, size_t k_local, const float* A_local,
                          const int8_t* B_local, const float* scale, float* C, int kernel,
                          int accumulate, unsigned flags, llme_comm_t* comm, void* stream);
int llme_matmul_f32_rowpar(size_t m, size_t n, size_t k_local, const float* A_local,
                           const float* B_local, float* C, int kernel, int accumulate,
                           unsigned flags, llme_comm_t* comm, void* stream);

/* llme_batch_run for row-parallel products (m = 1..8) with the sum over the ranks taken inside
 * the launch, the multi-GPU form of the grouped step. Every rank creates its batch from
 * products of the same shapes in the same order (equal shards, equally aligned pointers), so
 * every rank's CTA c runs the same units; CTA c sends each unit's finished columns to every
 * rank over NVLink (plain peer stores into the communicator's receive areas), waits once for
 * the other ranks' CTA c and writes the rank-ordered sums to C. No separate all-reduce launch.
 * A product's accumulate applies as given: set it on one rank only to add C once. Needs a
 * peer-enabled communicator (llme_comm_enable_peer) of 2 to 8 ranks; LLME_E_UNSUPPORTED for an
 * m >= 128 batch or a batch whose busiest CTA's values exceed the receive area (4096 floats).
 * A rank that breaks the same-shapes promise gets LLME_E_TIMEOUT from llme_comm_status. */
int llme_batch_run_rowpar(llme_batch_t* batch, llme_comm_t* comm, unsigned flags, void* stream);

/* ---- the transformer engine (the reference's CudaTransformer, optionally tensor-parallel) -- *
 * The reference's Llama-architecture model (src/model.h; its GPU form CudaTransformer,
 * src/cuda_model.cu:164-270) run by this library from C++: every matmul through the kernels
 * above, attention through llme_attention, one model object per GPU.
 *   world = 1: the whole model on the current GPU.
 *   world > 1: rank `rank` holds a slice of every layer: attention heads split by kv head
 *     (kv heads [rank * n_kv / world, ...) and the query heads that read them, so RoPE, the
 *     KV cache and attention stay local); wqkv, w13 and the classifier column-parallel (this
 *     rank's q, k, v / gate, up / vocabulary columns); wo and w2 row-parallel (the rows that
 *     multiply this rank's heads / hidden units), each followed by one sum all-reduce of the
 *     residual stream with the residual add folded in (rank 0 adds it before the sum). int8
 *     weights are quantised per column over the whole matrix, as the reference's quantize_q8
 *     does, so every rank's int8 values are exactly the reference's. With a communicator
 *     (llme_comm_init) the all-reduces run on it; without one, llme_model_group_forward runs
 *     `world` rank models held by one process on one GPU and sums their partials in rank order
 *     (the all-reduce's arithmetic), so the decomposition is testable on one device.
 * A step of at most 8 tokens fuses RoPE with the KV-cache write into the wqkv product and
 * SwiGLU into the w13 product (the GEMV epilogue; w13's gate and up columns are kept
 * interleaved in pairs for it); wider steps run them as separate kernels.
 * Positions follow the reference (its check_feed, src/model.cpp:165-177): tokens in
 * [0, vocab), pos + n <= seq_len, pos <= the number of positions already cached; otherwise
 * LLME_E_RANGE. Every call below runs on the model's own stream and returns when the logits
 * (vocab floats, host memory; the whole vocabulary on every rank) are written. */
typedef struct {
    int dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len;
} llme_model_config;
typedef struct llme_model llme_model_t;

/* Loads a llama2.c checkpoint (the reference's load_checkpoint, src/model.cpp:113-163: the
 * same header and size checks and error texts; LLME_E_INVALID) onto the current GPU; q8:
 * int8 projections. world > 1 without `comm` builds a rank for llme_model_group_forward. */
int llme_model_load(const char* checkpoint, int q8, int world, int rank, llme_comm_t* comm,
                    llme_model_t** model);
/* A model of cfg's shape with weights drawn on the device (projections N(0, 0.02^2),
 * embedding U(-1, 1), unit RMSNorm weights), each rank drawing only its own slices: for
 * benchmarks at sizes no host checkpoint is needed for. */
int llme_model_synthetic(const llme_model_config* cfg, int q8, int world, int rank,
                         llme_comm_t* comm, unsigned long long seed, llme_model_t** model);
int llme_model_get_config(const llme_model_t* model, llme_model_config* cfg);
/* Host only (no GPU): the checkpoint's header and size checks of llme_model_load, and its
 * configuration. */
int llme_checkpoint_config(const char* checkpoint, llme_model_config* cfg);
/* Host only: rank `rank`'s slice of a model split over `world` ranks -- query heads
 * [q0, q0 + nq), kv heads [kv0, kv0 + nkv), hidden units [h0, h0 + hc), vocabulary
 * [v0, v0 + vc) (hidden units and vocabulary in contiguous blocks, the first total % world
 * ranks one larger). LLME_E_INVALID when the kv heads do not split evenly. */
typedef struct {
    int q0, nq, kv0, nkv;
    size_t h0, hc, v0, vc;
} llme_model_slice;
int llme_model_partition(const llme_model_config* cfg, int world, int rank, llme_model_slice* out);
/* This rank's slice: query heads, kv heads, hidden units, vocabulary entries. */
int llme_model_local(const llme_model_t* model, int* q_heads, int* kv_heads, int* hidden,
                     int* vocab);
/* Device bytes this rank streams per decoded token: its projection weights (+ scales) and,
 * per cached position, its keys and values. */
int llme_model_stream_bytes(const llme_model_t* model, size_t* weight_bytes,
                            size_t* kv_bytes_per_position);
/* Feeds tokens[0..n) at positions [pos, pos + n); logits of the last one. */
int llme_model_forward(llme_model_t* model, const int* tokens, size_t n, size_t pos,
                       float* logits);
/* One token through the decode step captured as a CUDA graph (captured after an eager first
 * step, and again whenever a longer step has reallocated the buffers it reads or the
 * library's scratch generation moved, as the reference's CudaTransformer re-captures). */
int llme_model_decode(llme_model_t* model, int token, size_t pos, float* logits);
/* How many times the decode graph has been captured (0 before the first llme_model_decode). */
size_t llme_model_captures(const llme_model_t* model);
/* Benchmark helpers: fill the first `positions` cache rows of every layer with U(-1, 1) and
 * count them as cached; replay the captured decode step `times` times on `stream` (its last
 * token and position, asynchronously, logits left in device memory). */
int llme_model_fill_history(llme_model_t* model, size_t positions, unsigned long long seed);
int llme_model_replay(llme_model_t* model, size_t times, void* stream);
/* One forward over `world` rank models on the current GPU (built with world > 1 and no
 * communicator, ranks 0..world-1 in order), their partial results summed in rank order at
 * every reduction point; rank 0's logits. */
int llme_model_group_forward(llme_model_t* const* ranks, int world, const int* tokens, size_t n,
                             size_t pos, float* logits);
int llme_model_destroy(llme_model_t* model);

/* ---- host-side planning, exposed so the dispatch logic can be tested without a GPU -------- */
enum {
    LLME_PATH_NONE = 0,        /* nothing to launch (m == 0 or n == 0) */
    LLME_PATH_ZERO = 1,        /* k == 0: memset of C */
    LLME_PATH_NAIVE = 2,
    LLME_PATH_GEMV_TMA = 3,    /* weight-streaming GEMV, TMA ring (aligned B, m <= 8; fp32 B
                                  up to 16 rows in LLME_MATH_FP32) */
    LLME_PATH_GEMV_LDG = 4,    /* weight-streaming GEMV, plain loads (ragged B) */
    LLME_PATH_TILED_SIMT = 5,  /* fp32 SIMT tiles, k split across CTAs */
    LLME_PATH_TCGEN05 = 6,     /* tcgen05/TMEM tensor-core GEMM, TF32 (fp32 weights) */
    LLME_PATH_TCGEN05_Q8 = 7,  /* tcgen05/TMEM tensor-core GEMM, int8 weights (kind::i8 on a
                                  two-term int8 split of the activation rows) */
    LLME_PATH_TCGEN05_SKINNY = 8, /* decode-shaped int8 products on tcgen05: three-term split
                                     (fp32-decode accuracy), k slices reduced in a
                                     thread-block cluster as exact int64 sums */
    LLME_PATH_TCGEN05_F32_SKINNY = 9  /* decode-shaped fp32 products on tcgen05 in three TF32
                                         terms (fp32-decode accuracy), k slices reduced in a
                                         thread-block cluster */
};

typedef struct {
    int path;             /* LLME_PATH_* */
    int kernel;           /* the kernel choice after resolving LLME_KERNEL_AUTOMATIC */
    int rms_prepass;      /* 1 if rms_weight is applied by a separate pass over A */
    int grid_x, grid_y;   /* launch grid of the main kernel */
    int slices;           /* k slices reduced deterministically across CTAs (1 = none) */
    int cluster;          /* CTAs per thread-block cluster (slices reduced through DSMEM) */
    int span;             /* rows of k per slice */
    int tile_m, tile_n;   /* rows and columns of C per CTA */
    size_t split_bytes;   /* split-K scratch: partial sums (0 when slices == 1) */
    size_t counter_slots; /* split-K tickets needed (one per output tile) */
    size_t norm_bytes;    /* scratch for the normalised copy of A (rms_prepass) */
    size_t operand_bytes; /* scratch for re-laid-out operands: the int8 hi / lo (/ third)
                             activation rows and row scales of the int8 tensor-core GEMMs, or
                             B^T for the TF32 GEMM at m >= 6144 */
} llme_plan_t;

/* The plan llme_matmul_f32 (is_q8 == 0) or llme_matmul_q8 (is_q8 == 1) would follow on a
 * device with `sm_count` SMs, for A, B and the RMSNorm weight at the given device addresses
 * (rms_addr 0 = no RMSNorm). No GPU is touched. Returns LLME_E_INVALID (with the same
 * message) where the call would. One difference: a GEMV's k slices form thread-block clusters,
 * and on a device the calls take the driver's count of clusters it can hold at once where this
 * function assumes 2 x sm_count / (cluster size); the device may then use fewer slices. */
int llme_plan(size_t m, size_t n, size_t k, int is_q8, int kernel, int accumulate,
              uintptr_t a_addr, uintptr_t b_addr, uintptr_t rms_addr, int sm_count, int math,
              llme_plan_t* out);
/* llme_plan for a device that holds gemv_clusters[c - 1] GEMV clusters of c CTAs at once
 * (c = 1..8, as llme_gemv_cluster_capacity reports; NULL: as llme_plan), so an offline plan
 * matches the one the calls take on that device. No GPU is touched. */
int llme_plan_clusters(size_t m, size_t n, size_t k, int is_q8, int kernel, int accumulate,
                       uintptr_t a_addr, uintptr_t b_addr, uintptr_t rms_addr, int sm_count,
                       int math, const int* gemv_clusters, llme_plan_t* out);
/* The current device's capacity for the weight-streaming GEMV's thread-block clusters:
 * out[c - 1] = clusters of c CTAs it holds at once, c = 1..8 (the driver's occupancy
 * answer, two CTAs per SM; below 2 x SMs / c where clusters do not pack every GPC). */
int llme_gemv_cluster_capacity(int* out);

#ifdef __cplusplus
}
#endif

#endif /* LLME_B200_H */
