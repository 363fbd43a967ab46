// The transformer engine: the reference's Llama-architecture model (src/model.h, its GPU form
// CudaTransformer in src/cuda_model.cu:164-270) run by this library from C++, optionally
// tensor-parallel over one process per GPU.
//
// A forward is a sequence of segments separated by the points where tensor-parallel ranks
// must sum partial results: per layer, (1) RMSNorm + wqkv, RoPE + KV-cache write, attention,
// wo into the residual stream; (2) RMSNorm + w13, SwiGLU, w2 into the residual stream; then
// (3) RMSNorm + classifier into the logits. After each segment the residual stream (or the
// logits) is summed over the ranks: inside the wo / w2 GEMV itself when the ranks' shards are
// equal and the communicator has peer receive areas (each CTA exchanges its finished columns
// with the same CTA of every rank over NVLink), else by the communicator's all-reduce (NCCL or
// the NVLink peer all-reduce), or, for ranks emulated in one process, by a rank-order sum on
// the device. Rank 0 adds the residual before the sum (accumulate), the others contribute
// their partial only.
// At most 8 tokens per step: RoPE + cache write and SwiGLU are the GEMV's epilogues; wider
// steps run the separate kernels of decode_ops.cu. The one-token step is captured as a CUDA
// graph reading its token and position from device memory, so one graph serves every
// position, as the reference's CudaTransformer does (src/cuda_model.cu:189-230).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace {

struct Proj {
    void* w = nullptr;        // k x n, int8 or fp32
    float* scale = nullptr;   // n floats (int8 only)
    size_t k = 0, n = 0;
};

struct Layer {
    float* rms_att = nullptr;
    float* rms_ffn = nullptr;
    Proj wqkv, wo, w13, w2;   // w13: gate and up of each hidden unit in adjacent columns
    float* kc = nullptr;      // seq_len x (nkv * head_size)
    float* vc = nullptr;
};

// [start, start + count) of `total` for `rank`: the first total % world ranks take one more.
void shard_range(size_t total, int world, int rank, size_t* start, size_t* count) {
    const size_t base = total / world, extra = total % world;
    *start = rank * base + std::min<size_t>(rank, extra);
    *count = base + (static_cast<size_t>(rank) < extra ? 1 : 0);
}

}  // namespace

struct llme_model {
    llme_model_config cfg{};
    int world = 1, rank = 0;
    bool q8 = false;
    llme_comm_t* comm = nullptr;
    int hs = 0, q0 = 0, nq = 0, kv0 = 0, nkv = 0;
    size_t h0 = 0, hc = 0, v0 = 0, vc = 0, qkv_cols = 0;
    std::vector<void*> allocs;  // every device buffer the model owns
    float* emb = nullptr;
    float* rms_final = nullptr;
    Proj wcls;
    std::vector<Layer> layers;
    float* cos = nullptr;
    float* sin = nullptr;
    int* feed = nullptr;       // device: [position, tokens...]
    int* feed_host = nullptr;  // pinned
    float* logits = nullptr;
    float* x = nullptr;        // activation rows, grown to the widest step so far
    float* qkv = nullptr;
    float* att = nullptr;
    float* gu = nullptr;
    float* hb = nullptr;
    float* scratch = nullptr;
    size_t rows = 0;
    size_t own_generation = 0;  // bumped when the activation rows are reallocated
    size_t filled = 0;
    cudaStream_t stream = nullptr;
    cudaGraphExec_t graph = nullptr;
    size_t graph_generation = 0;
    size_t captures = 0;
    float** group_bufs = nullptr;  // device pointer table for the emulated-rank sums
    llme_attention_shape shape{};
};

namespace {

using llme::set_cuda_error;
using llme::set_error;

int cu(cudaError_t e, const char* what) { return e == cudaSuccess ? LLME_OK : set_cuda_error(e, what); }

template <typename T>
int dalloc(llme_model& m, size_t count, T** out, bool zero = true) {
    void* p = nullptr;
    const size_t bytes = std::max<size_t>(count * sizeof(T), 16);
    int st = cu(cudaMalloc(&p, bytes), "model: alloc");
    if (st) return st;
    m.allocs.push_back(p);
    if (zero) {
        st = cu(cudaMemset(p, 0, bytes), "model: zero");
        if (st) return st;
    }
    *out = static_cast<T*>(p);
    return LLME_OK;
}

void dfree(llme_model& m, void* p) {
    if (!p) return;
    auto it = std::find(m.allocs.begin(), m.allocs.end(), p);
    if (it != m.allocs.end()) m.allocs.erase(it);
    cudaFree(p);
}

int upload(llme_model& m, const float* host, size_t count, float** out) {
    int st = dalloc(m, count, out, false);
    if (st) return st;
    return cu(cudaMemcpy(*out, host, count * sizeof(float), cudaMemcpyHostToDevice), "model: upload");
}

// A projection of k x n fp32 values already on the device (dev_full, freed here): kept as is
// (fp32), or quantised per column over all k rows as the reference's quantize_q8 does; with
// rows != nullptr only rows [rows[0], rows[0] + rows[1]) are kept (the whole scale vector
// stays: it multiplies each row-parallel partial sum).
int finish_proj(llme_model& m, float* dev_full, size_t k, size_t n, const size_t* rows, Proj* out) {
    const size_t r0 = rows ? rows[0] : 0, rc = rows ? rows[1] : k;
    out->k = rc;
    out->n = n;
    if (!m.q8) {
        if (!rows) {
            out->w = dev_full;
            return LLME_OK;
        }
        float* w = nullptr;
        int st = dalloc(m, rc * n, &w, false);
        if (!st) st = cu(cudaMemcpy(w, dev_full + r0 * n, rc * n * sizeof(float), cudaMemcpyDeviceToDevice),
                         "model: slice");
        dfree(m, dev_full);
        out->w = w;
        return st;
    }
    int8_t* q = nullptr;
    int st = dalloc(m, k * n, &q, false);
    if (!st) st = dalloc(m, n, &out->scale, false);
    if (!st) st = llme_quantize_q8(k, n, dev_full, q, out->scale, m.stream);
    if (!st) st = cu(cudaStreamSynchronize(m.stream), "model: quantise");
    dfree(m, dev_full);
    if (st) return st;
    if (!rows) {
        out->w = q;
        return LLME_OK;
    }
    int8_t* qs = nullptr;
    st = dalloc(m, rc * n, &qs, false);
    if (!st) st = cu(cudaMemcpy(qs, q + r0 * n, rc * n, cudaMemcpyDeviceToDevice), "model: slice");
    dfree(m, q);
    out->w = qs;
    return st;
}

// Partition of heads, hidden units and vocabulary for (world, rank); LLME_E_INVALID when the
// configuration is not a model or the kv heads do not split evenly.
int slice_of(const llme_model_config& c, int world, int rank, llme_model_slice* out) {
    if (c.dim <= 0 || c.hidden_dim <= 0 || c.n_layers <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 ||
        c.vocab_size <= 0 || c.seq_len <= 0)
        return set_error(LLME_E_INVALID, "model: every configuration field must be positive");
    if (c.dim % c.n_heads != 0 || (c.dim / c.n_heads) % 2 != 0 || c.n_heads % c.n_kv_heads != 0)
        return set_error(LLME_E_INVALID, "model: dim must split into even-sized heads, and query "
                                         "heads into whole groups per kv head");
    if (world < 1 || rank < 0 || rank >= world)
        return set_error(LLME_E_INVALID, "model: rank " + std::to_string(rank) + " of " + std::to_string(world));
    if (c.n_kv_heads % world != 0)
        return set_error(LLME_E_INVALID, "tensor parallel: " + std::to_string(c.n_kv_heads) +
                                             " kv heads do not split over " + std::to_string(world) + " ranks");
    const int group = c.n_heads / c.n_kv_heads;
    out->nkv = c.n_kv_heads / world;
    out->kv0 = rank * out->nkv;
    out->nq = out->nkv * group;
    out->q0 = out->kv0 * group;
    shard_range(c.hidden_dim, world, rank, &out->h0, &out->hc);
    shard_range(c.vocab_size, world, rank, &out->v0, &out->vc);
    return LLME_OK;
}

int partition(llme_model& m) {
    llme_model_slice sl;
    int st = slice_of(m.cfg, m.world, m.rank, &sl);
    if (st) return st;
    if (m.comm && (llme_comm_size(m.comm) != m.world || llme_comm_rank(m.comm) != m.rank))
        return set_error(LLME_E_INVALID, "model: the communicator's ranks differ from the model's");
    const llme_model_config& c = m.cfg;
    m.hs = c.dim / c.n_heads;
    m.q0 = sl.q0;
    m.nq = sl.nq;
    m.kv0 = sl.kv0;
    m.nkv = sl.nkv;
    m.h0 = sl.h0;
    m.hc = sl.hc;
    m.v0 = sl.v0;
    m.vc = sl.vc;
    m.qkv_cols = static_cast<size_t>(m.nq + 2 * m.nkv) * m.hs;
    m.shape.n_heads = m.nq;
    m.shape.n_kv_heads = m.nkv;
    m.shape.head_size = m.hs;
    m.shape.seq_len = c.seq_len;
    m.shape.q_stride = m.qkv_cols;
    m.shape.kv_stride = static_cast<size_t>(m.nkv) * m.hs;
    m.shape.out_stride = static_cast<size_t>(m.nq) * m.hs;
    return llme_attention_check(&m.shape, LLME_ATTN_AUTOMATIC);
}

// Everything but the weights: caches, RoPE tables, feed, logits, the stream.
int common_setup(llme_model& m) {
    const llme_model_config& c = m.cfg;
    int st = cu(cudaStreamCreateWithFlags(&m.stream, cudaStreamNonBlocking), "model: stream");
    if (st) return st;
    st = cu(cudaMallocHost(&m.feed_host, (c.seq_len + 1) * sizeof(int)), "model: pinned feed");
    if (st) return st;
    std::memset(m.feed_host, 0, (c.seq_len + 1) * sizeof(int));
    st = dalloc(m, c.seq_len + 1, &m.feed);
    if (!st) st = dalloc(m, c.vocab_size, &m.logits);
    const size_t kvd = static_cast<size_t>(m.nkv) * m.hs;
    for (size_t l = 0; !st && l < m.layers.size(); ++l) {
        st = dalloc(m, c.seq_len * kvd, &m.layers[l].kc);
        if (!st) st = dalloc(m, c.seq_len * kvd, &m.layers[l].vc);
    }
    if (st) return st;
    std::vector<float> cs(static_cast<size_t>(c.seq_len) * m.hs / 2), sn(cs.size());
    llme::rope_tables(c.seq_len, m.hs, cs.data(), sn.data());
    st = upload(m, cs.data(), cs.size(), &m.cos);
    if (!st) st = upload(m, sn.data(), sn.size(), &m.sin);
    return st;
}

int reserve(llme_model& m, size_t n) {
    if (n <= m.rows) return LLME_OK;
    for (float* p : {m.x, m.qkv, m.att, m.gu, m.hb, m.scratch}) dfree(m, p);
    m.x = m.qkv = m.att = m.gu = m.hb = m.scratch = nullptr;
    m.rows = 0;
    const llme_model_config& c = m.cfg;
    int st = dalloc(m, n * c.dim, &m.x);
    if (!st) st = dalloc(m, n * m.qkv_cols, &m.qkv);
    if (!st) st = dalloc(m, n * m.nq * m.hs, &m.att);
    if (!st) st = dalloc(m, n * 2 * m.hc, &m.gu);
    if (!st) st = dalloc(m, n * m.hc, &m.hb);
    if (!st) st = dalloc(m, std::max<size_t>(1, llme_attention_scratch_floats(&m.shape, n, LLME_ATTN_AUTOMATIC)),
                         &m.scratch);
    if (st) return st;
    m.rows = n;
    ++m.own_generation;
    return LLME_OK;
}

size_t generation(const llme_model& m) { return m.own_generation + llme_scratch_generation(); }

int check_feed(const llme_model& m, const int* tokens, size_t n, size_t pos) {
    for (size_t i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= m.cfg.vocab_size)
            return set_error(LLME_E_RANGE, "forward: token " + std::to_string(tokens[i]) + " outside vocab");
    if (pos + n > static_cast<size_t>(m.cfg.seq_len) || pos > m.filled)
        return set_error(LLME_E_RANGE, "forward: positions " + std::to_string(pos) + ".." +
                                           std::to_string(pos + n - 1) + " with " +
                                           std::to_string(m.filled) + " cached of " +
                                           std::to_string(m.cfg.seq_len));
    return LLME_OK;
}

int product(llme_model& m, size_t rows, const Proj& w, const float* A, float* C, bool accumulate,
            const float* rms, cudaStream_t s) {
    return llme::run_product(rows, w.n, w.k, A, w.w, w.scale, C, m.q8, LLME_KERNEL_AUTOMATIC,
                             accumulate, rms, LLME_FLAG_WEIGHTS_STATIC, s);
}

// The product with its fused epilogue when the GEMV path takes it, else the plain product
// (the caller then runs the separate kernel). *fused tells which happened.
int product_fused(llme_model& m, size_t rows, const Proj& w, const float* A, float* C,
                  const float* rms, const llme::GemvEpilogue& epi, cudaStream_t s, bool* fused) {
    llme_plan_t p;
    int st = llme::plan_product(rows, w.n, w.k, m.q8, A, w.w, rms, &p);
    if (st) return st;
    *fused = p.path == LLME_PATH_GEMV_TMA && w.n % 2 == 0;
    if (!*fused) return product(m, rows, w, A, C, false, rms, s);
    return llme::run_product_epilogue(rows, w.n, w.k, A, w.w, w.scale, C, m.q8, rms,
                                      LLME_FLAG_WEIGHTS_STATIC, s, epi);
}

// A row-parallel product (wo, w2) whose sum over the ranks is taken inside the GEMV when every
// rank's shard has the same size (so every rank follows the same plan) and the communicator has
// its peer receive areas; *summed tells the caller to skip the separate all-reduce. Otherwise
// the plain product (rank 0 adds the residual), summed by the caller.
int rowpar_product(llme_model& m, size_t rows, const Proj& w, const float* A, float* C, bool lead,
                   bool equal_shards, cudaStream_t s, bool* summed) {
    *summed = false;
    llme::GemvEpilogue epi;
    if (m.world > 1 && m.comm && equal_shards && llme::comm_peer_sum(m.comm, &epi) == LLME_OK) {
        const int st = llme::run_product_epilogue(rows, w.n, w.k, A, w.w, w.scale, C, m.q8, nullptr,
                                                  LLME_FLAG_WEIGHTS_STATIC, s, epi, lead);
        if (st != LLME_E_UNSUPPORTED) {
            *summed = st == LLME_OK;
            return st;
        }
    }
    return product(m, rows, w, A, C, lead, nullptr, s);
}

int segments(const llme_model& m) { return 2 * m.cfg.n_layers + 1; }

// The buffer summed over the ranks after segment `seg`.
void reduction_buffer(const llme_model& m, int seg, size_t n, float** buf, size_t* count) {
    if (seg == segments(m) - 1) {
        *buf = m.logits;
        *count = m.cfg.vocab_size;
    } else {
        *buf = m.x;
        *count = n * m.cfg.dim;
    }
}

int run_segment(llme_model& m, int seg, size_t n, cudaStream_t s, bool* summed) {
    const int D = m.cfg.dim;
    *summed = false;
    const bool lead = m.rank == 0;  // adds the residual before the sum
    if (seg == segments(m) - 1) {
        int st = cu(cudaMemsetAsync(m.logits, 0, m.cfg.vocab_size * sizeof(float), s), "model: logits");
        if (st) return st;
        return product(m, 1, m.wcls, m.x + (n - 1) * D, m.logits + m.v0, false, m.rms_final, s);
    }
    Layer& L = m.layers[seg / 2];
    int st = LLME_OK;
    bool fused = false;
    if (seg % 2 == 0) {
        if (seg == 0) st = cu(llme::launch_embed_rows(static_cast<int>(n), D, m.feed, m.emb, m.x, s), "model: embed");
        llme::GemvEpilogue rope;
        rope.kind = llme::kEpiRopeCache;
        rope.nq = m.nq;
        rope.nkv = m.nkv;
        rope.head_size = m.hs;
        rope.feed = m.feed;
        rope.cos = m.cos;
        rope.sin = m.sin;
        rope.key_cache = L.kc;
        rope.value_cache = L.vc;
        if (!st) st = product_fused(m, n, L.wqkv, m.x, m.qkv, L.rms_att, rope, s, &fused);
        if (!st && !fused)
            st = cu(llme::launch_rope_cache(static_cast<int>(n), m.nq, m.nkv, m.hs, m.feed, m.cos, m.sin,
                                            m.qkv, L.kc, L.vc, s),
                    "model: rope");
        if (!st)
            st = llme_attention(&m.shape, n, m.feed, m.qkv, L.kc, L.vc, m.att, m.scratch,
                                LLME_ATTN_AUTOMATIC, s);
        // Heads split evenly over the ranks, so wo's shards are always the same size.
        if (!st) st = rowpar_product(m, n, L.wo, m.att, m.x, lead, true, s, summed);
        return st;
    }
    llme::GemvEpilogue swiglu;
    swiglu.kind = llme::kEpiSwiglu;
    swiglu.out = m.hb;
    st = product_fused(m, n, L.w13, m.x, m.gu, L.rms_ffn, swiglu, s, &fused);
    if (!st && !fused)
        st = cu(llme::launch_swiglu(static_cast<int>(n), static_cast<int>(m.hc), m.gu, m.hb, s), "model: swiglu");
    if (!st)
        st = rowpar_product(m, n, L.w2, m.hb, m.x, lead, m.cfg.hidden_dim % m.world == 0, s, summed);
    return st;
}

// Feed upload, every segment and (with a communicator) every all-reduce, on stream s.
int enqueue_step(llme_model& m, size_t n, cudaStream_t s) {
    int st = cu(cudaMemcpyAsync(m.feed, m.feed_host, (n + 1) * sizeof(int), cudaMemcpyHostToDevice, s),
                "model: feed");
    for (int seg = 0; !st && seg < segments(m); ++seg) {
        bool summed = false;
        st = run_segment(m, seg, n, s, &summed);
        if (!st && m.world > 1 && !summed) {
            float* buf;
            size_t count;
            reduction_buffer(m, seg, n, &buf, &count);
            st = llme_allreduce_sum_f32(buf, count, m.comm, s);
        }
    }
    return st;
}

void set_feed(llme_model& m, const int* tokens, size_t n, size_t pos) {
    m.feed_host[0] = static_cast<int>(pos);
    for (size_t i = 0; i < n; ++i) m.feed_host[1 + i] = tokens[i];
}

int finish(llme_model& m, float* logits) {
    int st = LLME_OK;
    if (logits)
        st = cu(cudaMemcpyAsync(logits, m.logits, m.cfg.vocab_size * sizeof(float), cudaMemcpyDeviceToHost,
                                m.stream),
                "model: logits");
    int st2 = cu(cudaStreamSynchronize(m.stream), "model: step");
    if (!st) st = st2;
    if (!st) st = llme_device_status();
    return st;
}

int forward(llme_model& m, const int* tokens, size_t n, size_t pos, float* logits) {
    if (n == 0) return set_error(LLME_E_INVALID, "prefill: no tokens");
    if (!tokens) return set_error(LLME_E_INVALID, "forward: null tokens");
    if (m.world > 1 && !m.comm)
        return set_error(LLME_E_INVALID, "tensor parallel: a rank without a communicator runs only "
                                         "through llme_model_group_forward");
    int st = check_feed(m, tokens, n, pos);
    if (st) return st;
    st = reserve(m, n);
    if (st) return st;
    // The stream is idle here (every call ends synchronised), so the pinned feed is free.
    set_feed(m, tokens, n, pos);
    st = enqueue_step(m, n, m.stream);
    if (!st) st = finish(m, logits);
    if (!st) m.filled = pos + n;
    return st;
}

int capture(llme_model& m) {
    if (m.graph) {
        cudaGraphExecDestroy(m.graph);
        m.graph = nullptr;
    }
    int st = cu(cudaStreamBeginCapture(m.stream, cudaStreamCaptureModeThreadLocal), "model: capture");
    if (st) return st;
    st = enqueue_step(m, 1, m.stream);
    cudaGraph_t g = nullptr;
    const int end = cu(cudaStreamEndCapture(m.stream, &g), "model: capture");
    if (!st) st = end;
    if (!st) st = cu(cudaGraphInstantiate(&m.graph, g, 0), "model: instantiate");
    if (g) cudaGraphDestroy(g);
    if (st) return st;
    m.graph_generation = generation(m);
    ++m.captures;
    return LLME_OK;
}

int decode(llme_model& m, int token, size_t pos, float* logits) {
    if (m.world > 1 && !m.comm)
        return set_error(LLME_E_INVALID, "tensor parallel: graphs need a communicator");
    int st = check_feed(m, &token, 1, pos);
    if (st) return st;
    if (!m.graph || m.graph_generation != generation(m)) {
        // Eager first (grows every buffer and the library's scratch), then capture.
        st = forward(m, &token, 1, pos, logits);
        return st ? st : capture(m);
    }
    set_feed(m, &token, 1, pos);
    st = cu(cudaGraphLaunch(m.graph, m.stream), "model: replay");
    if (!st) st = finish(m, logits);
    if (!st) m.filled = pos + 1;
    return st;
}

// The group forward: the ranks' segments on one stream, a rank-order sum after each.
int group_forward(llme_model* const* r, int world, const int* tokens, size_t n, size_t pos, float* logits) {
    if (world < 2 || world > 8) return set_error(LLME_E_INVALID, "group forward: 2 to 8 ranks");
    for (int i = 0; i < world; ++i) {
        if (!r[i]) return set_error(LLME_E_INVALID, "group forward: null rank");
        if (r[i]->world != world || r[i]->rank != i || r[i]->comm ||
            std::memcmp(&r[i]->cfg, &r[0]->cfg, sizeof(llme_model_config)) != 0 || r[i]->q8 != r[0]->q8)
            return set_error(LLME_E_INVALID, "group forward: ranks must be 0..world-1 of one model, "
                                             "without communicators");
    }
    if (n == 0) return set_error(LLME_E_INVALID, "prefill: no tokens");
    if (!tokens) return set_error(LLME_E_INVALID, "forward: null tokens");
    llme_model& m0 = *r[0];
    int st = check_feed(m0, tokens, n, pos);
    for (int i = 0; !st && i < world; ++i) {
        st = reserve(*r[i], n);
        if (!st) set_feed(*r[i], tokens, n, pos);
    }
    if (!st && !m0.group_bufs) st = dalloc(m0, 16, &m0.group_bufs);
    if (st) return st;
    cudaStream_t s = m0.stream;
    float* host_tab[16] = {};
    for (int i = 0; i < world; ++i) {
        host_tab[i] = r[i]->x;
        host_tab[8 + i] = r[i]->logits;
    }
    st = cu(cudaMemcpy(m0.group_bufs, host_tab, sizeof(host_tab), cudaMemcpyHostToDevice), "group: table");
    for (int i = 0; !st && i < world; ++i)
        st = cu(cudaMemcpyAsync(r[i]->feed, r[i]->feed_host, (n + 1) * sizeof(int), cudaMemcpyHostToDevice, s),
                "group: feed");
    for (int seg = 0; !st && seg < segments(m0); ++seg) {
        bool summed = false;  // group ranks have no communicator: always summed here
        for (int i = 0; !st && i < world; ++i) st = run_segment(*r[i], seg, n, s, &summed);
        if (st) break;
        const bool last = seg == segments(m0) - 1;
        st = cu(llme::launch_rank_sum(m0.group_bufs + (last ? 8 : 0), world,
                                      last ? static_cast<size_t>(m0.cfg.vocab_size) : n * m0.cfg.dim, s),
                "group: sum");
    }
    if (!st && logits)
        st = cu(cudaMemcpyAsync(logits, m0.logits, m0.cfg.vocab_size * sizeof(float), cudaMemcpyDeviceToHost, s),
                "group: logits");
    const int st2 = cu(cudaStreamSynchronize(s), "group: step");
    if (!st) st = st2;
    if (!st) st = llme_device_status();
    if (!st)
        for (int i = 0; i < world; ++i) r[i]->filled = pos + n;
    return st;
}

void destroy(llme_model* m) {
    if (!m) return;
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->graph) cudaGraphExecDestroy(m->graph);
    for (void* p : m->allocs) cudaFree(p);
    if (m->feed_host) cudaFreeHost(m->feed_host);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

// ---- checkpoints (llama2.c layout, as the reference reads them) -----------------------------

struct Checkpoint {
    llme_model_config cfg{};
    bool shared = false;
    std::vector<float> data;  // every float after the header
};

// The reference's header rules (src/model.cpp:62-75) and size rule (:77-86), with its texts.
int read_header(const char* path, Checkpoint* ck, FILE** fp_out, uint64_t* file_size) {
    const std::string p = path ? path : "";
    FILE* fp = path ? std::fopen(path, "rb") : nullptr;
    if (!fp) return set_error(LLME_E_INVALID, "cannot open checkpoint " + p);
    std::fseek(fp, 0, SEEK_END);
    const uint64_t size = static_cast<uint64_t>(std::ftell(fp));
    std::fseek(fp, 0, SEEK_SET);
    int32_t h[7];
    if (size < sizeof(h) || std::fread(h, sizeof(int32_t), 7, fp) != 7) {
        std::fclose(fp);
        return set_error(LLME_E_INVALID, "checkpoint " + p + " ended early");
    }
    ck->shared = h[5] > 0;
    for (int i = 0; i < 7; ++i) {
        if (h[i] == 0 || (i != 5 && h[i] < 0)) {
            std::fclose(fp);
            return set_error(LLME_E_INVALID, "checkpoint " + p + ": bad header field " + std::to_string(i) +
                                                 " = " + std::to_string(h[i]));
        }
    }
    auto u = [](int32_t v) { return static_cast<int>(v < 0 ? -static_cast<int64_t>(v) : v); };
    llme_model_config& c = ck->cfg;
    c.dim = u(h[0]);
    c.hidden_dim = u(h[1]);
    c.n_layers = u(h[2]);
    c.n_heads = u(h[3]);
    c.n_kv_heads = u(h[4]);
    c.vocab_size = u(h[5]);
    c.seq_len = u(h[6]);
    if (c.dim % c.n_heads != 0 || (c.dim / c.n_heads) % 2 != 0 || c.n_heads % c.n_kv_heads != 0) {
        std::fclose(fp);
        return set_error(LLME_E_INVALID, "checkpoint " + p + ": dim must split into even-sized heads, "
                                                             "and query heads into whole groups per kv head");
    }
    const uint64_t D = c.dim, H = c.hidden_dim, hs = D / c.n_heads, KV = c.n_kv_heads * hs,
                   V = c.vocab_size;
    const uint64_t per_layer = 2 * D + 2 * D * D + 2 * D * KV + 3 * D * H;
    uint64_t floats = V * D + c.n_layers * per_layer + D + static_cast<uint64_t>(c.seq_len) * hs;
    if (!ck->shared) floats += V * D;
    const uint64_t want = 7 * sizeof(int32_t) + floats * sizeof(float);
    if (size != want) {
        std::fclose(fp);
        return set_error(LLME_E_INVALID, "checkpoint " + p + " is " + std::to_string(size) +
                                             " bytes, header implies " + std::to_string(want));
    }
    *fp_out = fp;
    *file_size = size;
    return LLME_OK;
}

int read_checkpoint(const char* path, Checkpoint* ck) {
    FILE* fp = nullptr;
    uint64_t size = 0;
    int st = read_header(path, ck, &fp, &size);
    if (st) return st;
    ck->data.resize((size - 28) / 4);
    const size_t got = std::fread(ck->data.data(), sizeof(float), ck->data.size(), fp);
    std::fclose(fp);
    if (got != ck->data.size())
        return set_error(LLME_E_INVALID, "checkpoint " + std::string(path) + " ended early");
    return LLME_OK;
}

// Columns `outs` of a weight stored (out x in) in the file, as a k = in by n = outs.size()
// matrix (in x out, the layout the products take).
std::vector<float> gather(const float* w, size_t in, const std::vector<size_t>& outs) {
    std::vector<float> r(in * outs.size());
    for (size_t j = 0; j < outs.size(); ++j) {
        const float* src = w + outs[j] * in;
        for (size_t i = 0; i < in; ++i) r[i * outs.size() + j] = src[i];
    }
    return r;
}

std::vector<size_t> range_of(size_t start, size_t count) {
    std::vector<size_t> v(count);
    for (size_t i = 0; i < count; ++i) v[i] = start + i;
    return v;
}

int host_proj(llme_model& m, const std::vector<float>& host, size_t k, size_t n, const size_t* rows, Proj* out) {
    float* dev = nullptr;
    int st = upload(m, host.data(), k * n, &dev);
    return st ? st : finish_proj(m, dev, k, n, rows, out);
}

int load_weights(llme_model& m, const Checkpoint& ck) {
    const llme_model_config& c = m.cfg;
    const size_t D = c.dim, H = c.hidden_dim, KV = static_cast<size_t>(c.n_kv_heads) * m.hs, V = c.vocab_size,
                 NL = c.n_layers, hs = m.hs;
    const float* f = ck.data.data();
    const float* emb = f;
    const float* rms_att = emb + V * D;
    const float* wq = rms_att + NL * D;
    const float* wk = wq + NL * D * D;
    const float* wv = wk + NL * KV * D;
    const float* wo = wv + NL * KV * D;
    const float* rms_ffn = wo + NL * D * D;
    const float* w1 = rms_ffn + NL * D;
    const float* w2 = w1 + NL * H * D;
    const float* w3 = w2 + NL * D * H;
    const float* rms_final = w3 + NL * H * D;
    const float* wcls = ck.shared ? emb : rms_final + D + static_cast<size_t>(c.seq_len) * hs;

    int st = upload(m, emb, V * D, &m.emb);
    if (!st) st = upload(m, rms_final, D, &m.rms_final);
    if (!st) st = host_proj(m, gather(wcls, D, range_of(m.v0, m.vc)), D, m.vc, nullptr, &m.wcls);
    const auto q_outs = range_of(m.q0 * hs, m.nq * hs), kv_outs = range_of(m.kv0 * hs, m.nkv * hs);
    const auto all_d = range_of(0, D);
    for (size_t l = 0; !st && l < NL; ++l) {
        Layer& L = m.layers[l];
        st = upload(m, rms_att + l * D, D, &L.rms_att);
        if (!st) st = upload(m, rms_ffn + l * D, D, &L.rms_ffn);
        if (st) break;
        // wqkv: this rank's q heads, then its k heads, then its v heads.
        const auto q = gather(wq + l * D * D, D, q_outs);
        const auto k = gather(wk + l * KV * D, D, kv_outs);
        const auto v = gather(wv + l * KV * D, D, kv_outs);
        std::vector<float> qkv(D * m.qkv_cols);
        const size_t nqc = q_outs.size(), nkc = kv_outs.size();
        for (size_t i = 0; i < D; ++i) {
            std::copy(&q[i * nqc], &q[i * nqc] + nqc, &qkv[i * m.qkv_cols]);
            std::copy(&k[i * nkc], &k[i * nkc] + nkc, &qkv[i * m.qkv_cols + nqc]);
            std::copy(&v[i * nkc], &v[i * nkc] + nkc, &qkv[i * m.qkv_cols + nqc + nkc]);
        }
        st = host_proj(m, qkv, D, m.qkv_cols, nullptr, &L.wqkv);
        // wo: every row (quantised over all of them), this rank's head rows kept.
        const size_t wo_rows[2] = {static_cast<size_t>(m.q0) * hs, static_cast<size_t>(m.nq) * hs};
        if (!st) st = host_proj(m, gather(wo + l * D * D, D, all_d), D, D, wo_rows, &L.wo);
        // w13: gate and up of each of this rank's hidden units in adjacent columns.
        if (!st) {
            const auto hid = range_of(m.h0, m.hc);
            const auto g = gather(w1 + l * H * D, D, hid), u = gather(w3 + l * H * D, D, hid);
            std::vector<float> w13(D * 2 * m.hc);
            for (size_t i = 0; i < D; ++i)
                for (size_t j = 0; j < m.hc; ++j) {
                    w13[i * 2 * m.hc + 2 * j] = g[i * m.hc + j];
                    w13[i * 2 * m.hc + 2 * j + 1] = u[i * m.hc + j];
                }
            st = host_proj(m, w13, D, 2 * m.hc, nullptr, &L.w13);
        }
        const size_t w2_rows[2] = {m.h0, m.hc};
        if (!st) st = host_proj(m, gather(w2 + l * D * H, H, all_d), H, D, w2_rows, &L.w2);
    }
    return st;
}

int synthetic_weights(llme_model& m, uint64_t seed) {
    const llme_model_config& c = m.cfg;
    const size_t D = c.dim, hs = m.hs;
    uint64_t tensor = 0;
    auto fresh = [&](size_t k, size_t n, Proj* out) {
        float* dev = nullptr;
        int st = dalloc(m, k * n, &dev, false);
        if (!st) st = cu(llme::launch_fill_normal(dev, k * n, seed * 1000003ull + 7919ull * ++tensor + m.rank, 0.02f,
                                                  m.stream),
                         "model: draw");
        if (!st) st = cu(cudaStreamSynchronize(m.stream), "model: draw");
        return st ? st : finish_proj(m, dev, k, n, nullptr, out);
    };
    auto ones = [&](size_t count, float** out) {
        std::vector<float> h(count, 1.0f);
        return upload(m, h.data(), count, out);
    };
    int st = dalloc(m, static_cast<size_t>(c.vocab_size) * D, &m.emb, false);
    if (!st) st = cu(llme::launch_fill_uniform(m.emb, static_cast<size_t>(c.vocab_size) * D, seed * 31 + 17, -1.0f,
                                               1.0f, m.stream),
                     "model: draw");
    if (!st) st = ones(D, &m.rms_final);
    if (!st) st = fresh(D, m.vc, &m.wcls);
    for (size_t l = 0; !st && l < m.layers.size(); ++l) {
        Layer& L = m.layers[l];
        st = ones(D, &L.rms_att);
        if (!st) st = ones(D, &L.rms_ffn);
        if (!st) st = fresh(D, m.qkv_cols, &L.wqkv);
        if (!st) st = fresh(static_cast<size_t>(m.nq) * hs, D, &L.wo);
        if (!st) st = fresh(D, 2 * m.hc, &L.w13);
        if (!st) st = fresh(m.hc, D, &L.w2);
    }
    if (!st) st = cu(cudaStreamSynchronize(m.stream), "model: draw");
    return st;
}

int create(const llme_model_config& cfg, bool q8, int world, int rank, llme_comm_t* comm, llme_model_t** out) {
    if (!out) return set_error(LLME_E_INVALID, "model: null output");
    *out = nullptr;
    if (world > 8 && comm == nullptr) return set_error(LLME_E_INVALID, "model: at most 8 emulated ranks");
    llme_model* m = new llme_model;
    m->cfg = cfg;
    m->q8 = q8;
    m->world = world;
    m->rank = rank;
    m->comm = comm;
    int st = partition(*m);
    if (!st) {
        m->layers.resize(cfg.n_layers);
        st = common_setup(*m);
    }
    if (st) {
        destroy(m);
        return st;
    }
    *out = m;
    return LLME_OK;
}

}  // namespace

extern "C" {

int llme_model_load(const char* path, int q8, int world, int rank, llme_comm_t* comm, llme_model_t** model) {
    return llme::guarded([&]() -> int {
        Checkpoint ck;
        int st = read_checkpoint(path, &ck);
        if (st) return st;
        st = create(ck.cfg, q8 != 0, world, rank, comm, model);
        if (st) return st;
        st = load_weights(**model, ck);
        if (st) {
            destroy(*model);
            *model = nullptr;
        }
        return st;
    });
}

int llme_model_synthetic(const llme_model_config* cfg, int q8, int world, int rank, llme_comm_t* comm,
                         unsigned long long seed, llme_model_t** model) {
    return llme::guarded([&]() -> int {
        if (!cfg) return set_error(LLME_E_INVALID, "model: null configuration");
        int st = create(*cfg, q8 != 0, world, rank, comm, model);
        if (st) return st;
        st = synthetic_weights(**model, seed);
        if (st) {
            destroy(*model);
            *model = nullptr;
        }
        return st;
    });
}

int llme_checkpoint_config(const char* path, llme_model_config* cfg) {
    return llme::guarded([&]() -> int {
        Checkpoint ck;
        FILE* fp = nullptr;
        uint64_t size = 0;
        int st = read_header(path, &ck, &fp, &size);
        if (st) return st;
        std::fclose(fp);
        if (cfg) *cfg = ck.cfg;
        return LLME_OK;
    });
}

int llme_model_partition(const llme_model_config* cfg, int world, int rank, llme_model_slice* out) {
    return llme::guarded([&]() -> int {
        if (!cfg || !out) return set_error(LLME_E_INVALID, "model: null argument");
        return slice_of(*cfg, world, rank, out);
    });
}

int llme_model_get_config(const llme_model_t* m, llme_model_config* cfg) {
    return llme::guarded([&]() -> int {
        if (!m || !cfg) return set_error(LLME_E_INVALID, "model: null argument");
        *cfg = m->cfg;
        return LLME_OK;
    });
}

int llme_model_local(const llme_model_t* m, int* q_heads, int* kv_heads, int* hidden, int* vocab) {
    return llme::guarded([&]() -> int {
        if (!m) return set_error(LLME_E_INVALID, "model: null model");
        if (q_heads) *q_heads = m->nq;
        if (kv_heads) *kv_heads = m->nkv;
        if (hidden) *hidden = static_cast<int>(m->hc);
        if (vocab) *vocab = static_cast<int>(m->vc);
        return LLME_OK;
    });
}

int llme_model_stream_bytes(const llme_model_t* m, size_t* weight_bytes, size_t* kv_bytes_per_position) {
    return llme::guarded([&]() -> int {
        if (!m) return set_error(LLME_E_INVALID, "model: null model");
        auto bytes = [&](const Proj& p) { return m->q8 ? p.k * p.n + 4 * p.n : 4 * p.k * p.n; };
        size_t w = bytes(m->wcls);
        for (const Layer& L : m->layers) w += bytes(L.wqkv) + bytes(L.wo) + bytes(L.w13) + bytes(L.w2);
        if (weight_bytes) *weight_bytes = w;
        if (kv_bytes_per_position)
            *kv_bytes_per_position = 2 * m->layers.size() * static_cast<size_t>(m->nkv) * m->hs * sizeof(float);
        return LLME_OK;
    });
}

int llme_model_forward(llme_model_t* m, const int* tokens, size_t n, size_t pos, float* logits) {
    return llme::guarded([&]() -> int {
        if (!m) return set_error(LLME_E_INVALID, "model: null model");
        return forward(*m, tokens, n, pos, logits);
    });
}

int llme_model_decode(llme_model_t* m, int token, size_t pos, float* logits) {
    return llme::guarded([&]() -> int {
        if (!m) return set_error(LLME_E_INVALID, "model: null model");
        return decode(*m, token, pos, logits);
    });
}

size_t llme_model_captures(const llme_model_t* m) { return m ? m->captures : 0; }

int llme_model_fill_history(llme_model_t* m, size_t positions, unsigned long long seed) {
    return llme::guarded([&]() -> int {
        if (!m) return set_error(LLME_E_INVALID, "model: null model");
        if (positions > static_cast<size_t>(m->cfg.seq_len))
            return set_error(LLME_E_RANGE, "fill_history: more positions than seq_len");
        const size_t kvd = static_cast<size_t>(m->nkv) * m->hs;
        int st = LLME_OK;
        for (size_t l = 0; !st && l < m->layers.size() && positions; ++l) {
            st = cu(llme::launch_fill_uniform(m->layers[l].kc, positions * kvd, seed * 977 + 2 * l, -1.0f, 1.0f,
                                              m->stream),
                    "model: history");
            if (!st)
                st = cu(llme::launch_fill_uniform(m->layers[l].vc, positions * kvd, seed * 977 + 2 * l + 1, -1.0f,
                                                  1.0f, m->stream),
                        "model: history");
        }
        if (!st) st = cu(cudaStreamSynchronize(m->stream), "model: history");
        if (!st) m->filled = positions;
        return st;
    });
}

int llme_model_replay(llme_model_t* m, size_t times, void* stream) {
    return llme::guarded([&]() -> int {
        if (!m) return set_error(LLME_E_INVALID, "model: null model");
        if (!m->graph || m->graph_generation != generation(*m))
            return set_error(LLME_E_INVALID, "model: no current decode graph (run llme_model_decode first)");
        cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : cudaStreamPerThread;
        for (size_t i = 0; i < times; ++i) {
            int st = cu(cudaGraphLaunch(m->graph, s), "model: replay");
            if (st) return st;
        }
        return LLME_OK;
    });
}

int llme_model_group_forward(llme_model_t* const* ranks, int world, const int* tokens, size_t n, size_t pos,
                             float* logits) {
    return llme::guarded([&]() -> int {
        if (!ranks) return set_error(LLME_E_INVALID, "group forward: null ranks");
        return group_forward(ranks, world, tokens, n, pos, logits);
    });
}

int llme_model_destroy(llme_model_t* m) {
    return llme::guarded([&]() -> int {
        destroy(m);
        return LLME_OK;
    });
}

}  // extern "C"
