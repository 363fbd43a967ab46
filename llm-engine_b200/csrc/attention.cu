// Causal decode attention over a KV cache (the interface of the reference's
// src/cuda_attention.h; its kernels are src/cuda_attention.cu:37-257).
//
// split (flash-decoding; the decode path, few rows): one CTA per (group of G query heads
// sharing a kv head, row, chunk of positions). Each CTA brings its whole K chunk and V chunk
// into shared memory at once -- 2D TMA boxes of 16 positions x head_size floats over the
// caches (per-position bulk copies for heads wider than 256), completing two mbarriers -- so
// all of the chunk's bytes are in flight from the start; while they land it stages the
// queries. Scores: a group of lanes per position (head_size / 4 lanes, one float4 each, at
// most 32), the G queries' float4s held in registers, the dot products finished by shuffles.
// The chunk's softmax is kept unnormalised (max m, sum l of exp(score - m)) and the
// exp-weighted sum of values o is formed with one thread per (head, float4 of the head) and
// position slots. A context that fits one chunk is normalised and written directly;
// otherwise each CTA writes (o, m, l) to scratch and leaves. The merge is a second launch
// (programmatic dependent launch: it becomes resident while the chunks run and waits for
// them), parallel over (head, row, 32 of the head's dimensions): M = max m_c, the chunk
// weights w_c = exp(m_c - M) and L = sum w_c l_c, then O = sum w_c o_c in chunk order
// (deterministic), out = O / L; no CTA of the split launch waits on a ticket or merges a
// group of chunks alone. Chunks are sized for
// about three CTAs per SM (a tensor-parallel rank's 16 or 8 heads get shorter chunks in one
// wave); the grid is sized for seq_len and the context length is
// read from device memory, so a graph captured once serves every position; chunks past the
// context exit at once.
//
// single_block (many rows): one CTA per (query head, row), the whole context's scores in
// shared memory: a warp per position for the dot products (coalesced key reads), block
// reductions for the softmax, threads over the head's dimensions and position slots for the
// weighted sum.
//
// Every mbarrier wait is bounded (common.cuh).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace llme {
namespace {

__device__ unsigned int g_attn_error;

constexpr int kAttnThreads = 256;
constexpr int kMinChunk = 64;               // positions per split CTA, at least
constexpr int kTargetCtas = 444;            // split CTAs a single row aims for (3 per SM)
// A split CTA's shared memory, at most: three CTAs per SM, so some load while others compute
// (measured on B200: 7B MHA decode 41 us against 47 us with two larger CTAs per SM).
constexpr size_t kSplitSmemBudget = 72 * 1024;
constexpr size_t kSingleSmemMax = 48 * 1024;     // the interface's documented cap
constexpr std::size_t kSplitMaxRows = 8;         // automatic: split up to this many rows
constexpr int kAttnSmemAttr = 200 * 1024;        // dynamic shared memory the kernels may ask for

constexpr int kBoxRows = 16;                // positions per TMA box of keys / values

// Positions per chunk: a multiple of the box height, so only a context's last chunk reads a
// partial box.
__host__ __device__ inline int chunk_size(int n_ctx, int splits) {
    int c = (n_ctx + splits - 1) / splits;
    c = c > kMinChunk ? c : kMinChunk;
    return (c + kBoxRows - 1) / kBoxRows * kBoxRows;
}

constexpr int kMergeDims4 = 8;    // float4s of a head's dimensions per merge CTA (32 floats)
constexpr int kMergeSlots = kAttnThreads / kMergeDims4;  // chunk slots per float4

// out[i][h][d] = sum_c w_c o_c[d] / L over the chunks c < n of (head h, row i): one CTA per
// (head, row, kMergeDims4 float4s of the head). Launched after the split kernel with
// programmatic dependent launch; the partials are read through L2 (__ldcg) after the wait.
__global__ void __launch_bounds__(kAttnThreads) attn_merge_kernel(AttnArgs a, int splits) {
    extern __shared__ __align__(16) float wts[];  // splits weights, then kAttnThreads float4s
    __shared__ float red_s[kAttnThreads / 32];
    const int h = blockIdx.x, i = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hs4 = a.head_size / 4;
    if (tid == 0) pdl_launch_dependents();
    pdl_wait();  // the chunks' partials come from the split launch
    const int n_ctx = *a.pos + i + 1;
    const int chunk = chunk_size(n_ctx, splits);
    const int n = (n_ctx + chunk - 1) / chunk;
    if (n == 1) return;  // the split kernel normalised and wrote this row itself
    const size_t rb = static_cast<size_t>(i) * a.scratch_row;
    const float2* ml = a.part_ml + rb / 2 + static_cast<size_t>(h) * splits;
    // M = max m_c, then w_c = exp(m_c - M) and L = sum w_c l_c (block reductions, fixed order).
    float m = -INFINITY;
    for (int c = tid; c < n; c += kAttnThreads) m = fmaxf(m, __ldcg(&ml[c]).x);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red_s[warp] = m;
    __syncthreads();
    m = red_s[0];
    for (int w = 1; w < kAttnThreads / 32; ++w) m = fmaxf(m, red_s[w]);
    float l = 0.0f;
    for (int c = tid; c < n; c += kAttnThreads) {
        const float2 p = __ldcg(&ml[c]);
        const float w = expf(p.x - m);
        wts[c] = w;
        l += w * p.y;
    }
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    __syncthreads();  // every thread has read red_s's maxima before it is rewritten
    if (lane == 0) red_s[warp] = l;
    __syncthreads();
    l = red_s[0];
    for (int w = 1; w < kAttnThreads / 32; ++w) l += red_s[w];
    // O for float4 d4 of this CTA's slice: slot r takes chunks r, r + kMergeSlots, ...
    const int d4 = blockIdx.z * kMergeDims4 + tid % kMergeDims4, r = tid / kMergeDims4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (d4 < hs4) {
        const float4* po = reinterpret_cast<const float4*>(a.part_o + rb) +
                           static_cast<size_t>(h) * splits * hs4 + d4;
        int c = r;
        for (; c + 3 * kMergeSlots < n; c += 4 * kMergeSlots) {
            float4 o[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) o[u] = __ldcg(po + static_cast<size_t>(c + u * kMergeSlots) * hs4);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float w = wts[c + u * kMergeSlots];
                acc.x += w * o[u].x;
                acc.y += w * o[u].y;
                acc.z += w * o[u].z;
                acc.w += w * o[u].w;
            }
        }
        for (; c < n; c += kMergeSlots) {
            const float4 o = __ldcg(po + static_cast<size_t>(c) * hs4);
            const float w = wts[c];
            acc.x += w * o.x;
            acc.y += w * o.y;
            acc.z += w * o.z;
            acc.w += w * o.w;
        }
    }
    float4* slot_sum = reinterpret_cast<float4*>(wts + (splits + 3) / 4 * 4);
    slot_sum[tid] = acc;
    __syncthreads();
    if (r == 0 && d4 < hs4) {
        float4 o = slot_sum[tid];
        for (int q = 1; q < kMergeSlots; ++q) {  // slots in order
            const float4 x = slot_sum[q * kMergeDims4 + tid];
            o.x += x.x;
            o.y += x.y;
            o.z += x.z;
            o.w += x.w;
        }
        const float inv = 1.0f / l;
        reinterpret_cast<float4*>(a.out + static_cast<size_t>(i) * a.out_stride +
                                  static_cast<size_t>(h) * a.head_size)[d4] =
            make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
    }
}

// The G queries of one lane: float4 number sub + j * lpp of each head, j < QV.
template <int G, int QV>
__global__ void __launch_bounds__(kAttnThreads)
    attn_split_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                      AttnArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    // TMA destinations start on 128-byte boundaries (the launch adds 128 bytes of slack).
    float* smem = reinterpret_cast<float*>(smem_raw + ((128 - (smem_u32(smem_raw) & 127)) & 127));
    const int hs = a.head_size, hs4 = hs / 4;
    const int cap = a.chunk_cap;
    float* sK = smem;                              // cap x hs
    float* sV = sK + static_cast<size_t>(cap) * hs;  // cap x hs
    float* sQ = sV + static_cast<size_t>(cap) * hs;  // G x hs
    float* sc = sQ + G * hs;                       // G x cap4 scores
    const int cap4 = (cap + 3) / 4 * 4;
    float4* red = reinterpret_cast<float4*>(sc + G * cap4);  // slots x G x hs4
    __shared__ uint64_t bar[2];
    __shared__ float2 ml[G];

    const int hg = blockIdx.x, i = blockIdx.y, s = blockIdx.z, splits = gridDim.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // The next launch (a product staging its static weights) may become resident once every
    // CTA of this grid has started; it reads this kernel's output only after its own
    // griddepcontrol.wait, which waits for this whole grid to finish.
    if (tid == 0) pdl_launch_dependents();
    pdl_wait();  // q, the caches and the position come from earlier launches
    const int n_ctx = *a.pos + i + 1;
    const int chunk = chunk_size(n_ctx, splits);
    const int n = (n_ctx + chunk - 1) / chunk;  // chunks with work
    const int t0 = s * chunk;
    if (t0 >= n_ctx) return;  // uniform across the CTA
    const int len = min(chunk, n_ctx - t0);
    const int h0 = hg * G, kv_off = (h0 / a.group) * hs;

    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (a.boxes) {
        // Boxes of kBoxRows positions x head_size floats; the last box of a context's final
        // chunk may cover positions past it (zero fill past the cache) that are never used.
        if (tid == 0) {
            const int nbox = (len + kBoxRows - 1) / kBoxRows;
            const uint32_t box = static_cast<uint32_t>(kBoxRows * hs) * 4;
            mbar_arrive_expect_tx(&bar[0], box * nbox);
            mbar_arrive_expect_tx(&bar[1], box * nbox);
            for (int b = 0; b < nbox; ++b)
                tma_load_2d_nohint(sK + static_cast<size_t>(b) * kBoxRows * hs, &tmK, kv_off,
                                   t0 + b * kBoxRows, &bar[0]);
            for (int b = 0; b < nbox; ++b)
                tma_load_2d_nohint(sV + static_cast<size_t>(b) * kBoxRows * hs, &tmV, kv_off,
                                   t0 + b * kBoxRows, &bar[1]);
        }
    } else if (warp == 0) {
        const uint32_t bytes = static_cast<uint32_t>(hs) * 4;
        if (lane == 0) {
            mbar_arrive_expect_tx(&bar[0], bytes * len);
            mbar_arrive_expect_tx(&bar[1], bytes * len);
        }
        __syncwarp();
        const float* kb = a.k + static_cast<size_t>(t0) * a.kv_stride + kv_off;
        const float* vb = a.v + static_cast<size_t>(t0) * a.kv_stride + kv_off;
        for (int t = lane; t < len; t += 32)
            bulk_load_g2s(sK + static_cast<size_t>(t) * hs, kb + static_cast<size_t>(t) * a.kv_stride,
                          bytes, &bar[0]);
        for (int t = lane; t < len; t += 32)
            bulk_load_g2s(sV + static_cast<size_t>(t) * hs, vb + static_cast<size_t>(t) * a.kv_stride,
                          bytes, &bar[1]);
    }
    // The G heads are contiguous in q.
    const float4* qg = reinterpret_cast<const float4*>(a.q + static_cast<size_t>(i) * a.q_stride +
                                                       static_cast<size_t>(h0) * hs);
    for (int j = tid; j < G * hs4; j += kAttnThreads) reinterpret_cast<float4*>(sQ)[j] = qg[j];
    __syncthreads();

    // Scores: lpp lanes per position; each lane keeps its float4s of the G queries.
    int lpp = 1;
    while (lpp < hs4 && lpp < 32) lpp *= 2;
    const int sub = lane % lpp, per_warp = 32 / lpp;
    float4 qr[G][QV];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int j = 0; j < QV; ++j) {
            const int d = sub + j * lpp;
            qr[g][j] = d < hs4 ? reinterpret_cast<const float4*>(sQ)[g * hs4 + d]
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    const bool landed_k = mbar_wait(&bar[0], 0, &g_attn_error);
    const float scale = 1.0f / sqrtf(static_cast<float>(hs));
    // Every lane runs the same trip count so the shuffles see whole warps.
    for (int base = warp * per_warp; base < len; base += (kAttnThreads / 32) * per_warp) {
        const int t = base + lane / lpp;
        float dot[G];
#pragma unroll
        for (int g = 0; g < G; ++g) dot[g] = 0.0f;
        if (t < len && landed_k) {
            const float4* kr = reinterpret_cast<const float4*>(sK + static_cast<size_t>(t) * hs);
#pragma unroll
            for (int j = 0; j < QV; ++j) {
                const int d = sub + j * lpp;
                if (d < hs4) {
                    const float4 kv = kr[d];
#pragma unroll
                    for (int g = 0; g < G; ++g)
                        dot[g] += qr[g][j].x * kv.x + qr[g][j].y * kv.y + qr[g][j].z * kv.z +
                                  qr[g][j].w * kv.w;
                }
            }
        }
        for (int o = lpp / 2; o > 0; o >>= 1)
#pragma unroll
            for (int g = 0; g < G; ++g) dot[g] += __shfl_xor_sync(0xffffffffu, dot[g], o);
        if (t < len && sub == 0)
#pragma unroll
            for (int g = 0; g < G; ++g) sc[g * cap4 + t] = dot[g] * scale;
    }
    __syncthreads();

    // The chunk's softmax, one warp per head, unnormalised.
    for (int g = warp; g < G; g += kAttnThreads / 32) {
        float* p = sc + g * cap4;
        float m = -INFINITY;
        for (int t = lane; t < len; t += 32) m = fmaxf(m, p[t]);
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.0f;
        for (int t = lane; t < len; t += 32) {
            p[t] = expf(p[t] - m);
            l += p[t];
        }
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) ml[g] = make_float2(m, l);
    }
    const bool landed_v = mbar_wait(&bar[1], 0, &g_attn_error);
    __syncthreads();

    // o[g][d4] = sum over t of p[g][t] v[t][d4]; slots of positions, then a fixed-order sum.
    const int pairs = G * hs4;
    const int slots = max(1, kAttnThreads / pairs);
    for (int base = 0; base < pairs; base += kAttnThreads) {
        const int j = base + tid % (slots > 1 ? pairs : kAttnThreads);
        const int r = slots > 1 ? tid / pairs : 0;
        if (j < pairs && r < slots) {
            const int g = j / hs4, d4 = j % hs4;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            if (landed_v) {
                for (int t = r; t < len; t += slots) {
                    const float p = sc[g * cap4 + t];
                    const float4 v = reinterpret_cast<const float4*>(sV + static_cast<size_t>(t) * hs)[d4];
                    acc.x += p * v.x;
                    acc.y += p * v.y;
                    acc.z += p * v.z;
                    acc.w += p * v.w;
                }
            }
            red[r * pairs + j] = acc;
        }
    }
    __syncthreads();

    // This row's block of the scratch: [chunk partials o | chunk (m, l)], at a stride that
    // depends on the shape only; the merge launch reads them.
    const size_t rb = static_cast<size_t>(i) * a.scratch_row;
    float* part_o = a.part_o + rb;
    float2* part_ml = a.part_ml + rb / 2;
    for (int j = tid; j < pairs; j += kAttnThreads) {
        const int g = j / hs4, d4 = j % hs4;
        float4 o = red[j];
        for (int r = 1; r < slots; ++r) {
            const float4 x = red[r * pairs + j];
            o.x += x.x;
            o.y += x.y;
            o.z += x.z;
            o.w += x.w;
        }
        if (n == 1) {
            const float inv = 1.0f / ml[g].y;
            reinterpret_cast<float4*>(a.out + static_cast<size_t>(i) * a.out_stride +
                                      static_cast<size_t>(h0 + g) * hs)[d4] =
                make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
        } else {
            reinterpret_cast<float4*>(part_o)[(static_cast<size_t>(h0 + g) * splits + s) * hs4 + d4] = o;
        }
    }
    if (n > 1 && tid < G) part_ml[static_cast<size_t>(h0 + tid) * splits + s] = ml[tid];
}

__device__ __forceinline__ float block_max(float v, float* red) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = red[0];
    for (int w = 1; w < kAttnThreads / 32; ++w) r = fmaxf(r, red[w]);
    __syncthreads();
    return r;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = red[0];
    for (int w = 1; w < kAttnThreads / 32; ++w) r += red[w];
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(kAttnThreads) attn_single_kernel(AttnArgs a) {
    extern __shared__ __align__(16) float smem[];
    float* q = smem;
    float* scores = smem + a.head_size;
    __shared__ float red[kAttnThreads / 32];
    const int hs = a.head_size;
    const int h = blockIdx.x, i = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) pdl_launch_dependents();  // as in the split kernel
    pdl_wait();
    const int n_ctx = *a.pos + i + 1;
    const int kv_off = (h / a.group) * hs;
    const float* qg = a.q + static_cast<size_t>(i) * a.q_stride + static_cast<size_t>(h) * hs;
    for (int d = tid; d < hs; d += kAttnThreads) q[d] = qg[d];
    __syncthreads();

    const float scale = 1.0f / sqrtf(static_cast<float>(hs));
    float mx = -INFINITY;
    for (int t = warp; t < n_ctx; t += kAttnThreads / 32) {
        const float* k = a.k + static_cast<size_t>(t) * a.kv_stride + kv_off;
        float dot = 0.0f;
        for (int d = lane; d < hs; d += 32) dot += q[d] * __ldg(k + d);
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        if (lane == 0) scores[t] = dot * scale;
        mx = fmaxf(mx, dot * scale);
    }
    mx = block_max(mx, red);  // its barriers also publish the scores
    float sum = 0.0f;
    for (int t = tid; t < n_ctx; t += kAttnThreads) {
        scores[t] = expf(scores[t] - mx);
        sum += scores[t];
    }
    const float inv = 1.0f / block_sum(sum, red);

    // out[d] = sum over t of p[t] v[t][d]: threads over d (coalesced value rows); when the head
    // is narrower than the CTA, `slots` groups of hs threads take every slots-th position and
    // their sums are added in slot order.
    float* out = a.out + static_cast<size_t>(i) * a.out_stride + static_cast<size_t>(h) * hs;
    const int slots = max(1, kAttnThreads / hs);
    if (slots > 1) {
        float* part = scores + ((n_ctx + 3) / 4) * 4;  // after the scores (slots x hs floats)
        const int r = tid / hs, d = tid % hs;
        if (r < slots) {
            const float* v = a.v + kv_off + d;
            float acc = 0.0f;
            for (int t = r; t < n_ctx; t += slots)
                acc += scores[t] * __ldg(v + static_cast<size_t>(t) * a.kv_stride);
            part[r * hs + d] = acc;
        }
        __syncthreads();
        for (int dd = tid; dd < hs; dd += kAttnThreads) {
            float acc = part[dd];
            for (int rr = 1; rr < slots; ++rr) acc += part[rr * hs + dd];
            out[dd] = acc * inv;
        }
    } else {
        for (int d = tid; d < hs; d += kAttnThreads) {
            const float* v = a.v + kv_off + d;
            float acc = 0.0f;
            for (int t = 0; t < n_ctx; ++t)
                acc += scores[t] * __ldg(v + static_cast<size_t>(t) * a.kv_stride);
            out[d] = acc * inv;
        }
    }
}

// ---- host side ------------------------------------------------------------------------------

int heads_per_block(const llme_attention_shape& s) {
    const int group = s.n_heads / s.n_kv_heads;
    for (int g : {8, 4, 2})
        if (group % g == 0) return g;
    return 1;
}

// Splits (grid z) and the largest chunk a CTA can get, sized so one CTA's K + V chunk fits
// the shared-memory budget.
struct SplitGeo {
    int splits, cap;
    size_t smem;
};

// K and V chunks, the queries, the scores and the slot sums.
size_t split_smem_bytes(const llme_attention_shape& s, int cap) {
    const size_t G = heads_per_block(s), hs = s.head_size, hs4 = hs / 4;
    const size_t cap4 = (static_cast<size_t>(cap) + 3) / 4 * 4;
    const size_t pairs = G * hs4;
    const size_t slots = std::max<size_t>(1, kAttnThreads / pairs);
    return (2 * static_cast<size_t>(cap) * hs + G * hs + G * cap4) * sizeof(float) +
           slots * pairs * 16 + 128;  // + alignment slack
}

// The merge launch: the chunk weights, then one float4 per thread.
size_t merge_smem_bytes(int splits) {
    return (static_cast<size_t>(splits) + 3) / 4 * 4 * sizeof(float) + kAttnThreads * 16;
}

// Splits: enough for one row to give about kTargetCtas CTAs, no chunk below kMinChunk
// positions, and more whenever a chunk's keys and values would not fit the shared-memory
// budget. Independent of the number of rows, so the scratch grows in proportion to rows.
SplitGeo split_geo(const llme_attention_shape& s) {
    const int groups = s.n_heads / heads_per_block(s);
    const int most = std::max(1, (s.seq_len + kMinChunk - 1) / kMinChunk);
    int splits = std::min(most, std::max(1, (kTargetCtas + groups - 1) / groups));
    int cap = chunk_size(s.seq_len, splits);
    while (split_smem_bytes(s, cap) > kSplitSmemBudget && cap > kMinChunk) {
        ++splits;
        cap = chunk_size(s.seq_len, splits);
    }
    return {splits, cap, split_smem_bytes(s, cap)};
}

size_t single_smem_bytes(const llme_attention_shape& s) {
    const size_t hs = s.head_size, slots = std::max<size_t>(1, kAttnThreads / hs);
    const size_t base = (hs + static_cast<size_t>(s.seq_len)) * sizeof(float);
    // the position slots' partial sums reuse the space after the scores
    return base + (slots > 1 ? (slots * hs + 4) * sizeof(float) : 0);
}

// The interface's shared-memory rule for single_block: head_size + seq_len floats.
bool single_fits(const llme_attention_shape& s) {
    return (static_cast<size_t>(s.head_size) + static_cast<size_t>(s.seq_len)) * sizeof(float) <=
           kSingleSmemMax;
}

int resolve(const llme_attention_shape& s, int kernel, size_t rows) {
    if (kernel != LLME_ATTN_AUTOMATIC) return kernel;
    return rows <= kSplitMaxRows || !single_fits(s) ? LLME_ATTN_SPLIT : LLME_ATTN_SINGLE_BLOCK;
}

// Scratch (floats): one block per row, at a stride that depends on the shape only --
// [chunk partials o | chunk (m, l)], each part 16-byte aligned. Offsets are within a row's
// block; a call with fewer rows uses a prefix of the blocks. Every partial is written before
// the merge reads it, so the scratch needs no initial contents.
struct ScratchLayout {
    size_t o, ml, row;
};

ScratchLayout scratch_layout(const llme_attention_shape& s) {
    const SplitGeo g = split_geo(s);
    const size_t chunks = static_cast<size_t>(s.n_heads) * static_cast<size_t>(g.splits);
    auto up4 = [](size_t x) { return (x + 3) / 4 * 4; };
    ScratchLayout l{};
    l.o = 0;
    l.ml = l.o + up4(chunks * static_cast<size_t>(s.head_size));
    l.row = l.ml + up4(2 * chunks);
    return l;
}

int check(const llme_attention_shape& s, int kernel) {
    if (kernel < LLME_ATTN_AUTOMATIC || kernel > LLME_ATTN_SPLIT)
        return set_error(LLME_E_INVALID, "attention: unknown kernel " + std::to_string(kernel));
    if (s.n_heads <= 0 || s.n_kv_heads <= 0 || s.head_size <= 0 || s.seq_len <= 0 ||
        s.n_heads % s.n_kv_heads != 0)
        return set_error(LLME_E_INVALID, "attention: bad shape");
    if (static_cast<size_t>(s.seq_len) * s.kv_stride >= (size_t{1} << 31) ||
        s.q_stride >= (size_t{1} << 31) || s.out_stride >= (size_t{1} << 31))
        return set_error(LLME_E_INVALID, "attention: cache past 32-bit indexing");
    const bool single = kernel == LLME_ATTN_SINGLE_BLOCK;
    if (!single && (s.head_size % 4 || s.head_size > 512 || s.q_stride % 4 ||
                    s.kv_stride % 4 || s.out_stride % 4))
        return set_error(LLME_E_INVALID,
                         "attention: split needs head_size and strides divisible by 4");
    if (single && !single_fits(s))
        return set_error(LLME_E_INVALID,
                         "attention: seq_len " + std::to_string(s.seq_len) + " needs " +
                             std::to_string((s.head_size + static_cast<size_t>(s.seq_len)) * 4) +
                             " bytes of shared memory, more than " + std::to_string(kSingleSmemMax));
    return LLME_OK;
}

template <int G, int QV>
cudaError_t launch_split(const CUtensorMap& tmK, const CUtensorMap& tmV, const AttnArgs& a,
                         dim3 grid, size_t smem, cudaStream_t stream) {
    static unsigned configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 32 && !(configured & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(attn_split_kernel<G, QV>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kAttnSmemAttr);
        if (e != cudaSuccess) return e;
        configured |= 1u << dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, attn_split_kernel<G, QV>, tmK, tmV, a);
}

// The merge of the chunks' partials: one CTA per (head, row, 32 dimensions of the head).
cudaError_t launch_merge(const AttnArgs& a, size_t rows, int splits, cudaStream_t stream) {
    const size_t smem = merge_smem_bytes(splits);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(attn_merge_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kAttnSmemAttr);
        if (e != cudaSuccess) return e;
    }
    const int hs4 = a.head_size / 4;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(a.n_heads), static_cast<unsigned>(rows),
                       static_cast<unsigned>((hs4 + kMergeDims4 - 1) / kMergeDims4));
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, attn_merge_kernel, a, splits);
}

template <int G>
cudaError_t launch_split_g(const CUtensorMap& tmK, const CUtensorMap& tmV, const AttnArgs& a,
                           dim3 grid, size_t smem, cudaStream_t stream) {
    const int hs4 = a.head_size / 4;
    int lpp = 1;
    while (lpp < hs4 && lpp < 32) lpp *= 2;
    const int qv = (hs4 + lpp - 1) / lpp;
    if (qv <= 1) return launch_split<G, 1>(tmK, tmV, a, grid, smem, stream);
    if (qv <= 2) return launch_split<G, 2>(tmK, tmV, a, grid, smem, stream);
    return launch_split<G, 4>(tmK, tmV, a, grid, smem, stream);  // head_size <= 512
}

}  // namespace

unsigned read_and_clear_attn_error() {
    unsigned v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_attn_error, sizeof(v)) != cudaSuccess) return 0;
    if (v) cudaMemcpyToSymbol(g_attn_error, &zero, sizeof(zero));
    return v;
}

}  // namespace llme

using namespace llme;

extern "C" {

int llme_attention_check(const llme_attention_shape* s, int kernel) {
    return llme::guarded([&]() -> int {
        if (!s) return set_error(LLME_E_INVALID, "attention: null shape");
        return check(*s, kernel);
    });
}

size_t llme_attention_scratch_floats(const llme_attention_shape* s, size_t rows, int kernel) {
    if (!s || kernel == LLME_ATTN_SINGLE_BLOCK) return 0;
    if (s->n_heads <= 0 || s->n_kv_heads <= 0 || s->head_size <= 0 || s->seq_len <= 0 ||
        s->n_heads % s->n_kv_heads != 0)
        return 0;
    // The most rows a call of up to `rows` rows splits.
    if (kernel == LLME_ATTN_AUTOMATIC && single_fits(*s)) rows = std::min(rows, kSplitMaxRows);
    return scratch_layout(*s).row * rows;
}

size_t llme_attention_launches(const llme_attention_shape* s, size_t rows, int kernel) {
    try {
        if (!s || rows == 0 || check(*s, kernel) != LLME_OK) return 0;
        kernel = resolve(*s, kernel, rows);
        if (check(*s, kernel) != LLME_OK) return 0;
        if (kernel == LLME_ATTN_SINGLE_BLOCK) return 1;
        return split_geo(*s).splits > 1 ? 2 : 1;
    } catch (...) {
        return 0;
    }
}

int llme_attention(const llme_attention_shape* s, size_t rows, const int* pos_dev, const float* q,
                   const float* key_cache, const float* value_cache, float* out, float* scratch,
                   int kernel, void* stream_ptr) {
    return llme::guarded([&]() -> int {
        if (!s) return set_error(LLME_E_INVALID, "attention: null shape");
        int st = check(*s, kernel);
        if (st) return st;
        if (rows == 0) return LLME_OK;
        if (!pos_dev || !q || !key_cache || !value_cache || !out)
            return set_error(LLME_E_INVALID, "attention: null pointer");
        kernel = resolve(*s, kernel, rows);
        st = check(*s, kernel);
        if (st) return st;
        if (rows > 65535) return set_error(LLME_E_INVALID, "attention: more than 65535 rows");
        cudaStream_t stream = stream_ptr ? static_cast<cudaStream_t>(stream_ptr) : cudaStreamPerThread;
        AttnArgs a;
        a.n_heads = s->n_heads;
        a.head_size = s->head_size;
        a.group = s->n_heads / s->n_kv_heads;
        a.q_stride = s->q_stride;
        a.kv_stride = s->kv_stride;
        a.out_stride = s->out_stride;
        a.pos = pos_dev;
        a.q = q;
        a.k = key_cache;
        a.v = value_cache;
        a.out = out;
        cudaError_t e;
        if (kernel == LLME_ATTN_SINGLE_BLOCK) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(static_cast<unsigned>(s->n_heads), static_cast<unsigned>(rows));
            cfg.blockDim = dim3(kAttnThreads);
            cfg.dynamicSmemBytes = single_smem_bytes(*s);
            cfg.stream = stream;
            if (cfg.dynamicSmemBytes > 48 * 1024) {
                e = cudaFuncSetAttribute(attn_single_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kAttnSmemAttr);
                if (e != cudaSuccess) return set_cuda_error(e, "attention");
            }
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            e = cudaLaunchKernelEx(&cfg, attn_single_kernel, a);
        } else {
            // The caches are read by bulk copies: their rows must start on 16-byte boundaries.
            if ((reinterpret_cast<uintptr_t>(key_cache) | reinterpret_cast<uintptr_t>(value_cache) |
                 reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) % 16)
                return set_error(LLME_E_INVALID, "attention: split needs 16-byte aligned q, caches and out");
            if (!scratch) return set_error(LLME_E_INVALID, "attention: split needs scratch");
            const SplitGeo g = split_geo(*s);
            const ScratchLayout l = scratch_layout(*s);
            a.chunk_cap = g.cap;
            a.part_o = scratch + l.o;
            a.part_ml = reinterpret_cast<float2*>(scratch + l.ml);
            a.scratch_row = l.row;
            const int G = heads_per_block(*s);
            const dim3 grid(static_cast<unsigned>(s->n_heads / G), static_cast<unsigned>(rows),
                            static_cast<unsigned>(g.splits));
            // Keys and values by TMA boxes over the whole cache (kv_stride floats a row); a head
            // wider than one box (256 elements) takes the per-position copies.
            CUtensorMap tmK, tmV;
            std::memset(&tmK, 0, sizeof(tmK));
            std::memset(&tmV, 0, sizeof(tmV));
            a.boxes = s->head_size <= 256;
            if (a.boxes) {
                st = tensor_map_2d(key_cache, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, s->seq_len,
                                   s->kv_stride, s->kv_stride * 4, s->head_size, kBoxRows, &tmK);
                if (!st)
                    st = tensor_map_2d(value_cache, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, s->seq_len,
                                       s->kv_stride, s->kv_stride * 4, s->head_size, kBoxRows, &tmV);
                if (st) return st;
            }
            switch (G) {
                case 8: e = launch_split_g<8>(tmK, tmV, a, grid, g.smem, stream); break;
                case 4: e = launch_split_g<4>(tmK, tmV, a, grid, g.smem, stream); break;
                case 2: e = launch_split_g<2>(tmK, tmV, a, grid, g.smem, stream); break;
                default: e = launch_split_g<1>(tmK, tmV, a, grid, g.smem, stream); break;
            }
            if (e == cudaSuccess && g.splits > 1) e = launch_merge(a, rows, g.splits, stream);
        }
        return e == cudaSuccess ? LLME_OK : set_cuda_error(e, "attention");
    });
}

}  // extern "C"
