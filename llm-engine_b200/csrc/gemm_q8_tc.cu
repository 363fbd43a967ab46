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
// Layout in shared memory, per pipeline stage (128 k per stage):
//   hi tile: 128 rows x 128 bytes, K-major, 128-byte swizzle (TMA box 128 x 128)
//   lo tile: the same for the lo rows
//   B tile:  TBN/128 boxes of 128 k-rows x 128 columns, MN-major (W as stored,
//            k x n with n contiguous), 128-byte swizzle; the MMA descriptor
//            steps 1 KB per 8 k-rows (SBO) and one box (16 KB) per 128 columns
//            (LBO).
// Warp roles (192 threads, one CTA per SM, persistent over output tiles):
//   warp 0     TMA producer (one thread) over a ring of kStages stages;
//   warp 1     TMEM allocation (all 512 columns) and MMA issue (one thread):
//              per stage and 32-deep K step, one MMA into the Hi accumulator
//              and one into the Lo accumulator; tcgen05.commit frees the stage;
//   warps 2-5  epilogue: tcgen05.ld of Hi and Lo (each warp its TMEM lane
//              quadrant), scale, optional residual add, fp32 stores.
// With TBN = 128 the CTA holds two accumulator pairs, so the epilogue of one
// tile overlaps the MMAs of the next; with TBN = 256 one pair fills TMEM.
// Every mbarrier wait is bounded (common.cuh): a wait that runs out sets the
// file's error word and the kernel winds down instead of hanging.
#include "kernels.h"
#include "tc_common.cuh"

namespace llme {
namespace {

__device__ unsigned int g_q8tc_error;

constexpr int TBM = 128;       // rows of C per tile (TMEM lanes)
constexpr int TBK = 128;       // k per stage: 128 int8 = one 128-byte swizzle row
constexpr int kThreads = 192;
constexpr int kRingBudget = 196608;  // bytes of shared memory for the stage ring
constexpr int kGroupM = 8;           // row tiles that share each column panel (L2 reuse)

template <int TBN>
struct Cfg {
    static constexpr int kABytes = TBM * TBK;           // one of hi / lo: 16 KB
    static constexpr int kBBytes = TBK * TBN;           // 16 or 32 KB
    static constexpr int kStageBytes = 2 * kABytes + kBBytes;
    static constexpr int kStages = kRingBudget / kStageBytes;  // 4 or 3
    static constexpr int kAccCols = 2 * TBN;            // Hi + Lo
    static constexpr int kAccBufs = 512 / kAccCols;     // 2 or 1
    static constexpr int kSmemBytes = kStages * kStageBytes + 256 + 1024;
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
// A K-major, B MN-major.
constexpr uint32_t idesc_i8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | (1u << 16) |
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

// Tile t -> (row tile, column tile), kGroupM row tiles per column panel.
__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int* tm, int* tn) {
    const int group = kGroupM * tiles_n;
    const int first_m = (t / group) * kGroupM;
    const int gm = min(tiles_m - first_m, kGroupM);
    *tm = first_m + (t % group) % gm;
    *tn = (t % group) / gm;
}

template <int TBN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_q8_tc_kernel(const __grid_constant__ CUtensorMap tmHi,
                      const __grid_constant__ CUtensorMap tmLo,
                      const __grid_constant__ CUtensorMap tmB, const Q8TcArgs a) {
    using C = Cfg<TBN>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
    uint64_t* empty = full + C::kStages;
    uint64_t* acc_full = empty + C::kStages;
    uint64_t* acc_empty = acc_full + C::kAccBufs;
    uint64_t* drain = acc_empty + C::kAccBufs;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_m = (a.m + TBM - 1) / TBM;
    const int tiles_n = (a.n + TBN - 1) / TBN;
    const int tiles = tiles_m * tiles_n;
    const int nk = (a.k + TBK - 1) / TBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < C::kAccBufs; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
        }
        mbar_init(drain, 1);
        fence_mbar_init();
        prefetch_tensormap(&tmHi);
        prefetch_tensormap(&tmLo);
        prefetch_tensormap(&tmB);
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            pdl_wait();  // the split rows come from the kernel before this one
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                int tm, tn;
                tile_coords(t, tiles_m, tiles_n, &tm, &tn);
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % C::kStages;
                    if (it >= C::kStages &&
                        !mbar_wait(&empty[s], ((it / C::kStages) - 1) & 1, &g_q8tc_error)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = smem + s * C::kStageBytes;
                    mbar_arrive_expect_tx(&full[s], C::kStageBytes);
                    tma_load_2d_nohint(st, &tmHi, kb * TBK, tm * TBM, &full[s]);
                    tma_load_2d_nohint(st + C::kABytes, &tmLo, kb * TBK, tm * TBM, &full[s]);
#pragma unroll
                    for (int j = 0; j < TBN / 128; ++j)
                        tma_load_2d_nohint(st + 2 * C::kABytes + j * TBK * 128, &tmB,
                                           tn * TBN + j * 128, kb * TBK, &full[s]);
                }
            }
            // Before the CTA may exit, every copy issued into its shared memory has landed
            // (already true unless a wait above gave up).
            for (int j = it - 1; j >= 0 && j >= it - C::kStages; --j)
                mbar_wait(&full[j % C::kStages], (j / C::kStages) & 1, &g_q8tc_error);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(TBM, TBN);
            int it = 0, use = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++use) {
                const int buf = use % C::kAccBufs;
                const int round = use / C::kAccBufs;
                if (round > 0 && !mbar_wait(&acc_empty[buf], (round - 1) & 1, &g_q8tc_error)) break;
                tc::fence_after_sync();
                const uint32_t d_hi = tmem + buf * C::kAccCols;
                const uint32_t d_lo = d_hi + TBN;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % C::kStages;
                    if (!mbar_wait(&full[s], (it / C::kStages) & 1, &g_q8tc_error)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint32_t hi = smem_u32(smem + s * C::kStageBytes);
                    const uint32_t lo = hi + C::kABytes;
                    const uint32_t bb = lo + C::kABytes;
#pragma unroll
                    for (int kk = 0; kk < TBK / 32; ++kk) {
                        // A: K-major 128-byte rows, the 32-deep K step is 32 bytes into the row.
                        // B: MN-major, 32 k-rows of 128 bytes per K step; LBO = one box.
                        const uint64_t bd = tc::smem_desc_sw128(bb + kk * 32 * 128, TBK * 128, 1024);
                        const uint32_t acc = (kb | kk) != 0 ? 1u : 0u;
                        mma_i8(d_hi, tc::smem_desc_sw128(hi + kk * 32, 16, 1024), bd, idesc, acc);
                        mma_i8(d_lo, tc::smem_desc_sw128(lo + kk * 32, 16, 1024), bd, idesc, acc);
                    }
                    tc::commit(&empty[s]);
                }
                tc::commit(&acc_full[buf]);
            }
            // No MMA may still be writing TMEM when it is released.
            tc::commit(drain);
            mbar_wait(drain, 0, &g_q8tc_error);
        }
    } else {
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        pdl_wait();              // C may be read by the kernel before this one
        int use = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++use) {
            int tm, tn;
            tile_coords(t, tiles_m, tiles_n, &tm, &tn);
            const int buf = use % C::kAccBufs;
            const int round = use / C::kAccBufs;
            if (!mbar_wait(&acc_full[buf], round & 1, &g_q8tc_error)) break;
            tc::fence_after_sync();
            const int row = tm * TBM + q * 32 + lane;
            const bool row_ok = row < a.m;
            const float rs = row_ok ? a.row_scale[row] : 0.0f;
            float* out = a.C + static_cast<size_t>(row_ok ? row : 0) * a.n;
            const uint32_t base = tmem + (static_cast<uint32_t>(q * 32) << 16) + buf * C::kAccCols;
            const bool vec = ((reinterpret_cast<uintptr_t>(a.scale) |
                               reinterpret_cast<uintptr_t>(a.C)) & 15) == 0;
#pragma unroll 1
            for (int c = 0; c < TBN / 32; ++c) {
                __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp, converged
                uint32_t h[32], l[32];
                tc::tmem_ld_32x32b_x32(base + c * 32, h);
                tc::tmem_ld_32x32b_x32(base + TBN + c * 32, l);
                const int col0 = tn * TBN + c * 32;
                if (!row_ok || col0 >= a.n) continue;
                if (vec && col0 + 32 <= a.n) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        const float4 sc = *reinterpret_cast<const float4*>(a.scale + col0 + j);
                        float4* o = reinterpret_cast<float4*>(out + col0 + j);
                        float4 v = make_float4(finish(h[j], l[j], rs, sc.x), finish(h[j + 1], l[j + 1], rs, sc.y),
                                               finish(h[j + 2], l[j + 2], rs, sc.z), finish(h[j + 3], l[j + 3], rs, sc.w));
                        if (a.accumulate) {
                            const float4 p = *o;
                            v = make_float4(__fadd_rn(p.x, v.x), __fadd_rn(p.y, v.y),
                                            __fadd_rn(p.z, v.z), __fadd_rn(p.w, v.w));
                        }
                        *o = v;
                    }
                } else {
                    // n % 16 == 0: the last chunk of a row has 16 or 32 columns.
#pragma unroll
                    for (int j = 0; j < 32; j += 16) {
                        if (col0 + j >= a.n) continue;
#pragma unroll
                        for (int u = 0; u < 16; ++u) {
                            const float v = finish(h[j + u], l[j + u], rs, a.scale[col0 + j + u]);
                            out[col0 + j + u] = a.accumulate ? __fadd_rn(out[col0 + j + u], v) : v;
                        }
                    }
                }
            }
            // This warp's reads of the buffer are complete (tcgen05.ld waits inside the helper).
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, 512);
    }
}

// One CTA per row of A: the row (RMS-normalised when w is set: x = a * inv_rms * w) is split
// into hi / lo int8 rows of pitch kp and a row scale (see the file comment). Rows whose
// largest magnitude is not finite get a NaN row scale, so their outputs are NaN, as an fp32
// product with that row would be.
constexpr int kSplitThreads = 256;

__global__ void __launch_bounds__(kSplitThreads)
    split_rows_kernel(int k, int kp, const float* __restrict__ A, const float* __restrict__ w,
                      int8_t* __restrict__ hi, int8_t* __restrict__ lo,
                      float* __restrict__ row_scale) {
    __shared__ float red_ss[kSplitThreads / 32], red_mx[kSplitThreads / 32];
    pdl_launch_dependents();
    pdl_wait();
    const float* in = A + static_cast<size_t>(blockIdx.x) * k;
    int8_t* oh = hi + static_cast<size_t>(blockIdx.x) * kp;
    int8_t* ol = lo + static_cast<size_t>(blockIdx.x) * kp;
    const bool vec = (k & 3) == 0 && (reinterpret_cast<uintptr_t>(in) & 15) == 0 &&
                     (w == nullptr || (reinterpret_cast<uintptr_t>(w) & 15) == 0);
    // Pass 1: sum of squares (for the norm) and the largest |a * w| (or |a|).
    float ss = 0.0f, mx = 0.0f;
    if (vec) {
        for (int j = threadIdx.x * 4; j < k; j += kSplitThreads * 4) {
            const float4 v = *reinterpret_cast<const float4*>(in + j);
            float4 u = v;
            if (w) {
                const float4 g = *reinterpret_cast<const float4*>(w + j);
                ss = fmaf(v.x, v.x, ss);
                ss = fmaf(v.y, v.y, ss);
                ss = fmaf(v.z, v.z, ss);
                ss = fmaf(v.w, v.w, ss);
                u = make_float4(v.x * g.x, v.y * g.y, v.z * g.z, v.w * g.w);
            }
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(u.x), fabsf(u.y)), fmaxf(fabsf(u.z), fabsf(u.w))));
            // fmaxf drops NaN; keep it visible.
            if (u.x != u.x || u.y != u.y || u.z != u.z || u.w != u.w) mx = __int_as_float(0x7f800000);
        }
    } else {
        for (int j = threadIdx.x; j < k; j += kSplitThreads) {
            const float v = in[j];
            float u = v;
            if (w) {
                ss = fmaf(v, v, ss);
                u = v * w[j];
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
    const float inv_rms = w ? 1.0f / sqrtf(total / static_cast<float>(k) + kRmsEps) : 1.0f;
    amax *= inv_rms;
    // Multiplier to the hi grid (127 at the row's largest magnitude). Rows so small that
    // 127 / amax overflows are first brought up by 2^64 (exact).
    float pre = 1.0f;
    if (amax > 0.0f && amax < 1e-30f) pre = 18446744073709551616.0f;  // 2^64
    const float q = amax > 0.0f ? 127.0f / (amax * pre) : 0.0f;
    if (threadIdx.x == 0) {
        float s = amax / 127.0f;
        if (!(amax <= 3.402823466e38f)) s = __int_as_float(0x7fc00000);  // inf / NaN rows
        row_scale[blockIdx.x] = s;
    }
    auto split1 = [&](float a, float g, int8_t* h8, int8_t* l8) {
        float x = w ? a * inv_rms * g : a;
        float y = pre == 1.0f ? x * q : (x * pre) * q;
        if (!(fabsf(y) <= 128.0f)) y = 0.0f;  // non-finite rows: row scale is NaN
        float h = fminf(fmaxf(rintf(y), -127.0f), 127.0f);
        float r = (y - h) * 256.0f;
        float l = fminf(fmaxf(rintf(r), -127.0f), 127.0f);
        *h8 = static_cast<int8_t>(static_cast<int>(h));
        *l8 = static_cast<int8_t>(static_cast<int>(l));
    };
    if (vec) {
        for (int j = threadIdx.x * 4; j < k; j += kSplitThreads * 4) {
            const float4 v = *reinterpret_cast<const float4*>(in + j);
            float4 g = make_float4(1.f, 1.f, 1.f, 1.f);
            if (w) g = *reinterpret_cast<const float4*>(w + j);
            char4 h4, l4;
            split1(v.x, g.x, &h4.x, &l4.x);
            split1(v.y, g.y, &h4.y, &l4.y);
            split1(v.z, g.z, &h4.z, &l4.z);
            split1(v.w, g.w, &h4.w, &l4.w);
            *reinterpret_cast<char4*>(oh + j) = h4;
            *reinterpret_cast<char4*>(ol + j) = l4;
        }
    } else {
        for (int j = threadIdx.x; j < k; j += kSplitThreads) {
            int8_t h8, l8;
            split1(in[j], w ? w[j] : 1.0f, &h8, &l8);
            oh[j] = h8;
            ol[j] = l8;
        }
    }
}

template <int TBN>
cudaError_t launch_tbn(const Q8TcArgs& a, const CUtensorMap& tmHi, const CUtensorMap& tmLo,
                       const CUtensorMap& tmB) {
    static unsigned configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 32 && !(configured & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(gemm_q8_tc_kernel<TBN>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Cfg<TBN>::kSmemBytes);
        if (e != cudaSuccess) return e;
        configured |= 1u << dev;
    }
    const int tiles = ((a.m + TBM - 1) / TBM) * ((a.n + TBN - 1) / TBN);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::max(1, std::min(tiles, a.grid)));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = Cfg<TBN>::kSmemBytes;
    cfg.stream = a.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemm_q8_tc_kernel<TBN>, tmHi, tmLo, tmB, a);
}

}  // namespace

int q8tc_tile_m() { return TBM; }

cudaError_t launch_split_rows(int m, int k, int kp, const float* A, const float* w, int8_t* hi,
                              int8_t* lo, float* row_scale, cudaStream_t stream, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(m);
    cfg.blockDim = dim3(kSplitThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, split_rows_kernel, k, kp, A, w, hi, lo, row_scale);
}

cudaError_t launch_gemm_q8_tc(const Q8TcArgs& a, const CUtensorMap& tmHi, const CUtensorMap& tmLo,
                              const CUtensorMap& tmB) {
    if (a.tile_n == 256) return launch_tbn<256>(a, tmHi, tmLo, tmB);
    if (a.tile_n == 128) return launch_tbn<128>(a, tmHi, tmLo, tmB);
    return cudaErrorInvalidValue;
}

unsigned read_and_clear_q8tc_error() {
    unsigned v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_q8tc_error, sizeof(v)) != cudaSuccess) return 0;
    if (v) cudaMemcpyToSymbol(g_q8tc_error, &zero, sizeof(zero));
    return v;
}

}  // namespace llme
