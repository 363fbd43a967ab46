// Prefill-shaped products (m >= 128) on the 5th-generation tensor cores:
// C (+)= A x B with fp32 A and B multiplied in TF32 (kind::tf32), fp32
// accumulation in TMEM.
//
// The reference runs these shapes on its SIMT sgemm_tiled<128,8>
// (src/cuda_matmul.cu:71-125). Here one CTA per SM computes a 128 x 256 tile:
//   warp 0      one thread issues TMA loads into a 4-stage ring guarded by
//               mbarriers: A K-major (128-byte swizzle); B either straight
//               from the caller's k x n weights as the MN-major operand --
//               eight 32-column boxes per stage in the 128-byte swizzle with
//               32-byte atoms, the layout tcgen05 takes for 32-bit MN-major
//               operands -- or, for m large enough to repay a transpose pass
//               (the MN-major MMAs run ~9% slower), from B^T written by that
//               pass, K-major like A;
//   warp 1      allocates 256 TMEM columns; one thread issues
//               tcgen05.mma.kind::tf32 (M=128, N=256, K=8) four times per
//               32-deep stage and releases each stage with tcgen05.commit;
//   warps 2-5   wait for the final commit, read the accumulator with
//               tcgen05.ld (each warp its 32-lane TMEM quadrant) and write C,
//               adding to it for MatmulFusion::accumulate.
// Tiles are rasterised in groups of 8 along m so concurrently running CTAs
// share B panels in L2. Every mbarrier wait is bounded (common.cuh).
#include "kernels.h"
#include "tc_common.cuh"

namespace llme {
namespace {

__device__ unsigned int g_tc_error;

constexpr int TBM = 128, TBN = 256, TBK = 32;  // 32 fp32 = 128 bytes along K
constexpr int kStages = 4;
constexpr int kThreads = 192;
constexpr int kABytes = TBM * TBK * 4;        // 16 KB
constexpr int kBBytes = TBK * TBN * 4;        // 32 KB: B^T box of 256 rows (n) x 32 (k), or
constexpr int kBBoxBytes = TBK * 32 * 4;      // 8 MN-major boxes of 32 rows (k) x 32 columns
constexpr int kRingBytes = kStages * (kABytes + kBBytes);
constexpr int kSmemBytes = kRingBytes + 256 + 1024;  // barriers + alignment slack
constexpr int kGroupM = 8;
constexpr uint32_t kTmemCols = 256;

template <bool BMn>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tf32_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const TcArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 128B-swizzled TMA destinations and descriptors assume 1024-byte aligned atoms.
    uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint8_t* sA = smem;
    uint8_t* sB = smem + kStages * kABytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kRingBytes);
    uint64_t* empty = full + kStages;
    uint64_t* done = empty + kStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Grouped rasterisation: kGroupM row-tiles share each column panel.
    const int tile = blockIdx.x;
    const int group_size = kGroupM * a.tiles_n;
    const int first_m = (tile / group_size) * kGroupM;
    const int gm = min(a.tiles_m - first_m, kGroupM);
    const int tm = first_m + (tile % group_size) % gm;
    const int tn = (tile % group_size) / gm;
    const int m0 = tm * TBM, n0 = tn * TBN;
    const int nk = (a.k + TBK - 1) / TBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    if (threadIdx.x == 0) pdl_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            pdl_wait();
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % kStages;
                if (kb >= kStages && !mbar_wait(&empty[s], ((kb / kStages) - 1) & 1, &g_tc_error))
                    break;
                mbar_arrive_expect_tx(&full[s], kABytes + kBBytes);
                tma_load_2d_nohint(sA + s * kABytes, &tmA, kb * TBK, m0, &full[s]);
                if (BMn) {
#pragma unroll
                    for (int j = 0; j < TBN / 32; ++j)
                        tma_load_2d_nohint(sB + s * kBBytes + j * kBBoxBytes, &tmB, n0 + j * 32,
                                           kb * TBK, &full[s]);
                } else {
                    tma_load_2d_nohint(sB + s * kBBytes, &tmB, kb * TBK, n0, &full[s]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = tc::instr_desc(tc::kFmtTF32, tc::kFmtTF32, false, BMn, TBM, TBN);
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % kStages;
                if (!mbar_wait(&full[s], (kb / kStages) & 1, &g_tc_error)) break;
                tc::fence_after_sync();
                const uint32_t abase = smem_u32(sA + s * kABytes);
                const uint32_t bbase = smem_u32(sB + s * kBBytes);
#pragma unroll
                for (int kk = 0; kk < TBK / 8; ++kk) {
                    // K-major rows of 128 B (8-row groups 1 KB apart), the 8-deep K step
                    // 32 B into each row; MN-major B: the K step is 8 rows = 1 KB.
                    const uint64_t ad = tc::smem_desc_sw128(abase + kk * 32, 16, 1024);
                    const uint64_t bd = BMn ? tc::smem_desc_sw128_32b(bbase + kk * 1024, kBBoxBytes)
                                            : tc::smem_desc_sw128(bbase + kk * 32, 16, 1024);
                    tc::mma_tf32(tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
                }
                tc::commit(&empty[s]);
            }
            tc::commit(done);
        }
    } else {
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        const int row = m0 + q * 32 + lane;
        pdl_wait();
        const bool ok = mbar_wait(done, 0, &g_tc_error);
        tc::fence_after_sync();
        if (ok) {
            const bool vec = (a.n & 3) == 0;
#pragma unroll 1
            for (int c = 0; c < TBN / 32; ++c) {
                __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp, converged
                uint32_t r[32];
                tc::tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(q * 32) << 16) + c * 32, r);
                const int col0 = n0 + c * 32;
                if (row >= a.m || col0 >= a.n) continue;
                float* out = a.C + static_cast<size_t>(row) * a.n + col0;
                if (vec && col0 + 32 <= a.n) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        float4 v = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                               __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
                        if (a.accumulate) {
                            const float4 o = *reinterpret_cast<const float4*>(out + j);
                            v.x += o.x;
                            v.y += o.y;
                            v.z += o.z;
                            v.w += o.w;
                        }
                        *reinterpret_cast<float4*>(out + j) = v;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        if (col0 + j < a.n) {
                            const float v = __uint_as_float(r[j]);
                            out[j] = a.accumulate ? out[j] + v : v;
                        }
                    }
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
}

// out (n x k) = B^T for B k x n, fp32, through 32 x 32 shared-memory tiles so both the
// reads and the writes are coalesced.
__global__ void __launch_bounds__(256) transpose_kernel(const float* __restrict__ B,
                                                         float* __restrict__ out, int k, int n) {
    __shared__ float tile[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
    for (int i = ty; i < 32; i += 8) {
        const int r = r0 + i, c = c0 + tx;
        if (r < k && c < n) tile[i][tx] = B[static_cast<size_t>(r) * n + c];
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
        const int c = c0 + i, r = r0 + tx;  // out row c (a column of B), column r
        if (c < n && r < k) out[static_cast<size_t>(c) * k + r] = tile[tx][i];
    }
}

template <bool BMn>
cudaError_t launch_t(const TcArgs& a, const CUtensorMap& tmA, const CUtensorMap& tmB) {
    static unsigned configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 32 && !(configured & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(gemm_tf32_kernel<BMn>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        if (e != cudaSuccess) return e;
        configured |= 1u << dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.tiles_m * a.tiles_n);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = a.stream;
    cudaLaunchAttribute attr[1];
    if (a.pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, gemm_tf32_kernel<BMn>, tmA, tmB, a);
}

}  // namespace

cudaError_t launch_transpose(const float* B, float* out, int k, int n, cudaStream_t stream) {
    const dim3 grid((n + 31) / 32, (k + 31) / 32);
    transpose_kernel<<<grid, 256, 0, stream>>>(B, out, k, n);
    return cudaGetLastError();
}

int tc_tile_m() { return TBM; }
int tc_tile_n() { return TBN; }

cudaError_t launch_gemm_tf32(const TcArgs& a, const CUtensorMap& tmA, const CUtensorMap& tmB) {
    return a.b_transposed ? launch_t<false>(a, tmA, tmB) : launch_t<true>(a, tmA, tmB);
}

unsigned read_and_clear_tc_error() {
    unsigned v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(v)) != cudaSuccess) return 0;
    if (v) cudaMemcpyToSymbol(g_tc_error, &zero, sizeof(zero));
    return v;
}

}  // namespace llme
