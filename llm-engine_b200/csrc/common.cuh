// Device helpers shared by the sm_100a kernels: mbarrier waits with a time
// limit, TMA (cp.async.bulk.tensor) loads, programmatic-dependent-launch
// controls and the int8 -> fp32 conversion used by the weight-streaming GEMV.
//
// Every spin on an mbarrier is bounded: after kWaitLimitNs of global time the
// waiting thread records LLME_E_TIMEOUT in its translation unit's device error
// word and gives up, so a logic error shows up as a status on the host
// (llme_device_status) instead of a hung GPU.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "llme_b200.h"

namespace llme {

// 2 s: far above any legitimate wait (a whole 7B decode chain is ~1 ms).
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long global_timer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Makes mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking test. On sm_100 mbarrier.try_wait takes ~190 cycles to report a phase that
// has already completed and test_wait ~15, so the waits below test first and only then
// let try_wait suspend the thread.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete. Returns false (after
// setting *err) if kWaitLimitNs passed first.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int* err) {
    if (mbar_test_wait(bar, parity)) return true;
    const unsigned long long t0 = global_timer_ns();
    for (uint32_t i = 0;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63) == 63 && global_timer_ns() - t0 > kWaitLimitNs) {
            atomicExch(err, static_cast<unsigned int>(LLME_E_TIMEOUT));
            return false;
        }
    }
}

// As mbar_wait, with cluster-scope acquire: for barriers that the other CTA of a cluster
// arrives on.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_test_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity,
                                                  unsigned int* err) {
    if (mbar_test_wait_cluster(bar, parity)) return true;
    const unsigned long long t0 = global_timer_ns();
    for (uint32_t i = 0;; ++i) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if ((i & 63) == 63 && global_timer_ns() - t0 > kWaitLimitNs) {
            atomicExch(err, static_cast<unsigned int>(LLME_E_TIMEOUT));
            return false;
        }
    }
}

// L2 policy for data read exactly once (weights streamed by the GEMV).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2D tiled TMA load of the box at (x = inner coordinate, y = outer) into smem,
// completing `bar`'s transaction count.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::"
        "cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Brings the box at (x, y) into L2 only (no shared memory, no barrier): a hint that is safe
// to issue before griddepcontrol.wait, since L2 is where every write of the previous grid
// lands and a later load still reads the current contents.
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void tma_load_2d_nohint(void* dst, const CUtensorMap* map, int x, int y,
                                                   uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_1d(void* dst, const CUtensorMap* map, int x,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.1d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2}], [%3];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(smem_u32(bar))
        : "memory");
}

// Untiled bulk copy global -> shared (both 16-byte aligned, bytes a multiple of 16),
// completing `bar`'s transaction count.
__device__ __forceinline__ void bulk_load_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Programmatic dependent launch. wait: block until the grids this one depends
// on have finished and their writes are visible (a no-op when launched
// without the attribute). launch_dependents: allow the next grid on the
// stream to start its prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Barrier over the first `threads` threads of the block (named barrier `id`).
__device__ __forceinline__ void named_barrier(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Four signed bytes to four exact floats without I2F: each byte, offset by
// 128, becomes the low mantissa byte of 2^23 (0x4B0000xx = 2^23 + xx); one
// subtraction of 2^23 + 128 recovers the value. One PRMT and one FADD per
// element, both full-rate pipes.
__device__ __forceinline__ void s8x4_to_f32(uint32_t w, float (&x)[4]) {
    const uint32_t u = w ^ 0x80808080u;
    constexpr float kBias = 8388736.0f;  // 2^23 + 128
    x[0] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - kBias;
    x[1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - kBias;
    x[2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - kBias;
    x[3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - kBias;
}

// System-scope acquire load and release store of a 32-bit flag (cross-GPU handshakes over
// peer memory).
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// A 64-bit word written and read as one access at system scope: a value and its tag that
// cross NVLink together.
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Reads the tagged word at p once its tag (high 32 bits) equals `tag`, returning the value
// (low 32 bits as a float); after kWaitLimitNs sets *err and returns 0.
__device__ __forceinline__ float wait_tagged(const unsigned long long* p, unsigned tag,
                                             unsigned* err) {
    unsigned long long w = ld_relaxed_sys_u64(p);
    if (static_cast<unsigned>(w >> 32) == tag) return __uint_as_float(static_cast<unsigned>(w));
    const unsigned long long t0 = global_timer_ns();
    for (uint32_t i = 0;; ++i) {
        w = ld_relaxed_sys_u64(p);
        if (static_cast<unsigned>(w >> 32) == tag) return __uint_as_float(static_cast<unsigned>(w));
        if ((i & 255) == 255 && global_timer_ns() - t0 > kWaitLimitNs) {
            atomicExch(err, static_cast<unsigned>(LLME_E_TIMEOUT));
            return 0.0f;
        }
    }
}
__device__ __forceinline__ unsigned long long tagged(float v, unsigned tag) {
    return (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
}

// RMSNorm's eps, as the reference's ops.h / cuda_util.cuh.
constexpr float kRmsEps = 1e-5f;

// The int8 digits of y (|y| <= 127 up to one rounding) in base 256:
// y ~ t0 + t1 / 256 + t2 / 65536. Each residual times 256 is exact in fp32 (y - rint(y) is a
// multiple of y's unit in the last place, at most 1/2 in size). A second digit that rounds to
// +128 (y - t0 = 1/2 with t0 rounded to even below y) carries one into t0 and becomes -128,
// so every digit fits int8 and the error stays at most 2^-16 (2^-17 unless the last digit
// is clamped to 127).
__device__ __forceinline__ void int8_digits(float y, int& t0, int& t1, int& t2) {
    const float f0 = fminf(fmaxf(rintf(y), -127.0f), 127.0f);
    const float r1 = (y - f0) * 256.0f;  // [-128, 128]
    const float g1 = rintf(r1);
    const float f2 = fminf(fmaxf(rintf((r1 - g1) * 256.0f), -128.0f), 127.0f);
    const int carry = g1 > 127.0f ? 1 : 0;
    t0 = static_cast<int>(f0) + carry;
    t1 = static_cast<int>(g1) - 256 * carry;
    t2 = static_cast<int>(f2);
}

}  // namespace llme
