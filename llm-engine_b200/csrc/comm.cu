// Tensor-parallel products over NCCL (include/llme_b200.h, "multi-GPU").
//
// The reference has no collective; tensor parallelism adds exactly one: a sum all-reduce of the
// row-parallel (k-split) partial outputs of wo and w2. NCCL (libnccl.so.2) is opened with
// dlopen on first use, so single-GPU users of the library need no NCCL at all, and a process
// that already loaded NCCL (PyTorch does) shares that copy.
//
// Communicators are created non-blocking and polled against a host deadline, so a rank that
// never joins ends in LLME_E_TIMEOUT plus ncclCommAbort rather than a hang.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "llme_b200.h"

namespace {
constexpr int kPeerMaxRanks = 16;
constexpr int kPeerCtas = 64;
constexpr int kPeerThreads = 256;

// Device-side view of the peer all-reduce: every rank's symmetric buffer mapped into this
// process (own included), laid out as [2 slots][nranks sources][slot_words] epoch-tagged
// 64-bit words, plus this rank's per-CTA call counters.
struct PeerArgs {
    unsigned long long* base[kPeerMaxRanks];
    size_t slot_words;
    unsigned* epoch;   // kPeerCtas counters (local memory)
    unsigned* err;     // device error word
    int nranks, rank;
};
}  // namespace

struct llme_comm {
    ncclComm_t comm = nullptr;
    int nranks = 0;
    int rank = 0;
    // NVLink peer all-reduce (llme_comm_enable_peer)
    bool peer = false;
    size_t peer_max_floats = 0;
    void* peer_buf = nullptr;
    void* peer_epoch = nullptr;
    void* peer_opened[kPeerMaxRanks] = {};
    PeerArgs pargs{};
    // The GEMV's in-kernel rank sum (kEpiPeerSum): receive areas behind the all-reduce's in the
    // same shared buffer, one epoch counter per CTA slot.
    void* push_epoch = nullptr;
    llme::PeerSum push{};
};

namespace {

struct NcclApi {
    decltype(&ncclGetUniqueId) getUniqueId = nullptr;
    decltype(&ncclCommInitRankConfig) initRankConfig = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclCommAbort) abort = nullptr;
    decltype(&ncclCommGetAsyncError) asyncError = nullptr;
    decltype(&ncclAllReduce) allReduce = nullptr;
    decltype(&ncclAllGather) allGather = nullptr;
    decltype(&ncclGetErrorString) errorString = nullptr;
    bool ok = false;
    std::string why;
};

NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            const char* e = dlerror();
            api.why = std::string("cannot load libnccl.so.2: ") + (e ? e : "?");
            return;
        }
        auto sym = [&](const char* name) { return dlsym(h, name); };
        api.getUniqueId = reinterpret_cast<decltype(api.getUniqueId)>(sym("ncclGetUniqueId"));
        api.initRankConfig =
            reinterpret_cast<decltype(api.initRankConfig)>(sym("ncclCommInitRankConfig"));
        api.destroy = reinterpret_cast<decltype(api.destroy)>(sym("ncclCommDestroy"));
        api.abort = reinterpret_cast<decltype(api.abort)>(sym("ncclCommAbort"));
        api.asyncError = reinterpret_cast<decltype(api.asyncError)>(sym("ncclCommGetAsyncError"));
        api.allReduce = reinterpret_cast<decltype(api.allReduce)>(sym("ncclAllReduce"));
        api.allGather = reinterpret_cast<decltype(api.allGather)>(sym("ncclAllGather"));
        api.errorString = reinterpret_cast<decltype(api.errorString)>(sym("ncclGetErrorString"));
        api.ok = api.getUniqueId && api.initRankConfig && api.destroy && api.abort &&
                 api.asyncError && api.allReduce && api.allGather && api.errorString;
        if (!api.ok) api.why = "libnccl.so.2 lacks a needed symbol";
    });
    return api;
}

int nccl_fail(ncclResult_t r, const char* what) {
    NcclApi& api = nccl();
    return llme::set_error(LLME_E_NCCL, std::string("nccl: ") + what + ": " +
                                            (api.errorString ? api.errorString(r) : "error"));
}

int need_nccl() {
    NcclApi& api = nccl();
    return api.ok ? LLME_OK : llme::set_error(LLME_E_UNSUPPORTED, api.why);
}

// Polls a non-blocking communicator until its pending operation leaves ncclInProgress.
int wait_ready(llme_comm* c, double timeout_s, const char* what) {
    NcclApi& api = nccl();
    const auto deadline =
        std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s);
    for (;;) {
        ncclResult_t st = ncclSuccess;
        ncclResult_t r = api.asyncError(c->comm, &st);
        if (r != ncclSuccess) return nccl_fail(r, what);
        if (st == ncclSuccess) return LLME_OK;
        if (st != ncclInProgress) return nccl_fail(st, what);
        if (std::chrono::steady_clock::now() > deadline)
            return llme::set_error(LLME_E_TIMEOUT, std::string("nccl: ") + what +
                                                       ": not finished within the timeout");
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

// Enqueue-side waits of a non-blocking communicator (the GPU work itself stays async).
constexpr double kEnqueueTimeoutS = 60.0;

__device__ unsigned int g_comm_error;

// One-shot all-reduce over NVLink peer memory, in place on `data` (count floats, identical
// on every rank). CTA b owns elements [b*chunk, (b+1)*chunk). Each thread writes its elements
// into source row `rank` of slot (epoch & 1) of every rank's buffer as 64-bit words, the value's
// bits tagged with the call's epoch (one relaxed system-scope store: value and tag cross NVLink
// together), then reads the same elements back from its own buffer, source by source in rank
// order, each once its tag matches (bounded wait), and stores the sum -- so every rank gets the
// same bits, with no fence, flag or remote read. Two slots and monotonic per-CTA epochs make
// back-to-back calls (and CUDA-graph replays) safe: a rank writes epoch e + 2 of CTA b only
// after reading every peer's e + 1, written after that peer's kernel of epoch e had finished.
__global__ void __launch_bounds__(kPeerThreads) peer_allreduce_kernel(float* __restrict__ data,
                                                                        size_t count,
                                                                        const PeerArgs p) {
    __shared__ unsigned s_epoch;
    const int b = blockIdx.x, tid = threadIdx.x;
    if (tid == 0) {
        s_epoch = p.epoch[b] + 1;
        p.epoch[b] = s_epoch;
    }
    __syncthreads();
    const unsigned e = s_epoch;
    const size_t chunk = ((count + gridDim.x - 1) / gridDim.x + 3) / 4 * 4;
    const size_t lo = min(count, b * chunk), hi = min(count, lo + chunk);
    const size_t row = p.slot_words;                        // words of one source row
    const size_t slot = (e & 1u) * static_cast<size_t>(p.nranks) * row;
    for (size_t i = lo + tid; i < hi; i += kPeerThreads) {
        const unsigned long long w = llme::tagged(data[i], e);
        for (int q = 0; q < p.nranks; ++q)
            llme::st_relaxed_sys_u64(p.base[q] + slot + static_cast<size_t>(p.rank) * row + i, w);
    }
    for (size_t i = lo + tid; i < hi; i += kPeerThreads) {
        const unsigned long long* mine = p.base[p.rank] + slot + i;
        float v = llme::wait_tagged(mine, e, p.err);
        for (int r = 1; r < p.nranks; ++r) v += llme::wait_tagged(mine + static_cast<size_t>(r) * row, e, p.err);
        data[i] = v;
    }
}

}  // namespace

namespace llme {
int comm_peer_sum(llme_comm_t* c, GemvEpilogue* epi) {
    if (!c || !c->peer || c->push.world < 2)
        return set_error(LLME_E_UNSUPPORTED, "in-kernel rank sum: no peer-enabled communicator of "
                                             "2 to 8 ranks");
    *epi = GemvEpilogue{};
    epi->kind = kEpiPeerSum;
    epi->peer = c->push;
    return LLME_OK;
}
}  // namespace llme

extern "C" {

int llme_comm_unique_id(void* id) {
    return llme::guarded([&]() -> int {
        if (!id) return llme::set_error(LLME_E_INVALID, "llme_comm_unique_id: null id");
        int st = need_nccl();
        if (st) return st;
        static_assert(sizeof(ncclUniqueId) == LLME_COMM_ID_BYTES, "NCCL unique id size");
        ncclUniqueId u;
        ncclResult_t r = nccl().getUniqueId(&u);
        if (r != ncclSuccess) return nccl_fail(r, "get unique id");
        std::memcpy(id, &u, sizeof(u));
        return LLME_OK;
    });
}

int llme_comm_init(llme_comm_t** out, int nranks, int rank, const void* id, double timeout_s) {
    return llme::guarded([&]() -> int {
        if (!out || !id) return llme::set_error(LLME_E_INVALID, "llme_comm_init: null pointer");
        *out = nullptr;
        int st = need_nccl();
        if (st) return st;
        if (nranks < 1 || rank < 0 || rank >= nranks)
            return llme::set_error(LLME_E_INVALID, "llme_comm_init: rank " + std::to_string(rank) +
                                                       " of " + std::to_string(nranks));
        NcclApi& api = nccl();
        ncclUniqueId u;
        std::memcpy(&u, id, sizeof(u));
        ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
        cfg.blocking = 0;
        auto* c = new llme_comm;
        c->nranks = nranks;
        c->rank = rank;
        ncclResult_t r = api.initRankConfig(&c->comm, nranks, u, rank, &cfg);
        if (r != ncclSuccess && r != ncclInProgress) {
            delete c;
            return nccl_fail(r, "init");
        }
        st = wait_ready(c, timeout_s, "init");
        if (st) {
            if (c->comm) api.abort(c->comm);
            delete c;
            return st;
        }
        *out = c;
        return LLME_OK;
    });
}

static void peer_release(llme_comm* c) {
    for (int r = 0; r < kPeerMaxRanks; ++r)
        if (c->peer_opened[r]) cudaIpcCloseMemHandle(c->peer_opened[r]);
    if (c->peer_buf) cudaFree(c->peer_buf);
    if (c->peer_epoch) cudaFree(c->peer_epoch);
    if (c->push_epoch) cudaFree(c->push_epoch);
    c->peer_buf = c->peer_epoch = c->push_epoch = nullptr;
    c->push = llme::PeerSum{};
    c->peer = false;
}

int llme_comm_enable_peer(llme_comm_t* c, size_t max_floats) {
    return llme::guarded([&]() -> int {
        if (!c) return llme::set_error(LLME_E_INVALID, "llme_comm_enable_peer: no communicator");
        if (c->peer) return LLME_OK;
        if (c->nranks > kPeerMaxRanks)
            return llme::set_error(LLME_E_UNSUPPORTED, "llme_comm_enable_peer: more than 16 ranks");
        const size_t slot = (max_floats + 63) / 64 * 64;
        const size_t ar_bytes = 2 * static_cast<size_t>(c->nranks) * slot * sizeof(unsigned long long);
        // The GEMVs' in-kernel rank sum: per slot, per CTA of a resident grid (two per SM),
        // per source rank, the epoch-tagged 64-bit words of the values a CTA owns (a per-call
        // GEMV CTA at most 8 rows x 128 columns, a grouped CTA its units' strips, up to 2048).
        int dev = 0, sms = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const int units = 2 * (sms > 0 ? sms : 148);
        const int unit_words = 2048;
        const bool push = c->nranks <= llme::kPeerSumMaxRanks;
        const size_t push_off = (ar_bytes + 255) / 256 * 256;
        const size_t push_bytes =
            2 * static_cast<size_t>(units) * c->nranks * unit_words * sizeof(unsigned long long);
        const size_t bytes = push ? push_off + push_bytes : ar_bytes;
        cudaError_t e = cudaMalloc(&c->peer_buf, bytes);
        if (e == cudaSuccess) e = cudaMemset(c->peer_buf, 0, bytes);
        if (e == cudaSuccess) e = cudaMalloc(&c->peer_epoch, kPeerCtas * sizeof(unsigned));
        if (e == cudaSuccess) e = cudaMemset(c->peer_epoch, 0, kPeerCtas * sizeof(unsigned));
        if (e == cudaSuccess && push) e = cudaMalloc(&c->push_epoch, units * sizeof(unsigned));
        if (e == cudaSuccess && push) e = cudaMemset(c->push_epoch, 0, units * sizeof(unsigned));
        cudaIpcMemHandle_t mine;
        if (e == cudaSuccess) e = cudaIpcGetMemHandle(&mine, c->peer_buf);
        if (e != cudaSuccess) {
            peer_release(c);
            return llme::set_cuda_error(e, "peer buffer");
        }
        // Exchange the handles over the communicator itself.
        void* d_handles = nullptr;
        e = cudaMalloc(&d_handles, sizeof(cudaIpcMemHandle_t) * (c->nranks + 1));
        if (e != cudaSuccess) {
            peer_release(c);
            return llme::set_cuda_error(e, "peer handles");
        }
        char* dh = static_cast<char*>(d_handles);
        cudaMemcpy(dh + sizeof(cudaIpcMemHandle_t) * c->nranks, &mine, sizeof(mine), cudaMemcpyHostToDevice);
        cudaStream_t st;
        cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
        ncclResult_t r = nccl().allGather(dh + sizeof(cudaIpcMemHandle_t) * c->nranks, dh,
                                          sizeof(cudaIpcMemHandle_t), ncclUint8, c->comm, st);
        int status = LLME_OK;
        if (r == ncclInProgress) status = wait_ready(c, kEnqueueTimeoutS, "exchange peer handles");
        else if (r != ncclSuccess) status = nccl_fail(r, "exchange peer handles");
        std::vector<cudaIpcMemHandle_t> all(c->nranks);
        if (!status) {
            cudaStreamSynchronize(st);
            e = cudaMemcpy(all.data(), dh, sizeof(cudaIpcMemHandle_t) * c->nranks, cudaMemcpyDeviceToHost);
            if (e != cudaSuccess) status = llme::set_cuda_error(e, "peer handles");
        }
        cudaStreamDestroy(st);
        cudaFree(d_handles);
        if (status) {
            peer_release(c);
            return status;
        }
        PeerArgs& pa = c->pargs;
        for (int q = 0; q < c->nranks; ++q) {
            if (q == c->rank) {
                pa.base[q] = static_cast<unsigned long long*>(c->peer_buf);
                continue;
            }
            void* ptr = nullptr;
            e = cudaIpcOpenMemHandle(&ptr, all[q], cudaIpcMemLazyEnablePeerAccess);
            if (e != cudaSuccess) {
                peer_release(c);
                return llme::set_cuda_error(e, "open peer buffer");
            }
            c->peer_opened[q] = ptr;
            pa.base[q] = static_cast<unsigned long long*>(ptr);
        }
        void* err = nullptr;
        cudaGetSymbolAddress(&err, g_comm_error);
        pa.slot_words = slot;
        pa.epoch = static_cast<unsigned*>(c->peer_epoch);
        pa.err = static_cast<unsigned*>(err);
        pa.nranks = c->nranks;
        pa.rank = c->rank;
        if (push) {
            llme::PeerSum& ps = c->push;
            for (int q = 0; q < c->nranks; ++q)
                ps.base[q] = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(pa.base[q]) +
                                                                   push_off);
            ps.units = units;
            ps.unit_words = unit_words;
            ps.epoch = static_cast<unsigned*>(c->push_epoch);
            ps.err = pa.err;
            ps.world = c->nranks;
            ps.rank = c->rank;
        }
        c->peer_max_floats = max_floats;
        c->peer = true;
        return LLME_OK;
    });
}

int llme_comm_status(void) {
    return llme::guarded([&]() -> int {
        unsigned v = 0, zero = 0;
        cudaError_t e = cudaMemcpyFromSymbol(&v, g_comm_error, sizeof(v));
        if (e != cudaSuccess) return llme::set_cuda_error(e, "read comm status");
        if (v) {
            cudaMemcpyToSymbol(g_comm_error, &zero, sizeof(zero));
            return llme::set_error(LLME_E_TIMEOUT, "peer all-reduce: a peer did not arrive in time");
        }
        return LLME_OK;
    });
}

int llme_comm_destroy(llme_comm_t* c) {
    return llme::guarded([&]() -> int {
        if (!c) return LLME_OK;
        peer_release(c);
        NcclApi& api = nccl();
        ncclResult_t r = api.destroy(c->comm);
        int st = LLME_OK;
        if (r == ncclInProgress) {
            st = wait_ready(c, kEnqueueTimeoutS, "destroy");
        } else if (r != ncclSuccess) {
            st = nccl_fail(r, "destroy");
        }
        delete c;
        return st;
    });
}

int llme_comm_abort(llme_comm_t* c) {
    return llme::guarded([&]() -> int {
        if (!c) return LLME_OK;
        peer_release(c);
        ncclResult_t r = nccl().abort(c->comm);
        delete c;
        return r == ncclSuccess ? LLME_OK : nccl_fail(r, "abort");
    });
}

int llme_comm_size(const llme_comm_t* c) { return c ? c->nranks : 0; }
int llme_comm_rank(const llme_comm_t* c) { return c ? c->rank : -1; }

int llme_allreduce_sum_f32(float* buf, size_t count, llme_comm_t* c, void* stream_ptr) {
    return llme::guarded([&]() -> int {
        if (!c) return llme::set_error(LLME_E_INVALID, "llme_allreduce_sum_f32: no communicator");
        if (c->nranks == 1 || count == 0) return LLME_OK;
        if (!buf) return llme::set_error(LLME_E_INVALID, "llme_allreduce_sum_f32: null buffer");
        cudaStream_t stream = stream_ptr ? static_cast<cudaStream_t>(stream_ptr) : cudaStreamPerThread;
        if (c->peer && count <= c->peer_max_floats) {
            peer_allreduce_kernel<<<kPeerCtas, kPeerThreads, 0, stream>>>(buf, count, c->pargs);
            cudaError_t e = cudaGetLastError();
            return e == cudaSuccess ? LLME_OK : llme::set_cuda_error(e, "launch");
        }
        ncclResult_t r = nccl().allReduce(buf, buf, count, ncclFloat32, ncclSum, c->comm, stream);
        if (r == ncclInProgress) return wait_ready(c, kEnqueueTimeoutS, "all-reduce");
        return r == ncclSuccess ? LLME_OK : nccl_fail(r, "all-reduce");
    });
}

static int rowpar(size_t m, size_t n, size_t k_local, const float* A, const void* B,
                  const float* scale, float* C, bool q8, int kernel, int accumulate,
                  unsigned flags, llme_comm_t* c, void* stream) {
    if (!c) return llme::set_error(LLME_E_INVALID, "row-parallel product: no communicator");
    // Only rank 0 adds the existing C, so after the sum it is counted once.
    const bool acc = accumulate != 0 && c->rank == 0;
    const unsigned kflags = flags & ~static_cast<unsigned>(LLME_FLAG_SAME_SHARDS);
    if ((flags & LLME_FLAG_SAME_SHARDS) && c->nranks > 1 && kernel == LLME_KERNEL_AUTOMATIC) {
        // Every rank runs the same plan: the sum is taken inside the GEMV when it takes it.
        llme::GemvEpilogue epi;
        if (llme::comm_peer_sum(c, &epi) == LLME_OK) {
            const int st = llme::run_product_epilogue(m, n, k_local, A, B, scale, C, q8, nullptr,
                                                      kflags, stream, epi, acc);
            if (st != LLME_E_UNSUPPORTED) return st;
        }
    }
    int st = llme::run_product(m, n, k_local, A, B, scale, C, q8, kernel, acc, nullptr, kflags,
                               stream);
    if (st) return st;
    return llme_allreduce_sum_f32(C, m * n, c, stream);
}

int llme_matmul_q8_rowpar(size_t m, size_t n, size_t k_local, const float* A_local,
                          const int8_t* B_local, const float* scale, float* C, int kernel,
                          int accumulate, unsigned flags, llme_comm_t* comm, void* stream) {
    return llme::guarded([&]() -> int {
        return rowpar(m, n, k_local, A_local, B_local, scale, C, true, kernel, accumulate, flags, comm,
                      stream);
    });
}

int llme_matmul_f32_rowpar(size_t m, size_t n, size_t k_local, const float* A_local,
                           const float* B_local, float* C, int kernel, int accumulate,
                           unsigned flags, llme_comm_t* comm, void* stream) {
    return llme::guarded([&]() -> int {
        return rowpar(m, n, k_local, A_local, B_local, nullptr, C, false, kernel, accumulate, flags,
                      comm, stream);
    });
}

}  // extern "C"
