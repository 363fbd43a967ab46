// Tensor-parallel products over NCCL (include/llme_b200.h, "multi-GPU").
//
// The reference has no collective; the north star adds exactly one: a sum all-reduce of the
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

#include "kernels.h"
#include "llme_b200.h"

struct llme_comm {
    ncclComm_t comm = nullptr;
    int nranks = 0;
    int rank = 0;
};

namespace {

struct NcclApi {
    decltype(&ncclGetUniqueId) getUniqueId = nullptr;
    decltype(&ncclCommInitRankConfig) initRankConfig = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclCommAbort) abort = nullptr;
    decltype(&ncclCommGetAsyncError) asyncError = nullptr;
    decltype(&ncclAllReduce) allReduce = nullptr;
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
        api.errorString = reinterpret_cast<decltype(api.errorString)>(sym("ncclGetErrorString"));
        api.ok = api.getUniqueId && api.initRankConfig && api.destroy && api.abort &&
                 api.asyncError && api.allReduce && api.errorString;
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

}  // namespace

extern "C" {

int llme_comm_unique_id(void* id) {
    int st = need_nccl();
    if (st) return st;
    static_assert(sizeof(ncclUniqueId) == LLME_COMM_ID_BYTES, "NCCL unique id size");
    ncclUniqueId u;
    ncclResult_t r = nccl().getUniqueId(&u);
    if (r != ncclSuccess) return nccl_fail(r, "get unique id");
    std::memcpy(id, &u, sizeof(u));
    return LLME_OK;
}

int llme_comm_init(llme_comm_t** out, int nranks, int rank, const void* id, double timeout_s) {
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
}

int llme_comm_destroy(llme_comm_t* c) {
    if (!c) return LLME_OK;
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
}

int llme_comm_abort(llme_comm_t* c) {
    if (!c) return LLME_OK;
    ncclResult_t r = nccl().abort(c->comm);
    delete c;
    return r == ncclSuccess ? LLME_OK : nccl_fail(r, "abort");
}

int llme_comm_size(const llme_comm_t* c) { return c ? c->nranks : 0; }
int llme_comm_rank(const llme_comm_t* c) { return c ? c->rank : -1; }

int llme_allreduce_sum_f32(float* buf, size_t count, llme_comm_t* c, void* stream_ptr) {
    if (!c) return llme::set_error(LLME_E_INVALID, "llme_allreduce_sum_f32: no communicator");
    if (c->nranks == 1 || count == 0) return LLME_OK;
    cudaStream_t stream = stream_ptr ? static_cast<cudaStream_t>(stream_ptr) : cudaStreamPerThread;
    ncclResult_t r = nccl().allReduce(buf, buf, count, ncclFloat32, ncclSum, c->comm, stream);
    if (r == ncclInProgress) return wait_ready(c, kEnqueueTimeoutS, "all-reduce");
    return r == ncclSuccess ? LLME_OK : nccl_fail(r, "all-reduce");
}

static int rowpar(size_t m, size_t n, size_t k_local, const float* A, const void* B,
                  const float* scale, float* C, bool q8, int kernel, int accumulate,
                  unsigned flags, llme_comm_t* c, void* stream) {
    if (!c) return llme::set_error(LLME_E_INVALID, "row-parallel product: no communicator");
    // Only rank 0 adds the existing C, so after the sum it is counted once.
    const bool acc = accumulate != 0 && c->rank == 0;
    int st = llme::run_product(m, n, k_local, A, B, scale, C, q8, kernel, acc, nullptr, flags,
                               stream);
    if (st) return st;
    return llme_allreduce_sum_f32(C, m * n, c, stream);
}

int llme_matmul_q8_rowpar(size_t m, size_t n, size_t k_local, const float* A_local,
                          const int8_t* B_local, const float* scale, float* C, int kernel,
                          int accumulate, unsigned flags, llme_comm_t* comm, void* stream) {
    return rowpar(m, n, k_local, A_local, B_local, scale, C, true, kernel, accumulate, flags, comm,
                  stream);
}

int llme_matmul_f32_rowpar(size_t m, size_t n, size_t k_local, const float* A_local,
                           const float* B_local, float* C, int kernel, int accumulate,
                           unsigned flags, llme_comm_t* comm, void* stream) {
    return rowpar(m, n, k_local, A_local, B_local, nullptr, C, false, kernel, accumulate, flags,
                  comm, stream);
}

}  // extern "C"
