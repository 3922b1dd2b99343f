// ============================================================================
//  api/dist.cpp -- the row-partitioned forward over several GPUs behind the
//  C ABI (tg_dist_*): one process per GPU, an NCCL communicator, equal 1-D
//  row blocks, Model::forward_rows with an in-place NCCL all-gather of each
//  layer's exchanged rows.
//
//  NCCL is loaded when tg_dist_init runs (dlopen of libnccl.so.2 -- the copy
//  already in the process, e.g. torch's, or the system one), so the library
//  itself does not depend on it.  The communicator is non-blocking: joining
//  and every collective are polled with the caller's timeout, and a wait
//  that runs out aborts the communicator (which ends its kernels) and
//  returns TG_ERR_TIMEOUT -- a rank that never joins or dies mid-forward
//  cannot leave the others waiting for ever.
//
//  Rank 0 writes the communicator's unique id to `id_path` (written to a
//  temporary name, then renamed); the other ranks wait for the file.
// ============================================================================
#include <dlfcn.h>
#include <unistd.h>
#include <nccl.h>

#include <chrono>
#include <cstdio>
#include <fstream>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>

#include "internal.hpp"
#include "tinygnn/model.hpp"

namespace tg {
void set_last_error(const std::string& m);
}  // namespace tg

namespace {

struct NcclError : std::runtime_error {
    tg_status status;
    NcclError(tg_status s, const std::string& m) : std::runtime_error(m), status(s) {}
};

// The NCCL entry points used here, resolved from the loaded library.
struct Nccl {
    ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*commInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*commGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*allGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*commAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
    const char* (*getErrorString)(ncclResult_t) = nullptr;
};

const Nccl& nccl() {
    static Nccl api;
    static std::string error;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            error = std::string("tg_dist: cannot load NCCL (libnccl.so.2): ") + dlerror();
            return;
        }
        auto sym = [&](const char* name) {
            void* p = dlsym(h, name);
            if (!p) error = std::string("tg_dist: NCCL has no ") + name;
            return p;
        };
        api.getUniqueId = reinterpret_cast<decltype(api.getUniqueId)>(sym("ncclGetUniqueId"));
        api.commInitRankConfig = reinterpret_cast<decltype(api.commInitRankConfig)>(sym("ncclCommInitRankConfig"));
        api.commGetAsyncError = reinterpret_cast<decltype(api.commGetAsyncError)>(sym("ncclCommGetAsyncError"));
        api.allGather = reinterpret_cast<decltype(api.allGather)>(sym("ncclAllGather"));
        api.commAbort = reinterpret_cast<decltype(api.commAbort)>(sym("ncclCommAbort"));
        api.commDestroy = reinterpret_cast<decltype(api.commDestroy)>(sym("ncclCommDestroy"));
        api.getErrorString = reinterpret_cast<decltype(api.getErrorString)>(sym("ncclGetErrorString"));
    });
    if (!error.empty()) throw NcclError(TG_ERR_NCCL, error);
    return api;
}

std::string nccl_text(ncclResult_t r) {
    const char* s = nccl().getErrorString ? nccl().getErrorString(r) : nullptr;
    return s ? s : ("NCCL error " + std::to_string(static_cast<int>(r)));
}

using Clock = std::chrono::steady_clock;

}  // namespace

struct tg_dist_s : tinygnn::RowExchange {
    ncclComm_t comm = nullptr;
    int world_ = 1, rank_ = 0, device = 0;
    int timeout_ms = 60000;
    bool aborted = false;
    // NCCL runs on a stream of its own, ordered against the calling thread's
    // stream by events: the per-thread default stream is a pseudo-handle
    // that names a different stream in whichever thread uses it, and NCCL
    // may enqueue a non-blocking communicator's work from its own thread.
    cudaStream_t ns = nullptr;
    cudaEvent_t ready = nullptr, gathered = nullptr;

    ~tg_dist_s() {
        if (gathered) cudaEventDestroy(gathered);
        if (ready) cudaEventDestroy(ready);
        if (ns) cudaStreamDestroy(ns);
    }

    int world() const override { return world_; }
    int rank() const override { return rank_; }

    // Polls the communicator until its pending operation is accepted (or the
    // deadline passes: abort, TG_ERR_TIMEOUT).
    void settle(ncclResult_t r, const char* what) {
        const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
        while (r == ncclInProgress) {
            if (Clock::now() > deadline) fail_timeout(what);
            std::this_thread::sleep_for(std::chrono::microseconds(100));
            ncclResult_t st = ncclSuccess;
            const ncclResult_t q = nccl().commGetAsyncError(comm, &st);
            r = q != ncclSuccess ? q : st;
        }
        if (r != ncclSuccess) throw NcclError(TG_ERR_NCCL, std::string("tg_dist: ") + what + ": " + nccl_text(r));
    }

    [[noreturn]] void fail_timeout(const char* what) {
        if (comm && !aborted) {
            nccl().commAbort(comm);
            aborted = true;
            comm = nullptr;
        }
        throw NcclError(TG_ERR_TIMEOUT, std::string("tg_dist: ") + what + " did not complete within " +
                                            std::to_string(timeout_ms) + " ms (a rank missing?); the communicator "
                                                                         "was aborted");
    }

    void all_gather(float* buf, std::size_t count) override {
        if (aborted || !comm) throw NcclError(TG_ERR_NCCL, "tg_dist: the communicator was aborted");
        if (world_ == 1) return;
        const float* mine = buf + static_cast<std::size_t>(rank_) * count;
        const cudaStream_t cs = tinygnn::detail::cstream();
        tinygnn::detail::cuda(cudaEventRecord(ready, cs), "tg_dist all-gather");
        tinygnn::detail::cuda(cudaStreamWaitEvent(ns, ready, 0), "tg_dist all-gather");
        settle(nccl().allGather(mine, buf, count, ncclFloat, comm, ns), "all-gather");
        tinygnn::detail::cuda(cudaEventRecord(gathered, ns), "tg_dist all-gather");
        tinygnn::detail::cuda(cudaStreamWaitEvent(cs, gathered, 0), "tg_dist all-gather");
    }

    // Waits for the calling thread's stream, watching the communicator.
    void drain(const char* what) {
        const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
        for (;;) {
            cudaError_t e = cudaStreamQuery(tinygnn::detail::cstream());
            if (e == cudaSuccess && ns) e = cudaStreamQuery(ns);
            if (e == cudaSuccess) return;
            if (e != cudaErrorNotReady) tinygnn::detail::cuda(e, what);
            ncclResult_t st = ncclSuccess;
            if (comm) nccl().commGetAsyncError(comm, &st);
            if (st != ncclSuccess && st != ncclInProgress)
                throw NcclError(TG_ERR_NCCL, std::string("tg_dist: ") + what + ": " + nccl_text(st));
            if (Clock::now() > deadline) fail_timeout(what);
            std::this_thread::sleep_for(std::chrono::microseconds(50));
        }
    }
};


namespace {

template <class F>
tg_status dist_api(F&& f) noexcept {
    try {
        f();
        return TG_OK;
    } catch (const NcclError& e) {
        tg::set_last_error(e.what());
        return e.status;
    } catch (const std::invalid_argument& e) {
        tg::set_last_error(e.what());
        return TG_ERR_INVALID_ARGUMENT;
    } catch (const std::exception& e) {
        tg::set_last_error(e.what());
        return TG_ERR_RUNTIME;
    } catch (...) {
        tg::set_last_error("unknown error");
        return TG_ERR_RUNTIME;
    }
}

void need(const void* p, const char* what) {
    if (!p) throw std::invalid_argument(std::string(what) + " is NULL");
}

}  // namespace

extern "C" {

TG_API tg_status tg_dist_partition_csr(int32_t world, int32_t rank, int64_t n, const int32_t* row_ptr,
                                       int64_t* row_begin, int64_t* row_end, int64_t* entry_begin,
                                       int64_t* entry_end) {
    return dist_api([&] {
        if (world < 1 || rank < 0 || rank >= world) throw std::invalid_argument("tg_dist_partition_csr: bad world / rank");
        if (n < 0) throw std::invalid_argument("tg_dist_partition_csr: negative size");
        const int64_t R = (n + world - 1) / world;
        const int64_t r0 = std::min<int64_t>(n, static_cast<int64_t>(rank) * R), r1 = std::min<int64_t>(n, r0 + R);
        if (row_begin) *row_begin = r0;
        if (row_end) *row_end = r1;
        if (entry_begin || entry_end) {
            need(row_ptr, "tg_dist_partition_csr: row_ptr");
            if (entry_begin) *entry_begin = row_ptr[r0];
            if (entry_end) *entry_end = row_ptr[r1];
        }
    });
}

TG_API tg_status tg_dist_init(int32_t world, int32_t rank, int32_t device, const char* id_path, int32_t timeout_ms,
                              tg_dist* out) {
    return dist_api([&] {
        need(out, "tg_dist_init: out");
        need(id_path, "tg_dist_init: id_path");
        *out = nullptr;
        if (world < 1 || rank < 0 || rank >= world) throw std::invalid_argument("tg_dist_init: bad world / rank");
        if (timeout_ms <= 0) throw std::invalid_argument("tg_dist_init: timeout_ms must be > 0");
        int ndev = 0;
        if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
            cudaGetLastError();
            throw NcclError(TG_ERR_NO_DEVICE, "tinygnn_b200: no CUDA device is visible; this library has no CPU path");
        }
        if (device < 0 || device >= ndev) throw std::invalid_argument("tg_dist_init: no such device");
        tinygnn::detail::cuda(cudaSetDevice(device), "tg_dist_init");
        const Nccl& api = nccl();
        auto d = std::make_unique<tg_dist_s>();
        d->world_ = world;
        d->rank_ = rank;
        d->device = device;
        d->timeout_ms = timeout_ms;
        tinygnn::detail::cuda(cudaStreamCreateWithFlags(&d->ns, cudaStreamNonBlocking), "tg_dist_init");
        tinygnn::detail::cuda(cudaEventCreateWithFlags(&d->ready, cudaEventDisableTiming), "tg_dist_init");
        tinygnn::detail::cuda(cudaEventCreateWithFlags(&d->gathered, cudaEventDisableTiming), "tg_dist_init");
        ncclUniqueId id;
        const std::string path(id_path);
        if (rank == 0) {
            const ncclResult_t r = api.getUniqueId(&id);
            if (r != ncclSuccess) throw NcclError(TG_ERR_NCCL, "tg_dist_init: ncclGetUniqueId: " + nccl_text(r));
            const std::string tmp = path + ".tmp" + std::to_string(static_cast<long>(::getpid()));
            {
                std::ofstream f(tmp, std::ios::binary);
                f.write(reinterpret_cast<const char*>(&id), sizeof(id));
                if (!f) throw std::runtime_error("tg_dist_init: cannot write " + tmp);
            }
            if (std::rename(tmp.c_str(), path.c_str()) != 0)
                throw std::runtime_error("tg_dist_init: cannot rename " + tmp + " to " + path);
        } else {
            const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
            for (;;) {
                std::ifstream f(path, std::ios::binary);
                if (f && f.read(reinterpret_cast<char*>(&id), sizeof(id))) break;
                if (Clock::now() > deadline)
                    throw NcclError(TG_ERR_TIMEOUT, "tg_dist_init: rank 0's id file " + path + " did not appear within " +
                                                        std::to_string(timeout_ms) + " ms");
                std::this_thread::sleep_for(std::chrono::milliseconds(5));
            }
        }
        ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
        cfg.blocking = 0;  // joining is polled with the timeout
        ncclComm_t comm = nullptr;
        const ncclResult_t r = api.commInitRankConfig(&comm, world, id, rank, &cfg);
        d->comm = comm;
        d->settle(r, "joining the communicator");
        *out = d.release();
    });
}

TG_API tg_status tg_dist_forward(tg_dist d, tg_model m, int64_t n, tg_tensor adjacency_rows, tg_tensor feature_rows,
                                 tg_tensor* out) {
    return dist_api([&] {
        need(d, "tg_dist_forward: d");
        need(m, "tg_dist_forward: m");
        need(adjacency_rows, "tg_dist_forward: adjacency_rows");
        need(feature_rows, "tg_dist_forward: feature_rows");
        need(out, "tg_dist_forward: out");
        *out = nullptr;
        if (n < 0) throw std::invalid_argument("tg_dist_forward: negative size");
        tinygnn::detail::cuda(cudaSetDevice(d->device), "tg_dist_forward");
        auto h = std::make_unique<tg_tensor_s>(
            tg_tensor_s{m->m.forward_rows(adjacency_rows->t, static_cast<std::size_t>(n), feature_rows->t, *d)});
        d->drain("the partitioned forward");
        *out = h.release();
    });
}

TG_API tg_status tg_dist_finalize(tg_dist d) {
    return dist_api([&] {
        if (!d) return;
        std::unique_ptr<tg_dist_s> own(d);
        if (own->comm && !own->aborted) {
            const ncclResult_t r = nccl().commDestroy(own->comm);
            own->comm = nullptr;
            if (r != ncclSuccess) throw NcclError(TG_ERR_NCCL, "tg_dist_finalize: " + nccl_text(r));
        }
    });
}

}  // extern "C"
