// ============================================================================
//  peer.cu -- the fused GEMM -> exchange over NVLink (one process per GPU).
//
//  The row-partitioned layer computes this rank's rows of H.W and every rank
//  needs all of them.  Instead of a GEMM followed by an NCCL all-gather, the
//  tensor-core GEMM's epilogue stores each output tile into every peer's
//  copy of the gathered operand as well as its own (plain stores to peer
//  memory mapped with CUDA IPC), so the transfer overlaps the GEMM tile by
//  tile; after a tile has landed everywhere the CTA adds 1 to this rank's
//  completion counter in each peer's memory (release, system scope).  A
//  rank then waits -- on its own GPU, bounded in time -- until every peer's
//  counter has reached the number of tiles that peer owns, and gathers.
//
//    tg_ipc_get_handle / tg_ipc_open_handle / tg_ipc_close_handle  mapping
//    tg_gemm_peers_f32                                             GEMM + stores + signal
//    tg_wait_flags                                                 the bounded wait
//
//  No TMA reads peer memory (the GEMM's TMA loads read this GPU's A and B
//  only), and no kernel waits on another kernel of the same GPU.
// ============================================================================
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <vector>

#include "launch.cuh"
#include "mbarrier.cuh"

namespace tg {

void gemm_tc(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb, float* C,
             int64_t ldc, const float* bias, int act, float alpha, cudaStream_t s, const PeerOut& peers,
             bool c_cols_padded, const float* row_scale);
bool gemm_tc_supported(int64_t N, int64_t K, const float* A, int64_t lda);

namespace {

__device__ int g_peer_error = 0;  // first wait timeout seen: 20 + the flag's index

constexpr int kMaxFlags = 8;
struct Targets {
    unsigned long long v[kMaxFlags];
};

// Thread i waits until flags[i] >= t.v[i] (0 = nothing to wait for), reading
// with acquire semantics at system scope; gives up after timeout_ns.
__global__ void wait_flags_kernel(const unsigned long long* flags, Targets t, int n, unsigned long long timeout_ns,
                                  int* err) {
    const int i = threadIdx.x;
    if (i < n && t.v[i] != 0) {
        const uint64_t t0 = mb::global_ns();
        for (uint32_t it = 0;; ++it) {
            unsigned long long v;
            asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flags + i) : "memory");
            if (v >= t.v[i]) break;
            if ((it & 15) == 15 && mb::global_ns() - t0 > timeout_ns) {
                atomicCAS(err, 0, 20 + i);
                break;
            }
            __nanosleep(128);
        }
    }
    __syncthreads();
}

int* peer_error_word() {
    static std::mutex mu;
    static std::vector<int*> words;
    int dev = 0;
    TG_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(mu);
    if (static_cast<int>(words.size()) <= dev) words.resize(dev + 1, nullptr);
    if (!words[dev]) TG_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&words[dev]), g_peer_error));
    return words[dev];
}

PFN_cuMemGetAddressRange_v3020 address_range_fn() {
    static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
        else
            cudaGetLastError();
    });
    if (!fn) fail(TG_ERR_CUDA, "ipc: cuMemGetAddressRange is unavailable");
    return fn;
}

}  // namespace

// Reads and clears the wait kernel's error word (synchronises `s`).
int peer_take_error(cudaStream_t s) {
    int h = 0;
    TG_CUDA(cudaStreamSynchronize(s));
    TG_CUDA(cudaMemcpyFromSymbol(&h, g_peer_error, sizeof(int)));
    if (h) {
        const int zero = 0;
        TG_CUDA(cudaMemcpyToSymbol(g_peer_error, &zero, sizeof(int)));
    }
    return h;
}

}  // namespace tg

using namespace tg;

extern "C" {

TG_API tg_status tg_ipc_get_handle(const void* ptr, void* handle_out, int64_t* offset_out) {
    return guard([&] {
        require_device();
        check_ptr("ipc_get_handle", "ptr", ptr, true);
        check_ptr("ipc_get_handle", "handle_out", handle_out, true);
        check_ptr("ipc_get_handle", "offset_out", offset_out, true);
        CUdeviceptr base = 0;
        size_t size = 0;
        if (address_range_fn()(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
            invalid("ipc_get_handle: ptr is not device memory of this process");
        cudaIpcMemHandle_t h;
        TG_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
        std::memcpy(handle_out, &h, sizeof(h));
        *offset_out = static_cast<int64_t>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base));
    });
}

TG_API tg_status tg_ipc_open_handle(const void* handle, void** base_out) {
    return guard([&] {
        require_device();
        check_ptr("ipc_open_handle", "handle", handle, true);
        check_ptr("ipc_open_handle", "base_out", base_out, true);
        cudaIpcMemHandle_t h;
        std::memcpy(&h, handle, sizeof(h));
        TG_CUDA(cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess));
    });
}

TG_API tg_status tg_ipc_close_handle(void* base) {
    return guard([&] {
        require_device();
        check_ptr("ipc_close_handle", "base", base, true);
        TG_CUDA(cudaIpcCloseMemHandle(base));
    });
}

TG_API tg_status tg_gemm_peers_f32(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B,
                                   int64_t ldb, float* C, int64_t ldc, const float* bias, int32_t act, float alpha,
                                   const float* row_scale, int32_t npeers, float* const* peer_C,
                                   uint64_t* const* peer_flags, int32_t flags, void* stream) {
    return guard([&] {
        require_device();
        if (M < 0 || N < 0 || K < 0) invalid("gemm_peers: negative size");
        if (npeers < 0 || npeers > kMaxPeers)
            invalid("gemm_peers: npeers = " + std::to_string(npeers) + " (at most " + std::to_string(kMaxPeers) + ")");
        check_ld("gemm_peers", "A", lda, K);
        check_ld("gemm_peers", "B", ldb, N);
        check_ld("gemm_peers", "C", ldc, N);
        if (M == 0 || N == 0) return;
        check_ptr("gemm_peers", "A", A, K > 0);
        check_ptr("gemm_peers", "B", B, K > 0);
        check_ptr("gemm_peers", "C", C, true);
        if (!gemm_tc_supported(N, K, A, lda))
            invalid("gemm_peers: the tensor-core path needs N <= 256, lda % 4 == 0 and A 16-byte aligned");
        PeerOut peers;
        peers.n = npeers;
        for (int p = 0; p < npeers; ++p) {
            check_ptr("gemm_peers", "peer_C[p]", peer_C ? peer_C[p] : nullptr, true);
            check_ptr("gemm_peers", "peer_flags[p]", peer_flags ? peer_flags[p] : nullptr, true);
            peers.c[p] = peer_C[p];
            peers.flag[p] = reinterpret_cast<unsigned long long*>(peer_flags[p]);
        }
        gemm_tc(M, N, K, A, lda, B, ldb, C, ldc, bias, act, alpha, as_stream(stream), peers,
                (flags & TG_FLAG_C_COLS_PADDED) != 0, row_scale);
    });
}

TG_API tg_status tg_wait_flags(const uint64_t* flags, const uint64_t* targets, int32_t n, int64_t timeout_ns,
                               void* stream) {
    return guard([&] {
        require_device();
        if (n < 0 || n > kMaxFlags) invalid("wait_flags: n = " + std::to_string(n) + " (at most 8)");
        if (timeout_ns <= 0) invalid("wait_flags: timeout_ns must be positive");
        if (n == 0) return;
        check_ptr("wait_flags", "flags", flags, true);
        check_ptr("wait_flags", "targets", targets, true);
        Targets t{};
        for (int i = 0; i < n; ++i) t.v[i] = targets[i];
        launch("wait_flags", wait_flags_kernel, dim3(1), dim3(32), 0, as_stream(stream),
               reinterpret_cast<const unsigned long long*>(flags), t, static_cast<int>(n),
               static_cast<unsigned long long>(timeout_ns), peer_error_word());
    });
}

}  // extern "C"
