// ============================================================================
//  runtime.cu -- library-wide state: last-error text, device properties,
//  the stream-ordered scratch pool and the kernel launch counter.
// ============================================================================
#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "launch.cuh"

namespace tg {

namespace {
thread_local std::string g_last_error;
thread_local bool g_csr_checks = true;
std::atomic<uint64_t> g_launches{0};
std::mutex g_dev_mu;
std::vector<int> g_sms;           // per device, 0 = not queried yet
std::vector<char> g_pool_ready;   // per device
}  // namespace

void set_last_error(const std::string& m) { g_last_error = m; }

bool csr_checks_enabled() { return g_csr_checks; }

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

static int current_device() {
    int dev = 0;
    TG_CUDA(cudaGetDevice(&dev));
    return dev;
}

int num_sms() {
    const int dev = current_device();
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (static_cast<int>(g_sms.size()) <= dev) g_sms.resize(dev + 1, 0);
    if (!g_sms[dev]) TG_CUDA(cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev));
    return g_sms[dev];
}

SideStream& side_stream() {
    // Per host thread, so concurrent callers never share the events; created
    // on first use and kept for the thread's life (never destroyed: at exit
    // the CUDA context may already be gone).
    thread_local std::vector<SideStream*> per_dev;
    const int dev = current_device();
    if (static_cast<int>(per_dev.size()) <= dev) per_dev.resize(dev + 1, nullptr);
    if (!per_dev[dev]) {
        auto* ss = new SideStream();
        int least = 0, greatest = 0;
        TG_CUDA(cudaDeviceGetStreamPriorityRange(&least, &greatest));
        TG_CUDA(cudaStreamCreateWithPriority(&ss->s, cudaStreamNonBlocking, greatest));
        TG_CUDA(cudaEventCreateWithFlags(&ss->fork, cudaEventDisableTiming));
        TG_CUDA(cudaEventCreateWithFlags(&ss->join, cudaEventDisableTiming));
        per_dev[dev] = ss;
    }
    return *per_dev[dev];
}

// The default pool of each device keeps freed blocks (release threshold =
// max), so scratch reuse across calls costs no new mappings.
static void ensure_pool(int dev) {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (static_cast<int>(g_pool_ready.size()) <= dev) g_pool_ready.resize(dev + 1, 0);
    if (g_pool_ready[dev]) return;
    cudaMemPool_t pool;
    TG_CUDA(cudaDeviceGetDefaultMemPool(&pool, dev));
    uint64_t thr = ~0ull;
    TG_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr));
    g_pool_ready[dev] = 1;
}

void* scratch_alloc(size_t bytes, cudaStream_t s) {
    ensure_pool(current_device());
    void* p = nullptr;
    const cudaError_t e = cudaMallocAsync(&p, bytes, s);
    if (e != cudaSuccess) {
        cudaGetLastError();
        fail(TG_ERR_CUDA, "scratch allocation of " + std::to_string(bytes) +
                              " bytes failed: " + cudaGetErrorString(e));
    }
    return p;
}

void scratch_free(void* p, cudaStream_t s) {
    // Called from destructors: never throws.
    if (cudaFreeAsync(p, s) != cudaSuccess) cudaGetLastError();
}

void require_device() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        fail(TG_ERR_NO_DEVICE,
             "tinygnn_b200: no CUDA device is visible; this library has no CPU path");
    }
}

}  // namespace tg

extern "C" {

TG_API const char* tg_last_error_message(void) { return tg::g_last_error.c_str(); }

TG_API const char* tg_version(void) { return "tinygnn_b200 0.1.0 (sm_100a)"; }

TG_API int32_t tg_abi_version(void) { return 2; }

TG_API int32_t tg_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

TG_API uint64_t tg_kernel_launch_count(void) {
    return tg::g_launches.load(std::memory_order_relaxed);
}

TG_API int32_t tg_set_csr_checks(int32_t enabled) {
    const int32_t prev = tg::g_csr_checks ? 1 : 0;
    tg::g_csr_checks = enabled != 0;
    return prev;
}

}  // extern "C"
