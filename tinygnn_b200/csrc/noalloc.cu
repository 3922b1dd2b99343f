// ============================================================================
//  noalloc.cu -- a GCN layer forward that allocates no device memory.
//
//  Some callers cannot let a library allocate: real-time serving loops that
//  must not call cudaMalloc/cudaMallocAsync after start-up (an allocation can
//  block on the driver and break the latency budget), and host runtimes that
//  own all device memory through their own allocator and forbid
//  library-side allocations.  tg_gcn_layer_f32 needs an N x F_out scratch
//  for H.W (taken from the stream-ordered pool); this variant keeps that
//  intermediate in a fixed array in the library's own device memory instead.
//
//  The array is a file-scope __device__ variable of TG_NOALLOC_SCRATCH_BYTES
//  (16 MiB).  Every GPU that loads the library holds it until the process
//  exits.  Host code cannot use the variable's name as a device address (in
//  host code it names a host-side stand-in), so each device's address is
//  looked up once with cudaGetSymbolAddress, with that device current, on
//  the first call made on that device.
// ============================================================================
#include <mutex>
#include <vector>

#include "gather.cuh"
#include "launch.cuh"

namespace tg {

void gemm_exact(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb,
                float* C, int64_t ldc, const float* bias, int act, float alpha, cudaStream_t s);

namespace {

static __device__ __align__(256) float g_noalloc_scratch[TG_NOALLOC_SCRATCH_BYTES / sizeof(float)];
// The input CSR check's result words (the allocating entry points take them
// from the pool).
static __device__ __align__(256) unsigned long long g_noalloc_check[kCsrCheckWordsBytes / 8];

struct Addresses {
    float* scratch = nullptr;
    void* check = nullptr;
};
std::mutex g_mu;
std::vector<Addresses> g_addr;  // per device; nullptr = not looked up yet

void* symbol_address(const void* sym) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, sym);
    if (e != cudaSuccess) {
        cudaGetLastError();
        fail(TG_ERR_CUDA, std::string("gcn_layer (no-alloc): cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
    }
    return p;
}

// The fixed arrays' device addresses on the current device.
Addresses addresses() {
    int dev = 0;
    TG_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(g_mu);
    if (static_cast<int>(g_addr.size()) <= dev) g_addr.resize(dev + 1);
    if (!g_addr[dev].scratch) {
        Addresses a;
        a.scratch = static_cast<float*>(symbol_address(g_noalloc_scratch));
        a.check = symbol_address(g_noalloc_check);
        g_addr[dev] = a;
    }
    return g_addr[dev];
}

}  // namespace

}  // namespace tg

using namespace tg;

extern "C" {

TG_API tg_status tg_gcn_layer_noalloc_f32(int64_t N, int64_t nnz, const int32_t* row_ptr, const int32_t* col_ind,
                                          const float* values, const float* H, int64_t ldh, int64_t F_in,
                                          int64_t F_out, const float* W, const float* bias, int32_t act, float* out,
                                          int64_t ldo, const int32_t* row_order, void* stream) {
    return guard([&] {
        require_device();
        if (nnz < 0) invalid("GCNLayer::forward: negative nnz");
        if (F_in <= 0) invalid("GCNLayer: in_features must be > 0.");
        if (F_out <= 0) invalid("GCNLayer: out_features must be > 0.");
        if (N < 0) invalid("GCNLayer::forward: negative node count");
        check_ld("GCNLayer::forward", "H", ldh, F_in);
        check_ld("GCNLayer::forward", "out", ldo, F_out);
        // Limits are checked by division first, so that no product below can
        // overflow: F_out and N are each bounded by the array's size.
        constexpr int64_t cap_floats = static_cast<int64_t>(TG_NOALLOC_SCRATCH_BYTES / sizeof(float));
        const int64_t ldw = F_out <= cap_floats ? (F_out + 3) / 4 * 4 : cap_floats + 1;
        if (ldw > cap_floats || N > cap_floats / ldw)
            invalid("gcn_layer (no-alloc): N x F_out = " + std::to_string(N) + " x " + std::to_string(F_out) +
                    " needs more than the " + std::to_string(static_cast<long long>(TG_NOALLOC_SCRATCH_BYTES)) +
                    " bytes the fixed scratch holds (N * round_up(F_out, 4) * 4 bytes; use tg_gcn_layer_f32, "
                    "which allocates)");
        if (N == 0) return;
        const cudaStream_t s = as_stream(stream);
        const Addresses fixed = addresses();
        check_csr_input(N, N, nnz, row_ptr, col_ind, s, row_order, fixed.check);
        float* HW = fixed.scratch;
        // Every element the gather reads is written by this GEMM first, so
        // nothing carried over from an earlier call needs clearing.
        gemm_exact(N, F_out, F_in, H, ldh, W, F_out, HW, ldw, nullptr, TG_ACT_NONE, 0.0f, s);
        GatherArgs a;
        a.M = N; a.rp = row_ptr; a.ci = col_ind; a.val = values; a.order = row_order;
        a.B = HW; a.ldb = ldw; a.b_padded = true; a.F = F_out;
        a.C = out; a.ldc = ldo; a.bias = bias; a.act = act; a.op = GATHER_SUM;
        a.allow_auto_order = false;  // a schedule would need pool memory
        a.allow_heavy = false;       // so would the hub-row kernel's counter and side stream
        gather_rows(a, s);
    });
}

}  // extern "C"
