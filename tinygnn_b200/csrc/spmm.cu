// ============================================================================
//  spmm.cu -- CSR row-gather entry points: spmm, SAGE aggregation, the
//  transform-first SAGE combine, and the degree-ordered row schedule.
//
//  Reference: TinyGNN spmm (src/ops.cpp:198-297), SAGE mean/max aggregation
//  (src/layers.cpp:588-637, 674-700), sage_max_aggregate (359-435).
//
//  Layout in HBM: CSR row_ptr/col_ind int32, values fp32; dense operands
//  row-major fp32 with a leading dimension.  The kernel (gather_kernel.cuh)
//  is HBM/L2-bound: algorithmic traffic nnz*(8 + 4F) + M*(4 + 4F) bytes for
//  spmm (nnz*(4 + 4F) + ... without values).
// ============================================================================
#include <algorithm>
#include <cstdlib>
#include <memory>
#include <mutex>
#include <vector>

#include "gather.cuh"
#include "gather_heavy.cuh"
#include "gather_kernel.cuh"
#include "launch.cuh"

namespace tg {

namespace {

// Row count from which a gather without a schedule computes a degree order.
constexpr int64_t kAutoOrderRows = 16384;

inline bool aligned(const void* p, int bytes) {
    return (reinterpret_cast<uintptr_t>(p) % static_cast<uintptr_t>(bytes)) == 0;
}

template <int VEC, int LPR, int SPL, bool CVEC>
void launch_gather(const GatherArgs& a, cudaStream_t s) {
    constexpr int RPB = (256 / 32) * (32 / LPR);  // rows per block
    // Gathered rows in flight per batch (sweep on the Reddit-shaped graph,
    // degree-ordered: 4 for 32-lane rows, 8 for narrower ones).
    constexpr int U = (SPL >= 4) ? 2 : (SPL == 2 ? 4 : (LPR == 32 ? 4 : 8));
    const int64_t per_pass = static_cast<int64_t>(LPR) * SPL * VEC;
    const int64_t passes = ceil_div(a.F, per_pass);
    dim3 grid(static_cast<unsigned>(ceil_div(a.M, RPB)), static_cast<unsigned>(passes));
    if (a.op == GATHER_SUM)
        launch("gather_rows<sum>", gk::gather_rows_kernel<VEC, LPR, SPL, GATHER_SUM, U, CVEC>, grid, dim3(256), 0,
               s, a);
    else
        launch("gather_rows<max>", gk::gather_rows_kernel<VEC, LPR, SPL, GATHER_MAX, U, CVEC>, grid, dim3(256), 0,
               s, a);
}

// Lanes per row (LPR) x vectors per lane (SPL) for a row of S vector slots.
// Each load instruction should cover few 128-byte lines: the L1TEX data
// pipe's wavefronts, not the idle lanes, bound the narrow gathers.  Measured
// on the Reddit-shaped layer-2 gather (41-float rows, 11 float4 slots): 16
// lanes x 1 vector (two rows per instruction, 5 of 16 lanes idle) 1.75 ms;
// 4 lanes x 3 vectors (eight rows per instruction, 11 of 12 slots busy)
// 2.25 ms -- each instruction touched ~12 lines for 512 bytes.
template <int VEC, bool CVEC>
void dispatch_lpr(const GatherArgs& a, cudaStream_t s) {
    const int64_t S = ceil_div(a.F, VEC);  // vector slots per row
    if (S <= 4) launch_gather<VEC, 4, 1, CVEC>(a, s);
    else if (S <= 8) launch_gather<VEC, 8, 1, CVEC>(a, s);
    else if (S <= 16) launch_gather<VEC, 16, 1, CVEC>(a, s);
    else if (S <= 32) launch_gather<VEC, 32, 1, CVEC>(a, s);
    else if (S <= 64) launch_gather<VEC, 32, 2, CVEC>(a, s);
    else launch_gather<VEC, 32, 4, CVEC>(a, s);  // feature passes of 128 vectors beyond
}

template <int VEC>
void dispatch_cvec(const GatherArgs& a, cudaStream_t s) {
    bool cvec = a.ldc % VEC == 0 && aligned(a.C, 4 * VEC);
    if (a.self) cvec = cvec && a.lds % VEC == 0 && aligned(a.self, 4 * VEC);
    if (a.bias) cvec = cvec && aligned(a.bias, 4 * VEC);
    if (cvec) dispatch_lpr<VEC, true>(a, s);
    else dispatch_lpr<VEC, false>(a, s);
}

// ── Heavy rows ───────────────────────────────────────────────────────────
// The first slots of a schedule whose rows are long enough to be the
// launch's critical path go to the heavy-row kernel (gather_heavy.cuh) on
// the side stream, beside the sub-warp kernel.  heavy_prefix_kernel counts
// them on the device (threshold from the nnz) among the first kHeavyScan
// slots.  TINYGNN_B200_HEAVY_MIN_LEN sets a fixed threshold instead (a
// negative value below -1 turns the heavy kernel off).
constexpr int64_t kHeavyScan = 16384;

__device__ int g_gather_error = 0;  // first heavy-kernel timeout code (0 = none)

// -1: threshold from the nnz; >= 0: fixed; < -1: heavy kernel off.
int32_t heavy_min_len() {
    static const int32_t v = [] {
        const char* e = std::getenv("TINYGNN_B200_HEAVY_MIN_LEN");
        return e ? static_cast<int32_t>(std::atoi(e)) : -1;
    }();
    return v;
}

int* gather_error_word() {
    static std::mutex mu;
    static std::vector<int*> words;
    int dev = 0;
    TG_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(mu);
    if (static_cast<int>(words.size()) <= dev) words.resize(dev + 1, nullptr);
    if (!words[dev]) TG_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&words[dev]), g_gather_error));
    return words[dev];
}

template <int OP>
void launch_heavy_t(const GatherArgs& a, int passes, int64_t groups, cudaStream_t s) {
    auto kern = gk::gather_heavy_kernel<OP>;
    const size_t smem = sizeof(gk::HeavySmem);
    TG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    launch("gather_heavy", kern, dim3(static_cast<unsigned>(passes * groups)), dim3(gk::kHeavyThreads), smem, s, a,
           passes, gather_error_word());
}

// One CTA per (row group, 32-feature slice); all of them resident at once.
void launch_heavy(const GatherArgs& a, cudaStream_t s) {
    const int passes = static_cast<int>(ceil_div(a.F, gk::kHeavySlice));
    const int64_t resident = static_cast<int64_t>(gk::kHeavyCtasPerSm) * num_sms();
    const int64_t groups = std::max<int64_t>(1, std::min<int64_t>(std::min(kHeavyScan, a.M), resident / passes));
    if (a.op == GATHER_SUM) launch_heavy_t<GATHER_SUM>(a, passes, groups, s);
    else launch_heavy_t<GATHER_MAX>(a, passes, groups, s);
}

void dispatch_light(const GatherArgs& a, cudaStream_t s) {
    // Load width: the widest vector dividing B's leading dimension with B
    // aligned, and dividing F unless B's rows are padded; narrower when it
    // would leave fewer than 4 vectors per row (the narrowest sub-warp).
    auto ok = [&](int v) {
        if (a.F % v && !a.b_padded) return false;
        return a.ldb % v == 0 && aligned(a.B, 4 * v);
    };
    int vec = 4;
    while (vec > 1 && (!ok(vec) || ceil_div(a.F, vec) < 4)) vec /= 2;
    if (vec == 4) dispatch_cvec<4>(a, s);
    else if (vec == 2) dispatch_cvec<2>(a, s);
    else dispatch_cvec<1>(a, s);
}

}  // namespace

void csr_degree_order(int64_t M, const int32_t* rp, int32_t* out, cudaStream_t s);

// Reads and clears the heavy-row kernel's error word (synchronises `s`).
int gather_take_error(cudaStream_t s) {
    int h = 0;
    TG_CUDA(cudaStreamSynchronize(s));
    TG_CUDA(cudaMemcpyFromSymbol(&h, g_gather_error, sizeof(int)));
    if (h) {
        const int zero = 0;
        TG_CUDA(cudaMemcpyToSymbol(g_gather_error, &zero, sizeof(int)));
    }
    return h;
}

void gather_rows(const GatherArgs& args, cudaStream_t s) {
    if (args.M == 0 || args.F == 0) return;
    GatherArgs a = args;
    // Without a caller-given schedule, large launches start their longest
    // rows first: a hub row left to the end of the grid is a serial tail
    // (measured 5.8 -> 3.7 ms on the Reddit-shaped layer-1 gather).
    std::unique_ptr<Scratch<int32_t>> order;
    if (!a.order && a.allow_auto_order && a.M >= kAutoOrderRows) {
        order.reset(new Scratch<int32_t>(static_cast<size_t>(a.M), s));
        csr_degree_order(a.M, a.rp, order->p, s);
        a.order = order->p;
    }
    // Long rows go to the heavy-row kernel on the side stream, launched
    // first so its CTAs are placed before the sub-warp kernel's.
    const int32_t minlen = heavy_min_len();
    const bool heavy = a.allow_heavy && a.order && minlen >= -1 && a.ldb % 4 == 0 && aligned(a.B, 16);
    SideStream* side = nullptr;
    std::unique_ptr<Scratch<int32_t>> count;
    if (heavy) {
        count.reset(new Scratch<int32_t>(1, s));
        launch("heavy_prefix", gk::heavy_prefix_kernel, dim3(1), dim3(gk::kHeavyScanThreads), 0, s, a.M, a.rp,
               a.order, std::min(kHeavyScan, a.M), minlen, count->p);
        a.heavy_count = count->p;
        side = &side_stream();
        TG_CUDA(cudaEventRecord(side->fork, s));
        TG_CUDA(cudaStreamWaitEvent(side->s, side->fork, 0));
        launch_heavy(a, side->s);
        TG_CUDA(cudaEventRecord(side->join, side->s));
    }
    dispatch_light(a, s);
    if (side) TG_CUDA(cudaStreamWaitEvent(s, side->join, 0));
}

// ── Degree order: a stable bucket sort of rows by decreasing length ─────────
// Length classes, longest first: four per power of two -- x = len + 1 falls
// in [2^k, 2^(k+1)), and the two bits below its leading one split that range
// into quarters.  Rows that share a warp (up to 8 in the narrow gathers) then
// differ in length by at most ~25 % within a class.  Every class boundary
// 2^k - 1 stays a boundary, so the rows of at least 2^k - 1 entries lead the
// schedule (the hub-row prefix relies on it).  Three passes: per-block class
// counts, one exclusive scan over (class, block), then a stable scatter
// (ranks from warp match/popc and per-warp prefix counts in shared memory).
namespace {
constexpr int ORDER_BLOCK = 1024;
constexpr int NBUCKET = 128;

__device__ __forceinline__ int row_bucket(const int32_t* rp, int64_t i) {
    const uint32_t x = static_cast<uint32_t>(__ldg(rp + i + 1) - __ldg(rp + i)) + 1u;  // >= 1
    const int lz = __clz(x);                     // 0 for the longest rows, 31 for empty ones
    const uint32_t q = (x << lz) >> 29 & 3u;     // the two bits below the leading one
    return lz * 4 + 3 - static_cast<int>(q);     // 0 .. 127
}

__global__ void order_count_kernel(int64_t M, const int32_t* rp, int32_t* counts /*[NBUCKET][nblocks]*/) {
    __shared__ int32_t c[NBUCKET];
    if (threadIdx.x < NBUCKET) c[threadIdx.x] = 0;
    __syncthreads();
    const int64_t i = static_cast<int64_t>(blockIdx.x) * ORDER_BLOCK + threadIdx.x;
    if (i < M) atomicAdd(&c[row_bucket(rp, i)], 1);
    __syncthreads();
    if (threadIdx.x < NBUCKET) counts[static_cast<int64_t>(threadIdx.x) * gridDim.x + blockIdx.x] = c[threadIdx.x];
}

// Single-block exclusive scan over n ints, in place (n = NBUCKET * nblocks).
// Thread t owns one contiguous run of ceil(n / blockDim) entries: it sums
// its run, the block scans the 1024 run sums once (warp shuffles, then the
// warp totals), and each thread writes its run's prefixes.  With SMEM the
// counts are staged through shared memory with coalesced loads and stores
// (the runs are then read at an odd stride: no bank conflicts); a run read
// straight from global memory is a chain of dependent-latency loads (~25 us
// for the Reddit-shaped graph's 29,184 counts).
template <bool SMEM>
__global__ void order_scan_kernel(int32_t* x, int64_t n) {
    extern __shared__ int32_t sx[];
    __shared__ int32_t warp_sums[32];
    int32_t* v = x;
    if (SMEM) {
        for (int64_t i = threadIdx.x; i < n; i += blockDim.x) sx[i] = x[i];
        __syncthreads();
        v = sx;
    }
    const int64_t per = (n + blockDim.x - 1) / blockDim.x;
    const int64_t b = static_cast<int64_t>(threadIdx.x) * per;
    const int64_t e = b + per < n ? b + per : n;
    int32_t sum = 0;
    for (int64_t i = b; i < e; ++i) sum += v[i];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int32_t incl = sum;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int32_t t = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += t;
    }
    if (lane == 31) warp_sums[w] = incl;
    __syncthreads();
    if (w == 0) {
        int32_t ws = lane < static_cast<int>(blockDim.x >> 5) ? warp_sums[lane] : 0;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int32_t t = __shfl_up_sync(0xffffffffu, ws, d);
            if (lane >= d) ws += t;
        }
        warp_sums[lane] = ws;  // inclusive over warps
    }
    __syncthreads();
    int32_t run = (w ? warp_sums[w - 1] : 0) + incl - sum;  // exclusive prefix of this thread's run
    for (int64_t i = b; i < e; ++i) {
        const int32_t c = v[i];
        v[i] = run;
        run += c;
    }
    if (SMEM) {
        __syncthreads();
        for (int64_t i = threadIdx.x; i < n; i += blockDim.x) x[i] = sx[i];
    }
}

__global__ void order_scatter_kernel(int64_t M, const int32_t* rp, const int32_t* offsets, int32_t* out) {
    __shared__ int32_t wc[ORDER_BLOCK / 32][NBUCKET];  // per-warp bucket counts -> exclusive prefix
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    for (int k = threadIdx.x; k < (ORDER_BLOCK / 32) * NBUCKET; k += blockDim.x) (&wc[0][0])[k] = 0;
    __syncthreads();
    const int64_t i = static_cast<int64_t>(blockIdx.x) * ORDER_BLOCK + threadIdx.x;
    const bool valid = i < M;
    const int b = valid ? row_bucket(rp, i) : NBUCKET;  // NBUCKET = no bucket
    const unsigned peers = __match_any_sync(0xffffffffu, b);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (valid && rank == 0) wc[w][b] = __popc(peers);
    __syncthreads();
    if (threadIdx.x < NBUCKET) {  // prefix over warps, per bucket
        int32_t run = 0;
        for (int ww = 0; ww < ORDER_BLOCK / 32; ++ww) {
            const int32_t t = wc[ww][threadIdx.x];
            wc[ww][threadIdx.x] = run;
            run += t;
        }
    }
    __syncthreads();
    if (valid) {
        const int64_t dst = static_cast<int64_t>(offsets[static_cast<int64_t>(b) * gridDim.x + blockIdx.x]) + wc[w][b] + rank;
        out[dst] = static_cast<int32_t>(i);
    }
}
}  // namespace

// splits[q*M + i] = first entry of row i with column >= q*width (rows sorted
// by column); splits[0*M + i] = row_ptr[i], splits[nb*M + i] = row_ptr[i+1].
__global__ void column_splits_kernel(int64_t M, const int32_t* rp, const int32_t* ci, int nb, int64_t width,
                                     int32_t* out) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= M * (nb + 1)) return;
    const int q = static_cast<int>(t / M);
    const int64_t i = t % M;
    int32_t lo = rp[i], hi = rp[i + 1];
    if (q == 0) { out[t] = lo; return; }
    if (q == nb) { out[t] = hi; return; }
    const int64_t key = static_cast<int64_t>(q) * width;
    while (lo < hi) {  // lower_bound
        const int32_t mid = lo + (hi - lo) / 2;
        if (static_cast<int64_t>(ci[mid]) < key) lo = mid + 1;
        else hi = mid;
    }
    out[t] = lo;
}

void csr_degree_order(int64_t M, const int32_t* rp, int32_t* out, cudaStream_t s) {
    if (M == 0) return;
    const int64_t nb = ceil_div(M, ORDER_BLOCK);
    Scratch<int32_t> counts(static_cast<size_t>(nb) * NBUCKET, s);
    launch("order_count", order_count_kernel, dim3(static_cast<unsigned>(nb)), dim3(ORDER_BLOCK), 0, s, M, rp, counts.p);
    const int64_t n = nb * NBUCKET;
    constexpr int64_t kScanSmemMax = 200 * 1024;  // counts staged through shared memory up to this size
    if (n * 4 <= kScanSmemMax) {
        const int smem = static_cast<int>(n * 4);
        TG_CUDA(cudaFuncSetAttribute(order_scan_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        launch("order_scan", order_scan_kernel<true>, dim3(1), dim3(1024), static_cast<size_t>(smem), s, counts.p, n);
    } else {
        launch("order_scan", order_scan_kernel<false>, dim3(1), dim3(1024), 0, s, counts.p, n);
    }
    launch("order_scatter", order_scatter_kernel, dim3(static_cast<unsigned>(nb)), dim3(ORDER_BLOCK), 0, s, M, rp,
           static_cast<const int32_t*>(counts.p), out);
}

}  // namespace tg

// ── C ABI ───────────────────────────────────────────────────────────────────
using namespace tg;

extern "C" {

TG_API tg_status tg_spmm_f32(int64_t M, int64_t K, int64_t nnz, const int32_t* row_ptr,
                             const int32_t* col_ind, const float* values, const float* B,
                             int64_t F, int64_t ldb, float* C, int64_t ldc, const float* bias,
                             int32_t act, float alpha, const int32_t* row_order, int32_t mode,
                             void* stream) {
    return guard([&] {
        require_device();
        if (M < 0 || K < 0 || F < 0 || nnz < 0) invalid("spmm: negative size");
        check_ld("spmm", "B", ldb, F);
        check_ld("spmm", "C", ldc, F);
        check_ptr("spmm", "row_ptr", row_ptr, M > 0);
        check_ptr("spmm", "col_ind", col_ind, nnz > 0);  // values == NULL: every entry 1.0
        check_ptr("spmm", "B", B, nnz > 0 && F > 0);
        check_ptr("spmm", "C", C, M > 0 && F > 0);
        check_csr_input(M, K, nnz, row_ptr, col_ind, as_stream(stream), row_order);
        GatherArgs a;
        a.M = M; a.rp = row_ptr; a.ci = col_ind; a.val = values; a.order = row_order;
        a.B = B; a.ldb = ldb; a.F = F; a.C = C; a.ldc = ldc;
        a.bias = bias; a.act = act; a.alpha = alpha; a.op = GATHER_SUM;
        a.b_padded = (mode & TG_FLAG_B_ROWS_PADDED) != 0;
        gather_rows(a, as_stream(stream));
    });
}

TG_API tg_status tg_sage_mean_combine_f32(int64_t M, int64_t K, int64_t nnz, const int32_t* row_ptr,
                                          const int32_t* col_ind, const float* Tn, int64_t F, int64_t ldn,
                                          const float* Ts, int64_t lds, const float* bias, int32_t act, float* out,
                                          int64_t ldo, const int32_t* row_order, int32_t mode, void* stream) {
    return guard([&] {
        require_device();
        if (M < 0 || F < 0) invalid("sage_mean_combine: negative size");
        check_ld("sage_mean_combine", "Tn", ldn, F);
        check_ld("sage_mean_combine", "Ts", lds, F);
        check_ld("sage_mean_combine", "out", ldo, F);
        check_csr_input(M, K, nnz, row_ptr, col_ind, as_stream(stream), row_order);
        GatherArgs a;
        a.M = M; a.rp = row_ptr; a.ci = col_ind; a.order = row_order;
        a.B = Tn; a.ldb = ldn; a.F = F; a.self = Ts; a.lds = lds;
        a.C = out; a.ldc = ldo; a.bias = bias; a.act = act; a.op = GATHER_SUM; a.mean = 1;
        a.b_padded = (mode & TG_FLAG_B_ROWS_PADDED) != 0;
        gather_rows(a, as_stream(stream));
    });
}

TG_API tg_status tg_csr_column_splits(int64_t M, const int32_t* row_ptr, const int32_t* col_ind, int32_t nblocks,
                                      int64_t width, int32_t* splits_out, void* stream) {
    return guard([&] {
        require_device();
        if (M < 0 || nblocks < 1 || width < 1) invalid("csr_column_splits: need M >= 0, nblocks >= 1, width >= 1");
        const int64_t total = M * (nblocks + 1);
        if (total == 0) return;
        check_csr_input(M, -1, -1, row_ptr, col_ind, as_stream(stream));  // columns only compared
        launch("column_splits", column_splits_kernel, dim3(static_cast<unsigned>(ceil_div(total, 256))), dim3(256), 0,
               as_stream(stream), M, row_ptr, col_ind, static_cast<int>(nblocks), width, splits_out);
    });
}

TG_API tg_status tg_spmm_segment_f32(int64_t M, int64_t K, const int32_t* row_ptr, const int32_t* col_ind,
                                     const float* values, const int32_t* seg_begin, const int32_t* seg_end,
                                     const float* B, int64_t F, int64_t ldb, float* C, int64_t ldc, const float* bias,
                                     int32_t act, float alpha, const int32_t* row_order, int32_t carry, int32_t last,
                                     int32_t mode, void* stream) {
    return guard([&] {
        require_device();
        if (M < 0 || F < 0) invalid("spmm_segment: negative size");
        check_ld("spmm_segment", "B", ldb, F);
        check_ld("spmm_segment", "C", ldc, F);
        check_ptr("spmm_segment", "seg_begin/seg_end", seg_begin && seg_end ? seg_begin : nullptr, M > 0);
        check_csr_input(M, K, -1, row_ptr, col_ind, as_stream(stream), row_order);
        GatherArgs a;
        a.M = M; a.rp = row_ptr; a.ci = col_ind; a.val = values; a.order = row_order;
        a.B = B; a.ldb = ldb; a.F = F; a.C = C; a.ldc = ldc;
        a.bias = bias; a.act = act; a.alpha = alpha; a.op = GATHER_SUM;
        a.b_padded = (mode & TG_FLAG_B_ROWS_PADDED) != 0;
        a.seg_lo = seg_begin; a.seg_hi = seg_end; a.carry = carry != 0; a.last = last != 0;
        gather_rows(a, as_stream(stream));
    });
}

TG_API tg_status tg_sage_mean_combine_segment_f32(int64_t M, int64_t K, const int32_t* row_ptr,
                                                  const int32_t* col_ind, const int32_t* seg_begin,
                                                  const int32_t* seg_end, const float* Tn, int64_t F, int64_t ldn,
                                                  const float* Ts, int64_t lds, const float* bias, int32_t act,
                                                  float* out, int64_t ldo, const int32_t* row_order, int32_t carry,
                                                  int32_t last, int32_t mode, void* stream) {
    return guard([&] {
        require_device();
        if (M < 0 || F < 0) invalid("sage_mean_combine_segment: negative size");
        check_ld("sage_mean_combine_segment", "Tn", ldn, F);
        check_ld("sage_mean_combine_segment", "Ts", lds, F);
        check_ld("sage_mean_combine_segment", "out", ldo, F);
        check_csr_input(M, K, -1, row_ptr, col_ind, as_stream(stream), row_order);
        GatherArgs a;
        a.M = M; a.rp = row_ptr; a.ci = col_ind; a.order = row_order;
        a.B = Tn; a.ldb = ldn; a.F = F; a.self = Ts; a.lds = lds;
        a.C = out; a.ldc = ldo; a.bias = bias; a.act = act; a.op = GATHER_SUM; a.mean = 1;
        a.b_padded = (mode & TG_FLAG_B_ROWS_PADDED) != 0;
        a.seg_lo = seg_begin; a.seg_hi = seg_end; a.carry = carry != 0; a.last = last != 0;
        gather_rows(a, as_stream(stream));
    });
}

TG_API tg_status tg_gcn_aggregate_f32(int64_t M, int64_t K, int64_t nnz, const int32_t* row_ptr,
                                      const int32_t* col_ind, const float* values, const float* Hs, int64_t F,
                                      int64_t ldh, const float* Hs_self, int64_t lds, const float* dis,
                                      const float* bias, int32_t act, float* out, int64_t ldo,
                                      const int32_t* row_order, const int32_t* seg_begin, const int32_t* seg_end,
                                      int32_t carry, int32_t last, int32_t mode, void* stream) {
    return guard([&] {
        require_device();
        if (M < 0 || K < 0 || F < 0 || nnz < 0) invalid("gcn_aggregate: negative size");
        check_ld("gcn_aggregate", "Hs", ldh, F);
        check_ld("gcn_aggregate", "Hs_self", lds, F);
        check_ld("gcn_aggregate", "out", ldo, F);
        check_ptr("gcn_aggregate", "row_ptr/Hs_self/dis/out", row_ptr && Hs_self && dis && out ? row_ptr : nullptr,
                  M > 0 && F > 0);
        check_ptr("gcn_aggregate", "col_ind/Hs", col_ind && Hs ? col_ind : nullptr, nnz > 0 && F > 0);  // values may be NULL
        if ((seg_begin == nullptr) != (seg_end == nullptr)) invalid("gcn_aggregate: seg_begin and seg_end go together");
        // with segments the CSR may be a row-offset view: its entry count is row_ptr[M]
        check_csr_input(M, K, seg_begin ? -1 : nnz, row_ptr, col_ind, as_stream(stream), row_order);
        GatherArgs a;
        a.M = M; a.rp = row_ptr; a.ci = col_ind; a.val = values; a.order = row_order;
        a.B = Hs; a.ldb = ldh; a.F = F; a.C = out; a.ldc = ldo;
        a.self = Hs_self; a.lds = lds; a.row_scale = dis;
        a.bias = bias; a.act = act; a.op = GATHER_SUM;
        a.b_padded = (mode & TG_FLAG_B_ROWS_PADDED) != 0;
        a.seg_lo = seg_begin; a.seg_hi = seg_end; a.carry = carry != 0; a.last = last != 0;
        gather_rows(a, as_stream(stream));
    });
}

TG_API tg_status tg_csr_degree_order(int64_t M, const int32_t* row_ptr, int32_t* order_out,
                                     void* stream) {
    return guard([&] {
        require_device();
        if (M < 0) invalid("csr_degree_order: negative size");
        check_ptr("csr_degree_order", "row_ptr/order_out", row_ptr && order_out ? row_ptr : nullptr, M > 0);
        csr_degree_order(M, row_ptr, order_out, as_stream(stream));
    });
}

TG_API tg_status tg_sage_aggregate_f32(int64_t M, int64_t K, int64_t nnz,
                                       const int32_t* row_ptr, const int32_t* col_ind,
                                       const float* H, int64_t F, int64_t ldh, float* out,
                                       int64_t ldo, int32_t aggregator, void* stream) {
    return guard([&] {
        require_device();
        if (M < 0 || F < 0) invalid("sage_aggregate: negative size");
        check_ld("sage_aggregate", "H", ldh, F);
        check_ld("sage_aggregate", "out", ldo, F);
        check_csr_input(M, K, nnz, row_ptr, col_ind, as_stream(stream));
        GatherArgs a;
        a.M = M; a.rp = row_ptr; a.ci = col_ind; a.B = H; a.ldb = ldh; a.F = F;
        a.C = out; a.ldc = ldo;
        if (aggregator == TG_AGG_MAX) {
            a.op = GATHER_MAX;
            a.max_avx_cols = 0;  // SAGELayer Max uses std::max on every column
        } else {
            a.op = GATHER_SUM;
            a.mean = 1;
        }
        gather_rows(a, as_stream(stream));
    });
}

TG_API tg_status tg_sage_max_aggregate_f32(int64_t M, int64_t K, int64_t nnz,
                                           const int32_t* row_ptr, const int32_t* col_ind,
                                           const float* H, int64_t F, int64_t ldh, float* out,
                                           int64_t ldo, void* stream) {
    return guard([&] {
        require_device();
        if (M < 0 || F < 0) invalid("sage_max_aggregate: negative size");
        check_ld("sage_max_aggregate", "H", ldh, F);
        check_ld("sage_max_aggregate", "out", ldo, F);
        check_csr_input(M, K, nnz, row_ptr, col_ind, as_stream(stream));
        GatherArgs a;
        a.M = M; a.rp = row_ptr; a.ci = col_ind; a.B = H; a.ldb = ldh; a.F = F;
        a.C = out; a.ldc = ldo; a.op = GATHER_MAX;
        a.max_avx_cols = (F / 8) * 8;  // AVX2 body on full groups of 8 (layers.cpp:411-416)
        gather_rows(a, as_stream(stream));
    });
}

}  // extern "C"
