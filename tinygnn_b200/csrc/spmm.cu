// ============================================================================
//  spmm.cu -- CSR row-gather kernels: spmm, SAGE aggregation, degree order.
//
//  Reference: TinyGNN spmm (src/ops.cpp:198-297), SAGE mean/max aggregation
//  (src/layers.cpp:588-637, 674-700), sage_max_aggregate (359-435).
//
//  Layout in HBM: CSR row_ptr/col_ind int32, values fp32; dense operands
//  row-major fp32 with a leading dimension.  A row is owned by a sub-warp of
//  LPR lanes; lane l holds SPL vectors of VEC floats of the output row
//  (features (s*LPR + l)*VEC .. +VEC-1).  The row's col/val are read LPR at a
//  time (coalesced) and broadcast with shuffles; U gathered rows are loaded
//  before their fused multiply-adds are applied in stored order, which keeps
//  U*SPL 4..16-byte loads per lane in flight.  The kernel is HBM-bound: its
//  algorithmic traffic is nnz*(8 + 4F) + M*(4 + 4F) bytes.
// ============================================================================
#include <algorithm>

#include "gather.cuh"
#include "launch.cuh"

namespace tg {

namespace {

template <int V>
struct VecT;
template <>
struct VecT<1> { using T = float; };
template <>
struct VecT<2> { using T = float2; };
template <>
struct VecT<4> { using T = float4; };

template <int V>
__device__ __forceinline__ void ldv(const float* p, float (&x)[V]) {
    if constexpr (V == 4) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(p));
        x[0] = t.x; x[1] = t.y; x[2] = t.z; x[3] = t.w;
    } else if constexpr (V == 2) {
        const float2 t = __ldg(reinterpret_cast<const float2*>(p));
        x[0] = t.x; x[1] = t.y;
    } else {
        x[0] = __ldg(p);
    }
}

template <int V>
__device__ __forceinline__ void stv(float* p, const float (&x)[V]) {
    if constexpr (V == 4) {
        *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
    } else if constexpr (V == 2) {
        *reinterpret_cast<float2*>(p) = make_float2(x[0], x[1]);
    } else {
        p[0] = x[0];
    }
}

template <int OP>
__device__ __forceinline__ float reduce_step(float acc, float w, float h, bool avx_col) {
    if constexpr (OP == GATHER_SUM) {
        return fmaf(w, h, acc);  // acc += w * h, one rounding (reference FMA chain)
    } else {
        // _mm256_max_ps(r, h) on full 8-groups vs std::max(r, h) elsewhere.
        return avx_col ? ((acc > h) ? acc : h) : ((acc < h) ? h : acc);
    }
}

// Kernel: one sub-warp of LPR lanes per output row; gridDim.y feature passes.
template <int VEC, int LPR, int SPL, int OP>
__global__ void __launch_bounds__(256) gather_rows_kernel(const GatherArgs a) {
    constexpr int RPW = 32 / LPR;                 // rows per warp
    constexpr int U = (SPL >= 4) ? 2 : (SPL == 2 ? 4 : 8);  // gathered rows in flight
    const int lane = threadIdx.x & 31;
    const int sub = lane / LPR;
    const int l = lane % LPR;
    const unsigned mask = (LPR == 32) ? 0xffffffffu : (((1u << LPR) - 1u) << (sub * LPR));

    const int64_t slot = (static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW + sub;
    if (slot >= a.M) return;  // whole sub-warps leave together
    const int64_t row = a.order ? static_cast<int64_t>(__ldg(a.order + slot)) : slot;

    const int64_t f0 = static_cast<int64_t>(blockIdx.y) * (LPR * SPL * VEC);  // feature pass
    bool live[SPL], full[SPL];
    int64_t fo[SPL];
#pragma unroll
    for (int s = 0; s < SPL; ++s) {
        fo[s] = f0 + static_cast<int64_t>(s * LPR + l) * VEC;
        live[s] = fo[s] < a.F;          // vector starts inside the row
        full[s] = fo[s] + VEC <= a.F;   // ... and ends inside it (else B is padded)
    }

    float acc[SPL][VEC];
    const float init = (OP == GATHER_SUM) ? 0.0f : -INFINITY;
#pragma unroll
    for (int s = 0; s < SPL; ++s)
#pragma unroll
        for (int k = 0; k < VEC; ++k) acc[s][k] = init;

    bool avx[SPL][VEC];
#pragma unroll
    for (int s = 0; s < SPL; ++s)
#pragma unroll
        for (int k = 0; k < VEC; ++k) avx[s][k] = (fo[s] + k) < a.max_avx_cols;

    const int32_t start = __ldg(a.rp + row);
    const int32_t end = __ldg(a.rp + row + 1);

    for (int32_t base = start; base < end; base += LPR) {
        const int n = min(LPR, end - base);
        int my_c = 0;
        float my_w = 1.0f;
        if (l < n) {
            my_c = __ldg(a.ci + base + l);
            if (a.val) my_w = __ldg(a.val + base + l);
        }
        int e = 0;
        for (; e + U <= n; e += U) {
            int c[U];
            float w[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                c[u] = __shfl_sync(mask, my_c, e + u, LPR);
                w[u] = __shfl_sync(mask, my_w, e + u, LPR);
            }
            float h[U][SPL][VEC];
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int s = 0; s < SPL; ++s)
                    if (live[s]) ldv<VEC>(a.B + static_cast<int64_t>(c[u]) * a.ldb + fo[s], h[u][s]);
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int s = 0; s < SPL; ++s)
                    if (live[s])
#pragma unroll
                        for (int k = 0; k < VEC; ++k)
                            acc[s][k] = reduce_step<OP>(acc[s][k], w[u], h[u][s][k], avx[s][k]);
        }
        for (; e < n; ++e) {
            const int c = __shfl_sync(mask, my_c, e, LPR);
            const float w = __shfl_sync(mask, my_w, e, LPR);
#pragma unroll
            for (int s = 0; s < SPL; ++s)
                if (live[s]) {
                    float h[VEC];
                    ldv<VEC>(a.B + static_cast<int64_t>(c) * a.ldb + fo[s], h);
#pragma unroll
                    for (int k = 0; k < VEC; ++k) acc[s][k] = reduce_step<OP>(acc[s][k], w, h[k], avx[s][k]);
                }
        }
    }

    // Epilogue: (mean) -> (+ self) -> (+ bias) -> activation, each one rounding.
    const int32_t deg = end - start;
    const float inv_deg = (OP == GATHER_SUM && a.mean && deg > 0) ? __fdiv_rn(1.0f, static_cast<float>(deg)) : 1.0f;
#pragma unroll
    for (int s = 0; s < SPL; ++s) {
        if (!live[s]) continue;
        float x[VEC];
        float sv[VEC], bv[VEC];
        if (full[s]) {
            if (a.self) ldv<VEC>(a.self + row * a.lds + fo[s], sv);
            if (a.bias) ldv<VEC>(a.bias + fo[s], bv);
        } else {
#pragma unroll
            for (int k = 0; k < VEC; ++k) {
                const bool in = fo[s] + k < a.F;
                sv[k] = (a.self && in) ? a.self[row * a.lds + fo[s] + k] : 0.0f;
                bv[k] = (a.bias && in) ? a.bias[fo[s] + k] : 0.0f;
            }
        }
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
            float v = acc[s][k];
            if (OP == GATHER_MAX && deg == 0) v = 0.0f;
            if (OP == GATHER_SUM && a.mean && deg > 0) v = __fmul_rn(v, inv_deg);
            if (a.self) v = __fadd_rn(v, sv[k]);
            if (a.bias) v = __fadd_rn(v, bv[k]);
            x[k] = apply_act(a.act, v, a.alpha);
        }
        if (full[s]) {
            stv<VEC>(a.C + row * a.ldc + fo[s], x);
        } else {
#pragma unroll
            for (int k = 0; k < VEC; ++k)
                if (fo[s] + k < a.F) a.C[row * a.ldc + fo[s] + k] = x[k];
        }
    }
}

template <int VEC, int LPR, int SPL>
void launch_gather(const GatherArgs& a, cudaStream_t s) {
    constexpr int RPB = (256 / 32) * (32 / LPR);  // rows per block
    const int64_t per_pass = static_cast<int64_t>(LPR) * SPL * VEC;
    const int64_t passes = ceil_div(a.F, per_pass);
    dim3 grid(static_cast<unsigned>(ceil_div(a.M, RPB)), static_cast<unsigned>(passes));
    if (a.op == GATHER_SUM)
        launch("gather_rows<sum>", gather_rows_kernel<VEC, LPR, SPL, GATHER_SUM>, grid, dim3(256), 0, s, a);
    else
        launch("gather_rows<max>", gather_rows_kernel<VEC, LPR, SPL, GATHER_MAX>, grid, dim3(256), 0, s, a);
}

template <int VEC>
void dispatch_lpr(const GatherArgs& a, cudaStream_t s) {
    const int64_t S = ceil_div(a.F, VEC);  // vector slots per row
    if (S <= 8) launch_gather<VEC, 8, 1>(a, s);
    else if (S <= 16) launch_gather<VEC, 16, 1>(a, s);
    else if (S <= 32) launch_gather<VEC, 32, 1>(a, s);
    else if (S <= 64) launch_gather<VEC, 32, 2>(a, s);
    else launch_gather<VEC, 32, 4>(a, s);  // feature passes of 128 vectors beyond
}

inline bool aligned(const void* p, int bytes) {
    return (reinterpret_cast<uintptr_t>(p) % static_cast<uintptr_t>(bytes)) == 0;
}

}  // namespace

void gather_rows(const GatherArgs& a, cudaStream_t s) {
    if (a.M == 0 || a.F == 0) return;
    // Widest vector that divides F and every leading dimension and keeps
    // every base aligned; narrower when it would leave fewer than 8 vectors.
    int vec = 4;
    auto ok = [&](int v) {
        if ((a.F % v && !a.b_padded) || a.ldb % v || a.ldc % v) return false;
        if (!aligned(a.B, 4 * v) || !aligned(a.C, 4 * v)) return false;
        if (a.self && (a.lds % v || !aligned(a.self, 4 * v))) return false;
        if (a.bias && !aligned(a.bias, 4 * v)) return false;
        return true;
    };
    while (vec > 1 && (!ok(vec) || ceil_div(a.F, vec) < 8)) vec /= 2;
    if (vec == 4) dispatch_lpr<4>(a, s);
    else if (vec == 2) dispatch_lpr<2>(a, s);
    else dispatch_lpr<1>(a, s);
}

// ── Degree order: a stable bucket sort of rows by decreasing length ─────────
// Bucket b(i) = 31 - floor(log2(len_i + 1)) (longest rows in bucket 0..).
// Three passes: per-block bucket counts, one exclusive scan over
// (bucket, block), then a stable scatter (ranks from warp match/popc and
// per-warp prefix counts in shared memory).
namespace {
constexpr int ORDER_BLOCK = 1024;
constexpr int NBUCKET = 32;

__device__ __forceinline__ int row_bucket(const int32_t* rp, int64_t i) {
    const int32_t len = __ldg(rp + i + 1) - __ldg(rp + i);
    return __clz(len + 1);  // len+1 >= 1: 0 for the longest, 31 for empty rows
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
__global__ void order_scan_kernel(int32_t* x, int64_t n) {
    __shared__ int32_t warp_sums[32];
    __shared__ int32_t carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int64_t base = 0; base < n; base += blockDim.x) {
        const int64_t i = base + threadIdx.x;
        const int32_t v = i < n ? x[i] : 0;
        int32_t incl = v;
        const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int32_t t = __shfl_up_sync(0xffffffffu, incl, d);
            if (lane >= d) incl += t;
        }
        if (lane == 31) warp_sums[w] = incl;
        __syncthreads();
        if (w == 0) {
            int32_t ws = lane < (blockDim.x >> 5) ? warp_sums[lane] : 0;
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const int32_t t = __shfl_up_sync(0xffffffffu, ws, d);
                if (lane >= d) ws += t;
            }
            warp_sums[lane] = ws;  // inclusive over warps
        }
        __syncthreads();
        const int32_t warp_off = w ? warp_sums[w - 1] : 0;
        if (i < n) x[i] = carry + warp_off + incl - v;
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) carry += warp_off + incl;
        __syncthreads();
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

void csr_degree_order(int64_t M, const int32_t* rp, int32_t* out, cudaStream_t s) {
    if (M == 0) return;
    const int64_t nb = ceil_div(M, ORDER_BLOCK);
    Scratch<int32_t> counts(static_cast<size_t>(nb) * NBUCKET, s);
    launch("order_count", order_count_kernel, dim3(static_cast<unsigned>(nb)), dim3(ORDER_BLOCK), 0, s, M, rp, counts.p);
    launch("order_scan", order_scan_kernel, dim3(1), dim3(1024), 0, s, counts.p, nb * NBUCKET);
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
        check_ptr("spmm", "col_ind/values", col_ind && values ? col_ind : nullptr, nnz > 0);
        check_ptr("spmm", "B", B, nnz > 0 && F > 0);
        check_ptr("spmm", "C", C, M > 0 && F > 0);
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
        (void)K; (void)nnz;
        if (M < 0 || F < 0) invalid("sage_mean_combine: negative size");
        check_ld("sage_mean_combine", "Tn", ldn, F);
        check_ld("sage_mean_combine", "Ts", lds, F);
        check_ld("sage_mean_combine", "out", ldo, F);
        GatherArgs a;
        a.M = M; a.rp = row_ptr; a.ci = col_ind; a.order = row_order;
        a.B = Tn; a.ldb = ldn; a.F = F; a.self = Ts; a.lds = lds;
        a.C = out; a.ldc = ldo; a.bias = bias; a.act = act; a.op = GATHER_SUM; a.mean = 1;
        a.b_padded = (mode & TG_FLAG_B_ROWS_PADDED) != 0;
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
        (void)K; (void)nnz;
        check_ld("sage_aggregate", "H", ldh, F);
        check_ld("sage_aggregate", "out", ldo, F);
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
        (void)K; (void)nnz;
        check_ld("sage_max_aggregate", "H", ldh, F);
        check_ld("sage_max_aggregate", "out", ldo, F);
        GatherArgs a;
        a.M = M; a.rp = row_ptr; a.ci = col_ind; a.B = H; a.ldb = ldh; a.F = F;
        a.C = out; a.ldc = ldo; a.op = GATHER_MAX;
        a.max_avx_cols = (F / 8) * 8;  // AVX2 body on full groups of 8 (layers.cpp:411-416)
        gather_rows(a, as_stream(stream));
    });
}

}  // extern "C"
