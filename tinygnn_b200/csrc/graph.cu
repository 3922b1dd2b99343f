// ============================================================================
//  graph.cu -- bit-exact graph construction on the device.
//
//  edge_list_to_csr   GraphLoader::edge_list_to_csr, src/graph_loader.cpp:211-281
//  add_self_loops     src/layers.cpp:71-144
//  gcn_norm           src/layers.cpp:158-208
//  csr_validate       Tensor::sparse_csr checks, src/tensor.cpp:46-86
//
//  The CSR build is count (atomic histogram) -> exclusive scan -> scatter
//  through per-row cursors -> per-row sort.  Rows are sorted by size class:
//  <= 32 entries in one warp (register bitonic network), <= 32768 in one CTA
//  (shared-memory bitonic sort), longer rows by a counting sort over the
//  column range.  Values are plain integers with no payload, so the result is
//  identical to the reference's std::sort whatever the scatter order.
//
//  gcn_norm and add_self_loops give one warp per row: the diagonal search and
//  the insertion point are warp ballots, the degree is the reference's
//  sequential float sum (every lane folds the row in stored order), and the
//  scale is (v * dis_i) * dis_j with IEEE division and square root.
// ============================================================================
#include <algorithm>
#include <climits>
#include <memory>
#include <vector>

#include "launch.cuh"

namespace tg {

void inclusive_scan_i32(int32_t* x, int64_t n, cudaStream_t s);

namespace {

// ── Scan: per-block inclusive scan + block sums, one-block scan of sums, add ─
constexpr int SCAN_T = 1024;
constexpr int SCAN_PER = 4;
constexpr int SCAN_TILE = SCAN_T * SCAN_PER;

__device__ __forceinline__ int32_t block_inclusive(int32_t v, int32_t* warp_tot) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int32_t t = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += t;
    }
    if (lane == 31) warp_tot[w] = v;
    __syncthreads();
    if (w == 0) {
        int32_t t = lane < static_cast<int>(blockDim.x >> 5) ? warp_tot[lane] : 0;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int32_t u = __shfl_up_sync(0xffffffffu, t, d);
            if (lane >= d) t += u;
        }
        warp_tot[lane] = t;
    }
    __syncthreads();
    const int32_t r = v + (w ? warp_tot[w - 1] : 0);
    __syncthreads();
    return r;
}

__global__ void scan_tiles_kernel(int32_t* x, int64_t n, int32_t* tile_sums) {
    __shared__ int32_t wt[32];
    const int64_t base = static_cast<int64_t>(blockIdx.x) * SCAN_TILE + static_cast<int64_t>(threadIdx.x) * SCAN_PER;
    int32_t v[SCAN_PER];
    int32_t run = 0;
#pragma unroll
    for (int q = 0; q < SCAN_PER; ++q) {
        v[q] = (base + q < n) ? x[base + q] : 0;
        run += v[q];
        v[q] = run;
    }
    const int32_t incl = block_inclusive(run, wt);
    const int32_t off = incl - run;
#pragma unroll
    for (int q = 0; q < SCAN_PER; ++q)
        if (base + q < n) x[base + q] = v[q] + off;
    if (threadIdx.x == blockDim.x - 1) tile_sums[blockIdx.x] = incl;
}

// Exclusive scan of the tile sums in one CTA (any count).
__global__ void scan_sums_kernel(int32_t* sums, int64_t n) {
    __shared__ int32_t wt[32];
    __shared__ int32_t carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int64_t b = 0; b < n; b += blockDim.x) {
        const int64_t i = b + threadIdx.x;
        const int32_t v = i < n ? sums[i] : 0;
        const int32_t incl = block_inclusive(v, wt);
        const int32_t c = carry;
        if (i < n) sums[i] = c + incl - v;
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) carry = c + incl;
        __syncthreads();
    }
}

__global__ void scan_add_kernel(int32_t* x, int64_t n, const int32_t* sums) {
    const int32_t off = sums[blockIdx.x];
    if (off == 0) return;
    const int64_t base = static_cast<int64_t>(blockIdx.x) * SCAN_TILE;
    for (int t = threadIdx.x; t < SCAN_TILE; t += blockDim.x)
        if (base + t < n) x[base + t] += off;
}

// ── CSR validation (Tensor::sparse_csr) ──────────────────────────────────────
struct CheckWords {
    unsigned long long first_bad_col;    // index of the first out-of-range col_ind
    unsigned long long first_bad_rp;     // first i with row_ptr[i] < row_ptr[i-1]
    unsigned long long first_bad_order;  // first i with row_order[i] outside [0, rows)
    int32_t rp_first, rp_last;           // row_ptr[0], row_ptr[rows]
};
static_assert(sizeof(CheckWords) == kCsrCheckWordsBytes, "CheckWords size");

__global__ void csr_check_kernel(int64_t rows, int64_t cols, int64_t nnz, const int32_t* rp, const int32_t* ci,
                                 const int32_t* order, CheckWords* w) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (tid == 0 && rp) {
        w->rp_first = rp[0];
        w->rp_last = rp[rows];
    }
    if (cols >= 0) {
        // nnz < 0: the column array holds row_ptr[rows] entries
        const int64_t n = nnz >= 0 ? nnz : (rp ? max(0, rp[rows]) : 0);
        for (int64_t t = tid; t < n; t += stride) {
            const int32_t c = ci[t];
            if (c < 0 || c >= cols) atomicMin(&w->first_bad_col, static_cast<unsigned long long>(t));
        }
    }
    for (int64_t t = tid + 1; t <= rows; t += stride)
        if (rp[t] < rp[t - 1]) atomicMin(&w->first_bad_rp, static_cast<unsigned long long>(t));
    if (order)
        for (int64_t t = tid; t < rows; t += stride)
            if (order[t] < 0 || order[t] >= rows) atomicMin(&w->first_bad_order, static_cast<unsigned long long>(t));
}

// ── edge_list_to_csr ────────────────────────────────────────────────────────
__global__ void edge_check_kernel(int64_t N, int64_t E, const int32_t* src, const int32_t* dst,
                                  unsigned long long* first_bad) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < E; e += stride) {
        const int32_t s = src[e], d = dst[e];
        if (s < 0 || s >= N || d < 0 || d >= N) atomicMin(first_bad, static_cast<unsigned long long>(e));
    }
}

__global__ void edge_count_kernel(int64_t E, const int32_t* src, int32_t* rp /*[N+1], zeroed*/) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < E; e += stride)
        atomicAdd(rp + src[e] + 1, 1);
}

__global__ void edge_scatter_kernel(int64_t E, const int32_t* src, const int32_t* dst, const int32_t* rp,
                                    int32_t* cursor, int32_t* ci, float* v) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < E; e += stride) {
        const int32_t s = src[e];
        const int32_t pos = rp[s] + atomicAdd(cursor + s, 1);
        ci[pos] = dst[e];
        v[e] = 1.0f;
    }
}

// Rows of <= 32 entries: one warp per row, bitonic network on registers.
__global__ void sort_rows_warp_kernel(int64_t N, const int32_t* rp, int32_t* ci) {
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (row >= N) return;
    const int lane = threadIdx.x & 31;
    const int32_t s = rp[row], len = rp[row + 1] - s;
    if (len <= 1 || len > 32) return;
    int32_t x = lane < len ? ci[s + lane] : INT_MAX;
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const int32_t y = __shfl_xor_sync(0xffffffffu, x, j);
            const bool up = ((lane & k) == 0);
            const bool lower = ((lane & j) == 0);
            x = (lower == up) ? min(x, y) : max(x, y);
        }
    }
    if (lane < len) ci[s + lane] = x;
}

// Rows of 33..cap entries: one CTA per listed row, bitonic sort in shared memory.
__global__ void sort_rows_block_kernel(const int32_t* rows, int64_t nrows, const int32_t* rp, int32_t* ci, int cap) {
    extern __shared__ int32_t sh[];
    for (int64_t r = blockIdx.x; r < nrows; r += gridDim.x) {
        const int32_t row = rows[r];
        const int32_t s = rp[row], len = rp[row + 1] - s;
        int P = 64;
        while (P < len) P <<= 1;
        for (int t = threadIdx.x; t < P; t += blockDim.x) sh[t] = t < len ? ci[s + t] : INT_MAX;
        __syncthreads();
        for (int k = 2; k <= P; k <<= 1) {
            for (int j = k >> 1; j > 0; j >>= 1) {
                for (int t = threadIdx.x; t < P; t += blockDim.x) {
                    const int p = t ^ j;
                    if (p > t) {
                        const int32_t a = sh[t], b = sh[p];
                        const bool up = ((t & k) == 0);
                        if ((a > b) == up) { sh[t] = b; sh[p] = a; }
                    }
                }
                __syncthreads();
            }
        }
        for (int t = threadIdx.x; t < len; t += blockDim.x) ci[s + t] = sh[t];
        __syncthreads();
        (void)cap;
    }
}

__global__ void classify_rows_kernel(int64_t N, const int32_t* rp, int cap, int32_t* mid_rows, int32_t* n_mid,
                                     int32_t* big_rows, int32_t* n_big) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= N) return;
    const int32_t len = rp[i + 1] - rp[i];
    if (len > 32 && len <= cap) mid_rows[atomicAdd(n_mid, 1)] = static_cast<int32_t>(i);
    else if (len > cap) big_rows[atomicAdd(n_big, 1)] = static_cast<int32_t>(i);
}

// Counting sort of one long row over the column range [0, N).
__global__ void row_hist_kernel(const int32_t* ci, int32_t s, int32_t len, int32_t* hist) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < len; t += stride)
        atomicAdd(hist + ci[s + t] + 1, 1);
}

__global__ void row_expand_kernel(int64_t N, const int32_t* hist_scan, int32_t* ci, int32_t s) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < N; c += stride)
        for (int32_t p = hist_scan[c]; p < hist_scan[c + 1]; ++p) ci[s + p] = static_cast<int32_t>(c);
}

// ── add_self_loops / gcn_norm ───────────────────────────────────────────────
// Two row passes (one warp per row) over a block of rows of a square matrix
// whose local row i is global row i + off (the whole matrix: off = 0).
//
// Pass 1 (self_loop_rows_kernel): whether the row holds its diagonal, where
// add_self_loops inserts it otherwise -- before the first column > i in
// stored order, else at the end (src/layers.cpp:104-133) -- as insert[i]
// (-1: the row has one), the new length into out_rp[i+1], and for gcn_norm
// 1/sqrt(deg) of the self-looped row (src/layers.cpp:168-187).
//
// The degree is the reference's sequential float sum of the row's values in
// stored order, with every diagonal entry as v + 1 and an inserted one as 1.
// When every value is an integer and len * (max|v| + 1) + 1 < 2^24, every
// partial sum of any subset is an integer below 2^24 -- exact in fp32 -- so
// any summation order gives the sequential result bit for bit, and the warp
// adds its lanes' partial sums as a tree (always the case for unweighted
// graphs).  Otherwise the row is summed again as one sequential chain.
//
// Pass 2 (self_loop_fill_kernel): the self-looped row -- columns copied with
// the diagonal inserted, diagonal values v + 1 -- and for gcn_norm each value
// scaled (v * dis_row[i]) * dis_col[j], two roundings in that order
// (src/layers.cpp:192-198).  dis_col is indexed by global column.
// Each warp keeps CH chunks of 32 entries in flight (one load per lane per
// array per chunk, all issued before any is used).
constexpr int kSlChunks = 4;

template <bool DEG>
__global__ void self_loop_rows_kernel(int64_t N, int64_t off, const int32_t* rp, const int32_t* ci, const float* v,
                                      const int32_t* order, int32_t* out_rp, int32_t* insert, float* dis) {
    const int64_t slot = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (slot >= N) return;
    const int64_t row = order ? static_cast<int64_t>(order[slot]) : slot;
    const int lane = threadIdx.x & 31;
    const int32_t s = rp[row], e = rp[row + 1];
    const int32_t i32 = static_cast<int32_t>(row + off);
    bool has = false;
    int32_t ins = -1;                 // offset of the first column > i, -1 = none seen
    float part = 0.0f;                // this lane's partial degree (integer rows)
    bool integral = true;
    uint32_t max_bits = 0;            // max |v| as bits (order-preserving for |v|)
    for (int32_t b = s; b < e; b += 32 * kSlChunks) {
        int32_t c[kSlChunks];
        float x[kSlChunks];
#pragma unroll
        for (int u = 0; u < kSlChunks; ++u) {
            const int32_t t = b + 32 * u + lane;
            c[u] = t < e ? ci[t] : INT32_MIN;
            if (DEG) x[u] = t < e ? v[t] : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < kSlChunks; ++u) {
            const bool diag = c[u] == i32;
            const unsigned gt = __ballot_sync(0xffffffffu, c[u] > i32);
            if (ins < 0 && gt) ins = (b + 32 * u - s) + __ffs(gt) - 1;
            has = has || __any_sync(0xffffffffu, diag);
            if (DEG) {
                part = __fadd_rn(part, diag ? __fadd_rn(x[u], 1.0f) : x[u]);
                integral = integral && (x[u] == truncf(x[u]));
                max_bits = max(max_bits, __float_as_uint(x[u]) & 0x7fffffffu);
            }
        }
        if (!DEG && has) break;  // add_self_loops alone only needs to know that it is there
    }
    const int32_t len = e - s;
    const int32_t pos = has ? -1 : (ins >= 0 ? ins : len);
    if (DEG) {
        integral = __all_sync(0xffffffffu, integral);
        max_bits = __reduce_max_sync(0xffffffffu, max_bits);
        float deg;
        if (integral && static_cast<double>(len) * (static_cast<double>(__uint_as_float(max_bits)) + 1.0) + 1.0 <
                            16777216.0) {
            for (int d = 16; d > 0; d >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, d));
            deg = has ? part : __fadd_rn(part, 1.0f);
        } else {
            // the reference's chain: d = 0; d += v in stored order
            deg = 0.0f;
            for (int32_t b = s; b < e; b += 32) {
                const int32_t t = b + lane;
                float x = t < e ? v[t] : 0.0f;
                if (t < e && ci[t] == i32) x = __fadd_rn(x, 1.0f);
                const int n = min(32, e - b);
                for (int k = 0; k < n; ++k) {
                    if (b - s + k == pos) deg = __fadd_rn(deg, 1.0f);
                    deg = __fadd_rn(deg, __shfl_sync(0xffffffffu, x, k));
                }
            }
            if (pos == len) deg = __fadd_rn(deg, 1.0f);
        }
        if (lane == 0) dis[row] = deg > 0.0f ? __fdiv_rn(1.0f, __fsqrt_rn(deg)) : 0.0f;
    }
    if (lane == 0) {
        out_rp[row + 1] = len + (has ? 0 : 1);
        insert[row] = pos;
        if (row == 0) out_rp[0] = 0;
    }
}

template <bool NORM>
__global__ void self_loop_fill_kernel(int64_t N, int64_t off, const int32_t* rp, const int32_t* ci, const float* v,
                                      const int32_t* order, const int32_t* out_rp, const int32_t* insert,
                                      const float* dis_row, const float* dis_col, int32_t* out_ci, float* out_v) {
    const int64_t slot = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (slot >= N) return;
    const int64_t row = order ? static_cast<int64_t>(order[slot]) : slot;
    const int lane = threadIdx.x & 31;
    const int32_t s = rp[row], e = rp[row + 1];
    const int32_t o = out_rp[row];
    const int32_t ins = insert[row];
    const int32_t i32 = static_cast<int32_t>(row + off);
    const float di = NORM ? dis_row[row] : 1.0f;
    // Software-pipelined: the next group's (col, value) loads are issued
    // before this group's dis_col gathers are consumed and its stores made.
    int32_t c[kSlChunks];
    float x[kSlChunks];
#pragma unroll
    for (int u = 0; u < kSlChunks; ++u) {
        const int32_t t = s + 32 * u + lane;
        c[u] = t < e ? ci[t] : 0;
        x[u] = t < e ? v[t] : 0.0f;
    }
    for (int32_t b = s; b < e; b += 32 * kSlChunks) {
        float dj[kSlChunks];
        if (NORM) {
#pragma unroll
            for (int u = 0; u < kSlChunks; ++u) dj[u] = (b + 32 * u + lane < e) ? dis_col[c[u]] : 0.0f;
        }
        int32_t cn[kSlChunks];
        float xn[kSlChunks];
        const int32_t bn = b + 32 * kSlChunks;
#pragma unroll
        for (int u = 0; u < kSlChunks; ++u) {
            const int32_t t = bn + 32 * u + lane;
            cn[u] = t < e ? ci[t] : 0;
            xn[u] = t < e ? v[t] : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < kSlChunks; ++u) {
            const int32_t t = b + 32 * u + lane;
            if (t < e) {
                const int32_t rel = t - s;
                const int32_t p = o + rel + ((ins >= 0 && rel >= ins) ? 1 : 0);
                const float xs = (c[u] == i32) ? __fadd_rn(x[u], 1.0f) : x[u];
                out_ci[p] = c[u];
                out_v[p] = NORM ? __fmul_rn(__fmul_rn(xs, di), dj[u]) : xs;
            }
        }
#pragma unroll
        for (int u = 0; u < kSlChunks; ++u) {
            c[u] = cn[u];
            x[u] = xn[u];
        }
    }
    if (ins >= 0 && lane == 0) {
        out_ci[o + ins] = i32;
        out_v[o + ins] = NORM ? __fmul_rn(__fmul_rn(1.0f, di), dis_col[i32]) : 1.0f;
    }
}

// FAST gcn_norm scale: dis[i] = 1/sqrt(sum of row i's values + 1), the sum in
// any order (a warp tree; exact for integer rows within 2^24).
// v == nullptr: an unweighted CSR (every entry 1.0).  Below 2^24 entries
// every partial sum of ones is an exact integer, so the row sum is the row
// length whatever the order -- taken from row_ptr without reading entries;
// longer rows run the same tree over ones.
__global__ void gcn_scale_rows_kernel(int64_t N, const int32_t* rp, const float* v, float* dis) {
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (row >= N) return;
    const int lane = threadIdx.x & 31;
    const int32_t s = rp[row], e = rp[row + 1];
    float part = 0.0f;
    if (v == nullptr && e - s < (1 << 24)) {
        part = static_cast<float>(e - s);
    } else {
        for (int32_t b = s; b < e; b += 32 * kSlChunks) {
            float x[kSlChunks];
#pragma unroll
            for (int u = 0; u < kSlChunks; ++u)
                x[u] = (b + 32 * u + lane < e) ? (v ? v[b + 32 * u + lane] : 1.0f) : 0.0f;
#pragma unroll
            for (int u = 0; u < kSlChunks; ++u) part = __fadd_rn(part, x[u]);
        }
        for (int k = 16; k > 0; k >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, k));
    }
    const float d = __fadd_rn(part, 1.0f);
    if (lane == 0) dis[row] = d > 0.0f ? __fdiv_rn(1.0f, __fsqrt_rn(d)) : 0.0f;
}

// Degree (sequential float sum of a self-looped row) and 1/sqrt(deg): the
// standalone form for rows that already hold their self-loops.
__global__ void gcn_degree_kernel(int64_t N, const int32_t* rp, const float* v, float* dis) {
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (row >= N) return;
    const int lane = threadIdx.x & 31;
    const int32_t s = rp[row], e = rp[row + 1];
    float part = 0.0f;
    bool integral = true;
    uint32_t max_bits = 0;
    for (int32_t b = s; b < e; b += 32) {
        const float x = (b + lane < e) ? v[b + lane] : 0.0f;
        part = __fadd_rn(part, x);
        integral = integral && (x == truncf(x));
        max_bits = max(max_bits, __float_as_uint(x) & 0x7fffffffu);
    }
    integral = __all_sync(0xffffffffu, integral);
    max_bits = __reduce_max_sync(0xffffffffu, max_bits);
    float d;
    if (integral && static_cast<double>(e - s) * static_cast<double>(__uint_as_float(max_bits)) < 16777216.0) {
        for (int k = 16; k > 0; k >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, k));
        d = part;  // exact: see self_loop_rows_kernel
    } else {
        d = 0.0f;
        for (int32_t b = s; b < e; b += 32) {
            const float x = (b + lane < e) ? v[b + lane] : 0.0f;
            const int n = min(32, e - b);
            for (int k = 0; k < n; ++k) d = __fadd_rn(d, __shfl_sync(0xffffffffu, x, k));
        }
    }
    if (lane == 0) dis[row] = d > 0.0f ? __fdiv_rn(1.0f, __fsqrt_rn(d)) : 0.0f;
}

__global__ void gcn_scale_kernel(int64_t N, const int32_t* rp, const int32_t* ci, float* v, const float* dis_row,
                                 const float* dis_col) {
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (row >= N) return;
    const int lane = threadIdx.x & 31;
    const float di = dis_row[row];
    for (int32_t t = rp[row] + lane; t < rp[row + 1]; t += 32) v[t] = __fmul_rn(__fmul_rn(v[t], di), dis_col[ci[t]]);
}

unsigned stride_grid(int64_t n, int threads) {
    const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
    return static_cast<unsigned>(std::max<int64_t>(1, std::min(cap, ceil_div(n, threads))));
}

unsigned warp_rows_grid(int64_t rows) { return static_cast<unsigned>(ceil_div(rows * 32, 256)); }

template <class T>
T read_back(const T* dev, cudaStream_t s) {
    T h{};
    TG_CUDA(cudaMemcpyAsync(&h, dev, sizeof(T), cudaMemcpyDeviceToHost, s));
    TG_CUDA(cudaStreamSynchronize(s));
    return h;
}

constexpr int BLOCK_SORT_CAP = 32768;

}  // namespace

void inclusive_scan_i32(int32_t* x, int64_t n, cudaStream_t s) {
    if (n <= 0) return;
    const int64_t tiles = ceil_div(n, SCAN_TILE);
    Scratch<int32_t> sums(static_cast<size_t>(tiles), s);
    launch("scan_tiles", scan_tiles_kernel, dim3(static_cast<unsigned>(tiles)), dim3(SCAN_T), 0, s, x, n, sums.p);
    if (tiles > 1) {
        launch("scan_sums", scan_sums_kernel, dim3(1), dim3(1024), 0, s, sums.p, tiles);
        launch("scan_add", scan_add_kernel, dim3(static_cast<unsigned>(tiles)), dim3(256), 0, s, x, n,
               static_cast<const int32_t*>(sums.p));
    }
}

void csr_validate(int64_t rows, int64_t cols, int64_t nnz, const int32_t* rp, const int32_t* ci, cudaStream_t s,
                  const int32_t* order, void* words) {
    if (rows < 0) invalid("Tensor::sparse_csr: negative size");
    if (rows > 0 && !rp) invalid("Tensor::sparse_csr: row_ptr is NULL");
    if (nnz > 0 && !ci && cols >= 0) invalid("Tensor::sparse_csr: col_ind is NULL");
    if (rows == 0 && nnz <= 0 && !rp) return;
    std::unique_ptr<Scratch<CheckWords>> own;
    CheckWords* w = static_cast<CheckWords*>(words);
    if (!w) {
        own.reset(new Scratch<CheckWords>(1, s));
        w = own->p;
    }
    TG_CUDA(cudaMemsetAsync(w, 0xff, sizeof(CheckWords), s));
    const int64_t span = std::max<int64_t>(std::max<int64_t>(nnz, rows), 1);
    launch("csr_check", csr_check_kernel, dim3(stride_grid(span, 256)), dim3(256), 0, s, rows, cols, nnz, rp, ci, order,
           w);
    const CheckWords h = read_back(w, s);
    if (rp && h.rp_first < 0)
        invalid("Tensor::sparse_csr: row_ptr[0] (" + std::to_string(h.rp_first) + ") must be >= 0");
    if (nnz >= 0 && rp && static_cast<int64_t>(h.rp_last) != nnz)
        invalid("Tensor::sparse_csr: row_ptr.back() (" + std::to_string(h.rp_last) +
                ") must equal values.size() (" + std::to_string(nnz) + ")");
    if (h.first_bad_col != ~0ull) {
        const int32_t c = read_back(ci + h.first_bad_col, s);
        invalid("Tensor::sparse_csr: col_ind[" + std::to_string(h.first_bad_col) + "] = " + std::to_string(c) +
                " is out of bounds for cols=" + std::to_string(cols));
    }
    if (h.first_bad_rp != ~0ull) {
        const int32_t a = read_back(rp + h.first_bad_rp, s), b = read_back(rp + h.first_bad_rp - 1, s);
        invalid("Tensor::sparse_csr: row_ptr must be non-decreasing; row_ptr[" + std::to_string(h.first_bad_rp) +
                "] = " + std::to_string(a) + " < row_ptr[" + std::to_string(h.first_bad_rp - 1) +
                "] = " + std::to_string(b));
    }
    if (h.first_bad_order != ~0ull) {
        const int32_t o = read_back(order + h.first_bad_order, s);
        invalid("row_order[" + std::to_string(h.first_bad_order) + "] = " + std::to_string(o) +
                " is out of range [0, " + std::to_string(rows) + ")");
    }
}

void edge_list_to_csr(int64_t N, int64_t E, const int32_t* src, const int32_t* dst, int32_t* rp, int32_t* ci,
                      float* v, cudaStream_t s) {
    if (N == 0) {
        if (E != 0)
            invalid("GraphLoader::edge_list_to_csr: num_nodes is 0 but edges is non-empty");
        TG_CUDA(cudaMemsetAsync(rp, 0, sizeof(int32_t), s));
        return;
    }
    if (E > INT32_MAX) invalid("GraphLoader::edge_list_to_csr: more than 2^31-1 edges do not fit int32 row_ptr");
    if (E > 0) {
        Scratch<unsigned long long> bad(1, s);
        TG_CUDA(cudaMemsetAsync(bad.p, 0xff, sizeof(unsigned long long), s));
        launch("edge_check", edge_check_kernel, dim3(stride_grid(E, 256)), dim3(256), 0, s, N, E, src, dst, bad.p);
        const unsigned long long e = read_back(bad.p, s);
        if (e != ~0ull) {
            const int32_t a = read_back(src + e, s), b = read_back(dst + e, s);
            const std::string range = " out of range [0, " + std::to_string(N) + ")";
            if (a < 0 || a >= N)
                invalid("GraphLoader::edge_list_to_csr: edge[" + std::to_string(e) + "].src = " + std::to_string(a) + range);
            invalid("GraphLoader::edge_list_to_csr: edge[" + std::to_string(e) + "].dst = " + std::to_string(b) + range);
        }
    }
    TG_CUDA(cudaMemsetAsync(rp, 0, static_cast<size_t>(N + 1) * sizeof(int32_t), s));
    if (E == 0) return;
    launch("edge_count", edge_count_kernel, dim3(stride_grid(E, 256)), dim3(256), 0, s, E, src, rp);
    inclusive_scan_i32(rp + 1, N, s);
    {
        Scratch<int32_t> cursor(static_cast<size_t>(N), s);
        TG_CUDA(cudaMemsetAsync(cursor.p, 0, static_cast<size_t>(N) * sizeof(int32_t), s));
        launch("edge_scatter", edge_scatter_kernel, dim3(stride_grid(E, 256)), dim3(256), 0, s, E, src, dst,
               static_cast<const int32_t*>(rp), cursor.p, ci, v);
    }
    // Per-row sort by size class.
    launch("sort_rows_warp", sort_rows_warp_kernel, dim3(warp_rows_grid(N)), dim3(256), 0, s, N,
           static_cast<const int32_t*>(rp), ci);
    Scratch<int32_t> lists(static_cast<size_t>(2 * N + 2), s);
    int32_t* mid = lists.p;
    int32_t* big = lists.p + N;
    int32_t* counts = lists.p + 2 * N;
    TG_CUDA(cudaMemsetAsync(counts, 0, 2 * sizeof(int32_t), s));
    launch("classify_rows", classify_rows_kernel, dim3(static_cast<unsigned>(ceil_div(N, 256))), dim3(256), 0, s, N,
           static_cast<const int32_t*>(rp), BLOCK_SORT_CAP, mid, counts, big, counts + 1);
    int32_t hc[2];
    TG_CUDA(cudaMemcpyAsync(hc, counts, sizeof(hc), cudaMemcpyDeviceToHost, s));
    TG_CUDA(cudaStreamSynchronize(s));
    if (hc[0] > 0) {
        // Size classes: up to 4096 entries with 16 KB of shared memory, the
        // rest with 128 KB; both kernels read each listed row's length.
        const size_t smem = static_cast<size_t>(BLOCK_SORT_CAP) * sizeof(int32_t);
        TG_CUDA(cudaFuncSetAttribute(sort_rows_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem)));
        launch("sort_rows_block", sort_rows_block_kernel, dim3(static_cast<unsigned>(std::min<int64_t>(hc[0], 4 * num_sms()))),
               dim3(1024), smem, s, static_cast<const int32_t*>(mid), static_cast<int64_t>(hc[0]),
               static_cast<const int32_t*>(rp), ci, BLOCK_SORT_CAP);
    }
    if (hc[1] > 0) {
        std::vector<int32_t> rows(static_cast<size_t>(hc[1]));
        TG_CUDA(cudaMemcpyAsync(rows.data(), big, rows.size() * sizeof(int32_t), cudaMemcpyDeviceToHost, s));
        std::vector<int32_t> hrp(2);
        Scratch<int32_t> hist(static_cast<size_t>(N + 1), s);
        TG_CUDA(cudaStreamSynchronize(s));
        for (int32_t r : rows) {
            TG_CUDA(cudaMemcpyAsync(hrp.data(), rp + r, 2 * sizeof(int32_t), cudaMemcpyDeviceToHost, s));
            TG_CUDA(cudaStreamSynchronize(s));
            const int32_t st = hrp[0], len = hrp[1] - hrp[0];
            TG_CUDA(cudaMemsetAsync(hist.p, 0, static_cast<size_t>(N + 1) * sizeof(int32_t), s));
            launch("row_hist", row_hist_kernel, dim3(stride_grid(len, 256)), dim3(256), 0, s,
                   static_cast<const int32_t*>(ci), st, len, hist.p);
            inclusive_scan_i32(hist.p + 1, N, s);
            launch("row_expand", row_expand_kernel, dim3(stride_grid(N, 256)), dim3(256), 0, s, N,
                   static_cast<const int32_t*>(hist.p), ci, st);
        }
    }
}

// Pass 1 of a row block: out_rp (scanned), insert[], and with DEG dis[].
void self_loop_rows(int64_t N, int64_t off, const int32_t* rp, const int32_t* ci, const float* v,
                    const int32_t* order, int32_t* orp, int32_t* insert, float* dis, cudaStream_t s) {
    if (N == 0) {
        TG_CUDA(cudaMemsetAsync(orp, 0, sizeof(int32_t), s));
        return;
    }
    if (dis)
        launch("self_loop_rows<deg>", self_loop_rows_kernel<true>, dim3(warp_rows_grid(N)), dim3(256), 0, s, N, off,
               rp, ci, v, order, orp, insert, dis);
    else
        launch("self_loop_rows", self_loop_rows_kernel<false>, dim3(warp_rows_grid(N)), dim3(256), 0, s, N, off, rp,
               ci, v, order, orp, insert, dis);
    inclusive_scan_i32(orp + 1, N, s);
}

// Pass 2 of a row block; dis_row == nullptr: add_self_loops alone.
void self_loop_fill(int64_t N, int64_t off, const int32_t* rp, const int32_t* ci, const float* v,
                    const int32_t* order, const int32_t* orp, const int32_t* insert, const float* dis_row,
                    const float* dis_col, int32_t* oci, float* ov, cudaStream_t s) {
    if (N == 0) return;
    if (dis_row)
        launch("self_loop_fill<norm>", self_loop_fill_kernel<true>, dim3(warp_rows_grid(N)), dim3(256), 0, s, N, off,
               rp, ci, v, order, orp, insert, dis_row, dis_col, oci, ov);
    else
        launch("self_loop_fill", self_loop_fill_kernel<false>, dim3(warp_rows_grid(N)), dim3(256), 0, s, N, off, rp,
               ci, v, order, orp, insert, dis_row, dis_col, oci, ov);
}

int64_t add_self_loops(int64_t N, int64_t off, const int32_t* rp, const int32_t* ci, const float* v, int32_t* orp,
                       int32_t* oci, float* ov, cudaStream_t s) {
    if (N == 0) {
        TG_CUDA(cudaMemsetAsync(orp, 0, sizeof(int32_t), s));
        return 0;
    }
    Scratch<int32_t> insert(static_cast<size_t>(N), s);
    self_loop_rows(N, off, rp, ci, v, nullptr, orp, insert.p, nullptr, s);
    self_loop_fill(N, off, rp, ci, v, nullptr, orp, insert.p, nullptr, nullptr, oci, ov, s);
    return read_back(orp + N, s);
}

void degree_inv_sqrt(int64_t N, const int32_t* rp, const float* v, float* dis, cudaStream_t s) {
    launch("gcn_degree", gcn_degree_kernel, dim3(warp_rows_grid(N)), dim3(256), 0, s, N, rp, v, dis);
}

void scale_sym(int64_t N, const int32_t* rp, const int32_t* ci, float* v, const float* dis_row, const float* dis_col,
               cudaStream_t s) {
    launch("gcn_scale", gcn_scale_kernel, dim3(warp_rows_grid(N)), dim3(256), 0, s, N, rp, ci, v, dis_row, dis_col);
}

int64_t gcn_norm(int64_t N, const int32_t* rp, const int32_t* ci, const float* v, int32_t* orp, int32_t* oci,
                 float* ov, cudaStream_t s) {
    if (N == 0) {
        TG_CUDA(cudaMemsetAsync(orp, 0, sizeof(int32_t), s));
        return 0;
    }
    Scratch<int32_t> insert(static_cast<size_t>(N), s);
    Scratch<float> dis(static_cast<size_t>(N), s);
    self_loop_rows(N, 0, rp, ci, v, nullptr, orp, insert.p, dis.p, s);
    self_loop_fill(N, 0, rp, ci, v, nullptr, orp, insert.p, dis.p, dis.p, oci, ov, s);
    return read_back(orp + N, s);
}

}  // namespace tg

using namespace tg;

extern "C" {

TG_API tg_status tg_edge_list_to_csr(int64_t num_nodes, int64_t E, const int32_t* src, const int32_t* dst,
                                     int32_t* row_ptr_out, int32_t* col_ind_out, float* values_out,
                                     void* stream) {
    return guard([&] {
        require_device();
        if (num_nodes < 0 || E < 0) invalid("GraphLoader::edge_list_to_csr: negative size");
        check_ptr("edge_list_to_csr", "row_ptr_out", row_ptr_out, true);
        check_ptr("edge_list_to_csr", "src/dst/col_ind_out/values_out",
                  src && dst && col_ind_out && values_out ? src : nullptr, E > 0);
        edge_list_to_csr(num_nodes, E, src, dst, row_ptr_out, col_ind_out, values_out, as_stream(stream));
    });
}

TG_API tg_status tg_add_self_loops_f32(int64_t N, int64_t nnz, const int32_t* row_ptr, const int32_t* col_ind,
                                       const float* values, int32_t* row_ptr_out, int32_t* col_ind_out,
                                       float* values_out, int64_t* nnz_out, void* stream) {
    return guard([&] {
        require_device();
        if (N < 0 || nnz < 0) invalid("add_self_loops: negative size");
        if (nnz + N > INT32_MAX) invalid("add_self_loops: result does not fit int32 row_ptr");
        check_csr_input(N, N, nnz, row_ptr, col_ind, as_stream(stream));
        const int64_t n = add_self_loops(N, 0, row_ptr, col_ind, values, row_ptr_out, col_ind_out, values_out,
                                         as_stream(stream));
        if (nnz_out) *nnz_out = n;
    });
}

TG_API tg_status tg_gcn_norm_f32(int64_t N, int64_t nnz, const int32_t* row_ptr, const int32_t* col_ind,
                                 const float* values, int32_t* row_ptr_out, int32_t* col_ind_out,
                                 float* values_out, int64_t* nnz_out, void* stream) {
    return guard([&] {
        require_device();
        if (N < 0 || nnz < 0) invalid("gcn_norm: negative size");
        if (nnz + N > INT32_MAX) invalid("gcn_norm: result does not fit int32 row_ptr");
        check_csr_input(N, N, nnz, row_ptr, col_ind, as_stream(stream));
        const int64_t n = gcn_norm(N, row_ptr, col_ind, values, row_ptr_out, col_ind_out, values_out,
                                   as_stream(stream));
        if (nnz_out) *nnz_out = n;
    });
}

TG_API tg_status tg_add_self_loops_rows_f32(int64_t rows, int64_t row_offset, int64_t nnz, const int32_t* row_ptr,
                                            const int32_t* col_ind, const float* values, int32_t* row_ptr_out,
                                            int32_t* col_ind_out, float* values_out, int64_t* nnz_out,
                                            void* stream) {
    return guard([&] {
        require_device();
        if (rows < 0 || row_offset < 0 || nnz < 0) invalid("add_self_loops: negative size");
        if (nnz + rows > INT32_MAX) invalid("add_self_loops: result does not fit int32 row_ptr");
        check_csr_input(rows, -1, nnz, row_ptr, col_ind, as_stream(stream));  // columns only compared
        const int64_t n = add_self_loops(rows, row_offset, row_ptr, col_ind, values, row_ptr_out, col_ind_out,
                                         values_out, as_stream(stream));
        if (nnz_out) *nnz_out = n;
    });
}

TG_API tg_status tg_gcn_norm_rows_degrees_f32(int64_t rows, int64_t row_offset, int64_t nnz, const int32_t* row_ptr,
                                              const int32_t* col_ind, const float* values, const int32_t* row_order,
                                              int32_t* row_ptr_out, int32_t* insert_out, float* dis_out,
                                              void* stream) {
    return guard([&] {
        require_device();
        if (rows < 0 || row_offset < 0 || nnz < 0) invalid("gcn_norm: negative size");
        if (nnz + rows > INT32_MAX) invalid("gcn_norm: result does not fit int32 row_ptr");
        check_ptr("gcn_norm", "row_ptr_out", row_ptr_out, true);
        check_ptr("gcn_norm", "row_ptr/insert_out/dis_out", row_ptr && insert_out && dis_out ? row_ptr : nullptr,
                  rows > 0);
        check_ptr("gcn_norm", "col_ind/values", col_ind && values ? col_ind : nullptr, nnz > 0);
        check_csr_input(rows, -1, nnz, row_ptr, col_ind, as_stream(stream), row_order);  // columns only compared
        self_loop_rows(rows, row_offset, row_ptr, col_ind, values, row_order, row_ptr_out, insert_out, dis_out,
                       as_stream(stream));
    });
}

TG_API tg_status tg_gcn_norm_rows_fill_f32(int64_t rows, int64_t row_offset, int64_t n_cols, const int32_t* row_ptr,
                                           const int32_t* col_ind, const float* values, const int32_t* row_order,
                                           const int32_t* row_ptr_out, const int32_t* insert, const float* dis_row,
                                           const float* dis_col, int32_t* col_ind_out, float* values_out,
                                           void* stream) {
    return guard([&] {
        require_device();
        if (rows < 0 || row_offset < 0 || n_cols < 0) invalid("gcn_norm: negative size");
        if (row_offset + rows > n_cols) invalid("gcn_norm: rows [row_offset, row_offset + rows) exceed n_cols");
        check_csr_input(rows, n_cols, -1, row_ptr, col_ind, as_stream(stream), row_order);
        check_ptr("gcn_norm", "row_ptr/row_ptr_out/insert/dis_row/dis_col/col_ind_out/values_out",
                  row_ptr && row_ptr_out && insert && dis_row && dis_col && col_ind_out && values_out ? row_ptr
                                                                                                      : nullptr,
                  rows > 0);
        self_loop_fill(rows, row_offset, row_ptr, col_ind, values, row_order, row_ptr_out, insert, dis_row, dis_col,
                       col_ind_out, values_out, as_stream(stream));
    });
}

TG_API tg_status tg_gcn_norm_scale_f32(int64_t rows, int64_t nnz, const int32_t* row_ptr, const float* values,
                                       float* dis_out, void* stream) {
    return guard([&] {
        require_device();
        if (rows < 0 || nnz < 0) invalid("gcn_norm: negative size");
        if (rows == 0) return;
        check_ptr("gcn_norm", "row_ptr/dis_out", row_ptr && dis_out ? row_ptr : nullptr, true);
        // values == NULL: an unweighted CSR (every entry 1.0)
        check_csr_input(rows, -1, -1, row_ptr, nullptr, as_stream(stream));  // values read by row only
        launch("gcn_scale_rows", gcn_scale_rows_kernel, dim3(warp_rows_grid(rows)), dim3(256), 0, as_stream(stream),
               rows, row_ptr, values, dis_out);
    });
}

TG_API tg_status tg_csr_degree_inv_sqrt_f32(int64_t rows, const int32_t* row_ptr, const float* values,
                                            float* dis_out, void* stream) {
    return guard([&] {
        require_device();
        if (rows < 0) invalid("gcn_norm: negative size");
        check_csr_input(rows, -1, -1, row_ptr, nullptr, as_stream(stream));
        if (rows) degree_inv_sqrt(rows, row_ptr, values, dis_out, as_stream(stream));
    });
}

TG_API tg_status tg_csr_scale_sym_f32(int64_t rows, const int32_t* row_ptr, const int32_t* col_ind, float* values,
                                      const float* dis_row, const float* dis_col, void* stream) {
    return guard([&] {
        require_device();
        if (rows < 0) invalid("gcn_norm: negative size");
        check_csr_input(rows, -1, -1, row_ptr, col_ind, as_stream(stream));  // col_ind must index dis_col
        if (rows) scale_sym(rows, row_ptr, col_ind, values, dis_row, dis_col, as_stream(stream));
    });
}

TG_API tg_status tg_csr_validate(int64_t rows, int64_t cols, int64_t nnz, const int32_t* row_ptr,
                                 const int32_t* col_ind, void* stream) {
    return guard([&] {
        require_device();
        if (rows < 0 || cols < 0 || nnz < 0) invalid("Tensor::sparse_csr: negative size");
        csr_validate(rows, cols, nnz, row_ptr, col_ind, as_stream(stream));
    });
}

}  // extern "C"
