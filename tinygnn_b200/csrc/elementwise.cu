// ============================================================================
//  elementwise.cu -- activations, bias, row softmax / log_softmax,
//  edge_softmax.
//
//  Reference: src/ops.cpp:304-661 (activations, softmax, log_softmax,
//  add_bias), src/layers.cpp:768-822 (edge_softmax).  The row kernels give
//  each row to one thread and walk it in the reference's sequential order
//  (max, then a running sum), so the only differences from the CPU are the
//  last bits of expf/logf.  These passes are HBM-bound; on the layer path
//  they are fused into the producing kernel's epilogue instead.
// ============================================================================
#include <algorithm>

#include "launch.cuh"

namespace tg {

namespace {

__global__ void activation_kernel(int act, float alpha, float* X, int64_t rows, int64_t cols, int64_t ld) {
    const int64_t total = rows * cols;
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = t / cols, c = t % cols;
        float* p = X + r * ld + c;
        *p = apply_act(act, *p, alpha);
    }
}

__global__ void add_bias_kernel(float* X, int64_t rows, int64_t cols, int64_t ld, const float* b) {
    const int64_t total = rows * cols;
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = t / cols, c = t % cols;
        float* p = X + r * ld + c;
        *p = __fadd_rn(*p, __ldg(b + c));
    }
}

// softmax (ops.cpp:525-547) / log_softmax (ops.cpp:584-604) of one row in
// place, in the reference's order: max, then the exp sum left to right.
template <bool LOG>
__device__ __forceinline__ void softmax_row(float* row, int64_t cols) {
    float mx = row[0];
    for (int64_t j = 1; j < cols; ++j)
        if (row[j] > mx) mx = row[j];
    float s = 0.0f;
    if (LOG) {
        for (int64_t j = 0; j < cols; ++j) s = __fadd_rn(s, expf(__fsub_rn(row[j], mx)));
        const float lse = __fadd_rn(mx, logf(s));
        for (int64_t j = 0; j < cols; ++j) row[j] = __fsub_rn(row[j], lse);
    } else {
        for (int64_t j = 0; j < cols; ++j) {
            const float e = expf(__fsub_rn(row[j], mx));
            row[j] = e;
            s = __fadd_rn(s, e);
        }
        const float inv = __fdiv_rn(1.0f, s);
        for (int64_t j = 0; j < cols; ++j) row[j] = __fmul_rn(row[j], inv);
    }
}

// Rows of up to 256 columns: a block of TR threads stages TR rows in shared
// memory (TR = 128 / 64 / 32 for up to 64 / 128 / 256 columns, ~33 KB),
// each thread runs softmax_row on its row there (odd stride: no bank
// conflicts), and the rows go back.  Both copies walk the block's elements
// in row-major order, TR threads apart (consecutive threads touch
// consecutive columns: coalesced), eight independent loads ahead.
constexpr int kCopyAhead = 8;

// Element position (row, col) of flat index t + k * step, advanced without
// a division per step.
struct TilePos {
    int r, c, qr, qc, cols;
    __device__ TilePos(int t, int cols_, int step) : r(t / cols_), c(t % cols_), qr(step / cols_),
                                                     qc(step % cols_), cols(cols_) {}
    __device__ void next() {
        r += qr;
        c += qc;
        if (c >= cols) {
            c -= cols;
            ++r;
        }
    }
};

template <bool LOG, int TR>
__global__ void __launch_bounds__(TR) row_softmax_tile_kernel(float* X, int64_t rows, int64_t cols, int64_t ld) {
    extern __shared__ float tile[];
    const int nc = static_cast<int>(cols);
    const int stride = nc | 1;
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * TR;
    const int nr = static_cast<int>(min(static_cast<int64_t>(TR), rows - r0));
    const int total = nr * nc;
    float* base = X + r0 * ld;
    {
        TilePos p(threadIdx.x, nc, TR);
        for (int i = threadIdx.x; i < total; i += kCopyAhead * TR) {
            float v[kCopyAhead];
            TilePos q = p;
#pragma unroll
            for (int u = 0; u < kCopyAhead; ++u) {
                if (i + u * TR < total) v[u] = base[q.r * ld + q.c];
                q.next();
            }
#pragma unroll
            for (int u = 0; u < kCopyAhead; ++u) {
                if (i + u * TR < total) tile[p.r * stride + p.c] = v[u];
                p.next();
            }
        }
    }
    __syncthreads();
    if (static_cast<int>(threadIdx.x) < nr) softmax_row<LOG>(tile + threadIdx.x * stride, cols);
    __syncthreads();
    {
        TilePos p(threadIdx.x, nc, TR);
        for (int i = threadIdx.x; i < total; i += kCopyAhead * TR) {
            float v[kCopyAhead];
            TilePos q = p;
#pragma unroll
            for (int u = 0; u < kCopyAhead; ++u) {
                if (i + u * TR < total) v[u] = tile[q.r * stride + q.c];
                q.next();
            }
#pragma unroll
            for (int u = 0; u < kCopyAhead; ++u) {
                if (i + u * TR < total) base[p.r * ld + p.c] = v[u];
                p.next();
            }
        }
    }
}

// Wider rows: one row per thread in global memory.
template <bool LOG>
__global__ void row_softmax_kernel(float* X, int64_t rows, int64_t cols, int64_t ld) {
    const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    softmax_row<LOG>(X + r * ld, cols);
}

// edge_softmax (layers.cpp:791-812), one CSR row per thread.
__global__ void edge_softmax_kernel(int64_t M, const int32_t* rp, const float* v, float* out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= M) return;
    const int32_t s = rp[i], e = rp[i + 1];
    if (s == e) return;
    float mx = v[s];
    for (int32_t k = s + 1; k < e; ++k) mx = (mx < v[k]) ? v[k] : mx;  // std::max(mx, v)
    float sum = 0.0f;
    for (int32_t k = s; k < e; ++k) {
        const float x = expf(__fsub_rn(v[k], mx));
        out[k] = x;
        sum = __fadd_rn(sum, x);
    }
    if (sum > 0.0f) {
        const float inv = __fdiv_rn(1.0f, sum);
        for (int32_t k = s; k < e; ++k) out[k] = __fmul_rn(out[k], inv);
    }
}

unsigned grid_for(int64_t total, int threads) {
    const int64_t cap = static_cast<int64_t>(num_sms()) * 16;
    return static_cast<unsigned>(std::max<int64_t>(1, std::min(cap, ceil_div(total, threads))));
}

}  // namespace

void activation(int act, float alpha, float* X, int64_t rows, int64_t cols, int64_t ld, cudaStream_t s) {
    if (rows == 0 || cols == 0 || act == TG_ACT_NONE) return;
    launch("activation", activation_kernel, dim3(grid_for(rows * cols, 256)), dim3(256), 0, s, act, alpha,
           X, rows, cols, ld);
}

void add_bias(float* X, int64_t rows, int64_t cols, int64_t ld, const float* b, cudaStream_t s) {
    if (rows == 0 || cols == 0) return;
    launch("add_bias", add_bias_kernel, dim3(grid_for(rows * cols, 256)), dim3(256), 0, s, X, rows, cols, ld, b);
}

void row_softmax(bool log, float* X, int64_t rows, int64_t cols, int64_t ld, cudaStream_t s) {
    if (rows == 0) return;
    const dim3 grid(static_cast<unsigned>(ceil_div(rows, 128)));
    if (cols <= 256) {
        const int tr = cols <= 64 ? 128 : (cols <= 128 ? 64 : 32);
        const dim3 tgrid(static_cast<unsigned>(ceil_div(rows, tr)));
        const size_t smem = static_cast<size_t>(tr) * (static_cast<size_t>(cols) | 1) * sizeof(float);
        auto kern = log ? (tr == 128 ? row_softmax_tile_kernel<true, 128>
                           : tr == 64 ? row_softmax_tile_kernel<true, 64> : row_softmax_tile_kernel<true, 32>)
                        : (tr == 128 ? row_softmax_tile_kernel<false, 128>
                           : tr == 64 ? row_softmax_tile_kernel<false, 64> : row_softmax_tile_kernel<false, 32>);
        launch(log ? "log_softmax" : "softmax", kern, tgrid, dim3(tr), smem, s, X, rows, cols, ld);
        return;
    }
    if (log) launch("log_softmax", row_softmax_kernel<true>, grid, dim3(128), 0, s, X, rows, cols, ld);
    else launch("softmax", row_softmax_kernel<false>, grid, dim3(128), 0, s, X, rows, cols, ld);
}

namespace {
__global__ void fill_kernel(float* p, int64_t n, float v) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < n; t += stride) p[t] = v;
}
}  // namespace

// p[0..n) = v, queued on s (the values of an unweighted CSR).
void fill_f32(float* p, int64_t n, float v, cudaStream_t s) {
    if (n <= 0) return;
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(ceil_div(n, 256), 8 * num_sms()));
    launch("fill", fill_kernel, dim3(grid), dim3(256), 0, s, p, n, v);
}

}  // namespace tg

using namespace tg;

extern "C" {

TG_API tg_status tg_activation_f32(int32_t act, float alpha, float* X, int64_t rows, int64_t cols,
                                   int64_t ld, void* stream) {
    return guard([&] {
        require_device();
        if (act < TG_ACT_NONE || act > TG_ACT_GELU) invalid("activation: unknown activation kind");
        check_ld("activation", "X", ld, cols);
        activation(act, alpha, X, rows, cols, ld, as_stream(stream));
    });
}

TG_API tg_status tg_softmax_rows_f32(float* X, int64_t rows, int64_t cols, int64_t ld, void* stream) {
    return guard([&] {
        require_device();
        if (cols == 0)
            invalid("softmax_inplace: tensor has 0 columns — softmax over an empty set is undefined.");
        check_ld("softmax_inplace", "X", ld, cols);
        row_softmax(false, X, rows, cols, ld, as_stream(stream));
    });
}

TG_API tg_status tg_log_softmax_rows_f32(float* X, int64_t rows, int64_t cols, int64_t ld, void* stream) {
    return guard([&] {
        require_device();
        if (cols == 0)
            invalid("log_softmax_inplace: tensor has 0 columns — log-softmax over an empty set is undefined.");
        check_ld("log_softmax_inplace", "X", ld, cols);
        row_softmax(true, X, rows, cols, ld, as_stream(stream));
    });
}

TG_API tg_status tg_add_bias_f32(float* X, int64_t rows, int64_t cols, int64_t ld, const float* bias,
                                 void* stream) {
    return guard([&] {
        require_device();
        check_ld("add_bias", "X", ld, cols);
        check_ptr("add_bias", "bias", bias, cols > 0);
        add_bias(X, rows, cols, ld, bias, as_stream(stream));
    });
}

TG_API tg_status tg_edge_softmax_f32(int64_t M, int64_t nnz, const int32_t* row_ptr, const float* values,
                                     float* values_out, void* stream) {
    return guard([&] {
        require_device();
        if (M < 0 || nnz < 0) invalid("edge_softmax: negative size");
        if (M == 0) return;
        check_csr_input(M, -1, nnz, row_ptr, nullptr, as_stream(stream));  // reads values by row only
        const dim3 grid(static_cast<unsigned>(ceil_div(M, 128)));
        launch("edge_softmax", edge_softmax_kernel, grid, dim3(128), 0, as_stream(stream), M, row_ptr,
               values, values_out);
    });
}

}  // extern "C"
