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

// softmax (ops.cpp:525-547) / log_softmax (ops.cpp:584-604), one row per thread.
template <bool LOG>
__global__ void row_softmax_kernel(float* X, int64_t rows, int64_t cols, int64_t ld) {
    const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    float* row = X + r * ld;
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
    if (log) launch("log_softmax", row_softmax_kernel<true>, grid, dim3(128), 0, s, X, rows, cols, ld);
    else launch("softmax", row_softmax_kernel<false>, grid, dim3(128), 0, s, X, rows, cols, ld);
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
        (void)nnz;
        const dim3 grid(static_cast<unsigned>(ceil_div(M, 128)));
        launch("edge_softmax", edge_softmax_kernel, grid, dim3(128), 0, as_stream(stream), M, row_ptr,
               values, values_out);
    });
}

}  // extern "C"
