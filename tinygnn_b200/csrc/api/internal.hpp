// ============================================================================
//  api/internal.hpp -- shared helpers of the C++ API (not installed).
// ============================================================================
#pragma once

#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "tinygnn/model.hpp"
#include "tinygnn/tensor.hpp"
#include "tinygnn_b200.h"

namespace tinygnn {
namespace detail {

// Every C++ API call runs on the calling thread's default stream.
inline void* stream() { return reinterpret_cast<void*>(cudaStreamPerThread); }
inline cudaStream_t cstream() { return cudaStreamPerThread; }

// tg_status -> the exception TinyGNN throws for that condition.
inline void check(tg_status s) {
    if (s == TG_OK) return;
    const std::string msg = tg_last_error_message();
    if (s == TG_ERR_INVALID_ARGUMENT) throw std::invalid_argument(msg);
    if (s == TG_ERR_OUT_OF_RANGE) throw std::out_of_range(msg);
    throw std::runtime_error(msg);
}

inline void cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

inline int mode() { return fast_math() ? TG_MODE_FAST : TG_MODE_EXACT; }

// The API's CSR Tensors are validated where they are built
// (Tensor::sparse_csr) or come from the library itself, so the C-ABI calls
// made for them skip the ABI's own input checks (restored on scope exit).
struct TrustedCsr {
    int32_t prev;
    TrustedCsr() : prev(tg_set_csr_checks(0)) {}
    ~TrustedCsr() { tg_set_csr_checks(prev); }
    TrustedCsr(const TrustedCsr&) = delete;
    TrustedCsr& operator=(const TrustedCsr&) = delete;
};

inline std::size_t pad4(std::size_t n) { return (n + 3) / 4 * 4; }

// A device array from the stream-ordered pool (the calling thread's
// stream), freed on scope exit in stream order.
template <class T>
struct DevArray {
    T* p = nullptr;
    explicit DevArray(std::size_t n) {
        void* q = nullptr;
        cuda(cudaMallocAsync(&q, (n ? n : 1) * sizeof(T), cstream()), "tinygnn allocation");
        p = static_cast<T*>(q);
    }
    ~DevArray() {
        if (p && cudaFreeAsync(p, cstream()) != cudaSuccess) cudaGetLastError();
    }
    DevArray(const DevArray&) = delete;
    DevArray& operator=(const DevArray&) = delete;
};

// A gathered operand above this size is aggregated in column-block passes
// (each pass's slice of the operand stays in L2; measured on B200 for the
// 119 MB Reddit-shaped layer-1 operand: 2 passes, -6 %).
constexpr std::size_t kPassBytes = std::size_t(64) << 20;

// Two weight matrices (same shape) as device arrays with ld == cols, the
// layout tg_gemm_pair_f32 takes (Tensor rows are padded to 16 bytes).
struct DevWeights {
    const float* wn = nullptr;
    const float* ws = nullptr;
    float* owned = nullptr;
    DevWeights(const Tensor& a, const Tensor& b) {
        const std::size_t r = a.rows(), c = a.cols();
        if (a.device_ld() == c && b.device_ld() == c) {
            wn = a.device_data();
            ws = b.device_data();
            return;
        }
        void* q = nullptr;
        detail::cuda(cudaMallocAsync(&q, (r * c > 0 ? 2 * r * c : 1) * sizeof(float), detail::cstream()),
                     "tinygnn allocation");
        owned = static_cast<float*>(q);
        detail::cuda(cudaMemcpy2DAsync(owned, c * sizeof(float), a.device_data(), a.device_ld() * sizeof(float),
                                       c * sizeof(float), r, cudaMemcpyDeviceToDevice, detail::cstream()),
                     "SAGELayer weights");
        detail::cuda(cudaMemcpy2DAsync(owned + r * c, c * sizeof(float), b.device_data(), b.device_ld() * sizeof(float),
                                       c * sizeof(float), r, cudaMemcpyDeviceToDevice, detail::cstream()),
                     "SAGELayer weights");
        wn = owned;
        ws = owned + r * c;
    }
    ~DevWeights() {
        if (owned && cudaFreeAsync(owned, detail::cstream()) != cudaSuccess) cudaGetLastError();
    }
    DevWeights(const DevWeights&) = delete;
    DevWeights& operator=(const DevWeights&) = delete;
};

inline std::string shape_str(std::size_t r, std::size_t c) {
    return "(" + std::to_string(r) + "\xC3\x97" + std::to_string(c) + ")";
}

}  // namespace detail

// Constructs tensors over device buffers the API has just produced.
struct TensorAccess {
    static Tensor csr_from_device(std::size_t rows, std::size_t cols, int32_t* d_rp, int32_t* d_ci, float* d_v,
                                  std::size_t nnz);
};

}  // namespace tinygnn

// The objects behind the handle C ABI's opaque pointers.
struct tg_tensor_s {
    tinygnn::Tensor t;
};
struct tg_model_s {
    tinygnn::Model m;
};
struct tg_graph_s {
    tinygnn::ForwardGraph g;
};
