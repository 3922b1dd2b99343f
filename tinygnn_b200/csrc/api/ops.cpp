// ============================================================================
//  api/ops.cpp -- tinygnn:: operators on device tensors (reference
//  src/ops.cpp:70-661): host-side validation with the reference's
//  messages, then one C-ABI call per op.
// ============================================================================
#include "tinygnn/ops.hpp"

#include "internal.hpp"

namespace tinygnn {

using detail::check;
using detail::stream;

namespace {
void require_dense(const Tensor& X, const char* fn) {
    if (X.format() != StorageFormat::Dense)
        throw std::invalid_argument(std::string(fn) +
                                    ": tensor must be Dense (got SparseCSR). "
                                    "Activations operate on dense feature matrices only.");
}

void act(Tensor& X, int kind, float alpha, const char* fn) {
    require_dense(X, fn);
    if (X.rows() == 0 || X.cols() == 0) return;
    check(tg_activation_f32(kind, alpha, X.mutable_device_data(), static_cast<int64_t>(X.rows()),
                            static_cast<int64_t>(X.cols()), static_cast<int64_t>(X.device_ld()), stream()));
}
}  // namespace

Tensor matmul(const Tensor& A, const Tensor& B) {
    if (A.format() != StorageFormat::Dense)
        throw std::invalid_argument(
            "matmul: tensor A must be Dense (got SparseCSR). Sparse-dense matmul is planned for Phase 4 (SpMM kernel).");
    if (B.format() != StorageFormat::Dense)
        throw std::invalid_argument(
            "matmul: tensor B must be Dense (got SparseCSR). Sparse-dense matmul is planned for Phase 4 (SpMM kernel).");
    const std::size_t M = A.rows(), K = A.cols(), K2 = B.rows(), N = B.cols();
    if (K != K2)
        throw std::invalid_argument("matmul: dimension mismatch \xE2\x80\x94 A is " + detail::shape_str(M, K) +
                                    " but B is " + detail::shape_str(K2, N) +
                                    ". Required: A.cols() == B.rows() (both = " + std::to_string(K) + " vs " +
                                    std::to_string(K2) + ").");
    Tensor C = Tensor::dense_device(M, N);
    if (M == 0 || N == 0) return C;
    check(tg_gemm_f32(static_cast<int64_t>(M), static_cast<int64_t>(N), static_cast<int64_t>(K),
                      K ? A.device_data() : nullptr, static_cast<int64_t>(A.device_ld()),
                      K ? B.device_data() : nullptr, static_cast<int64_t>(B.device_ld()), C.mutable_device_data(),
                      static_cast<int64_t>(C.device_ld()), nullptr, TG_ACT_NONE, 0.0f, detail::mode(), stream()));
    return C;
}

Tensor spmm(const Tensor& A, const Tensor& B) {
    if (A.format() != StorageFormat::SparseCSR)
        throw std::invalid_argument(
            "spmm: tensor A must be SparseCSR (got Dense). For Dense \xC3\x97 Dense, use matmul() instead.");
    if (B.format() != StorageFormat::Dense)
        throw std::invalid_argument(
            "spmm: tensor B must be Dense (got SparseCSR). Sparse \xC3\x97 Sparse multiplication is not supported.");
    const std::size_t M = A.rows(), K = A.cols(), K2 = B.rows(), N = B.cols();
    if (K != K2)
        throw std::invalid_argument("spmm: dimension mismatch \xE2\x80\x94 A is (" + std::to_string(M) + "\xC3\x97" +
                                    std::to_string(K) + ", SparseCSR) but B is (" + std::to_string(K2) + "\xC3\x97" +
                                    std::to_string(N) + ", Dense). Required: A.cols() == B.rows() (" +
                                    std::to_string(K) + " vs " + std::to_string(K2) + ").");
    Tensor C = Tensor::dense_device(M, N);
    if (M == 0 || N == 0 || A.nnz() == 0) return C;  // zeros (ops.cpp:234)
    const detail::TrustedCsr trusted_csr;
    check(tg_spmm_f32(static_cast<int64_t>(M), static_cast<int64_t>(K), static_cast<int64_t>(A.nnz()),
                      A.device_row_ptr(), A.device_col_ind(), A.device_data(), B.device_data(),
                      static_cast<int64_t>(N), static_cast<int64_t>(B.device_ld()), C.mutable_device_data(),
                      static_cast<int64_t>(C.device_ld()), nullptr, TG_ACT_NONE, 0.0f, nullptr,
                      detail::mode() | TG_FLAG_B_ROWS_PADDED, stream()));
    return C;
}

void relu_inplace(Tensor& X) { act(X, TG_ACT_RELU, 0.0f, "relu_inplace"); }
void leaky_relu_inplace(Tensor& X, float alpha) { act(X, TG_ACT_LEAKY_RELU, alpha, "leaky_relu_inplace"); }
void elu_inplace(Tensor& X, float alpha) { act(X, TG_ACT_ELU, alpha, "elu_inplace"); }
void sigmoid_inplace(Tensor& X) { act(X, TG_ACT_SIGMOID, 0.0f, "sigmoid_inplace"); }
void tanh_inplace(Tensor& X) { act(X, TG_ACT_TANH, 0.0f, "tanh_inplace"); }
void gelu_inplace(Tensor& X) { act(X, TG_ACT_GELU, 0.0f, "gelu_inplace"); }

void softmax_inplace(Tensor& X) {
    require_dense(X, "softmax_inplace");
    if (X.cols() == 0)
        throw std::invalid_argument(
            "softmax_inplace: tensor has 0 columns \xE2\x80\x94 softmax over an empty set is undefined.");
    if (X.rows() == 0) return;
    check(tg_softmax_rows_f32(X.mutable_device_data(), static_cast<int64_t>(X.rows()),
                              static_cast<int64_t>(X.cols()), static_cast<int64_t>(X.device_ld()), stream()));
}

void log_softmax_inplace(Tensor& X) {
    require_dense(X, "log_softmax_inplace");
    if (X.cols() == 0)
        throw std::invalid_argument(
            "log_softmax_inplace: tensor has 0 columns \xE2\x80\x94 log-softmax over an empty set is undefined.");
    if (X.rows() == 0) return;
    check(tg_log_softmax_rows_f32(X.mutable_device_data(), static_cast<int64_t>(X.rows()),
                                  static_cast<int64_t>(X.cols()), static_cast<int64_t>(X.device_ld()), stream()));
}

void add_bias(Tensor& X, const Tensor& bias) {
    require_dense(X, "add_bias (X)");
    if (bias.format() != StorageFormat::Dense)
        throw std::invalid_argument("add_bias: bias tensor must be Dense (got SparseCSR).");
    const std::size_t N = X.cols();
    if (bias.rows() != 1 || bias.cols() != N)
        throw std::invalid_argument("add_bias: bias must be shape (1\xC3\x97" + std::to_string(N) +
                                    ") to match X columns, but got " + detail::shape_str(bias.rows(), bias.cols()) +
                                    ".");
    if (X.rows() == 0 || N == 0) return;
    check(tg_add_bias_f32(X.mutable_device_data(), static_cast<int64_t>(X.rows()), static_cast<int64_t>(N),
                          static_cast<int64_t>(X.device_ld()), bias.device_data(), stream()));
}

}  // namespace tinygnn
