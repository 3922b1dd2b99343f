// ============================================================================
//  tinygnn/tensor.hpp -- device-resident Tensor with TinyGNN's interface.
//
//  Source-compatible with TinyGNN's Tensor (include/tinygnn/tensor.hpp:25-94
//  of the reference): Dense (row-major fp32) or SparseCSR (int32 row_ptr /
//  col_ind, fp32 values), the same factories, observers, accessors and
//  exceptions.  The authoritative copy lives in B200 HBM; the host vectors
//  returned by data() / row_ptr() / col_ind() / at() are a mirror that is
//  downloaded on first host access after the device copy changed, and a
//  non-const host access (data(), at()) marks the mirror as newer, so the
//  next device use uploads it.  Copies are deep (device to device); moves
//  are cheap.  Dense device rows are padded to a multiple of 4 floats
//  (16-byte rows for vector loads and TMA); device_ld() gives the stride.
// ============================================================================
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <vector>

namespace tinygnn {

enum class StorageFormat : uint8_t {
    Dense = 0,      // row-major fp32
    SparseCSR = 1   // compressed sparse row
};

struct Tensor {
    // ── construction (tensor.hpp:28-46 of the reference) ────────────────────
    Tensor();
    static Tensor dense(std::size_t rows, std::size_t cols);
    static Tensor dense(std::size_t rows, std::size_t cols, std::vector<float> data);
    static Tensor sparse_csr(std::size_t rows, std::size_t cols, std::vector<int32_t> row_ptr,
                             std::vector<int32_t> col_ind, std::vector<float> values);

    Tensor(const Tensor& other);
    Tensor& operator=(const Tensor& other);
    Tensor(Tensor&&) noexcept;
    Tensor& operator=(Tensor&&) noexcept;
    ~Tensor();

    // ── observers ───────────────────────────────────────────────────────────
    StorageFormat format() const noexcept;
    std::size_t rows() const noexcept;
    std::size_t cols() const noexcept;
    std::size_t numel() const noexcept;
    std::size_t ndim() const noexcept;
    std::size_t nnz() const noexcept;
    std::size_t memory_footprint_bytes() const noexcept;
    const std::vector<std::size_t>& shape() const noexcept;
    const std::vector<std::size_t>& strides() const noexcept;

    // ── host accessors (synchronise the mirror) ─────────────────────────────
    const std::vector<float>& data() const;
    std::vector<float>& data();
    const std::vector<int32_t>& row_ptr() const;
    const std::vector<int32_t>& col_ind() const;
    float at(std::size_t row, std::size_t col) const;
    float& at(std::size_t row, std::size_t col);
    std::string repr() const;

    // ── device side (B200 extension) ────────────────────────────────────────
    // Dense: rows x cols on the device, zero-filled, no host mirror yet.
    static Tensor dense_device(std::size_t rows, std::size_t cols);
    const float* device_data() const;      // values (dense or CSR), uploaded if the host is newer
    float* mutable_device_data();          // the host mirror becomes stale
    const int32_t* device_row_ptr() const;
    const int32_t* device_col_ind() const;
    std::size_t device_ld() const noexcept;  // dense: device row stride (>= cols)

    // Tensors over caller-owned device memory on the current device (zero
    // copy; DLPack / torch interop).  The tensor reads and writes that
    // memory in place and never frees it; `owner` (may be null) is kept
    // alive while the tensor exists and released after the tensor's pending
    // device work has finished.  Copies of such a tensor own their memory.
    // Dense: rows x cols at row stride `ld` >= cols floats.
    static Tensor dense_from_device(std::size_t rows, std::size_t cols, std::size_t ld, float* data,
                                    std::shared_ptr<void> owner);
    // CSR: row_ptr[rows + 1], col_ind[nnz], values[nnz]; validated on the
    // device with Tensor::sparse_csr's checks and messages.
    static Tensor sparse_csr_from_device(std::size_t rows, std::size_t cols, std::size_t nnz, int32_t* row_ptr,
                                         int32_t* col_ind, float* values, std::shared_ptr<void> owner);

    struct Impl;

private:
    std::unique_ptr<Impl> impl_;
    explicit Tensor(std::unique_ptr<Impl> impl);
    friend struct TensorAccess;
};

// Selects the arithmetic of the ops/layers/Model entry points of this API:
// exact (default; bit-identical to TinyGNN's CPU library where the kernel is
// exact) or fast (3xTF32 tensor-core GEMMs, SAGE transform-first; within
// |d| <= 1e-5 + 1e-4|ref|).  Per thread.
void set_fast_math(bool fast) noexcept;
bool fast_math() noexcept;

}  // namespace tinygnn
