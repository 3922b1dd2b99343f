// ============================================================================
//  api/tensor.cpp -- tinygnn::Tensor over device memory with a host mirror.
//
//  Construction and validation follow the reference's src/tensor.cpp:17-176
//  (same checks in the same order, same messages).  State: the device
//  buffers hold the values once they have been uploaded or produced by a
//  kernel; `host_valid` says whether the host vectors are current,
//  `device_valid` whether the device copy is.  Const host accessors download
//  when needed; non-const host accessors make the host copy authoritative;
//  device accessors upload when needed.  The CSR structure (row_ptr,
//  col_ind) never changes after construction.
// ============================================================================
#include <cstring>
#include <sstream>
#include <utility>

#include "internal.hpp"

namespace tinygnn {

namespace {
thread_local bool g_fast = false;

template <class T>
T* dev_alloc(std::size_t n) {
    void* p = nullptr;
    detail::cuda(cudaMallocAsync(&p, (n ? n : 1) * sizeof(T), detail::cstream()), "tinygnn::Tensor allocation");
    return static_cast<T*>(p);
}

void dev_free(void* p) {
    if (p && cudaFreeAsync(p, detail::cstream()) != cudaSuccess) cudaGetLastError();
}
}  // namespace

void set_fast_math(bool fast) noexcept { g_fast = fast; }
bool fast_math() noexcept { return g_fast; }

struct Tensor::Impl {
    StorageFormat format = StorageFormat::Dense;
    std::vector<std::size_t> shape{0, 0};
    std::vector<std::size_t> strides{0, 0};
    std::size_t nnz = 0;  // CSR entries

    mutable std::vector<float> h_data;
    mutable std::vector<int32_t> h_rp, h_ci;
    mutable bool host_valid = true;
    mutable bool host_struct_valid = true;  // CSR row_ptr / col_ind mirrors

    mutable float* d_data = nullptr;
    mutable int32_t* d_rp = nullptr;
    mutable int32_t* d_ci = nullptr;
    mutable bool device_valid = false;
    std::size_t ld = 0;  // dense device row stride

    // Set for tensors over caller-owned device memory: the buffers are not
    // ours to free, and the owner goes only after our queued work is done.
    std::shared_ptr<void> owner;
    bool external = false;

    ~Impl() {
        if (external) {
            if (cudaStreamSynchronize(detail::cstream()) != cudaSuccess) cudaGetLastError();
            owner.reset();
            return;
        }
        dev_free(d_data);
        dev_free(d_rp);
        dev_free(d_ci);
    }

    std::size_t rows() const { return shape[0]; }
    std::size_t cols() const { return shape[1]; }
    std::size_t count() const { return format == StorageFormat::Dense ? rows() * cols() : nnz; }

    void upload() const {
        if (device_valid) return;
        if (format == StorageFormat::Dense) {
            if (!d_data) d_data = dev_alloc<float>(rows() * ld);
            if (rows() && cols())
                detail::cuda(cudaMemcpy2DAsync(d_data, ld * sizeof(float), h_data.data(), cols() * sizeof(float),
                                               cols() * sizeof(float), rows(), cudaMemcpyHostToDevice,
                                               detail::cstream()),
                             "tinygnn::Tensor upload");
        } else {
            if (!d_rp) {
                d_rp = dev_alloc<int32_t>(rows() + 1);
                d_ci = dev_alloc<int32_t>(nnz);
                detail::cuda(cudaMemcpyAsync(d_rp, h_rp.data(), (rows() + 1) * sizeof(int32_t),
                                             cudaMemcpyHostToDevice, detail::cstream()),
                             "tinygnn::Tensor upload");
                if (nnz)
                    detail::cuda(cudaMemcpyAsync(d_ci, h_ci.data(), nnz * sizeof(int32_t), cudaMemcpyHostToDevice,
                                                 detail::cstream()),
                                 "tinygnn::Tensor upload");
            }
            if (!d_data) d_data = dev_alloc<float>(nnz);
            if (nnz)
                detail::cuda(cudaMemcpyAsync(d_data, h_data.data(), nnz * sizeof(float), cudaMemcpyHostToDevice,
                                             detail::cstream()),
                             "tinygnn::Tensor upload");
        }
        // The host vectors may be changed after this call returns: finish the copy.
        detail::cuda(cudaStreamSynchronize(detail::cstream()), "tinygnn::Tensor upload");
        device_valid = true;
    }

    void download() const {
        if (host_valid) return;
        h_data.resize(count());
        if (format == StorageFormat::Dense) {
            if (rows() && cols())
                detail::cuda(cudaMemcpy2DAsync(h_data.data(), cols() * sizeof(float), d_data, ld * sizeof(float),
                                               cols() * sizeof(float), rows(), cudaMemcpyDeviceToHost,
                                               detail::cstream()),
                             "tinygnn::Tensor download");
        } else if (nnz) {
            detail::cuda(cudaMemcpyAsync(h_data.data(), d_data, nnz * sizeof(float), cudaMemcpyDeviceToHost,
                                         detail::cstream()),
                         "tinygnn::Tensor download");
        }
        detail::cuda(cudaStreamSynchronize(detail::cstream()), "tinygnn::Tensor download");
        host_valid = true;
    }

    void download_struct() const {
        if (host_struct_valid || format != StorageFormat::SparseCSR) return;
        h_rp.resize(rows() + 1);
        h_ci.resize(nnz);
        detail::cuda(cudaMemcpyAsync(h_rp.data(), d_rp, (rows() + 1) * sizeof(int32_t), cudaMemcpyDeviceToHost,
                                     detail::cstream()),
                     "tinygnn::Tensor download");
        if (nnz)
            detail::cuda(cudaMemcpyAsync(h_ci.data(), d_ci, nnz * sizeof(int32_t), cudaMemcpyDeviceToHost,
                                         detail::cstream()),
                         "tinygnn::Tensor download");
        detail::cuda(cudaStreamSynchronize(detail::cstream()), "tinygnn::Tensor download");
        host_struct_valid = true;
    }

    std::unique_ptr<Impl> clone() const {
        auto c = std::make_unique<Impl>();
        c->format = format;
        c->shape = shape;
        c->strides = strides;
        c->nnz = nnz;
        c->ld = ld;
        c->host_valid = host_valid;
        c->host_struct_valid = host_struct_valid;
        if (host_valid) c->h_data = h_data;
        if (host_struct_valid) {
            c->h_rp = h_rp;
            c->h_ci = h_ci;
        }
        if (device_valid) {
            const std::size_t n = format == StorageFormat::Dense ? rows() * ld : nnz;
            c->d_data = dev_alloc<float>(n);
            if (n)
                detail::cuda(cudaMemcpyAsync(c->d_data, d_data, n * sizeof(float), cudaMemcpyDeviceToDevice,
                                             detail::cstream()),
                             "tinygnn::Tensor copy");
            c->device_valid = true;
        }
        if (format == StorageFormat::SparseCSR && d_rp && (device_valid || !host_struct_valid)) {
            c->d_rp = dev_alloc<int32_t>(rows() + 1);
            c->d_ci = dev_alloc<int32_t>(nnz);
            detail::cuda(cudaMemcpyAsync(c->d_rp, d_rp, (rows() + 1) * sizeof(int32_t), cudaMemcpyDeviceToDevice,
                                         detail::cstream()),
                         "tinygnn::Tensor copy");
            if (nnz)
                detail::cuda(cudaMemcpyAsync(c->d_ci, d_ci, nnz * sizeof(int32_t), cudaMemcpyDeviceToDevice,
                                             detail::cstream()),
                             "tinygnn::Tensor copy");
        }
        return c;
    }
};

Tensor::Tensor() : impl_(std::make_unique<Impl>()) {}
Tensor::Tensor(std::unique_ptr<Impl> impl) : impl_(std::move(impl)) {}
Tensor::Tensor(const Tensor& o) : impl_(o.impl_->clone()) {}
Tensor& Tensor::operator=(const Tensor& o) {
    if (this != &o) impl_ = o.impl_->clone();
    return *this;
}
Tensor::Tensor(Tensor&&) noexcept = default;
Tensor& Tensor::operator=(Tensor&&) noexcept = default;
Tensor::~Tensor() = default;

Tensor Tensor::dense(std::size_t rows, std::size_t cols) {
    return dense(rows, cols, std::vector<float>(rows * cols, 0.0f));
}

Tensor Tensor::dense(std::size_t rows, std::size_t cols, std::vector<float> data) {
    if (data.size() != rows * cols)
        throw std::invalid_argument("Tensor::dense: data.size() (" + std::to_string(data.size()) +
                                    ") != rows*cols (" + std::to_string(rows * cols) + ")");
    auto p = std::make_unique<Impl>();
    p->format = StorageFormat::Dense;
    p->shape = {rows, cols};
    p->strides = {cols, 1};
    p->ld = detail::pad4(cols);
    p->h_data = std::move(data);
    return Tensor(std::move(p));
}

Tensor Tensor::dense_device(std::size_t rows, std::size_t cols) {
    auto p = std::make_unique<Impl>();
    p->format = StorageFormat::Dense;
    p->shape = {rows, cols};
    p->strides = {cols, 1};
    p->ld = detail::pad4(cols);
    p->d_data = dev_alloc<float>(rows * p->ld);
    if (rows && p->ld)
        detail::cuda(cudaMemsetAsync(p->d_data, 0, rows * p->ld * sizeof(float), detail::cstream()),
                     "tinygnn::Tensor");
    p->device_valid = true;
    p->host_valid = false;
    return Tensor(std::move(p));
}

Tensor Tensor::sparse_csr(std::size_t rows, std::size_t cols, std::vector<int32_t> row_ptr,
                          std::vector<int32_t> col_ind, std::vector<float> values) {
    // The reference's checks and messages, in its order (src/tensor.cpp:142-182).
    if (row_ptr.size() != rows + 1)
        throw std::invalid_argument("Tensor::sparse_csr: row_ptr.size() (" + std::to_string(row_ptr.size()) +
                                    ") must equal rows+1 (" + std::to_string(rows + 1) + ")");
    if (col_ind.size() != values.size())
        throw std::invalid_argument("Tensor::sparse_csr: col_ind.size() (" + std::to_string(col_ind.size()) +
                                    ") must equal values.size() (" + std::to_string(values.size()) + ")");
    const auto nnz = static_cast<std::size_t>(row_ptr.back());
    if (nnz != values.size())
        throw std::invalid_argument("Tensor::sparse_csr: row_ptr.back() (" + std::to_string(nnz) +
                                    ") must equal values.size() (" + std::to_string(values.size()) + ")");
    for (std::size_t i = 0; i < col_ind.size(); ++i)
        if (col_ind[i] < 0 || static_cast<std::size_t>(col_ind[i]) >= cols)
            throw std::invalid_argument("Tensor::sparse_csr: col_ind[" + std::to_string(i) + "] = " +
                                        std::to_string(col_ind[i]) + " is out of bounds for cols=" +
                                        std::to_string(cols));
    for (std::size_t i = 1; i < row_ptr.size(); ++i)
        if (row_ptr[i] < row_ptr[i - 1])
            throw std::invalid_argument("Tensor::sparse_csr: row_ptr must be non-decreasing; row_ptr[" +
                                        std::to_string(i) + "] = " + std::to_string(row_ptr[i]) + " < row_ptr[" +
                                        std::to_string(i - 1) + "] = " + std::to_string(row_ptr[i - 1]));
    auto p = std::make_unique<Impl>();
    p->format = StorageFormat::SparseCSR;
    p->shape = {rows, cols};
    p->strides = {};
    p->nnz = nnz;
    p->h_rp = std::move(row_ptr);
    p->h_ci = std::move(col_ind);
    p->h_data = std::move(values);
    return Tensor(std::move(p));
}

Tensor Tensor::dense_from_device(std::size_t rows, std::size_t cols, std::size_t ld, float* data,
                                 std::shared_ptr<void> owner) {
    if (ld < cols)
        throw std::invalid_argument("Tensor::dense_from_device: row stride " + std::to_string(ld) + " < cols (" +
                                    std::to_string(cols) + ")");
    if (!data && rows && cols) throw std::invalid_argument("Tensor::dense_from_device: null data");
    auto p = std::make_unique<Impl>();
    p->format = StorageFormat::Dense;
    p->shape = {rows, cols};
    p->strides = {cols, 1};
    p->ld = ld;
    p->d_data = data;
    p->device_valid = true;
    p->host_valid = false;
    p->owner = std::move(owner);
    p->external = true;
    return Tensor(std::move(p));
}

Tensor Tensor::sparse_csr_from_device(std::size_t rows, std::size_t cols, std::size_t nnz, int32_t* row_ptr,
                                      int32_t* col_ind, float* values, std::shared_ptr<void> owner) {
    if (!row_ptr || ((!col_ind || !values) && nnz))
        throw std::invalid_argument("Tensor::sparse_csr_from_device: null array");
    detail::check(tg_csr_validate(static_cast<int64_t>(rows), static_cast<int64_t>(cols), static_cast<int64_t>(nnz),
                                  row_ptr, col_ind, detail::stream()));
    auto p = std::make_unique<Impl>();
    p->format = StorageFormat::SparseCSR;
    p->shape = {rows, cols};
    p->strides = {};
    p->nnz = nnz;
    p->d_rp = row_ptr;
    p->d_ci = col_ind;
    p->d_data = values;
    p->device_valid = true;
    p->host_valid = false;
    p->host_struct_valid = false;
    p->owner = std::move(owner);
    p->external = true;
    return Tensor(std::move(p));
}

Tensor TensorAccess::csr_from_device(std::size_t rows, std::size_t cols, int32_t* d_rp, int32_t* d_ci, float* d_v,
                                     std::size_t nnz) {
    auto p = std::make_unique<Tensor::Impl>();
    p->format = StorageFormat::SparseCSR;
    p->shape = {rows, cols};
    p->strides = {};
    p->nnz = nnz;
    p->d_rp = d_rp;
    p->d_ci = d_ci;
    p->d_data = d_v;
    p->device_valid = true;
    p->host_valid = false;
    p->host_struct_valid = false;
    return Tensor(std::move(p));
}

StorageFormat Tensor::format() const noexcept { return impl_->format; }
std::size_t Tensor::rows() const noexcept { return impl_->shape[0]; }
std::size_t Tensor::cols() const noexcept { return impl_->shape[1]; }
std::size_t Tensor::numel() const noexcept { return impl_->count(); }
std::size_t Tensor::ndim() const noexcept { return impl_->shape.size(); }
std::size_t Tensor::nnz() const noexcept { return impl_->count(); }
const std::vector<std::size_t>& Tensor::shape() const noexcept { return impl_->shape; }
const std::vector<std::size_t>& Tensor::strides() const noexcept { return impl_->strides; }
std::size_t Tensor::device_ld() const noexcept { return impl_->ld; }

std::size_t Tensor::memory_footprint_bytes() const noexcept {
    if (impl_->format == StorageFormat::Dense) return impl_->count() * sizeof(float);
    return impl_->nnz * (sizeof(float) + sizeof(int32_t)) + (rows() + 1) * sizeof(int32_t);
}

const std::vector<float>& Tensor::data() const {
    impl_->download();
    return impl_->h_data;
}

std::vector<float>& Tensor::data() {
    impl_->download();
    impl_->device_valid = false;  // the caller may write through the reference
    return impl_->h_data;
}

const std::vector<int32_t>& Tensor::row_ptr() const {
    impl_->download_struct();
    return impl_->h_rp;
}

const std::vector<int32_t>& Tensor::col_ind() const {
    impl_->download_struct();
    return impl_->h_ci;
}

float Tensor::at(std::size_t row, std::size_t col) const {
    if (impl_->format != StorageFormat::Dense)
        throw std::runtime_error("Tensor::at() is only supported for Dense tensors");
    if (row >= rows() || col >= cols())
        throw std::out_of_range("Tensor::at(" + std::to_string(row) + ", " + std::to_string(col) +
                                ") out of range for shape (" + std::to_string(rows()) + ", " +
                                std::to_string(cols()) + ")");
    return data()[row * cols() + col];
}

float& Tensor::at(std::size_t row, std::size_t col) {
    if (impl_->format != StorageFormat::Dense)
        throw std::runtime_error("Tensor::at() is only supported for Dense tensors");
    if (row >= rows() || col >= cols())
        throw std::out_of_range("Tensor::at(" + std::to_string(row) + ", " + std::to_string(col) +
                                ") out of range for shape (" + std::to_string(rows()) + ", " +
                                std::to_string(cols()) + ")");
    return data()[row * cols() + col];
}

std::string Tensor::repr() const {
    std::ostringstream os;
    os << "Tensor(" << rows() << "x" << cols() << ", "
       << (impl_->format == StorageFormat::Dense ? "Dense" : "SparseCSR") << ", " << memory_footprint_bytes()
       << " bytes)";
    return os.str();
}

const float* Tensor::device_data() const {
    impl_->upload();
    return impl_->d_data;
}

float* Tensor::mutable_device_data() {
    impl_->upload();
    impl_->host_valid = false;
    return impl_->d_data;
}

const int32_t* Tensor::device_row_ptr() const {
    if (impl_->format != StorageFormat::SparseCSR) return nullptr;
    impl_->upload();
    return impl_->d_rp;
}

const int32_t* Tensor::device_col_ind() const {
    if (impl_->format != StorageFormat::SparseCSR) return nullptr;
    impl_->upload();
    return impl_->d_ci;
}

}  // namespace tinygnn
