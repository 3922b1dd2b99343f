// ============================================================================
//  api/capi.cpp -- the handle half of the C ABI: tinygnn::Tensor and
//  tinygnn::Model behind opaque pointers (tg_tensor, tg_model), so that a
//  caller in any language that binds C (ctypes, cgo, JNI, N-API) drives the
//  same drop-in API as C++ code: build tensors from host buffers, build a
//  model, load its weights, run Model::forward, read the logits back.
//
//  Host buffers are only read (or written) inside the call: uploads and
//  downloads complete before it returns, from pinned memory at full PCIe
//  rate, from pageable memory through the driver's staging.  A CSR is
//  checked on the device after its upload with Tensor::sparse_csr's checks
//  (src/tensor.cpp:46-86) and refused with the reference's message.
// ============================================================================
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>

#include "internal.hpp"
#include "tinygnn/model.hpp"

namespace tg {
void set_last_error(const std::string& m);
void fill_f32(float* p, int64_t n, float v, cudaStream_t s);
}  // namespace tg


namespace {

using tinygnn::Tensor;
using tinygnn::detail::cstream;
using tinygnn::detail::cuda;

struct NoDevice : std::runtime_error {
    NoDevice() : std::runtime_error("tinygnn_b200: no CUDA device is visible; this library has no CPU path") {}
};

template <class F>
tg_status api(F&& f) noexcept {
    try {
        f();
        return TG_OK;
    } catch (const NoDevice& e) {
        tg::set_last_error(e.what());
        return TG_ERR_NO_DEVICE;
    } catch (const std::invalid_argument& e) {
        tg::set_last_error(e.what());
        return TG_ERR_INVALID_ARGUMENT;
    } catch (const std::out_of_range& e) {
        tg::set_last_error(e.what());
        return TG_ERR_OUT_OF_RANGE;
    } catch (const std::exception& e) {
        tg::set_last_error(e.what());
        return TG_ERR_RUNTIME;
    } catch (...) {
        tg::set_last_error("unknown error");
        return TG_ERR_RUNTIME;
    }
}

void need(const void* p, const char* what) {
    if (!p) throw std::invalid_argument(std::string(what) + " is NULL");
}

void no_device_check() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        throw NoDevice();
    }
}

tinygnn::Activation act_of(int32_t a) {
    if (a == TG_ACT_NONE) return tinygnn::Activation::None;
    if (a == TG_ACT_RELU) return tinygnn::Activation::ReLU;
    throw std::invalid_argument("layer activation must be TG_ACT_NONE or TG_ACT_RELU");
}

tinygnn::Model::InterActivation post_of(int32_t p) {
    if (p == 0) return tinygnn::Model::InterActivation::None;
    if (p == 1) return tinygnn::Model::InterActivation::ReLU;
    if (p == 2) return tinygnn::Model::InterActivation::ELU;
    throw std::invalid_argument("post activation must be 0 (none), 1 (ReLU) or 2 (ELU)");
}

template <class T>
T* device_alloc(std::size_t n) {
    void* p = nullptr;
    cuda(cudaMallocAsync(&p, (n ? n : 1) * sizeof(T), cstream()), "tinygnn allocation");
    return static_cast<T*>(p);
}

}  // namespace

extern "C" {

TG_API tg_status tg_tensor_create_dense(int64_t rows, int64_t cols, const float* host, int64_t ld, tg_tensor* out) {
    return api([&] {
        need(out, "tg_tensor_create_dense: out");
        *out = nullptr;
        if (rows < 0 || cols < 0) throw std::invalid_argument("Tensor::dense: negative size");
        if (host && ld < cols) throw std::invalid_argument("Tensor::dense: ld < cols");
        no_device_check();
        auto h = std::make_unique<tg_tensor_s>(tg_tensor_s{Tensor::dense_device(static_cast<std::size_t>(rows),
                                                                               static_cast<std::size_t>(cols))});
        const auto r = static_cast<std::size_t>(rows), c = static_cast<std::size_t>(cols);
        const std::size_t dld = h->t.device_ld();
        if (host && r && c) {
            if (static_cast<std::size_t>(ld) == dld) {
                cuda(cudaMemcpyAsync(h->t.mutable_device_data(), host, r * dld * sizeof(float), cudaMemcpyHostToDevice,
                                     cstream()),
                     "tg_tensor_create_dense");
            } else {
                // One DMA of the host rows as they lie, then the repack to the
                // device's 16-byte row stride on the device: a pitched host
                // copy moves each row separately.
                float* land = device_alloc<float>(r * static_cast<std::size_t>(ld));
                cuda(cudaMemcpyAsync(land, host, r * static_cast<std::size_t>(ld) * sizeof(float),
                                     cudaMemcpyHostToDevice, cstream()),
                     "tg_tensor_create_dense");
                cuda(cudaMemcpy2DAsync(h->t.mutable_device_data(), dld * sizeof(float), land,
                                       static_cast<std::size_t>(ld) * sizeof(float), c * sizeof(float), r,
                                       cudaMemcpyDeviceToDevice, cstream()),
                     "tg_tensor_create_dense");
                cuda(cudaFreeAsync(land, cstream()), "tg_tensor_create_dense");
            }
        }
        cuda(cudaStreamSynchronize(cstream()), "tg_tensor_create_dense");
        *out = h.release();
    });
}

TG_API tg_status tg_tensor_create_csr(int64_t rows, int64_t cols, int64_t nnz, const int32_t* row_ptr,
                                      const int32_t* col_ind, const float* values, tg_tensor* out) {
    return api([&] {
        need(out, "tg_tensor_create_csr: out");
        *out = nullptr;
        if (rows < 0 || cols < 0 || nnz < 0) throw std::invalid_argument("Tensor::sparse_csr: negative size");
        need(row_ptr, "Tensor::sparse_csr: row_ptr");
        if (nnz > 0) need(col_ind, "Tensor::sparse_csr: col_ind");
        no_device_check();
        const auto n1 = static_cast<std::size_t>(rows) + 1, nz = static_cast<std::size_t>(nnz);
        int32_t* d_rp = device_alloc<int32_t>(n1);
        int32_t* d_ci = device_alloc<int32_t>(nz);
        float* d_v = device_alloc<float>(nz);
        std::shared_ptr<void> owner(d_rp, [d_ci, d_v](void* p) {
            cudaFreeAsync(p, cstream());
            cudaFreeAsync(d_ci, cstream());
            cudaFreeAsync(d_v, cstream());
        });
        cuda(cudaMemcpyAsync(d_rp, row_ptr, n1 * sizeof(int32_t), cudaMemcpyHostToDevice, cstream()),
             "tg_tensor_create_csr");
        if (nz) {
            cuda(cudaMemcpyAsync(d_ci, col_ind, nz * sizeof(int32_t), cudaMemcpyHostToDevice, cstream()),
                 "tg_tensor_create_csr");
            if (values)
                cuda(cudaMemcpyAsync(d_v, values, nz * sizeof(float), cudaMemcpyHostToDevice, cstream()),
                     "tg_tensor_create_csr");
            else
                tg::fill_f32(d_v, nnz, 1.0f, cstream());  // an unweighted graph: every value 1.0
        }
        // validates on the device (the reference's messages) and synchronises
        auto h = std::make_unique<tg_tensor_s>(tg_tensor_s{Tensor::sparse_csr_from_device(
            static_cast<std::size_t>(rows), static_cast<std::size_t>(cols), nz, d_rp, d_ci, d_v, owner)});
        *out = h.release();
    });
}

}  // extern "C"

namespace {

// A dense tensor's values into host rows of stride ld; complete on return.
void download_dense(const Tensor& x, float* host, int64_t ld) {
    if (x.format() != tinygnn::StorageFormat::Dense)
        throw std::invalid_argument("tg_tensor_download: only Dense tensors can be downloaded");
    if (ld < static_cast<int64_t>(x.cols())) throw std::invalid_argument("tg_tensor_download: ld < cols");
    const std::size_t r = x.rows(), c = x.cols(), dld = x.device_ld();
    if (r && c) {
        if (static_cast<std::size_t>(ld) == dld) {
            cuda(cudaMemcpyAsync(host, x.device_data(), r * dld * sizeof(float), cudaMemcpyDeviceToHost, cstream()),
                 "tg_tensor_download");
        } else {
            // pack to the host's stride on the device, then one DMA
            float* pack = device_alloc<float>(r * static_cast<std::size_t>(ld));
            cuda(cudaMemcpy2DAsync(pack, static_cast<std::size_t>(ld) * sizeof(float), x.device_data(),
                                   dld * sizeof(float), c * sizeof(float), r, cudaMemcpyDeviceToDevice,
                                   cstream()),
                 "tg_tensor_download");
            cuda(cudaMemcpyAsync(host, pack, r * static_cast<std::size_t>(ld) * sizeof(float),
                                 cudaMemcpyDeviceToHost, cstream()),
                 "tg_tensor_download");
            cuda(cudaFreeAsync(pack, cstream()), "tg_tensor_download");
        }
    }
    cuda(cudaStreamSynchronize(cstream()), "tg_tensor_download");
}

}  // namespace

extern "C" {

TG_API tg_status tg_tensor_upload(tg_tensor t, const float* host, int64_t ld) {
    return api([&] {
        need(t, "tg_tensor_upload: t");
        need(host, "tg_tensor_upload: host");
        no_device_check();
        Tensor& x = t->t;
        if (x.format() == tinygnn::StorageFormat::SparseCSR) {
            if (x.nnz())
                cuda(cudaMemcpyAsync(x.mutable_device_data(), host, x.nnz() * sizeof(float), cudaMemcpyHostToDevice,
                                     cstream()),
                     "tg_tensor_upload");
        } else {
            const std::size_t r = x.rows(), c = x.cols(), dld = x.device_ld();
            if (ld < static_cast<int64_t>(c)) throw std::invalid_argument("tg_tensor_upload: ld < cols");
            if (r && c) {
                if (static_cast<std::size_t>(ld) == dld) {
                    cuda(cudaMemcpyAsync(x.mutable_device_data(), host, r * dld * sizeof(float),
                                         cudaMemcpyHostToDevice, cstream()),
                         "tg_tensor_upload");
                } else {  // one DMA of the host rows as they lie, then the repack on the device
                    float* land = device_alloc<float>(r * static_cast<std::size_t>(ld));
                    cuda(cudaMemcpyAsync(land, host, r * static_cast<std::size_t>(ld) * sizeof(float),
                                         cudaMemcpyHostToDevice, cstream()),
                         "tg_tensor_upload");
                    cuda(cudaMemcpy2DAsync(x.mutable_device_data(), dld * sizeof(float), land,
                                           static_cast<std::size_t>(ld) * sizeof(float), c * sizeof(float), r,
                                           cudaMemcpyDeviceToDevice, cstream()),
                         "tg_tensor_upload");
                    cuda(cudaFreeAsync(land, cstream()), "tg_tensor_upload");
                }
            }
        }
        cuda(cudaStreamSynchronize(cstream()), "tg_tensor_upload");
    });
}

TG_API tg_status tg_tensor_download(tg_tensor t, float* host, int64_t ld) {
    return api([&] {
        need(t, "tg_tensor_download: t");
        need(host, "tg_tensor_download: host");
        download_dense(t->t, host, ld);
    });
}

TG_API tg_status tg_tensor_shape(tg_tensor t, int64_t* rows, int64_t* cols, int64_t* nnz, int32_t* is_csr) {
    return api([&] {
        need(t, "tg_tensor_shape: t");
        if (rows) *rows = static_cast<int64_t>(t->t.rows());
        if (cols) *cols = static_cast<int64_t>(t->t.cols());
        if (nnz) *nnz = static_cast<int64_t>(t->t.nnz());
        if (is_csr) *is_csr = t->t.format() == tinygnn::StorageFormat::SparseCSR ? 1 : 0;
    });
}

TG_API void tg_tensor_free(tg_tensor t) { delete t; }

TG_API tg_status tg_model_create(tg_model* out) {
    return api([&] {
        need(out, "tg_model_create: out");
        *out = new tg_model_s();
    });
}

TG_API tg_status tg_model_add_gcn(tg_model m, int64_t in_f, int64_t out_f, int32_t bias, int32_t act, int32_t post) {
    return api([&] {
        need(m, "tg_model_add_gcn: m");
        if (in_f <= 0 || out_f <= 0) throw std::invalid_argument("GCNLayer: in_features and out_features must be > 0.");
        m->m.add_gcn_layer(static_cast<std::size_t>(in_f), static_cast<std::size_t>(out_f), bias != 0, act_of(act),
                           post_of(post));
    });
}

TG_API tg_status tg_model_add_sage(tg_model m, int64_t in_f, int64_t out_f, int32_t aggregator, int32_t bias,
                                   int32_t act, int32_t post) {
    return api([&] {
        need(m, "tg_model_add_sage: m");
        if (in_f <= 0 || out_f <= 0) throw std::invalid_argument("SAGELayer: in_features and out_features must be > 0.");
        m->m.add_sage_layer(static_cast<std::size_t>(in_f), static_cast<std::size_t>(out_f),
                            aggregator == TG_AGG_MAX ? tinygnn::SAGELayer::Aggregator::Max
                                                     : tinygnn::SAGELayer::Aggregator::Mean,
                            bias != 0, act_of(act), post_of(post));
    });
}

TG_API tg_status tg_model_add_gat(tg_model m, int64_t in_f, int64_t out_f, int64_t heads, int32_t concat, float slope,
                                  int32_t bias, int32_t act, int32_t post) {
    return api([&] {
        need(m, "tg_model_add_gat: m");
        if (in_f <= 0 || out_f <= 0 || heads <= 0)
            throw std::invalid_argument("GATLayer: in_features, out_features and heads must be > 0.");
        m->m.add_gat_layer(static_cast<std::size_t>(in_f), static_cast<std::size_t>(out_f),
                           static_cast<std::size_t>(heads), concat != 0, slope, bias != 0, act_of(act), post_of(post));
    });
}

TG_API tg_status tg_model_load_weights_file(tg_model m, const char* path) {
    return api([&] {
        need(m, "tg_model_load_weights_file: m");
        need(path, "tg_model_load_weights_file: path");
        m->m.load_weights(std::string(path));
    });
}

TG_API tg_status tg_model_load_weights(tg_model m, int32_t count, const char* const* names, const float* const* data,
                                       const int64_t* rows, const int64_t* cols) {
    return api([&] {
        need(m, "tg_model_load_weights: m");
        if (count < 0) throw std::invalid_argument("tg_model_load_weights: negative count");
        if (count > 0) {
            need(names, "tg_model_load_weights: names");
            need(data, "tg_model_load_weights: data");
            need(rows, "tg_model_load_weights: rows");
            need(cols, "tg_model_load_weights: cols");
        }
        tinygnn::WeightFile wf;
        for (int32_t i = 0; i < count; ++i) {
            need(names[i], "tg_model_load_weights: names[i]");
            if (rows[i] < 0 || cols[i] < 0) throw std::invalid_argument("tg_model_load_weights: negative shape");
            const auto r = static_cast<std::size_t>(rows[i]), c = static_cast<std::size_t>(cols[i]);
            if (r * c != 0) need(data[i], "tg_model_load_weights: data[i]");
            std::vector<float> v(r * c);
            if (r * c != 0) std::memcpy(v.data(), data[i], r * c * sizeof(float));
            wf.tensors.emplace(std::string(names[i]), Tensor::dense(r, c, std::move(v)));
        }
        m->m.load_weights(wf);
    });
}

TG_API tg_status tg_model_forward(tg_model m, tg_tensor adjacency, tg_tensor features, tg_tensor* out) {
    return api([&] {
        need(m, "tg_model_forward: m");
        need(adjacency, "tg_model_forward: adjacency");
        need(features, "tg_model_forward: features");
        need(out, "tg_model_forward: out");
        *out = nullptr;
        no_device_check();
        auto h = std::make_unique<tg_tensor_s>(tg_tensor_s{m->m.forward(adjacency->t, features->t)});
        cuda(cudaStreamSynchronize(cstream()), "tg_model_forward");  // complete on return, like every handle call
        *out = h.release();
    });
}

TG_API tg_status tg_model_forward_host(tg_model m, int64_t n, int64_t nnz, const int32_t* row_ptr,
                                       const int32_t* col_ind, const float* values, const float* features,
                                       int64_t feature_cols, int64_t ld_features, float* out, int64_t out_cols,
                                       int64_t ld_out) {
    return api([&] {
        need(m, "tg_model_forward_host: m");
        if (n < 0 || nnz < 0 || feature_cols < 0 || ld_features < 0 || out_cols < 0 || ld_out < 0)
            throw std::invalid_argument("tg_model_forward_host: negative size");
        need(row_ptr, "tg_model_forward_host: row_ptr");
        no_device_check();
        m->m.forward_host(static_cast<std::size_t>(n), static_cast<std::size_t>(nnz), row_ptr, col_ind, values,
                          features, static_cast<std::size_t>(feature_cols), static_cast<std::size_t>(ld_features),
                          out, static_cast<std::size_t>(out_cols), static_cast<std::size_t>(ld_out));
    });
}

TG_API void tg_model_free(tg_model m) { delete m; }

TG_API tg_status tg_model_capture(tg_model m, tg_tensor adjacency, tg_tensor features, tg_graph* out) {
    return api([&] {
        need(m, "tg_model_capture: m");
        need(adjacency, "tg_model_capture: adjacency");
        need(features, "tg_model_capture: features");
        need(out, "tg_model_capture: out");
        *out = nullptr;
        no_device_check();
        auto h = std::make_unique<tg_graph_s>(tg_graph_s{m->m.capture(adjacency->t, features->t)});
        *out = h.release();
    });
}

TG_API tg_status tg_graph_replay(tg_graph g) {
    return api([&] {
        need(g, "tg_graph_replay: g");
        g->g.replay();
        cuda(cudaStreamSynchronize(cstream()), "tg_graph_replay");
    });
}

TG_API tg_status tg_graph_download(tg_graph g, float* host, int64_t ld) {
    return api([&] {
        need(g, "tg_graph_download: g");
        need(host, "tg_graph_download: host");
        download_dense(g->g.output(), host, ld);
    });
}

TG_API void tg_graph_free(tg_graph g) { delete g; }

TG_API int32_t tg_set_fast_math(int32_t fast) {
    const int32_t prev = tinygnn::fast_math() ? 1 : 0;
    tinygnn::set_fast_math(fast != 0);
    return prev;
}

}  // extern "C"
