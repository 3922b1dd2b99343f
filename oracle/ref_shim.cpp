// ============================================================================
//  oracle/ref_shim.cpp -- TEST INFRASTRUCTURE ONLY.
//
//  A flat extern "C" surface over the *unmodified* TinyGNN CPU library,
//  compiled from the reference sources with the namespace renamed to
//  `tinygnn_ref` (see oracle/Makefile).  The resulting
//  oracle/_ref/libtinygnn_ref.so is the reference implementation itself; the
//  parity tests call it to pin the C restatement (oracle/tg_oracle.c) and the
//  CUDA path, and bench.py's reference arm times it.  Nothing in the product
//  library (tinygnn_b200/) links or loads this file.
//
//  Every function returns 0 on success, or 1/2/3 when the reference threw
//  std::invalid_argument / std::out_of_range / another exception; the message
//  is available from ref_last_error().
// ============================================================================
#include "tinygnn/graph_loader.hpp"
#include "tinygnn/layers.hpp"
#include "tinygnn/model.hpp"
#include "tinygnn/ops.hpp"
#include "tinygnn/tensor.hpp"

#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace R = tinygnn_ref;

namespace {
thread_local std::string g_err;

template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::invalid_argument& e) {
        g_err = e.what();
        return 1;
    } catch (const std::out_of_range& e) {
        g_err = e.what();
        return 2;
    } catch (const std::exception& e) {
        g_err = e.what();
        return 3;
    }
}

R::Tensor csr(int64_t rows, int64_t cols, int64_t nnz, const int32_t* rp,
              const int32_t* ci, const float* v) {
    return R::Tensor::sparse_csr(
        static_cast<std::size_t>(rows), static_cast<std::size_t>(cols),
        std::vector<int32_t>(rp, rp + rows + 1),
        std::vector<int32_t>(ci, ci + nnz), std::vector<float>(v, v + nnz));
}

R::Tensor dense(int64_t rows, int64_t cols, const float* x) {
    return R::Tensor::dense(static_cast<std::size_t>(rows),
                            static_cast<std::size_t>(cols),
                            std::vector<float>(x, x + rows * cols));
}

void out_dense(const R::Tensor& t, float* out) {
    std::memcpy(out, t.data().data(), t.data().size() * sizeof(float));
}

// Copies a CSR result out; *nnz_io holds the capacity on entry and the
// number of stored entries on return.
void out_csr(const R::Tensor& t, int32_t* rp, int32_t* ci, float* v,
             int64_t* nnz_io) {
    const auto nnz = static_cast<int64_t>(t.nnz());
    if (nnz > *nnz_io) throw std::runtime_error("ref_shim: output capacity too small");
    std::memcpy(rp, t.row_ptr().data(), t.row_ptr().size() * sizeof(int32_t));
    std::memcpy(ci, t.col_ind().data(), static_cast<std::size_t>(nnz) * sizeof(int32_t));
    std::memcpy(v, t.data().data(), static_cast<std::size_t>(nnz) * sizeof(float));
    *nnz_io = nnz;
}

R::Activation act_of(int a) { return a ? R::Activation::ReLU : R::Activation::None; }
}  // namespace

extern "C" {

const char* ref_last_error(void) { return g_err.c_str(); }

void ref_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int ref_get_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

int ref_matmul(int64_t M, int64_t K, int64_t N, const float* A, const float* B,
               float* C) {
    return guarded([&] { out_dense(R::matmul(dense(M, K, A), dense(K, N, B)), C); });
}

int ref_spmm(int64_t M, int64_t K, int64_t nnz, const int32_t* rp,
             const int32_t* ci, const float* v, const float* B, int64_t F,
             float* C) {
    return guarded([&] { out_dense(R::spmm(csr(M, K, nnz, rp, ci, v), dense(K, F, B)), C); });
}

// kind: 0 relu, 1 leaky_relu(alpha), 2 elu(alpha), 3 sigmoid, 4 tanh,
//       5 gelu, 6 softmax, 7 log_softmax
int ref_activation(int kind, float alpha, float* X, int64_t rows, int64_t cols) {
    return guarded([&] {
        R::Tensor t = dense(rows, cols, X);
        switch (kind) {
            case 0: R::relu_inplace(t); break;
            case 1: R::leaky_relu_inplace(t, alpha); break;
            case 2: R::elu_inplace(t, alpha); break;
            case 3: R::sigmoid_inplace(t); break;
            case 4: R::tanh_inplace(t); break;
            case 5: R::gelu_inplace(t); break;
            case 6: R::softmax_inplace(t); break;
            case 7: R::log_softmax_inplace(t); break;
            default: throw std::invalid_argument("ref_activation: bad kind");
        }
        out_dense(t, X);
    });
}

int ref_add_bias(float* X, int64_t rows, int64_t cols, const float* b,
                 int64_t b_rows, int64_t b_cols) {
    return guarded([&] {
        R::Tensor t = dense(rows, cols, X);
        R::add_bias(t, dense(b_rows, b_cols, b));
        out_dense(t, X);
    });
}

int ref_add_self_loops(int64_t N, int64_t nnz, const int32_t* rp,
                       const int32_t* ci, const float* v, int32_t* rp_out,
                       int32_t* ci_out, float* v_out, int64_t* nnz_io) {
    return guarded([&] {
        out_csr(R::add_self_loops(csr(N, N, nnz, rp, ci, v)), rp_out, ci_out, v_out, nnz_io);
    });
}

int ref_gcn_norm(int64_t N, int64_t nnz, const int32_t* rp, const int32_t* ci,
                 const float* v, int32_t* rp_out, int32_t* ci_out,
                 float* v_out, int64_t* nnz_io) {
    return guarded([&] {
        out_csr(R::gcn_norm(csr(N, N, nnz, rp, ci, v)), rp_out, ci_out, v_out, nnz_io);
    });
}

int ref_edge_softmax(int64_t rows, int64_t cols, int64_t nnz, const int32_t* rp,
                     const int32_t* ci, const float* v, float* v_out) {
    return guarded([&] {
        R::Tensor t = R::edge_softmax(csr(rows, cols, nnz, rp, ci, v));
        std::memcpy(v_out, t.data().data(), static_cast<std::size_t>(nnz) * sizeof(float));
    });
}

int ref_sage_max_aggregate(int64_t rows, int64_t cols, int64_t nnz,
                           const int32_t* rp, const int32_t* ci,
                           const float* v, const float* H, int64_t F,
                           float* out) {
    return guarded([&] {
        out_dense(R::sage_max_aggregate(csr(rows, cols, nnz, rp, ci, v), dense(cols, F, H)), out);
    });
}

int ref_edge_list_to_csr(int64_t num_nodes, int64_t E, const int32_t* src,
                         const int32_t* dst, int32_t* rp_out, int32_t* ci_out,
                         float* v_out) {
    return guarded([&] {
        std::vector<std::pair<int32_t, int32_t>> edges(static_cast<std::size_t>(E));
        for (int64_t i = 0; i < E; ++i) edges[static_cast<std::size_t>(i)] = {src[i], dst[i]};
        R::Tensor t = R::GraphLoader::edge_list_to_csr(edges, static_cast<std::size_t>(num_nodes));
        int64_t cap = E;
        out_csr(t, rp_out, ci_out, v_out, &cap);
    });
}

int ref_gcn_layer(int64_t N, int64_t nnz, const int32_t* rp, const int32_t* ci,
                  const float* v, const float* H, int64_t F_in, int64_t F_out,
                  const float* W, const float* bias, int act, float* out) {
    return guarded([&] {
        R::GCNLayer layer(static_cast<std::size_t>(F_in), static_cast<std::size_t>(F_out),
                          bias != nullptr, act_of(act));
        layer.set_weight(dense(F_in, F_out, W));
        if (bias) layer.set_bias(dense(1, F_out, bias));
        out_dense(layer.forward(csr(N, N, nnz, rp, ci, v), dense(N, F_in, H)), out);
    });
}

int ref_sage_layer(int64_t N, int64_t nnz, const int32_t* rp, const int32_t* ci,
                   const float* v, const float* H, int64_t F_in, int64_t F_out,
                   const float* Wn, const float* Ws, const float* bias,
                   int agg_max, int act, float* out) {
    return guarded([&] {
        R::SAGELayer layer(static_cast<std::size_t>(F_in), static_cast<std::size_t>(F_out),
                           agg_max ? R::SAGELayer::Aggregator::Max : R::SAGELayer::Aggregator::Mean,
                           bias != nullptr, act_of(act));
        layer.set_weight_neigh(dense(F_in, F_out, Wn));
        layer.set_weight_self(dense(F_in, F_out, Ws));
        if (bias) layer.set_bias(dense(1, F_out, bias));
        out_dense(layer.forward(csr(N, N, nnz, rp, ci, v), dense(N, F_in, H)), out);
    });
}

int ref_gat_layer(int64_t N, int64_t nnz, const int32_t* rp, const int32_t* ci,
                  const float* v, const float* H, int64_t F_in, int64_t F_out,
                  const float* W, const float* a_l, const float* a_r,
                  const float* bias, float neg_slope, int act, float* out) {
    return guarded([&] {
        R::GATLayer layer(static_cast<std::size_t>(F_in), static_cast<std::size_t>(F_out),
                          neg_slope, bias != nullptr, act_of(act));
        layer.set_weight(dense(F_in, F_out, W));
        layer.set_attn_left(dense(1, F_out, a_l));
        layer.set_attn_right(dense(1, F_out, a_r));
        if (bias) layer.set_bias(dense(1, F_out, bias));
        out_dense(layer.forward(csr(N, N, nnz, rp, ci, v), dense(N, F_in, H)), out);
    });
}

// ── Model: built incrementally, weights staged by name, then forward ──────
struct RefModel {
    R::Model model;
    R::WeightFile wf;
    std::size_t out_cols = 0;
};

void* ref_model_create(void) { return new RefModel(); }
void ref_model_free(void* m) { delete static_cast<RefModel*>(m); }

int ref_model_add_gcn(void* m, int64_t in_f, int64_t out_f, int bias, int act, int post) {
    return guarded([&] {
        auto* rm = static_cast<RefModel*>(m);
        rm->model.add_gcn_layer(static_cast<std::size_t>(in_f), static_cast<std::size_t>(out_f),
                                bias != 0, act_of(act),
                                static_cast<R::Model::InterActivation>(post));
        rm->out_cols = static_cast<std::size_t>(out_f);
    });
}

int ref_model_add_sage(void* m, int64_t in_f, int64_t out_f, int agg_max, int bias,
                       int act, int post) {
    return guarded([&] {
        auto* rm = static_cast<RefModel*>(m);
        rm->model.add_sage_layer(static_cast<std::size_t>(in_f), static_cast<std::size_t>(out_f),
                                 agg_max ? R::SAGELayer::Aggregator::Max
                                         : R::SAGELayer::Aggregator::Mean,
                                 bias != 0, act_of(act),
                                 static_cast<R::Model::InterActivation>(post));
        rm->out_cols = static_cast<std::size_t>(out_f);
    });
}

int ref_model_add_gat(void* m, int64_t in_f, int64_t out_f, int64_t heads, int concat,
                      float neg_slope, int bias, int act, int post) {
    return guarded([&] {
        auto* rm = static_cast<RefModel*>(m);
        rm->model.add_gat_layer(static_cast<std::size_t>(in_f), static_cast<std::size_t>(out_f),
                                static_cast<std::size_t>(heads), concat != 0, neg_slope,
                                bias != 0, act_of(act),
                                static_cast<R::Model::InterActivation>(post));
        rm->out_cols = static_cast<std::size_t>(concat ? out_f * heads : out_f);
    });
}

int ref_model_set_tensor(void* m, const char* name, const float* data, int64_t rows,
                         int64_t cols) {
    return guarded([&] {
        static_cast<RefModel*>(m)->wf.tensors[name] = dense(rows, cols, data);
    });
}

int ref_model_load(void* m) {
    return guarded([&] {
        auto* rm = static_cast<RefModel*>(m);
        rm->model.load_weights(rm->wf);
    });
}

int ref_model_load_file(void* m, const char* path) {
    return guarded([&] { static_cast<RefModel*>(m)->model.load_weights(std::string(path)); });
}

// Full Model::forward on a raw (no self-loop) adjacency; the caller then
// applies log_softmax separately when the reference test does.
int ref_model_forward(void* m, int64_t N, int64_t nnz, const int32_t* rp,
                      const int32_t* ci, const float* v, const float* X,
                      int64_t F, float* out) {
    return guarded([&] {
        auto* rm = static_cast<RefModel*>(m);
        out_dense(rm->model.forward(csr(N, N, nnz, rp, ci, v), dense(N, F, X)), out);
    });
}

// Same forward on Tensors that the caller pre-built once, so timing loops
// measure Model::forward itself rather than the copies into std::vector.
void* ref_tensor_csr(int64_t N, int64_t nnz, const int32_t* rp, const int32_t* ci,
                     const float* v) {
    try {
        return new R::Tensor(csr(N, N, nnz, rp, ci, v));
    } catch (const std::exception& e) {
        g_err = e.what();
        return nullptr;
    }
}

void* ref_tensor_dense(int64_t rows, int64_t cols, const float* x) {
    try {
        return new R::Tensor(dense(rows, cols, x));
    } catch (const std::exception& e) {
        g_err = e.what();
        return nullptr;
    }
}

void ref_tensor_free(void* t) { delete static_cast<R::Tensor*>(t); }

int ref_model_forward_tensors(void* m, const void* adj, const void* X, float* out,
                              int log_softmax) {
    return guarded([&] {
        auto* rm = static_cast<RefModel*>(m);
        R::Tensor y = rm->model.forward(*static_cast<const R::Tensor*>(adj),
                                        *static_cast<const R::Tensor*>(X));
        if (log_softmax) R::log_softmax_inplace(y);
        if (out) out_dense(y, out);
    });
}

// ── The layers alone ──────────────────────────────────────────────────────
// A stack of the reference's GCN / SAGE layer objects run on an adjacency
// prepared once (gcn_norm for GCN layers, the raw one for SAGE): what
// Model::forward does per layer, without its per-call normalisation
// (src/model.cpp:365-381), for timing the layer forwards by themselves.
struct RefStack {
    std::vector<int> kind;     // 0 GCN, 1 SAGE
    std::vector<int> post;     // 0 none, 1 ReLU, 2 ELU (alpha 1)
    std::vector<R::GCNLayer> gcn;
    std::vector<R::SAGELayer> sage;
};

void* ref_stack_create(void) { return new RefStack(); }
void ref_stack_free(void* s) { delete static_cast<RefStack*>(s); }

int ref_stack_add_gcn(void* s, int64_t in_f, int64_t out_f, int act, int post, const float* W,
                      const float* b) {
    return guarded([&] {
        auto* st = static_cast<RefStack*>(s);
        R::GCNLayer L(static_cast<std::size_t>(in_f), static_cast<std::size_t>(out_f), b != nullptr,
                      act_of(act));
        L.set_weight(dense(in_f, out_f, W));
        if (b) L.set_bias(dense(1, out_f, b));
        st->gcn.push_back(std::move(L));
        st->kind.push_back(0);
        st->post.push_back(post);
    });
}

int ref_stack_add_sage(void* s, int64_t in_f, int64_t out_f, int agg_max, int act, int post,
                       const float* Wn, const float* Ws, const float* b) {
    return guarded([&] {
        auto* st = static_cast<RefStack*>(s);
        R::SAGELayer L(static_cast<std::size_t>(in_f), static_cast<std::size_t>(out_f),
                       agg_max ? R::SAGELayer::Aggregator::Max : R::SAGELayer::Aggregator::Mean,
                       b != nullptr, act_of(act));
        L.set_weight_neigh(dense(in_f, out_f, Wn));
        L.set_weight_self(dense(in_f, out_f, Ws));
        if (b) L.set_bias(dense(1, out_f, b));
        st->sage.push_back(std::move(L));
        st->kind.push_back(1);
        st->post.push_back(post);
    });
}

// gcn_norm of a pre-built CSR Tensor, as a new Tensor (free with ref_tensor_free).
void* ref_gcn_norm_tensor(const void* A) {
    try {
        return new R::Tensor(R::gcn_norm(*static_cast<const R::Tensor*>(A)));
    } catch (const std::exception& e) {
        g_err = e.what();
        return nullptr;
    }
}

int ref_stack_forward_tensors(void* s, const void* A_norm, const void* A_raw, const void* X,
                              int log_softmax, float* out) {
    return guarded([&] {
        auto* st = static_cast<RefStack*>(s);
        const R::Tensor* H = static_cast<const R::Tensor*>(X);
        R::Tensor cur;
        std::size_t ig = 0, is = 0;
        for (std::size_t l = 0; l < st->kind.size(); ++l) {
            cur = st->kind[l] == 0 ? st->gcn[ig++].forward(*static_cast<const R::Tensor*>(A_norm), *H)
                                   : st->sage[is++].forward(*static_cast<const R::Tensor*>(A_raw), *H);
            if (st->post[l] == 1) R::relu_inplace(cur);
            if (st->post[l] == 2) R::elu_inplace(cur, 1.0f);
            H = &cur;
        }
        if (log_softmax) R::log_softmax_inplace(cur);
        if (out) out_dense(cur, out);
    });
}

int ref_spmm_tensors(const void* A, const void* B, float* out) {
    return guarded([&] {
        R::Tensor y = R::spmm(*static_cast<const R::Tensor*>(A),
                              *static_cast<const R::Tensor*>(B));
        if (out) out_dense(y, out);
    });
}

}  // extern "C"
