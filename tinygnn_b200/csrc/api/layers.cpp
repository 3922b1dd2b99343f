// ============================================================================
//  api/layers.cpp -- tinygnn:: graph utilities and layers (reference
//  src/layers.cpp:44-1129): the reference's constructor / setter / forward
//  validation and messages, then the fused device kernels through the C ABI.
// ============================================================================
#include "tinygnn/layers.hpp"

#include <algorithm>

#include "internal.hpp"

namespace tinygnn {

using detail::check;
using detail::stream;

namespace {

void require_square_csr(const Tensor& A, const char* fn) {
    if (A.format() != StorageFormat::SparseCSR)
        throw std::invalid_argument(std::string(fn) + ": A must be SparseCSR (got Dense).");
    if (A.rows() != A.cols())
        throw std::invalid_argument(std::string(fn) + ": A must be square \xE2\x80\x94 got " +
                                    detail::shape_str(A.rows(), A.cols()) + ".");
}

template <class T>
T* dalloc(std::size_t n) {
    void* p = nullptr;
    detail::cuda(cudaMallocAsync(&p, (n ? n : 1) * sizeof(T), detail::cstream()), "tinygnn allocation");
    return static_cast<T*>(p);
}

Tensor expand_csr(const Tensor& A, bool norm) {
    const std::size_t N = A.rows(), nnz = A.nnz(), cap = nnz + N;
    int32_t* rp = dalloc<int32_t>(N + 1);
    int32_t* ci = dalloc<int32_t>(cap);
    float* v = dalloc<float>(cap);
    int64_t out_nnz = 0;
    const detail::TrustedCsr trusted_csr;
    const auto fn = norm ? tg_gcn_norm_f32 : tg_add_self_loops_f32;
    const tg_status st = fn(static_cast<int64_t>(N), static_cast<int64_t>(nnz), A.device_row_ptr(),
                            A.device_col_ind(), A.device_data(), rp, ci, v, &out_nnz, stream());
    Tensor t = TensorAccess::csr_from_device(N, N, rp, ci, v, static_cast<std::size_t>(out_nnz));
    check(st);
    return t;
}

// A contiguous (ld == cols) device copy of a small dense tensor when its
// device rows are padded; returns the pointer to use.
struct Contig {
    float* owned = nullptr;
    const float* ptr = nullptr;
    Contig(const Tensor& t) {
        if (t.device_ld() == t.cols() || t.rows() * t.cols() == 0) {
            ptr = t.device_data();
            return;
        }
        owned = dalloc<float>(t.rows() * t.cols());
        detail::cuda(cudaMemcpy2DAsync(owned, t.cols() * sizeof(float), t.device_data(), t.device_ld() * sizeof(float),
                                       t.cols() * sizeof(float), t.rows(), cudaMemcpyDeviceToDevice,
                                       detail::cstream()),
                     "tinygnn copy");
        ptr = owned;
    }
    ~Contig() {
        if (owned && cudaFreeAsync(owned, detail::cstream()) != cudaSuccess) cudaGetLastError();
    }
};

int act_code(Activation a) { return a == Activation::ReLU ? TG_ACT_RELU : TG_ACT_NONE; }

void check_weight(const Tensor& w, std::size_t in, std::size_t out, const std::string& who) {
    if (w.format() != StorageFormat::Dense) throw std::invalid_argument(who + ": weight must be Dense.");
    if (w.rows() != in || w.cols() != out)
        throw std::invalid_argument(who + ": expected shape " + detail::shape_str(in, out) + ", got " +
                                    detail::shape_str(w.rows(), w.cols()) + ".");
}

void check_row(const Tensor& b, std::size_t out, const std::string& who, const char* what) {
    if (b.format() != StorageFormat::Dense) throw std::invalid_argument(who + ": " + what + " must be Dense.");
    if (b.rows() != 1 || b.cols() != out)
        throw std::invalid_argument(who + ": expected shape (1\xC3\x97" + std::to_string(out) + "), got " +
                                    detail::shape_str(b.rows(), b.cols()) + ".");
}

}  // namespace

Tensor add_self_loops(const Tensor& A) {
    require_square_csr(A, "add_self_loops");
    return expand_csr(A, false);
}

Tensor gcn_norm(const Tensor& A) {
    require_square_csr(A, "gcn_norm");
    return expand_csr(A, true);
}

Tensor sage_max_aggregate(const Tensor& A, const Tensor& H) {
    if (A.format() != StorageFormat::SparseCSR)
        throw std::invalid_argument("sage_max_aggregate: A must be SparseCSR (got Dense).");
    if (H.format() != StorageFormat::Dense)
        throw std::invalid_argument("sage_max_aggregate: H must be Dense (got SparseCSR).");
    if (A.cols() != H.rows())
        throw std::invalid_argument("sage_max_aggregate: A.cols() (" + std::to_string(A.cols()) + ") != H.rows() (" +
                                    std::to_string(H.rows()) + ").");
    Tensor out = Tensor::dense_device(A.rows(), H.cols());
    if (A.rows() == 0 || H.cols() == 0) return out;
    const detail::TrustedCsr trusted_csr;
    check(tg_sage_max_aggregate_f32(static_cast<int64_t>(A.rows()), static_cast<int64_t>(A.cols()),
                                    static_cast<int64_t>(A.nnz()), A.device_row_ptr(), A.device_col_ind(),
                                    H.device_data(), static_cast<int64_t>(H.cols()),
                                    static_cast<int64_t>(H.device_ld()), out.mutable_device_data(),
                                    static_cast<int64_t>(out.device_ld()), stream()));
    return out;
}

Tensor edge_softmax(const Tensor& A) {
    if (A.format() != StorageFormat::SparseCSR)
        throw std::invalid_argument("edge_softmax: input must be SparseCSR (got Dense).");
    const std::size_t N = A.rows(), nnz = A.nnz();
    int32_t* rp = dalloc<int32_t>(N + 1);
    int32_t* ci = dalloc<int32_t>(nnz);
    float* v = dalloc<float>(nnz);
    detail::cuda(cudaMemcpyAsync(rp, A.device_row_ptr(), (N + 1) * sizeof(int32_t), cudaMemcpyDeviceToDevice,
                                 detail::cstream()),
                 "edge_softmax");
    if (nnz) {
        detail::cuda(cudaMemcpyAsync(ci, A.device_col_ind(), nnz * sizeof(int32_t), cudaMemcpyDeviceToDevice,
                                     detail::cstream()),
                     "edge_softmax");
        detail::cuda(cudaMemsetAsync(v, 0, nnz * sizeof(float), detail::cstream()), "edge_softmax");
    }
    Tensor t = TensorAccess::csr_from_device(N, A.cols(), rp, ci, v, nnz);
    const detail::TrustedCsr trusted_csr;
    if (N) check(tg_edge_softmax_f32(static_cast<int64_t>(N), static_cast<int64_t>(nnz), t.device_row_ptr(),
                                     A.device_data(), t.mutable_device_data(), stream()));
    return t;
}

// ── GCNLayer (layers.cpp:213-339) ──────────────────────────────────────────
GCNLayer::GCNLayer(std::size_t in_features, std::size_t out_features, bool use_bias, Activation act)
    : in_features_(in_features), out_features_(out_features), use_bias_(use_bias), activation_(act),
      weight_(Tensor::dense(in_features, out_features)), bias_(Tensor::dense(1, out_features)) {
    if (in_features == 0) throw std::invalid_argument("GCNLayer: in_features must be > 0.");
    if (out_features == 0) throw std::invalid_argument("GCNLayer: out_features must be > 0.");
}

void GCNLayer::set_weight(Tensor w) {
    check_weight(w, in_features_, out_features_, "GCNLayer::set_weight");
    weight_ = std::move(w);
}

void GCNLayer::set_bias(Tensor b) {
    if (!use_bias_) throw std::invalid_argument("GCNLayer::set_bias: layer was constructed with use_bias=false.");
    check_row(b, out_features_, "GCNLayer::set_bias", "bias");
    bias_ = std::move(b);
}

Tensor GCNLayer::forward(const Tensor& A_norm, const Tensor& H) const {
    if (A_norm.format() != StorageFormat::SparseCSR)
        throw std::invalid_argument(
            "GCNLayer::forward: A_norm must be SparseCSR (got Dense). Use gcn_norm() to precompute the normalized "
            "adjacency.");
    if (A_norm.rows() != A_norm.cols())
        throw std::invalid_argument("GCNLayer::forward: A_norm must be square \xE2\x80\x94 got " +
                                    detail::shape_str(A_norm.rows(), A_norm.cols()) + ".");
    if (H.format() != StorageFormat::Dense)
        throw std::invalid_argument("GCNLayer::forward: H must be Dense (got SparseCSR).");
    if (H.cols() != in_features_)
        throw std::invalid_argument("GCNLayer::forward: H has " + std::to_string(H.cols()) +
                                    " columns but layer expects in_features=" + std::to_string(in_features_) + ".");
    if (A_norm.rows() != H.rows())
        throw std::invalid_argument("GCNLayer::forward: A_norm has " + std::to_string(A_norm.rows()) +
                                    " rows but H has " + std::to_string(H.rows()) +
                                    " rows. They must match (N nodes).");
    const std::size_t N = H.rows();
    Tensor out = Tensor::dense_device(N, out_features_);
    if (N == 0) return out;
    // HW = H . W into a row-padded intermediate, then the fused gather.
    Tensor HW = Tensor::dense_device(N, out_features_);
    check(tg_gemm_f32(static_cast<int64_t>(N), static_cast<int64_t>(out_features_), static_cast<int64_t>(in_features_),
                      H.device_data(), static_cast<int64_t>(H.device_ld()), weight_.device_data(),
                      static_cast<int64_t>(weight_.device_ld()), HW.mutable_device_data(),
                      static_cast<int64_t>(HW.device_ld()), nullptr, TG_ACT_NONE, 0.0f,
                      detail::mode() | TG_FLAG_C_COLS_PADDED, stream()));
    const detail::TrustedCsr trusted_csr;
    check(tg_spmm_f32(static_cast<int64_t>(N), static_cast<int64_t>(N), static_cast<int64_t>(A_norm.nnz()),
                      A_norm.device_row_ptr(), A_norm.device_col_ind(), A_norm.device_data(), HW.device_data(),
                      static_cast<int64_t>(out_features_), static_cast<int64_t>(HW.device_ld()),
                      out.mutable_device_data(), static_cast<int64_t>(out.device_ld()),
                      use_bias_ ? bias_.device_data() : nullptr, act_code(activation_), 0.0f, nullptr,
                      detail::mode() | TG_FLAG_B_ROWS_PADDED, stream()));
    return out;
}

// ── SAGELayer (layers.cpp:440-752) ─────────────────────────────────────────
SAGELayer::SAGELayer(std::size_t in_features, std::size_t out_features, Aggregator agg, bool use_bias,
                     Activation act)
    : in_features_(in_features), out_features_(out_features), aggregator_(agg), use_bias_(use_bias),
      activation_(act), weight_neigh_(Tensor::dense(in_features, out_features)),
      weight_self_(Tensor::dense(in_features, out_features)), bias_(Tensor::dense(1, out_features)) {
    if (in_features == 0) throw std::invalid_argument("SAGELayer: in_features must be > 0.");
    if (out_features == 0) throw std::invalid_argument("SAGELayer: out_features must be > 0.");
}

void SAGELayer::set_weight_neigh(Tensor w) {
    check_weight(w, in_features_, out_features_, "SAGELayer::set_weight_neigh");
    weight_neigh_ = std::move(w);
}

void SAGELayer::set_weight_self(Tensor w) {
    check_weight(w, in_features_, out_features_, "SAGELayer::set_weight_self");
    weight_self_ = std::move(w);
}

void SAGELayer::set_bias(Tensor b) {
    if (!use_bias_) throw std::invalid_argument("SAGELayer::set_bias: layer was constructed with use_bias=false.");
    check_row(b, out_features_, "SAGELayer::set_bias", "bias");
    bias_ = std::move(b);
}

Tensor SAGELayer::forward(const Tensor& A, const Tensor& H) const {
    if (A.format() != StorageFormat::SparseCSR)
        throw std::invalid_argument("SAGELayer::forward: A must be SparseCSR (got Dense).");
    if (H.format() != StorageFormat::Dense)
        throw std::invalid_argument("SAGELayer::forward: H must be Dense (got SparseCSR).");
    if (H.cols() != in_features_)
        throw std::invalid_argument("SAGELayer::forward: H has " + std::to_string(H.cols()) +
                                    " columns but layer expects in_features=" + std::to_string(in_features_) + ".");
    if (A.cols() != H.rows())
        throw std::invalid_argument("SAGELayer::forward: A.cols() (" + std::to_string(A.cols()) + ") != H.rows() (" +
                                    std::to_string(H.rows()) + ").");
    const std::size_t N = H.rows(), Fi = in_features_, Fo = out_features_;
    Tensor out = Tensor::dense_device(N, Fo);
    if (N == 0) return out;
    const bool max = aggregator_ == Aggregator::Max;
    const float* bias = use_bias_ ? bias_.device_data() : nullptr;
    if (fast_math() && !max && Fi > Fo) {  // transform first: gather F_out instead of F_in floats per edge
        // W_neigh and W_self in one tensor-core pass over H (weights are dense with ld == cols)
        Tensor Tn = Tensor::dense_device(N, Fo), Ts = Tensor::dense_device(N, Fo);
        detail::DevWeights w(weight_neigh_, weight_self_);
        check(tg_gemm_pair_f32(static_cast<int64_t>(N), static_cast<int64_t>(Fo), static_cast<int64_t>(Fi),
                               H.device_data(), static_cast<int64_t>(H.device_ld()), w.wn, w.ws,
                               static_cast<int64_t>(Fo), Tn.mutable_device_data(), static_cast<int64_t>(Tn.device_ld()),
                               Ts.mutable_device_data(), static_cast<int64_t>(Ts.device_ld()),
                               TG_MODE_FAST | TG_FLAG_C_COLS_PADDED, stream()));
        // The combine gathers Tn rows in a longest-first schedule, in column
        // passes when Tn is larger than kPassBytes (each pass's slice stays
        // in L2; the passes carry each output element's chain through out).
        const detail::TrustedCsr trusted_csr;
        const std::size_t K = A.cols();
        const int64_t M = static_cast<int64_t>(N);
        detail::DevArray<int32_t> order(N);
        check(tg_csr_degree_order(M, A.device_row_ptr(), order.p, stream()));
        const int passes = static_cast<int>(std::max<std::size_t>(
            1, (K * Tn.device_ld() * sizeof(float) + detail::kPassBytes - 1) / detail::kPassBytes));
        if (passes == 1) {
            check(tg_sage_mean_combine_f32(M, static_cast<int64_t>(K), static_cast<int64_t>(A.nnz()),
                                           A.device_row_ptr(), A.device_col_ind(), Tn.device_data(),
                                           static_cast<int64_t>(Fo), static_cast<int64_t>(Tn.device_ld()),
                                           Ts.device_data(), static_cast<int64_t>(Ts.device_ld()), bias,
                                           act_code(activation_), out.mutable_device_data(),
                                           static_cast<int64_t>(out.device_ld()), order.p, TG_FLAG_B_ROWS_PADDED,
                                           stream()));
            return out;
        }
        detail::DevArray<int32_t> sp(N * static_cast<std::size_t>(passes + 1));
        check(tg_csr_column_splits(M, A.device_row_ptr(), A.device_col_ind(), passes,
                                   static_cast<int64_t>((K + passes - 1) / passes), sp.p, stream()));
        for (int q = 0; q < passes; ++q)
            check(tg_sage_mean_combine_segment_f32(
                M, static_cast<int64_t>(K), A.device_row_ptr(), A.device_col_ind(), sp.p + static_cast<std::size_t>(q) * N,
                sp.p + static_cast<std::size_t>(q + 1) * N, Tn.device_data(), static_cast<int64_t>(Fo),
                static_cast<int64_t>(Tn.device_ld()), Ts.device_data(), static_cast<int64_t>(Ts.device_ld()), bias,
                act_code(activation_), out.mutable_device_data(), static_cast<int64_t>(out.device_ld()), order.p,
                q > 0, q == passes - 1, TG_FLAG_B_ROWS_PADDED, stream()));
        return out;
    }
    // Aggregate first, then the interleaved dual product (bit-identical), or
    // in FAST mode one tensor-core GEMM [agg | H] . [Wn; Ws].
    Tensor agg = Tensor::dense_device(N, Fi);
    const detail::TrustedCsr trusted_csr;
    check(tg_sage_aggregate_f32(static_cast<int64_t>(N), static_cast<int64_t>(A.cols()), static_cast<int64_t>(A.nnz()),
                                A.device_row_ptr(), A.device_col_ind(), H.device_data(), static_cast<int64_t>(Fi),
                                static_cast<int64_t>(H.device_ld()), agg.mutable_device_data(),
                                static_cast<int64_t>(agg.device_ld()), max ? TG_AGG_MAX : TG_AGG_MEAN, stream()));
    if (fast_math()) {
        check(tg_gemm_cat_f32(static_cast<int64_t>(N), static_cast<int64_t>(Fo), static_cast<int64_t>(Fi),
                              agg.device_data(), static_cast<int64_t>(agg.device_ld()), static_cast<int64_t>(Fi),
                              H.device_data(), static_cast<int64_t>(H.device_ld()), weight_neigh_.device_data(),
                              static_cast<int64_t>(weight_neigh_.device_ld()), weight_self_.device_data(),
                              static_cast<int64_t>(weight_self_.device_ld()), out.mutable_device_data(),
                              static_cast<int64_t>(out.device_ld()), bias, act_code(activation_), 0.0f, TG_MODE_FAST,
                              stream()));
        return out;
    }
    check(tg_gemm_dual_f32(static_cast<int64_t>(N), static_cast<int64_t>(Fo), static_cast<int64_t>(Fi),
                           agg.device_data(), static_cast<int64_t>(agg.device_ld()), H.device_data(),
                           static_cast<int64_t>(H.device_ld()), weight_neigh_.device_data(),
                           weight_self_.device_data(), static_cast<int64_t>(weight_neigh_.device_ld()),
                           out.mutable_device_data(), static_cast<int64_t>(out.device_ld()), bias,
                           act_code(activation_), 0.0f, stream()));
    return out;
}

// ── GATLayer (layers.cpp:827-1129) ─────────────────────────────────────────
GATLayer::GATLayer(std::size_t in_features, std::size_t out_features, float negative_slope, bool use_bias,
                   Activation act)
    : in_features_(in_features), out_features_(out_features), negative_slope_(negative_slope),
      use_bias_(use_bias), activation_(act), weight_(Tensor::dense(in_features, out_features)),
      attn_left_(Tensor::dense(1, out_features)), attn_right_(Tensor::dense(1, out_features)),
      bias_(Tensor::dense(1, out_features)) {
    if (in_features == 0) throw std::invalid_argument("GATLayer: in_features must be > 0.");
    if (out_features == 0) throw std::invalid_argument("GATLayer: out_features must be > 0.");
}

void GATLayer::set_weight(Tensor w) {
    check_weight(w, in_features_, out_features_, "GATLayer::set_weight");
    weight_ = std::move(w);
}

void GATLayer::set_attn_left(Tensor a) {
    check_row(a, out_features_, "GATLayer::set_attn_left", "attention vector");
    attn_left_ = std::move(a);
}

void GATLayer::set_attn_right(Tensor a) {
    check_row(a, out_features_, "GATLayer::set_attn_right", "attention vector");
    attn_right_ = std::move(a);
}

void GATLayer::set_bias(Tensor b) {
    if (!use_bias_) throw std::invalid_argument("GATLayer::set_bias: layer was constructed with use_bias=false.");
    check_row(b, out_features_, "GATLayer::set_bias", "bias");
    bias_ = std::move(b);
}

Tensor GATLayer::forward(const Tensor& A, const Tensor& H) const {
    if (A.format() != StorageFormat::SparseCSR)
        throw std::invalid_argument(
            "GATLayer::forward: A must be SparseCSR (got Dense). Use add_self_loops() to prepare the adjacency.");
    if (A.rows() != A.cols())
        throw std::invalid_argument("GATLayer::forward: A must be square \xE2\x80\x94 got " +
                                    detail::shape_str(A.rows(), A.cols()) + ".");
    if (H.format() != StorageFormat::Dense)
        throw std::invalid_argument("GATLayer::forward: H must be Dense (got SparseCSR).");
    if (H.cols() != in_features_)
        throw std::invalid_argument("GATLayer::forward: H has " + std::to_string(H.cols()) +
                                    " columns but layer expects in_features=" + std::to_string(in_features_) + ".");
    if (A.rows() != H.rows())
        throw std::invalid_argument("GATLayer::forward: A has " + std::to_string(A.rows()) + " rows but H has " +
                                    std::to_string(H.rows()) + " rows. They must match (N nodes).");
    const std::size_t N = H.rows();
    Tensor out = Tensor::dense_device(N, out_features_);
    if (N == 0) return out;
    const Contig W(weight_);
    const detail::TrustedCsr trusted_csr;
    check(tg_gat_layer_f32(static_cast<int64_t>(N), static_cast<int64_t>(A.nnz()), A.device_row_ptr(),
                           A.device_col_ind(), H.device_data(), static_cast<int64_t>(H.device_ld()),
                           static_cast<int64_t>(in_features_), 1, static_cast<int64_t>(out_features_), W.ptr,
                           attn_left_.device_data(), attn_right_.device_data(),
                           use_bias_ ? bias_.device_data() : nullptr, negative_slope_, 1, act_code(activation_),
                           out.mutable_device_data(), static_cast<int64_t>(out.device_ld()), nullptr, detail::mode(),
                           stream()));
    return out;
}

}  // namespace tinygnn
