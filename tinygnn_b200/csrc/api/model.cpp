// ============================================================================
//  api/model.cpp -- Model (execution graph) and the binary loaders (reference
//  src/model.cpp:30-439).
//
//  The file formats are TinyGNN's (cora_graph.bin: N, F, C, E as uint32
//  LE, features, labels, three masks, src[E], dst[E]; TGNN weight files:
//  magic, version 1, accuracy, named tensors), read on the host; the
//  adjacency CSR is built on the device (edge_list_to_csr, bit-identical).
//  Model::forward normalises on the device once per call, like the
//  reference, runs every layer's fused kernels, and runs a multi-head GAT
//  layer as one pass over the graph for all heads.
// ============================================================================
#include "tinygnn/model.hpp"

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <utility>
#include <fstream>

#include "internal.hpp"
#include "tinygnn/graph_loader.hpp"
#include "tinygnn/ops.hpp"

namespace tg {
void fill_f32(float* p, int64_t n, float v, cudaStream_t s);
}  // namespace tg

namespace tinygnn {

using detail::check;
using detail::stream;

namespace {

void read_exact(std::ifstream& f, void* buf, std::size_t n, const char* ctx) {
    f.read(reinterpret_cast<char*>(buf), static_cast<std::streamsize>(n));
    if (!f) throw std::runtime_error(std::string(ctx) + ": unexpected end of file or read error.");
}

template <class T>
T read_le(std::ifstream& f, const char* ctx) {
    T v{};
    read_exact(f, &v, sizeof(T), ctx);  // little-endian host
    return v;
}

using DevBuf = detail::DevArray<float>;

// Packs rows x cols of `src` (device, row stride ld) into dst at column offset.
void pack(float* dst, std::size_t dst_ld, std::size_t col0, const Tensor& src) {
    if (src.rows() * src.cols() == 0) return;
    detail::cuda(cudaMemcpy2DAsync(dst + col0, dst_ld * sizeof(float), src.device_data(),
                                   src.device_ld() * sizeof(float), src.cols() * sizeof(float), src.rows(),
                                   cudaMemcpyDeviceToDevice, detail::cstream()),
                 "Model::forward");
}

}  // namespace

CoraData load_cora_binary(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f.is_open()) throw std::runtime_error("load_cora_binary: cannot open " + path);
    const char* ctx = "load_cora_binary";
    CoraData cd;
    cd.num_nodes = read_le<uint32_t>(f, ctx);
    cd.num_features = read_le<uint32_t>(f, ctx);
    cd.num_classes = read_le<uint32_t>(f, ctx);
    cd.num_edges = read_le<uint32_t>(f, ctx);
    const std::size_t N = cd.num_nodes, F = cd.num_features, E = cd.num_edges;
    std::vector<float> feat(N * F);
    read_exact(f, feat.data(), N * F * sizeof(float), ctx);
    cd.features = Tensor::dense(N, F, std::move(feat));
    cd.labels.resize(N);
    read_exact(f, cd.labels.data(), N * sizeof(int32_t), ctx);
    cd.train_mask.resize(N);
    cd.val_mask.resize(N);
    cd.test_mask.resize(N);
    read_exact(f, cd.train_mask.data(), N, ctx);
    read_exact(f, cd.val_mask.data(), N, ctx);
    read_exact(f, cd.test_mask.data(), N, ctx);
    std::vector<int32_t> src(E), dst(E);
    read_exact(f, src.data(), E * sizeof(int32_t), ctx);
    read_exact(f, dst.data(), E * sizeof(int32_t), ctx);
    std::vector<std::pair<int32_t, int32_t>> edges(E);
    for (std::size_t e = 0; e < E; ++e) edges[e] = {src[e], dst[e]};
    cd.adjacency = GraphLoader::edge_list_to_csr(edges, N);  // same CSR algorithm (model.cpp:89-122)
    return cd;
}

WeightFile load_weight_file(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f.is_open()) throw std::runtime_error("load_weight_file: cannot open " + path);
    const char* ctx = "load_weight_file";
    char magic[4]{};
    read_exact(f, magic, 4, ctx);
    if (std::memcmp(magic, "TGNN", 4) != 0) throw std::runtime_error("load_weight_file: invalid magic in " + path);
    const uint32_t version = read_le<uint32_t>(f, ctx);
    if (version != 1)
        throw std::runtime_error("load_weight_file: unsupported version " + std::to_string(version) + " in " + path);
    WeightFile wf;
    wf.test_accuracy = read_le<float>(f, ctx);
    const uint32_t count = read_le<uint32_t>(f, ctx);
    for (uint32_t t = 0; t < count; ++t) {
        const uint32_t len = read_le<uint32_t>(f, ctx);
        std::string name(len, '\0');
        read_exact(f, name.data(), len, ctx);
        const uint32_t rows = read_le<uint32_t>(f, ctx), cols = read_le<uint32_t>(f, ctx);
        std::vector<float> data(static_cast<std::size_t>(rows) * cols);
        read_exact(f, data.data(), data.size() * sizeof(float), ctx);
        wf.tensors[name] = Tensor::dense(rows, cols, std::move(data));
    }
    return wf;
}

std::size_t Model::add_gcn_layer(std::size_t in_f, std::size_t out_f, bool bias, Activation act,
                                 InterActivation post) {
    gcn_layers_.emplace_back(in_f, out_f, bias, act);
    layers_.push_back({LayerEntry::Type::GCN, gcn_layers_.size() - 1, 1, false, post});
    return layers_.size() - 1;
}

std::size_t Model::add_sage_layer(std::size_t in_f, std::size_t out_f, SAGELayer::Aggregator agg, bool bias,
                                  Activation act, InterActivation post) {
    sage_layers_.emplace_back(in_f, out_f, agg, bias, act);
    layers_.push_back({LayerEntry::Type::SAGE, sage_layers_.size() - 1, 1, false, post});
    return layers_.size() - 1;
}

std::size_t Model::add_gat_layer(std::size_t in_f, std::size_t out_f, std::size_t num_heads, bool concat,
                                 float neg_slope, bool bias, Activation act, InterActivation post) {
    const std::size_t idx = gat_layers_.size();
    for (std::size_t h = 0; h < num_heads; ++h) gat_layers_.emplace_back(in_f, out_f, neg_slope, bias, act);
    layers_.push_back({LayerEntry::Type::GAT, idx, num_heads, concat, post});
    return layers_.size() - 1;
}

void Model::load_weights(const std::string& path) { load_weights(load_weight_file(path)); }

void Model::load_weights(const WeightFile& wf) {
    auto get = [&](const std::string& name) -> const Tensor& {
        auto it = wf.tensors.find(name);
        if (it == wf.tensors.end()) throw std::runtime_error("Model::load_weights: missing tensor '" + name + "'");
        return it->second;
    };
    for (std::size_t li = 0; li < layers_.size(); ++li) {
        const auto& e = layers_[li];
        const std::string p = "layer" + std::to_string(li);
        switch (e.type) {
            case LayerEntry::Type::GCN: {
                auto& l = gcn_layers_[e.start_idx];
                l.set_weight(get(p + ".weight"));
                if (l.has_bias()) l.set_bias(get(p + ".bias"));
                break;
            }
            case LayerEntry::Type::SAGE: {
                auto& l = sage_layers_[e.start_idx];
                l.set_weight_neigh(get(p + ".weight_neigh"));
                l.set_weight_self(get(p + ".weight_self"));
                if (l.has_bias()) l.set_bias(get(p + ".bias"));
                break;
            }
            case LayerEntry::Type::GAT:
                for (std::size_t h = 0; h < e.count; ++h) {
                    auto& l = gat_layers_[e.start_idx + h];
                    const std::string hp = p + ".head" + std::to_string(h);
                    l.set_weight(get(hp + ".weight"));
                    l.set_attn_left(get(hp + ".attn_left"));
                    l.set_attn_right(get(hp + ".attn_right"));
                    if (l.has_bias()) l.set_bias(get(hp + ".bias"));
                }
                break;
        }
    }
}

namespace {

using DevInts = detail::DevArray<int32_t>;

// The raw adjacency prepared once per forward for FAST GCN layers without a
// normalised copy: dis[i] = 1/sqrt(row sum + 1) (tg_gcn_norm_scale_f32), a
// longest-first row schedule, and column splits per pass count.
struct ScaledGraph {
    const Tensor& A;
    std::size_t n;
    DevBuf dis;
    DevInts order;
    std::vector<std::pair<int, std::unique_ptr<DevInts>>> splits;

    explicit ScaledGraph(const Tensor& adj) : A(adj), n(adj.rows()), dis(adj.rows()), order(adj.rows()) {
        const detail::TrustedCsr trusted_csr;
        check(tg_gcn_norm_scale_f32(static_cast<int64_t>(n), static_cast<int64_t>(A.nnz()), A.device_row_ptr(),
                                    A.device_data(), dis.p, stream()));
        check(tg_csr_degree_order(static_cast<int64_t>(n), A.device_row_ptr(), order.p, stream()));
    }

    const int32_t* split_points(int passes) {
        for (auto& sp : splits)
            if (sp.first == passes) return sp.second->p;
        auto buf = std::make_unique<DevInts>(n * static_cast<std::size_t>(passes + 1));
        const detail::TrustedCsr trusted_csr;
        check(tg_csr_column_splits(static_cast<int64_t>(n), A.device_row_ptr(), A.device_col_ind(), passes,
                                   static_cast<int64_t>((n + passes - 1) / passes), buf->p, stream()));
        splits.emplace_back(passes, std::move(buf));
        return splits.back().second->p;
    }
};

using detail::kPassBytes;

// GCNLayer::forward on the raw adjacency in FAST mode: Hs = diag(dis) . (H . W)
// on the tensor cores, then out = act(dis * (A . Hs + Hs_self) + b) in
// stored order -- D^-1/2 (A + I) D^-1/2 . HW without the normalised copy.
Tensor gcn_forward_scaled(const GCNLayer& L, ScaledGraph& g, const Tensor& H) {
    if (H.format() != StorageFormat::Dense)
        throw std::invalid_argument("GCNLayer::forward: H must be Dense (got SparseCSR).");
    if (H.cols() != L.in_features())
        throw std::invalid_argument("GCNLayer::forward: H has " + std::to_string(H.cols()) +
                                    " columns but layer expects in_features=" + std::to_string(L.in_features()) +
                                    ".");
    if (g.n != H.rows())
        throw std::invalid_argument("GCNLayer::forward: A_norm has " + std::to_string(g.n) + " rows but H has " +
                                    std::to_string(H.rows()) + " rows. They must match (N nodes).");
    const std::size_t N = g.n, Fo = L.out_features();
    Tensor out = Tensor::dense_device(N, Fo);
    if (N == 0) return out;
    Tensor Hs = Tensor::dense_device(N, Fo);  // rows padded to 16 bytes; the padding stays 0
    check(tg_gemm_rowscale_f32(static_cast<int64_t>(N), static_cast<int64_t>(Fo),
                               static_cast<int64_t>(L.in_features()), H.device_data(),
                               static_cast<int64_t>(H.device_ld()), L.weight().device_data(),
                               static_cast<int64_t>(L.weight().device_ld()), Hs.mutable_device_data(),
                               static_cast<int64_t>(Hs.device_ld()), g.dis.p, nullptr, TG_ACT_NONE, 0.0f,
                               TG_MODE_FAST | TG_FLAG_C_COLS_PADDED, stream()));
    const int passes = static_cast<int>(
        std::max<std::size_t>(1, (N * Hs.device_ld() * sizeof(float) + kPassBytes - 1) / kPassBytes));
    const int32_t* sp = passes > 1 ? g.split_points(passes) : nullptr;
    const detail::TrustedCsr trusted_csr;
    for (int q = 0; q < passes; ++q)
        check(tg_gcn_aggregate_f32(
            static_cast<int64_t>(N), static_cast<int64_t>(N), static_cast<int64_t>(g.A.nnz()), g.A.device_row_ptr(),
            g.A.device_col_ind(), g.A.device_data(), Hs.device_data(), static_cast<int64_t>(Fo),
            static_cast<int64_t>(Hs.device_ld()), Hs.device_data(), static_cast<int64_t>(Hs.device_ld()), g.dis.p,
            L.has_bias() ? L.bias().device_data() : nullptr,
            L.activation() == Activation::ReLU ? TG_ACT_RELU : TG_ACT_NONE, out.mutable_device_data(),
            static_cast<int64_t>(out.device_ld()), g.order.p, sp ? sp + static_cast<std::size_t>(q) * N : nullptr,
            sp ? sp + static_cast<std::size_t>(q + 1) * N : nullptr, q > 0, q == passes - 1, TG_FLAG_B_ROWS_PADDED,
            stream()));
    return out;
}

}  // namespace

namespace detail {

// The adjacency variants one forward call uses (src/model.cpp:363-381): the
// raw adjacency for SAGE; for GCN layers gcn_norm(A) (EXACT) or the raw
// adjacency with its per-row scale (FAST, ScaledGraph); add_self_loops(A)
// for GAT.
struct ForwardGraphs {
    const Tensor& adjacency;
    std::unique_ptr<ScaledGraph> sg;
    Tensor A_gcn, A_sl;

    ForwardGraphs(const Tensor& adj, bool need_norm, bool need_sl) : adjacency(adj) {
        // EXACT (the default): gcn_norm once per call, bit for bit, like the
        // reference (src/model.cpp:365-381).  FAST: the GCN layers run on the
        // raw adjacency with gcn_norm as per-row scale factors (within the
        // fp32 tolerance); the same validation as gcn_norm's.
        if (need_norm && fast_math()) {
            if (adj.format() != StorageFormat::SparseCSR)
                throw std::invalid_argument("gcn_norm: A must be SparseCSR (got Dense).");
            if (adj.rows() != adj.cols())
                throw std::invalid_argument("gcn_norm: A must be square \xE2\x80\x94 got " +
                                            detail::shape_str(adj.rows(), adj.cols()) + ".");
            sg = std::make_unique<ScaledGraph>(adj);
        } else if (need_norm) {
            A_gcn = gcn_norm(adj);
        }
        if (need_sl) A_sl = add_self_loops(adj);
    }
};

}  // namespace detail

Tensor Model::run_layer(std::size_t li, detail::ForwardGraphs& g, const Tensor& in_t) const {
    const LayerEntry& e = layers_[li];
    const Tensor* in = &in_t;
    Tensor out;
    switch (e.type) {
        case LayerEntry::Type::GCN:
            out = g.sg ? gcn_forward_scaled(gcn_layers_[e.start_idx], *g.sg, *in)
                       : gcn_layers_[e.start_idx].forward(g.A_gcn, *in);
            break;
        case LayerEntry::Type::SAGE: out = sage_layers_[e.start_idx].forward(g.adjacency, *in); break;
        case LayerEntry::Type::GAT: {
            const Tensor& A_sl = g.A_sl;
            if (e.count == 1) {
                out = gat_layers_[e.start_idx].forward(A_sl, *in);
                break;
            }
            // All heads in one pass: W = [W_0 | W_1 | ...], a_l / a_r / b stacked.
            const GATLayer& h0 = gat_layers_[e.start_idx];
            const std::size_t heads = e.count, d = h0.out_features(), fi = h0.in_features();
            if (in->format() != StorageFormat::Dense || in->cols() != fi || in->rows() != A_sl.rows())
                h0.forward(A_sl, *in);  // raises the reference's validation error
            DevBuf W(fi * heads * d), al(heads * d), ar(heads * d), b(heads * d);
            for (std::size_t h = 0; h < heads; ++h) {
                const GATLayer& L = gat_layers_[e.start_idx + h];
                pack(W.p, heads * d, h * d, L.weight());
                pack(al.p, heads * d, h * d, L.attn_left());
                pack(ar.p, heads * d, h * d, L.attn_right());
                pack(b.p, heads * d, h * d, L.bias());
            }
            const std::size_t ocols = e.gat_concat ? heads * d : d;
            out = Tensor::dense_device(in->rows(), ocols);
            const detail::TrustedCsr trusted_csr;
            check(tg_gat_layer_f32(static_cast<int64_t>(in->rows()), static_cast<int64_t>(A_sl.nnz()),
                                   A_sl.device_row_ptr(), A_sl.device_col_ind(), in->device_data(),
                                   static_cast<int64_t>(in->device_ld()), static_cast<int64_t>(fi),
                                   static_cast<int64_t>(heads), static_cast<int64_t>(d), W.p, al.p, ar.p,
                                   h0.has_bias() ? b.p : nullptr, h0.negative_slope(), e.gat_concat ? 1 : 0,
                                   h0.activation() == Activation::ReLU ? TG_ACT_RELU : TG_ACT_NONE,
                                   out.mutable_device_data(), static_cast<int64_t>(out.device_ld()), nullptr,
                                   detail::mode(), stream()));
            break;
        }
    }
    if (e.post_act == InterActivation::ReLU) relu_inplace(out);
    else if (e.post_act == InterActivation::ELU) elu_inplace(out);
    return out;
}

Tensor Model::forward(const Tensor& adjacency, const Tensor& features) const {
    if (layers_.empty()) throw std::runtime_error("Model::forward: no layers configured.");
    bool need_norm = false, need_sl = false;
    for (const auto& e : layers_) {
        need_norm |= e.type == LayerEntry::Type::GCN;
        need_sl |= e.type == LayerEntry::Type::GAT;
    }
    detail::ForwardGraphs g(adjacency, need_norm, need_sl);
    Tensor H;
    const Tensor* in = &features;
    for (std::size_t li = 0; li < layers_.size(); ++li) {
        H = run_layer(li, g, *in);
        in = &H;
    }
    return H;
}


// ── Captured forward (CUDA graph) ───────────────────────────────────────────
struct ForwardGraph::Impl {
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    Tensor out;
    ~Impl() {
        if (exec) cudaGraphExecDestroy(exec);
        if (graph) cudaGraphDestroy(graph);
    }
};

ForwardGraph::ForwardGraph() = default;
ForwardGraph::ForwardGraph(ForwardGraph&&) noexcept = default;
ForwardGraph& ForwardGraph::operator=(ForwardGraph&&) noexcept = default;
ForwardGraph::~ForwardGraph() = default;

const Tensor& ForwardGraph::output() const {
    if (!impl_) throw std::runtime_error("ForwardGraph: empty (not captured)");
    return impl_->out;
}

const Tensor& ForwardGraph::replay() {
    if (!impl_) throw std::runtime_error("ForwardGraph: empty (not captured)");
    detail::cuda(cudaGraphLaunch(impl_->exec, detail::cstream()), "ForwardGraph::replay");
    return impl_->out;
}

ForwardGraph Model::capture(const Tensor& adjacency, const Tensor& features) const {
    // One eager run first: it uploads host-newer inputs and weights, and sets
    // up what the kernels create on first use (attributes, the side stream).
    const Tensor first = forward(adjacency, features);
    auto impl = std::make_unique<ForwardGraph::Impl>();
    impl->out = Tensor::dense_device(first.rows(), first.cols());
    const cudaStream_t s = detail::cstream();
    detail::cuda(cudaStreamSynchronize(s), "Model::capture");
    detail::cuda(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "Model::capture");
    cudaGraph_t g = nullptr;
    try {
        // the forward's temporaries (its output included) are allocated and
        // freed inside the graph; the result is copied into impl->out
        const Tensor y = forward(adjacency, features);
        if (y.rows() > 0 && y.cols() > 0)
            detail::cuda(cudaMemcpy2DAsync(impl->out.mutable_device_data(), impl->out.device_ld() * sizeof(float),
                                           y.device_data(), y.device_ld() * sizeof(float), y.cols() * sizeof(float),
                                           y.rows(), cudaMemcpyDeviceToDevice, s),
                         "Model::capture");
    } catch (...) {
        cudaStreamEndCapture(s, &g);
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        throw std::runtime_error(
            "Model::capture: this forward cannot be recorded as a CUDA graph (a step reads a size back to the "
            "host: EXACT gcn_norm, GAT self-loops); use FAST mode GCN / SAGE layers, or forward()");
    }
    const cudaError_t e = cudaStreamEndCapture(s, &g);
    if (e != cudaSuccess || !g) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        throw std::runtime_error(std::string("Model::capture: recording failed: ") + cudaGetErrorString(e));
    }
    impl->graph = g;
    detail::cuda(cudaGraphInstantiate(&impl->exec, g, 0), "Model::capture");
    ForwardGraph fg;
    fg.impl_ = std::move(impl);
    return fg;
}


// ── Forward from host buffers ──────────────────────────────────────────────
namespace {

// Feature row blocks (and layer-1 column passes) of the host-input forward
// when its first layer is a FAST GCN layer: the GEMM and gather pass of
// block q overlap the upload of block q + 1, and the gather work left after
// the last block has landed is one block's pass.  Row chunks of the last
// layer's gather (one-pass FAST GCN layers): chunk c's output crosses PCIe
// while chunk c + 1 gathers.  TINYGNN_B200_HOST_BLOCKS /
// TINYGNN_B200_HOST_OUT_CHUNKS override the counts.
int env_count(const char* name, int dflt) {
    const char* e = std::getenv(name);
    const int v = e ? std::atoi(e) : 0;
    return v > 0 && v <= 64 ? v : dflt;
}
int host_blocks() {
    static const int v = env_count("TINYGNN_B200_HOST_BLOCKS", 16);
    return v;
}
int out_chunks() {
    static const int v = env_count("TINYGNN_B200_HOST_OUT_CHUNKS", 3);
    return v;
}

// The calling thread's copy stream on the current device (non-blocking, so
// it runs beside the per-thread default stream the compute uses).
cudaStream_t copy_stream() {
    thread_local std::vector<cudaStream_t> per_device;
    int dev = 0;
    detail::cuda(cudaGetDevice(&dev), "Model::forward_host");
    if (static_cast<int>(per_device.size()) <= dev) per_device.resize(static_cast<std::size_t>(dev) + 1, nullptr);
    cudaStream_t& s = per_device[static_cast<std::size_t>(dev)];
    if (!s) detail::cuda(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "Model::forward_host");
    return s;
}

struct Event {
    cudaEvent_t e = nullptr;
    Event() { detail::cuda(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "Model::forward_host"); }
    ~Event() {
        if (e) cudaEventDestroy(e);
    }
    Event(const Event&) = delete;
    Event& operator=(const Event&) = delete;
    void record(cudaStream_t s) { detail::cuda(cudaEventRecord(e, s), "Model::forward_host"); }
    void wait_in(cudaStream_t s) { detail::cuda(cudaStreamWaitEvent(s, e, 0), "Model::forward_host"); }
};

// On scope exit the compute stream waits for everything queued on the copy
// stream, so buffers freed (stream-ordered) on the compute stream afterwards
// -- on error paths too -- are no longer being copied.
struct JoinCopies {
    cudaStream_t cs;
    Event done;
    explicit JoinCopies(cudaStream_t c) : cs(c) {}
    ~JoinCopies() {
        if (cudaEventRecord(done.e, cs) != cudaSuccess ||
            cudaStreamWaitEvent(detail::cstream(), done.e, 0) != cudaSuccess) {
            cudaGetLastError();
            cudaStreamSynchronize(cs);
        }
    }
};

// rows x cols of a device matrix (row stride dld) into host memory at row
// stride ld, on stream s: one DMA when the strides match, else a device-side
// repack into `pack` (rows x ld floats) first.
void download_rows(float* host, std::size_t ld, const float* dev, std::size_t dld, std::size_t rows,
                   std::size_t cols, float* pack, cudaStream_t s) {
    if (!rows || !cols) return;
    if (ld == dld) {
        detail::cuda(cudaMemcpyAsync(host, dev, rows * ld * sizeof(float), cudaMemcpyDeviceToHost, s),
                     "Model::forward_host");
        return;
    }
    detail::cuda(cudaMemcpy2DAsync(pack, ld * sizeof(float), dev, dld * sizeof(float), cols * sizeof(float), rows,
                                   cudaMemcpyDeviceToDevice, s),
                 "Model::forward_host");
    detail::cuda(cudaMemcpyAsync(host, pack, rows * ld * sizeof(float), cudaMemcpyDeviceToHost, s),
                 "Model::forward_host");
}

}  // namespace

void Model::forward_host(std::size_t n, std::size_t nnz, const int32_t* row_ptr, const int32_t* col_ind,
                         const float* values, const float* features, std::size_t feature_cols,
                         std::size_t ld_features, float* out, std::size_t out_cols, std::size_t ld_out) const {
    if (layers_.empty()) throw std::runtime_error("Model::forward: no layers configured.");
    if (!row_ptr || (nnz && !col_ind)) throw std::invalid_argument("Model::forward_host: null CSR array");
    if (n && (!features || !out)) throw std::invalid_argument("Model::forward_host: null features or out");
    if (ld_features < feature_cols) throw std::invalid_argument("Model::forward_host: ld_features < feature_cols");
    if (ld_out < out_cols) throw std::invalid_argument("Model::forward_host: ld_out < out_cols");
    if (nnz > static_cast<std::size_t>(INT32_MAX))
        throw std::invalid_argument("Model::forward_host: nnz exceeds the int32 CSR limit");
    bool need_norm = false, need_sl = false;
    for (const auto& e : layers_) {
        need_norm |= e.type == LayerEntry::Type::GCN;
        need_sl |= e.type == LayerEntry::Type::GAT;
    }
    const cudaStream_t s = detail::cstream(), cs = copy_stream();
    const bool first_scaled = layers_[0].type == LayerEntry::Type::GCN && fast_math() && n > 0;
    // a FAST transform-first SAGE-mean first layer pipelines the same way
    bool first_sage = false;
    if (layers_[0].type == LayerEntry::Type::SAGE && fast_math() && n > 0) {
        const SAGELayer& L = sage_layers_[layers_[0].start_idx];
        first_sage = L.aggregator() == SAGELayer::Aggregator::Mean && L.in_features() > L.out_features() &&
                     feature_cols == L.in_features();
    }
    const bool pipelined = first_scaled || first_sage;
    const int blocks = pipelined ? static_cast<int>(std::min<std::size_t>(host_blocks(), n)) : 1;
    const std::size_t width = n ? (n + static_cast<std::size_t>(blocks) - 1) / static_cast<std::size_t>(blocks) : 0;

    // device buffers (stream-ordered on the compute stream; the CSR arrays
    // pass to the adjacency tensor once it has been checked)
    DevInts d_rp(n + 1), d_ci(nnz);
    DevBuf d_v(nnz);
    const std::size_t ldx = detail::pad4(feature_cols);
    std::unique_ptr<DevBuf> landing;
    if (ld_features != ldx && n && feature_cols) landing = std::make_unique<DevBuf>(n * ld_features);
    Event allocated, csr_ready;
    std::vector<std::unique_ptr<Event>> x_ready;
    // The copies may start once their destinations exist; the features'
    // device tensor (zero-filled: 0.1 ms for 561 MB) is created after that
    // point when they land in a separate buffer first.
    Tensor X;
    if (landing) allocated.record(s);
    X = Tensor::dense_device(n, feature_cols);
    if (!landing) allocated.record(s);
    float* x_dst = landing ? landing->p : X.mutable_device_data();
    JoinCopies join(cs);  // declared after the buffers: runs before they are freed
    allocated.wait_in(cs);

    // the uploads, all queued before any host wait
    detail::cuda(cudaMemcpyAsync(d_rp.p, row_ptr, (n + 1) * sizeof(int32_t), cudaMemcpyHostToDevice, cs),
                 "Model::forward_host");
    if (nnz) {
        detail::cuda(cudaMemcpyAsync(d_ci.p, col_ind, nnz * sizeof(int32_t), cudaMemcpyHostToDevice, cs),
                     "Model::forward_host");
        if (values)
            detail::cuda(cudaMemcpyAsync(d_v.p, values, nnz * sizeof(float), cudaMemcpyHostToDevice, cs),
                         "Model::forward_host");
    }
    csr_ready.record(cs);
    for (int q = 0; q < blocks; ++q) {
        const std::size_t a = std::min(n, static_cast<std::size_t>(q) * width), b = std::min(n, a + width);
        if (b > a && feature_cols)
            detail::cuda(cudaMemcpyAsync(x_dst + a * (landing ? ld_features : ldx), features + a * ld_features,
                                         (b - a) * ld_features * sizeof(float), cudaMemcpyHostToDevice, cs),
                         "Model::forward_host");
        x_ready.push_back(std::make_unique<Event>());
        x_ready.back()->record(cs);
    }

    // the adjacency: checked on the device as soon as it has landed
    if (nnz && !values) tg::fill_f32(d_v.p, static_cast<int64_t>(nnz), 1.0f, s);
    csr_ready.wait_in(s);
    check(tg_csr_validate(static_cast<int64_t>(n), static_cast<int64_t>(n), static_cast<int64_t>(nnz), d_rp.p, d_ci.p,
                          stream()));
    Tensor A = TensorAccess::csr_from_device(n, n, d_rp.p, d_ci.p, d_v.p, nnz);
    d_rp.p = nullptr;  // owned by A from here
    d_ci.p = nullptr;
    d_v.p = nullptr;
    detail::ForwardGraphs g(A, need_norm, need_sl);

    auto repack = [&](std::size_t a, std::size_t b) {
        if (!landing || b <= a) return;
        detail::cuda(cudaMemcpy2DAsync(X.mutable_device_data() + a * ldx, ldx * sizeof(float),
                                       landing->p + a * ld_features, ld_features * sizeof(float),
                                       feature_cols * sizeof(float), b - a, cudaMemcpyDeviceToDevice, s),
                     "Model::forward_host");
    };

    Tensor H;
    std::size_t first = 0;
    if (first_scaled) {
        // Layer 1 per feature block: Hs rows of block q = diag(dis) . X . W,
        // then the gather pass over the columns of block q (passes in column
        // order: each output element's chain keeps its stored order).
        const GCNLayer& L = gcn_layers_[layers_[0].start_idx];
        if (feature_cols != L.in_features())
            throw std::invalid_argument("GCNLayer::forward: H has " + std::to_string(feature_cols) +
                                        " columns but layer expects in_features=" + std::to_string(L.in_features()) +
                                        ".");
        const std::size_t Fo = L.out_features();
        Tensor Hs = Tensor::dense_device(n, Fo);
        Tensor o = Tensor::dense_device(n, Fo);
        const std::size_t ldh = Hs.device_ld();
        const int32_t* sp = blocks > 1 ? g.sg->split_points(blocks) : nullptr;
        const detail::TrustedCsr trusted_csr;
        for (int q = 0; q < blocks; ++q) {
            const std::size_t a = std::min(n, static_cast<std::size_t>(q) * width), b = std::min(n, a + width);
            x_ready[static_cast<std::size_t>(q)]->wait_in(s);
            repack(a, b);
            if (b > a)
                check(tg_gemm_rowscale_f32(static_cast<int64_t>(b - a), static_cast<int64_t>(Fo),
                                           static_cast<int64_t>(feature_cols), X.device_data() + a * ldx,
                                           static_cast<int64_t>(ldx), L.weight().device_data(),
                                           static_cast<int64_t>(L.weight().device_ld()),
                                           Hs.mutable_device_data() + a * ldh, static_cast<int64_t>(ldh), g.sg->dis.p + a,
                                           nullptr, TG_ACT_NONE, 0.0f, TG_MODE_FAST | TG_FLAG_C_COLS_PADDED, stream()));
            check(tg_gcn_aggregate_f32(
                static_cast<int64_t>(n), static_cast<int64_t>(n), static_cast<int64_t>(nnz), A.device_row_ptr(),
                A.device_col_ind(), A.device_data(), Hs.device_data(), static_cast<int64_t>(Fo),
                static_cast<int64_t>(ldh), Hs.device_data(), static_cast<int64_t>(ldh), g.sg->dis.p,
                L.has_bias() ? L.bias().device_data() : nullptr,
                L.activation() == Activation::ReLU ? TG_ACT_RELU : TG_ACT_NONE, o.mutable_device_data(),
                static_cast<int64_t>(o.device_ld()), g.sg->order.p, sp ? sp + static_cast<std::size_t>(q) * n : nullptr,
                sp ? sp + static_cast<std::size_t>(q + 1) * n : nullptr, q > 0, q == blocks - 1,
                TG_FLAG_B_ROWS_PADDED, stream()));
        }
        if (layers_[0].post_act == InterActivation::ReLU) relu_inplace(o);
        else if (layers_[0].post_act == InterActivation::ELU) elu_inplace(o);
        H = std::move(o);
        first = 1;
    } else if (first_sage) {
        // Layer 1 per feature block: Tn and Ts rows of block q = X . W_neigh
        // and X . W_self (one tensor-core pass), then the combine pass over
        // the columns of block q; the last pass adds Ts, bias, activation.
        const SAGELayer& L = sage_layers_[layers_[0].start_idx];
        const std::size_t Fo = L.out_features();
        Tensor Tn = Tensor::dense_device(n, Fo), Ts = Tensor::dense_device(n, Fo);
        Tensor o = Tensor::dense_device(n, Fo);
        const std::size_t ldn = Tn.device_ld(), lds = Ts.device_ld();
        const detail::DevWeights w(L.weight_neigh(), L.weight_self());
        DevInts order(n);
        const detail::TrustedCsr trusted_csr;
        check(tg_csr_degree_order(static_cast<int64_t>(n), A.device_row_ptr(), order.p, stream()));
        std::unique_ptr<DevInts> sp;
        if (blocks > 1) {
            sp = std::make_unique<DevInts>(n * static_cast<std::size_t>(blocks + 1));
            check(tg_csr_column_splits(static_cast<int64_t>(n), A.device_row_ptr(), A.device_col_ind(), blocks,
                                       static_cast<int64_t>(width), sp->p, stream()));
        }
        const float* bias = L.has_bias() ? L.bias().device_data() : nullptr;
        const int act = L.activation() == Activation::ReLU ? TG_ACT_RELU : TG_ACT_NONE;
        for (int q = 0; q < blocks; ++q) {
            const std::size_t a = std::min(n, static_cast<std::size_t>(q) * width), b = std::min(n, a + width);
            x_ready[static_cast<std::size_t>(q)]->wait_in(s);
            repack(a, b);
            if (b > a)
                check(tg_gemm_pair_f32(static_cast<int64_t>(b - a), static_cast<int64_t>(Fo),
                                       static_cast<int64_t>(feature_cols), X.device_data() + a * ldx,
                                       static_cast<int64_t>(ldx), w.wn, w.ws, static_cast<int64_t>(Fo),
                                       Tn.mutable_device_data() + a * ldn, static_cast<int64_t>(ldn),
                                       Ts.mutable_device_data() + a * lds, static_cast<int64_t>(lds),
                                       TG_MODE_FAST | TG_FLAG_C_COLS_PADDED, stream()));
            if (sp)
                check(tg_sage_mean_combine_segment_f32(
                    static_cast<int64_t>(n), static_cast<int64_t>(n), A.device_row_ptr(), A.device_col_ind(),
                    sp->p + static_cast<std::size_t>(q) * n, sp->p + static_cast<std::size_t>(q + 1) * n,
                    Tn.device_data(), static_cast<int64_t>(Fo), static_cast<int64_t>(ldn), Ts.device_data(),
                    static_cast<int64_t>(lds), bias, act, o.mutable_device_data(), static_cast<int64_t>(o.device_ld()),
                    order.p, q > 0, q == blocks - 1, TG_FLAG_B_ROWS_PADDED, stream()));
            else
                check(tg_sage_mean_combine_f32(static_cast<int64_t>(n), static_cast<int64_t>(n),
                                               static_cast<int64_t>(nnz), A.device_row_ptr(), A.device_col_ind(),
                                               Tn.device_data(), static_cast<int64_t>(Fo), static_cast<int64_t>(ldn),
                                               Ts.device_data(), static_cast<int64_t>(lds), bias, act,
                                               o.mutable_device_data(), static_cast<int64_t>(o.device_ld()), order.p,
                                               TG_FLAG_B_ROWS_PADDED, stream()));
        }
        if (layers_[0].post_act == InterActivation::ReLU) relu_inplace(o);
        else if (layers_[0].post_act == InterActivation::ELU) elu_inplace(o);
        H = std::move(o);
        first = 1;
    } else {
        x_ready.back()->wait_in(s);
        repack(0, n);
    }
    if (pipelined) X = Tensor();  // not read again
    else H = std::move(X);

    const std::size_t last = layers_.size() - 1;
    for (std::size_t li = first; li < last; ++li) H = run_layer(li, g, H);

    // The last layer, then its output to the host.
    const LayerEntry& e = layers_[last];
    bool chunked = false;
    std::size_t Fo = 0;
    const int chunks = out_chunks();
    if (first <= last && e.type == LayerEntry::Type::GCN && g.sg && n >= 2 * static_cast<std::size_t>(chunks) &&
        e.post_act == InterActivation::None) {
        const GCNLayer& L = gcn_layers_[e.start_idx];
        Fo = L.out_features();
        chunked = H.format() == StorageFormat::Dense && H.cols() == L.in_features() && H.rows() == n &&
                  n * detail::pad4(Fo) * sizeof(float) <= kPassBytes;
    }
    if (first <= last && !chunked) H = run_layer(last, g, H);
    if (!chunked) {
        if (H.cols() != out_cols)
            throw std::invalid_argument("Model::forward_host: the last layer has " + std::to_string(H.cols()) +
                                        " columns, out_cols is " + std::to_string(out_cols));
        std::unique_ptr<DevBuf> pack;
        if (ld_out != H.device_ld() && n && out_cols) pack = std::make_unique<DevBuf>(n * ld_out);
        download_rows(out, ld_out, H.device_data(), H.device_ld(), n, out_cols, pack ? pack->p : nullptr, s);
        detail::cuda(cudaStreamSynchronize(s), "Model::forward_host");
        return;
    }
    if (Fo != out_cols)
        throw std::invalid_argument("Model::forward_host: the last layer has " + std::to_string(Fo) +
                                    " columns, out_cols is " + std::to_string(out_cols));
    // One-pass FAST GCN layer in row chunks (row-offset views of the CSR,
    // each chunk with its own longest-first schedule): per row the same
    // arithmetic as one launch; chunk c's rows go back on the copy stream
    // while chunk c + 1 gathers.
    const GCNLayer& L = gcn_layers_[e.start_idx];
    Tensor Hs = Tensor::dense_device(n, Fo);
    const std::size_t ldh = Hs.device_ld();
    check(tg_gemm_rowscale_f32(static_cast<int64_t>(n), static_cast<int64_t>(Fo), static_cast<int64_t>(H.cols()),
                               H.device_data(), static_cast<int64_t>(H.device_ld()), L.weight().device_data(),
                               static_cast<int64_t>(L.weight().device_ld()), Hs.mutable_device_data(),
                               static_cast<int64_t>(ldh), g.sg->dis.p, nullptr, TG_ACT_NONE, 0.0f, TG_MODE_FAST,
                               stream()));
    Tensor o = Tensor::dense_device(n, Fo);
    const std::size_t ldo = o.device_ld();
    std::unique_ptr<DevBuf> pack;
    if (ld_out != ldo) pack = std::make_unique<DevBuf>(n * ld_out);
    JoinCopies join_out(cs);  // the downloads read o and pack
    const std::size_t step = (n + static_cast<std::size_t>(chunks) - 1) / static_cast<std::size_t>(chunks);
    DevInts order(n);
    std::vector<std::unique_ptr<Event>> chunk_done;
    const detail::TrustedCsr trusted_csr;
    for (std::size_t a = 0; a < n; a += step) {
        const std::size_t b = std::min(n, a + step);
        const int64_t m = static_cast<int64_t>(b - a);
        check(tg_csr_degree_order(m, A.device_row_ptr() + a, order.p + a, stream()));
        check(tg_gcn_aggregate_f32(m, static_cast<int64_t>(n), static_cast<int64_t>(nnz), A.device_row_ptr() + a,
                                   A.device_col_ind(), A.device_data(), Hs.device_data(), static_cast<int64_t>(Fo),
                                   static_cast<int64_t>(ldh), Hs.device_data() + a * ldh, static_cast<int64_t>(ldh),
                                   g.sg->dis.p + a, L.has_bias() ? L.bias().device_data() : nullptr,
                                   L.activation() == Activation::ReLU ? TG_ACT_RELU : TG_ACT_NONE,
                                   o.mutable_device_data() + a * ldo, static_cast<int64_t>(ldo), order.p + a, nullptr,
                                   nullptr, 0, 1, TG_FLAG_B_ROWS_PADDED, stream()));
        chunk_done.push_back(std::make_unique<Event>());
        chunk_done.back()->record(s);
        chunk_done.back()->wait_in(cs);
        download_rows(out + a * ld_out, ld_out, o.device_data() + a * ldo, ldo, b - a, Fo,
                      pack ? pack->p + a * ld_out : nullptr, cs);
    }
    Event copied;
    copied.record(cs);
    copied.wait_in(s);
    detail::cuda(cudaStreamSynchronize(s), "Model::forward_host");
}


// ── Row-partitioned forward ─────────────────────────────────────────────────
namespace {

// A (world * R) x ld exchange buffer whose row j is node j; this rank's
// block starts at row rank * R.
struct Gathered {
    DevBuf buf;
    std::size_t R, ld;
    Gathered(std::size_t P, std::size_t R_, std::size_t ld_) : buf(P * R_ * ld_), R(R_), ld(ld_) {
        detail::cuda(cudaMemsetAsync(buf.p, 0, P * R_ * ld_ * sizeof(float), detail::cstream()), "forward_rows");
    }
    float* block(int rank) { return buf.p + static_cast<std::size_t>(rank) * R * ld; }
};

int act_of(Activation a) { return a == Activation::ReLU ? TG_ACT_RELU : TG_ACT_NONE; }

}  // namespace

Tensor Model::forward_rows(const Tensor& A, std::size_t n, const Tensor& X, RowExchange& ex) const {
    if (layers_.empty()) throw std::runtime_error("Model::forward: no layers configured.");
    const int P = ex.world(), r = ex.rank();
    if (P < 1 || r < 0 || r >= P) throw std::invalid_argument("Model::forward_rows: bad world / rank");
    const std::size_t R = (n + static_cast<std::size_t>(P) - 1) / static_cast<std::size_t>(P);
    const std::size_t row0 = std::min(n, static_cast<std::size_t>(r) * R);
    const std::size_t rows = std::min(R, n - row0);
    if (A.format() != StorageFormat::SparseCSR)
        throw std::invalid_argument("Model::forward_rows: adjacency rows must be SparseCSR (got Dense).");
    if (A.rows() != rows || A.cols() != n)
        throw std::invalid_argument("Model::forward_rows: rank " + std::to_string(r) + " holds rows [" +
                                    std::to_string(row0) + ", " + std::to_string(row0 + rows) + ") of " +
                                    std::to_string(n) + "; adjacency rows are " +
                                    detail::shape_str(A.rows(), A.cols()));
    if (X.format() != StorageFormat::Dense || X.rows() != rows)
        throw std::invalid_argument("Model::forward_rows: feature rows must be Dense with " + std::to_string(rows) +
                                    " rows");
    bool need_norm = false;
    for (const auto& e : layers_) {
        if (e.type == LayerEntry::Type::GAT)
            throw std::invalid_argument("Model::forward_rows: GAT layers are not supported on partitioned graphs");
        need_norm |= e.type == LayerEntry::Type::GCN;
    }
    const bool fast = fast_math();
    const int64_t M = static_cast<int64_t>(rows), K = static_cast<int64_t>(n);
    const detail::TrustedCsr trusted_csr;  // A was checked where it was built

    // Per graph: a longest-first schedule of this block's rows; for GCN in
    // FAST mode this block's 1/sqrt(deg) (rank-local), in EXACT mode the
    // normalised block (its degrees all-gathered for the column scale).
    DevInts order(rows);
    if (rows) check(tg_csr_degree_order(M, A.device_row_ptr(), order.p, stream()));
    DevBuf dis(std::max<std::size_t>(rows, 1));
    Tensor A_gcn;
    std::unique_ptr<DevInts> rp_n, ci_n;
    std::unique_ptr<DevBuf> v_n;
    if (need_norm && fast && rows) {
        check(tg_gcn_norm_scale_f32(M, static_cast<int64_t>(A.nnz()), A.device_row_ptr(), A.device_data(), dis.p,
                                    stream()));
    } else if (need_norm) {
        Gathered dis_all(static_cast<std::size_t>(P), R, 1);
        rp_n = std::make_unique<DevInts>(rows + 1);
        DevInts ins(rows);
        check(tg_gcn_norm_rows_degrees_f32(M, static_cast<int64_t>(row0), static_cast<int64_t>(A.nnz()),
                                           A.device_row_ptr(), A.device_col_ind(), A.device_data(), order.p,
                                           rp_n->p, ins.p, dis_all.block(r), stream()));
        ex.all_gather(dis_all.buf.p, R);
        int32_t nnz_n = 0;
        detail::cuda(cudaMemcpyAsync(&nnz_n, rp_n->p + rows, sizeof(int32_t), cudaMemcpyDeviceToHost,
                                     detail::cstream()),
                     "forward_rows");
        detail::cuda(cudaStreamSynchronize(detail::cstream()), "forward_rows");
        ci_n = std::make_unique<DevInts>(static_cast<std::size_t>(nnz_n));
        v_n = std::make_unique<DevBuf>(static_cast<std::size_t>(nnz_n));
        check(tg_gcn_norm_rows_fill_f32(M, static_cast<int64_t>(row0), K, A.device_row_ptr(), A.device_col_ind(),
                                        A.device_data(), order.p, rp_n->p, ins.p, dis_all.block(r), dis_all.buf.p,
                                        ci_n->p, v_n->p, stream()));
        // the tensor takes the three arrays over (same stream-ordered pool)
        A_gcn = TensorAccess::csr_from_device(rows, n, rp_n->p, ci_n->p, v_n->p, static_cast<std::size_t>(nnz_n));
        rp_n->p = nullptr;
        ci_n->p = nullptr;
        v_n->p = nullptr;
    }

    Tensor H;
    const Tensor* in = &X;
    for (const auto& e : layers_) {
        Tensor out;
        if (e.type == LayerEntry::Type::GCN) {
            const GCNLayer& L = gcn_layers_[e.start_idx];
            if (in->cols() != L.in_features())
                throw std::invalid_argument("GCNLayer::forward: H has " + std::to_string(in->cols()) +
                                            " columns but layer expects in_features=" +
                                            std::to_string(L.in_features()) + ".");
            const std::size_t Fo = L.out_features(), ld = detail::pad4(Fo);
            Gathered full(static_cast<std::size_t>(P), R, ld);
            out = Tensor::dense_device(rows, Fo);
            if (rows) {
                if (fast)  // Hs = diag(dis) . H . W for this block's rows
                    check(tg_gemm_rowscale_f32(M, static_cast<int64_t>(Fo), static_cast<int64_t>(L.in_features()),
                                               in->device_data(), static_cast<int64_t>(in->device_ld()),
                                               L.weight().device_data(), static_cast<int64_t>(L.weight().device_ld()),
                                               full.block(r), static_cast<int64_t>(ld), dis.p, nullptr, TG_ACT_NONE,
                                               0.0f, TG_MODE_FAST, stream()));
                else
                    check(tg_gemm_f32(M, static_cast<int64_t>(Fo), static_cast<int64_t>(L.in_features()),
                                      in->device_data(), static_cast<int64_t>(in->device_ld()), L.weight().device_data(),
                                      static_cast<int64_t>(L.weight().device_ld()), full.block(r),
                                      static_cast<int64_t>(ld), nullptr, TG_ACT_NONE, 0.0f, TG_MODE_EXACT, stream()));
            }
            ex.all_gather(full.buf.p, R * ld);
            if (rows) {
                const float* b = L.has_bias() ? L.bias().device_data() : nullptr;
                if (fast)
                    check(tg_gcn_aggregate_f32(M, K, static_cast<int64_t>(A.nnz()), A.device_row_ptr(),
                                               A.device_col_ind(), A.device_data(), full.buf.p,
                                               static_cast<int64_t>(Fo), static_cast<int64_t>(ld), full.block(r),
                                               static_cast<int64_t>(ld), dis.p, b, act_of(L.activation()),
                                               out.mutable_device_data(), static_cast<int64_t>(out.device_ld()),
                                               order.p, nullptr, nullptr, 0, 1, TG_FLAG_B_ROWS_PADDED, stream()));
                else
                    check(tg_spmm_f32(M, K, static_cast<int64_t>(A_gcn.nnz()), A_gcn.device_row_ptr(),
                                      A_gcn.device_col_ind(), A_gcn.device_data(), full.buf.p, static_cast<int64_t>(Fo),
                                      static_cast<int64_t>(ld), out.mutable_device_data(),
                                      static_cast<int64_t>(out.device_ld()), b, act_of(L.activation()), 0.0f, order.p,
                                      TG_MODE_EXACT | TG_FLAG_B_ROWS_PADDED, stream()));
            }
        } else {  // SAGE
            const SAGELayer& L = sage_layers_[e.start_idx];
            const std::size_t Fi = L.in_features(), Fo = L.out_features();
            if (in->cols() != Fi)
                throw std::invalid_argument("SAGELayer::forward: H has " + std::to_string(in->cols()) +
                                            " columns but layer expects in_features=" + std::to_string(Fi) + ".");
            const bool max = L.aggregator() == SAGELayer::Aggregator::Max;
            const float* b = L.has_bias() ? L.bias().device_data() : nullptr;
            out = Tensor::dense_device(rows, Fo);
            if (fast && !max && Fi > Fo) {
                // transform first: Tn = H . Wn exchanged, Ts = H . Ws local
                const std::size_t ld = detail::pad4(Fo);
                Gathered full(static_cast<std::size_t>(P), R, ld);
                Tensor Ts = Tensor::dense_device(rows, Fo);
                if (rows) {  // both products in one pass over H (column-split epilogue)
                    const detail::DevWeights w(L.weight_neigh(), L.weight_self());
                    check(tg_gemm_pair_f32(M, static_cast<int64_t>(Fo), static_cast<int64_t>(Fi), in->device_data(),
                                           static_cast<int64_t>(in->device_ld()), w.wn, w.ws,
                                           static_cast<int64_t>(Fo), full.block(r), static_cast<int64_t>(ld),
                                           Ts.mutable_device_data(), static_cast<int64_t>(Ts.device_ld()),
                                           TG_MODE_FAST, stream()));
                }
                ex.all_gather(full.buf.p, R * ld);
                if (rows)
                    check(tg_sage_mean_combine_f32(M, K, static_cast<int64_t>(A.nnz()), A.device_row_ptr(),
                                                   A.device_col_ind(), full.buf.p, static_cast<int64_t>(Fo),
                                                   static_cast<int64_t>(ld), Ts.device_data(),
                                                   static_cast<int64_t>(Ts.device_ld()), b, act_of(L.activation()),
                                                   out.mutable_device_data(), static_cast<int64_t>(out.device_ld()),
                                                   order.p, TG_FLAG_B_ROWS_PADDED, stream()));
            } else {
                // aggregate first: every node's H rows exchanged, this block's
                // rows aggregated, then the layer's product
                const std::size_t ld = detail::pad4(Fi);
                Gathered full(static_cast<std::size_t>(P), R, ld);
                if (rows)
                    detail::cuda(cudaMemcpy2DAsync(full.block(r), ld * sizeof(float), in->device_data(),
                                                   in->device_ld() * sizeof(float), Fi * sizeof(float), rows,
                                                   cudaMemcpyDeviceToDevice, detail::cstream()),
                                 "forward_rows");
                ex.all_gather(full.buf.p, R * ld);
                if (rows) {
                    Tensor agg = Tensor::dense_device(rows, Fi);
                    check(tg_sage_aggregate_f32(M, K, static_cast<int64_t>(A.nnz()), A.device_row_ptr(),
                                                A.device_col_ind(), full.buf.p, static_cast<int64_t>(Fi),
                                                static_cast<int64_t>(ld), agg.mutable_device_data(),
                                                static_cast<int64_t>(agg.device_ld()), max ? TG_AGG_MAX : TG_AGG_MEAN,
                                                stream()));
                    if (fast)
                        check(tg_gemm_cat_f32(M, static_cast<int64_t>(Fo), static_cast<int64_t>(Fi), agg.device_data(),
                                              static_cast<int64_t>(agg.device_ld()), static_cast<int64_t>(Fi),
                                              in->device_data(), static_cast<int64_t>(in->device_ld()),
                                              L.weight_neigh().device_data(),
                                              static_cast<int64_t>(L.weight_neigh().device_ld()),
                                              L.weight_self().device_data(),
                                              static_cast<int64_t>(L.weight_self().device_ld()),
                                              out.mutable_device_data(), static_cast<int64_t>(out.device_ld()), b,
                                              act_of(L.activation()), 0.0f, TG_MODE_FAST, stream()));
                    else
                        check(tg_gemm_dual_f32(M, static_cast<int64_t>(Fo), static_cast<int64_t>(Fi),
                                               agg.device_data(), static_cast<int64_t>(agg.device_ld()),
                                               in->device_data(), static_cast<int64_t>(in->device_ld()),
                                               L.weight_neigh().device_data(), L.weight_self().device_data(),
                                               static_cast<int64_t>(L.weight_neigh().device_ld()),
                                               out.mutable_device_data(), static_cast<int64_t>(out.device_ld()), b,
                                               act_of(L.activation()), 0.0f, stream()));
                }
            }
        }
        if (e.post_act == InterActivation::ReLU) relu_inplace(out);
        else if (e.post_act == InterActivation::ELU) elu_inplace(out);
        H = std::move(out);
        in = &H;
    }
    return H;
}

}  // namespace tinygnn
