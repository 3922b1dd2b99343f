// ============================================================================
//  tinygnn/model.hpp -- Model (execution graph) and the binary file loaders.
//
//  Same interface as the reference's include/tinygnn/model.hpp:42-164:
//  load_cora_binary, the TGNN weight file format (magic "TGNN", version 1,
//  test accuracy, named row-major fp32 tensors), Model::add_*_layer,
//  load_weights (names layer{i}.weight|bias|weight_neigh|weight_self|
//  head{j}.{weight,attn_left,attn_right,bias}) and forward.  forward runs on
//  the device: gcn_norm / add_self_loops once per call, every layer's fused
//  kernels, and a multi-head GAT layer as one pass over the graph for all
//  heads (heads concatenated or averaged as in model.cpp:403-422).
// ============================================================================
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "tinygnn/layers.hpp"
#include "tinygnn/tensor.hpp"

namespace tinygnn {

struct CoraData {
    std::size_t num_nodes = 0, num_features = 0, num_classes = 0, num_edges = 0;
    Tensor adjacency;   // SparseCSR N x N, values 1.0
    Tensor features;    // Dense N x F
    std::vector<int32_t> labels;
    std::vector<uint8_t> train_mask, val_mask, test_mask;
};

CoraData load_cora_binary(const std::string& path);

struct WeightFile {
    float test_accuracy = 0.0f;
    std::unordered_map<std::string, Tensor> tensors;
};

WeightFile load_weight_file(const std::string& path);

namespace detail {
struct ForwardGraphs;  // the adjacency variants one forward call uses
}

// A Model::forward recorded once as a CUDA graph and replayed (no
// counterpart in the reference).  For small graphs a forward is a couple of
// dozen short kernels whose launches cost more than their work; a replay
// issues them as one graph launch.  The graph reads the adjacency and
// feature tensors it was captured with -- their device memory, with
// whatever it holds at replay time -- so those tensors must outlive it and
// keep their shapes; the output lives in the graph's own tensor.
class ForwardGraph {
public:
    ForwardGraph();
    ForwardGraph(ForwardGraph&&) noexcept;
    ForwardGraph& operator=(ForwardGraph&&) noexcept;
    ~ForwardGraph();
    // Runs the captured forward again on the calling thread's stream and
    // returns its output (complete when the stream reaches it).
    const Tensor& replay();
    const Tensor& output() const;

    struct Impl;

private:
    friend class Model;
    std::unique_ptr<Impl> impl_;
};

// The exchange step of a row-partitioned forward (no counterpart in the
// reference): `world` processes, each holding one equal block of
// R = ceil(n / world) rows; all_gather(buf, count) runs on the calling
// thread's stream and leaves block q's `count` floats (at buf + q * count,
// this rank's block filled by the caller) in every rank's buf.
class RowExchange {
public:
    virtual ~RowExchange() = default;
    virtual int world() const = 0;
    virtual int rank() const = 0;
    virtual void all_gather(float* buf, std::size_t count) = 0;
};

class Model {
public:
    enum class InterActivation : uint8_t { None = 0, ReLU = 1, ELU = 2 };

    std::size_t add_gcn_layer(std::size_t in_f, std::size_t out_f, bool bias = true,
                              Activation act = Activation::ReLU,
                              InterActivation post = InterActivation::None);
    std::size_t add_sage_layer(std::size_t in_f, std::size_t out_f,
                               SAGELayer::Aggregator agg = SAGELayer::Aggregator::Mean, bool bias = true,
                               Activation act = Activation::ReLU,
                               InterActivation post = InterActivation::None);
    std::size_t add_gat_layer(std::size_t in_f, std::size_t out_f, std::size_t num_heads = 1,
                              bool concat = true, float neg_slope = 0.2f, bool bias = true,
                              Activation act = Activation::None,
                              InterActivation post = InterActivation::None);
    std::size_t num_layers() const noexcept { return layers_.size(); }

    void load_weights(const std::string& path);
    void load_weights(const WeightFile& wf);

    Tensor forward(const Tensor& adjacency, const Tensor& features) const;

    // Model::forward on this process's block of an n-node graph partitioned
    // into equal row blocks (rows [rank * R, rank * R + rows), R = ceil(n /
    // world)): adjacency_rows is that block's rows with global column ids
    // (rows x n), feature_rows its feature rows; returns its output rows.
    // Every process calls it with the same model.  GCN and SAGE layers; the
    // result equals the rows of forward() on the whole graph (bit for bit in
    // EXACT mode).  No counterpart in the reference.
    Tensor forward_rows(const Tensor& adjacency_rows, std::size_t n, const Tensor& feature_rows,
                        RowExchange& exchange) const;

    // forward() from host buffers, for callers that hold the graph and the
    // features in host memory (no counterpart in the reference): the raw
    // adjacency as CSR arrays (values NULL: an unweighted graph, every value
    // 1.0, written on the device instead of crossing PCIe) and the n x
    // feature_cols features at row stride ld_features in; the last layer's
    // n x out_cols output written to `out` at row stride ld_out before the
    // call returns.  The uploads run on a copy stream, overlapped with the
    // compute: the CSR first (checked on the device with Tensor::sparse_csr's
    // checks as soon as it has landed), then the features in row blocks.
    // When the first layer is a GCN layer (or a transform-first SAGE-mean
    // layer) in FAST mode, its GEMM and its gather pass over block q's
    // columns start as soon as block q has landed,
    // and when the last layer is a one-pass FAST GCN layer it runs in row
    // chunks whose outputs go back while the next chunk runs.  Same results
    // as forward() on tensors holding the same data.  Host buffers in pinned
    // (page-locked) memory let the copies overlap; pageable ones work, with
    // the driver's staging and less overlap.
    void forward_host(std::size_t n, std::size_t nnz, const int32_t* row_ptr, const int32_t* col_ind,
                      const float* values, const float* features, std::size_t feature_cols,
                      std::size_t ld_features, float* out, std::size_t out_cols, std::size_t ld_out) const;

    // forward(adjacency, features) recorded as a CUDA graph after one eager
    // run (no counterpart in the reference).  Every call the forward makes
    // must be asynchronous: FAST-mode GCN and SAGE layers are; EXACT
    // gcn_norm and GAT's self-loops read a size back to the host, and their
    // capture is refused (std::runtime_error).  Output equals forward()'s.
    ForwardGraph capture(const Tensor& adjacency, const Tensor& features) const;

private:
    Tensor run_layer(std::size_t li, detail::ForwardGraphs& g, const Tensor& in) const;

    struct LayerEntry {
        enum class Type : uint8_t { GCN, SAGE, GAT };
        Type type;
        std::size_t start_idx, count;
        bool gat_concat;
        InterActivation post_act;
    };
    std::vector<LayerEntry> layers_;
    std::vector<GCNLayer> gcn_layers_;
    std::vector<SAGELayer> sage_layers_;
    std::vector<GATLayer> gat_layers_;
};

}  // namespace tinygnn
