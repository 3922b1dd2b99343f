// ============================================================================
//  tinygnn/layers.hpp -- graph utilities and GNN layers on device tensors.
//
//  Same interface and validation as the reference's include/tinygnn/
//  layers.hpp:91-443 (constructor defaults, set_* shape checks, messages).
//  forward() runs the fused sm_100a kernels: GCN = GEMM + gather with
//  bias/activation epilogue; SAGE = aggregate + interleaved dual product;
//  GAT = GEMM + exact scores + one-pass online-softmax aggregation.
// ============================================================================
#pragma once

#include <cstddef>
#include <cstdint>

#include "tinygnn/tensor.hpp"

namespace tinygnn {

enum class Activation : uint8_t { None = 0, ReLU = 1 };

Tensor add_self_loops(const Tensor& A);                 // layers.hpp:121
Tensor gcn_norm(const Tensor& A);                        // layers.hpp:145
Tensor sage_max_aggregate(const Tensor& A, const Tensor& H);  // layers.hpp:324
Tensor edge_softmax(const Tensor& A);                    // layers.hpp:349

struct GCNLayer {
    GCNLayer(std::size_t in_features, std::size_t out_features, bool use_bias = true,
             Activation act = Activation::ReLU);
    void set_weight(Tensor w);
    void set_bias(Tensor b);
    Tensor forward(const Tensor& A_norm, const Tensor& H) const;
    std::size_t in_features() const noexcept { return in_features_; }
    std::size_t out_features() const noexcept { return out_features_; }
    bool has_bias() const noexcept { return use_bias_; }
    Activation activation() const noexcept { return activation_; }
    const Tensor& weight() const noexcept { return weight_; }
    const Tensor& bias() const noexcept { return bias_; }

private:
    std::size_t in_features_, out_features_;
    bool use_bias_;
    Activation activation_;
    Tensor weight_, bias_;
};

struct SAGELayer {
    enum class Aggregator : uint8_t { Mean = 0, Max = 1 };
    SAGELayer(std::size_t in_features, std::size_t out_features, Aggregator agg = Aggregator::Mean,
              bool use_bias = true, Activation act = Activation::ReLU);
    void set_weight_neigh(Tensor w);
    void set_weight_self(Tensor w);
    void set_bias(Tensor b);
    Tensor forward(const Tensor& A, const Tensor& H) const;
    std::size_t in_features() const noexcept { return in_features_; }
    std::size_t out_features() const noexcept { return out_features_; }
    Aggregator aggregator() const noexcept { return aggregator_; }
    bool has_bias() const noexcept { return use_bias_; }
    Activation activation() const noexcept { return activation_; }
    const Tensor& weight_neigh() const noexcept { return weight_neigh_; }
    const Tensor& weight_self() const noexcept { return weight_self_; }
    const Tensor& bias() const noexcept { return bias_; }

private:
    std::size_t in_features_, out_features_;
    Aggregator aggregator_;
    bool use_bias_;
    Activation activation_;
    Tensor weight_neigh_, weight_self_, bias_;
};

struct GATLayer {
    GATLayer(std::size_t in_features, std::size_t out_features, float negative_slope = 0.2f,
             bool use_bias = true, Activation act = Activation::None);
    void set_weight(Tensor w);
    void set_attn_left(Tensor a);
    void set_attn_right(Tensor a);
    void set_bias(Tensor b);
    Tensor forward(const Tensor& A, const Tensor& H) const;
    std::size_t in_features() const noexcept { return in_features_; }
    std::size_t out_features() const noexcept { return out_features_; }
    float negative_slope() const noexcept { return negative_slope_; }
    bool has_bias() const noexcept { return use_bias_; }
    Activation activation() const noexcept { return activation_; }
    const Tensor& weight() const noexcept { return weight_; }
    const Tensor& attn_left() const noexcept { return attn_left_; }
    const Tensor& attn_right() const noexcept { return attn_right_; }
    const Tensor& bias() const noexcept { return bias_; }

private:
    std::size_t in_features_, out_features_;
    float negative_slope_;
    bool use_bias_;
    Activation activation_;
    Tensor weight_, attn_left_, attn_right_, bias_;
};

}  // namespace tinygnn
