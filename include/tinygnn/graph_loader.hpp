// ============================================================================
//  tinygnn/graph_loader.hpp -- CSR construction (and the CSV loaders).
//
//  Same interface as the reference's include/tinygnn/graph_loader.hpp:41-86.
//  edge_list_to_csr runs on the device and is bit-identical to the
//  reference (count, scan, scatter, per-row sort, values 1.0, no dedup).
//  The CSV readers parse on the host (header sniffing, CRLF, zero-padding of
//  feature rows, the reference's error messages) and hand the arrays to the
//  device build.
// ============================================================================
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <utility>
#include <vector>

#include "tinygnn/tensor.hpp"

namespace tinygnn {

struct GraphData {
    Tensor adjacency;       // SparseCSR num_nodes x num_nodes, values 1.0
    Tensor node_features;   // Dense num_nodes x num_features
    std::size_t num_nodes = 0, num_edges = 0, num_features = 0;
};

class GraphLoader {
public:
    static std::vector<std::pair<int32_t, int32_t>> parse_edges(const std::string& path);
    static Tensor parse_features(const std::string& path);
    static Tensor edge_list_to_csr(const std::vector<std::pair<int32_t, int32_t>>& edges, std::size_t num_nodes);
    static GraphData load(const std::string& edges_path, const std::string& features_path);
};

}  // namespace tinygnn
