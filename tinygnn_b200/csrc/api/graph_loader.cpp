// ============================================================================
//  api/graph_loader.cpp -- GraphLoader (reference src/graph_loader.cpp).
//
//  CSV parsing runs on the host with the reference's rules: lines are
//  trimmed and blank lines dropped; a first line whose first field contains
//  a letter or '_' is a header; edges are "src,dst"; features are
//  "node_id,f0,f1,..." placed at row node_id of a (max id + 1) x F matrix.
//  The CSR is built on the device (tg_edge_list_to_csr, bit-identical).
// ============================================================================
#include "tinygnn/graph_loader.hpp"

#include <algorithm>
#include <cctype>
#include <fstream>
#include <sstream>

#include "internal.hpp"

namespace tinygnn {

using detail::check;
using detail::stream;

namespace {

std::string strip(const std::string& s) {
    const auto a = s.find_first_not_of(" \t\r\n");
    if (a == std::string::npos) return {};
    const auto b = s.find_last_not_of(" \t\r\n");
    return s.substr(a, b - a + 1);
}

bool header_line(const std::string& line) {
    for (char c : strip(line)) {
        if (c == ',' || c == ' ' || c == '\t') break;
        if (std::isalpha(static_cast<unsigned char>(c)) || c == '_') return true;
    }
    return false;
}

std::vector<std::string> lines_of(const std::string& path) {
    std::ifstream f(path);
    if (!f.is_open()) throw std::runtime_error("GraphLoader: cannot open file '" + path + "'");
    std::vector<std::string> out;
    std::string raw;
    while (std::getline(f, raw)) {
        std::string t = strip(raw);
        if (!t.empty()) out.push_back(std::move(t));
    }
    return out;
}

template <class T>
T* dalloc(std::size_t n) {
    void* p = nullptr;
    detail::cuda(cudaMallocAsync(&p, (n ? n : 1) * sizeof(T), detail::cstream()), "tinygnn allocation");
    return static_cast<T*>(p);
}

}  // namespace

std::vector<std::pair<int32_t, int32_t>> GraphLoader::parse_edges(const std::string& path) {
    const auto lines = lines_of(path);
    if (lines.empty()) throw std::runtime_error("GraphLoader::parse_edges: file is empty: '" + path + "'");
    std::vector<std::pair<int32_t, int32_t>> edges;
    for (std::size_t i = header_line(lines[0]) ? 1 : 0; i < lines.size(); ++i) {
        const auto& line = lines[i];
        const auto comma = line.find(',');
        if (comma == std::string::npos)
            throw std::runtime_error("GraphLoader::parse_edges: malformed line " + std::to_string(i + 1) + ": '" +
                                     line + "'");
        int32_t s = 0, d = 0;
        try {
            s = static_cast<int32_t>(std::stoi(line.substr(0, comma)));
            d = static_cast<int32_t>(std::stoi(line.substr(comma + 1)));
        } catch (const std::exception&) {
            throw std::runtime_error("GraphLoader::parse_edges: invalid integer on line " + std::to_string(i + 1) +
                                     ": '" + line + "'");
        }
        if (s < 0 || d < 0)
            throw std::runtime_error("GraphLoader::parse_edges: negative node ID on line " + std::to_string(i + 1) +
                                     ": src=" + std::to_string(s) + ", dst=" + std::to_string(d));
        edges.emplace_back(s, d);
    }
    return edges;
}

Tensor GraphLoader::parse_features(const std::string& path) {
    const auto lines = lines_of(path);
    if (lines.empty()) throw std::runtime_error("GraphLoader::parse_features: file is empty: '" + path + "'");
    const std::size_t first = header_line(lines[0]) ? 1 : 0;
    if (lines.size() == first)
        throw std::runtime_error("GraphLoader::parse_features: no data rows in '" + path + "'");
    std::size_t F = 0;
    int32_t max_id = -1;
    std::vector<std::pair<int32_t, std::vector<float>>> rows;
    for (std::size_t i = first; i < lines.size(); ++i) {
        std::istringstream ss(lines[i]);
        std::string tok;
        if (!std::getline(ss, tok, ','))
            throw std::runtime_error("GraphLoader::parse_features: empty line " + std::to_string(i + 1));
        int32_t id = 0;
        try {
            id = static_cast<int32_t>(std::stoi(strip(tok)));
        } catch (const std::exception&) {
            throw std::runtime_error("GraphLoader::parse_features: invalid node_id on line " + std::to_string(i + 1) +
                                     ": '" + tok + "'");
        }
        if (id < 0)
            throw std::runtime_error("GraphLoader::parse_features: negative node_id on line " + std::to_string(i + 1));
        max_id = std::max(max_id, id);
        std::vector<float> feats;
        while (std::getline(ss, tok, ',')) {
            try {
                feats.push_back(std::stof(strip(tok)));
            } catch (const std::exception&) {
                throw std::runtime_error("GraphLoader::parse_features: invalid feature on line " +
                                         std::to_string(i + 1) + ": '" + tok + "'");
            }
        }
        if (F == 0) {
            F = feats.size();
            if (F == 0)
                throw std::runtime_error("GraphLoader::parse_features: no features on line " + std::to_string(i + 1));
        } else if (feats.size() != F) {
            throw std::runtime_error("GraphLoader::parse_features: inconsistent feature count on line " +
                                     std::to_string(i + 1) + ": expected " + std::to_string(F) + " but got " +
                                     std::to_string(feats.size()));
        }
        rows.emplace_back(id, std::move(feats));
    }
    const std::size_t n = static_cast<std::size_t>(max_id + 1);
    std::vector<float> data(n * F, 0.0f);
    for (const auto& [id, f] : rows) std::copy(f.begin(), f.end(), data.begin() + static_cast<std::ptrdiff_t>(id * F));
    return Tensor::dense(n, F, std::move(data));
}

Tensor GraphLoader::edge_list_to_csr(const std::vector<std::pair<int32_t, int32_t>>& edges, std::size_t num_nodes) {
    const std::size_t E = edges.size();
    std::vector<int32_t> src(E), dst(E);
    for (std::size_t e = 0; e < E; ++e) {
        src[e] = edges[e].first;
        dst[e] = edges[e].second;
    }
    int32_t* d_src = dalloc<int32_t>(E);
    int32_t* d_dst = dalloc<int32_t>(E);
    if (E) {
        detail::cuda(cudaMemcpyAsync(d_src, src.data(), E * sizeof(int32_t), cudaMemcpyHostToDevice, detail::cstream()),
                     "edge_list_to_csr");
        detail::cuda(cudaMemcpyAsync(d_dst, dst.data(), E * sizeof(int32_t), cudaMemcpyHostToDevice, detail::cstream()),
                     "edge_list_to_csr");
    }
    int32_t* rp = dalloc<int32_t>(num_nodes + 1);
    int32_t* ci = dalloc<int32_t>(E);
    float* v = dalloc<float>(E);
    const tg_status st = tg_edge_list_to_csr(static_cast<int64_t>(num_nodes), static_cast<int64_t>(E), d_src, d_dst,
                                             rp, ci, v, stream());
    cudaFreeAsync(d_src, detail::cstream());
    cudaFreeAsync(d_dst, detail::cstream());
    Tensor t = TensorAccess::csr_from_device(num_nodes, num_nodes, rp, ci, v, E);
    check(st);
    return t;
}

GraphData GraphLoader::load(const std::string& edges_path, const std::string& features_path) {
    auto edges = parse_edges(edges_path);
    auto features = parse_features(features_path);
    int32_t max_e = -1;
    for (const auto& [s, d] : edges) max_e = std::max({max_e, s, d});
    const std::size_t from_edges = edges.empty() ? 0 : static_cast<std::size_t>(max_e + 1);
    const std::size_t n = std::max(from_edges, features.rows());
    GraphData gd;
    gd.adjacency = edge_list_to_csr(edges, n);
    if (features.rows() < n) {  // zero-pad rows of nodes that only appear in edges
        const std::size_t F = features.cols();
        std::vector<float> grown(n * F, 0.0f);
        const auto& fd = features.data();
        std::copy(fd.begin(), fd.end(), grown.begin());
        features = Tensor::dense(n, F, std::move(grown));
    }
    gd.node_features = std::move(features);
    gd.num_nodes = n;
    gd.num_edges = edges.size();
    gd.num_features = gd.node_features.cols();
    return gd;
}

}  // namespace tinygnn
