// C++ API (include/tinygnn/*.hpp) on the device: TinyGNN's known answers
// (tests/test_spmm.cpp:198, test_matmul.cpp:160, test_gcn.cpp:288,514,
// test_graphsage.cpp:362,509, test_gat.cpp:332,370,
// test_graph_loader.cpp:330) and its exceptions, through tinygnn::Tensor /
// ops / layers / Model / GraphLoader.  Exit code 0 = all passed.
#include <cmath>
#include <cstdio>
#include <fstream>
#include <functional>
#include <stdexcept>
#include <string>
#include <vector>

#include "tinygnn/graph_loader.hpp"
#include "tinygnn/layers.hpp"
#include "tinygnn/model.hpp"
#include "tinygnn/ops.hpp"
#include "tinygnn/tensor.hpp"

using namespace tinygnn;

static int g_fail = 0, g_pass = 0;
#define CHECK(cond)                                                                \
    do {                                                                           \
        if (cond) ++g_pass;                                                        \
        else {                                                                     \
            ++g_fail;                                                              \
            std::printf("FAIL %s:%d: %s\n", __FILE__, __LINE__, #cond);            \
        }                                                                          \
    } while (0)
#define NEAR(a, b, tol) CHECK(std::fabs(double(a) - double(b)) <= (tol))

template <class E>
static bool throws(const std::function<void()>& f, const char* needle = nullptr) {
    try {
        f();
    } catch (const E& e) {
        return !needle || std::string(e.what()).find(needle) != std::string::npos;
    } catch (...) {
        return false;
    }
    return false;
}

static Tensor undirected(std::size_t n, std::vector<std::pair<int, int>> pairs) {
    std::vector<std::pair<int32_t, int32_t>> e;
    for (auto [u, v] : pairs) {
        e.emplace_back(u, v);
        e.emplace_back(v, u);
    }
    return GraphLoader::edge_list_to_csr(e, n);
}

int main(int argc, char** argv) {
    // scratch files go to the directory the caller gives (a per-test temp dir)
    const std::string tmpdir = argc > 1 ? argv[1] : ".";
    // spmm 3x3 (test_spmm.cpp:198)
    {
        auto A = Tensor::sparse_csr(3, 3, {0, 2, 3, 5}, {0, 1, 1, 0, 2}, {1, 1, 1, 1, 1});
        auto B = Tensor::dense(3, 2, {1, 2, 3, 4, 5, 6});
        auto C = spmm(A, B);
        const std::vector<float> want = {4, 6, 3, 4, 6, 8};
        CHECK(C.rows() == 3 && C.cols() == 2 && C.format() == StorageFormat::Dense);
        for (int i = 0; i < 6; ++i) NEAR(C.data()[i], want[i], 1e-4);
        CHECK(throws<std::invalid_argument>([&] { spmm(A, Tensor::dense(4, 2)); }, "spmm: dimension mismatch"));
        CHECK(throws<std::invalid_argument>([&] { spmm(B, B); }, "spmm: tensor A must be SparseCSR"));
    }
    // matmul 4x4 (test_matmul.cpp:160)
    {
        std::vector<float> a(16), b(16);
        for (int i = 0; i < 16; ++i) { a[i] = float(i + 1); b[i] = float(i + 17); }
        auto C = matmul(Tensor::dense(4, 4, a), Tensor::dense(4, 4, b));
        NEAR(C.at(0, 0), 250, 1e-4);
        NEAR(C.at(3, 3), 1528, 1e-4);
        NEAR(C.at(1, 2), 670, 1e-4);
        CHECK(throws<std::invalid_argument>([&] { matmul(Tensor::dense(2, 3), Tensor::dense(2, 3)); },
                                            "matmul: dimension mismatch"));
    }
    // gcn_norm 3-node path (test_gcn.cpp:288)
    {
        auto An = gcn_norm(undirected(3, {{0, 1}, {1, 2}}));
        const double s6 = 1.0 / std::sqrt(6.0);
        const std::vector<int32_t> rp = {0, 2, 5, 7}, ci = {0, 1, 0, 1, 2, 1, 2};
        const std::vector<double> v = {0.5, s6, s6, 1.0 / 3, s6, s6, 0.5};
        CHECK(An.nnz() == 7 && An.row_ptr() == rp && An.col_ind() == ci);
        for (int i = 0; i < 7; ++i) NEAR(An.data()[i], v[i], 1e-5);
    }
    // GCN forward 3-node (test_gcn.cpp:514)
    {
        auto An = gcn_norm(undirected(3, {{0, 1}, {1, 2}}));
        GCNLayer layer(2, 2, true, Activation::ReLU);
        layer.set_weight(Tensor::dense(2, 2, {1.0f, 0.5f, 0.5f, 1.0f}));
        layer.set_bias(Tensor::dense(1, 2, {0.1f, -0.1f}));
        auto out = layer.forward(An, Tensor::dense(3, 2, {1, 0, 0, 1, 1, 1}));
        NEAR(out.at(0, 0), 0.804124, 1e-4);
        NEAR(out.at(0, 1), 0.558248, 1e-4);
        NEAR(out.at(1, 0), 1.287287, 1e-4);
        NEAR(out.at(1, 1), 1.049829, 1e-4);
        NEAR(out.at(2, 0), 1.054124, 1e-4);
        NEAR(out.at(2, 1), 1.058248, 1e-4);
        CHECK(throws<std::invalid_argument>([&] { layer.set_weight(Tensor::dense(3, 2)); },
                                            "GCNLayer::set_weight: expected shape"));
        CHECK(throws<std::invalid_argument>([&] { layer.forward(An, Tensor::dense(3, 5)); },
                                            "columns but layer expects in_features=2"));
    }
    // SAGE mean and max (test_graphsage.cpp:362, 509)
    {
        auto A = undirected(3, {{0, 1}, {1, 2}});
        auto H = Tensor::dense(3, 2, {1, 0, 0, 1, 1, 1});
        SAGELayer mean(2, 2, SAGELayer::Aggregator::Mean, true, Activation::ReLU);
        mean.set_weight_neigh(Tensor::dense(2, 2, {1, 0.5f, 0.5f, 1}));
        mean.set_weight_self(Tensor::dense(2, 2, {0.5f, 0, 0, 0.5f}));
        mean.set_bias(Tensor::dense(1, 2, {0.1f, -0.1f}));
        auto o = mean.forward(A, H);
        const std::vector<float> want = {1.1f, 0.9f, 1.35f, 1.4f, 1.1f, 1.4f};
        for (int i = 0; i < 6; ++i) NEAR(o.data()[i], want[i], 1e-4);
        SAGELayer mx(2, 2, SAGELayer::Aggregator::Max, false, Activation::None);
        mx.set_weight_neigh(Tensor::dense(2, 2, {1, 0, 0, 1}));
        mx.set_weight_self(Tensor::dense(2, 2, {1, 0, 0, 1}));
        auto m = mx.forward(A, H);
        const std::vector<float> wm = {1, 1, 1, 2, 1, 2};
        for (int i = 0; i < 6; ++i) NEAR(m.data()[i], wm[i], 1e-5);
        CHECK(throws<std::invalid_argument>([&] { mx.set_bias(Tensor::dense(1, 2)); }, "use_bias=false"));
    }
    // GAT 2-node and uniform attention (test_gat.cpp:332, 370)
    {
        auto A = add_self_loops(undirected(2, {{0, 1}}));
        GATLayer g(2, 2, 0.2f, false, Activation::None);
        g.set_weight(Tensor::dense(2, 2, {1, 0, 0, 1}));
        g.set_attn_left(Tensor::dense(1, 2, {1, 0}));
        g.set_attn_right(Tensor::dense(1, 2, {0, 1}));
        auto o = g.forward(A, Tensor::dense(2, 2, {1, 0, 0, 1}));
        const double e1 = std::exp(1.0), e2 = std::exp(2.0);
        NEAR(o.at(0, 0), e1 / (e1 + e2), 1e-5);
        NEAR(o.at(0, 1), e2 / (e1 + e2), 1e-5);
        NEAR(o.at(1, 0), 1 / (1 + e1), 1e-5);
        NEAR(o.at(1, 1), e1 / (1 + e1), 1e-5);
        auto A3 = add_self_loops(undirected(3, {{0, 1}, {1, 2}}));
        GATLayer u(2, 2, 0.2f, false, Activation::None);
        u.set_weight(Tensor::dense(2, 2, {1, 0, 0, 1}));
        auto uo = u.forward(A3, Tensor::dense(3, 2, {1, 2, 3, 4, 5, 6}));
        const std::vector<float> want = {2, 3, 3, 4, 4, 5};
        for (int i = 0; i < 6; ++i) NEAR(uo.data()[i], want[i], 1e-5);
    }
    // edge_list_to_csr known graph (test_graph_loader.cpp:330)
    {
        std::vector<std::pair<int32_t, int32_t>> e = {{0, 1}, {0, 2}, {1, 0}, {1, 3}, {2, 0},
                                                      {2, 3}, {2, 4}, {3, 1}, {3, 2}, {4, 2}};
        auto adj = GraphLoader::edge_list_to_csr(e, 5);
        CHECK(adj.row_ptr() == std::vector<int32_t>({0, 2, 4, 7, 9, 10}));
        CHECK(adj.col_ind() == std::vector<int32_t>({1, 2, 0, 3, 0, 3, 4, 1, 2, 2}));
        CHECK(adj.memory_footprint_bytes() == 10 * 8 + 6 * 4);
        CHECK(throws<std::invalid_argument>([&] { GraphLoader::edge_list_to_csr({{0, 7}}, 3); },
                                            "edge[0].dst = 7 out of range [0, 3)"));
    }
    // Tensor semantics: validation, at(), host edits reach the device, deep copies
    {
        CHECK(throws<std::invalid_argument>([] { Tensor::sparse_csr(2, 2, {0, 1, 3}, {0, 1}, {1, 1}); },
                                            "row_ptr.back() (3) must equal values.size() (2)"));
        CHECK(throws<std::invalid_argument>([] { Tensor::sparse_csr(2, 2, {0, 1, 2}, {0, 5}, {1, 1}); },
                                            "col_ind[1] = 5 is out of bounds for cols=2"));
        auto X = Tensor::dense(2, 3, {-1, 2, -3, 4, -5, 6});
        CHECK(throws<std::out_of_range>([&] { X.at(2, 0); }));
        relu_inplace(X);  // on the device
        NEAR(X.at(0, 0), 0, 0);
        NEAR(X.at(1, 2), 6, 0);
        X.at(0, 1) = -7.0f;  // host edit, then a device op must see it
        relu_inplace(X);
        NEAR(X.at(0, 1), 0, 0);
        Tensor Y = X;  // deep copy
        Y.at(1, 2) = 100.0f;
        NEAR(X.at(1, 2), 6, 0);
        CHECK(X.repr() == "Tensor(2x3, Dense, 24 bytes)");
        auto S = Tensor::dense(2, 3, {1, 2, 3, 1, 1, 1});
        log_softmax_inplace(S);
        double s = 0;
        for (int j = 0; j < 3; ++j) s += std::exp(S.at(0, j));
        NEAR(s, 1.0, 1e-6);
    }
    // Model: weights from a TGNN file, multi-head GAT (concat + ELU) then GCN
    {
        const std::string path_s = tmpdir + "/tinygnn_b200_cpp_api_weights.bin";
        const char* path = path_s.c_str();
        std::vector<std::pair<std::string, std::vector<float>>> ts;
        std::vector<std::pair<uint32_t, uint32_t>> shapes;
        auto add = [&](const std::string& n, uint32_t r, uint32_t c, float seed) {
            std::vector<float> v(r * c);
            for (std::size_t i = 0; i < v.size(); ++i) v[i] = std::sin(seed + 0.37f * float(i)) * 0.5f;
            ts.emplace_back(n, v);
            shapes.emplace_back(r, c);
        };
        for (int h = 0; h < 3; ++h) {
            const std::string p = "layer0.head" + std::to_string(h);
            add(p + ".weight", 4, 2, 1.0f + h);
            add(p + ".attn_left", 1, 2, 2.0f + h);
            add(p + ".attn_right", 1, 2, 3.0f + h);
            add(p + ".bias", 1, 2, 4.0f + h);
        }
        add("layer1.weight", 6, 3, 5.0f);
        add("layer1.bias", 1, 3, 6.0f);
        {
            std::ofstream f(path, std::ios::binary);
            f.write("TGNN", 4);
            const uint32_t ver = 1, n = static_cast<uint32_t>(ts.size());
            const float acc = 0.5f;
            f.write(reinterpret_cast<const char*>(&ver), 4);
            f.write(reinterpret_cast<const char*>(&acc), 4);
            f.write(reinterpret_cast<const char*>(&n), 4);
            for (std::size_t i = 0; i < ts.size(); ++i) {
                const uint32_t len = static_cast<uint32_t>(ts[i].first.size());
                f.write(reinterpret_cast<const char*>(&len), 4);
                f.write(ts[i].first.data(), len);
                f.write(reinterpret_cast<const char*>(&shapes[i].first), 4);
                f.write(reinterpret_cast<const char*>(&shapes[i].second), 4);
                f.write(reinterpret_cast<const char*>(ts[i].second.data()),
                        static_cast<std::streamsize>(ts[i].second.size() * 4));
            }
        }
        Model m;
        m.add_gat_layer(4, 2, 3, true, 0.2f, true, Activation::None, Model::InterActivation::ELU);
        m.add_gcn_layer(6, 3, true, Activation::None);
        m.load_weights(path);
        auto A = undirected(6, {{0, 1}, {1, 2}, {2, 3}, {3, 4}, {4, 5}, {0, 5}, {1, 4}});
        std::vector<float> xv(24);
        for (int i = 0; i < 24; ++i) xv[i] = std::cos(0.3f * i);
        auto X = Tensor::dense(6, 4, xv);
        auto Y = m.forward(A, X);
        // the same composition by hand: three single-head layers, concat, ELU, GCN
        auto wf = load_weight_file(path);
        NEAR(wf.test_accuracy, 0.5, 0);
        auto Asl = add_self_loops(A);
        std::vector<float> cat(6 * 6);
        for (int h = 0; h < 3; ++h) {
            const std::string p = "layer0.head" + std::to_string(h);
            GATLayer g(4, 2);
            g.set_weight(wf.tensors.at(p + ".weight"));
            g.set_attn_left(wf.tensors.at(p + ".attn_left"));
            g.set_attn_right(wf.tensors.at(p + ".attn_right"));
            g.set_bias(wf.tensors.at(p + ".bias"));
            auto o = g.forward(Asl, X);
            for (int i = 0; i < 6; ++i)
                for (int j = 0; j < 2; ++j) cat[i * 6 + h * 2 + j] = o.at(i, j);
        }
        auto C = Tensor::dense(6, 6, cat);
        elu_inplace(C);
        GCNLayer g1(6, 3, true, Activation::None);
        g1.set_weight(wf.tensors.at("layer1.weight"));
        g1.set_bias(wf.tensors.at("layer1.bias"));
        auto Y2 = g1.forward(gcn_norm(A), C);
        CHECK(Y.rows() == 6 && Y.cols() == 3);
        for (int i = 0; i < 18; ++i) NEAR(Y.data()[i], Y2.data()[i], 1e-5 + 1e-4 * std::fabs(Y2.data()[i]));
        Model empty;
        CHECK(throws<std::runtime_error>([&] { empty.forward(A, X); }, "no layers configured"));
        CHECK(throws<std::runtime_error>([&] { load_weight_file("/nonexistent/file.bin"); }, "cannot open"));
        std::remove(path);
    }
    std::printf("C++ API: %d passed, %d failed\n", g_pass, g_fail);
    return g_fail == 0 ? 0 : 1;
}
