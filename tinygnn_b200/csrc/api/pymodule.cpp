// ============================================================================
//  pymodule.cpp -- the Python module `tinygnn_b200.tinygnn._core`.
//
//  The same Python surface as TinyGNN's pybind module (python/tinygnn_ext.cpp
//  and python/tinygnn/__init__.py of the reference): Tensor with the NumPy /
//  SciPy / edge_index constructors and accessors, the ops, the graph
//  utilities, GCN / SAGE / GAT layers, Model, CoraData / WeightFile and their
//  loaders, GraphData / GraphLoader, set_num_threads / get_max_threads --
//  same names, argument names and defaults -- bound to this library's C++
//  mirror (include/tinygnn/*.hpp), so every call runs on the GPU.  Device
//  work runs with the GIL released.  Additions: set_fast_math / fast_math,
//  and zero-copy DLPack interop (torch, CuPy, ...): Tensor.from_dlpack,
//  Tensor.sparse_csr_from_dlpack, Tensor.__dlpack__ / __dlpack_device__ and
//  the CSR arrays' *_dlpack capsules.
// ============================================================================
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cuda_runtime.h>

#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "tinygnn/graph_loader.hpp"
#include "tinygnn/layers.hpp"
#include "tinygnn/model.hpp"
#include "tinygnn/ops.hpp"
#include "tinygnn/tensor.hpp"

namespace py = pybind11;
using namespace tinygnn;

namespace {

using FloatArray = py::array_t<float, py::array::c_style | py::array::forcecast>;
using IntArray = py::array_t<int32_t, py::array::c_style | py::array::forcecast>;
using Release = py::call_guard<py::gil_scoped_release>;

Tensor dense_from_array(const FloatArray& a, const char* who) {
    if (a.ndim() != 2)
        throw std::invalid_argument(std::string(who) + ": expected 2D array, got " + std::to_string(a.ndim()) + "D");
    const auto rows = static_cast<std::size_t>(a.shape(0)), cols = static_cast<std::size_t>(a.shape(1));
    return Tensor::dense(rows, cols, std::vector<float>(a.data(), a.data() + rows * cols));
}

Tensor dense_from_array_1d(const FloatArray& a) {
    if (a.ndim() == 1) {
        const auto n = static_cast<std::size_t>(a.shape(0));
        return Tensor::dense(1, n, std::vector<float>(a.data(), a.data() + n));
    }
    if (a.ndim() == 2) return dense_from_array(a, "Tensor.from_numpy_1d");
    throw std::invalid_argument("Tensor.from_numpy_1d: expected 1D or 2D array, got " + std::to_string(a.ndim()) +
                                "D");
}

py::array_t<float> dense_to_array(const Tensor& t) {
    if (t.format() != StorageFormat::Dense)
        throw std::invalid_argument("to_numpy: only Dense tensors can be converted to NumPy.");
    const auto& d = t.data();  // synchronises the host mirror
    py::array_t<float> out({static_cast<py::ssize_t>(t.rows()), static_cast<py::ssize_t>(t.cols())});
    std::copy(d.begin(), d.begin() + static_cast<std::ptrdiff_t>(t.rows() * t.cols()), out.mutable_data());
    return out;
}

Tensor csr_from_scipy(const py::object& m) {
    const IntArray indptr = m.attr("indptr").cast<IntArray>();
    const IntArray indices = m.attr("indices").cast<IntArray>();
    const FloatArray values = m.attr("data").cast<FloatArray>();
    const py::tuple shape = m.attr("shape").cast<py::tuple>();
    const auto rows = shape[0].cast<std::size_t>(), cols = shape[1].cast<std::size_t>();
    if (static_cast<std::size_t>(indptr.size()) != rows + 1)
        throw std::invalid_argument("Tensor.from_scipy_csr: indptr has " + std::to_string(indptr.size()) +
                                    " entries, expected rows + 1 = " + std::to_string(rows + 1));
    const auto nnz = static_cast<std::size_t>(indptr.data()[rows]);
    if (static_cast<std::size_t>(indices.size()) < nnz || static_cast<std::size_t>(values.size()) < nnz)
        throw std::invalid_argument("Tensor.from_scipy_csr: indices / data shorter than indptr[rows]");
    return Tensor::sparse_csr(rows, cols, std::vector<int32_t>(indptr.data(), indptr.data() + rows + 1),
                              std::vector<int32_t>(indices.data(), indices.data() + nnz),
                              std::vector<float>(values.data(), values.data() + nnz));
}

// PyG edge_index (2 x E, row 0 = source) -> row = source CSR with values 1,
// columns sorted within each row: GraphLoader::edge_list_to_csr's layout
// (built on the device), which also checks every id against num_nodes.
Tensor csr_from_edge_index(const IntArray& ei, std::size_t num_nodes) {
    if (ei.ndim() != 2 || ei.shape(0) != 2)
        throw std::invalid_argument("from_edge_index: expected shape (2, E), got (" +
                                    std::to_string(ei.ndim() > 0 ? ei.shape(0) : 0) + ", " +
                                    std::to_string(ei.ndim() > 1 ? ei.shape(1) : 0) + ")");
    const auto E = static_cast<std::size_t>(ei.shape(1));
    std::vector<std::pair<int32_t, int32_t>> edges(E);
    for (std::size_t e = 0; e < E; ++e) edges[e] = {ei.data()[e], ei.data()[E + e]};
    py::gil_scoped_release release;
    return GraphLoader::edge_list_to_csr(edges, num_nodes);
}

py::array_t<int32_t> int_vector(const std::vector<int32_t>& v) {
    return py::array_t<int32_t>(static_cast<py::ssize_t>(v.size()), v.data());
}

// ── DLPack (the data-api exchange ABI, v0.8 unversioned capsules) ──────────
// The structures below are DLPack's published C ABI (dlpack.h), declared
// here because the toolchain ships no copy of the header.
enum : int32_t { kDLCPU = 1, kDLCUDA = 2, kDLCUDAHost = 3 };
enum : uint8_t { kDLInt = 0, kDLFloat = 2 };
struct DLDevice {
    int32_t device_type;
    int32_t device_id;
};
struct DLDataType {
    uint8_t code;
    uint8_t bits;
    uint16_t lanes;
};
struct DLTensor {
    void* data;
    DLDevice device;
    int32_t ndim;
    DLDataType dtype;
    int64_t* shape;
    int64_t* strides;
    uint64_t byte_offset;
};
struct DLManagedTensor {
    DLTensor dl_tensor;
    void* manager_ctx;
    void (*deleter)(DLManagedTensor*);
};

int current_device() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) {
        cudaGetLastError();
        throw std::runtime_error("tinygnn: no CUDA device (DLPack interop needs one)");
    }
    return d;
}

// Takes ownership of a "dltensor" capsule: renames it "used_dltensor" and
// returns the managed tensor with a releaser that runs its deleter.
std::shared_ptr<DLManagedTensor> consume_capsule(const py::object& cap, const char* who) {
    PyObject* c = cap.ptr();
    if (!PyCapsule_IsValid(c, "dltensor"))
        throw std::invalid_argument(std::string(who) + ": expected an unconsumed DLPack capsule (\"dltensor\")");
    auto* m = static_cast<DLManagedTensor*>(PyCapsule_GetPointer(c, "dltensor"));
    PyCapsule_SetName(c, "used_dltensor");
    return std::shared_ptr<DLManagedTensor>(m, [](DLManagedTensor* mt) {
        if (mt && mt->deleter) {
            py::gil_scoped_acquire gil;
            mt->deleter(mt);
        }
    });
}

// The producer's capsule for `obj` (an object with __dlpack__, or a capsule).
// CUDA producers are asked to order their work before the legacy default
// stream (DLPack stream 1), which the API's per-thread stream waits on.
py::object capsule_of(const py::object& obj, bool& on_cuda) {
    on_cuda = false;
    if (!py::hasattr(obj, "__dlpack__")) return obj;
    const auto dev = obj.attr("__dlpack_device__")().cast<std::pair<int, int>>();
    on_cuda = dev.first == kDLCUDA;
    if (on_cuda) return obj.attr("__dlpack__")(py::arg("stream") = 1);
    return obj.attr("__dlpack__")();
}

void check_dtype(const DLTensor& t, uint8_t code, const char* what, const char* who) {
    if (t.dtype.code != code || t.dtype.bits != 32 || t.dtype.lanes != 1)
        throw std::invalid_argument(std::string(who) + ": " + what + " must be " +
                                    (code == kDLFloat ? "float32" : "int32"));
}

// A contiguous 1-D int32 / float32 device array of `n` elements.
template <class T>
T* device_vector(const DLTensor& t, std::size_t n, uint8_t code, const char* what, const char* who) {
    check_dtype(t, code, what, who);
    if (t.device.device_type != kDLCUDA || t.device.device_id != current_device())
        throw std::invalid_argument(std::string(who) + ": " + what + " must be on the current CUDA device");
    if (t.ndim != 1 || static_cast<std::size_t>(t.shape[0]) != n)
        throw std::invalid_argument(std::string(who) + ": " + what + " must be 1-D with " + std::to_string(n) +
                                    " elements");
    if (t.strides && t.shape[0] > 1 && t.strides[0] != 1)
        throw std::invalid_argument(std::string(who) + ": " + what + " must be contiguous");
    return reinterpret_cast<T*>(static_cast<char*>(t.data) + t.byte_offset);
}

// Tensor.from_dlpack: CUDA memory is used in place (the producer stays alive
// as the tensor's owner); host memory is copied into a new tensor.
Tensor tensor_from_dlpack(const py::object& obj) {
    const char* who = "Tensor.from_dlpack";
    bool on_cuda = false;
    auto m = consume_capsule(capsule_of(obj, on_cuda), who);
    const DLTensor& t = m->dl_tensor;
    check_dtype(t, kDLFloat, "the array", who);
    if (t.ndim != 1 && t.ndim != 2)
        throw std::invalid_argument(std::string(who) + ": expected 1D or 2D array, got " + std::to_string(t.ndim) +
                                    "D");
    const std::size_t rows = t.ndim == 2 ? static_cast<std::size_t>(t.shape[0]) : 1;
    const std::size_t cols = static_cast<std::size_t>(t.shape[t.ndim - 1]);
    const int64_t s_col = t.strides ? t.strides[t.ndim - 1] : 1;
    const int64_t s_row = t.ndim == 2 ? (t.strides ? t.strides[0] : static_cast<int64_t>(cols))
                                      : static_cast<int64_t>(cols);
    float* base = reinterpret_cast<float*>(static_cast<char*>(t.data) + t.byte_offset);
    if (t.device.device_type == kDLCPU || t.device.device_type == kDLCUDAHost) {
        std::vector<float> host(rows * cols);
        for (std::size_t r = 0; r < rows; ++r)
            for (std::size_t c = 0; c < cols; ++c) host[r * cols + c] = base[r * s_row + c * s_col];
        return Tensor::dense(rows, cols, std::move(host));
    }
    if (t.device.device_type != kDLCUDA)
        throw std::invalid_argument(std::string(who) + ": unsupported device type " +
                                    std::to_string(t.device.device_type));
    if (t.device.device_id != current_device())
        throw std::invalid_argument(std::string(who) + ": the array is on CUDA device " +
                                    std::to_string(t.device.device_id) + ", not the current device " +
                                    std::to_string(current_device()));
    if ((s_col != 1 && cols > 1) || (rows > 1 && s_row < static_cast<int64_t>(cols)))
        throw std::invalid_argument(std::string(who) + ": a CUDA array needs unit column stride and row stride "
                                    ">= cols (use .contiguous())");
    const std::size_t ld = rows > 1 ? static_cast<std::size_t>(s_row) : cols;
    return Tensor::dense_from_device(rows, cols, ld, base, std::static_pointer_cast<void>(m));
}

Tensor csr_from_dlpack(std::size_t rows, std::size_t cols, const py::object& rp, const py::object& ci,
                       const py::object& vals) {
    const char* who = "Tensor.sparse_csr_from_dlpack";
    bool c0 = false, c1 = false, c2 = false;
    auto mrp = consume_capsule(capsule_of(rp, c0), who);
    auto mci = consume_capsule(capsule_of(ci, c1), who);
    auto mv = consume_capsule(capsule_of(vals, c2), who);
    const std::size_t nnz = mci->dl_tensor.ndim == 1 ? static_cast<std::size_t>(mci->dl_tensor.shape[0]) : 0;
    int32_t* d_rp = device_vector<int32_t>(mrp->dl_tensor, rows + 1, kDLInt, "row_ptr", who);
    int32_t* d_ci = device_vector<int32_t>(mci->dl_tensor, nnz, kDLInt, "col_ind", who);
    float* d_v = device_vector<float>(mv->dl_tensor, nnz, kDLFloat, "values", who);
    auto owner = std::make_shared<std::vector<std::shared_ptr<DLManagedTensor>>>(
        std::vector<std::shared_ptr<DLManagedTensor>>{mrp, mci, mv});
    py::gil_scoped_release release;
    return Tensor::sparse_csr_from_device(rows, cols, nnz, d_rp, d_ci, d_v, std::static_pointer_cast<void>(owner));
}

// Export: a capsule over the tensor's device memory that keeps the Python
// tensor alive until the consumer releases it.  Work queued on the API's
// per-thread stream is ordered before `stream` (DLPack numbering: None or 1
// = legacy default stream, 2 = per-thread default stream, -1 = no sync,
// else a cudaStream_t handle).
struct ExportCtx {
    py::object keep;
    int64_t shape[2];
    int64_t strides[2];
};

void order_before(const py::object& stream) {
    if (!stream.is_none() && stream.cast<int64_t>() == -1) return;
    const int64_t s = stream.is_none() ? 1 : stream.cast<int64_t>();
    if (s == 2) return;  // the same stream
    cudaStream_t consumer = s == 1 ? cudaStreamLegacy : reinterpret_cast<cudaStream_t>(s);
    cudaEvent_t ev;
    if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventRecord(ev, cudaStreamPerThread) != cudaSuccess || cudaStreamWaitEvent(consumer, ev, 0) != cudaSuccess)
        throw std::runtime_error("tinygnn: DLPack stream synchronisation failed: " +
                                 std::string(cudaGetErrorString(cudaGetLastError())));
    cudaEventDestroy(ev);
}

py::capsule export_capsule(const py::object& self, void* data, int ndim, int64_t d0, int64_t d1, int64_t s0,
                           uint8_t code) {
    auto* ctx = new ExportCtx{self, {d0, d1}, {s0, 1}};
    auto* m = new DLManagedTensor{};
    m->dl_tensor.data = data;
    m->dl_tensor.device = DLDevice{kDLCUDA, current_device()};
    m->dl_tensor.ndim = ndim;
    m->dl_tensor.dtype = DLDataType{code, 32, 1};
    m->dl_tensor.shape = ctx->shape;
    m->dl_tensor.strides = ndim == 2 ? ctx->strides : nullptr;
    m->manager_ctx = ctx;
    m->deleter = [](DLManagedTensor* mt) {
        py::gil_scoped_acquire gil;
        delete static_cast<ExportCtx*>(mt->manager_ctx);
        delete mt;
    };
    return py::capsule(m, "dltensor", [](PyObject* cap) {
        if (PyCapsule_IsValid(cap, "dltensor")) {  // never consumed
            auto* mt = static_cast<DLManagedTensor*>(PyCapsule_GetPointer(cap, "dltensor"));
            mt->deleter(mt);
        }
    });
}

py::capsule dense_dlpack(const py::object& self, const py::object& stream) {
    Tensor& t = self.cast<Tensor&>();
    if (t.format() != StorageFormat::Dense)
        throw py::buffer_error("__dlpack__: only Dense tensors export as one array (use the *_dlpack methods of "
                               "a SparseCSR tensor)");
    float* p = t.mutable_device_data();  // uploads if needed; the consumer may write
    order_before(stream);
    return export_capsule(self, p, 2, static_cast<int64_t>(t.rows()), static_cast<int64_t>(t.cols()),
                          static_cast<int64_t>(t.device_ld()), kDLFloat);
}

py::capsule csr_part_dlpack(const py::object& self, int which) {
    Tensor& t = self.cast<Tensor&>();
    if (t.format() != StorageFormat::SparseCSR)
        throw std::invalid_argument("row_ptr_dlpack / col_ind_dlpack / values_dlpack: SparseCSR tensors only");
    void* p = which == 0 ? static_cast<void*>(const_cast<int32_t*>(t.device_row_ptr()))
                         : which == 1 ? static_cast<void*>(const_cast<int32_t*>(t.device_col_ind()))
                                      : static_cast<void*>(const_cast<float*>(t.device_data()));
    order_before(py::int_(1));
    const int64_t n = which == 0 ? static_cast<int64_t>(t.rows()) + 1 : static_cast<int64_t>(t.nnz());
    return export_capsule(self, p, 1, n, 0, 1, which == 2 ? kDLFloat : kDLInt);
}

}  // namespace

PYBIND11_MODULE(_core, m) {
    m.doc() = "TinyGNN's Python API on the B200 (every call runs on the GPU)";

    py::enum_<StorageFormat>(m, "StorageFormat")
        .value("Dense", StorageFormat::Dense)
        .value("SparseCSR", StorageFormat::SparseCSR)
        .export_values();
    py::enum_<Activation>(m, "Activation")
        .value("NONE", Activation::None)
        .value("RELU", Activation::ReLU)
        .export_values();

    py::class_<Tensor>(m, "Tensor")
        .def(py::init<>())
        .def_static("dense", py::overload_cast<std::size_t, std::size_t>(&Tensor::dense), py::arg("rows"),
                    py::arg("cols"))
        .def_static(
            "dense_from_data",
            [](std::size_t rows, std::size_t cols, std::vector<float> data) {
                return Tensor::dense(rows, cols, std::move(data));
            },
            py::arg("rows"), py::arg("cols"), py::arg("data"))
        .def_static("sparse_csr", &Tensor::sparse_csr, py::arg("rows"), py::arg("cols"), py::arg("row_ptr"),
                    py::arg("col_ind"), py::arg("values"))
        .def_static(
            "from_numpy", [](const FloatArray& a) { return dense_from_array(a, "Tensor.from_numpy"); },
            py::arg("array"))
        .def_static("from_numpy_1d", &dense_from_array_1d, py::arg("array"))
        .def_static("from_scipy_csr", &csr_from_scipy, py::arg("csr_matrix"))
        .def_static("from_edge_index", &csr_from_edge_index, py::arg("edge_index"), py::arg("num_nodes"))
        .def("to_numpy", &dense_to_array)
        .def("row_ptr_numpy", [](const Tensor& t) { return int_vector(t.row_ptr()); })
        .def("col_ind_numpy", [](const Tensor& t) { return int_vector(t.col_ind()); })
        .def("values_numpy",
             [](const Tensor& t) {
                 const auto& v = t.data();
                 return py::array_t<float>(static_cast<py::ssize_t>(v.size()), v.data());
             })
        .def_property_readonly("format", &Tensor::format)
        .def_property_readonly("rows", &Tensor::rows)
        .def_property_readonly("cols", &Tensor::cols)
        .def_property_readonly("numel", &Tensor::numel)
        .def_property_readonly("nnz", &Tensor::nnz)
        .def_property_readonly("memory_footprint_bytes", &Tensor::memory_footprint_bytes)
        .def("at", py::overload_cast<std::size_t, std::size_t>(&Tensor::at, py::const_), py::arg("row"),
             py::arg("col"))
        .def("repr", &Tensor::repr)
        .def("__repr__", &Tensor::repr)
        .def_static("from_dlpack", &tensor_from_dlpack, py::arg("array"))
        .def_static("sparse_csr_from_dlpack", &csr_from_dlpack, py::arg("rows"), py::arg("cols"),
                    py::arg("row_ptr"), py::arg("col_ind"), py::arg("values"))
        .def(
            "__dlpack__",
            [](const py::object& self, const py::object& stream, const py::kwargs&) {
                return dense_dlpack(self, stream);
            },
            py::kw_only(), py::arg("stream") = py::none())
        .def("__dlpack_device__",
             [](const Tensor&) { return std::make_pair(static_cast<int>(kDLCUDA), current_device()); })
        .def("row_ptr_dlpack", [](const py::object& self) { return csr_part_dlpack(self, 0); })
        .def("col_ind_dlpack", [](const py::object& self) { return csr_part_dlpack(self, 1); })
        .def("values_dlpack", [](const py::object& self) { return csr_part_dlpack(self, 2); });

    m.def("matmul", &matmul, py::arg("A"), py::arg("B"), Release());
    m.def("spmm", &spmm, py::arg("A"), py::arg("B"), Release());
    m.def("relu_inplace", &relu_inplace, py::arg("X"), Release());
    m.def("leaky_relu_inplace", &leaky_relu_inplace, py::arg("X"), py::arg("alpha") = 0.01f, Release());
    m.def("elu_inplace", &elu_inplace, py::arg("X"), py::arg("alpha") = 1.0f, Release());
    m.def("sigmoid_inplace", &sigmoid_inplace, py::arg("X"), Release());
    m.def("tanh_inplace", &tanh_inplace, py::arg("X"), Release());
    m.def("gelu_inplace", &gelu_inplace, py::arg("X"), Release());
    m.def("softmax_inplace", &softmax_inplace, py::arg("X"), Release());
    m.def("log_softmax_inplace", &log_softmax_inplace, py::arg("X"), Release());
    m.def("add_bias", &add_bias, py::arg("X"), py::arg("bias"), Release());
    m.def("add_self_loops", &add_self_loops, py::arg("A"), Release());
    m.def("gcn_norm", &gcn_norm, py::arg("A"), Release());
    m.def("edge_softmax", &edge_softmax, py::arg("A"), Release());
    m.def("sage_max_aggregate", &sage_max_aggregate, py::arg("A"), py::arg("H"), Release());

    py::class_<GCNLayer>(m, "GCNLayer")
        .def(py::init<std::size_t, std::size_t, bool, Activation>(), py::arg("in_features"), py::arg("out_features"),
             py::arg("use_bias") = true, py::arg("activation") = Activation::ReLU)
        .def("set_weight", &GCNLayer::set_weight, py::arg("w"))
        .def("set_bias", &GCNLayer::set_bias, py::arg("b"))
        .def("forward", &GCNLayer::forward, py::arg("A_norm"), py::arg("H"), Release())
        .def_property_readonly("in_features", &GCNLayer::in_features)
        .def_property_readonly("out_features", &GCNLayer::out_features)
        .def_property_readonly("has_bias", &GCNLayer::has_bias)
        .def_property_readonly("activation", &GCNLayer::activation)
        .def_property_readonly("weight", &GCNLayer::weight)
        .def_property_readonly("bias", &GCNLayer::bias);

    py::class_<SAGELayer> sage(m, "SAGELayer");
    py::enum_<SAGELayer::Aggregator>(sage, "Aggregator")
        .value("Mean", SAGELayer::Aggregator::Mean)
        .value("Max", SAGELayer::Aggregator::Max)
        .export_values();
    sage.def(py::init<std::size_t, std::size_t, SAGELayer::Aggregator, bool, Activation>(), py::arg("in_features"),
             py::arg("out_features"), py::arg("aggregator") = SAGELayer::Aggregator::Mean,
             py::arg("use_bias") = true, py::arg("activation") = Activation::ReLU)
        .def("set_weight_neigh", &SAGELayer::set_weight_neigh, py::arg("w"))
        .def("set_weight_self", &SAGELayer::set_weight_self, py::arg("w"))
        .def("set_bias", &SAGELayer::set_bias, py::arg("b"))
        .def("forward", &SAGELayer::forward, py::arg("A"), py::arg("H"), Release())
        .def_property_readonly("in_features", &SAGELayer::in_features)
        .def_property_readonly("out_features", &SAGELayer::out_features)
        .def_property_readonly("has_bias", &SAGELayer::has_bias)
        .def_property_readonly("activation", &SAGELayer::activation)
        .def_property_readonly("aggregator", &SAGELayer::aggregator)
        .def_property_readonly("weight_neigh", &SAGELayer::weight_neigh)
        .def_property_readonly("weight_self", &SAGELayer::weight_self)
        .def_property_readonly("bias", &SAGELayer::bias);

    py::class_<GATLayer>(m, "GATLayer")
        .def(py::init<std::size_t, std::size_t, float, bool, Activation>(), py::arg("in_features"),
             py::arg("out_features"), py::arg("negative_slope") = 0.2f, py::arg("use_bias") = true,
             py::arg("activation") = Activation::None)
        .def("set_weight", &GATLayer::set_weight, py::arg("w"))
        .def("set_attn_left", &GATLayer::set_attn_left, py::arg("a"))
        .def("set_attn_right", &GATLayer::set_attn_right, py::arg("a"))
        .def("set_bias", &GATLayer::set_bias, py::arg("b"))
        .def("forward", &GATLayer::forward, py::arg("A"), py::arg("H"), Release())
        .def_property_readonly("in_features", &GATLayer::in_features)
        .def_property_readonly("out_features", &GATLayer::out_features)
        .def_property_readonly("negative_slope", &GATLayer::negative_slope)
        .def_property_readonly("has_bias", &GATLayer::has_bias)
        .def_property_readonly("activation", &GATLayer::activation)
        .def_property_readonly("weight", &GATLayer::weight)
        .def_property_readonly("attn_left", &GATLayer::attn_left)
        .def_property_readonly("attn_right", &GATLayer::attn_right)
        .def_property_readonly("bias", &GATLayer::bias);

    py::class_<Model> model(m, "Model");
    py::enum_<Model::InterActivation>(model, "InterActivation")
        .value("NONE", Model::InterActivation::None)
        .value("RELU", Model::InterActivation::ReLU)
        .value("ELU", Model::InterActivation::ELU)
        .export_values();
    model.def(py::init<>())
        .def("add_gcn_layer", &Model::add_gcn_layer, py::arg("in_f"), py::arg("out_f"), py::arg("bias") = true,
             py::arg("act") = Activation::ReLU, py::arg("post") = Model::InterActivation::None)
        .def("add_sage_layer", &Model::add_sage_layer, py::arg("in_f"), py::arg("out_f"),
             py::arg("agg") = SAGELayer::Aggregator::Mean, py::arg("bias") = true, py::arg("act") = Activation::ReLU,
             py::arg("post") = Model::InterActivation::None)
        .def("add_gat_layer", &Model::add_gat_layer, py::arg("in_f"), py::arg("out_f"),
             py::arg("num_heads") = static_cast<std::size_t>(1), py::arg("concat") = true,
             py::arg("neg_slope") = 0.2f, py::arg("bias") = true, py::arg("act") = Activation::None,
             py::arg("post") = Model::InterActivation::None)
        .def("load_weights", py::overload_cast<const std::string&>(&Model::load_weights), py::arg("path"))
        .def("load_weights_from_file", py::overload_cast<const WeightFile&>(&Model::load_weights),
             py::arg("weight_file"))
        .def("forward", &Model::forward, py::arg("adjacency"), py::arg("features"), Release())
        .def_property_readonly("num_layers", &Model::num_layers);

    py::class_<CoraData>(m, "CoraData")
        .def_readonly("num_nodes", &CoraData::num_nodes)
        .def_readonly("num_features", &CoraData::num_features)
        .def_readonly("num_classes", &CoraData::num_classes)
        .def_readonly("num_edges", &CoraData::num_edges)
        .def_readonly("adjacency", &CoraData::adjacency)
        .def_readonly("features", &CoraData::features)
        .def_readonly("labels", &CoraData::labels)
        .def_readonly("train_mask", &CoraData::train_mask)
        .def_readonly("val_mask", &CoraData::val_mask)
        .def_readonly("test_mask", &CoraData::test_mask);
    py::class_<WeightFile>(m, "WeightFile")
        .def_readonly("test_accuracy", &WeightFile::test_accuracy)
        .def_readonly("tensors", &WeightFile::tensors);
    m.def("load_cora_binary", &load_cora_binary, py::arg("path"));
    m.def("load_weight_file", &load_weight_file, py::arg("path"));

    py::class_<GraphData>(m, "GraphData")
        .def_readonly("adjacency", &GraphData::adjacency)
        .def_readonly("node_features", &GraphData::node_features)
        .def_readonly("num_nodes", &GraphData::num_nodes)
        .def_readonly("num_edges", &GraphData::num_edges)
        .def_readonly("num_features", &GraphData::num_features);
    py::class_<GraphLoader>(m, "GraphLoader")
        .def_static("parse_edges", &GraphLoader::parse_edges, py::arg("path"))
        .def_static("parse_features", &GraphLoader::parse_features, py::arg("path"))
        .def_static("edge_list_to_csr", &GraphLoader::edge_list_to_csr, py::arg("edges"), py::arg("num_nodes"))
        .def_static("load", &GraphLoader::load, py::arg("edges_path"), py::arg("features_path"));

    // Host thread count: the reference parallelises on the CPU; here every
    // call runs on the GPU, so the count is accepted and has no effect.
    m.def("set_num_threads", [](int) {}, py::arg("n"));
    m.def("get_max_threads", []() { return 1; });
    m.def("set_fast_math", &set_fast_math, py::arg("fast"));
    m.def("fast_math", &fast_math);
}
