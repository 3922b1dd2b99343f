"""The Python module tinygnn_b200.tinygnn (pybind11 over the C++ API): it
imports without a GPU and has TinyGNN's Python surface -- the names of
python/tinygnn/__init__.py and the argument names, defaults and argument
errors of python/tinygnn_ext.cpp.  Nothing here runs a kernel."""
import re

import numpy as np
import pytest

tg = pytest.importorskip("tinygnn_b200.tinygnn", reason="the native module is not built", exc_type=ImportError)

# python/tinygnn/__init__.py:43-73 (re-exports) and tinygnn_ext.cpp:454-468.
REFERENCE_NAMES = [
    "StorageFormat", "Activation", "Tensor", "matmul", "spmm", "relu_inplace", "leaky_relu_inplace",
    "elu_inplace", "sigmoid_inplace", "tanh_inplace", "gelu_inplace", "softmax_inplace", "log_softmax_inplace",
    "add_bias", "add_self_loops", "gcn_norm", "edge_softmax", "sage_max_aggregate", "GCNLayer", "SAGELayer",
    "GATLayer", "Model", "CoraData", "WeightFile", "load_cora_binary", "load_weight_file", "GraphData",
    "GraphLoader", "set_num_threads", "get_max_threads",
]

# (callable path, [(argument, default or None), ...]) as bound in
# python/tinygnn_ext.cpp:197-461.
SIGNATURES = [
    ("matmul", [("A", None), ("B", None)]),
    ("spmm", [("A", None), ("B", None)]),
    ("relu_inplace", [("X", None)]),
    ("leaky_relu_inplace", [("X", None), ("alpha", "0.01")]),
    ("elu_inplace", [("X", None), ("alpha", "1")]),
    ("sigmoid_inplace", [("X", None)]),
    ("tanh_inplace", [("X", None)]),
    ("gelu_inplace", [("X", None)]),
    ("softmax_inplace", [("X", None)]),
    ("log_softmax_inplace", [("X", None)]),
    ("add_bias", [("X", None), ("bias", None)]),
    ("add_self_loops", [("A", None)]),
    ("gcn_norm", [("A", None)]),
    ("edge_softmax", [("A", None)]),
    ("sage_max_aggregate", [("A", None), ("H", None)]),
    ("load_cora_binary", [("path", None)]),
    ("load_weight_file", [("path", None)]),
    ("set_num_threads", [("n", None)]),
    ("Tensor.dense", [("rows", None), ("cols", None)]),
    ("Tensor.dense_from_data", [("rows", None), ("cols", None), ("data", None)]),
    ("Tensor.sparse_csr", [("rows", None), ("cols", None), ("row_ptr", None), ("col_ind", None),
                           ("values", None)]),
    ("Tensor.from_numpy", [("array", None)]),
    ("Tensor.from_numpy_1d", [("array", None)]),
    ("Tensor.from_scipy_csr", [("csr_matrix", None)]),
    ("Tensor.from_edge_index", [("edge_index", None), ("num_nodes", None)]),
    ("Tensor.at", [("row", None), ("col", None)]),
    ("GCNLayer.__init__", [("in_features", None), ("out_features", None), ("use_bias", "True"),
                           ("activation", "Activation.RELU")]),
    ("GCNLayer.set_weight", [("w", None)]),
    ("GCNLayer.set_bias", [("b", None)]),
    ("GCNLayer.forward", [("A_norm", None), ("H", None)]),
    ("SAGELayer.__init__", [("in_features", None), ("out_features", None), ("aggregator", "Aggregator.Mean"),
                            ("use_bias", "True"), ("activation", "Activation.RELU")]),
    ("SAGELayer.set_weight_neigh", [("w", None)]),
    ("SAGELayer.set_weight_self", [("w", None)]),
    ("SAGELayer.set_bias", [("b", None)]),
    ("SAGELayer.forward", [("A", None), ("H", None)]),
    ("GATLayer.__init__", [("in_features", None), ("out_features", None), ("negative_slope", "0.2"),
                           ("use_bias", "True"), ("activation", "Activation.NONE")]),
    ("GATLayer.set_weight", [("w", None)]),
    ("GATLayer.set_attn_left", [("a", None)]),
    ("GATLayer.set_attn_right", [("a", None)]),
    ("GATLayer.set_bias", [("b", None)]),
    ("GATLayer.forward", [("A", None), ("H", None)]),
    ("Model.add_gcn_layer", [("in_f", None), ("out_f", None), ("bias", "True"), ("act", "Activation.RELU"),
                             ("post", "InterActivation.NONE")]),
    ("Model.add_sage_layer", [("in_f", None), ("out_f", None), ("agg", "Aggregator.Mean"), ("bias", "True"),
                              ("act", "Activation.RELU"), ("post", "InterActivation.NONE")]),
    ("Model.add_gat_layer", [("in_f", None), ("out_f", None), ("num_heads", "1"), ("concat", "True"),
                             ("neg_slope", "0.2"), ("bias", "True"), ("act", "Activation.NONE"),
                             ("post", "InterActivation.NONE")]),
    ("Model.load_weights", [("path", None)]),
    ("Model.load_weights_from_file", [("weight_file", None)]),
    ("Model.forward", [("adjacency", None), ("features", None)]),
    ("GraphLoader.parse_edges", [("path", None)]),
    ("GraphLoader.parse_features", [("path", None)]),
    ("GraphLoader.edge_list_to_csr", [("edges", None), ("num_nodes", None)]),
    ("GraphLoader.load", [("edges_path", None), ("features_path", None)]),
]

PROPERTIES = {
    "Tensor": ["format", "rows", "cols", "numel", "nnz", "memory_footprint_bytes"],
    "GCNLayer": ["in_features", "out_features", "has_bias", "activation", "weight", "bias"],
    "SAGELayer": ["in_features", "out_features", "has_bias", "activation", "aggregator", "weight_neigh",
                  "weight_self", "bias"],
    "GATLayer": ["in_features", "out_features", "negative_slope", "has_bias", "activation", "weight",
                 "attn_left", "attn_right", "bias"],
    "Model": ["num_layers"],
    "CoraData": ["num_nodes", "num_features", "num_classes", "num_edges", "adjacency", "features", "labels",
                 "train_mask", "val_mask", "test_mask"],
    "WeightFile": ["test_accuracy", "tensors"],
    "GraphData": ["adjacency", "node_features", "num_nodes", "num_edges", "num_features"],
}


def _resolve(path):
    obj = tg
    for part in path.split("."):
        obj = getattr(obj, part)
    return obj


def _split_top(s):
    """Splits a pybind11 parameter list on top-level commas."""
    out, depth, cur = [], 0, ""
    for ch in s:
        if ch in "[(<":
            depth += 1
        elif ch in "])>":
            depth -= 1
        if ch == "," and depth == 0:
            out.append(cur.strip())
            cur = ""
        else:
            cur += ch
    if cur.strip():
        out.append(cur.strip())
    return out


def _normalise_default(d):
    if d.startswith("<"):
        return d[1:].split(":")[0]  # "<Activation.NONE: 0>" -> "Activation.NONE"
    try:
        return f"{float(d):.6g}"
    except ValueError:
        return d


def _params(fn):
    """[(name, default)] from the first signature line of a pybind11 docstring."""
    line = fn.__doc__.strip().splitlines()[0]
    inner = line[line.index("(") + 1:line.rindex(")")]
    out = []
    for p in _split_top(inner):
        name, _, rest = p.partition(":")
        default = rest.split(" = ", 1)[1] if " = " in rest else None
        if name.strip() != "self":
            out.append((name.strip(), None if default is None else _normalise_default(default.strip())))
    return out


def test_module_exports_the_reference_names():
    missing = [n for n in REFERENCE_NAMES if not hasattr(tg, n)]
    assert not missing, missing
    assert set(REFERENCE_NAMES) <= set(tg.__all__)
    assert tg._core.__file__.startswith(tg.__path__[0]), "module must be the in-tree build"


@pytest.mark.parametrize("path,expected", SIGNATURES, ids=[s[0] for s in SIGNATURES])
def test_argument_names_and_defaults(path, expected):
    assert _params(_resolve(path)) == expected


def test_properties_and_enums():
    for cls, props in PROPERTIES.items():
        for p in props:
            assert isinstance(getattr(getattr(tg, cls), p), property), f"{cls}.{p}"
    assert {m for m in tg.StorageFormat.__members__} == {"Dense", "SparseCSR"}
    assert {m for m in tg.Activation.__members__} == {"NONE", "RELU"}
    assert {m for m in tg.SAGELayer.Aggregator.__members__} == {"Mean", "Max"}
    assert {m for m in tg.Model.InterActivation.__members__} == {"NONE", "RELU", "ELU"}
    assert int(tg.Activation.RELU) == 1 and int(tg.Model.InterActivation.ELU) == 2


def test_host_side_argument_errors():
    """The reference's argument checks and messages (tinygnn_ext.cpp:41-160,
    tensor.cpp sparse_csr validation), raised before any device work."""
    with pytest.raises(ValueError, match=re.escape("Tensor.from_numpy: expected 2D array, got 3D")):
        tg.Tensor.from_numpy(np.zeros((2, 2, 2), np.float32))
    with pytest.raises(ValueError, match=re.escape("Tensor.from_numpy_1d: expected 1D or 2D array, got 3D")):
        tg.Tensor.from_numpy_1d(np.zeros((2, 2, 2), np.float32))
    with pytest.raises(ValueError, match=re.escape("from_edge_index: expected shape (2, E), got (3, 4)")):
        tg.Tensor.from_edge_index(np.zeros((3, 4), np.int32), 5)
    with pytest.raises(ValueError, match="col_ind"):
        tg.Tensor.sparse_csr(2, 3, [0, 2, 4], [0, 1, 1, 3], [1.0] * 4)
    with pytest.raises(ValueError, match="only Dense tensors"):
        tg.Tensor.sparse_csr(2, 3, [0, 2, 4], [0, 1, 1, 2], [1.0] * 4).to_numpy()
    with pytest.raises(ValueError, match="dimension mismatch"):
        tg.matmul(tg.Tensor.dense(2, 3), tg.Tensor.dense(2, 3))
    with pytest.raises(ValueError, match=re.escape("expected shape (4×8), got (3×8)")):
        tg.GCNLayer(4, 8).set_weight(tg.Tensor.dense(3, 8))
    with pytest.raises(RuntimeError, match="cannot open"):
        tg.load_weight_file("/nonexistent/weights.bin")


def test_host_mirrors_and_csv_parsing(tmp_path):
    """Constructors, host copies and CSV parsing (no kernel runs)."""
    a = np.arange(6, dtype=np.float64).reshape(2, 3)
    t = tg.Tensor.from_numpy(a)  # forcecast to float32, like the reference
    assert (t.rows, t.cols, t.numel, t.format) == (2, 3, 6, tg.StorageFormat.Dense)
    assert np.array_equal(t.to_numpy(), a.astype(np.float32))
    assert t.to_numpy().dtype == np.float32
    assert tg.Tensor.from_numpy_1d(np.arange(4)).to_numpy().shape == (1, 4)
    s = tg.Tensor.sparse_csr(2, 3, [0, 2, 4], [0, 1, 1, 2], [1.0, 2.0, 3.0, 4.0])
    assert (s.nnz, s.format) == (4, tg.StorageFormat.SparseCSR)
    assert np.array_equal(s.row_ptr_numpy(), [0, 2, 4]) and s.row_ptr_numpy().dtype == np.int32
    assert np.array_equal(s.col_ind_numpy(), [0, 1, 1, 2])
    assert np.array_equal(s.values_numpy(), [1, 2, 3, 4])
    assert "SparseCSR" in repr(s)
    e = tmp_path / "edges.csv"
    e.write_text("src,dst\n0,1\n\n 1 , 2 \n2,0\n")
    assert tg.GraphLoader.parse_edges(str(e)) == [(0, 1), (1, 2), (2, 0)]
    f = tmp_path / "feat.csv"
    f.write_text("node_id,f0,f1\n0,1.0,2.0\n2,3.0,4.0\n1,5,6\n")
    assert np.array_equal(tg.GraphLoader.parse_features(str(f)).to_numpy(), [[1, 2], [5, 6], [3, 4]])
    tg.set_num_threads(4)
    assert tg.get_max_threads() == 1


def test_dlpack_host_import_copies():
    """Tensor.from_dlpack of host arrays (NumPy, torch CPU; any strides)
    copies into a new tensor; the DLPack methods exist with their names."""
    torch = pytest.importorskip("torch")
    a = np.arange(12, dtype=np.float32).reshape(3, 4)
    assert np.array_equal(tg.Tensor.from_dlpack(a).to_numpy(), a)
    assert np.array_equal(tg.Tensor.from_dlpack(a[:, ::2]).to_numpy(), a[:, ::2])
    tt = torch.arange(6, dtype=torch.float32).reshape(2, 3).t()
    assert np.array_equal(tg.Tensor.from_dlpack(tt).to_numpy(), tt.numpy())
    assert tg.Tensor.from_dlpack(torch.arange(5, dtype=torch.float32)).to_numpy().shape == (1, 5)
    with pytest.raises(ValueError, match="must be float32"):
        tg.Tensor.from_dlpack(np.zeros((2, 2), np.float64))
    with pytest.raises(ValueError, match="expected 1D or 2D array, got 3D"):
        tg.Tensor.from_dlpack(np.zeros((2, 2, 2), np.float32))
    with pytest.raises(ValueError, match="DLPack capsule"):
        tg.Tensor.from_dlpack(object())
    assert _params(tg.Tensor.from_dlpack) == [("array", None)]
    assert _params(tg.Tensor.sparse_csr_from_dlpack) == [("rows", None), ("cols", None), ("row_ptr", None),
                                                         ("col_ind", None), ("values", None)]
    for name in ("__dlpack__", "__dlpack_device__", "row_ptr_dlpack", "col_ind_dlpack", "values_dlpack"):
        assert callable(getattr(tg.Tensor, name))
    # CSR arrays are wrapped in place only: host arrays and other index types are refused
    rp, ci, v = np.array([0, 1], np.int32), np.array([0], np.int32), np.array([1.0], np.float32)
    with pytest.raises(ValueError, match="row_ptr must be on the current CUDA device"):
        tg.Tensor.sparse_csr_from_dlpack(1, 1, rp, ci, v)
    with pytest.raises(ValueError, match="row_ptr must be int32"):
        tg.Tensor.sparse_csr_from_dlpack(1, 1, rp.astype(np.int64), ci, v)
