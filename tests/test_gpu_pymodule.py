"""tinygnn_b200.tinygnn (TinyGNN's Python API) on the device, against the
oracle: the reference's post-install smoke cases (python/tinygnn/tests/
smoke_tests.py C1-C12) with their known answers, then every op, layer,
constructor and loader with the exactness the kernel tests require --
bit-identical for CSR construction, self-loops, gcn_norm, spmm, matmul,
ReLU / leaky ReLU, add_bias, SAGE max aggregation, GCN and SAGE layers;
|d| <= 1e-5 + 1e-4 |ref| for the transcendental ops, GAT and whole models."""
import struct

import numpy as np
import pytest

import oracle
from tests.helpers import assert_bits_equal, assert_close, powerlaw_csr, rand_csr

pytestmark = pytest.mark.gpu
P = oracle.port


@pytest.fixture(scope="module")
def tg():
    import torch

    assert torch.cuda.is_available()
    import tinygnn_b200.tinygnn as m
    return m


def _triangle(tg):
    return tg.Tensor.sparse_csr(3, 3, [0, 2, 4, 6], [1, 2, 0, 2, 0, 1], [1.0] * 6)


def _csr(tg, rp, ci, v, cols=None):
    return tg.Tensor.sparse_csr(rp.size - 1, rp.size - 1 if cols is None else cols, rp, ci, v)


def _arrays(t):
    return t.row_ptr_numpy(), t.col_ind_numpy(), t.values_numpy()


def _write_weights(path, tensors, acc=0.0):
    """TGNN weight file: magic, version 1, accuracy, count, then per tensor
    name length, name, rows, cols, row-major fp32 (src/model.cpp:130-190)."""
    with open(path, "wb") as fh:
        fh.write(b"TGNN" + struct.pack("<IfI", 1, acc, len(tensors)))
        for name, a in tensors.items():
            a = np.asarray(a, np.float32)
            a = a.reshape(1, -1) if a.ndim == 1 else a
            nb = name.encode()
            fh.write(struct.pack("<I", len(nb)) + nb + struct.pack("<II", *a.shape) + a.tobytes())


def test_reference_smoke_cases(tg, tmp_path):
    # C1 tensor creation
    t = tg.Tensor.dense(4, 3)
    assert (t.rows, t.cols, t.numel) == (4, 3, 12)
    assert np.array_equal(t.to_numpy(), np.zeros((4, 3), np.float32))
    s = _triangle(tg)
    assert (s.nnz, s.rows, s.cols) == (6, 3, 3)
    # C2 numpy round trip
    arr = np.random.default_rng(2).standard_normal((5, 7)).astype(np.float32)
    assert_bits_equal(tg.Tensor.from_numpy(arr).to_numpy(), arr, "round trip")
    # C3 matmul
    C = tg.matmul(tg.Tensor.dense_from_data(2, 2, [1, 2, 3, 4]), tg.Tensor.dense_from_data(2, 2, [5, 6, 7, 8]))
    assert np.array_equal(C.to_numpy(), [[19, 22], [43, 50]])
    # C4 spmm
    A = tg.Tensor.sparse_csr(2, 3, [0, 2, 4], [0, 1, 1, 2], [1.0, 1.0, 1.0, 1.0])
    B = tg.Tensor.from_numpy(np.array([[1, 0], [0, 1], [2, 2]], np.float32))
    assert np.array_equal(tg.spmm(A, B).to_numpy(), [[1, 1], [2, 3]])
    # C5 relu
    X = tg.Tensor.from_numpy(np.array([[-3, -1, 0, 1, 4]], np.float32))
    tg.relu_inplace(X)
    assert np.array_equal(X.to_numpy(), [[0, 0, 0, 1, 4]])
    # C6 / C7 self-loops and normalisation
    Asl = tg.add_self_loops(s)
    assert Asl.nnz == 9
    An = tg.gcn_norm(Asl)
    rs = tg.spmm(An, tg.Tensor.from_numpy(np.ones((3, 1), np.float32))).to_numpy().ravel()
    assert np.all((rs > 0) & (rs <= 1 + 1e-5))
    # C8-C11 layers: shapes and finiteness (exact values in the tests below)
    rng = np.random.default_rng(8)
    H = tg.Tensor.from_numpy(rng.standard_normal((3, 4)).astype(np.float32))
    w = lambda r, c: tg.Tensor.from_numpy((rng.standard_normal((r, c)) * 0.1).astype(np.float32))  # noqa: E731
    g = tg.GCNLayer(4, 8, True, tg.Activation.RELU)
    g.set_weight(w(4, 8))
    g.set_bias(tg.Tensor.from_numpy(np.zeros((1, 8), np.float32)))
    outs = [g.forward(tg.gcn_norm(s), H)]
    for agg in (tg.SAGELayer.Aggregator.Mean, tg.SAGELayer.Aggregator.Max):
        L = tg.SAGELayer(4, 8, agg, True, tg.Activation.RELU)
        L.set_weight_neigh(w(4, 8))
        L.set_weight_self(w(4, 8))
        L.set_bias(tg.Tensor.from_numpy(np.zeros((1, 8), np.float32)))
        outs.append(L.forward(s, H))
    G = tg.GATLayer(4, 8, 0.2, True, tg.Activation.RELU)
    G.set_weight(w(4, 8))
    G.set_attn_left(w(1, 8))
    G.set_attn_right(w(1, 8))
    G.set_bias(tg.Tensor.from_numpy(np.zeros((1, 8), np.float32)))
    outs.append(G.forward(Asl, H))
    for o in outs:
        o = o.to_numpy()
        assert o.shape == (3, 8) and np.all(np.isfinite(o))
    # C12 two-layer model from a weight file
    m = tg.Model()
    m.add_gcn_layer(4, 8, True, tg.Activation.RELU)
    m.add_gcn_layer(8, 3, True, tg.Activation.NONE)
    assert m.num_layers == 2
    wts = {"layer0.weight": rng.standard_normal((4, 8)) * 0.1, "layer0.bias": np.zeros((1, 8)),
           "layer1.weight": rng.standard_normal((8, 3)) * 0.1, "layer1.bias": np.zeros((1, 3))}
    _write_weights(tmp_path / "w.bin", wts)
    m.load_weights(str(tmp_path / "w.bin"))
    o = m.forward(s, H).to_numpy()
    assert o.shape == (3, 3) and np.all(np.isfinite(o))


def test_ops_match_the_oracle(tg):
    rng = np.random.default_rng(11)
    n, f = 3000, 44
    rp, ci, v = powerlaw_csr(rng, n, 9)
    A = _csr(tg, rp, ci, v)
    X = rng.standard_normal((n, f)).astype(np.float32)
    W = rng.standard_normal((f, 20)).astype(np.float32)
    b = rng.standard_normal(f).astype(np.float32)
    T = tg.Tensor.from_numpy(X)
    assert_bits_equal(tg.spmm(A, T).to_numpy(), P.spmm(rp, ci, v, X), "spmm")
    assert_bits_equal(tg.matmul(T, tg.Tensor.from_numpy(W)).to_numpy(), P.matmul(X, W), "matmul")
    for name, alpha, exact in [("relu", 0.0, True), ("leaky_relu", 0.05, True), ("elu", 0.7, False),
                               ("sigmoid", 0.0, False), ("tanh", 0.0, False), ("gelu", 0.0, False),
                               ("softmax", 0.0, False), ("log_softmax", 0.0, False)]:
        Y = tg.Tensor.from_numpy(X)
        fn = getattr(tg, name + "_inplace")
        fn(Y, alpha) if name in ("leaky_relu", "elu") else fn(Y)
        (assert_bits_equal if exact else assert_close)(Y.to_numpy(), P.activation(name, X, alpha), name)
    Y = tg.Tensor.from_numpy(X)
    tg.add_bias(Y, tg.Tensor.from_numpy_1d(b))
    assert_bits_equal(Y.to_numpy(), P.add_bias(X, b), "add_bias")
    for name in ("add_self_loops", "gcn_norm"):
        got, ref = _arrays(getattr(tg, name)(A)), getattr(P, name)(rp, ci, v)
        for g_, r_, k in zip(got, ref, ("row_ptr", "col_ind", "values")):
            assert_bits_equal(g_, r_, f"{name}.{k}")
    Es = tg.edge_softmax(A)
    assert_bits_equal(Es.row_ptr_numpy(), rp, "edge_softmax.row_ptr")
    assert_close(Es.values_numpy(), P.edge_softmax(rp, ci, v), "edge_softmax")
    assert_bits_equal(tg.sage_max_aggregate(A, T).to_numpy(), P.sage_max_aggregate(rp, ci, v, X), "sage_max")
    Xd = X[:4]
    assert Xd.shape == (4, f) and tg.Tensor.from_numpy(Xd).at(3, 5) == Xd[3, 5]


@pytest.mark.parametrize("agg", ["mean", "max"])
def test_layers_match_the_oracle(tg, agg):
    rng = np.random.default_rng(5)
    n, fi, fo = 2500, 96, 40
    rp, ci, v = rand_csr(rng, n, n, 7, weighted=False, diag=False, empty_frac=0.05)
    X = rng.standard_normal((n, fi)).astype(np.float32)
    H = tg.Tensor.from_numpy(X)
    A = _csr(tg, rp, ci, v)
    W, Wn, Ws = ((rng.standard_normal((fi, fo)) * 0.1).astype(np.float32) for _ in range(3))
    b = (rng.standard_normal(fo) * 0.1).astype(np.float32)
    dn = tg.Tensor.from_numpy
    g = tg.GCNLayer(fi, fo)
    g.set_weight(dn(W))
    g.set_bias(tg.Tensor.from_numpy_1d(b))
    An = tg.gcn_norm(A)
    assert_bits_equal(g.forward(An, H).to_numpy(), P.gcn_layer(*_arrays(An), X, W, b, True), "GCNLayer")
    assert (g.in_features, g.out_features, g.has_bias, g.activation) == (fi, fo, True, tg.Activation.RELU)
    assert_bits_equal(g.weight.to_numpy(), W, "GCNLayer.weight")
    aggr = tg.SAGELayer.Aggregator.Mean if agg == "mean" else tg.SAGELayer.Aggregator.Max
    s = tg.SAGELayer(fi, fo, aggr, True, tg.Activation.NONE)
    s.set_weight_neigh(dn(Wn))
    s.set_weight_self(dn(Ws))
    s.set_bias(tg.Tensor.from_numpy_1d(b))
    assert_bits_equal(s.forward(A, H).to_numpy(), P.sage_layer(rp, ci, v, X, Wn, Ws, b, agg, False),
                      f"SAGELayer {agg}")
    assert s.aggregator == aggr
    a_l, a_r = (rng.standard_normal(fo) * 0.5).astype(np.float32), (rng.standard_normal(fo) * 0.5).astype(np.float32)
    G = tg.GATLayer(fi, fo, 0.15, True, tg.Activation.RELU)
    G.set_weight(dn(W))
    G.set_attn_left(tg.Tensor.from_numpy_1d(a_l))
    G.set_attn_right(tg.Tensor.from_numpy_1d(a_r))
    G.set_bias(tg.Tensor.from_numpy_1d(b))
    Asl = tg.add_self_loops(A)
    assert_close(G.forward(Asl, H).to_numpy(), P.gat_layer(*_arrays(Asl), X, W, a_l, a_r, b, 0.15, True), "GATLayer")


def _weights(rng, spec):
    w = {}
    for li, L in enumerate(spec):
        p = f"layer{li}"
        r = lambda *s: (rng.standard_normal(s) * 0.2).astype(np.float32)  # noqa: E731
        if L["type"] == "gcn":
            w[f"{p}.weight"], w[f"{p}.bias"] = r(L["in"], L["out"]), r(L["out"])
        elif L["type"] == "sage":
            w[f"{p}.weight_neigh"], w[f"{p}.weight_self"], w[f"{p}.bias"] = (r(L["in"], L["out"]),
                                                                              r(L["in"], L["out"]), r(L["out"]))
        else:
            for h in range(L["heads"]):
                q = f"{p}.head{h}"
                w[f"{q}.weight"], w[f"{q}.attn_left"], w[f"{q}.attn_right"], w[f"{q}.bias"] = (
                    r(L["in"], L["out"]), r(L["out"]), r(L["out"]), r(L["out"]))
    return w


@pytest.mark.parametrize("name", ["gcn", "sage", "gat"])
def test_model_from_weight_file_matches_the_oracle(tg, tmp_path, name):
    rng = np.random.default_rng(len(name) + 40)
    n = 2000
    rp, ci, v = powerlaw_csr(rng, n, 8, weighted=False, diag=False)
    m = tg.Model()
    if name == "gcn":
        spec = [dict(type="gcn", **{"in": 120, "out": 16}, act="relu"), dict(type="gcn", **{"in": 16, "out": 7})]
        m.add_gcn_layer(120, 16)
        m.add_gcn_layer(16, 7, act=tg.Activation.NONE)
    elif name == "sage":
        spec = [dict(type="sage", **{"in": 120, "out": 32}, agg="max", act="relu"),
                dict(type="sage", **{"in": 32, "out": 7}, post="relu")]
        m.add_sage_layer(120, 32, agg=tg.SAGELayer.Aggregator.Max)
        m.add_sage_layer(32, 7, act=tg.Activation.NONE, post=tg.Model.InterActivation.RELU)
    else:
        spec = [dict(type="gat", **{"in": 120, "out": 8}, heads=4, concat=True, post="elu"),
                dict(type="gat", **{"in": 32, "out": 7}, heads=2, concat=False)]
        m.add_gat_layer(120, 8, num_heads=4, post=tg.Model.InterActivation.ELU)
        m.add_gat_layer(32, 7, num_heads=2, concat=False)
    w = _weights(rng, spec)
    path = str(tmp_path / f"{name}.bin")
    _write_weights(path, w, acc=0.8125)
    wf = tg.load_weight_file(path)
    assert wf.test_accuracy == np.float32(0.8125) and set(wf.tensors) == set(w)
    m.load_weights_from_file(wf)
    X = rng.standard_normal((n, 120)).astype(np.float32)
    A, H = _csr(tg, rp, ci, v), tg.Tensor.from_numpy(X)
    ref = oracle.model_forward(P, spec, w, rp, ci, v, X)
    assert_close(m.forward(A, H).to_numpy(), ref, f"Model {name}")
    m2 = tg.Model()
    for L in spec:  # same layers, weights through load_weights(path)
        if L["type"] == "gcn":
            m2.add_gcn_layer(L["in"], L["out"], act=tg.Activation.RELU if L.get("act") else tg.Activation.NONE)
        elif L["type"] == "sage":
            m2.add_sage_layer(L["in"], L["out"], agg=tg.SAGELayer.Aggregator.Max if L.get("agg") == "max"
                              else tg.SAGELayer.Aggregator.Mean,
                              act=tg.Activation.RELU if L.get("act") else tg.Activation.NONE,
                              post=tg.Model.InterActivation.RELU if L.get("post") else tg.Model.InterActivation.NONE)
        else:
            m2.add_gat_layer(L["in"], L["out"], num_heads=L["heads"], concat=L["concat"],
                             post=tg.Model.InterActivation.ELU if L.get("post") else tg.Model.InterActivation.NONE)
    m2.load_weights(path)
    assert_bits_equal(m2.forward(A, H).to_numpy(), m.forward(A, H).to_numpy(), f"Model {name} reload")


def test_constructors_match_the_oracle(tg):
    scipy_sparse = pytest.importorskip("scipy.sparse")
    rng = np.random.default_rng(3)
    n, E = 700, 5000
    src, dst = rng.integers(0, n, E).astype(np.int32), rng.integers(0, n, E).astype(np.int32)
    src[:50], dst[:50] = src[50:100], dst[50:100]  # duplicate edges stay (src/graph_loader.cpp:244-274)
    t = tg.Tensor.from_edge_index(np.stack([src, dst]), n)
    for g_, r_, k in zip(_arrays(t), P.edge_list_to_csr(src, dst, n), ("row_ptr", "col_ind", "values")):
        assert_bits_equal(g_, r_, f"from_edge_index.{k}")
    e = tg.GraphLoader.edge_list_to_csr(list(zip(src.tolist(), dst.tolist())), n)
    assert_bits_equal(e.col_ind_numpy(), t.col_ind_numpy(), "edge_list_to_csr")
    assert tg.Tensor.from_edge_index(np.zeros((2, 0), np.int32), 0).nnz == 0
    with pytest.raises(ValueError, match="out of range"):
        tg.Tensor.from_edge_index(np.array([[0, 1], [1, n]], np.int32), n)
    S = scipy_sparse.random(400, 300, density=0.02, format="csr", random_state=1, dtype=np.float64)
    t = tg.Tensor.from_scipy_csr(S)
    assert (t.rows, t.cols, t.nnz) == (400, 300, S.nnz)
    assert_bits_equal(t.values_numpy(), S.data.astype(np.float32), "from_scipy_csr values")
    B = rng.standard_normal((300, 16)).astype(np.float32)
    assert_bits_equal(tg.spmm(t, tg.Tensor.from_numpy(B)).to_numpy(),
                      P.spmm(S.indptr, S.indices, S.data.astype(np.float32), B), "spmm(from_scipy_csr)")


def test_loaders_match_the_oracle(tg, tmp_path):
    rng = np.random.default_rng(4)
    n, F, C, E = 300, 12, 5, 1400
    src, dst = rng.integers(0, n, E).astype(np.int32), rng.integers(0, n, E).astype(np.int32)
    X = rng.standard_normal((n, F)).astype(np.float32)
    ref = P.edge_list_to_csr(src, dst, n)
    # GraphLoader.load: CSV edges + features (node ids out of order)
    (tmp_path / "e.csv").write_text("src,dst\n" + "".join(f"{a},{b}\n" for a, b in zip(src, dst)))
    order = rng.permutation(n)
    (tmp_path / "f.csv").write_text("node_id," + ",".join(f"f{j}" for j in range(F)) + "\n" +
                                    "".join(f"{i}," + ",".join(repr(float(x)) for x in X[i]) + "\n" for i in order))
    gd = tg.GraphLoader.load(str(tmp_path / "e.csv"), str(tmp_path / "f.csv"))
    assert (gd.num_nodes, gd.num_edges, gd.num_features) == (n, E, F)
    assert_bits_equal(gd.node_features.to_numpy(), X, "GraphData.node_features")
    for g_, r_, k in zip(_arrays(gd.adjacency), ref, ("row_ptr", "col_ind", "values")):
        assert_bits_equal(g_, r_, f"GraphData.adjacency.{k}")
    # load_cora_binary: N, F, C, E (uint32), features, labels, 3 masks, src, dst
    labels = rng.integers(0, C, n).astype(np.int32)
    masks = [(rng.random(n) < p).astype(np.uint8) for p in (0.2, 0.3, 0.5)]
    blob = struct.pack("<4I", n, F, C, E) + X.tobytes() + labels.tobytes() + b"".join(m.tobytes() for m in masks)
    (tmp_path / "cora.bin").write_bytes(blob + src.tobytes() + dst.tobytes())
    cd = tg.load_cora_binary(str(tmp_path / "cora.bin"))
    assert (cd.num_nodes, cd.num_features, cd.num_classes, cd.num_edges) == (n, F, C, E)
    assert_bits_equal(cd.features.to_numpy(), X, "CoraData.features")
    assert list(cd.labels) == labels.tolist() and list(cd.test_mask) == masks[2].tolist()
    for g_, r_, k in zip(_arrays(cd.adjacency), ref, ("row_ptr", "col_ind", "values")):
        assert_bits_equal(g_, r_, f"CoraData.adjacency.{k}")


def test_dlpack_zero_copy_with_torch(tg):
    """torch CUDA tensors in and out without copies: the same device memory,
    ops on imported tensors bit-identical to the oracle, in-place ops visible
    to torch, the producer kept alive by the tensor."""
    import gc

    import torch
    rng = np.random.default_rng(21)
    n, f = 1500, 41
    rp, ci, v = rand_csr(rng, n, n, 6)
    X = rng.standard_normal((n, 44)).astype(np.float32)
    xt = torch.as_tensor(X).cuda()
    view = xt[:, :f]                        # row stride 44, 41 columns
    T = tg.Tensor.from_dlpack(view)
    assert (T.rows, T.cols) == (n, f)
    back = torch.from_dlpack(T)
    assert back.data_ptr() == view.data_ptr() and back.stride() == (44, 1)
    # CSR arrays from torch, used in place and validated on the device
    d = lambda a: torch.as_tensor(a).cuda()  # noqa: E731
    A = tg.Tensor.sparse_csr_from_dlpack(n, n, d(rp), d(ci), d(v))
    ref = P.spmm(rp, ci, v, X[:, :f].copy())
    assert_bits_equal(tg.spmm(A, T).to_numpy(), ref, "spmm on DLPack tensors")
    An = tg.gcn_norm(A)
    for arr, r_, k in zip((An.row_ptr_dlpack(), An.col_ind_dlpack(), An.values_dlpack()),
                          P.gcn_norm(rp, ci, v), ("row_ptr", "col_ind", "values")):
        assert_bits_equal(torch.from_dlpack(arr).cpu().numpy(), r_, f"gcn_norm.{k} via DLPack")
    with pytest.raises(ValueError, match="out of bounds"):
        bad = ci.copy()
        bad[7] = n
        tg.Tensor.sparse_csr_from_dlpack(n, n, d(rp), d(bad), d(v))
    # in place through the shared memory; the producer outlives its name
    tg.relu_inplace(T)
    assert_bits_equal(xt[:, :f].cpu().numpy(), np.maximum(X[:, :f], 0), "relu_inplace seen by torch")
    assert_bits_equal(xt[:, f:].cpu().numpy(), X[:, f:], "padding columns untouched")
    del view, back, xt
    gc.collect()
    torch.cuda.empty_cache()
    assert_bits_equal(T.to_numpy(), np.maximum(X[:, :f], 0), "tensor alive after the producer's name is gone")
    # a host-created tensor exports after its upload
    H = tg.Tensor.from_numpy(X)
    assert_bits_equal(torch.from_dlpack(H).cpu().numpy(), X, "export of a host tensor")
    # a GCN layer whose operands all come from torch
    W = (rng.standard_normal((f, 16)) * 0.2).astype(np.float32)
    g = tg.GCNLayer(f, 16, False, tg.Activation.RELU)
    g.set_weight(tg.Tensor.from_dlpack(d(W)))
    Xc = np.maximum(X[:, :f], 0)
    got = torch.from_dlpack(g.forward(An, tg.Tensor.from_dlpack(d(Xc)))).cpu().numpy()
    assert_bits_equal(got, P.gcn_layer(*P.gcn_norm(rp, ci, v), Xc, W, None, True), "GCNLayer on DLPack tensors")
