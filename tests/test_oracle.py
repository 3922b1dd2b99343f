"""The oracle is pinned before anything is checked against it (CPU only).

* The C restatement (oracle.port) reproduces, bit for bit, the outputs of the
  reference library stored in tests/golden/golden_ref.npz.
* It meets the hand-computed known answers of TinyGNN's own unit tests
  (tests/golden/known_answers.json), within those tests' tolerances.
* Where the reference library itself is built (oracle/_ref), it is compared
  live on fresh seeded inputs, including heavy-tailed rows and edge cases.
"""
import numpy as np
import pytest

import oracle
from tests.helpers import (assert_bits_equal, assert_close, powerlaw_csr, rand_csr,
                           undirected_csr)

P = oracle.port
needs_ref = pytest.mark.skipif(oracle.ref is None, reason="oracle/_ref not built (no reference sources)")


def test_port_library_loaded():
    assert P is not None, "oracle/_build/libtg_oracle.so missing: run `make -C oracle`"


# ── golden_ref.npz: outputs of the reference library itself ─────────────────
def _port_output(case, g):
    if case.startswith("spmm_"):
        return P.spmm(g["rp"], g["ci"], g["v"], g["B"])
    if case.startswith("matmul_"):
        return P.matmul(g["A"], g["B"])
    if case.startswith("asl_"):
        return P.add_self_loops(g["rp"], g["ci"], g["v"])
    if case.startswith("gcnnorm_"):
        return P.gcn_norm(g["rp"], g["ci"], g["v"])
    if case == "el2csr":
        return P.edge_list_to_csr(g["src"], g["dst"], int(g["n"]))
    if case == "edge_softmax":
        return P.edge_softmax(g["rp"], g["ci"], g["v"])
    if case.startswith("sagemax_"):
        return P.sage_max_aggregate(g["rp"], g["ci"], g["v"], g["H"])
    if case.startswith("act_"):
        return P.activation(case[4:], g["X"], float(g["alpha"]))
    if case == "add_bias":
        return P.add_bias(g["X"], g["b"])
    if case.startswith("gcn_"):
        return P.gcn_layer(g["rp"], g["ci"], g["v"], g["H"], g["W"], g["b"], True)
    if case.startswith("sage_"):
        agg = case.split("_")[1]
        return P.sage_layer(g["rp"], g["ci"], None, g["H"], g["Wn"], g["Ws"], g["b"], agg, True)
    if case.startswith("gat_"):
        return P.gat_layer(g["rp"], g["ci"], None, g["H"], g["W"], g["al"], g["ar"], g["b"], 0.2, False)
    if case.startswith("model_"):
        spec, weights = model_spec(case, g)
        y = oracle.model_forward(P, spec, weights, g["rp"], g["ci"], g["v"], g["X"])
        return P.activation("log_softmax", y)
    raise KeyError(case)


def model_spec(case, g):
    """Layer spec + named weights of the model_* golden cases."""
    if case == "model_gcn":
        return ([dict(type="gcn", **{"in": 48, "out": 16}, act="relu"),
                 dict(type="gcn", **{"in": 16, "out": 7}, act=None)],
                {"layer0.weight": g["W0"], "layer0.bias": g["b0"], "layer1.weight": g["W1"], "layer1.bias": g["b1"]})
    if case == "model_sage":
        return ([dict(type="sage", **{"in": 48, "out": 32}, act="relu"),
                 dict(type="sage", **{"in": 32, "out": 10}, act=None)],
                {"layer0.weight_neigh": g["Wn0"], "layer0.weight_self": g["Ws0"], "layer0.bias": g["b0"],
                 "layer1.weight_neigh": g["Wn1"], "layer1.weight_self": g["Ws1"], "layer1.bias": g["b1"]})
    if case == "model_gat":
        w = {k.replace("_head", ".head").replace("_weight", ".weight").replace("_attn", ".attn")
             .replace("_bias", ".bias"): a for k, a in g.items() if k.startswith("layer")}
        return ([dict(type="gat", **{"in": 48, "out": 8}, heads=4, concat=True, post="elu"),
                 dict(type="gat", **{"in": 32, "out": 6}, heads=1, concat=True)], w)
    raise KeyError(case)


GOLDEN_CASES = None


def pytest_generate_tests(metafunc):
    if "golden_case" in metafunc.fixturenames:
        from tests.helpers import load_golden
        metafunc.parametrize("golden_case", load_golden().cases)


def test_port_matches_reference_outputs(golden, golden_case):
    g = golden[golden_case]
    got = _port_output(golden_case, g)
    if isinstance(got, tuple):
        keys = ("out_rp", "out_ci", "out_v")
        for k, a in zip(keys, got):
            assert_bits_equal(a, g[k], f"{golden_case}.{k}")
    else:
        assert_bits_equal(got, g["out"], golden_case)


# ── known answers from the reference's own unit tests ───────────────────────
def _ka_run(impl, c):
    op = c["op"]
    if op == "spmm":
        return impl.spmm(c["rp"], c["ci"], c["v"], np.array(c["B"], np.float32)), c["expect"]
    if op == "matmul":
        return impl.matmul(np.array(c["A"], np.float32), np.array(c["B"], np.float32)), c["expect"]
    if op in ("gcn_norm", "add_self_loops"):
        rp, ci, v = getattr(impl, op)(np.array(c["rp"]), np.array(c["ci"]), np.array(c["v"]))
        assert list(rp) == c["expect_rp"] and list(ci) == c["expect_ci"], c["src"]
        return v, c["expect_v"]
    if op == "edge_softmax":
        return impl.edge_softmax(np.array(c["rp"]), np.array(c["ci"]), np.array(c["v"])), c["expect_v"]
    if op == "edge_list_to_csr":
        e = np.array(c["edges"], np.int32).reshape(-1, 2)
        rp, ci, v = impl.edge_list_to_csr(e[:, 0], e[:, 1], c["n"])
        assert list(rp) == c["expect_rp"] and list(ci) == c["expect_ci"], c["src"]
        return v, [1.0] * len(c["expect_ci"])
    if op == "activation":
        return impl.activation(c["kind"], np.array(c["X"], np.float32), c.get("alpha", 0.0)), c["expect"]
    n, pairs = c["graph"]
    rp, ci, v = undirected_csr(n, [tuple(p) for p in pairs])
    H = np.array(c["H"], np.float32)
    b = None if c.get("bias") is None else np.array(c["bias"], np.float32)
    relu = c.get("act") == "relu"
    if op == "gcn_layer":
        A = impl.gcn_norm(rp, ci, v)
        return impl.gcn_layer(*A, H, np.array(c["W"], np.float32), b, relu), c["expect"]
    if op == "sage_layer":
        return impl.sage_layer(rp, ci, v, H, np.array(c["Wn"], np.float32), np.array(c["Ws"], np.float32), b,
                               c["agg"], relu), c["expect"]
    if op == "gat_layer":
        A = impl.add_self_loops(rp, ci, v)
        return impl.gat_layer(*A, H, np.array(c["W"], np.float32), np.array(c["a_l"], np.float32),
                              np.array(c["a_r"], np.float32), b, 0.2, relu), c["expect"]
    raise KeyError(op)


def test_port_known_answers(known_answers):
    for c in known_answers:
        got, expect = _ka_run(P, c)
        tol = c.get("tol", 0.0)
        np.testing.assert_allclose(np.asarray(got, np.float64), np.asarray(expect, np.float64), rtol=0,
                                   atol=max(tol, 1e-7), err_msg=c["src"])


@needs_ref
def test_reference_known_answers(known_answers):
    """The compiled reference itself passes its own known answers (sanity of the build)."""
    for c in known_answers:
        got, expect = _ka_run(oracle.ref, c)
        np.testing.assert_allclose(np.asarray(got, np.float64), np.asarray(expect, np.float64), rtol=0,
                                   atol=max(c.get("tol", 0.0), 1e-7), err_msg=c["src"])


# ── live comparison with the reference on fresh inputs ──────────────────────
@needs_ref
@pytest.mark.parametrize("seed", [1, 2, 3])
def test_port_vs_reference_live(seed):
    R = oracle.ref
    rng = np.random.default_rng(1000 + seed)
    n = 600
    rp, ci, v = powerlaw_csr(rng, n, 12)
    for F in (3, 8, 13, 41, 96):
        B = rng.standard_normal((n, F)).astype(np.float32)
        assert_bits_equal(P.spmm(rp, ci, v, B), R.spmm(rp, ci, v, B), f"spmm F={F}")
    for tag, (a, b) in {"asl": (P.add_self_loops, R.add_self_loops), "norm": (P.gcn_norm, R.gcn_norm)}.items():
        for x, y in zip(a(rp, ci, v), b(rp, ci, v)):
            assert_bits_equal(x, y, tag)
    src = rng.integers(0, 500, 20000).astype(np.int32)
    dst = rng.integers(0, 500, 20000).astype(np.int32)
    for x, y in zip(P.edge_list_to_csr(src, dst, 500), R.edge_list_to_csr(src, dst, 500)):
        assert_bits_equal(x, y, "edge_list_to_csr")
    H = rng.standard_normal((n, 24)).astype(np.float32)
    for Fo in (4, 12, 16, 33):
        W = (rng.standard_normal((24, Fo)) * 0.3).astype(np.float32)
        W2 = (rng.standard_normal((24, Fo)) * 0.3).astype(np.float32)
        bias = rng.standard_normal(Fo).astype(np.float32)
        al, ar = rng.standard_normal(Fo).astype(np.float32), rng.standard_normal(Fo).astype(np.float32)
        for agg in ("mean", "max"):
            assert_bits_equal(P.sage_layer(rp, ci, v, H, W, W2, bias, agg),
                              R.sage_layer(rp, ci, v, H, W, W2, bias, agg), f"sage {agg} {Fo}")
        sl = R.add_self_loops(rp, ci, v)
        assert_bits_equal(P.gat_layer(*sl, H, W, al, ar, bias), R.gat_layer(*sl, H, W, al, ar, bias), f"gat {Fo}")


@needs_ref
def test_model_forward_composition_matches_reference_model():
    """oracle.model_forward over the reference's layers == the reference's Model::forward."""
    R = oracle.ref
    rng = np.random.default_rng(7)
    rp, ci, v = rand_csr(rng, 200, 200, 6, weighted=False, diag=False)
    X = rng.standard_normal((200, 20)).astype(np.float32)
    w = {}
    for h in range(3):
        w[f"layer0.head{h}.weight"] = (rng.standard_normal((20, 8)) * 0.3).astype(np.float32)
        w[f"layer0.head{h}.attn_left"] = rng.standard_normal(8).astype(np.float32)
        w[f"layer0.head{h}.attn_right"] = rng.standard_normal(8).astype(np.float32)
        w[f"layer0.head{h}.bias"] = rng.standard_normal(8).astype(np.float32)
    w["layer1.weight"] = (rng.standard_normal((8, 5)) * 0.3).astype(np.float32)
    w["layer1.bias"] = rng.standard_normal(5).astype(np.float32)
    w["layer2.weight_neigh"] = (rng.standard_normal((5, 4)) * 0.3).astype(np.float32)
    w["layer2.weight_self"] = (rng.standard_normal((5, 4)) * 0.3).astype(np.float32)
    w["layer2.bias"] = rng.standard_normal(4).astype(np.float32)
    spec = [dict(type="gat", **{"in": 20, "out": 8}, heads=3, concat=False, post="elu"),
            dict(type="gcn", **{"in": 8, "out": 5}, act="relu", post="relu"),
            dict(type="sage", **{"in": 5, "out": 4}, act=None)]
    ours = oracle.model_forward(P, spec, w, rp, ci, v, X)
    theirs = R.model(spec, w).forward(rp, ci, v, X)
    assert_bits_equal(ours, theirs, "model")


# ── edge cases the reference tests cover ────────────────────────────────────
def test_port_edge_cases():
    # empty graph / rows / features
    rp = np.zeros(4, np.int32)
    ci = np.zeros(0, np.int32)
    v = np.zeros(0, np.float32)
    assert P.spmm(rp, ci, v, np.ones((3, 5), np.float32)).sum() == 0
    a = P.gcn_norm(rp, ci, v)
    assert list(a[0]) == [0, 1, 2, 3] and np.all(a[2] == 1.0)
    rp0, ci0, v0 = P.edge_list_to_csr(np.zeros(0, np.int32), np.zeros(0, np.int32), 3)
    assert list(rp0) == [0, 0, 0, 0]
    with pytest.raises(oracle.OracleError):
        P.edge_list_to_csr(np.array([0], np.int32), np.array([3], np.int32), 3)
    with pytest.raises(oracle.OracleError):
        P.activation("softmax", np.zeros((2, 0), np.float32))


@pytest.mark.skipif(oracle.ref is None, reason="the reference library is not built")
@pytest.mark.parametrize("kind", ["gcn", "sage"])
def test_reference_layer_stack_equals_model_forward(kind):
    """The reference's layer objects run on an adjacency normalised once (the
    CPU baseline's layers-only figure) give Model::forward's logits bit for
    bit."""
    rng = np.random.default_rng(17)
    n = 1500
    rp, ci, v = powerlaw_csr(rng, n, 9, weighted=False, diag=False)
    X = rng.standard_normal((n, 24)).astype(np.float32)
    if kind == "gcn":
        spec = [dict(type="gcn", **{"in": 24, "out": 16}, act="relu"), dict(type="gcn", **{"in": 16, "out": 5})]
        w = {"layer0.weight": rng.standard_normal((24, 16)).astype(np.float32) * 0.3,
             "layer0.bias": rng.standard_normal(16).astype(np.float32) * 0.1,
             "layer1.weight": rng.standard_normal((16, 5)).astype(np.float32) * 0.3,
             "layer1.bias": rng.standard_normal(5).astype(np.float32) * 0.1}
    else:
        spec = [dict(type="sage", **{"in": 24, "out": 16}, act="relu"), dict(type="sage", **{"in": 16, "out": 5})]
        w = {f"layer{i}.{k}": rng.standard_normal(s).astype(np.float32) * 0.3
             for i, (a, b) in enumerate([(24, 16), (16, 5)])
             for k, s in (("weight_neigh", (a, b)), ("weight_self", (a, b)), ("bias", (b,)))}
    R = oracle.ref
    ref = R.activation("log_softmax", R.model(spec, w).forward(rp, ci, v, X))
    st = R.stack(spec, w)
    A = R.lib.ref_tensor_csr(n, ci.size, rp.ctypes.data, ci.ctypes.data, v.ctypes.data)
    Xt = R.lib.ref_tensor_dense(n, 24, X.ctypes.data)
    An = st.gcn_norm_tensor(A)
    try:
        got = st.forward_tensors(An, A, Xt, True, rows=n)
    finally:
        for t in (A, Xt, An):
            R.lib.ref_tensor_free(t)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
