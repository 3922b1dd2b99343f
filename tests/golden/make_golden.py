"""Generate the golden fixtures in this folder (run in the build container).

Two files:

* ``known_answers.json`` -- the hand-computed cases of TinyGNN's own unit
  tests, restated as inputs, expected outputs and the test's tolerance, each
  citing the test it comes from (tests/test_*.cpp:line in TinyGNN).
* ``golden_ref.npz`` -- seeded small inputs and the outputs of the reference
  library itself (oracle/_ref/libtinygnn_ref.so, compiled from the TinyGNN
  sources by oracle/Makefile) on them.  The C restatement and the CUDA path
  are checked bit for bit against these where the path is exact.

Usage:  python tests/golden/make_golden.py   (needs oracle/_ref built)
"""
from __future__ import annotations

import json
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402


def undirected_csr(n, pairs):
    """make_undirected_csr of the reference tests: both directions, rows sorted."""
    src = [u for u, v in pairs] + [v for u, v in pairs]
    dst = [v for u, v in pairs] + [u for u, v in pairs]
    order = sorted(range(len(src)), key=lambda k: (src[k], dst[k]))
    rp = [0] * (n + 1)
    for k in order:
        rp[src[k] + 1] += 1
    for i in range(n):
        rp[i + 1] += rp[i]
    return rp, [dst[k] for k in order], [1.0] * len(order)


def known_answers():
    s6 = 1.0 / math.sqrt(6.0)
    e1, e2 = math.exp(1.0), math.exp(2.0)
    cases = []
    rp, ci, v = [0, 2, 3, 5], [0, 1, 1, 0, 2], [1, 1, 1, 1, 1]
    cases.append(dict(op="spmm", src="tests/test_spmm.cpp:198", rp=rp, ci=ci, v=v, n_cols=3,
                      B=[[1, 2], [3, 4], [5, 6]], expect=[[4, 6], [3, 4], [6, 8]], tol=1e-4))
    cases.append(dict(op="spmm", src="tests/test_spmm.cpp:288", rp=[0, 1, 3, 5, 7], ci=[0, 1, 2, 0, 3, 1, 2],
                      v=[2, 3, 1, 1, 2, 1, 1], n_cols=4, B=[[1, 0, 2], [0, 1, 0], [3, 0, 1], [0, 2, 0]],
                      expect=[[2, 0, 4], [3, 3, 1], [1, 4, 2], [3, 1, 1]], tol=1e-4))
    A = np.arange(1, 17, dtype=np.float32).reshape(4, 4)
    B = np.arange(17, 33, dtype=np.float32).reshape(4, 4)
    cases.append(dict(op="matmul", src="tests/test_matmul.cpp:160", A=A.tolist(), B=B.tolist(),
                      expect=[[250, 260, 270, 280], [618, 644, 670, 696], [986, 1028, 1070, 1112],
                              [1354, 1412, 1470, 1528]], tol=1e-4))
    rp, ci, v = undirected_csr(3, [(0, 1), (1, 2)])
    cases.append(dict(op="gcn_norm", src="tests/test_gcn.cpp:288", rp=rp, ci=ci, v=v,
                      expect_rp=[0, 2, 5, 7], expect_ci=[0, 1, 0, 1, 2, 1, 2],
                      expect_v=[0.5, s6, s6, 1 / 3, s6, s6, 0.5], tol=1e-5))
    rp, ci, v = undirected_csr(3, [(0, 1), (0, 2), (1, 2)])
    cases.append(dict(op="gcn_norm", src="tests/test_gcn.cpp:329", rp=rp, ci=ci, v=v,
                      expect_rp=[0, 3, 6, 9], expect_ci=[0, 1, 2] * 3, expect_v=[1 / 3] * 9, tol=1e-5))
    cases.append(dict(op="gcn_norm", src="tests/test_gcn.cpp:345", rp=[0, 0, 0], ci=[], v=[],
                      expect_rp=[0, 1, 2], expect_ci=[0, 1], expect_v=[1.0, 1.0], tol=1e-5))
    rp, ci, v = undirected_csr(3, [(0, 1), (1, 2)])
    cases.append(dict(op="add_self_loops", src="tests/test_gcn.cpp:158", rp=rp, ci=ci, v=v,
                      expect_rp=[0, 2, 5, 7], expect_ci=[0, 1, 0, 1, 2, 1, 2], expect_v=[1.0] * 7, tol=1e-6))
    cases.append(dict(op="gcn_layer", src="tests/test_gcn.cpp:514", graph=[3, [(0, 1), (1, 2)]],
                      H=[[1, 0], [0, 1], [1, 1]], W=[[1, 0.5], [0.5, 1]], bias=[0.1, -0.1], act="relu",
                      expect=[[0.804124, 0.558248], [1.287287, 1.049829], [1.054124, 1.058248]], tol=1e-4))
    cases.append(dict(op="sage_layer", src="tests/test_graphsage.cpp:362", graph=[3, [(0, 1), (1, 2)]],
                      H=[[1, 0], [0, 1], [1, 1]], Wn=[[1, 0.5], [0.5, 1]], Ws=[[0.5, 0], [0, 0.5]],
                      bias=[0.1, -0.1], agg="mean", act="relu",
                      expect=[[1.1, 0.9], [1.35, 1.4], [1.1, 1.4]], tol=1e-4))
    cases.append(dict(op="sage_layer", src="tests/test_graphsage.cpp:509", graph=[3, [(0, 1), (1, 2)]],
                      H=[[1, 0], [0, 1], [1, 1]], Wn=[[1, 0], [0, 1]], Ws=[[1, 0], [0, 1]], bias=None,
                      agg="max", act=None, expect=[[1, 1], [1, 2], [1, 2]], tol=1e-5))
    cases.append(dict(op="gat_layer", src="tests/test_gat.cpp:332", graph=[2, [(0, 1)]], self_loops=True,
                      H=[[1, 0], [0, 1]], W=[[1, 0], [0, 1]], a_l=[1, 0], a_r=[0, 1], bias=None, act=None,
                      expect=[[e1 / (e1 + e2), e2 / (e1 + e2)], [1 / (1 + e1), e1 / (1 + e1)]], tol=1e-5))
    cases.append(dict(op="gat_layer", src="tests/test_gat.cpp:370", graph=[3, [(0, 1), (1, 2)]], self_loops=True,
                      H=[[1, 2], [3, 4], [5, 6]], W=[[1, 0], [0, 1]], a_l=[0, 0], a_r=[0, 0], bias=None,
                      act=None, expect=[[2, 3], [3, 4], [4, 5]], tol=1e-5))
    rp, ci, v = undirected_csr(3, [(0, 1), (1, 2)])
    cases.append(dict(op="edge_softmax", src="tests/test_gat.cpp:133", rp=rp, ci=ci, v=v,
                      expect_v=[1.0, 0.5, 0.5, 1.0], tol=1e-6))
    em1 = math.exp(-1.0)
    cases.append(dict(op="edge_softmax", src="tests/test_gat.cpp:182", rp=[0, 2, 4], ci=[0, 1, 0, 1],
                      v=[1000, 1001, -500, -501], expect_v=[em1 / (em1 + 1), 1 / (em1 + 1), 1 / (1 + em1),
                                                            em1 / (1 + em1)], tol=1e-5))
    cases.append(dict(op="edge_softmax", src="tests/test_gat.cpp:205", rp=[0, 1, 1, 2], ci=[1, 0], v=[2.0, 3.0],
                      expect_v=[1.0, 1.0], tol=1e-6))
    cases.append(dict(op="edge_list_to_csr", src="tests/test_graph_loader.cpp:330", n=5,
                      edges=[[0, 1], [0, 2], [1, 0], [1, 3], [2, 0], [2, 3], [2, 4], [3, 1], [3, 2], [4, 2]],
                      expect_rp=[0, 2, 4, 7, 9, 10], expect_ci=[1, 2, 0, 3, 0, 3, 4, 1, 2, 2]))
    cases.append(dict(op="edge_list_to_csr", src="tests/test_graph_loader.cpp:377", n=4,
                      edges=[[0, 3], [0, 1], [0, 2]], expect_rp=[0, 3, 3, 3, 3], expect_ci=[1, 2, 3]))
    cases.append(dict(op="edge_list_to_csr", src="tests/test_graph_loader.cpp:393", n=3,
                      edges=[[0, 1], [0, 2]], expect_rp=[0, 2, 2, 2], expect_ci=[1, 2]))
    cases.append(dict(op="edge_list_to_csr", src="tests/test_graph_loader.cpp:409", n=2,
                      edges=[[0, 0], [0, 1], [1, 1]], expect_rp=[0, 2, 3], expect_ci=[0, 1, 1]))
    cases.append(dict(op="edge_list_to_csr", src="tests/test_graph_loader.cpp:427", n=3, edges=[],
                      expect_rp=[0, 0, 0, 0], expect_ci=[]))
    X = [[-3, -1, 0, 1, 3]]
    cases.append(dict(op="activation", kind="relu", src="tests/test_activations.cpp:139", X=X,
                      expect=[[0, 0, 0, 1, 3]], tol=0.0))
    cases.append(dict(op="activation", kind="leaky_relu", alpha=0.01, src="tests/test_activations.cpp:198",
                      X=[[-100, -1, 0, 1, 100]], expect=[[-1, -0.01, 0, 1, 100]], tol=1e-6))
    cases.append(dict(op="activation", kind="leaky_relu", alpha=0.2, src="tests/test_activations.cpp:212",
                      X=[[-5, -1, 0, 1, 5]], expect=[[-1, -0.2, 0, 1, 5]], tol=1e-6))
    return cases


def rand_csr(rng, n, m, deg, weighted=True, diag=True, empty_frac=0.0):
    e = n * deg
    s = rng.integers(0, n, e)
    d = rng.integers(0, m, e)
    if not diag:
        keep = s != d
        s, d = s[keep], d[keep]
    if empty_frac > 0:
        empty = rng.random(n) < empty_frac
        keep = ~empty[s]
        s, d = s[keep], d[keep]
    key = np.unique(s.astype(np.int64) * m + d)
    s, d = (key // m).astype(np.int32), (key % m).astype(np.int32)
    rp = np.zeros(n + 1, np.int64)
    np.add.at(rp, s + 1, 1)
    rp = np.cumsum(rp).astype(np.int32)
    v = (rng.random(d.size) + 0.05).astype(np.float32) if weighted else np.ones(d.size, np.float32)
    return rp, d, v


def ref_cases():
    R = oracle.ref
    assert R is not None, "oracle/_ref is not built: run `make -C oracle`"
    rng = np.random.default_rng(20260101)
    out = {}

    def put(name, **arrays):
        for k, a in arrays.items():
            out[f"{name}/{k}"] = np.asarray(a)

    f32 = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731
    for F in (1, 7, 16, 41, 64, 128):
        rp, ci, v = rand_csr(rng, 300, 250, 9, empty_frac=0.05)
        B = f32(250, F)
        put(f"spmm_F{F}", rp=rp, ci=ci, v=v, B=B, out=R.spmm(rp, ci, v, B))
    for (M, K, N) in ((37, 1433, 16), (50, 602, 41), (64, 64, 7), (33, 128, 128), (5, 3, 1)):
        A, B = f32(M, K), f32(K, N)
        put(f"matmul_{M}x{K}x{N}", A=A, B=B, out=R.matmul(A, B))
    for tag, kw in (("plain", dict(weighted=False, diag=False)), ("diag", dict(weighted=False, diag=True)),
                    ("weighted", dict(weighted=True, diag=True, empty_frac=0.1))):
        rp, ci, v = rand_csr(rng, 400, 400, 6, **kw)
        a = R.add_self_loops(rp, ci, v)
        g = R.gcn_norm(rp, ci, v)
        put(f"asl_{tag}", rp=rp, ci=ci, v=v, out_rp=a[0], out_ci=a[1], out_v=a[2])
        put(f"gcnnorm_{tag}", rp=rp, ci=ci, v=v, out_rp=g[0], out_ci=g[1], out_v=g[2])
    src = rng.integers(0, 350, 6000).astype(np.int32)
    dst = rng.integers(0, 350, 6000).astype(np.int32)
    e = R.edge_list_to_csr(src, dst, 350)
    put("el2csr", src=src, dst=dst, n=np.int64(350), out_rp=e[0], out_ci=e[1], out_v=e[2])
    rp, ci, v = rand_csr(rng, 300, 300, 7, empty_frac=0.05)
    v = (v * 20 - 10).astype(np.float32)
    put("edge_softmax", rp=rp, ci=ci, v=v, out=R.edge_softmax(rp, ci, v))
    for F in (5, 8, 19):
        rp, ci, v = rand_csr(rng, 300, 300, 5, empty_frac=0.05)
        H = f32(300, F)
        put(f"sagemax_F{F}", rp=rp, ci=ci, v=v, H=H, out=R.sage_max_aggregate(rp, ci, v, H))
    X = (f32(37, 41) * 4).astype(np.float32)
    for kind in oracle.ACT:
        put(f"act_{kind}", X=X, alpha=np.float32(0.3), out=R.activation(kind, X, 0.3))
    b = f32(41)
    put("add_bias", X=X, b=b, out=R.add_bias(X, b))
    for (Fi, Fo) in ((16, 8), (20, 41), (64, 40), (13, 7), (24, 13)):
        rp, ci, v = rand_csr(rng, 250, 250, 6, diag=False, empty_frac=0.05)
        H = f32(250, Fi)
        W, W2 = f32(Fi, Fo) * 0.3, f32(Fi, Fo) * 0.3
        bias = f32(Fo)
        al, ar = f32(Fo), f32(Fo)
        gn = R.gcn_norm(rp, ci, v)
        put(f"gcn_{Fi}x{Fo}", rp=gn[0], ci=gn[1], v=gn[2], H=H, W=W, b=bias,
            out=R.gcn_layer(gn[0], gn[1], gn[2], H, W, bias, True))
        for agg in ("mean", "max"):
            put(f"sage_{agg}_{Fi}x{Fo}", rp=rp, ci=ci, H=H, Wn=W, Ws=W2, b=bias,
                out=R.sage_layer(rp, ci, v, H, W, W2, bias, agg, True))
        sl = R.add_self_loops(rp, ci, v)
        put(f"gat_{Fi}x{Fo}", rp=sl[0], ci=sl[1], H=H, W=W, al=al, ar=ar, b=bias,
            out=R.gat_layer(sl[0], sl[1], sl[2], H, W, al, ar, bias, 0.2, False))
    # Whole-model forwards (Model::forward + caller log_softmax), small graphs.
    rp, ci, v = rand_csr(rng, 300, 300, 5, weighted=False, diag=False)
    X = f32(300, 48)
    W0, W1 = f32(48, 16) * 0.2, f32(16, 7) * 0.3
    b0, b1 = f32(16) * 0.1, f32(7) * 0.1
    spec = [dict(type="gcn", **{"in": 48, "out": 16}, act="relu"), dict(type="gcn", **{"in": 16, "out": 7}, act=None)]
    m = R.model(spec, {"layer0.weight": W0, "layer0.bias": b0, "layer1.weight": W1, "layer1.bias": b1})
    y = R.activation("log_softmax", m.forward(rp, ci, v, X))
    put("model_gcn", rp=rp, ci=ci, v=v, X=X, W0=W0, b0=b0, W1=W1, b1=b1, out=y)
    Wn0, Ws0, Wn1, Ws1 = f32(48, 32) * 0.2, f32(48, 32) * 0.2, f32(32, 10) * 0.2, f32(32, 10) * 0.2
    sb0, sb1 = f32(32) * 0.1, f32(10) * 0.1
    spec = [dict(type="sage", **{"in": 48, "out": 32}, act="relu"), dict(type="sage", **{"in": 32, "out": 10}, act=None)]
    m = R.model(spec, {"layer0.weight_neigh": Wn0, "layer0.weight_self": Ws0, "layer0.bias": sb0,
                       "layer1.weight_neigh": Wn1, "layer1.weight_self": Ws1, "layer1.bias": sb1})
    y = R.activation("log_softmax", m.forward(rp, ci, v, X))
    put("model_sage", rp=rp, ci=ci, v=v, X=X, Wn0=Wn0, Ws0=Ws0, b0=sb0, Wn1=Wn1, Ws1=Ws1, b1=sb1, out=y)
    heads, d1, d2 = 4, 8, 6
    w = {}
    for h in range(heads):
        w[f"layer0.head{h}.weight"] = f32(48, d1) * 0.2
        w[f"layer0.head{h}.attn_left"] = f32(d1) * 0.5
        w[f"layer0.head{h}.attn_right"] = f32(d1) * 0.5
        w[f"layer0.head{h}.bias"] = f32(d1) * 0.1
    w["layer1.head0.weight"] = f32(heads * d1, d2) * 0.2
    w["layer1.head0.attn_left"] = f32(d2) * 0.5
    w["layer1.head0.attn_right"] = f32(d2) * 0.5
    w["layer1.head0.bias"] = f32(d2) * 0.1
    spec = [dict(type="gat", **{"in": 48, "out": d1}, heads=heads, concat=True, post="elu"),
            dict(type="gat", **{"in": heads * d1, "out": d2}, heads=1, concat=True)]
    m = R.model(spec, w)
    y = R.activation("log_softmax", m.forward(rp, ci, v, X))
    put("model_gat", rp=rp, ci=ci, v=v, X=X, out=y, **{k.replace(".", "_"): a for k, a in w.items()})
    # Rows in stored (unsorted) column order, some holding their diagonal
    # twice, values integer or fractional: add_self_loops inserts before the
    # first column > i in stored order and adds 1 to every diagonal entry.
    rng2 = np.random.default_rng(20261202)
    n = 300
    lens = rng2.integers(0, 14, n)
    rp = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    ci = rng2.integers(0, n, rp[-1]).astype(np.int32)
    for i in rng2.choice(n, n // 3, replace=False):
        a, b = rp[i], rp[i + 1]
        if b > a:
            ci[rng2.integers(a, b)] = i
            if b - a > 3:
                ci[rng2.integers(a, b)] = i
    for tag, v in (("unsorted_int", rng2.integers(1, 4, ci.size)),
                   ("unsorted_frac", rng2.random(ci.size) + 0.1)):
        v = v.astype(np.float32)
        a = R.add_self_loops(rp, ci, v)
        g = R.gcn_norm(rp, ci, v)
        put(f"asl_{tag}", rp=rp, ci=ci, v=v, out_rp=a[0], out_ci=a[1], out_v=a[2])
        put(f"gcnnorm_{tag}", rp=rp, ci=ci, v=v, out_rp=g[0], out_ci=g[1], out_v=g[2])
    return out


def main():
    with open(os.path.join(HERE, "known_answers.json"), "w") as f:
        json.dump(known_answers(), f, indent=1)
    arrays = ref_cases()
    np.savez_compressed(os.path.join(HERE, "golden_ref.npz"), **arrays)
    size = os.path.getsize(os.path.join(HERE, "golden_ref.npz"))
    print(f"wrote {len(arrays)} arrays, {size / 1e6:.2f} MB")


if __name__ == "__main__":
    main()
