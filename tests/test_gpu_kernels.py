"""GPU parity of the kernels, through the C ABI (ctypes -> libtinygnn_b200.so).

Bar: bit-identical to the reference for CSR construction, self-loops,
gcn_norm, spmm, matmul, SAGE aggregation and the exact layers; within
|d| <= 1e-5 + 1e-4 |ref| where expf/logf/tanhf enter (their last bits differ
between CUDA and glibc).
"""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import (assert_bits_equal, assert_close, load_golden, powerlaw_csr, rand_csr,
                           undirected_csr)

pytestmark = pytest.mark.gpu
P = oracle.port


@pytest.fixture(scope="module")
def tg():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import tinygnn_b200
    return tinygnn_b200


def dev(a, dtype=None):
    t = torch.as_tensor(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def csr(tg, rp, ci, v=None, n_cols=None):
    return tg.CSR.from_numpy(rp, ci, v, n_cols=n_cols)


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


# ── golden_ref.npz (outputs of the reference library) ───────────────────────
EXACT_ACTS = {"relu", "leaky_relu"}


def test_golden_reference_outputs(tg):
    G = load_golden()
    checked = 0
    for case in G.cases:
        g = G[case]
        if case.startswith("spmm_"):
            A = csr(tg, g["rp"], g["ci"], g["v"], n_cols=g["B"].shape[0])
            assert_bits_equal(host(tg.spmm(A, dev(g["B"]))), g["out"], case)
        elif case.startswith("matmul_"):
            assert_bits_equal(host(tg.matmul(dev(g["A"]), dev(g["B"]))), g["out"], case)
        elif case.startswith("asl_") or case.startswith("gcnnorm_"):
            fn = tg.add_self_loops if case.startswith("asl_") else tg.gcn_norm
            r = fn(csr(tg, g["rp"], g["ci"], g["v"]))
            for k, t in zip(("out_rp", "out_ci", "out_v"), (r.row_ptr, r.col_ind, r.values)):
                assert_bits_equal(host(t), g[k], f"{case}.{k}")
        elif case == "el2csr":
            r = tg.edge_list_to_csr(dev(g["src"]), dev(g["dst"]), int(g["n"]))
            for k, t in zip(("out_rp", "out_ci", "out_v"), (r.row_ptr, r.col_ind, r.values)):
                assert_bits_equal(host(t), g[k], f"{case}.{k}")
        elif case == "edge_softmax":
            r = tg.edge_softmax(csr(tg, g["rp"], g["ci"], g["v"]))
            assert_close(host(r.values), g["out"], case)
        elif case.startswith("sagemax_"):
            assert_bits_equal(host(tg.sage_max_aggregate(csr(tg, g["rp"], g["ci"], g["v"]), dev(g["H"]))),
                              g["out"], case)
        elif case.startswith("act_"):
            kind = case[4:]
            X = dev(g["X"])
            if kind == "softmax":
                tg.softmax_(X)
            elif kind == "log_softmax":
                tg.log_softmax_(X)
            else:
                from tinygnn_b200.ops import activation_
                activation_(X, kind, float(g["alpha"]))
            (assert_bits_equal if kind in EXACT_ACTS else assert_close)(host(X), g["out"], case)
        elif case == "add_bias":
            X = dev(g["X"])
            tg.add_bias_(X, dev(g["b"]))
            assert_bits_equal(host(X), g["out"], case)
        elif case.startswith("gcn_"):
            out = tg.gcn_layer(csr(tg, g["rp"], g["ci"], g["v"]), dev(g["H"]), dev(g["W"]), dev(g["b"]), "relu")
            assert_bits_equal(host(out), g["out"], case)
        elif case.startswith("sage_"):
            agg = case.split("_")[1]
            A = csr(tg, g["rp"], g["ci"])
            out = tg.sage_layer(A, dev(g["H"]), dev(g["Wn"]), dev(g["Ws"]), dev(g["b"]), agg, "relu")
            assert_bits_equal(host(out), g["out"], case + " exact")
            fast = tg.sage_layer(A, dev(g["H"]), dev(g["Wn"]), dev(g["Ws"]), dev(g["b"]), agg, "relu", mode="fast")
            assert_close(host(fast), g["out"], case + " fast")
        elif case.startswith("gat_"):
            A = csr(tg, g["rp"], g["ci"])
            out = tg.gat_layer(A, dev(g["H"]), dev(g["W"]), dev(g["al"]), dev(g["ar"]), 1, dev(g["b"]))
            assert_close(host(out), g["out"], case)
        else:
            continue
        checked += 1
    assert checked >= 40


def test_golden_known_answers(tg, known_answers):
    for c in known_answers:
        op = c["op"]
        tol = max(c.get("tol", 0.0), 1e-6)
        if op == "spmm":
            got = host(tg.spmm(csr(tg, c["rp"], c["ci"], c["v"], n_cols=c["n_cols"]), dev(np.array(c["B"], np.float32))))
            expect = c["expect"]
        elif op == "matmul":
            got = host(tg.matmul(dev(np.array(c["A"], np.float32)), dev(np.array(c["B"], np.float32))))
            expect = c["expect"]
        elif op in ("gcn_norm", "add_self_loops"):
            r = getattr(tg, op)(csr(tg, c["rp"], c["ci"], c["v"]))
            assert list(host(r.row_ptr)) == c["expect_rp"] and list(host(r.col_ind)) == c["expect_ci"], c["src"]
            got, expect = host(r.values), c["expect_v"]
        elif op == "edge_softmax":
            got, expect = host(tg.edge_softmax(csr(tg, c["rp"], c["ci"], c["v"])).values), c["expect_v"]
        elif op == "edge_list_to_csr":
            e = np.array(c["edges"], np.int32).reshape(-1, 2)
            r = tg.edge_list_to_csr(dev(e[:, 0].copy()), dev(e[:, 1].copy()), c["n"])
            assert list(host(r.row_ptr)) == c["expect_rp"] and list(host(r.col_ind)) == c["expect_ci"], c["src"]
            continue
        elif op == "activation":
            from tinygnn_b200.ops import activation_
            X = dev(np.array(c["X"], np.float32))
            activation_(X, c["kind"], c.get("alpha", 0.0))
            got, expect = host(X), c["expect"]
        else:
            n, pairs = c["graph"]
            rp, ci, v = undirected_csr(n, [tuple(p) for p in pairs])
            A = csr(tg, rp, ci, v)
            H = dev(np.array(c["H"], np.float32))
            b = None if c.get("bias") is None else dev(np.array(c["bias"], np.float32))
            act = c.get("act")
            if op == "gcn_layer":
                got = host(tg.gcn_layer(tg.gcn_norm(A), H, dev(np.array(c["W"], np.float32)), b, act))
            elif op == "sage_layer":
                got = host(tg.sage_layer(A, H, dev(np.array(c["Wn"], np.float32)), dev(np.array(c["Ws"], np.float32)),
                                         b, c["agg"], act))
            else:
                got = host(tg.gat_layer(tg.add_self_loops(A), H, dev(np.array(c["W"], np.float32)),
                                        dev(np.array(c["a_l"], np.float32)), dev(np.array(c["a_r"], np.float32)), 1, b,
                                        act=act))
            expect = c["expect"]
        np.testing.assert_allclose(np.asarray(got, np.float64), np.asarray(expect, np.float64), rtol=0, atol=tol,
                                   err_msg=c["src"])


# ── spmm against the oracle on seeded inputs ────────────────────────────────
@pytest.mark.parametrize("F", [1, 2, 3, 7, 8, 16, 33, 41, 64, 100, 128, 256, 300, 602])
def test_spmm_exact_vs_oracle(tg, F):
    rng = np.random.default_rng(F)
    n = 3000
    rp, ci, v = powerlaw_csr(rng, n, 20)
    B = rng.standard_normal((n, F)).astype(np.float32)
    A = csr(tg, rp, ci, v)
    ref = P.spmm(rp, ci, v, B)
    assert_bits_equal(host(tg.spmm(A, dev(B))), ref, f"spmm F={F}")
    order = tg.degree_order(A)
    assert_bits_equal(host(tg.spmm(A, dev(B), row_order=order)), ref, f"spmm F={F} degree order")


@pytest.mark.parametrize("F", [16, 41, 128])
def test_spmm_large_auto_schedule_vs_oracle(tg, F):
    """Above 16,384 rows the library schedules longest rows first by itself."""
    rng = np.random.default_rng(100 + F)
    n = 40000
    rp, ci, v = powerlaw_csr(rng, n, 24)
    B = rng.standard_normal((n, F)).astype(np.float32)
    A = csr(tg, rp, ci, v)
    assert A.order is None
    assert_bits_equal(host(tg.spmm(A, dev(B))), P.spmm(rp, ci, v, B), f"spmm auto-ordered F={F}")
    H = rng.standard_normal((n, 12)).astype(np.float32)
    W = (rng.standard_normal((12, F)) * 0.3).astype(np.float32)
    An = P.gcn_norm(rp, ci, v)
    assert_bits_equal(host(tg.gcn_layer(csr(tg, *An), dev(H), dev(W), None, "relu")),
                      P.gcn_layer(*An, H, W, None, True), f"gcn auto-ordered F={F}")


@pytest.mark.parametrize("nblocks", [1, 2, 3, 8])
def test_column_block_passes_equal_one_pass(tg, nblocks):
    """Passes over column blocks in order reproduce spmm / the SAGE combine bit for bit."""
    rng = np.random.default_rng(nblocks)
    n, F = 20000, 41
    rp, ci, v = powerlaw_csr(rng, n, 16)
    A = csr(tg, rp, ci, v)
    B = torch.zeros((n, 44), device="cuda")
    B[:, :F] = dev(rng.standard_normal((n, F)).astype(np.float32))
    b = dev(rng.standard_normal(F).astype(np.float32))
    width = (n + nblocks - 1) // nblocks
    sp = tg.ops.column_splits(A, nblocks, width)
    h_sp = host(sp)
    assert np.array_equal(h_sp[0], rp[:-1]) and np.array_equal(h_sp[-1], rp[1:])
    ref = host(tg.spmm(A, B[:, :F], bias=b, act="relu"))
    out = torch.empty((n, F), device="cuda")
    for q in range(nblocks):
        tg.ops.spmm_segment(A, B[:, :F], sp[q], sp[q + 1], out, q > 0, q == nblocks - 1, bias=b, act="relu")
    assert_bits_equal(host(out), ref, f"spmm in {nblocks} passes")
    Ts = dev(rng.standard_normal((n, F)).astype(np.float32))
    ref = host(tg.ops.sage_mean_combine(A, B[:, :F], Ts, bias=b, act="relu"))
    for q in range(nblocks):
        tg.ops.sage_mean_combine_segment(A, B[:, :F], Ts, sp[q], sp[q + 1], out, q > 0, q == nblocks - 1, bias=b,
                                         act="relu")
    assert_bits_equal(host(out), ref, f"sage combine in {nblocks} passes")


def test_spmm_epilogue_and_strides(tg):
    rng = np.random.default_rng(5)
    n, F = 1000, 41
    rp, ci, v = powerlaw_csr(rng, n, 10)
    B = rng.standard_normal((n, F)).astype(np.float32)
    b = rng.standard_normal(F).astype(np.float32)
    ref = P.activation("relu", P.add_bias(P.spmm(rp, ci, v, B), b))
    A = csr(tg, rp, ci, v)
    assert_bits_equal(host(tg.spmm(A, dev(B), bias=dev(b), act="relu")), ref, "bias+relu epilogue")
    # B and C as column slices of wider buffers (leading dimension > F)
    Bw = torch.zeros((n, 48), device="cuda")
    Bw[:, 3:3 + F] = dev(B)
    Cw = torch.full((n, 50), 7.0, device="cuda")
    tg.spmm(A, Bw[:, 3:3 + F], out=Cw[:, 5:5 + F])
    Cw_h = host(Cw)
    assert_bits_equal(Cw_h[:, 5:5 + F], P.spmm(rp, ci, v, B), "strided")
    assert np.all(Cw_h[:, :5] == 7.0) and np.all(Cw_h[:, 5 + F:] == 7.0), "wrote outside the output slice"


def test_spmm_empty_and_rectangular(tg):
    rp = np.zeros(6, np.int32)
    A = csr(tg, rp, np.zeros(0, np.int32), np.zeros(0, np.float32), n_cols=4)
    out = host(tg.spmm(A, dev(np.ones((4, 9), np.float32))))
    assert out.shape == (5, 9) and np.all(out == 0)
    rng = np.random.default_rng(3)
    rp, ci, v = rand_csr(rng, 70, 500, 30)
    B = rng.standard_normal((500, 24)).astype(np.float32)
    assert_bits_equal(host(tg.spmm(csr(tg, rp, ci, v, n_cols=500), dev(B))), P.spmm(rp, ci, v, B), "70x500")
    with pytest.raises(ValueError, match="spmm: dimension mismatch"):
        tg.spmm(csr(tg, rp, ci, v, n_cols=500), dev(np.ones((499, 3), np.float32)))


def test_degree_order_is_a_descending_bucket_permutation(tg):
    rng = np.random.default_rng(11)
    rp, ci, v = powerlaw_csr(rng, 20000, 8)
    order = host(tg.degree_order(csr(tg, rp, ci, v)))
    assert np.array_equal(np.sort(order), np.arange(20000))
    lens = (rp[1:] - rp[:-1])[order]
    # length classes: x = len + 1 in [2^k, 2^(k+1)), split in quarters
    x = (lens + 1).astype(np.int64)
    k = np.floor(np.log2(x)).astype(np.int64)
    quarter = ((x - (1 << k)) * 4) >> k
    buckets = 4 * k + quarter
    assert np.all(np.diff(buckets) <= 0)
    assert len(np.unique(buckets)) > len(np.unique(k))  # finer than powers of two
    for b in np.unique(buckets):  # stable: rows ascending inside a bucket
        assert np.all(np.diff(order[buckets == b]) > 0)


# ── matmul ───────────────────────────────────────────────────────────────────
@pytest.mark.parametrize("shape", [(1, 1, 1), (37, 1433, 16), (300, 602, 41), (513, 256, 64), (1000, 128, 128),
                                   (257, 64, 7), (129, 300, 8), (64, 20, 200), (10, 0, 5)])
def test_matmul_exact_vs_oracle(tg, shape):
    M, K, N = shape
    rng = np.random.default_rng(M + K + N)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    assert_bits_equal(host(tg.matmul(dev(A), dev(B))), P.matmul(A, B), f"matmul {shape}")


def test_matmul_epilogue(tg):
    rng = np.random.default_rng(1)
    A = rng.standard_normal((200, 50)).astype(np.float32)
    B = rng.standard_normal((50, 41)).astype(np.float32)
    b = rng.standard_normal(41).astype(np.float32)
    ref = P.activation("relu", P.add_bias(P.matmul(A, B), b))
    assert_bits_equal(host(tg.matmul(dev(A), dev(B), bias=dev(b), act="relu")), ref, "matmul+bias+relu")
    with pytest.raises(ValueError, match="matmul: dimension mismatch"):
        tg.matmul(dev(A), dev(B[:40]))


# ── graph construction ───────────────────────────────────────────────────────
@pytest.mark.parametrize("case", ["uniform", "hub", "giant_rows", "dups"])
def test_edge_list_to_csr_vs_oracle(tg, case):
    rng = np.random.default_rng(hash(case) % 1000)
    if case == "uniform":
        N, E = 5000, 200000
        src, dst = rng.integers(0, N, E), rng.integers(0, N, E)
    elif case == "hub":       # rows in every size class (warp, CTA)
        N, E = 3000, 300000
        src = np.minimum(rng.zipf(1.3, E) - 1, N - 1)
        dst = rng.integers(0, N, E)
    elif case == "giant_rows":  # rows above the shared-memory sort limit
        N, E = 70000, 160000
        src = np.concatenate([np.full(40000, 5), np.full(50000, 69999), rng.integers(0, N, 70000)])
        dst = rng.integers(0, N, E)
    else:                     # heavy duplication
        N, E = 100, 100000
        src, dst = rng.integers(0, N, E), rng.integers(0, 10, E)
    src, dst = src.astype(np.int32), dst.astype(np.int32)
    r = tg.edge_list_to_csr(dev(src), dev(dst), N)
    ref = P.edge_list_to_csr(src, dst, N)
    for k, t, a in zip(("row_ptr", "col_ind", "values"), (r.row_ptr, r.col_ind, r.values), ref):
        assert_bits_equal(host(t), a, f"{case}.{k}")


def test_edge_list_to_csr_errors(tg):
    src = dev(np.array([0, 1, 2], np.int32))
    with pytest.raises(ValueError, match=r"edge\[2\]\.dst = 7 out of range \[0, 3\)"):
        tg.edge_list_to_csr(src, dev(np.array([1, 2, 7], np.int32)), 3)
    with pytest.raises(ValueError, match=r"edge\[1\]\.src = -1 out of range"):
        tg.edge_list_to_csr(dev(np.array([0, -1], np.int32)), dev(np.array([0, 0], np.int32)), 3)
    with pytest.raises(ValueError, match="num_nodes is 0 but edges is non-empty"):
        tg.edge_list_to_csr(src, src, 0)
    r = tg.edge_list_to_csr(dev(np.zeros(0, np.int32)), dev(np.zeros(0, np.int32)), 0)
    assert host(r.row_ptr).tolist() == [0]


def _unsorted_dup_diag(rng, n=3000, deg=20):
    """Rows in random column order, some holding their diagonal twice, with
    integer and fractional values mixed per row."""
    lens = rng.integers(0, 2 * deg, n)
    rp = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    ci = rng.integers(0, n, rp[-1]).astype(np.int32)
    for i in rng.choice(n, n // 4, replace=False):  # one or two diagonal entries
        a, b = rp[i], rp[i + 1]
        if b > a:
            ci[rng.integers(a, b)] = i
            if b - a > 3 and rng.random() < 0.5:
                ci[rng.integers(a, b)] = i
    v = np.where(rng.random(ci.size) < 0.5, rng.integers(1, 4, ci.size), rng.random(ci.size) + 0.1)
    return rp, ci, v.astype(np.float32)


@pytest.mark.parametrize("kind", ["plain", "with_diag", "weighted_empty_rows", "powerlaw", "integral_weights",
                                  "large_integral", "unsorted_dup_diag", "negative_integral"])
def test_self_loops_and_gcn_norm_vs_oracle(tg, kind):
    """Both degree paths: rows of integer values within the exactness bound
    (summed as a tree) and every other row (the sequential chain)."""
    rng = np.random.default_rng(len(kind))
    if kind == "powerlaw":
        rp, ci, v = powerlaw_csr(rng, 20000, 30, weighted=False, diag=False)
    elif kind in ("integral_weights", "large_integral", "negative_integral"):
        rp, ci, v = powerlaw_csr(rng, 20000, 30, weighted=False, diag=True)
        hi = {"integral_weights": 5, "large_integral": 1 << 20, "negative_integral": 3}[kind]
        v = rng.integers(1, hi, ci.size).astype(np.float32)
        if kind == "negative_integral":
            v *= np.where(rng.random(ci.size) < 0.3, -1, 1).astype(np.float32)
    elif kind == "unsorted_dup_diag":
        rp, ci, v = _unsorted_dup_diag(rng)
    else:
        rp, ci, v = rand_csr(rng, 8000, 8000, 12, weighted=kind.startswith("weighted"),
                             diag=kind == "with_diag" or kind.startswith("weighted"),
                             empty_frac=0.2 if "empty" in kind else 0.0)
    A = csr(tg, rp, ci, v)
    for name in ("add_self_loops", "gcn_norm"):
        r = getattr(tg, name)(A)
        ref = getattr(P, name)(rp, ci, v)
        for k, t, a in zip(("row_ptr", "col_ind", "values"), (r.row_ptr, r.col_ind, r.values), ref):
            assert_bits_equal(host(t), a, f"{name}.{k}")


def test_csr_validate_messages(tg):
    rp = np.array([0, 2, 1, 3], np.int32)
    ci = np.array([0, 1, 2], np.int32)
    with pytest.raises(ValueError, match=r"row_ptr must be non-decreasing; row_ptr\[2\] = 1 < row_ptr\[1\] = 2"):
        tg.csr_validate(csr(tg, rp, ci))
    with pytest.raises(ValueError, match=r"col_ind\[1\] = 9 is out of bounds for cols=3"):
        tg.csr_validate(csr(tg, np.array([0, 1, 2, 3], np.int32), np.array([0, 9, 1], np.int32)))
    with pytest.raises(ValueError, match=r"row_ptr.back\(\) \(3\) must equal values.size\(\) \(2\)"):
        A = csr(tg, np.array([0, 1, 3], np.int32), np.array([0, 1], np.int32))
        tg.csr_validate(A)
    tg.csr_validate(csr(tg, np.array([0, 1, 3], np.int32), np.array([0, 1, 0], np.int32)))
    with pytest.raises(ValueError, match="must be square"):
        tg.gcn_norm(csr(tg, np.array([0, 1], np.int32), np.array([1], np.int32), n_cols=2))


# ── elementwise ──────────────────────────────────────────────────────────────
def test_activations_and_softmax_vs_oracle(tg):
    from tinygnn_b200.ops import activation_
    rng = np.random.default_rng(9)
    X = (rng.standard_normal((5000, 41)) * 5).astype(np.float32)
    for kind in ("relu", "leaky_relu", "elu", "sigmoid", "tanh", "gelu"):
        T = dev(X)
        activation_(T, kind, 0.3)
        ref = P.activation(kind, X, 0.3)
        (assert_bits_equal if kind in EXACT_ACTS else assert_close)(host(T), ref, kind)
    for kind, fn in (("softmax", tg.softmax_), ("log_softmax", tg.log_softmax_)):
        T = dev(X)
        fn(T)
        assert_close(host(T), P.activation(kind, X), kind)
    with pytest.raises(ValueError, match="0 columns"):
        tg.softmax_(torch.zeros((3, 0), device="cuda"))


@pytest.mark.parametrize("rows,cols,ld", [(1, 1, 1), (129, 7, 7), (1000, 41, 44), (300, 64, 64), (300, 65, 65),
                                          (257, 128, 130), (100, 129, 129), (70, 256, 256), (33, 257, 257),
                                          (5, 600, 602)])
def test_row_softmax_shapes(tg, rows, cols, ld):
    """Row softmax / log_softmax across the staged-tile sizes (128 / 64 / 32
    rows for up to 64 / 128 / 256 columns, partial last tiles, strided rows)
    and the wide-row kernel, against the oracle; padding columns untouched."""
    rng = np.random.default_rng(rows * 1000 + cols)
    X = (rng.standard_normal((rows, ld)) * 4).astype(np.float32)
    for kind, fn in (("softmax", tg.softmax_), ("log_softmax", tg.log_softmax_)):
        T = dev(X)
        fn(T[:, :cols])
        got = host(T)
        assert_close(got[:, :cols], P.activation(kind, X[:, :cols].copy()), f"{kind} {rows}x{cols}")
        assert_bits_equal(got[:, cols:], X[:, cols:], "padding columns")


def test_edge_softmax_vs_oracle(tg):
    rng = np.random.default_rng(4)
    rp, ci, v = powerlaw_csr(rng, 5000, 12)
    v = (v * 30 - 15).astype(np.float32)
    r = tg.edge_softmax(csr(tg, rp, ci, v))
    assert_close(host(r.values), P.edge_softmax(rp, ci, v), "edge_softmax")


def test_sage_max_aggregate_vs_oracle(tg):
    rng = np.random.default_rng(8)
    for F in (3, 8, 19, 64, 130):
        rp, ci, v = powerlaw_csr(rng, 4000, 9)
        H = rng.standard_normal((4000, F)).astype(np.float32)
        assert_bits_equal(host(tg.sage_max_aggregate(csr(tg, rp, ci, v), dev(H))),
                          P.sage_max_aggregate(rp, ci, v, H), f"sage_max F={F}")


def test_unweighted_csr_equals_explicit_ones(tg):
    """values=None (an unweighted CSR: no values array, every entry 1.0) gives the
    bits an explicit array of ones gives: spmm (hub rows included, any schedule),
    the FAST gcn_norm scale and aggregate, and the FAST GCN forward."""
    from tinygnn_b200.dist import Comm, Layer, ShardedModel
    rng = np.random.default_rng(7)
    n = 20000
    rp, ci, _ = powerlaw_csr(rng, n, 30, weighted=False, diag=False)
    assert int(np.diff(rp).max()) >= 1023, "the graph should have hub rows for the heavy-row kernel"
    ones = csr(tg, rp, ci, np.ones(ci.size, np.float32))
    bare = tg.CSR(n, n, ones.row_ptr, ones.col_ind, None)
    B = dev(rng.standard_normal((n, 64)).astype(np.float32))
    for order in (None, tg.degree_order(ones)):
        assert_bits_equal(host(tg.spmm(bare, B, row_order=order)), host(tg.spmm(ones, B, row_order=order)), "spmm")
    d1, d0 = tg.ops.gcn_norm_scale(ones), tg.ops.gcn_norm_scale(bare)
    assert_bits_equal(host(d0), host(d1), "gcn_norm_scale")
    Hs = dev(rng.standard_normal((n, 44)).astype(np.float32))[:, :41]
    g1 = tg.ops.gcn_aggregate(ones, Hs, Hs, d1, act="relu")
    g0 = tg.ops.gcn_aggregate(bare, Hs, Hs, d0, act="relu")
    assert_bits_equal(host(g0), host(g1), "gcn_aggregate")
    W1 = dev((rng.standard_normal((32, 16)) * 0.2).astype(np.float32))
    W2 = dev((rng.standard_normal((16, 7)) * 0.2).astype(np.float32))
    X = dev(rng.standard_normal((n, 32)).astype(np.float32))
    m = ShardedModel([Layer("gcn", W1, None, "relu"), Layer("gcn", W2, None, None)], n, Comm(1, 0), "cuda",
                     mode="fast")
    y1 = m.forward_model(tg.CSR(n, n, ones.row_ptr, ones.col_ind, ones.values), X).clone()
    y0 = m.forward_model(tg.CSR(n, n, ones.row_ptr, ones.col_ind, None), X).clone()
    assert_bits_equal(host(y0), host(y1), "FAST GCN forward")
