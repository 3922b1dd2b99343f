"""GPU parity of the layer forwards and whole-model compositions vs the oracle."""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import assert_bits_equal, assert_close, assert_sage_fast_close, powerlaw_csr, rand_csr

pytestmark = pytest.mark.gpu
P = oracle.port


@pytest.fixture(scope="module")
def tg():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import tinygnn_b200
    return tinygnn_b200


def dev(a):
    return torch.as_tensor(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def glorot(rng, i, o):
    r = np.sqrt(6.0 / (i + o))
    return rng.uniform(-r, r, (i, o)).astype(np.float32)


@pytest.mark.parametrize("fi,fo", [(1433, 16), (16, 7), (602, 128), (128, 41), (64, 64)])
def test_gcn_layer_exact(tg, fi, fo):
    rng = np.random.default_rng(fi * 7 + fo)
    n = 2500
    rp, ci, v = powerlaw_csr(rng, n, 15, weighted=False, diag=False)
    A = P.gcn_norm(rp, ci, v)
    H = rng.standard_normal((n, fi)).astype(np.float32)
    W = glorot(rng, fi, fo)
    b = (rng.standard_normal(fo) * 0.1).astype(np.float32)
    ref = P.gcn_layer(*A, H, W, b, True)
    Ad = tg.CSR.from_numpy(*A)
    assert_bits_equal(host(tg.gcn_layer(Ad, dev(H), dev(W), dev(b), "relu")), ref, f"gcn {fi}->{fo}")
    assert_bits_equal(host(tg.gcn_layer(Ad, dev(H), dev(W), dev(b), "relu", row_order=tg.degree_order(Ad))), ref,
                      "gcn ordered")


@pytest.mark.parametrize("agg", ["mean", "max"])
@pytest.mark.parametrize("fi,fo", [(128, 128), (128, 40), (602, 128), (128, 41), (12, 5)])
def test_sage_layer(tg, agg, fi, fo):
    rng = np.random.default_rng(fi + fo)
    n = 2000
    rp, ci, v = powerlaw_csr(rng, n, 12, weighted=False, diag=False)
    H = rng.standard_normal((n, fi)).astype(np.float32)
    Wn, Ws = glorot(rng, fi, fo), glorot(rng, fi, fo)
    b = (rng.standard_normal(fo) * 0.1).astype(np.float32)
    ref = P.sage_layer(rp, ci, v, H, Wn, Ws, b, agg, True)
    A = tg.CSR.from_numpy(rp, ci, v)
    exact = host(tg.sage_layer(A, dev(H), dev(Wn), dev(Ws), dev(b), agg, "relu", mode="exact"))
    assert_bits_equal(exact, ref, f"sage {agg} exact")
    fast = host(tg.sage_layer(A, dev(H), dev(Wn), dev(Ws), dev(b), agg, "relu", mode="fast"))
    assert_sage_fast_close(fast, ref, rp, ci, H, Wn, Ws, f"sage {agg} fast")


@pytest.mark.parametrize("heads,d,fi,concat", [(8, 8, 256, True), (1, 16, 64, True), (4, 6, 20, True),
                                                (3, 5, 17, False), (2, 41, 30, True), (1, 7, 9, True)])
def test_gat_multihead_vs_oracle(tg, heads, d, fi, concat):
    rng = np.random.default_rng(heads * 100 + d)
    n = 3000
    rp, ci, v = powerlaw_csr(rng, n, 10, weighted=False, diag=False)
    A_sl = P.add_self_loops(rp, ci, v)
    H = rng.standard_normal((n, fi)).astype(np.float32)
    Ws = [glorot(rng, fi, d) for _ in range(heads)]
    al = [(rng.standard_normal(d) * 0.5).astype(np.float32) for _ in range(heads)]
    ar = [(rng.standard_normal(d) * 0.5).astype(np.float32) for _ in range(heads)]
    bs = [(rng.standard_normal(d) * 0.1).astype(np.float32) for _ in range(heads)]
    outs = [P.gat_layer(*A_sl, H, Ws[h], al[h], ar[h], bs[h], 0.2, False) for h in range(heads)]
    if concat:
        ref = np.concatenate(outs, axis=1)
    else:
        acc = np.zeros_like(outs[0])
        for o in outs:
            acc = (acc + o).astype(np.float32)
        ref = (acc * np.float32(1.0 / heads)).astype(np.float32)
    got = tg.gat_layer(tg.CSR.from_numpy(*A_sl), dev(H), dev(np.concatenate(Ws, axis=1)), dev(np.stack(al)),
                       dev(np.stack(ar)), heads, dev(np.stack(bs)), 0.2, concat)
    assert_close(host(got), ref, f"gat h={heads} d={d}")


def test_gat_isolated_rows_get_bias(tg):
    # Rows without entries (no self-loops added) give bias then activation.
    rp = np.array([0, 2, 2, 3], np.int32)
    ci = np.array([0, 2, 1], np.int32)
    H = np.arange(6, dtype=np.float32).reshape(3, 2)
    W = np.eye(2, dtype=np.float32)
    al = np.array([0.3, -0.2], np.float32)
    ar = np.array([0.1, 0.4], np.float32)
    b = np.array([0.5, -0.5], np.float32)
    ref = P.gat_layer(rp, ci, None, H, W, al, ar, b, 0.2, False)
    got = host(tg.gat_layer(tg.CSR.from_numpy(rp, ci), dev(H), dev(W), dev(al), dev(ar), 1, dev(b)))
    assert_close(got, ref, "gat isolated")
    assert np.allclose(got[1], b)


def _model_weights(rng, spec):
    w = {}
    for li, L in enumerate(spec):
        p = f"layer{li}"
        if L["type"] == "gcn":
            w[f"{p}.weight"] = glorot(rng, L["in"], L["out"])
            w[f"{p}.bias"] = (rng.standard_normal(L["out"]) * 0.1).astype(np.float32)
        elif L["type"] == "sage":
            w[f"{p}.weight_neigh"] = glorot(rng, L["in"], L["out"])
            w[f"{p}.weight_self"] = glorot(rng, L["in"], L["out"])
            w[f"{p}.bias"] = (rng.standard_normal(L["out"]) * 0.1).astype(np.float32)
        else:
            for h in range(L.get("heads", 1)):
                w[f"{p}.head{h}.weight"] = glorot(rng, L["in"], L["out"])
                w[f"{p}.head{h}.attn_left"] = (rng.standard_normal(L["out"]) * 0.5).astype(np.float32)
                w[f"{p}.head{h}.attn_right"] = (rng.standard_normal(L["out"]) * 0.5).astype(np.float32)
                w[f"{p}.head{h}.bias"] = (rng.standard_normal(L["out"]) * 0.1).astype(np.float32)
    return w


def _gpu_model_forward(tg, spec, w, rp, ci, v, X):
    """The composition Model::forward performs, on the device entry points."""
    A = tg.CSR.from_numpy(rp, ci, v)
    A_gcn = tg.gcn_norm(A) if any(L["type"] == "gcn" for L in spec) else None
    A_sl = tg.add_self_loops(A) if any(L["type"] == "gat" for L in spec) else None
    H = dev(X)
    for li, L in enumerate(spec):
        p = f"layer{li}"
        act = L.get("act")
        if L["type"] == "gcn":
            H = tg.gcn_layer(A_gcn, H, dev(w[f"{p}.weight"]), dev(w[f"{p}.bias"]), act)
        elif L["type"] == "sage":
            H = tg.sage_layer(A, H, dev(w[f"{p}.weight_neigh"]), dev(w[f"{p}.weight_self"]), dev(w[f"{p}.bias"]),
                              L.get("agg", "mean"), act)
        else:
            hs = range(L.get("heads", 1))
            H = tg.gat_layer(A_sl, H, dev(np.concatenate([w[f"{p}.head{h}.weight"] for h in hs], 1)),
                             dev(np.stack([w[f"{p}.head{h}.attn_left"] for h in hs])),
                             dev(np.stack([w[f"{p}.head{h}.attn_right"] for h in hs])), len(hs),
                             dev(np.stack([w[f"{p}.head{h}.bias"] for h in hs])), 0.2, L.get("concat", True), act)
        if L.get("post") == "elu":
            tg.elu_(H)
        elif L.get("post") == "relu":
            tg.relu_(H)
    return tg.log_softmax_(H)


@pytest.mark.parametrize("name", ["gcn", "sage", "gat"])
def test_model_compositions(tg, name):
    rng = np.random.default_rng(len(name))
    n = 4000
    rp, ci, v = powerlaw_csr(rng, n, 10, weighted=False, diag=False)
    if name == "gcn":
        spec = [dict(type="gcn", **{"in": 300, "out": 16}, act="relu"), dict(type="gcn", **{"in": 16, "out": 7})]
        fi = 300
    elif name == "sage":
        spec = [dict(type="sage", **{"in": 128, "out": 128}, act="relu"), dict(type="sage", **{"in": 128, "out": 40})]
        fi = 128
    else:
        spec = [dict(type="gat", **{"in": 64, "out": 8}, heads=8, concat=True, post="elu"),
                dict(type="gat", **{"in": 64, "out": 16}, heads=1)]
        fi = 64
    X = rng.standard_normal((n, fi)).astype(np.float32)
    w = _model_weights(rng, spec)
    ref = P.activation("log_softmax", oracle.model_forward(P, spec, w, rp, ci, v, X))
    got = host(_gpu_model_forward(tg, spec, w, rp, ci, v, X))
    assert_close(got, ref, f"model {name}")
