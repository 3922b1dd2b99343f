"""The handle C ABI (tg_tensor_* / tg_model_*): TinyGNN's Tensor and Model
driven through C with host buffers, checked against the oracle's
Model::forward + log_softmax -- bit for bit in EXACT mode, within the fp32
tolerance in FAST mode -- and malformed input refused with the reference's
message."""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import assert_bits_equal, assert_close, powerlaw_csr

pytestmark = pytest.mark.gpu
P = oracle.port


def _glorot(rng, i, o):
    r = np.sqrt(6.0 / (i + o))
    return rng.uniform(-r, r, (i, o)).astype(np.float32)


def _spec_weights(rng, kind, fin):
    if kind == "gcn":
        spec = [dict(type="gcn", **{"in": fin, "out": 24}, act="relu"), dict(type="gcn", **{"in": 24, "out": 7})]
        w = {"layer0.weight": _glorot(rng, fin, 24), "layer0.bias": rng.standard_normal(24).astype(np.float32) * .1,
             "layer1.weight": _glorot(rng, 24, 7), "layer1.bias": rng.standard_normal(7).astype(np.float32) * .1}
    elif kind == "sage":
        spec = [dict(type="sage", **{"in": fin, "out": 24}, act="relu"), dict(type="sage", **{"in": 24, "out": 7})]
        w = {"layer0.weight_neigh": _glorot(rng, fin, 24), "layer0.weight_self": _glorot(rng, fin, 24),
             "layer0.bias": rng.standard_normal(24).astype(np.float32) * .1,
             "layer1.weight_neigh": _glorot(rng, 24, 7), "layer1.weight_self": _glorot(rng, 24, 7),
             "layer1.bias": rng.standard_normal(7).astype(np.float32) * .1}
    else:
        spec = [dict(type="gat", **{"in": fin, "out": 8}, heads=3, concat=True, post="elu"),
                dict(type="gat", **{"in": 24, "out": 7}, heads=1)]
        w = {}
        for h in range(3):
            w[f"layer0.head{h}.weight"] = _glorot(rng, fin, 8)
            w[f"layer0.head{h}.attn_left"] = rng.standard_normal(8).astype(np.float32) * .5
            w[f"layer0.head{h}.attn_right"] = rng.standard_normal(8).astype(np.float32) * .5
            w[f"layer0.head{h}.bias"] = rng.standard_normal(8).astype(np.float32) * .1
        w.update({"layer1.head0.weight": _glorot(rng, 24, 7),
                  "layer1.head0.attn_left": rng.standard_normal(7).astype(np.float32) * .5,
                  "layer1.head0.attn_right": rng.standard_normal(7).astype(np.float32) * .5,
                  "layer1.head0.bias": rng.standard_normal(7).astype(np.float32) * .1})
    return spec, w


def _build(spec, w):
    from tinygnn_b200.handles import HModel
    m = HModel()
    for L in spec:
        if L["type"] == "gcn":
            m.add_gcn(L["in"], L["out"], act=L.get("act"))
        elif L["type"] == "sage":
            m.add_sage(L["in"], L["out"], act=L.get("act"))
        else:
            m.add_gat(L["in"], L["out"], heads=L.get("heads", 1), concat=L.get("concat", True), post=L.get("post"))
    m.load_weights(w)
    return m


@pytest.mark.parametrize("kind", ["gcn", "sage", "gat"])
@pytest.mark.parametrize("fast", [False, True])
@pytest.mark.parametrize("weighted", [False, True])
def test_handle_model_forward_vs_oracle(kind, fast, weighted):
    import tinygnn_b200 as tg
    from tinygnn_b200.handles import HTensor, set_fast_math
    rng = np.random.default_rng(len(kind) * 10 + fast * 2 + weighted)
    n, fin = 6000, 40
    rp, ci, v = powerlaw_csr(rng, n, 9, weighted=weighted, diag=False)
    X = rng.standard_normal((n, fin)).astype(np.float32)
    spec, w = _spec_weights(rng, kind, fin)
    prev = set_fast_math(fast)
    try:
        m = _build(spec, w)
        A = HTensor.csr(n, n, rp, ci, v if weighted else None)  # unweighted: values written on the device
        assert A.shape() == (n, n, ci.size, True)
        Xt = HTensor.dense(X, n, fin)
        logits = m.forward(A, Xt).download()
        tg.ops.take_device_error()
    finally:
        set_fast_math(prev)
    ref = oracle.model_forward(P, spec, w, rp, ci, v, X)
    if fast or kind == "gat":  # GAT's softmax goes through expf: the fp32 tolerance in either mode
        assert_close(P.activation("log_softmax", logits), P.activation("log_softmax", ref), f"{kind} fast={fast}")
    else:
        assert_bits_equal(logits, ref, f"{kind} exact")


def test_handle_tensors_from_pinned_torch_and_errors():
    """Pinned torch host tensors are accepted as host buffers; a malformed CSR
    is refused after its upload with the reference's message."""
    from tinygnn_b200 import _lib
    from tinygnn_b200.handles import HTensor
    X = torch.randn(100, 12).pin_memory()
    t = HTensor.dense(X, 100, 12)
    out = torch.empty(100, 12).pin_memory()
    t.download(out)
    assert torch.equal(out, X)
    rp = torch.tensor([0, 1, 3], dtype=torch.int32).pin_memory()
    ci = torch.tensor([0, 5, 1], dtype=torch.int32).pin_memory()
    with pytest.raises(ValueError, match=r"col_ind\[1\] = 5 is out of bounds for cols=2"):
        HTensor.csr(2, 2, rp, ci)
    rp_bad = np.array([0, 2, 1], np.int32)
    with pytest.raises(ValueError, match=r"row_ptr must be non-decreasing"):
        HTensor.csr(2, 2, rp_bad, np.array([0, 1], np.int32))
    assert _lib.lib.tg_tensor_download(None, None, 0) == _lib.INVALID_ARGUMENT


@pytest.mark.parametrize("kind", ["gcn", "sage", "gat"])
@pytest.mark.parametrize("fast", [False, True])
def test_forward_host_equals_forward(kind, fast):
    """tg_model_forward_host (uploads overlapped with the compute; a FAST GCN
    first layer in 16 feature blocks / column passes, a FAST GCN last layer in
    row chunks) gives tg_model_forward's output bit for bit, at the caller's
    feature stride (41: landing + device repack; 44: straight into place)
    and output stride (7: device pack; 8: one copy), twice in a row, from
    pinned and from pageable host buffers."""
    import tinygnn_b200 as tg
    from tinygnn_b200.handles import HTensor, set_fast_math
    rng = np.random.default_rng(100 + len(kind) * 10 + fast)
    n, fin = 6000, 41
    weighted = kind == "sage"
    rp, ci, v = powerlaw_csr(rng, n, 9, weighted=weighted, diag=False)
    X = rng.standard_normal((n, fin)).astype(np.float32)
    spec, w = _spec_weights(rng, kind, fin)
    prev = set_fast_math(fast)
    try:
        m = _build(spec, w)
        ref = m.forward(HTensor.csr(n, n, rp, ci, v if weighted else None), HTensor.dense(X, n, fin)).download()
        h_rp, h_ci = torch.from_numpy(rp).pin_memory(), torch.from_numpy(ci).pin_memory()
        h_v = torch.from_numpy(v).pin_memory() if weighted else None
        for ld_f in (fin, 44):
            Xh = torch.zeros((n, ld_f)).pin_memory()
            Xh[:, :fin] = torch.from_numpy(X)
            for ld_o in (7, 8):
                for _ in range(2):
                    out = torch.full((n, ld_o), float("nan")).pin_memory()
                    m.forward_host(h_rp, h_ci, h_v, Xh, fin, out, 7)
                    assert_bits_equal(out[:, :7].numpy(), ref, f"{kind} fast={fast} ld_f={ld_f} ld_o={ld_o}")
        out = np.full((n, 7), np.nan, np.float32)  # pageable numpy buffers
        m.forward_host(rp, ci, v if weighted else None, X, fin, out, 7)
        assert_bits_equal(out, ref, f"{kind} fast={fast} pageable")
        tg.ops.take_device_error()
    finally:
        set_fast_math(prev)


def test_forward_host_refuses_bad_input():
    """A malformed CSR is refused once it has landed, with the reference's
    message; wrong feature widths with the layer's message."""
    from tinygnn_b200.handles import set_fast_math
    rng = np.random.default_rng(7)
    spec, w = _spec_weights(rng, "gcn", 12)
    for fast in (False, True):
        prev = set_fast_math(fast)
        try:
            m = _build(spec, w)
            X = np.ones((3, 12), np.float32)
            out = np.zeros((3, 7), np.float32)
            rp = np.array([0, 1, 3, 3], np.int32)
            with pytest.raises(ValueError, match=r"col_ind\[2\] = 9 is out of bounds for cols=3"):
                m.forward_host(rp, np.array([0, 1, 9], np.int32), None, X, 12, out, 7)
            with pytest.raises(ValueError, match=r"in_features=12"):
                m.forward_host(rp, np.array([0, 1, 2], np.int32), None, np.ones((3, 10), np.float32), 10, out, 7)
            m.forward_host(rp, np.array([0, 1, 2], np.int32), None, X, 12, out, 7)  # still usable
            assert np.isfinite(out).all()
        finally:
            set_fast_math(prev)


@pytest.mark.parametrize("kind", ["gcn", "sage"])
def test_captured_forward_replays_forward(kind):
    """tg_model_capture records FAST Model::forward as a CUDA graph; replays
    give tg_model_forward's output bit for bit, repeatedly; forwards that read
    a size back to the host (EXACT gcn_norm, GAT self-loops) are refused."""
    import tinygnn_b200 as tg
    from tinygnn_b200.handles import HTensor, set_fast_math
    rng = np.random.default_rng(300 + len(kind))
    n, fin = 2708, 40  # Cora-sized: the launch-bound case the graph is for
    rp, ci, v = powerlaw_csr(rng, n, 4, weighted=False, diag=False)
    X = rng.standard_normal((n, fin)).astype(np.float32)
    spec, w = _spec_weights(rng, kind, fin)
    prev = set_fast_math(True)
    try:
        m = _build(spec, w)
        A, Xt = HTensor.csr(n, n, rp, ci, None), HTensor.dense(X, n, fin)
        ref = m.forward(A, Xt).download()
        g = m.capture(A, Xt)
        for _ in range(3):
            out = np.full((n, 7), np.nan, np.float32)
            g.replay().download(out)
            assert_bits_equal(out, ref, f"{kind} replay")
        g.free()
        tg.ops.take_device_error()
        set_fast_math(False)
        me = _build(spec, w)
        if kind == "gcn":
            with pytest.raises(RuntimeError, match="cannot be recorded"):
                me.capture(A, Xt)
        spec_g, w_g = _spec_weights(rng, "gat", fin)
        set_fast_math(True)
        mg = _build(spec_g, w_g)
        with pytest.raises(RuntimeError, match="cannot be recorded"):
            mg.capture(A, Xt)
        # the thread's stream is usable after a refused capture
        again = m.forward(A, Xt).download()
        assert_bits_equal(again, ref, f"{kind} after refused capture")
    finally:
        set_fast_math(prev)


def test_tensor_upload_feeds_a_captured_forward():
    """tg_tensor_upload writes new values into a tensor (dense rows at the
    host's stride, or a CSR's values): downloads read them back, and a
    captured forward replayed after new features and new edge weights were
    uploaded equals tg_model_forward on fresh tensors, bit for bit."""
    import tinygnn_b200 as tg
    from tinygnn_b200.handles import HTensor, set_fast_math
    rng = np.random.default_rng(410)
    n, fin = 3000, 41  # 41-wide host rows land beside the 44-float device stride
    rp, ci, v = powerlaw_csr(rng, n, 5, weighted=True, diag=False)
    X1 = rng.standard_normal((n, fin)).astype(np.float32)
    X2 = rng.standard_normal((n, fin)).astype(np.float32)
    v2 = (rng.random(ci.size) + 0.1).astype(np.float32)
    spec, w = _spec_weights(rng, "gcn", fin)
    prev = set_fast_math(True)
    try:
        m = _build(spec, w)
        A, Xt = HTensor.csr(n, n, rp, ci, v), HTensor.dense(X1, n, fin)
        g = m.capture(A, Xt)
        Xt.upload(X2)
        assert np.array_equal(Xt.download(), X2)
        A.upload(v2)
        out = np.empty((n, 7), np.float32)
        g.replay().download(out)
        ref = m.forward(HTensor.csr(n, n, rp, ci, v2), HTensor.dense(X2, n, fin)).download()
        assert_bits_equal(out, ref, "replay after uploads")
        g.free()
        tg.ops.take_device_error()
    finally:
        set_fast_math(prev)
