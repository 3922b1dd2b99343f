"""Malformed CSR input through the C ABI (Tensor::sparse_csr's checks,
src/tensor.cpp:46-86, plus row_ptr[0] >= 0 and row_order in range): every
entry point that reads a CSR refuses it with the reference's message before
any kernel reads through it -- the only launch is the device check itself.
No malformed array ever reaches a gather: these calls stop at the check."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _p(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _d(a):
    return torch.as_tensor(np.ascontiguousarray(a)).cuda()


# (row_ptr, col_ind, row_order, expected message) for a 3 x 4 CSR of 3 entries
BAD = [
    ([0, 1, 2, 3], [0, 9, 1], None, r"col_ind\[1\] = 9 is out of bounds for cols=4"),
    ([0, 1, 2, 3], [0, -1, 1], None, r"col_ind\[1\] = -1 is out of bounds for cols=4"),
    ([0, 2, 1, 3], [0, 1, 2], None, r"row_ptr must be non-decreasing; row_ptr\[2\] = 1 < row_ptr\[1\] = 2"),
    ([-1, 1, 2, 3], [0, 1, 2], None, r"row_ptr\[0\] \(-1\) must be >= 0"),
    ([0, 1, 2, 2], [0, 1, 2], None, r"row_ptr.back\(\) \(2\) must equal values.size\(\) \(3\)"),
    ([0, 1, 2, 3], [0, 1, 2], [0, 7, 1], r"row_order\[1\] = 7 is out of range \[0, 3\)"),
]


@pytest.mark.parametrize("case", range(len(BAD)))
def test_spmm_refuses_malformed_csr_before_gathering(case):
    import re

    import tinygnn_b200 as tg
    from tinygnn_b200 import _lib
    rp, ci, order, msg = BAD[case]
    rp, ci = _d(np.array(rp, np.int32)), _d(np.array(ci, np.int32))
    v = _d(np.ones(3, np.float32))
    o = None if order is None else _d(np.array(order, np.int32))
    B = _d(np.ones((4, 8), np.float32))
    out = torch.zeros((3, 8), device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert _lib.lib.tg_set_csr_checks(1) in (0, 1)
    n0 = tg.launches()
    st = _lib.lib.tg_spmm_f32(3, 4, 3, _p(rp), _p(ci), _p(v), _p(B), 8, 8, _p(out), 8, None, 0, 0.0, _p(o), 0, s)
    assert st == _lib.INVALID_ARGUMENT
    assert re.search(msg, _lib.last_error()), _lib.last_error()
    assert tg.launches() - n0 == 1  # the check kernel only: no gather ran
    assert torch.count_nonzero(out).item() == 0


def test_layers_and_aggregates_refuse_malformed_csr():
    """The same refusal from the layer and aggregation entry points (a column
    out of range), each before its first kernel."""
    import tinygnn_b200 as tg
    from tinygnn_b200 import _lib
    L = _lib.lib
    s = torch.cuda.current_stream().cuda_stream
    rp, ci = _d(np.array([0, 1, 2, 3], np.int32)), _d(np.array([0, 5, 1], np.int32))
    v = _d(np.ones(3, np.float32))
    H = _d(np.ones((3, 4), np.float32))
    W = _d(np.ones((4, 2), np.float32))
    a = _d(np.ones((1, 2), np.float32))
    out = torch.zeros((3, 4), device="cuda")
    calls = {
        "gcn_layer": lambda: L.tg_gcn_layer_f32(3, 3, _p(rp), _p(ci), _p(v), _p(H), 4, 4, 2, _p(W), None, 0,
                                                _p(out), 2, None, 0, s),
        "gcn_layer_noalloc": lambda: L.tg_gcn_layer_noalloc_f32(3, 3, _p(rp), _p(ci), _p(v), _p(H), 4, 4, 2, _p(W),
                                                                None, 0, _p(out), 2, None, s),
        "sage_layer": lambda: L.tg_sage_layer_f32(3, 3, _p(rp), _p(ci), _p(H), 4, 4, 2, _p(W), _p(W), None, 0, 0,
                                                  _p(out), 2, None, 0, s),
        "gat_layer": lambda: L.tg_gat_layer_f32(3, 3, _p(rp), _p(ci), _p(H), 4, 4, 1, 2, _p(W), _p(a), _p(a), None,
                                                0.2, 1, 0, _p(out), 2, None, 0, s),
        "sage_aggregate": lambda: L.tg_sage_aggregate_f32(3, 3, 3, _p(rp), _p(ci), _p(H), 4, 4, _p(out), 4, 0, s),
        "sage_max_aggregate": lambda: L.tg_sage_max_aggregate_f32(3, 3, 3, _p(rp), _p(ci), _p(H), 4, 4, _p(out),
                                                                  4, s),
        "gcn_norm": lambda: L.tg_gcn_norm_f32(3, 3, _p(rp), _p(ci), _p(v), _p(rp), _p(ci), _p(v), None, s),
    }
    for name, call in calls.items():
        n0 = tg.launches()
        assert call() == _lib.INVALID_ARGUMENT, name
        assert "col_ind[1] = 5 is out of bounds for cols=3" in _lib.last_error(), (name, _lib.last_error())
        assert tg.launches() - n0 == 1, name
    assert torch.count_nonzero(out).item() == 0


def test_python_csr_is_checked_once_and_library_csrs_are_trusted():
    """tinygnn_b200.ops: a caller's CSR is checked on its first use (a bad one
    raises ValueError); after that, and for CSRs the library built, the
    calls skip the check (one launch fewer)."""
    import tinygnn_b200 as tg
    bad = tg.CSR.from_numpy(np.array([0, 1, 2], np.int32), np.array([0, 4], np.int32), n_cols=3)
    with pytest.raises(ValueError, match=r"col_ind\[1\] = 4 is out of bounds for cols=3"):
        tg.spmm(bad, _d(np.ones((3, 4), np.float32)))
    assert not bad.validated
    rng = np.random.default_rng(0)
    rp = np.array([0, 2, 3, 5], np.int32)
    A = tg.CSR.from_numpy(rp, np.array([0, 2, 1, 0, 1], np.int32), rng.random(5).astype(np.float32))
    B = _d(rng.standard_normal((3, 4)).astype(np.float32))
    n0 = tg.launches()
    r1 = tg.spmm(A, B)
    first = tg.launches() - n0
    assert A.validated
    n0 = tg.launches()
    r2 = tg.spmm(A, B)
    assert tg.launches() - n0 == first - 1  # no check the second time
    assert torch.equal(r1, r2)
    An = tg.gcn_norm(A)
    assert An.validated
    from tinygnn_b200 import _lib
    assert _lib.lib.tg_set_csr_checks(1) == 1  # the calls restored the default
