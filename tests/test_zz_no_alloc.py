"""tg_gcn_layer_noalloc_f32: the GCN layer for callers that cannot let a
library allocate device memory (serving loops that must not call cudaMalloc
after start-up; runtimes that own all device memory).

Called through the C ABI (ctypes, device pointers from torch), twice in a
row on different inputs -- the fixed scratch array keeps the previous call's
contents, so a stale read would show -- and compared with the allocating
entry point tg_gcn_layer_f32 in exact mode, bit for bit (tighter than the
suite's fp32 tolerance).  The default memory pool's high-water mark must not
move during the calls, and an oversized layer must be refused.  The file is
named to be collected last; it also passes on its own in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from tests.helpers import assert_bits_equal, powerlaw_csr

pytestmark = pytest.mark.gpu


def _p(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _pool_high_water():
    from cuda.bindings import runtime as rt
    err, pool = rt.cudaDeviceGetDefaultMemPool(torch.cuda.current_device())
    assert err == rt.cudaError_t.cudaSuccess
    err, high = rt.cudaMemPoolGetAttribute(pool, rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh)
    assert err == rt.cudaError_t.cudaSuccess
    return pool, int(high)


def _reset_pool_high_water(pool):
    from cuda.bindings import driver as dr
    from cuda.bindings import runtime as rt
    zero = dr.cuuint64_t(0)
    err, = rt.cudaMemPoolSetAttribute(pool, rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh, zero)
    assert err == rt.cudaError_t.cudaSuccess


def _layer_inputs(seed, n=6000, fi=48, fo=41):
    rng = np.random.default_rng(seed)
    rp, ci, v = powerlaw_csr(rng, n, 9)
    d = lambda a: torch.as_tensor(np.ascontiguousarray(a)).cuda()  # noqa: E731
    H = d(rng.standard_normal((n, fi)).astype(np.float32))
    W = d((rng.standard_normal((fi, fo)) * 0.2).astype(np.float32))
    b = d((rng.standard_normal(fo) * 0.1).astype(np.float32))
    return n, d(rp), d(ci), d(v), H, W, b


def test_noalloc_gcn_layer_matches_allocating_entry_point_twice():
    from tinygnn_b200 import _lib
    lib = _lib.lib
    stream = torch.cuda.current_stream().cuda_stream
    outs = []
    for seed in (1, 2):  # two calls in a row, different inputs
        n, rp, ci, v, H, W, b = _layer_inputs(seed)
        fi, fo = W.shape
        ref = torch.empty((n, fo), device="cuda")
        _lib.check(lib.tg_gcn_layer_f32(n, ci.numel(), _p(rp), _p(ci), _p(v), _p(H), fi, fi, fo, _p(W), _p(b),
                                        _lib.ACT_RELU, _p(ref), fo, None, _lib.MODE_EXACT, stream))
        torch.cuda.synchronize()
        pool, _ = _pool_high_water()
        _reset_pool_high_water(pool)
        out = torch.full((n, fo), float("nan"), device="cuda")
        _lib.check(lib.tg_gcn_layer_noalloc_f32(n, ci.numel(), _p(rp), _p(ci), _p(v), _p(H), fi, fi, fo, _p(W),
                                                _p(b), _lib.ACT_RELU, _p(out), fo, None, stream))
        torch.cuda.synchronize()
        _, high = _pool_high_water()
        assert high == 0, f"the no-alloc entry point took {high} bytes from the memory pool"
        assert_bits_equal(out.cpu().numpy(), ref.cpu().numpy(), f"no-alloc call seed={seed}")
        outs.append(out.cpu().numpy())
    assert not np.array_equal(outs[0], outs[1])


def test_noalloc_gcn_layer_refuses_oversized_layers():
    from tinygnn_b200 import _lib
    lib = _lib.lib
    n, fo = 40000, 128  # 40000 x 128 x 4 B = 20.5 MB > the 16 MiB scratch
    st = lib.tg_gcn_layer_noalloc_f32(n, 0, None, None, None, None, 8, 8, fo, None, None, 0, None, fo, None,
                                      torch.cuda.current_stream().cuda_stream)
    assert st == _lib.INVALID_ARGUMENT
    assert "16777216 bytes the fixed scratch holds" in _lib.last_error()
    # a width whose N * F_out * 4 would overflow int64 is refused, not wrapped
    st = lib.tg_gcn_layer_noalloc_f32(4, 0, None, None, None, None, 8, 8, 1 << 62, None, None, 0, None, 1 << 62,
                                      None, torch.cuda.current_stream().cuda_stream)
    assert st == _lib.INVALID_ARGUMENT
    assert "fixed scratch holds" in _lib.last_error()


def _hub_inputs(seed, n=6000, fi=32, fo=41, hub_len=4000):
    """A power-law graph whose row 0 is a hub of ``hub_len`` entries (above
    the hub-row kernel's threshold of 1023), in CSR with sorted columns."""
    rng = np.random.default_rng(seed)
    rp, ci, v = powerlaw_csr(rng, n, 9)
    lens = np.diff(rp)
    hub = np.sort(rng.choice(n, hub_len, replace=False)).astype(np.int32)
    lens[0] = hub_len
    rp2 = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    ci2 = np.concatenate([hub, ci[rp[1]:]]).astype(np.int32)
    v2 = np.concatenate([rng.random(hub_len).astype(np.float32), v[rp[1]:]]).astype(np.float32)
    d = lambda a: torch.as_tensor(np.ascontiguousarray(a)).cuda()  # noqa: E731
    H = d(rng.standard_normal((n, fi)).astype(np.float32))
    W = d((rng.standard_normal((fi, fo)) * 0.2).astype(np.float32))
    b = d((rng.standard_normal(fo) * 0.1).astype(np.float32))
    return n, d(rp2), d(ci2), d(v2), H, W, b


def test_noalloc_gcn_layer_with_row_order_allocates_nothing():
    """A caller-given longest-rows-first schedule with a hub row: the
    allocating entry point sends the hub to the hub-row kernel (pool memory,
    side stream); the no-alloc one keeps it in the sub-warp kernel and must
    still allocate nothing and match bit for bit, twice in a row."""
    from tinygnn_b200 import _lib
    lib = _lib.lib
    stream = torch.cuda.current_stream().cuda_stream
    outs = []
    for seed in (3, 4):
        n, rp, ci, v, H, W, b = _hub_inputs(seed)
        fi, fo = W.shape
        order = torch.empty(n, dtype=torch.int32, device="cuda")
        _lib.check(lib.tg_csr_degree_order(n, _p(rp), _p(order), stream))
        ref = torch.empty((n, fo), device="cuda")
        _lib.check(lib.tg_gcn_layer_f32(n, ci.numel(), _p(rp), _p(ci), _p(v), _p(H), fi, fi, fo, _p(W), _p(b),
                                        _lib.ACT_RELU, _p(ref), fo, _p(order), _lib.MODE_EXACT, stream))
        torch.cuda.synchronize()
        assert int(order[0]) == 0  # the hub leads the schedule
        pool, _ = _pool_high_water()
        _reset_pool_high_water(pool)
        out = torch.full((n, fo), float("nan"), device="cuda")
        _lib.check(lib.tg_gcn_layer_noalloc_f32(n, ci.numel(), _p(rp), _p(ci), _p(v), _p(H), fi, fi, fo, _p(W),
                                                _p(b), _lib.ACT_RELU, _p(out), fo, _p(order), stream))
        torch.cuda.synchronize()
        _, high = _pool_high_water()
        assert high == 0, f"the no-alloc entry point took {high} bytes from the memory pool with a row order"
        assert_bits_equal(out.cpu().numpy(), ref.cpu().numpy(), f"no-alloc call with row order seed={seed}")
        outs.append(out.cpu().numpy())
    assert not np.array_equal(outs[0], outs[1])
