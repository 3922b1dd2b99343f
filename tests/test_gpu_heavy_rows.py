"""Long (hub) rows: the heavy-row gather kernel against the oracle.

The leading slots of a degree schedule whose rows have at least
max(1023, ~nnz/16384) entries (1023 for these graphs) are produced by the
heavy-row kernel (async copies into a shared-memory ring) on a side stream,
the rest by the sub-warp kernel.  Every
result must be bit-identical to the oracle's sequential chain, whichever
kernel produced a row: rows right at the threshold (1022 / 1023 / 1024
entries), a row over every column, empty rows, several feature passes
(F > 512), unweighted (SAGE) and max reductions, epilogues and
column-block passes.
"""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import assert_bits_equal

pytestmark = pytest.mark.gpu
P = oracle.port

HUB_LENS = (1022, 1023, 1024, 1500, 4096, 9000)


@pytest.fixture(scope="module")
def tg():
    assert torch.cuda.is_available()
    import tinygnn_b200
    return tinygnn_b200


def hub_graph(seed, n=20000, extra_full_row=True):
    """Short random rows, hubs of HUB_LENS entries (and one over every column), empty rows."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(0, 12, n)
    hubs = rng.choice(n, len(HUB_LENS) + 1, replace=False)
    lens[hubs[:len(HUB_LENS)]] = HUB_LENS
    if extra_full_row:
        lens[hubs[-1]] = n
    lens[rng.choice(n, 50, replace=False)] = 0
    rp = np.zeros(n + 1, np.int32)
    rp[1:] = np.cumsum(lens)
    ci = np.concatenate([np.sort(rng.choice(n, k, replace=False)) if k else np.zeros(0, np.int64)
                         for k in lens]).astype(np.int32)
    v = (rng.random(ci.size) + 0.05).astype(np.float32)
    return rng, rp, ci, v


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("F", [1, 5, 16, 41, 44, 128, 200, 300, 602])
def test_spmm_hub_rows_vs_oracle(tg, F):
    rng, rp, ci, v = hub_graph(F)
    n = rp.size - 1
    A = tg.CSR.from_numpy(rp, ci, v)
    Fp = (F + 3) // 4 * 4
    Bbuf = torch.zeros((n, Fp), device="cuda")  # ldb % 4 == 0: the heavy kernel's 16-byte copies apply
    B = rng.standard_normal((n, F)).astype(np.float32)
    Bbuf[:, :F] = torch.as_tensor(B).cuda()
    ref = P.spmm(rp, ci, v, B)
    assert_bits_equal(host(tg.spmm(A, Bbuf[:, :F])), ref, f"spmm F={F} (auto schedule)")
    order = tg.degree_order(A)
    assert_bits_equal(host(tg.spmm(A, Bbuf[:, :F], row_order=order)), ref, f"spmm F={F} (given schedule)")
    b = rng.standard_normal(F).astype(np.float32)
    ref_e = P.activation("relu", P.add_bias(ref, b))
    out = torch.full((n, F + 3), 5.0, device="cuda")
    tg.spmm(A, Bbuf[:, :F], bias=torch.as_tensor(b).cuda(), act="relu", out=out[:, 1:1 + F])
    got = host(out)
    assert_bits_equal(got[:, 1:1 + F], ref_e, f"spmm F={F} bias+relu into a strided output")
    assert np.all(got[:, 0] == 5.0) and np.all(got[:, 1 + F:] == 5.0), "wrote outside the output slice"
    tg.ops.take_device_error()


@pytest.mark.parametrize("F", [8, 41, 128, 300])
def test_sage_mean_and_max_hub_rows(tg, F):
    rng, rp, ci, v = hub_graph(50 + F)
    n = rp.size - 1
    A = tg.CSR.from_numpy(rp, ci, v)
    Fp = (F + 3) // 4 * 4
    Hbuf = torch.zeros((n, Fp), device="cuda")
    H = rng.standard_normal((n, F)).astype(np.float32)
    Hbuf[:, :F] = torch.as_tensor(H).cuda()
    assert_bits_equal(host(tg.sage_max_aggregate(A, Hbuf[:, :F])), P.sage_max_aggregate(rp, ci, v, H),
                      f"sage max F={F}")
    # mean: the unweighted sum chain, then one multiply by the rounded 1/deg
    s = P.spmm(rp, ci, np.ones_like(v), H)
    deg = np.diff(rp).astype(np.float32)
    inv = np.where(deg > 0, np.float32(1) / np.maximum(deg, np.float32(1)), np.float32(1)).astype(np.float32)
    mean = (s * inv[:, None]).astype(np.float32)
    assert_bits_equal(host(tg.ops.sage_aggregate(A, Hbuf[:, :F], "mean")), mean, f"sage mean F={F}")
    tg.ops.take_device_error()


@pytest.mark.parametrize("nblocks", [2, 5])
def test_hub_rows_in_column_block_passes(tg, nblocks):
    rng, rp, ci, v = hub_graph(7 + nblocks)
    n, F = rp.size - 1, 128
    A = tg.CSR.from_numpy(rp, ci, v).with_degree_order()
    B = torch.as_tensor(rng.standard_normal((n, F)).astype(np.float32)).cuda()
    Ts = torch.as_tensor(rng.standard_normal((n, F)).astype(np.float32)).cuda()
    b = torch.as_tensor(rng.standard_normal(F).astype(np.float32)).cuda()
    width = (n + nblocks - 1) // nblocks
    sp = tg.ops.column_splits(A, nblocks, width)
    one = host(tg.spmm(A, B, bias=b, act="relu"))
    assert_bits_equal(one, P.activation("relu", P.add_bias(P.spmm(rp, ci, v, host(B)), host(b))), "one pass")
    out = torch.empty((n, F), device="cuda")
    for q in range(nblocks):
        tg.ops.spmm_segment(A, B, sp[q], sp[q + 1], out, q > 0, q == nblocks - 1, bias=b, act="relu")
    assert_bits_equal(host(out), one, f"spmm in {nblocks} passes")
    ref = host(tg.ops.sage_mean_combine(A, B, Ts, bias=b, act="relu"))
    for q in range(nblocks):
        tg.ops.sage_mean_combine_segment(A, B, Ts, sp[q], sp[q + 1], out, q > 0, q == nblocks - 1, bias=b,
                                         act="relu")
    assert_bits_equal(host(out), ref, f"sage combine in {nblocks} passes")
    tg.ops.take_device_error()


def test_gcn_layer_with_hub_rows_vs_oracle(tg):
    rng, rp, ci, v = hub_graph(99)
    n = rp.size - 1
    An = P.gcn_norm(rp, ci, v)
    H = rng.standard_normal((n, 24)).astype(np.float32)
    W = (rng.standard_normal((24, 64)) * 0.3).astype(np.float32)
    b = (rng.standard_normal(64) * 0.1).astype(np.float32)
    got = tg.gcn_layer(tg.CSR.from_numpy(*An), torch.as_tensor(H).cuda(), torch.as_tensor(W).cuda(),
                       torch.as_tensor(b).cuda(), "relu")
    assert_bits_equal(host(got), P.gcn_layer(*An, H, W, b, True), "gcn layer with hub rows")
    tg.ops.take_device_error()


@pytest.mark.parametrize("heads,d,concat", [(8, 8, True), (1, 16, True), (4, 3, False), (2, 41, True)])
def test_gat_hub_rows_vs_oracle(tg, heads, d, concat):
    """GAT over hub rows: rows at and above the threshold are cut into
    512-entry chunks whose online-softmax states merge in order (1022..9000
    entries and one row over every column -- up to 40 chunks), the rest run
    as whole rows; every head of every row within the fp32 tolerance of the
    oracle's per-head GATLayer."""
    from tests.helpers import assert_close
    rng, rp, ci, v = hub_graph(7 + heads + d)
    Asl_np = P.add_self_loops(rp, ci, v)
    n = rp.size - 1
    fi = 24
    X = rng.standard_normal((n, fi)).astype(np.float32)
    W = (rng.standard_normal((fi, heads * d)) * 0.3).astype(np.float32)
    al = (rng.standard_normal((heads, d)) * 0.5).astype(np.float32)
    ar = (rng.standard_normal((heads, d)) * 0.5).astype(np.float32)
    b = (rng.standard_normal((heads, d)) * 0.1).astype(np.float32)
    A = tg.CSR.from_numpy(*Asl_np)
    dev = lambda a: torch.as_tensor(a).cuda()  # noqa: E731
    got = host(tg.gat_layer(A, dev(X), dev(W), dev(al), dev(ar), heads, dev(b), 0.2, concat, None))
    per_head = [P.gat_layer(*Asl_np, X, W[:, h * d:(h + 1) * d].copy(), al[h], ar[h], b[h], 0.2, False)
                for h in range(heads)]
    if concat:
        ref = np.concatenate(per_head, axis=1)
    else:
        acc = np.zeros_like(per_head[0])
        for t in per_head:
            acc = (acc + t).astype(np.float32)
        ref = (acc * np.float32(1.0 / heads)).astype(np.float32)
    assert_close(got, ref, f"GAT hub rows h={heads} d={d} concat={concat}")
    tg.ops.take_device_error()
