"""The benchmark configurations at their full sizes on the device, checked
against the oracle on a seeded sample of rows.

Every output row of spmm and of a GCN / SAGE / GAT layer depends only on its
own CSR row and the rows it gathers, so the oracle runs on the sample's
neighbourhood: the sampled rows first (so a row's self term stays row i),
then every column they touch, renumbered in that order; rows past the sample
stay empty, so the oracle's square layer functions apply unchanged.  The
eight longest rows (the hubs) are always sampled.  Bit-identical for spmm,
the exact GEMM, GCN and SAGE layers; |d| <= 1e-5 + 1e-4 |ref| for GAT.

Sizes (the configurations of the headline benchmark's suite): R-MAT
2^20 nodes / 2^24 draws with values U(0,1] and F in {16, 64, 128, 256};
SAGE on a symmetrised R-MAT of 2^18 nodes, 128 -> 128 -> 40; GAT on an
R-MAT of 2^20 nodes stored incoming plus self-loops, 256 -> 8 heads x 8
(concat, ELU) -> 16; GCN layer 1 of the Reddit-shaped graph (232,965 nodes,
114,615,892 edges, 602 -> 128); and the Cora-shaped GCN model whole
(2,708 nodes, 1433 -> 16 -> 7), every row.
"""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import assert_bits_equal, assert_close

pytestmark = pytest.mark.gpu
P = oracle.port


@pytest.fixture(scope="module")
def tg():
    assert torch.cuda.is_available()
    import tinygnn_b200 as m
    torch.cuda.set_device(0)
    return m


def _sample(rp: torch.Tensor, k: int, seed: int) -> torch.Tensor:
    lens = rp[1:] - rp[:-1]
    hubs = torch.topk(lens, 8).indices
    g = torch.Generator().manual_seed(seed)
    rnd = torch.randint(0, lens.numel(), (k,), generator=g).to(rp.device)
    return torch.unique(torch.cat([hubs.to(torch.int64), rnd]))


def _neighbourhood(rp: torch.Tensor, ci: torch.Tensor, v: torch.Tensor, rows: torch.Tensor):
    """(sub_rp, sub_ci, sub_v, ids) as numpy / a device index: the sampled
    rows' CSR over columns renumbered into ids (rows first), padded with
    empty rows to len(ids)."""
    dev = rp.device
    rp64 = rp.to(torch.int64)
    starts, lens = rp64[rows], rp64[rows + 1] - rp64[rows]
    total = int(lens.sum())
    first = torch.cumsum(lens, 0) - lens
    idx = torch.repeat_interleave(starts, lens) + (torch.arange(total, device=dev) -
                                                   torch.repeat_interleave(first, lens))
    cols = ci[idx].to(torch.int64)
    n = rp.numel() - 1
    mark = torch.zeros(n, dtype=torch.bool, device=dev)
    mark[cols] = True
    mark[rows] = False
    ids = torch.cat([rows, torch.nonzero(mark).flatten()])
    local = torch.full((n,), -1, dtype=torch.int64, device=dev)
    local[ids] = torch.arange(ids.numel(), device=dev)
    S, U = rows.numel(), ids.numel()
    sub_rp = torch.full((U + 1,), total, dtype=torch.int64, device=dev)
    sub_rp[0] = 0
    sub_rp[1:S + 1] = torch.cumsum(lens, 0)
    return (sub_rp.to(torch.int32).cpu().numpy(), local[cols].to(torch.int32).cpu().numpy(),
            v[idx].cpu().numpy(), ids)


def _host(t: torch.Tensor) -> np.ndarray:
    return np.ascontiguousarray(t.detach().float().cpu().numpy())


@pytest.mark.parametrize("F", [16, 64, 128, 256])
def test_spmm_sweep_rmat_2e20(tg, F):
    from tinygnn_b200 import synth
    n, rp, ci, v = synth.rmat_csr(20, 1 << 24, 3, device="cuda", values_seed=3)
    A = tg.CSR(n, n, rp, ci, v)
    B = synth.normal_rows(0, n, F, 4, 0, "cuda")
    out = tg.spmm(A, B)
    rows = _sample(rp, 1500, F)
    srp, sci, sv, ids = _neighbourhood(rp, ci, v, rows)
    ref = P.spmm(srp, sci, sv, _host(B[ids]))[:rows.numel()]
    assert_bits_equal(_host(out[rows]), ref, f"spmm R-MAT 2^20 F={F}")


def test_sage_rmat_2e18(tg):
    from tinygnn_b200 import synth
    n, rp, ci, v = synth.rmat_csr(18, 5_242_880, 5, device="cuda", symmetric=True, no_self=True)
    A = tg.CSR(n, n, rp, ci, v)
    X = synth.normal_rows(0, n, 128, 6, 0, "cuda")
    Wn1, Ws1 = synth.glorot(128, 128, 6, 1, "cuda"), synth.glorot(128, 128, 6, 2, "cuda")
    Wn2, Ws2 = synth.glorot(128, 40, 6, 3, "cuda"), synth.glorot(128, 40, 6, 4, "cuda")
    b1, b2 = torch.zeros(128, device="cuda"), torch.zeros(40, device="cuda")
    H1 = tg.sage_layer(A, X, Wn1, Ws1, b1, "mean", "relu")
    H2 = tg.sage_layer(A, H1, Wn2, Ws2, b2, "mean", None)
    rows = _sample(rp, 1500, 33)
    srp, sci, sv, ids = _neighbourhood(rp, ci, v, rows)
    S = rows.numel()
    ref1 = P.sage_layer(srp, sci, sv, _host(X[ids]), _host(Wn1), _host(Ws1), _host(b1), "mean", True)[:S]
    assert_bits_equal(_host(H1[rows]), ref1, "SAGE layer 1 (2^18, 128 -> 128)")
    ref2 = P.sage_layer(srp, sci, sv, _host(H1[ids]), _host(Wn2), _host(Ws2), _host(b2), "mean", False)[:S]
    assert_bits_equal(_host(H2[rows]), ref2, "SAGE layer 2 (128 -> 40)")


def test_gat_rmat_2e20(tg):
    from tinygnn_b200 import synth
    n, rp, ci, v = synth.rmat_csr(20, 1 << 24, 7, device="cuda", transpose=True)
    Asl = tg.add_self_loops(tg.CSR(n, n, rp, ci, v))
    X = synth.normal_rows(0, n, 256, 8, 0, "cuda")
    heads, d = 8, 8
    W = torch.cat([synth.glorot(256, d, 8, 10 + h, "cuda") for h in range(heads)], 1)
    al = torch.stack([synth.glorot(d, 1, 8, 30 + h, "cuda").flatten() for h in range(heads)])
    ar = torch.stack([synth.glorot(d, 1, 8, 50 + h, "cuda").flatten() for h in range(heads)])
    bias = torch.zeros((heads, d), device="cuda")
    H1 = tg.gat_layer(Asl, X, W, al, ar, heads, bias, 0.2, True, None)
    tg.elu_(H1)
    W2 = synth.glorot(64, 16, 8, 70, "cuda")
    al2, ar2 = synth.glorot(16, 1, 8, 71, "cuda").flatten(), synth.glorot(16, 1, 8, 72, "cuda").flatten()
    H2 = tg.gat_layer(Asl, H1, W2, al2.reshape(1, -1), ar2.reshape(1, -1), 1, torch.zeros((1, 16), device="cuda"),
                      0.2, True, None)
    rows = _sample(Asl.row_ptr, 1500, 44)
    srp, sci, sv, ids = _neighbourhood(Asl.row_ptr, Asl.col_ind, Asl.values, rows)
    S = rows.numel()
    Xs, Wh = _host(X[ids]), _host(W)
    ref1 = np.concatenate([P.gat_layer(srp, sci, sv, Xs, Wh[:, h * d:(h + 1) * d].copy(), _host(al[h]),
                                       _host(ar[h]), np.zeros(d, np.float32), 0.2, False)[:S]
                           for h in range(heads)], axis=1)
    ref1 = P.activation("elu", ref1, 1.0)
    assert_close(_host(H1[rows]), ref1, "GAT layer 1 (2^20, 8 heads x 8, ELU)")
    ref2 = P.gat_layer(srp, sci, sv, _host(H1[ids]), _host(W2), _host(al2), _host(ar2),
                       np.zeros(16, np.float32), 0.2, False)[:S]
    assert_close(_host(H2[rows]), ref2, "GAT layer 2 (64 -> 16)")


def test_gcn_layer1_reddit_shape(tg):
    """The exact GEMM rows and the gather rows of GCN layer 1 on the
    Reddit-shaped graph (each checked on the device's own operand), and the
    fused layer equal to their composition."""
    import bench
    from tinygnn_b200 import synth
    n, rp, ci, v = bench.make_graph(False, "cuda", 0)
    An = tg.gcn_norm(tg.CSR(n, n, rp, ci, v))
    X = synth.normal_rows(0, n, bench.FEATS, bench.FEAT_SEED, 0, "cuda")
    W = synth.glorot(bench.FEATS, bench.HIDDEN, bench.WEIGHT_SEED, 1, "cuda")
    b = torch.full((bench.HIDDEN,), 0.01, device="cuda")
    HW = tg.matmul(X, W, mode="exact")
    out = tg.spmm(An, HW, bias=b, act="relu")
    rows = _sample(An.row_ptr, 300, 55)
    assert_bits_equal(_host(HW[rows]), P.matmul(_host(X[rows]), _host(W)), "GEMM 232,965 x 602 x 128 rows")
    srp, sci, sv, ids = _neighbourhood(An.row_ptr, An.col_ind, An.values, rows)
    S = rows.numel()
    ref = P.activation("relu", P.add_bias(P.spmm(srp, sci, sv, _host(HW[ids])), _host(b)))[:S]
    assert_bits_equal(_host(out[rows]), ref, "gather rows (nnz 114,848,857, F = 128)")
    fused = tg.gcn_layer(An, X, W, b, "relu")
    assert torch.equal(fused.view(torch.int32), out.view(torch.int32)), "gcn_layer != matmul + spmm"


def test_gcn_cora_shape_full_model(tg):
    """The Cora-shaped configuration whole: gcn_norm, GCN 1433 -> 16 (ReLU)
    -> 7, log_softmax, exact mode -- every row against the oracle (and the
    reference library itself where it was built)."""
    from tinygnn_b200 import synth
    n, rp, ci, v, X = synth.cora_like(device="cuda")
    W0, W1 = synth.glorot(1433, 16, 2, 1, "cuda"), synth.glorot(16, 7, 2, 2, "cuda")
    b0, b1 = torch.zeros(16, device="cuda"), torch.zeros(7, device="cuda")
    An = tg.gcn_norm(tg.CSR(n, n, rp, ci, v))
    H1 = tg.gcn_layer(An, X, W0, b0, "relu")
    logits = tg.gcn_layer(An, H1, W1, b1, None)
    out = tg.log_softmax_(logits.clone())
    hrp, hci, hv = _host(rp).astype(np.int32), _host(ci).astype(np.int32), _host(v)
    spec = [dict(type="gcn", **{"in": 1433, "out": 16}, act="relu"), dict(type="gcn", **{"in": 16, "out": 7})]
    w = {"layer0.weight": _host(W0), "layer0.bias": _host(b0), "layer1.weight": _host(W1), "layer1.bias": _host(b1)}
    for impl in [P] + ([oracle.ref] if oracle.ref is not None else []):
        ref = oracle.model_forward(impl, spec, w, hrp, hci, hv, _host(X))
        assert_bits_equal(_host(logits), ref, f"Cora-shaped GCN logits vs {impl.name}")
        assert_close(_host(out), impl.activation("log_softmax", ref), f"Cora-shaped log_softmax vs {impl.name}")
    assert int(An.nnz) == 13_264 and n == 2708
