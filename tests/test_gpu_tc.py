"""The tcgen05 tensor-core GEMM (FAST mode, 3xTF32) against the exact oracle.

Tolerance |d| <= 1e-5 + 1e-4 |ref| scaled by the row's magnitude: the
3xTF32 product is within a few 1e-6 relative of fp32 per term, so the check
is on |d| <= 1e-5 + 1e-4 * sum_k |a_ik||b_kj| (the magnitude the rounding
acts on).  After every call the device error word must be clear.
"""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import assert_bits_equal

pytestmark = pytest.mark.gpu
P = oracle.port


@pytest.fixture(scope="module")
def tg():
    assert torch.cuda.is_available()
    import tinygnn_b200
    return tinygnn_b200


def padded(a, mult=4):
    """Device copy of a with the row stride rounded up (TMA needs 16-byte rows)."""
    M, K = a.shape
    ld = (K + mult - 1) // mult * mult
    t = torch.zeros((M, ld), dtype=torch.float32, device="cuda")
    t[:, :K] = torch.as_tensor(a).cuda()
    return t[:, :K]


def check(got, A, B, what, bias=None):
    ref = P.matmul(A, B)
    if bias is not None:
        ref = P.add_bias(ref, bias)
    mag = np.abs(A).astype(np.float64) @ np.abs(B).astype(np.float64)
    err = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    bad = err > 1e-5 + 1e-4 * mag
    assert not bad.any(), f"{what}: {bad.sum()} outside; max err {err.max():.3g}"
    # and the plain elementwise tolerance on these well-conditioned inputs
    rel = err / (1e-5 + 1e-4 * np.abs(ref))
    return float(rel.max())


@pytest.mark.parametrize("shape", [(128, 32, 16), (1, 8, 7), (130, 70, 41), (300, 602, 128), (257, 256, 64),
                                   (1000, 128, 41), (4099, 602, 256), (64, 1433, 16), (513, 33, 48), (200, 4, 1),
                                   (700, 128, 82), (300, 602, 96), (129, 40, 65)])
def test_tc_gemm_vs_oracle(tg, shape):
    M, K, N = shape
    rng = np.random.default_rng(M * 7 + K + N)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = (rng.standard_normal((K, N)) / np.sqrt(K)).astype(np.float32)
    out = tg.matmul(padded(A), torch.as_tensor(B).cuda(), mode="fast")
    torch.cuda.synchronize()
    tg.ops.take_device_error()
    check(out.cpu().numpy(), A, B, f"tc {shape}")


@pytest.mark.parametrize("N,padded_ok", [(41, False), (41, True), (44, False), (7, False)])
def test_tc_gemm_writes_nothing_past_n(tg, N, padded_ok):
    """An aligned output view whose rows have room past N (TMA-store epilogue):
    columns >= N stay untouched unless the caller declares them writable
    (cols_padded: up to round_up(N, 4), holding act(0) = 0 here)."""
    rng = np.random.default_rng(N)
    A = rng.standard_normal((700, 602)).astype(np.float32)
    B = (rng.standard_normal((602, N)) * 0.05).astype(np.float32)
    Cw = torch.full((700, 48), 5.0, device="cuda")
    tg.ops.matmul(padded(A), torch.as_tensor(B).cuda(), out=Cw[:, :N], mode="fast", cols_padded=padded_ok)
    torch.cuda.synchronize()
    tg.ops.take_device_error()
    h = Cw.cpu().numpy()
    check(h[:, :N], A, B, f"tc N={N}")
    n4 = (N + 3) // 4 * 4 if padded_ok else N
    assert np.all(h[:, N:n4] == 0.0), "declared padding holds act(0)"
    assert np.all(h[:, n4:] == 5.0), "written past the output's columns"


def test_tc_gemm_epilogue_and_strided_out(tg):
    rng = np.random.default_rng(3)
    A = rng.standard_normal((700, 602)).astype(np.float32)
    B = (rng.standard_normal((602, 41)) * 0.05).astype(np.float32)
    b = rng.standard_normal(41).astype(np.float32)
    Cw = torch.full((700, 48), 5.0, device="cuda")
    tg.matmul(padded(A), torch.as_tensor(B).cuda(), bias=torch.as_tensor(b).cuda(), out=Cw[:, 2:43], mode="fast")
    torch.cuda.synchronize()
    tg.ops.take_device_error()
    h = Cw.cpu().numpy()
    check(h[:, 2:43], A, B, "tc bias", bias=b)
    assert np.all(h[:, :2] == 5.0) and np.all(h[:, 43:] == 5.0)


def test_fast_mode_falls_back_when_rows_are_not_16B(tg):
    """lda % 4 != 0 cannot feed TMA: FAST mode then runs the exact kernel."""
    rng = np.random.default_rng(4)
    A = rng.standard_normal((100, 602)).astype(np.float32)   # contiguous: lda = 602
    B = rng.standard_normal((602, 16)).astype(np.float32)
    out = tg.matmul(torch.as_tensor(A).cuda(), torch.as_tensor(B).cuda(), mode="fast").cpu().numpy()
    assert np.array_equal(out.view(np.uint32), P.matmul(A, B).view(np.uint32))


def test_fast_layers_within_tolerance(tg):
    from tests.helpers import assert_close, powerlaw_csr
    rng = np.random.default_rng(5)
    n = 5000
    rp, ci, v = powerlaw_csr(rng, n, 12, weighted=False, diag=False)
    H = rng.standard_normal((n, 96)).astype(np.float32)
    W = (rng.standard_normal((96, 64)) * 0.1).astype(np.float32)
    W2 = (rng.standard_normal((96, 64)) * 0.1).astype(np.float32)
    b = rng.standard_normal(64).astype(np.float32) * 0.1
    An = P.gcn_norm(rp, ci, v)
    Hd = padded(H)
    got = tg.gcn_layer(tg.CSR.from_numpy(*An), Hd, torch.as_tensor(W).cuda(), torch.as_tensor(b).cuda(), "relu",
                       mode="fast")
    assert_close(got.cpu().numpy(), P.gcn_layer(*An, H, W, b, True), "gcn fast")
    got = tg.sage_layer(tg.CSR.from_numpy(rp, ci, v), Hd, torch.as_tensor(W).cuda(), torch.as_tensor(W2).cuda(),
                        torch.as_tensor(b).cuda(), "mean", "relu", mode="fast")
    assert_close(got.cpu().numpy(), P.sage_layer(rp, ci, v, H, W, W2, b, "mean", True), "sage fast")
    tg.ops.take_device_error()


@pytest.mark.parametrize("M,K,N", [(1000, 602, 128), (513, 128, 41), (300, 96, 20), (129, 33, 7)])
@pytest.mark.parametrize("persistent", ["0", "1"])
def test_tc_gemm_pair_vs_oracle(tg, M, K, N, persistent, monkeypatch):
    """C1 = A . B1, C2 = A . B2 in one tensor-core pass ([B1 | B2], columns
    split in the epilogue into two strided outputs); both kernels."""
    monkeypatch.setenv("TINYGNN_B200_GEMM_PERSISTENT", persistent)
    rng = np.random.default_rng(M + K + N)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B1 = (rng.standard_normal((K, N)) / np.sqrt(K)).astype(np.float32)
    B2 = (rng.standard_normal((K, N)) / np.sqrt(K)).astype(np.float32)
    ld = 2 * ((N + 3) // 4 * 4)
    T = torch.full((M, ld), 7.0, device="cuda")
    half = ld // 2
    tg.ops.gemm_pair(padded(A), torch.as_tensor(B1).cuda(), torch.as_tensor(B2).cuda(), T[:, :N], T[:, half:half + N])
    torch.cuda.synchronize()
    tg.ops.take_device_error()
    h = T.cpu().numpy()
    check(h[:, :N], A, B1, "pair C1")
    check(h[:, half:half + N], A, B2, "pair C2")
    assert np.all(h[:, N:half] == 7.0) and np.all(h[:, half + N:] == 7.0)


@pytest.mark.parametrize("N", [128, 64, 44, 41])
def test_tc_gemm_pair_persistent_matches_per_tile(tg, N, monkeypatch):
    """More tiles than SMs (each persistent CTA walks several, alternating its
    two accumulators), K > 256: the split outputs of both kernels bit-identical."""
    rng = np.random.default_rng(N)
    M, K = 40000, 300
    A = padded(rng.standard_normal((M, K)).astype(np.float32))
    B1 = torch.as_tensor((rng.standard_normal((K, N)) / np.sqrt(K)).astype(np.float32)).cuda()
    B2 = torch.as_tensor((rng.standard_normal((K, N)) / np.sqrt(K)).astype(np.float32)).cuda()
    half = (N + 3) // 4 * 4
    got = {}
    for persistent in ("0", "1"):
        monkeypatch.setenv("TINYGNN_B200_GEMM_PERSISTENT", persistent)
        T = torch.full((M, 2 * half), 7.0, device="cuda")
        tg.ops.gemm_pair(A, B1, B2, T[:, :N], T[:, half:half + N])
        torch.cuda.synchronize()
        got[persistent] = T.cpu().numpy()
    tg.ops.take_device_error()
    assert_bits_equal(got["1"], got["0"], "persistent vs per-tile (both outputs, padding untouched)")
    assert np.all(got["1"][:, N:half] == 7.0) and np.all(got["1"][:, half + N:] == 7.0)


@pytest.mark.parametrize("M,K1,K2,N", [(1000, 128, 128, 128), (700, 40, 602, 41), (300, 33, 70, 64), (129, 8, 8, 7)])
def test_tc_gemm_cat_vs_oracle(tg, M, K1, K2, N):
    """act([A1 | A2] . [B1; B2] + b) with the concatenation done by the
    operand loads (K1 not a multiple of the 32-column k-block included)."""
    rng = np.random.default_rng(M + K1 + K2 + N)
    A1 = rng.standard_normal((M, K1)).astype(np.float32)
    A2 = rng.standard_normal((M, K2)).astype(np.float32)
    B1 = (rng.standard_normal((K1, N)) / np.sqrt(K1 + K2)).astype(np.float32)
    B2 = (rng.standard_normal((K2, N)) / np.sqrt(K1 + K2)).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    got = tg.ops.gemm_cat(padded(A1), padded(A2), torch.as_tensor(B1).cuda(), torch.as_tensor(B2).cuda(),
                          bias=torch.as_tensor(b).cuda())
    torch.cuda.synchronize()
    tg.ops.take_device_error()
    A = np.concatenate([A1, A2], 1)
    B = np.concatenate([B1, B2], 0)
    check(got.cpu().numpy(), A, B, "cat", bias=b)
    # A2 not 16-byte aligned (a view one float into its buffer): the
    # two-product path, same tolerance
    buf = torch.zeros((M, K2 + 1), device="cuda")
    buf[:, 1:] = torch.as_tensor(A2).cuda()
    got = tg.ops.gemm_cat(padded(A1), buf[:, 1:], torch.as_tensor(B1).cuda(), torch.as_tensor(B2).cuda(),
                          bias=torch.as_tensor(b).cuda())
    check(got.cpu().numpy(), A, B, "cat (fallback when unaligned)", bias=b)


@pytest.mark.parametrize("fin,fout,agg", [(64, 128, "mean"), (128, 128, "mean"), (128, 40, "mean"),
                                          (40, 64, "max"), (602, 41, "mean")])
def test_fast_sage_layer_paths_vs_oracle(tg, fin, fout, agg):
    """FAST SAGELayer: aggregate-first with the concat-K tensor-core GEMM
    (F_in <= F_out, or max), transform-first with the pair GEMM (mean,
    F_in > F_out); within the tolerance of the reference's layer."""
    from tests.helpers import assert_sage_fast_close, powerlaw_csr
    rng = np.random.default_rng(fin * 3 + fout)
    n = 4000
    rp, ci, v = powerlaw_csr(rng, n, 10, weighted=False, diag=False)
    H = rng.standard_normal((n, fin)).astype(np.float32)
    Wn = (rng.standard_normal((fin, fout)) * 0.1).astype(np.float32)
    Ws = (rng.standard_normal((fin, fout)) * 0.1).astype(np.float32)
    b = (rng.standard_normal(fout) * 0.1).astype(np.float32)
    got = tg.sage_layer(tg.CSR.from_numpy(rp, ci, v), padded(H), torch.as_tensor(Wn).cuda(),
                        torch.as_tensor(Ws).cuda(), torch.as_tensor(b).cuda(), agg, "relu", mode="fast")
    torch.cuda.synchronize()
    tg.ops.take_device_error()
    assert_sage_fast_close(got.cpu().numpy(), P.sage_layer(rp, ci, v, H, Wn, Ws, b, agg, True), rp, ci, H, Wn, Ws,
                           f"sage fast {fin}->{fout} {agg}")
