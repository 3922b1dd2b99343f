"""The fused GEMM -> exchange pieces on one GPU.

tg_gemm_peers_f32 stores every output row into each "peer" copy and bumps a
counter per 128-row tile; here the peer copies and counters are other
buffers of the same GPU, which exercises the epilogue's extra stores and its
release increments without a second device.  tg_wait_flags is checked both
ways: targets already reached, and a flag nothing sets (a short timeout that
must come back as TG_ERR_TIMEOUT through tg_take_device_error, leaving the
context usable).  The cross-process path (IPC-mapped peers over NVLink) runs
in tests/dist_worker.py under torchrun.
"""
import numpy as np
import pytest
import torch

from tests.helpers import assert_bits_equal

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tg():
    assert torch.cuda.is_available()
    import tinygnn_b200
    return tinygnn_b200


@pytest.mark.parametrize("M,K,N,ld,padded", [(1000, 64, 128, 128, False), (300, 128, 41, 44, False),
                                              (300, 128, 41, 44, True), (129, 604, 128, 132, False),
                                              (1000, 96, 44, 44, False)])
@pytest.mark.parametrize("persistent", ["0", "1"])
def test_gemm_peers_stores_every_copy_and_counts_tiles(tg, M, K, N, ld, padded, persistent, monkeypatch):
    """Rows land in every copy; with padded rows (16-byte stores) the padding gets act(0) = 0.
    Both kernels: one CTA per tile, and the persistent one (TINYGNN_B200_GEMM_PERSISTENT=1)."""
    monkeypatch.setenv("TINYGNN_B200_GEMM_PERSISTENT", persistent)
    rng = np.random.default_rng(M + N)
    A = torch.as_tensor(rng.standard_normal((M, K)).astype(np.float32)).cuda()
    W = torch.as_tensor((rng.standard_normal((K, N)) * 0.1).astype(np.float32)).cuda()
    b = torch.as_tensor(rng.standard_normal(N).astype(np.float32)).cuda()
    ref = tg.ops.matmul(A, W, bias=b, act="relu", mode="fast")
    out = torch.full((M, ld), 7.0, device="cuda")
    peers = [torch.full((M, ld), 7.0, device="cuda") for _ in range(3)]
    flags = torch.zeros(3, dtype=torch.int64, device="cuda")
    tiles = -(-M // 128)
    for call in (1, 2):
        tg.ops.gemm_peers(A, W, out[:, :N], [p.data_ptr() for p in peers],
                          [flags.data_ptr() + 8 * i for i in range(3)], bias=b, act="relu", cols_padded=padded)
        torch.cuda.synchronize()
        assert_bits_equal(out[:, :N].cpu().numpy(), ref.cpu().numpy(), "local output")
        n4 = (N + 3) // 4 * 4 if padded else N
        for i, p in enumerate([out] + peers):
            assert_bits_equal(p[:, :N].cpu().numpy(), ref.cpu().numpy(), f"copy {i}")
            assert torch.all(p[:, N:n4] == 0.0), "padding columns must hold act(0)"
            assert torch.all(p[:, n4:] == 7.0), "stored outside the copy's columns"
        assert flags.tolist() == [call * tiles] * 3
    tg.ops.take_device_error()


@pytest.mark.parametrize("M,K,N,ld,padded", [(40000, 64, 128, 128, False), (40000, 128, 41, 44, True),
                                              (38001, 200, 256, 256, False)])
def test_gemm_peers_persistent_matches_per_tile(tg, M, K, N, ld, padded, monkeypatch):
    """More tiles than SMs (each persistent CTA walks several tiles, alternating its two
    accumulators), row scale + bias + activation: both kernels bit-identical in every copy."""
    rng = np.random.default_rng(M)
    A = torch.as_tensor(rng.standard_normal((M, K)).astype(np.float32)).cuda()
    W = torch.as_tensor((rng.standard_normal((K, N)) * 0.1).astype(np.float32)).cuda()
    b = torch.as_tensor(rng.standard_normal(N).astype(np.float32)).cuda()
    rs = torch.as_tensor(rng.uniform(0.1, 2.0, M).astype(np.float32)).cuda()
    got = {}
    for persistent in ("0", "1"):
        monkeypatch.setenv("TINYGNN_B200_GEMM_PERSISTENT", persistent)
        out = torch.full((M, ld), 7.0, device="cuda")
        peers = [torch.full((M, ld), 7.0, device="cuda") for _ in range(2)]
        flags = torch.zeros(2, dtype=torch.int64, device="cuda")
        tg.ops.gemm_peers(A, W, out[:, :N], [p.data_ptr() for p in peers],
                          [flags.data_ptr() + 8 * i for i in range(2)], bias=b, act="leaky_relu", alpha=0.1,
                          cols_padded=padded, row_scale=rs)
        torch.cuda.synchronize()
        assert flags.tolist() == [-(-M // 128)] * 2
        for i, p in enumerate(peers):
            assert torch.equal(p, out), f"copy {i} differs from the local output"
        got[persistent] = out.cpu().numpy()
    assert_bits_equal(got["1"], got["0"], "persistent vs per-tile")
    tg.ops.take_device_error()


def test_gemm_peers_argument_errors(tg):
    A = torch.zeros((10, 6), device="cuda")  # lda 6: not a multiple of 4
    W = torch.zeros((6, 8), device="cuda")
    with pytest.raises(ValueError, match="gemm_peers: the tensor-core path needs"):
        tg.ops.gemm_peers(A, W, torch.zeros((10, 8), device="cuda"), [], [])
    with pytest.raises(ValueError, match="npeers"):
        tg.ops.gemm_peers(torch.zeros((10, 8), device="cuda"), torch.zeros((8, 8), device="cuda"),
                          torch.zeros((10, 8), device="cuda"), [0] * 8, [0] * 8)


def test_wait_flags_reached_and_timeout(tg):
    flags = torch.tensor([5, 0, 9], dtype=torch.int64, device="cuda")
    tg.ops.wait_flags(flags, [3, 0, 9], timeout_ns=1_000_000)
    tg.ops.take_device_error()  # nothing to report
    tg.ops.wait_flags(flags, [3, 1, 0], timeout_ns=1_000_000)  # flag 1 never reaches 1
    from tinygnn_b200 import _lib
    with pytest.raises(_lib.TinyGNNError, match="flag 1 did not reach its target") as e:
        tg.ops.take_device_error()
    assert e.value.status == _lib.TIMEOUT
    tg.ops.take_device_error()  # cleared
    x = torch.ones(4, device="cuda") * 2  # the context is still usable
    assert float(x.sum()) == 8.0
