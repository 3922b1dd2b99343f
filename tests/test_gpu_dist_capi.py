"""The row-partitioned forward behind the C ABI (tg_dist_*): one rank on one
GPU equals tg_model_forward bit for bit (EXACT and FAST, GCN and SAGE); a
rank whose peers never join gets TG_ERR_TIMEOUT from its bounded wait (no
kernel is involved); with several GPUs, worker processes that use only the C
ABI (tests/dist_capi_worker.py) match the single-GPU forward bit for bit."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from tests.helpers import assert_bits_equal, powerlaw_csr

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _model(kind, fin, rng):
    from tinygnn_b200.handles import HModel
    g = lambda i, o: (rng.uniform(-1, 1, (i, o)) * np.sqrt(6.0 / (i + o))).astype(np.float32)  # noqa: E731
    m = HModel()
    if kind == "gcn":
        m.add_gcn(fin, 32, act="relu").add_gcn(32, 9, act=None)
        w = {"layer0.weight": g(fin, 32), "layer0.bias": rng.standard_normal(32).astype(np.float32) * .1,
             "layer1.weight": g(32, 9), "layer1.bias": rng.standard_normal(9).astype(np.float32) * .1}
    else:
        m.add_sage(fin, 32, act="relu").add_sage(32, 9, act=None)
        w = {"layer0.weight_neigh": g(fin, 32), "layer0.weight_self": g(fin, 32),
             "layer0.bias": rng.standard_normal(32).astype(np.float32) * .1,
             "layer1.weight_neigh": g(32, 9), "layer1.weight_self": g(32, 9),
             "layer1.bias": rng.standard_normal(9).astype(np.float32) * .1}
    m.load_weights(w)
    return m


@pytest.mark.parametrize("kind,fin", [("gcn", 40), ("sage", 40), ("sage", 24)])
@pytest.mark.parametrize("fast", [False, True])
def test_one_rank_dist_forward_equals_model_forward(tmp_path, kind, fin, fast):
    import tinygnn_b200 as tg
    from tinygnn_b200.handles import HDist, HTensor, set_fast_math
    rng = np.random.default_rng(7 + fast)
    n = 5000
    rp, ci, v = powerlaw_csr(rng, n, 8, weighted=False, diag=False)
    X = rng.standard_normal((n, fin)).astype(np.float32)
    prev = set_fast_math(fast)
    try:
        m = _model(kind, fin, rng)
        A, Xt = HTensor.csr(n, n, rp, ci, v), HTensor.dense(X, n, fin)
        want = m.forward(A, Xt).download()
        d = HDist(1, 0, torch.cuda.current_device(), str(tmp_path / "nccl.id"), 30000)
        got = d.forward(m, n, A, Xt).download()
        d.finalize()
        tg.ops.take_device_error()
    finally:
        set_fast_math(prev)
    assert_bits_equal(got, want, f"{kind} fast={fast}")


def test_rank_whose_peers_never_join_times_out(tmp_path):
    """world = 2 with only rank 0 started: joining the communicator gives up
    after the timeout with TG_ERR_TIMEOUT (run in a child process)."""
    code = ("import sys; sys.path.insert(0, %r)\n"
            "import ctypes as C\n"
            "from tinygnn_b200 import _lib\n"
            "h = C.c_void_p()\n"
            "st = _lib.lib.tg_dist_init(2, 0, 0, %r, 3000, C.byref(h))\n"
            "print('status', st, _lib.last_error())\n" % (ROOT, str(tmp_path / "id").encode()))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120,
                       env=dict(os.environ, NCCL_NVLS_ENABLE="0"))
    assert r.returncode == 0, r.stderr[-3000:]
    assert "status 6" in r.stdout and "did not complete within 3000 ms" in r.stdout, r.stdout


@pytest.mark.parametrize("world", [2, 4])
def test_c_abi_dist_forward_across_gpus(tmp_path, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs, {torch.cuda.device_count()} visible")
    procs = []
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    for r in range(world):
        procs.append(subprocess.Popen([sys.executable, os.path.join(ROOT, "tests", "dist_capi_worker.py"), str(world),
                                       str(r), str(tmp_path / "nccl.id"), str(tmp_path)],
                                      env=env, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True))
    outs = []
    for p in procs:
        try:
            o, e = p.communicate(timeout=300)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
        outs.append((p.returncode, o, e))
    for rc, o, e in outs:
        assert rc == 0, o[-2000:] + e[-3000:]
    assert "bit-identical=True" in outs[0][1], outs[0][1]
