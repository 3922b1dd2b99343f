"""Host logic of the row-partitioned path on CPU ranks (gloo), world sizes 2 and 3.

Each rank owns an equal row block, computes its rows' transform with the
oracle, exchanges them with the same in-place all-gather the GPU driver uses
(tinygnn_b200.dist.Comm), aggregates its rows, and the reassembled result
must equal the unpartitioned oracle forward bit for bit.  The row-block
gcn_norm (self-loops and degrees local, 1/sqrt(deg) all-gathered) must give
exactly the rows of the global gcn_norm.  A rank that leaves before a
collective makes the others' next collective fail within the process-group
timeout instead of hanging.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _graph(n=600, deg=9, seed=3):
    from tests.helpers import powerlaw_csr
    rng = np.random.default_rng(seed)
    rp, ci, v = powerlaw_csr(rng, n, deg, weighted=False, diag=False)
    X = rng.standard_normal((n, 24)).astype(np.float32)
    W0 = (rng.standard_normal((24, 16)) * 0.3).astype(np.float32)
    W1 = (rng.standard_normal((16, 5)) * 0.3).astype(np.float32)
    b0 = rng.standard_normal(16).astype(np.float32)
    b1 = rng.standard_normal(5).astype(np.float32)
    return n, rp, ci, v, X, W0, W1, b0, b1


def _rank_main(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        import oracle
        from tinygnn_b200.dist import Comm, row_block
        P = oracle.port
        n, rp, ci, v, X, W0, W1, b0, b1 = _graph()
        comm = Comm(world, rank)
        R, r0, r1 = row_block(n, world, rank)
        rows = r1 - r0
        # row-block gcn_norm: self-loops and degree on the block, dis exchanged
        srp, sci, sv = P.add_self_loops(rp, ci, v)
        a, b = srp[r0], srp[r1]
        lrp, lci, lv = srp[r0:r1 + 1] - a, sci[a:b], sv[a:b].copy()
        dis_all = torch.zeros(R * world, 1)
        for i in range(rows):
            d = np.float32(0.0)
            for k in range(lrp[i], lrp[i + 1]):
                d = np.float32(d + lv[k])
            dis_all[rank * R + i, 0] = float(np.float32(1.0) / np.sqrt(d)) if d > 0 else 0.0
        comm.all_gather_rows(dis_all, R)
        dis = dis_all[:, 0].numpy().astype(np.float32)
        for i in range(rows):
            for k in range(lrp[i], lrp[i + 1]):
                lv[k] = np.float32(np.float32(lv[k] * dis[r0 + i]) * dis[lci[k]])
        grp, gci, gv = P.gcn_norm(rp, ci, v)
        ga, gb = grp[r0], grp[r1]
        norm_ok = np.array_equal(lv.view(np.uint32), gv[ga:gb].view(np.uint32)) and np.array_equal(lci, gci[ga:gb])
        # two GCN layers with an all-gather of the transformed rows
        H = X[r0:r1]
        for W, bias, relu in ((W0, b0, True), (W1, b1, False)):
            full = torch.zeros(R * world, W.shape[1])
            full[rank * R:rank * R + rows] = torch.from_numpy(P.matmul(H, W))
            comm.all_gather_rows(full, R)
            out = P.spmm(lrp, lci, lv, full[:n].numpy())
            out = P.add_bias(out, bias)
            H = P.activation("relu", out) if relu else out
        parts = [None] * world
        dist.all_gather_object(parts, H)
        if rank == 0:
            got = np.concatenate(parts, axis=0)
            ref = P.gcn_layer(grp, gci, gv, P.gcn_layer(grp, gci, gv, X, W0, b0, True), W1, b1, False)
            q.put(("ok", bool(norm_ok), bool(np.array_equal(got.view(np.uint32), ref.view(np.uint32)))))
        else:
            q.put(("ok", bool(norm_ok), True))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put(("error", repr(e), False))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_row_partitioned_gcn_equals_unpartitioned(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(60)
    for status, norm_ok, fwd_ok in results:
        assert status == "ok", norm_ok
        assert norm_ok, "row-block gcn_norm differs from the global gcn_norm"
        assert fwd_ok, "partitioned forward differs from the unpartitioned oracle"


def _dropout_main(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    def report(msg):
        q.put(msg)
        q.close()
        q.join_thread()  # flush before leaving without cleanup

    if rank == 1:
        report(("left", ""))
        os._exit(0)  # leaves between steps, no collective in flight
    import sys
    sys.path.insert(0, ROOT)
    from tinygnn_b200.dist import Comm
    full = torch.zeros(4, 2)
    try:
        Comm(world, rank).all_gather_rows(full, 2)
        report(("no-error", ""))
    except Exception as e:
        report(("raised", type(e).__name__))
    os._exit(0)


def test_rank_dropout_is_detected_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dropout_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(30)
    assert ("left", "") in got
    assert any(s == "raised" for s, _ in got), got


def test_exchange_choice_is_validated():
    """ShardedModel's exchange: 'auto' / 'peer' / 'nccl', or one of the last two per layer."""
    from tinygnn_b200.dist import Comm, Layer, ShardedModel
    layers = [Layer("gcn", torch.zeros(8, 4), None, "relu"), Layer("gcn", torch.zeros(4, 2), None, None)]
    with pytest.raises(ValueError, match="one of 'peer' / 'nccl' per layer"):
        ShardedModel(layers, 16, Comm(1, 0), "cpu", mode="fast", exchange=["peer"])
    with pytest.raises(ValueError, match="one of 'peer' / 'nccl' per layer"):
        ShardedModel(layers, 16, Comm(1, 0), "cpu", mode="fast", exchange=["peer", "ring"])
    with pytest.raises(ValueError, match="exchange: 'auto', 'peer', 'nccl'"):
        ShardedModel(layers, 16, Comm(1, 0), "cpu", mode="fast", exchange="ring")
    with pytest.raises(ValueError, match="mode must be 'fast'"):
        ShardedModel(layers, 16, Comm(1, 0), "cpu", mode="exact", exchange=["nccl", "peer"])
