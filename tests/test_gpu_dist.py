"""The row-partitioned GCN / SAGE path on one GPU, P ranks emulated in lockstep.

Each emulated rank is a tinygnn_b200.dist.ShardedModel over its own row
block; the all-gather between the transform and aggregate phases is
emulated by copying every shard's block into every shard's gather buffer
(the layout NCCL's all_gather_into_tensor produces).  Results must equal the
unpartitioned forward bit for bit (exact mode), and the row-block gcn_norm
must equal the rows of the global gcn_norm.  The real NCCL path runs under
torchrun in tests/test_gpu_dist_nccl.py when several GPUs are visible.
"""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import assert_bits_equal, assert_close, powerlaw_csr

pytestmark = pytest.mark.gpu
P = oracle.port


@pytest.fixture(scope="module")
def tg():
    assert torch.cuda.is_available()
    import tinygnn_b200
    return tinygnn_b200


class LocalComm:
    """Comm stand-in for one shard when the exchange is done by the test."""

    def __init__(self, world, rank):
        self.world, self.rank, self.group = world, rank, None

    def all_gather_rows(self, full, R):
        pass


def _graph(n=30000, seed=1):
    rng = np.random.default_rng(seed)
    rp, ci, v = powerlaw_csr(rng, n, 14, weighted=False, diag=False)
    X = rng.standard_normal((n, 40)).astype(np.float32)
    return rng, rp, ci, v, X


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_row_block_gcn_norm_matches_global(tg, world):
    from tinygnn_b200.dist import row_block, slice_rows
    rng, rp, ci, v, X = _graph()
    n = rp.size - 1
    A = tg.CSR.from_numpy(rp, ci, v)
    G = P.gcn_norm(rp, ci, v)
    R = (n + world - 1) // world
    dis_all = torch.zeros(R * world, device="cuda")
    blocks = []
    for r in range(world):  # phase 1: local self-loops + degrees
        _, r0, r1 = row_block(n, world, r)
        Ar = slice_rows(A.row_ptr, A.col_ind, A.values, r0, r1, n)
        asl = tg.ops.add_self_loops_rows(Ar, r0)
        tg.ops.degree_inv_sqrt(asl, out=dis_all[r * R:r * R + (r1 - r0)])
        blocks.append((r0, r1, asl))
    for r, (r0, r1, asl) in enumerate(blocks):  # phase 2: scale with every rank's 1/sqrt(deg)
        tg.ops.scale_sym_(asl, dis_all[r * R:r * R + (r1 - r0)], dis_all)
        a, b = G[0][r0], G[0][r1]
        assert_bits_equal(asl.row_ptr.cpu().numpy(), (G[0][r0:r1 + 1] - a).astype(np.int32), "row_ptr")
        assert_bits_equal(asl.col_ind.cpu().numpy(), G[1][a:b], "col_ind")
        assert_bits_equal(asl.values.cpu().numpy(), G[2][a:b], "values")


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_two_pass_row_block_gcn_norm_matches_global(tg, world):
    """tg_gcn_norm_rows_degrees_f32 / _fill_f32 per row block, with an
    emulated all-gather of 1/sqrt(deg) between them, equal the rows of the
    global gcn_norm bit for bit (weighted rows too: the sequential degree)."""
    from tinygnn_b200.dist import row_block, slice_rows
    rng, rp, ci, v, X = _graph()
    n = rp.size - 1
    for weighted, ordered in ((False, False), (True, False), (False, True), (True, True)):
        vv = (rng.random(ci.size) + 0.25).astype(np.float32) if weighted else v
        A = tg.CSR.from_numpy(rp, ci, vv)
        G = P.gcn_norm(rp, ci, vv)
        R = (n + world - 1) // world
        dis_all = torch.zeros(R * world, device="cuda")
        firsts = []
        for r in range(world):
            _, r0, r1 = row_block(n, world, r)
            Ar = slice_rows(A.row_ptr, A.col_ind, A.values, r0, r1, n)
            if ordered:  # the longest-first schedule only orders the work
                Ar.order = tg.degree_order(Ar)
            firsts.append((r0, r1, Ar) + tg.ops.gcn_norm_rows_degrees(Ar, r0, dis_all[r * R:r * R + (r1 - r0)]))
        for r, (r0, r1, Ar, rpo, ins) in enumerate(firsts):
            B = tg.ops.gcn_norm_rows_fill(Ar, r0, rpo, ins, dis_all[r * R:r * R + (r1 - r0)], dis_all)
            a, b = G[0][r0], G[0][r1]
            assert_bits_equal(B.row_ptr.cpu().numpy(), (G[0][r0:r1 + 1] - a).astype(np.int32), "row_ptr")
            assert_bits_equal(B.col_ind.cpu().numpy(), G[1][a:b], "col_ind")
            assert_bits_equal(B.values.cpu().numpy(), G[2][a:b], f"values weighted={weighted} ordered={ordered}")


@pytest.mark.parametrize("workload,bpr", [("gcn", 2), ("gcn", 3), ("sage", 4)])
def test_single_gpu_column_passes_are_bit_identical(tg, workload, bpr):
    from tinygnn_b200.dist import Comm, Layer, ShardedModel, gcn_norm_rows
    rng, rp, ci, v, X = _graph(seed=bpr)
    n = rp.size - 1
    W0 = torch.as_tensor((rng.standard_normal((40, 32)) * 0.2).astype(np.float32)).cuda()
    W1 = torch.as_tensor((rng.standard_normal((32, 11)) * 0.2).astype(np.float32)).cuda()
    S0 = torch.as_tensor((rng.standard_normal((40, 32)) * 0.2).astype(np.float32)).cuda()
    S1 = torch.as_tensor((rng.standard_normal((32, 11)) * 0.2).astype(np.float32)).cuda()
    sage = workload == "sage"
    layers = [Layer(workload, W0, None, "relu", S0 if sage else None),
              Layer(workload, W1, None, None, S1 if sage else None)]
    A = tg.CSR.from_numpy(rp, ci, v)
    An = gcn_norm_rows(A, 0, n, Comm(1, 0)) if not sage else None
    Xd = torch.as_tensor(X).cuda()
    one = ShardedModel(layers, n, Comm(1, 0), "cuda", passes=1).forward(An, A, Xd).clone()
    blk = ShardedModel(layers, n, Comm(1, 0), "cuda", passes=bpr).forward(An, A, Xd)
    pip = ShardedModel(layers, n, Comm(1, 0), "cuda", blocks_per_rank=bpr, pipeline=True).forward(An, A, Xd)
    torch.cuda.synchronize()
    assert_bits_equal(blk.cpu().numpy(), one.cpu().numpy(), f"{workload} {bpr} passes")
    assert_bits_equal(pip.cpu().numpy(), one.cpu().numpy(), f"{workload} {bpr} blocks (pipelined path)")


@pytest.mark.parametrize("workload,mode,blocks,unweighted,fin,chunks", [
    ("gcn", "exact", 8, False, 40, 4), ("gcn", "fast", 5, False, 40, 1), ("sage", "fast", 1, False, 40, 4),
    ("gcn", "exact", 8, True, 37, 3), ("gcn", "fast", 8, True, 37, 4), ("sage", "fast", 1, True, 37, 7)])
def test_forward_from_host_equals_resident_forward(tg, workload, mode, blocks, unweighted, fin, chunks):
    """The pipelined host-input call (uploads overlapped with gcn_norm and the
    per-block layer-1 passes; features of a width that is not a multiple of 4
    repacked on the device; the last layer in row chunks whose logits stream
    back) returns exactly the resident forward's logits; an unweighted graph
    passes no values (1.0 written on the device)."""
    from tinygnn_b200.dist import Comm, Layer, ShardedModel, gcn_norm_rows
    rng, rp, ci, v, X = _graph(seed=11)
    if unweighted:
        v = np.ones_like(v)
    n = rp.size - 1
    W0 = torch.as_tensor((rng.standard_normal((fin, 32)) * 0.2).astype(np.float32)).cuda()
    W1 = torch.as_tensor((rng.standard_normal((32, 11)) * 0.2).astype(np.float32)).cuda()
    S0 = torch.as_tensor((rng.standard_normal((fin, 32)) * 0.2).astype(np.float32)).cuda()
    S1 = torch.as_tensor((rng.standard_normal((32, 11)) * 0.2).astype(np.float32)).cuda()
    b0 = torch.as_tensor((rng.standard_normal(32) * 0.1).astype(np.float32)).cuda()
    sage = workload == "sage"
    layers = [Layer(workload, W0, b0, "relu", S0 if sage else None),
              Layer(workload, W1, None, None, S1 if sage else None)]
    model = ShardedModel(layers, n, Comm(1, 0), "cuda", mode=mode)
    A = tg.CSR.from_numpy(rp, ci, v)
    Xd = torch.zeros((n, (fin + 3) // 4 * 4), device="cuda")[:, :fin]
    Xd[:] = torch.as_tensor(X[:, :fin]).cuda()
    # the resident Model::forward (EXACT: normalised copy; FAST: factored)
    ref = model.forward_model(A, Xd).cpu().numpy().copy()
    pin = lambda t: t.cpu().pin_memory()  # noqa: E731
    h_out = torch.empty((n, 11)).pin_memory()
    bufs = {}
    for _ in range(2):  # buffers reused on the second call
        h_out.zero_()
        model.forward_from_host(pin(A.row_ptr), pin(A.col_ind), None if unweighted else pin(A.values), pin(Xd),
                                h_out, bufs, feature_blocks=blocks, out_chunks=chunks)
        assert_bits_equal(h_out.numpy(), ref, f"{workload} {mode} from host")


@pytest.mark.parametrize("workload,world", [("gcn", 2), ("gcn", 4), ("sage", 3), ("gcn", 8)])
def test_sharded_forward_equals_unpartitioned(tg, workload, world):
    from tinygnn_b200.dist import Layer, ShardedModel, gcn_norm_rows, row_block, slice_rows
    rng, rp, ci, v, X = _graph(seed=world)
    n = rp.size - 1
    W0 = torch.as_tensor((rng.standard_normal((40, 32)) * 0.2).astype(np.float32)).cuda()
    W1 = torch.as_tensor((rng.standard_normal((32, 11)) * 0.2).astype(np.float32)).cuda()
    S0 = torch.as_tensor((rng.standard_normal((40, 32)) * 0.2).astype(np.float32)).cuda()
    S1 = torch.as_tensor((rng.standard_normal((32, 11)) * 0.2).astype(np.float32)).cuda()
    b0 = torch.as_tensor((rng.standard_normal(32) * 0.1).astype(np.float32)).cuda()
    b1 = torch.as_tensor((rng.standard_normal(11) * 0.1).astype(np.float32)).cuda()
    kind = workload
    layers = [Layer(kind, W0, b0, "relu", S0 if kind == "sage" else None),
              Layer(kind, W1, b1, None, S1 if kind == "sage" else None)]
    A = tg.CSR.from_numpy(rp, ci, v)
    Xd = torch.as_tensor(X).cuda()

    # reference: one shard holding everything
    one = ShardedModel(layers, n, LocalComm(1, 0), "cuda")
    from tinygnn_b200.dist import Comm
    An_full = gcn_norm_rows(A, 0, n, Comm(1, 0)) if kind == "gcn" else None
    ref = one.forward(An_full, A, Xd).clone()

    shards, graphs, H = [], [], []
    R = (n + world - 1) // world
    dis_all = torch.zeros(R * world, device="cuda")
    for r in range(world):
        _, r0, r1 = row_block(n, world, r)
        Ar = slice_rows(A.row_ptr, A.col_ind, A.values, r0, r1, n)
        shards.append(ShardedModel(layers, n, LocalComm(world, r), "cuda"))
        graphs.append([r0, r1, Ar, None])
        H.append(Xd[r0:r1])
    if kind == "gcn":
        asls = []
        for r, (r0, r1, Ar, _) in enumerate(graphs):
            asl = tg.ops.add_self_loops_rows(Ar, r0)
            tg.ops.degree_inv_sqrt(asl, out=dis_all[r * R:r * R + (r1 - r0)])
            asls.append(asl)
        for r, asl in enumerate(asls):
            r0, r1 = graphs[r][0], graphs[r][1]
            graphs[r][3] = tg.ops.scale_sym_(asl, dis_all[r * R:r * R + (r1 - r0)], dis_all)
    for li in range(2):
        for r, sh in enumerate(shards):
            sh.transform(li, H[r])
        for r, sh in enumerate(shards):  # emulated all-gather
            for q, src in enumerate(shards):
                if q != r:
                    sh.full[li][q * R:(q + 1) * R] = src.full[li][q * R:(q + 1) * R]
        H = [sh.aggregate(li, graphs[r][3], graphs[r][2]) for r, sh in enumerate(shards)]
    got = torch.cat([tg.log_softmax_(h) for h in H], 0)
    torch.cuda.synchronize()
    if kind == "gcn":
        assert_bits_equal(got.cpu().numpy(), ref.cpu().numpy(), f"{kind} x{world}")
    else:
        assert_close(got.cpu().numpy(), ref.cpu().numpy(), f"{kind} x{world}")
    # and the unpartitioned forward itself against the oracle
    spec = [dict(type=kind, **{"in": 40, "out": 32}, act="relu"), dict(type=kind, **{"in": 32, "out": 11})]
    w = ({"layer0.weight": W0, "layer0.bias": b0, "layer1.weight": W1, "layer1.bias": b1} if kind == "gcn" else
         {"layer0.weight_neigh": W0, "layer0.weight_self": S0, "layer0.bias": b0,
          "layer1.weight_neigh": W1, "layer1.weight_self": S1, "layer1.bias": b1})
    w = {k: t.cpu().numpy() for k, t in w.items()}
    oref = P.activation("log_softmax", oracle.model_forward(P, spec, w, rp, ci, v, X))
    assert_close(ref.cpu().numpy(), oref, f"{kind} vs oracle")


@pytest.mark.parametrize("world,weighted", [(1, False), (1, True), (2, False), (3, True), (8, False)])
def test_fast_factored_gcn_forward(tg, world, weighted):
    """FAST GCN without a normalised copy of A (per-row 1/sqrt(deg) folded
    into the GEMM and gather epilogues): emulated ranks equal one rank bit
    for bit (every factor is rank-local), and the logits are within the fp32
    tolerance of the oracle's Model::forward (gcn_norm, layers, log_softmax)."""
    from tinygnn_b200.dist import Layer, ShardedModel, row_block, slice_rows
    rng, rp, ci, v, X = _graph(seed=20 + world)
    if weighted:
        v = (rng.random(ci.size) + 0.25).astype(np.float32)
    n = rp.size - 1
    W0 = torch.as_tensor((rng.standard_normal((40, 32)) * 0.2).astype(np.float32)).cuda()
    W1 = torch.as_tensor((rng.standard_normal((32, 11)) * 0.2).astype(np.float32)).cuda()
    b0 = torch.as_tensor((rng.standard_normal(32) * 0.1).astype(np.float32)).cuda()
    b1 = torch.as_tensor((rng.standard_normal(11) * 0.1).astype(np.float32)).cuda()
    layers = [Layer("gcn", W0, b0, "relu"), Layer("gcn", W1, b1, None)]
    A = tg.CSR.from_numpy(rp, ci, v)
    Xd = torch.as_tensor(X).cuda()
    one = ShardedModel(layers, n, LocalComm(1, 0), "cuda", mode="fast")
    ref = one.forward_model(A, Xd).clone()

    R = (n + world - 1) // world
    shards, preps, H = [], [], []
    for r in range(world):
        _, r0, r1 = row_block(n, world, r)
        sh = ShardedModel(layers, n, LocalComm(world, r), "cuda", mode="fast")
        shards.append(sh)
        preps.append(sh.prepare(slice_rows(A.row_ptr, A.col_ind, A.values, r0, r1, n)))
        H.append(Xd[r0:r1])
    for li in range(2):
        for r, sh in enumerate(shards):
            sh.scale = preps[r][2]
            sh.transform(li, H[r])
        for r, sh in enumerate(shards):  # emulated all-gather
            for q, src in enumerate(shards):
                if q != r:
                    sh.full[li][q * R:(q + 1) * R] = src.full[li][q * R:(q + 1) * R]
        H = []
        for r, sh in enumerate(shards):
            sh.scale = preps[r][2]
            H.append(sh.aggregate(li, preps[r][0], preps[r][1]))
            sh.scale = None
    got = torch.cat([tg.log_softmax_(h) for h in H], 0)
    torch.cuda.synchronize()
    assert_bits_equal(got.cpu().numpy(), ref.cpu().numpy(), f"fast gcn x{world} vs one rank")
    spec = [dict(type="gcn", **{"in": 40, "out": 32}, act="relu"), dict(type="gcn", **{"in": 32, "out": 11})]
    w = {"layer0.weight": W0, "layer0.bias": b0, "layer1.weight": W1, "layer1.bias": b1}
    w = {k: t.cpu().numpy() for k, t in w.items()}
    oref = P.activation("log_softmax", oracle.model_forward(P, spec, w, rp, ci, v, X))
    assert_close(ref.cpu().numpy(), oref, f"fast factored gcn weighted={weighted} vs oracle")


def test_gcn_norm_scale_matches_gcn_norm_degrees(tg):
    """1/sqrt(row sum + 1) of the raw rows is gcn_norm's 1/sqrt(deg) of A + I:
    bit for bit on integer-valued rows (with and without diagonals), within
    the tolerance on fractional ones."""
    rng = np.random.default_rng(5)
    n = 30000
    rp, ci, v = powerlaw_csr(rng, n, 14, weighted=False, diag=True)  # some rows hold their diagonal
    for kind in ("unit", "integer", "fractional"):
        vv = {"unit": np.ones_like(v), "integer": rng.integers(1, 5, v.size).astype(np.float32),
              "fractional": (rng.random(v.size) + 0.1).astype(np.float32)}[kind]
        A = tg.CSR.from_numpy(rp, ci, vv)
        exact = torch.empty(n, device="cuda")
        tg.ops.gcn_norm_rows_degrees(A, 0, exact)
        fast = tg.ops.gcn_norm_scale(A)
        if kind == "fractional":
            assert_close(fast.cpu().numpy(), exact.cpu().numpy(), kind)
        else:
            assert_bits_equal(fast.cpu().numpy(), exact.cpu().numpy(), kind)


@pytest.mark.parametrize("fin", [40, 602])
def test_fast_sage_model_logits_vs_oracle(tg, fin):
    """FAST SAGE-mean Model::forward (transform-first, W_neigh and W_self in
    one tensor-core pass) -- logits within |d| <= 1e-5 + 1e-4 |ref| of the
    oracle's Model::forward + log_softmax, elementwise."""
    from tinygnn_b200.dist import Comm, Layer, ShardedModel
    rng, rp, ci, v, X = _graph(n=20000, seed=31 + fin)
    X = rng.standard_normal((rp.size - 1, fin)).astype(np.float32)
    n = rp.size - 1
    g = lambda i, o: (rng.uniform(-1, 1, (i, o)) * np.sqrt(6.0 / (i + o))).astype(np.float32)  # noqa: E731
    Wn0, Ws0, Wn1, Ws1 = g(fin, 32), g(fin, 32), g(32, 11), g(32, 11)
    b0 = (rng.standard_normal(32) * 0.1).astype(np.float32)
    b1 = (rng.standard_normal(11) * 0.1).astype(np.float32)
    d = lambda a: torch.as_tensor(a).cuda()  # noqa: E731
    layers = [Layer("sage", d(Wn0), d(b0), "relu", d(Ws0)), Layer("sage", d(Wn1), d(b1), None, d(Ws1))]
    Xd = torch.zeros((n, (fin + 3) // 4 * 4), device="cuda")[:, :fin]
    Xd[:] = d(X)
    got = ShardedModel(layers, n, Comm(1, 0), "cuda", mode="fast").forward_model(tg.CSR.from_numpy(rp, ci, v), Xd)
    spec = [dict(type="sage", **{"in": fin, "out": 32}, act="relu"), dict(type="sage", **{"in": 32, "out": 11})]
    w = {"layer0.weight_neigh": Wn0, "layer0.weight_self": Ws0, "layer0.bias": b0,
         "layer1.weight_neigh": Wn1, "layer1.weight_self": Ws1, "layer1.bias": b1}
    oref = P.activation("log_softmax", oracle.model_forward(P, spec, w, rp, ci, v, X))
    tg.ops.take_device_error()
    assert_close(got.cpu().numpy(), oref, f"fast sage model fin={fin}")


def test_fast_forward_model_reuses_its_buffers_across_graphs(tg):
    """forward_model keeps the per-call schedule and split points in buffers
    the model rewrites every call: forwards on different graphs in turn each
    give the prepared (own-buffer) forward's logits bit for bit."""
    from tinygnn_b200.dist import Comm, Layer, ShardedModel
    rng = np.random.default_rng(5)
    n, fin = 30000, 40
    W0 = torch.as_tensor((rng.standard_normal((fin, 32)) * 0.2).astype(np.float32)).cuda()
    W1 = torch.as_tensor((rng.standard_normal((32, 11)) * 0.2).astype(np.float32)).cuda()
    b0 = torch.as_tensor((rng.standard_normal(32) * 0.1).astype(np.float32)).cuda()
    b1 = torch.as_tensor((rng.standard_normal(11) * 0.1).astype(np.float32)).cuda()
    # passes=2: the layer-1 gather in column passes (split points in the model's buffer)
    m = ShardedModel([Layer("gcn", W0, b0, "relu"), Layer("gcn", W1, b1, None)], n, Comm(1, 0), "cuda",
                     mode="fast", passes=2)
    graphs = []
    for deg in (14, 3, 22):
        rp, ci, v = powerlaw_csr(rng, n, deg, weighted=False, diag=False)
        X = torch.as_tensor(rng.standard_normal((n, fin)).astype(np.float32)).cuda()
        A = tg.CSR.from_numpy(rp, ci, v)
        ref = m.forward_prepared(m.prepare(A), X).clone()
        graphs.append((A, X, ref))
    for _ in range(2):  # queued back to back: each call rewrites the buffers the previous one read
        for A, X, _ in graphs:
            m.forward_model(tg.CSR(A.n_rows, A.n_cols, A.row_ptr, A.col_ind, A.values), X)
    torch.cuda.synchronize()
    for (A, X, ref) in graphs:
        got = m.forward_model(tg.CSR(A.n_rows, A.n_cols, A.row_ptr, A.col_ind, A.values), X).clone()
        assert_bits_equal(got.cpu().numpy(), ref.cpu().numpy(), "forward_model after other graphs")
    tg.ops.take_device_error()
