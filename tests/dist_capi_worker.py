"""Worker for tests/test_gpu_dist_capi.py: one process per GPU, the C ABI only
(tg_tensor_*, tg_model_*, tg_dist_*).  Every rank builds the same seeded
graph, uploads its row block, runs tg_dist_forward for a GCN and a SAGE
model in EXACT and FAST mode and writes its logits; rank 0 compares the assembled logits with
tg_model_forward of the whole graph on its GPU (bit for bit).
Usage: dist_capi_worker.py WORLD RANK ID_PATH OUT_DIR"""
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402


def main() -> int:
    world, rank, id_path, out_dir = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3], sys.argv[4]
    from tinygnn_b200.handles import HDist, HModel, HTensor, partition_rows, set_fast_math
    from tests.helpers import powerlaw_csr
    rng = np.random.default_rng(123)
    n, fin = 20000, 40
    rp, ci, v = powerlaw_csr(rng, n, 10, weighted=False, diag=False)
    X = rng.standard_normal((n, fin)).astype(np.float32)
    g = lambda i, o: (rng.uniform(-1, 1, (i, o)) * np.sqrt(6.0 / (i + o))).astype(np.float32)  # noqa: E731
    w = {"layer0.weight": g(fin, 32), "layer0.bias": rng.standard_normal(32).astype(np.float32) * .1,
         "layer1.weight": g(32, 9), "layer1.bias": rng.standard_normal(9).astype(np.float32) * .1}
    ws = {"layer0.weight_neigh": g(fin, 32), "layer0.weight_self": g(fin, 32),
          "layer0.bias": rng.standard_normal(32).astype(np.float32) * .1,
          "layer1.weight_neigh": g(32, 9), "layer1.weight_self": g(32, 9),
          "layer1.bias": rng.standard_normal(9).astype(np.float32) * .1}
    r0, r1, e0, e1 = partition_rows(world, rank, n, rp)
    d = HDist(world, rank, rank, id_path, 60000)
    ok = True
    runs = [(kind, fast) for kind in ("gcn", "sage") for fast in (False, True)]
    for run, (kind, fast) in enumerate(runs):
        set_fast_math(fast)
        if kind == "gcn":
            m = HModel().add_gcn(fin, 32, act="relu").add_gcn(32, 9, act=None)
            m.load_weights(w)
        else:  # fin > 32: transform-first (the pair GEMM) in FAST mode
            m = HModel().add_sage(fin, 32, act="relu").add_sage(32, 9, act=None)
            m.load_weights(ws)
        A = HTensor.csr(r1 - r0, n, (rp[r0:r1 + 1] - e0).astype(np.int32), ci[e0:e1].copy(), None)
        Xt = HTensor.dense(np.ascontiguousarray(X[r0:r1]), r1 - r0, fin)
        part = d.forward(m, n, A, Xt).download()
        np.save(os.path.join(out_dir, f"part{run}_{rank}.npy"), part)
        open(os.path.join(out_dir, f"done{run}_{rank}"), "w").close()
        if rank == 0:
            full = m.forward(HTensor.csr(n, n, rp, ci, None), HTensor.dense(X, n, fin)).download()
            deadline = time.time() + 120
            while not all(os.path.exists(os.path.join(out_dir, f"done{run}_{q}")) for q in range(world)):
                if time.time() > deadline:
                    print("timeout waiting for the other ranks", flush=True)
                    return 1
                time.sleep(0.05)
            got = np.concatenate([np.load(os.path.join(out_dir, f"part{run}_{q}.npy")) for q in range(world)])
            same = bool(np.array_equal(got.view(np.uint32), full.view(np.uint32)))
            R = -(-n // world)
            blocks = [float(np.abs(got[q * R:(q + 1) * R] - full[q * R:(q + 1) * R]).max()) for q in range(world)]
            print(f"{kind} fast={fast} same={same} max |diff| per rank block {blocks}", flush=True)
            ok = ok and same
    d.finalize()
    if rank == 0:
        print(f"world={world} bit-identical={ok}", flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
