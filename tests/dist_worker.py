"""Worker for tests/test_gpu_dist_nccl.py, run under torchrun (one process per GPU).

Builds the same seeded graph on every rank, runs the row-partitioned GCN
forward over NCCL (tinygnn_b200.dist), gathers the logits on rank 0 and
compares them with the single-GPU forward of the whole graph (bit-identical
in exact mode).  Exit code 0 = pass.
"""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    import tinygnn_b200 as tg
    from tinygnn_b200 import synth
    from tinygnn_b200.dist import Comm, Layer, ShardedModel, gcn_norm_rows, row_block, slice_rows

    n, rp, ci, v = synth.chung_lu_csr(50000, 3_000_000, 5, device=dev)
    X = synth.normal_rows(0, n, 64, 6, 0, dev)
    W0, W1 = synth.glorot(64, 32, 7, 1, dev), synth.glorot(32, 9, 7, 2, dev)
    b0 = torch.zeros(32, device=dev)
    b1 = torch.full((9,), 0.1, device=dev)
    layers = [Layer("gcn", W0, b0, "relu"), Layer("gcn", W1, b1, None)]
    comm = Comm(world, rank)
    R, r0, r1 = row_block(n, world, rank)
    A = slice_rows(rp, ci, v, r0, r1, n)
    An = gcn_norm_rows(A, r0, R, comm)
    ok = True
    ref = None
    if rank == 0:
        full = tg.CSR(n, n, rp, ci, v)
        one = ShardedModel(layers, n, Comm(1, 0), dev, mode="exact")
        ref = one.forward(gcn_norm_rows(full, 0, n, Comm(1, 0)), full, X).clone()
    for pipeline, passes in ((False, 1), (False, 3), (True, "auto"), ("auto", "auto")):  # all-gather + passes / broadcasts
        model = ShardedModel(layers, n, comm, dev, mode="exact", pipeline=pipeline, passes=passes)
        out = model.forward(An, A, X[r0:r1].contiguous())
        parts = [torch.zeros((R, 9), device=dev) for _ in range(world)]
        mine = torch.zeros((R, 9), device=dev)
        mine[:r1 - r0] = out
        dist.all_gather(parts, mine)
        if rank == 0:
            same = bool(torch.equal(torch.cat(parts, 0)[:n], ref))
            print(f"pipeline={pipeline} passes={passes} same={same}", flush=True)
            ok = ok and same
    # FAST mode: the fused GEMM -> NVLink exchange (IPC-mapped peer buffers,
    # counters, device-side waits) against GEMM + NCCL all-gather.  Same
    # tensor-core GEMM and gathers, so the logits must match bit for bit;
    # three forwards use both buffer parities.
    nccl = ShardedModel(layers, n, comm, dev, mode="fast", exchange="nccl")
    peer = ShardedModel(layers, n, comm, dev, mode="fast", exchange="peer")
    mixed = ShardedModel(layers, n, comm, dev, mode="fast", exchange=["peer"] + ["nccl"] * (len(layers) - 1))
    for step in range(3):
        a = nccl.forward(An, A, X[r0:r1].contiguous()).clone()
        c = mixed.forward(An, A, X[r0:r1].contiguous()).clone()
        b = peer.forward(An, A, X[r0:r1].contiguous())
        torch.cuda.synchronize()
        same = bool(torch.equal(a, b)) and bool(torch.equal(a, c))
        if rank == 0:
            print(f"peer exchange step {step} same={same}", flush=True)
        ok = ok and same
    # FAST Model::forward without a normalised copy of A (1/sqrt(deg) in the
    # GEMM and gather epilogues): both exchanges, and the single GPU, agree
    # bit for bit -- every factor is rank-local.
    ref_fast = None
    if rank == 0:
        full = tg.CSR(n, n, rp, ci, v)
        ref_fast = ShardedModel(layers, n, Comm(1, 0), dev, mode="fast").forward_model(full, X).clone()
    for step in range(2):
        a = nccl.forward_model(A, X[r0:r1].contiguous()).clone()
        b = peer.forward_model(A, X[r0:r1].contiguous()).clone()
        torch.cuda.synchronize()
        parts = [torch.zeros((R, 9), device=dev) for _ in range(world)]
        mine = torch.zeros((R, 9), device=dev)
        mine[:r1 - r0] = b
        dist.all_gather(parts, mine)
        same = bool(torch.equal(a, b))
        if rank == 0:
            same = same and bool(torch.equal(torch.cat(parts, 0)[:n], ref_fast))
            print(f"factored fast step {step} same={same}", flush=True)
        ok = ok and same
    # The host-input call on every rank (its rows from pinned host memory,
    # features of a width that is not a multiple of 4, the last layer in row
    # chunks) against the same model's resident forward, with either exchange.
    Xh = synth.normal_rows(r0, r1 - r0, 61, 8, 0, dev)
    Xd = torch.zeros((r1 - r0, 64), device=dev)[:, :61]
    Xd[:] = Xh
    W61 = synth.glorot(61, 32, 7, 3, dev)
    pin = lambda t: t.cpu().pin_memory()  # noqa: E731
    h_v = None if bool(torch.all(A.values == 1.0)) else pin(A.values)
    for kind in ("nccl", "peer"):
        m = ShardedModel([Layer("gcn", W61, b0, "relu"), Layer("gcn", W1, b1, None)], n, comm, dev, mode="fast",
                         exchange=kind)
        want = m.forward_model(A, Xd).clone()
        h_out = torch.empty((r1 - r0, 9)).pin_memory()
        bufs = {}
        for step in range(2):
            h_out.zero_()
            m.forward_from_host(pin(A.row_ptr), pin(A.col_ind), h_v, pin(Xd), h_out, bufs)
            same = bool(torch.equal(h_out.to(dev), want))
            if rank == 0:
                print(f"forward_from_host {kind} step {step} same={same}", flush=True)
            ok = ok and same
        m.close()
    tg.ops.take_device_error()
    peer.close()
    mixed.close()
    if rank == 0:
        print(f"world={world} bit-identical={ok}", flush=True)
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.broadcast(flag, 0)
    dist.barrier()
    dist.destroy_process_group()
    return 0 if int(flag.item()) == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
