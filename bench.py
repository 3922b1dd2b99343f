"""Benchmark: 2-layer GCN (or SAGE-mean) forward on the Reddit-shaped graph.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload gcn|sage] [--small]

Workload (the configuration the headline metric is quoted
on at 1/2/4/8 GPUs): seeded Chung-Lu graph of 232,965 nodes and
114,615,892 directed edges (mean degree ~492, heavy tail), 602-wide N(0,1)
features, 602 -> 128 (ReLU) -> 41, log_softmax; Glorot weights, zero bias.
A step is one forward of the whole graph.  For N > 1 (torchrun, one process
per GPU) rows are split in equal blocks and each layer all-gathers its
transformed rows over NCCL (tinygnn_b200/dist.py).

Reported (rank 0, one JSON line):
  value   edges/s = nnz(A_norm) / forward time, inputs resident in HBM,
          normalised adjacency cached (max over ranks of CUDA-event time);
  e2e     the same metric through the public path with host inputs: every
          step uploads the raw CSR rows + feature rows from pinned memory,
          runs gcn_norm, the forward and log_softmax, and reads the logits
          back;
  roofline  the layer-1 gather (SpMM, F=128): algorithmic bytes
          nnz*(8+4F) + rows*(4+4F) + 4 per launch / its CUDA-event time,
          against the measured HBM copy bandwidth (MEASURED_PEAKS.json);
  cpu_baseline  the reference library (oracle/_ref) Model::forward on the
          same graph on this host's cores (rank 0, N = 1), and beside it
          (layers_only) its layer objects on an adjacency normalised once.
--impl reference times that reference forward alone (rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

NODES, EDGES, FEATS, HIDDEN, CLASSES = 232_965, 114_615_892, 602, 128, 41
SMALL = (20_000, 2_000_000)
GRAPH_SEED, FEAT_SEED, WEIGHT_SEED = 9, 10, 10


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["gcn", "sage"], default="gcn")
    ap.add_argument("--mode", choices=["fast", "exact"], default="fast",
                    help="fast: 3xTF32 tensor-core GEMMs (within fp32 tolerance); exact: bit-identical GEMMs")
    ap.add_argument("--small", action="store_true", help="a 20k-node graph (quick functional run)")
    ap.add_argument("--edges", type=int, default=0, help="override the edge count (profiling on a smaller graph)")
    ap.add_argument("--passes", default="auto",
                    help="column passes per gather after the all-gather (auto: operand bytes / 64 MB)")
    ap.add_argument("--exchange", default="auto",
                    help="N > 1: peer = the GEMM stores its tiles into every GPU's gather buffer over NVLink; "
                         "nccl = GEMM then NCCL all-gather / broadcasts (auto: peer in fast mode); "
                         "or one per layer, comma-separated (e.g. peer,nccl)")
    ap.add_argument("--pipeline", choices=["auto", "on", "off"], default="auto",
                    help="N > 1: per-rank async broadcasts with a gather pass per arriving block "
                         "(auto: on 2-4 GPUs, for the layers whose exchanged operand is >= 64 MB)")
    ap.add_argument("--blocks-per-rank", default="auto",
                    help="column blocks per rank for the gathers: 'auto' or a count")
    ap.add_argument("--micro", choices=["hub", "l2"], default=None,
                    help="hub: time one long row through spmm (the heavy-row path); l2: the random-row gather "
                         "rate of spmm over a 64 MB operand that stays in L2 (the ceiling of the gathers); "
                         "instead of the benchmark")
    ap.add_argument("--micro-entries", type=int, default=13_531)
    ap.add_argument("--micro-features", type=int, default=128)
    ap.add_argument("--suite", action="store_true",
                    help="one line per other benchmark configuration (Cora-shaped GCN, R-MAT spmm sweep, SAGE, "
                         "GAT): GPU time beside the reference's CPU time; not the headline line")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    return ap.parse_args()


# ── workload ─────────────────────────────────────────────────────────────────
def make_graph(small: bool, device, edges: int = 0):
    from tinygnn_b200 import synth
    n, e = SMALL if small else (NODES, EDGES)
    if edges:
        e = edges
    n, rp, ci, v = synth.chung_lu_csr(n, e, GRAPH_SEED, device=device)
    return n, rp, ci, v


def make_weights(workload: str, device):
    from tinygnn_b200 import synth
    g = lambda i, o, s: synth.glorot(i, o, WEIGHT_SEED, s, device)  # noqa: E731
    z = lambda o: torch.zeros(o, dtype=torch.float32, device=device)  # noqa: E731
    if workload == "gcn":
        return {"layer0.weight": g(FEATS, HIDDEN, 1), "layer0.bias": z(HIDDEN),
                "layer1.weight": g(HIDDEN, CLASSES, 2), "layer1.bias": z(CLASSES)}
    return {"layer0.weight_neigh": g(FEATS, HIDDEN, 1), "layer0.weight_self": g(FEATS, HIDDEN, 3),
            "layer0.bias": z(HIDDEN), "layer1.weight_neigh": g(HIDDEN, CLASSES, 2),
            "layer1.weight_self": g(HIDDEN, CLASSES, 4), "layer1.bias": z(CLASSES)}


def layer_stack(workload: str, w):
    from tinygnn_b200.dist import Layer
    if workload == "gcn":
        return [Layer("gcn", w["layer0.weight"], w["layer0.bias"], "relu"),
                Layer("gcn", w["layer1.weight"], w["layer1.bias"], None)]
    return [Layer("sage", w["layer0.weight_neigh"], w["layer0.bias"], "relu", w["layer0.weight_self"]),
            Layer("sage", w["layer1.weight_neigh"], w["layer1.bias"], None, w["layer1.weight_self"])]


def ref_spec(workload: str):
    t = workload
    return [dict(type=t, **{"in": FEATS, "out": HIDDEN}, act="relu"),
            dict(type=t, **{"in": HIDDEN, "out": CLASSES}, act=None)]


# ── clocks sampled during the timed region ───────────────────────────────────
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.samples = []
        self.proc = None
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            self.gpu = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        except Exception:
            self.gpu = str(device_index)
        self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.gpu, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.out, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except Exception:
            self.proc.kill()
        self.out.flush()
        rows = []
        with open(self.out.name) as f:
            for line in f:
                p = [x.strip() for x in line.split(",")]
                if len(p) < 7:
                    continue
                try:
                    rows.append((float(p[0]), float(p[1]), float(p[2]), p[3:7]))
                except ValueError:
                    continue
        os.unlink(self.out.name)
        if not rows:
            return None
        load = [r for r in rows if r[2] > 200.0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in load for i, x in enumerate(r[3]) if x.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in load), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(load), "power_w_max": max(r[2] for r in rows)}


# ── timing helpers ───────────────────────────────────────────────────────────
def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def time_steps(step, K: int, W: int, world: int) -> float:
    """ms for exactly K steps after W warm-up steps (CUDA events, max over ranks)."""
    for _ in range(W):
        step()
    barrier(world)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(K):
        step()
    e.record()
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(s.elapsed_time(e), world)


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def committed_traffic(kernel_tag: str):
    """Per-launch DRAM bytes of a kernel from the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        parts = line.split()
        if len(parts) >= 2 and parts[0] == kernel_tag:
            try:
                return float(parts[1])
            except ValueError:
                return None
    return None


# ── reference arm / CPU baseline ─────────────────────────────────────────────
def cpu_impl():
    """(kind, cores): the CPU implementation the reference arm and the
    cpu_baseline leg time -- the reference library compiled from its own
    sources (oracle/_ref) where it was built, else the C restatement of its
    algorithms (oracle/tg_oracle.c) -- set to every host core this process
    may run on (torchrun starts its ranks with OMP_NUM_THREADS=1)."""
    import oracle
    try:
        cores = len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        cores = os.cpu_count() or 1
    impl = ("reference", oracle.ref) if oracle.ref is not None else ("port", oracle.port)
    impl[1].set_num_threads(cores)
    return impl[0], impl[1].max_threads()


def _host(t, dtype):
    return np.ascontiguousarray(t.cpu().numpy(), dtype=dtype)


def port_forward_timer(workload, n, rp, ci, v, X, weights):
    """A callable running Model::forward + log_softmax once through the C
    restatement: gcn_norm of the raw adjacency every call (src/model.cpp:
    365-381), the layers, log_softmax (oracle.model_forward)."""
    import oracle
    P = oracle.port
    spec = ref_spec(workload)
    w = {k: t.cpu().numpy() for k, t in weights.items()}
    rp_h, ci_h, v_h, X_h = _host(rp, np.int32), _host(ci, np.int32), _host(v, np.float32), _host(X, np.float32)

    def run():
        P.activation("log_softmax", oracle.model_forward(P, spec, w, rp_h, ci_h, v_h, X_h))

    return run, lambda: None


def port_layers_timer(workload, n, rp, ci, v, X, weights):
    """The C restatement's layers + log_softmax on an adjacency normalised once."""
    import oracle
    P = oracle.port
    w = {k: t.cpu().numpy() for k, t in weights.items()}
    rp_h, ci_h, v_h, X_h = _host(rp, np.int32), _host(ci, np.int32), _host(v, np.float32), _host(X, np.float32)
    An = P.gcn_norm(rp_h, ci_h, v_h) if workload == "gcn" else None

    def run():
        if workload == "gcn":
            H = P.gcn_layer(*An, X_h, w["layer0.weight"], w["layer0.bias"], True)
            H = P.gcn_layer(*An, H, w["layer1.weight"], w["layer1.bias"], False)
        else:
            H = P.sage_layer(rp_h, ci_h, v_h, X_h, w["layer0.weight_neigh"], w["layer0.weight_self"],
                             w["layer0.bias"], "mean", True)
            H = P.sage_layer(rp_h, ci_h, v_h, H, w["layer1.weight_neigh"], w["layer1.weight_self"],
                             w["layer1.bias"], "mean", False)
        P.activation("log_softmax", H)

    return run, lambda: None


def reference_forward_timer(workload, n, rp, ci, v, X, weights):
    """A callable running the reference library's Model::forward + log_softmax
    once (the C restatement's where the reference library was not built)."""
    import oracle
    R = oracle.ref
    if R is None:
        return port_forward_timer(workload, n, rp, ci, v, X, weights)
    m = R.model(ref_spec(workload), {k: t.cpu().numpy() for k, t in weights.items()})
    rp_h = np.ascontiguousarray(rp.cpu().numpy(), dtype=np.int32)
    ci_h = np.ascontiguousarray(ci.cpu().numpy(), dtype=np.int32)
    v_h = np.ascontiguousarray(v.cpu().numpy(), dtype=np.float32)
    X_h = np.ascontiguousarray(X.cpu().numpy(), dtype=np.float32)
    lib = R.lib
    # The reference Tensors own copies of the arrays: the forward reads only them.
    A = lib.ref_tensor_csr(n, ci_h.size, rp_h.ctypes.data, ci_h.ctypes.data, v_h.ctypes.data)
    Xt = lib.ref_tensor_dense(X_h.shape[0], X_h.shape[1], X_h.ctypes.data)
    del rp_h, ci_h, v_h, X_h

    def run():
        rc = lib.ref_model_forward_tensors(m.h, A, Xt, None, 1)
        if rc:
            raise RuntimeError(lib.ref_last_error().decode())

    def free():
        lib.ref_tensor_free(A)
        lib.ref_tensor_free(Xt)

    return run, free


def reference_layers_timer(workload, n, rp, ci, v, X, weights):
    """A callable running the reference's layer objects (GCNLayer / SAGELayer)
    + log_softmax once on an adjacency normalised beforehand: the layer
    forwards of Model::forward without its per-call gcn_norm (the C
    restatement's where the reference library was not built)."""
    import oracle
    R = oracle.ref
    if R is None:
        return port_layers_timer(workload, n, rp, ci, v, X, weights)
    st = R.stack(ref_spec(workload), {k: t.cpu().numpy() for k, t in weights.items()})
    rp_h = np.ascontiguousarray(rp.cpu().numpy(), dtype=np.int32)
    ci_h = np.ascontiguousarray(ci.cpu().numpy(), dtype=np.int32)
    v_h = np.ascontiguousarray(v.cpu().numpy(), dtype=np.float32)
    X_h = np.ascontiguousarray(X.cpu().numpy(), dtype=np.float32)
    lib = R.lib
    A = lib.ref_tensor_csr(n, ci_h.size, rp_h.ctypes.data, ci_h.ctypes.data, v_h.ctypes.data)
    Xt = lib.ref_tensor_dense(X_h.shape[0], X_h.shape[1], X_h.ctypes.data)
    del rp_h, ci_h, v_h, X_h
    An = st.gcn_norm_tensor(A) if workload == "gcn" else None

    def run():
        st.forward_tensors(An if An is not None else A, A, Xt, True)

    def free():
        for t in (A, Xt, An):
            if t:
                lib.ref_tensor_free(t)

    return run, free


def time_reference(run, budget_s: float):
    """1 warm-up, then up to 5 timed calls within ``budget_s`` (at least 1):
    (median seconds per call, calls)."""
    run()
    times, t0 = [], time.perf_counter()
    while not times or (time.perf_counter() - t0 < budget_s and len(times) < 5):
        t = time.perf_counter()
        run()
        times.append(time.perf_counter() - t)
    return statistics.median(times), len(times)


def nnz_normalized(rp, ci, n):
    """nnz of gcn_norm(A) = nnz(A) + rows without a diagonal entry."""
    rows = torch.repeat_interleave(torch.arange(n, device=rp.device), (rp[1:] - rp[:-1]).long())
    has = torch.zeros(n, dtype=torch.bool, device=rp.device)
    has[rows[ci.long() == rows]] = True
    return int(ci.numel() + n - int(has.sum()))


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    kind, cores = cpu_impl()
    dev = "cuda" if torch.cuda.is_available() else "cpu"  # input synthesis only
    n, rp, ci, v = make_graph(args.small, dev, args.edges)
    from tinygnn_b200 import synth
    X = synth.normal_rows(0, n, FEATS, FEAT_SEED, 0, dev)
    w = make_weights(args.workload, dev)
    nnz = nnz_normalized(rp, ci, n) if args.workload == "gcn" else int(ci.numel())
    run, free = reference_forward_timer(args.workload, n, rp, ci, v, X, w)
    del rp, ci, v, X
    if dev == "cuda":
        torch.cuda.empty_cache()
    for _ in range(args.warmup):
        run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run()
    dt = (time.perf_counter() - t0) / args.steps
    free()
    value = nnz / dt
    unit = "edges/s"
    print(json.dumps({
        "impl": "reference", "metric": metric_name(args.workload), "value": value, "unit": unit,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": config_dict(args, n, nnz),
        "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": kind,
                         "sample": f"{args.steps} full Model::forward + log_softmax calls on the whole graph"
                                   + ("" if kind == "reference" else
                                      " through the C restatement of the reference (oracle/tg_oracle.c; the "
                                      "reference library is built only where its sources are)")},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))
    return 0


def metric_name(workload):
    return (f"{workload.upper()} forward edges/s (2-layer {FEATS}-{HIDDEN}-{CLASSES}, Reddit-shaped graph "
            f"{NODES} nodes / {EDGES} edges)")


def config_dict(args, n, nnz, exchange="nccl", peer_layers=()):
    if args.gpus > 1 and exchange == "peer":
        which = "every layer's" if all(peer_layers) else (
            "layer " + ", ".join(str(i + 1) for i, p in enumerate(peer_layers) if p) + "'s")
        partition = (f"1-D equal row blocks; {which} GEMM stores its output tiles into every GPU's gather "
                     "buffer over NVLink (peer memory) and signals per tile, each GPU waiting for its peers' tiles "
                     "on the device" + ("" if all(peer_layers) else "; the other layers exchange by one in-place "
                                        "NCCL all-gather") + "; then exact gather passes over column ranges")
    else:
        partition = None
    return {"workload": f"{args.workload}-reddit-shape" + ("-small" if args.small else ""),
            "nodes": n, "nnz": nnz, "features": FEATS, "hidden": HIDDEN, "classes": CLASSES,
            "partition": partition or "1-D equal row blocks; " + {
                "on": "each layer's transformed rows broadcast per rank block (NCCL, async), one exact gather "
                      "pass per arriving block",
                "off": "each layer's transformed rows exchanged by one in-place NCCL all-gather, then exact "
                       "gather passes over column ranges",
                "auto": "on 2-4 GPUs, layers whose exchanged operand is >= 64 MB broadcast per rank block "
                        "(NCCL, async) with one exact gather pass per arriving block; otherwise one in-place NCCL "
                        "all-gather, then exact gather passes over column ranges"}[args.pipeline],
            "parallelism": f"row-partition x{args.gpus}",
            "l2": "inputs larger than L2 (CSR 918 MB, features 561 MB); no flush between steps",
            "mode": ("fast: 3xTF32 tcgen05 GEMMs, order-preserving fp32 gathers" if args.mode == "fast"
                     else "exact: bit-identical FMA-chain GEMMs and gathers") +
                    ("" if args.workload == "gcn" else "; SAGE transform-first")}


# ── our arm ──────────────────────────────────────────────────────────────────
def run_ours(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        # rank 0's stdout carries exactly one JSON line: NCCL's own messages go to stderr
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)

    import tinygnn_b200 as tg
    from tinygnn_b200 import synth
    from tinygnn_b200.dist import Comm, ShardedModel, row_block, slice_rows
    from tinygnn_b200.ops import CSR

    comm = Comm(world, rank, group)
    n, rp, ci, v = make_graph(args.small, dev, args.edges)
    w = make_weights(args.workload, dev)
    bpr = args.blocks_per_rank if args.blocks_per_rank == "auto" else int(args.blocks_per_rank)
    passes = args.passes if args.passes == "auto" else int(args.passes)
    model = ShardedModel(layer_stack(args.workload, w), n, comm, dev, mode=args.mode, blocks_per_rank=bpr, passes=passes,
                         pipeline={"auto": "auto", "on": True, "off": False}[args.pipeline],
                         exchange=args.exchange.split(",") if "," in args.exchange else args.exchange)
    R, r0, r1 = model.R, model.row0, model.row1
    rows = r1 - r0
    A_raw = slice_rows(rp, ci, v, r0, r1, n)
    # The graph is checked once, as Tensor::sparse_csr checks it when the
    # caller builds it (src/tensor.cpp:46-86); Model::forward does not re-check.
    tg.csr_validate(A_raw)
    A_raw.validated = True
    # Feature rows live at a 16-byte row stride (602 -> 604 floats) so the
    # tensor-core GEMM can read them with TMA; the view is 602 wide.
    Xp = torch.zeros((rows, (FEATS + 3) // 4 * 4), dtype=torch.float32, device=dev)
    Xp[:, :FEATS] = synth.normal_rows(r0, rows, FEATS, FEAT_SEED, 0, dev)
    X = Xp[:, :FEATS]
    # edges of the normalised adjacency (GCN: A + I) this rank aggregates
    nnz_local = A_raw.nnz
    if args.workload == "gcn":
        lens = (A_raw.row_ptr[1:] - A_raw.row_ptr[:-1]).long()
        rows_of = torch.repeat_interleave(torch.arange(rows, device=dev), lens)
        has_diag = torch.zeros(rows, dtype=torch.bool, device=dev)
        has_diag[rows_of[A_raw.col_ind.long() == rows_of + r0]] = True
        nnz_local += int(rows - int(has_diag.sum()))
        del lens, rows_of, has_diag
    nnz_total = nnz_local
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([nnz_local], dtype=torch.int64, device=dev)
        dist.all_reduce(t)
        nnz_total = int(t.item())
    # keep the full graph only where the CPU baseline needs it
    want_cpu = rank == 0 and world == 1 and not args.no_cpu_baseline
    if not want_cpu:
        del rp, ci, v
    torch.cuda.synchronize()

    # roofline hook: CUDA events around the layer-1 gather of every step
    ev = {}  # (layer, phase) -> [start, end, start, end, ...] events

    def hook(li, what, edge):
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        ev.setdefault((li, what), []).append(e)

    dis_buf = torch.zeros(R * world, dtype=torch.float32, device=dev)

    def step():
        # What Model::forward does every call (src/model.cpp:359-439): the raw
        # adjacency is normalised (gcn_norm; in FAST mode as per-row scale
        # factors folded into the GEMM and gather epilogues) and scheduled
        # afresh, then the layers and log_softmax run.  Nothing derived from
        # the graph is kept between steps.
        Ar = CSR(A_raw.n_rows, A_raw.n_cols, A_raw.row_ptr, A_raw.col_ind, A_raw.values, validated=A_raw.validated)
        model.forward_model(Ar, X, dis_all=dis_buf)

    prepared = model.prepare(CSR(A_raw.n_rows, A_raw.n_cols, A_raw.row_ptr, A_raw.col_ind, A_raw.values,
                                 validated=A_raw.validated), dis_buf)

    def layers_step():
        # the layers alone on a graph normalised and scheduled once
        model.forward_prepared(prepared, X)

    sampler = ClockSampler(local)
    sampler.start()
    launches0 = tg.launches()
    model.timing = hook
    ms = time_steps(step, args.steps, args.warmup, world)
    model.timing = None
    launches = tg.launches() - launches0
    layers_ms = time_steps(layers_step, args.steps, min(args.warmup, 3), world)
    # Beside the step: the same step given the unweighted adjacency without
    # its values array (values=None: every entry 1.0).  The FAST gcn_norm
    # scale then takes each degree from row_ptr and the gathers read no
    # values; the logits are checked equal to the step's, bit for bit.
    unweighted = bool(torch.all(A_raw.values == 1.0).item())
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([1 if unweighted else 0], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        unweighted = bool(t.item())
    bare_info = None
    if unweighted and args.workload == "gcn" and args.mode == "fast":
        def bare_step():
            model.forward_model(CSR(A_raw.n_rows, A_raw.n_cols, A_raw.row_ptr, A_raw.col_ind, None,
                                    validated=A_raw.validated), X, dis_all=dis_buf)
        bare_ms = time_steps(bare_step, args.steps, min(args.warmup, 3), world)
        y_vals = model.forward_model(CSR(A_raw.n_rows, A_raw.n_cols, A_raw.row_ptr, A_raw.col_ind, A_raw.values,
                                         validated=A_raw.validated), X, dis_all=dis_buf).clone()
        y_bare = model.forward_model(CSR(A_raw.n_rows, A_raw.n_cols, A_raw.row_ptr, A_raw.col_ind, None,
                                         validated=A_raw.validated), X, dis_all=dis_buf)
        torch.cuda.synchronize()
        bare_info = {"ms_per_step": bare_ms / args.steps,
                     "logits_equal_bitwise": bool(torch.equal(y_bare, y_vals)),
                     "what": "the step on the unweighted adjacency given without its values array (values=None, "
                             "every entry 1.0): the FAST gcn_norm scale takes degrees from row_ptr, the gathers "
                             "read no values; TinyGNN's CSR stores the 1.0s, which the step above reads"}
        del y_vals
    def phase_ms(key):
        evs = ev.get(key, [])
        pairs = list(zip(evs[0::2], evs[1::2]))[-args.steps:]
        return statistics.mean(a.elapsed_time(b) for a, b in pairs) if pairs else None

    gather_ms = phase_ms((0, "gather"))
    phases = {f"layer{li}_{what}": phase_ms((li, what)) for li in range(2)
              for what in ("gemm", "exchange", "gather")}
    phases = {k: v for k, v in phases.items() if v is not None}
    rank_phases = [phases]
    if world > 1:  # every rank's phase times (the exchange absorbs imbalance)
        import torch.distributed as dist
        rank_phases = [None] * world
        dist.all_gather_object(rank_phases, phases)
    per_launch = launches / (args.steps + args.warmup)

    # e2e: host inputs -> device -> gcn_norm -> forward -> logits to host
    pin = lambda t: t.cpu().pin_memory()  # noqa: E731
    # An unweighted graph (every stored value 1.0, as Reddit's is) crosses as
    # its structure only; forward_from_host writes the 1.0s on the device.
    h_rp, h_ci, h_X = pin(A_raw.row_ptr), pin(A_raw.col_ind), pin(X)
    h_v = None if unweighted else pin(A_raw.values)
    h_out = torch.empty((rows, CLASSES), dtype=torch.float32).pin_memory()
    e2e_bufs = {}

    def e2e_sharded_step():
        # the row-partitioned Python API: this rank's host CSR rows + feature
        # rows in, host logits out, uploads pipelined with the compute
        model.forward_from_host(h_rp, h_ci, h_v, h_X, h_out, e2e_bufs)

    # At one GPU, e2e goes through the drop-in boundary a TinyGNN caller
    # binds: tg_model_forward_host (Model::forward from the pinned host CSR
    # arrays and features, the uploads overlapped with the compute, the
    # logits written to a pinned host buffer before it returns), every step.
    # Beside it, the same through the four separate handle calls
    # (tg_tensor_create_csr / _dense, tg_model_forward, tg_tensor_download),
    # each complete before it returns.
    hmodel = None
    h_Xc = None
    if world == 1 and not args.no_e2e:
        from tinygnn_b200.handles import HModel, HTensor, set_fast_math
        prev_fast = set_fast_math(args.mode == "fast")
        hmodel = HModel()
        for L in ref_spec(args.workload):
            if L["type"] == "gcn":
                hmodel.add_gcn(L["in"], L["out"], act=L.get("act"))
            else:
                hmodel.add_sage(L["in"], L["out"], act=L.get("act"))
        hmodel.load_weights({k: t.cpu().numpy() for k, t in w.items()})
        h_Xc = X.contiguous().cpu().pin_memory()  # rows of 602 floats, as a caller holds them
        h_out_api = torch.empty((rows, CLASSES), dtype=torch.float32).pin_memory()

        parts = {"upload_csr": 0.0, "upload_features": 0.0, "forward": 0.0, "download": 0.0, "free": 0.0}

        def e2e_step():
            hmodel.forward_host(h_rp, h_ci, h_v, h_Xc, FEATS, h_out_api, CLASSES)

        def e2e_calls_step():
            # each handle call completes before it returns: host timestamps time it
            t0 = time.perf_counter()
            A_t = HTensor.csr(n, n, h_rp, h_ci, h_v)
            t1 = time.perf_counter()
            X_t = HTensor.dense(h_Xc, n, FEATS)
            t2 = time.perf_counter()
            Y = hmodel.forward(A_t, X_t)
            Y.download(h_out_api)  # the forward's kernels finish inside this call
            t3 = time.perf_counter()
            for t in (Y, X_t, A_t):
                t.free()
            t4 = time.perf_counter()
            parts["upload_csr"] += t1 - t0
            parts["upload_features"] += t2 - t1
            parts["forward"] += t3 - t2
            parts["free"] += t4 - t3
    else:
        e2e_step = e2e_sharded_step

    e2e_ms = None if args.no_e2e else time_steps(e2e_step, args.steps, min(args.warmup, 3), world)
    host_api_out = None if hmodel is None else h_out_api.clone()
    e2e_parts = e2e_calls_ms = None
    if hmodel is not None:
        e2e_calls_ms = time_steps(e2e_calls_step, args.steps, min(args.warmup, 3), world)
        # per timed step (the warm-up steps are in the sums too)
        calls = args.steps + min(args.warmup, 3)
        e2e_parts = {k: v / calls * 1e3 for k, v in parts.items() if k != "download"}
        e2e_parts["forward+download"] = e2e_parts.pop("forward")
    e2e_sharded_ms = None
    if hmodel is not None:
        set_fast_math(prev_fast)
        e2e_sharded_ms = time_steps(e2e_sharded_step, args.steps, min(args.warmup, 3), world)
    clocks = sampler.stop()
    h2d = (h_rp.numel() + h_ci.numel()) * 4 + (0 if h_v is None else h_v.numel() * 4) + h_X.numel() * 4
    d2h = h_out.numel() * 4

    # parity spot check of the e2e logits against the device-resident run
    # (the ShardedModel path bit for bit; the handle path -- a different
    # kernel schedule for the same arithmetic -- within the fp32 tolerance)
    ref_out = model.forward_prepared(prepared, X)
    torch.cuda.synchronize()
    e2e_matches = None if args.no_e2e else bool(torch.equal(ref_out.cpu(), h_out))
    sharded_ms = e2e_sharded_ms if hmodel is not None else e2e_ms
    api_close = host_equals_calls = None
    if hmodel is not None:
        logits_ref = torch.log_softmax(ref_out.cpu().double(), 1)
        logits_api = torch.log_softmax(host_api_out.double(), 1)
        api_close = bool(((logits_api - logits_ref).abs() <= 1e-5 + 1e-4 * logits_ref.abs()).all())
        host_equals_calls = bool(torch.equal(host_api_out, h_out_api))  # h_out_api: the four-call path's
        hmodel.free()

    # roofline of the layer-1 gather (rank-local)
    F = HIDDEN
    alg_bytes = nnz_local * (8 + 4 * F) + rows * (4 + 4 * F) + 4
    if args.workload == "sage":
        alg_bytes = nnz_local * (4 + 4 * F) + rows * (4 + 8 * F) + 4  # no values; + self row
    alg_gbs = alg_bytes / (gather_ms * 1e-3) / 1e9
    peak, peak_kind = measured_peaks()
    traffic = committed_traffic(f"gather-{args.workload}-L1-{'small' if args.small else 'full'}-p{world}")
    l2_ceiling = committed_traffic("l2-random-gather-512B")
    # frac is the DRAM fraction: ncu's DRAM bytes per launch over this run's
    # launch time.  The no-reuse algorithmic model counts every gathered row
    # as a DRAM read although L2 serves most of them, so its "fraction" runs
    # above 1 (L2-assisted); it is reported beside, not as the fraction.
    dram_gbs = None if traffic is None else traffic / (gather_ms * 1e-3) / 1e9
    compulsory = (8 * nnz_local + 4 * (rows + 1) + 4 * n * HIDDEN + 4 * rows * HIDDEN)
    roof = {"kernel": "gather_rows + gather_heavy (layer-1 SpMM, F=128, fused bias+ReLU, column passes)",
            "bound": "hbm", "achieved": dram_gbs, "peak": peak, "unit": "GB/s",
            "frac": None if dram_gbs is None else dram_gbs / peak,
            "peak_source": (f"{peak_kind} HBM copy bandwidth (MEASURED_PEAKS.json)" if peak_kind == "measured"
                            else "fallback 6650 GB/s"),
            "traffic": traffic,
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum per launch (profiles/traffic.txt)",
            "ms_per_launch": gather_ms,
            "limiter": "L2 latency (long-scoreboard stalls; most gathered rows hit L2), not DRAM bandwidth",
            "algorithmic": {"label": "L2-assisted (algorithmic, no-reuse model nnz*(8+4F) + rows*(4+4F) + 4)",
                            "bytes_per_launch": alg_bytes, "achieved": alg_gbs, "frac_of_peak": alg_gbs / peak},
            "l2_bound": None if l2_ceiling is None else {
                "ceiling": l2_ceiling / 1e9, "unit": "GB/s", "frac": alg_gbs / (l2_ceiling / 1e9),
                "what": "the algorithmic bytes per launch against the rate the same kernel gathers uniformly random "
                        "512-byte rows from an L2-resident operand (bench.py --micro l2, profiles/traffic.txt)"},
            "compulsory_bytes_per_launch": compulsory}

    cpu = None
    if want_cpu:
        Xfull = X
        run, free = reference_forward_timer(args.workload, n, rp, ci, v, Xfull, w)
        if run is not None:
            kind, cores = cpu_impl()
            dt, reps = time_reference(run, args.cpu_seconds)
            free()
            cpu = {"value": nnz_total / dt, "unit": "edges/s", "cores": cores,
                   "kind": kind, "ms_per_forward": dt * 1e3,
                   "sample": f"median of {reps} full Model::forward + log_softmax calls (after 1 warm-up) on "
                             "the same graph"}
            run, free = reference_layers_timer(args.workload, n, rp, ci, v, Xfull, w)
            dt, reps = time_reference(run, args.cpu_seconds)
            free()
            cpu["layers_only"] = {
                "value": nnz_total / dt, "unit": "edges/s", "ms_per_forward": dt * 1e3,
                "sample": f"median of {reps} calls of the reference's layer objects + log_softmax on an "
                          "adjacency normalised once (Model::forward without its per-call gcn_norm)"}

    if rank == 0:
        value = nnz_total / (ms / args.steps * 1e-3)
        layers_value = nnz_total / (layers_ms / args.steps * 1e-3)
        e2e_val = None if e2e_ms is None else nnz_total / (e2e_ms / args.steps * 1e-3)
        line = {
            "metric": metric_name(args.workload), "value": value, "unit": "edges/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded Chung-Lu graph, N(0,1) features, Glorot weights, zero bias)",
            "config": config_dict(args, n, nnz_total, model.exchange_kind, model.peer_layers),
            "roofline": roof, "cpu_baseline": cpu,
            "e2e": {"value": e2e_val, "unit": "edges/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": None if e2e_ms is None else e2e_ms / args.steps,
                    "api": ("handle C ABI: tg_model_forward_host (Model::forward from pinned host CSR arrays + "
                            "features, uploads overlapped with the compute, gcn_norm inside, logits to a pinned host "
                            "buffer)"
                            if hmodel is not None else
                            "tinygnn_b200.dist.ShardedModel.forward_from_host: this rank's pinned host rows in, "
                            "host logits out"),
                    "log_softmax_within_tolerance_of_resident_run": api_close,
                    "equals_separate_calls": host_equals_calls,
                    "inputs": ("unweighted CSR: row_ptr + col_ind uploaded, values 1.0 written on the device"
                               if h_v is None else "CSR row_ptr + col_ind + values") + ", features fp32",
                    "note": "rank 0's bytes; every rank moves its own row block"},
            "e2e_separate_calls": None if e2e_calls_ms is None else {
                "value": nnz_total / (e2e_calls_ms / args.steps * 1e-3), "unit": "edges/s",
                "ms_per_step": e2e_calls_ms / args.steps, "call_ms": e2e_parts,
                "api": "tg_tensor_create_csr + tg_tensor_create_dense (pinned host buffers), tg_model_forward, "
                       "tg_tensor_download: four calls, each complete before it returns"},
            "e2e_sharded_pipelined": None if sharded_ms is None else {
                "value": nnz_total / (sharded_ms / args.steps * 1e-3), "unit": "edges/s",
                "ms_per_step": sharded_ms / args.steps, "logits_match_resident_run": e2e_matches,
                "api": "tinygnn_b200.dist.ShardedModel.forward_from_host (uploads overlapped with the compute)"},
            "step": ("Model::forward: gcn_norm of the raw adjacency, its row schedule, both layers, log_softmax"
                     if args.workload == "gcn" else
                     "Model::forward: the raw adjacency's row schedule, both layers, log_softmax"),
            "unweighted_csr": None if bare_info is None else dict(
                bare_info, value=nnz_total / (bare_info["ms_per_step"] * 1e-3), unit="edges/s"),
            "layers_only": {"value": layers_value, "unit": "edges/s", "ms_per_step": layers_ms / args.steps,
                            "what": "the layers + log_softmax on a graph normalised and scheduled once"},
            "clocks": clocks, "gpu_launches": int(per_launch * args.steps),
            "phase_ms": phases,
            "phase_ms_per_rank": rank_phases if world > 1 else None,
        }
        print(json.dumps(line))
    torch.cuda.synchronize()
    model.close()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_micro_hub(args):
    """One long row through the public spmm: the critical path the heavy-row
    kernel exists for (a Reddit-shaped hub has 13,531 entries).  Prints its
    own JSON line; not the benchmark contract's line."""
    import tinygnn_b200 as tg
    torch.cuda.set_device(0)
    rng = np.random.default_rng(1)
    n, F, reps = 240_000, args.micro_features, 20
    rp = np.zeros(n + 1, np.int32)
    rp[1:] = args.micro_entries  # row 0 holds every entry, the other rows are empty
    ci = np.sort(rng.choice(n, args.micro_entries, replace=False)).astype(np.int32)
    A = tg.CSR.from_numpy(rp, ci, np.ones(ci.size, np.float32)).with_degree_order()
    Fp = (F + 3) // 4 * 4
    B = torch.randn(n, Fp, device="cuda")[:, :F]
    out = torch.empty(n, F, device="cuda")
    for _ in range(3):
        tg.spmm(A, B, out=out)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        tg.spmm(A, B, out=out)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000 / reps
    print(json.dumps({"micro": "hub_row", "entries": args.micro_entries, "features": F, "us_per_call": us,
                      "ns_per_entry": us * 1000 / args.micro_entries,
                      "heavy_min_len": os.environ.get("TINYGNN_B200_HEAVY_MIN_LEN", "auto")}))
    tg.ops.take_device_error()
    return 0


def run_micro_l2(args):
    """The gather rate when every operand row hits in L2: 2^17 output rows of
    320 uniformly random entries each over an operand of 64 MB (under the
    126 MB L2), through the public spmm, for the two row widths the Reddit
    GCN gathers (128 and 41 features).  The bytes counted are the operand
    rows read (entries x features x 4); a gather whose operand spills to HBM
    cannot beat this rate.  Prints its own JSON lines."""
    import tinygnn_b200 as tg
    torch.cuda.set_device(0)
    rng = np.random.default_rng(2)
    rows, per_row, reps = 1 << 17, 320, 20
    for F in (128, 41):
        Fp = (F + 3) // 4 * 4
        n_cols = (64 << 20) // (Fp * 4)
        rp = np.arange(rows + 1, dtype=np.int64) * per_row
        # "uniform": random rows; "sequential": row i reads rows i*320 .. i*320+319
        # (mod n_cols) -- every 128-byte line of the operand used whole, the
        # L2 read rate with perfect locality
        for pattern in ("uniform", "sequential"):
            if pattern == "uniform":
                ci = np.sort(rng.integers(0, n_cols, (rows, per_row), dtype=np.int64), axis=1)
            else:
                ci = np.sort((np.arange(rows * per_row, dtype=np.int64) % n_cols).reshape(rows, per_row), axis=1)
            ci = ci.astype(np.int32).ravel()
            A = tg.CSR.from_numpy(rp.astype(np.int32), ci, np.ones(ci.size, np.float32), n_cols=n_cols)
            A = A.with_degree_order()
            B = torch.randn(n_cols, Fp, device="cuda")[:, :F]
            out = torch.empty(rows, F, device="cuda")
            ms = _gpu_ms(lambda: tg.spmm(A, B, out=out), reps=reps)
            nnz = rows * per_row
            print(json.dumps({"micro": "l2_gather", "pattern": pattern, "features": F,
                              "operand_mb": n_cols * Fp * 4 / 2**20, "entries": nnz, "ms_per_call": ms,
                              "operand_tb_s": nnz * F * 4 / (ms * 1e-3) / 1e12,
                              "with_indices_tb_s": nnz * (F * 4 + 8) / (ms * 1e-3) / 1e12}))
            del A, B, out
    tg.ops.take_device_error()
    return 0


# ── the other configurations (--suite) ──────────────────────────────────────
def _gpu_ms(fn, reps: int = 20, warm: int = 3) -> float:
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / reps


def _ref_model_runner(spec, weights, n, rp, ci, v, X):
    """The reference Model::forward + log_softmax on pre-built reference
    Tensors (through the C restatement where the reference library was not
    built)."""
    import oracle
    R = oracle.ref
    if R is None:
        P = oracle.port
        w = {k: np.asarray(t) for k, t in weights.items()}
        rp_h, ci_h, v_h, X_h = _host(rp, np.int32), _host(ci, np.int32), _host(v, np.float32), _host(X, np.float32)

        def run():
            P.activation("log_softmax", oracle.model_forward(P, spec, w, rp_h, ci_h, v_h, X_h))
        return run, lambda: None
    m = R.model(spec, {k: np.asarray(t) for k, t in weights.items()})
    rp_h = np.ascontiguousarray(rp.cpu().numpy(), dtype=np.int32)
    ci_h = np.ascontiguousarray(ci.cpu().numpy(), dtype=np.int32)
    v_h = np.ascontiguousarray(v.cpu().numpy(), dtype=np.float32)
    X_h = np.ascontiguousarray(X.cpu().numpy(), dtype=np.float32)
    A = R.lib.ref_tensor_csr(n, ci_h.size, rp_h.ctypes.data, ci_h.ctypes.data, v_h.ctypes.data)
    Xt = R.lib.ref_tensor_dense(X_h.shape[0], X_h.shape[1], X_h.ctypes.data)

    def run():
        R._chk(R.lib.ref_model_forward_tensors(m.h, A, Xt, None, 1))

    def free():
        R.lib.ref_tensor_free(A)
        R.lib.ref_tensor_free(Xt)

    return run, free


def run_suite(args):
    """One JSON line per benchmark configuration other than the headline one:
    the GPU time with inputs in HBM (CUDA events, warm; each call does what
    Model::forward does -- gcn_norm or self-loops, the layers, log_softmax)
    and the reference library's CPU time on the same inputs (median of up to
    5 calls after a warm-up, all host threads).  Synthetic seeded inputs of
    the configurations' shapes."""
    import oracle
    import tinygnn_b200 as tg
    from tinygnn_b200 import synth
    from tinygnn_b200.dist import Comm, Layer, ShardedModel
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    R = oracle.ref
    peak, _ = measured_peaks()
    h = lambda t: t.detach().cpu().numpy()  # noqa: E731

    kind, cores = cpu_impl()

    def emit(line, run=None, free=None):
        if run is not None:
            dt, reps = time_reference(run, args.cpu_seconds)
            free()
            line["cpu_ms"] = dt * 1e3
            line["cpu_cores"] = cores
            line["cpu_kind"] = kind
            line["speedup"] = line["cpu_ms"] / line["gpu_ms"]
        print(json.dumps(line), flush=True)

    # 1. Cora-shaped GCN 1433 -> 16 -> 7
    n, rp, ci, v, X = synth.cora_like(device=dev)
    W0, W1 = synth.glorot(1433, 16, 2, 1, dev), synth.glorot(16, 7, 2, 2, dev)
    b0, b1 = torch.zeros(16, device=dev), torch.zeros(7, device=dev)
    A = tg.CSR(n, n, rp, ci, v)
    tg.csr_validate(A)
    A.validated = True
    # Model::forward as the headline bench runs it (FAST: gcn_norm as a per-row
    # scale of the raw adjacency, both layers, log_softmax), per call
    cora_model = ShardedModel([Layer("gcn", W0, b0, "relu"), Layer("gcn", W1, b1, None)], n, Comm(1, 0), dev,
                              mode="fast")
    Xp = torch.zeros((n, 1436), dtype=torch.float32, device=dev)
    Xp[:, :1433] = X

    def cora():
        cora_model.forward_model(tg.CSR(n, n, rp, ci, v, validated=True), Xp[:, :1433])
    ms = _gpu_ms(cora, reps=200, warm=10)
    spec = [dict(type="gcn", **{"in": 1433, "out": 16}, act="relu"), dict(type="gcn", **{"in": 16, "out": 7})]
    w = {"layer0.weight": h(W0), "layer0.bias": h(b0), "layer1.weight": h(W1), "layer1.bias": h(b1)}
    # The same forward recorded once as a CUDA graph (tg_model_capture, FAST)
    # and replayed: one graph launch instead of ~20 kernel launches; each
    # tg_graph_replay call returns when the forward has finished.
    from tinygnn_b200.handles import HModel, HTensor, set_fast_math
    prev_fast = set_fast_math(True)
    hm = HModel().add_gcn(1433, 16, act="relu").add_gcn(16, 7, act=None)
    hm.load_weights(w)
    At = HTensor.csr(n, n, h(rp).astype(np.int32), h(ci).astype(np.int32), h(v).astype(np.float32))
    Xt = HTensor.dense(np.ascontiguousarray(h(X), dtype=np.float32), n, 1433)
    graph = hm.capture(At, Xt)
    for _ in range(10):
        graph.replay()
    reps = 500
    t0 = time.perf_counter()
    for _ in range(reps):
        graph.replay()
    graph_ms = (time.perf_counter() - t0) / reps * 1e3
    graph.free()
    hm.free()
    set_fast_math(prev_fast)
    emit({"suite": "gcn-cora-shape", "nodes": n, "nnz_norm": int(tg.gcn_norm(A).nnz), "gpu_ms": ms,
          "gpu_ms_graph_replay": graph_ms,
          "graph_replay": "Model::forward (FAST gcn_norm scale, both layers) recorded by tg_model_capture, "
                          "host-timed synchronous tg_graph_replay calls (launch + run + wait)"},
         *_ref_model_runner(spec, w, n, rp, ci, v, X))

    # 2. spmm, R-MAT 2^20 / 2^24 draws, values U(0,1], F in {16, 64, 128, 256}
    n, rp, ci, v = synth.rmat_csr(20, 1 << 24, 3, device=dev, values_seed=3)
    A = tg.CSR(n, n, rp, ci, v).with_degree_order()
    nnz = int(ci.numel())
    for F in (16, 64, 128, 256):
        B = synth.normal_rows(0, n, F, 4, 0, dev)
        out = torch.empty((n, F), device=dev)
        ms = _gpu_ms(lambda: tg.spmm(A, B, out=out))
        alg = nnz * (8 + 4 * F) + n * (4 + 4 * F)
        line = {"suite": "spmm-rmat-2^20", "F": F, "nnz": nnz, "gpu_ms": ms, "edges_per_s": nnz / (ms * 1e-3),
                "alg_GBps": alg / (ms * 1e-3) / 1e9, "hbm_frac_of_measured": alg / (ms * 1e-3) / 1e9 / peak}
        run = free = None
        if R is None:
            rp_h, ci_h, v_h, Bh = (np.ascontiguousarray(h(t)) for t in (rp, ci, v, B))

            def run(rp_h=rp_h, ci_h=ci_h, v_h=v_h, Bh=Bh):
                oracle.port.spmm(rp_h, ci_h, v_h, Bh)
            free = lambda: None  # noqa: E731
        else:
            rp_h, ci_h, v_h, Bh = (np.ascontiguousarray(h(t)) for t in (rp, ci, v, B))  # alive across the calls
            At = R.lib.ref_tensor_csr(n, nnz, rp_h.ctypes.data, ci_h.ctypes.data, v_h.ctypes.data)
            Bt = R.lib.ref_tensor_dense(n, F, Bh.ctypes.data)
            del rp_h, ci_h, v_h, Bh  # the reference Tensors hold their own copies

            def run(At=At, Bt=Bt):
                R._chk(R.lib.ref_spmm_tensors(At, Bt, None))

            def free(At=At, Bt=Bt):
                R.lib.ref_tensor_free(At)
                R.lib.ref_tensor_free(Bt)
        emit(line, run, free)
        del B, out

    # 3. SAGE-mean 128 -> 128 -> 40 on a symmetrised R-MAT 2^18
    n, rp, ci, v = synth.rmat_csr(18, 5_242_880, 5, device=dev, symmetric=True, no_self=True)
    X = synth.normal_rows(0, n, 128, 6, 0, dev)
    Wn1, Ws1 = synth.glorot(128, 128, 6, 1, dev), synth.glorot(128, 128, 6, 2, dev)
    Wn2, Ws2 = synth.glorot(128, 40, 6, 3, dev), synth.glorot(128, 40, 6, 4, dev)
    b1, b2 = torch.zeros(128, device=dev), torch.zeros(40, device=dev)
    model = ShardedModel([Layer("sage", Wn1, b1, "relu", Ws1), Layer("sage", Wn2, b2, None, Ws2)], n,
                         Comm(1, 0), dev, mode="fast")
    A = tg.CSR(n, n, rp, ci, v).with_degree_order()
    ms = _gpu_ms(lambda: model.forward(None, A, X))
    spec = [dict(type="sage", **{"in": 128, "out": 128}, act="relu"), dict(type="sage", **{"in": 128, "out": 40})]
    w = {"layer0.weight_neigh": h(Wn1), "layer0.weight_self": h(Ws1), "layer0.bias": h(b1),
         "layer1.weight_neigh": h(Wn2), "layer1.weight_self": h(Ws2), "layer1.bias": h(b2)}
    emit({"suite": "sage-rmat-2^18", "nodes": n, "nnz": int(ci.numel()), "gpu_ms": ms,
          "edges_per_s": int(ci.numel()) / (ms * 1e-3)},
         *_ref_model_runner(spec, w, n, rp, ci, v, X))
    del model

    # 4. GAT 256 -> 8 heads x 8 (concat, ELU) -> 16 on an R-MAT 2^20 stored incoming, self-loops per call
    n, rp, ci, v = synth.rmat_csr(20, 1 << 24, 7, device=dev, transpose=True)
    X = synth.normal_rows(0, n, 256, 8, 0, dev)
    heads, d = 8, 8
    Wh = [synth.glorot(256, d, 8, 10 + k, dev) for k in range(heads)]
    al = [synth.glorot(d, 1, 8, 30 + k, dev).flatten() for k in range(heads)]
    ar = [synth.glorot(d, 1, 8, 50 + k, dev).flatten() for k in range(heads)]
    W2 = synth.glorot(64, 16, 8, 70, dev)
    al2, ar2 = synth.glorot(16, 1, 8, 71, dev).flatten(), synth.glorot(16, 1, 8, 72, dev).flatten()
    W, AL, AR = torch.cat(Wh, 1), torch.stack(al), torch.stack(ar)
    z1, z2 = torch.zeros((heads, d), device=dev), torch.zeros((1, 16), device=dev)
    A = tg.CSR(n, n, rp, ci, v)

    def gat():
        Asl = tg.add_self_loops(A)
        H = tg.gat_layer(Asl, X, W, AL, AR, heads, z1, 0.2, True, None, mode="fast")
        tg.elu_(H)
        tg.log_softmax_(tg.gat_layer(Asl, H, W2, al2.reshape(1, -1), ar2.reshape(1, -1), 1, z2, 0.2, True, None,
                                     mode="fast"))
    ms = _gpu_ms(gat, reps=10)
    spec = [dict(type="gat", **{"in": 256, "out": d}, heads=heads, concat=True, post="elu"),
            dict(type="gat", **{"in": 64, "out": 16}, heads=1)]
    w = {}
    for k in range(heads):
        w[f"layer0.head{k}.weight"], w[f"layer0.head{k}.attn_left"] = h(Wh[k]), h(al[k])
        w[f"layer0.head{k}.attn_right"], w[f"layer0.head{k}.bias"] = h(ar[k]), np.zeros(d, np.float32)
    w.update({"layer1.head0.weight": h(W2), "layer1.head0.attn_left": h(al2), "layer1.head0.attn_right": h(ar2),
              "layer1.head0.bias": np.zeros(16, np.float32)})
    emit({"suite": "gat-rmat-2^20", "nodes": n, "nnz": int(ci.numel()), "gpu_ms": ms,
          "edges_per_s": int(ci.numel()) / (ms * 1e-3)},
         *_ref_model_runner(spec, w, n, rp, ci, v, X))


def main():
    args = parse()
    if args.suite:
        return run_suite(args)
    if args.micro == "hub":
        return run_micro_hub(args)
    if args.micro == "l2":
        return run_micro_l2(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
