"""Row-partitioned GCN / SAGE forward over several GPUs (one process per GPU).

Partitioning (1-D, by rows): with P ranks and N nodes, rank r owns global
rows [r*R, min(N, (r+1)*R)) where R = ceil(N/P) (rounded up to a multiple of
the column blocks per rank) -- its rows of the adjacency (global column ids)
and of the features.  Each layer's transformed rows are exchanged into a
(P*R) x F buffer whose row j is global node j, so gathers index it with the
global column ids directly (no remapping).  Hubs are never split across
ranks.

Per GCN layer on rank r (src/layers.cpp:286-339 per block of rows):
  1. HW[rR : rR + rows] = H_r . W          (this rank's rows)
  2. exchange HW over the ranks             (NCCL via torch.distributed)
  3. H'_r = act(A_norm[r-rows] . HW + b)    (gather, fused epilogue)
Step 2-3 run as column-block passes: every rank's block is broadcast
asynchronously, and the gather runs one pass per block in increasing column
order (tg_spmm_segment_f32), starting as soon as that block has arrived.
The passes carry each output element's FMA chain through the output, so the
result is bit-identical to the one-pass gather -- and to one GPU -- while
the transfer of block q+1 overlaps the pass over block q, and each pass
reads only one block of the gathered operand (an L2-sized working set).

gcn_norm of a row block (src/layers.cpp:158-208): self-loops and degrees are
row-local; the column scale needs every node's 1/sqrt(deg), which one
all-gather of the degree vector provides -- bit-identical to the
single-GPU gcn_norm.

SAGE (transform-first, mean): Tn_r = H_r . W_neigh is exchanged,
Ts_r = H_r . W_self stays local, H'_r = act(mean_j Tn[j] + Ts_r[i] + b).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from . import ops
from .ops import CSR


def row_block(n: int, world: int, rank: int, multiple: int = 1) -> Tuple[int, int, int]:
    """(R, row0, row1): the equal-size row block of ``rank`` (R a multiple of ``multiple``)."""
    R = (n + world - 1) // world
    R = (R + multiple - 1) // multiple * multiple
    r0 = min(n, rank * R)
    return R, r0, min(n, r0 + R)


def slice_rows(row_ptr: torch.Tensor, col_ind: torch.Tensor, values: torch.Tensor, r0: int, r1: int,
               n_cols: int) -> CSR:
    """Rows [r0, r1) of a CSR as a CSR with rebased row_ptr (same device)."""
    a = int(row_ptr[r0])
    b = int(row_ptr[r1])
    rp = (row_ptr[r0:r1 + 1] - a).to(torch.int32).contiguous()
    return CSR(r1 - r0, n_cols, rp, col_ind[a:b].contiguous(), values[a:b].contiguous())


def _pad4(n: int) -> int:
    return (n + 3) // 4 * 4


class Comm:
    """The exchange steps (NCCL through torch.distributed); nothing at P = 1."""

    def __init__(self, world: int, rank: int, group=None):
        self.world, self.rank, self.group = world, rank, group

    def all_gather_rows(self, full: torch.Tensor, R: int) -> None:
        """In-place all-gather: rank r's rows [rR, rR+R) of ``full`` go to every rank."""
        if self.world == 1:
            return
        mine = full[self.rank * R:(self.rank + 1) * R]
        dist.all_gather_into_tensor(full, mine, group=self.group)

    def broadcast_rows(self, full: torch.Tensor, R: int, src: int):
        """Start sending rank ``src``'s rows of ``full`` to every rank; returns a waitable."""
        if self.world == 1:
            return None
        return dist.broadcast(full[src * R:(src + 1) * R], src=src, group=self.group, async_op=True)

    def all_gather_object(self, obj) -> list:
        out = [None] * self.world
        dist.all_gather_object(out, obj, group=self.group)
        return out

    def barrier(self) -> None:
        dist.barrier(group=self.group)

    @property
    def distributed(self) -> bool:
        return self.world > 1 and dist.is_available() and dist.is_initialized()


class PeerExchange:
    """Exchange memory shared over NVLink by the ranks of a ShardedModel.

    One allocation per rank holds, per layer, two gather buffers
    ((P*R) x pad4(F_out); a layer's forward uses buffer epoch % 2) and a
    (layers x P) table of 64-bit completion counters: counter [l, q] counts
    the 128-row tiles of layer l that rank q has stored here.  Every rank maps
    every other rank's allocation (CUDA IPC), so the fused GEMM stores its
    tiles into all copies and bumps its counter in each.  Two buffers per
    layer are enough without a "consumed" handshake: a rank writes epoch e+1
    into a buffer that its peers last read at epoch e-1, and none of them can
    still be there -- the writer finished epoch e's gather, which waited for
    every peer's epoch-e tiles, which each peer stored after its epoch e-1
    gather.
    """

    TILE = 128  # rows per GEMM tile (one counter increment)
    ALIGN = 256

    def __init__(self, comm: "Comm", R: int, widths: List[int], device):
        self.comm, self.R, self.widths = comm, R, widths
        P = comm.world
        off, self.buf_off = 0, []
        for w in widths:
            pair = []
            for _ in range(2):
                pair.append(off)
                off += -(-P * R * w * 4 // self.ALIGN) * self.ALIGN
            self.buf_off.append(pair)
        self.cnt_off = off
        off += -(-len(widths) * P * 8 // self.ALIGN) * self.ALIGN
        self.blob = torch.zeros(off, dtype=torch.uint8, device=device)
        self.bufs = [[self.blob[o:o + P * R * w * 4].view(torch.float32).view(P * R, w) for o in pair]
                     for pair, w in zip(self.buf_off, widths)]
        self.counters = self.blob[self.cnt_off:self.cnt_off + len(widths) * P * 8].view(torch.int64).view(
            len(widths), P)
        torch.cuda.synchronize()  # zeroed before any peer may write here
        handle, offset = ops.ipc_get_handle(self.blob)
        table = comm.all_gather_object((handle, offset))
        self.opened, self.peer_base = [], {}
        for q, (h, o) in enumerate(table):
            if q == comm.rank:
                continue
            base = ops.ipc_open_handle(h)
            self.opened.append(base)
            self.peer_base[q] = base + o
        comm.barrier()
        self.epoch = [0] * len(widths)
        self.peers = [q for q in range(P) if q != comm.rank]
        self.tiles = [0] * P

    def set_rows(self, n: int) -> None:
        """Tiles each rank stores per layer, from the global node count."""
        P, R = self.comm.world, self.R
        self.tiles = [-(-max(0, min(R, n - q * R)) // self.TILE) for q in range(P)]

    def next_epoch(self, li: int) -> torch.Tensor:
        """Start layer li's next forward: its gather buffer (this epoch's parity)."""
        self.epoch[li] += 1
        return self.bufs[li][self.epoch[li] % 2]

    def peer_targets(self, li: int, row_off_floats: int):
        """(peer output addresses, peer counter addresses) for layer li's current buffer."""
        par = self.epoch[li] % 2
        P, me = self.comm.world, self.comm.rank
        outs = [self.peer_base[q] + self.buf_off[li][par] + row_off_floats * 4 for q in self.peers]
        flags = [self.peer_base[q] + self.cnt_off + (li * P + me) * 8 for q in self.peers]
        return outs, flags

    def wait(self, li: int) -> None:
        """In stream order: every peer's tiles of layer li's current epoch have landed here."""
        e = self.epoch[li]
        targets = [0 if q == self.comm.rank else self.tiles[q] * e for q in range(self.comm.world)]
        ops.wait_flags(self.counters[li], targets)

    def close(self) -> None:
        for base in self.opened:
            ops.ipc_close_handle(base)
        self.opened = []


def gcn_norm_rows(A: CSR, row0: int, R: int, comm: Comm, dis_all: Optional[torch.Tensor] = None) -> CSR:
    """gcn_norm of this rank's row block (global columns), bit-identical to the
    rows of the single-GPU gcn_norm: one pass for the self-looped row lengths
    and 1/sqrt(deg), the all-gather of 1/sqrt(deg), one pass writing the
    scaled self-looped rows."""
    if dis_all is None:
        dis_all = torch.zeros(R * comm.world, dtype=torch.float32, device=A.row_ptr.device)
    mine = dis_all[comm.rank * R:comm.rank * R + A.n_rows]
    rp, ins = ops.gcn_norm_rows_degrees(A, row0, mine)
    comm.all_gather_rows(dis_all.view(-1, 1), R)
    return ops.gcn_norm_rows_fill(A, row0, rp, ins, mine, dis_all)


def gcn_norm_rows_scheduled(A: CSR, row0: int, R: int, comm: Comm, dis_all: Optional[torch.Tensor] = None) -> CSR:
    """gcn_norm_rows with the raw rows' longest-first schedule computed once:
    both normalisation passes run in it, and the normalised block keeps it
    for the gathers (same arithmetic; the order changes speed only)."""
    if A.order is None:
        A = CSR(A.n_rows, A.n_cols, A.row_ptr, A.col_ind, A.values, ops.degree_order(A), A.validated)
    return gcn_norm_rows(A, row0, R, comm, dis_all)


@dataclass
class Layer:
    kind: str                      # "gcn" or "sage"
    W: torch.Tensor                # gcn: F_in x F_out; sage: W_neigh
    b: Optional[torch.Tensor]
    act: Optional[str]
    W_self: Optional[torch.Tensor] = None


class ShardedModel:
    """A stack of GCN / SAGE-mean layers over a row-partitioned graph.

    ``forward`` takes this rank's normalised (GCN) or raw (SAGE) adjacency
    rows and feature rows, already in HBM; buffers are allocated once.
    ``blocks_per_rank`` > 1 splits every rank's columns into that many
    column blocks (extra passes that each gather from a smaller working set).
    """

    # A rank's block of a gathered operand above this size is split into
    # column blocks (measured on B200: 2 blocks for the 119 MB F=128 operand
    # -6% time, more blocks or smaller operands slower).
    BLOCK_BYTES = 64 << 20

    def __init__(self, layers: List[Layer], n: int, comm: Comm, device, mode: str = "exact",
                 blocks_per_rank="auto", pipeline="auto", passes="auto", exchange="auto"):
        self.layers, self.n, self.comm, self.device, self.mode = layers, n, comm, device, mode
        # exchange: "peer" = the GEMM stores its tiles straight into every
        # rank's gather buffer over NVLink (PeerExchange; FAST mode, the
        # tensor-core GEMM); "nccl" = GEMM, then an NCCL all-gather or
        # broadcasts.  "auto" = peer when FAST under a real process group,
        # except, on 8+ ranks, for operands under BLOCK_BYTES.  Measured on
        # B200 (GCN, Reddit-shaped; forward, peer vs NCCL): P = 2 3.37 vs
        # 3.42 ms, P = 4 2.08 vs 2.20 ms, P = 8 1.443 vs 1.440 ms -- at P = 8
        # the 119 MB layer-1 exchange is faster fused (GEMM + exchange 0.29
        # vs 0.32 ms) and the 41 MB layer-2 one slower (0.16 vs 0.13 ms).
        # A list gives each layer's exchange ("peer" / "nccl").
        if isinstance(exchange, (list, tuple)):
            if len(exchange) != len(layers) or any(x not in ("peer", "nccl") for x in exchange):
                raise ValueError(f"exchange: one of 'peer' / 'nccl' per layer, got {exchange!r}")
            peer_layers = [x == "peer" for x in exchange]
            exchange = "peer" if any(peer_layers) else "nccl"
        elif exchange == "auto":
            exchange = ("peer" if mode == "fast" and getattr(comm, "distributed", False)
                        and all(L.W.shape[1] <= 256 for L in layers) else "nccl")
            peer_layers = [exchange == "peer" and (comm.world < 8 or n * _pad4(L.W.shape[1]) * 4 >= self.BLOCK_BYTES)
                           for L in layers]
        elif exchange in ("peer", "nccl"):
            peer_layers = [exchange == "peer"] * len(layers)
        else:
            raise ValueError(f"exchange: 'auto', 'peer', 'nccl' or one of the last two per layer, got {exchange!r}")
        if exchange == "peer" and mode != "fast":
            raise ValueError("exchange='peer' runs the tensor-core GEMM: mode must be 'fast'")
        self.exchange_kind = exchange
        self.peer_layers = peer_layers
        if exchange == "peer":
            pipeline = False
        # pipeline: per-rank async broadcasts with one gather pass per arriving
        # column block (blocks_per_rank blocks per rank); otherwise one
        # all-gather, then `passes` column passes over the whole operand.
        # "auto" pipelines, on 2-4 ranks, the layers whose exchanged operand
        # is at least BLOCK_BYTES.  Measured on B200 (GCN, Reddit-shaped):
        # P = 2 forward 3.52 -> 3.34 ms; P = 4 layer 1 (exchange + gather)
        # 1.25 -> 1.19 ms but the 41 MB layer 2 0.62 -> 0.72 ms; P = 8 layer
        # 1 0.82 -> 1.09 ms (eight serial broadcasts and eight passes).  P
        # broadcasts move less than one all-gather, which pays only where the
        # passes they overlap are long.
        if pipeline == "auto":
            self.pipe = [2 <= comm.world <= 4 and n * _pad4(L.W.shape[1]) * 4 >= self.BLOCK_BYTES for L in layers]
        else:
            self.pipe = [bool(pipeline)] * len(layers)
        self.pipeline = any(self.pipe)
        R0 = (n + comm.world - 1) // comm.world
        if blocks_per_rank == "auto":
            self.bprs = [max(1, -(-(R0 * _pad4(L.W.shape[1]) * 4) // self.BLOCK_BYTES)) for L in layers]
        else:
            self.bprs = [max(1, int(blocks_per_rank))] * len(layers)
        if passes == "auto":
            self.passes = [max(1, -(-(n * _pad4(L.W.shape[1]) * 4) // self.BLOCK_BYTES)) for L in layers]
        else:
            self.passes = [max(1, int(passes))] * len(layers)
        multiple = 1
        if self.pipeline:  # rank blocks split evenly into column blocks
            for b in self.bprs:
                multiple = multiple * b // math.gcd(multiple, b)
        self.R, self.row0, self.row1 = row_block(n, comm.world, comm.rank, multiple)
        self.rows = self.row1 - self.row0
        P = comm.world
        self.pex = None
        if exchange == "peer":
            self.pex = PeerExchange(comm, self.R, [_pad4(L.W.shape[1]) for L in layers], device)
            self.pex.set_rows(n)
        self.hpad = [None] * len(layers)  # 16-byte-aligned copies of unaligned layer inputs (peer exchange)
        self.full = []   # gathered operand per layer: (P*R) x pad4(F_out)
        self.outs = []
        self.selfs = []
        for li, L in enumerate(layers):
            fo = L.W.shape[1]
            self.full.append(self.pex.bufs[li][0] if self.pex else
                             torch.zeros((P * self.R, _pad4(fo)), dtype=torch.float32, device=device))
            self.outs.append(torch.empty((self.rows, fo), dtype=torch.float32, device=device))
            self.selfs.append(torch.empty((self.rows, _pad4(fo)), dtype=torch.float32, device=device)
                              if L.kind == "sage" else None)
        self.timing = None  # optional hook: (layer index, phase, "start"|"end") -> None
        # FAST GCN without a normalised copy of A: this rank's 1/sqrt(deg)
        # while a forward runs (set by forward_model / forward_from_host).
        self.scale: Optional[torch.Tensor] = None
        self.scale_buf = torch.empty(max(self.rows, 1), dtype=torch.float32, device=device)
        self._prep_stream = None  # _normalise's side stream (schedule, split points)
        self._prep_ready = None   # its completion, joined by the first gather
        self._order_buf = None    # the schedule of the rows, rewritten every forward
        self._split_bufs = {}     # column-pass split points by pass count

    def _scaled(self, li: int) -> bool:
        """Layer li is a GCN layer run in the factored FAST form."""
        return self.scale is not None and self.layers[li].kind == "gcn"

    def _self_rows(self, li: int, a: int = 0, b: Optional[int] = None) -> torch.Tensor:
        """This rank's rows [a, b) of layer li's gathered operand."""
        fo = self.layers[li].W.shape[1]
        r0 = self.comm.rank * self.R
        return self.full[li][r0 + a:r0 + (self.rows if b is None else b), :fo]

    def _mark(self, li: int, what: str, edge: str) -> None:
        if self.timing is not None:
            self.timing(li, what, edge)

    @staticmethod
    def _cached_splits(A: CSR, nblocks: int, width: int) -> torch.Tensor:
        cache = getattr(A, "_splits", None)
        if cache is None:
            cache = A._splits = {}
        key = (nblocks, width)
        if key not in cache:
            cache[key] = ops.column_splits(A, nblocks, width)
        return cache[key]

    def splits(self, A: CSR, bpr: int) -> Optional[torch.Tensor]:
        """Split points of A's rows into `bpr` column blocks per rank (pipelined exchange; cached on A)."""
        nblocks = self.comm.world * bpr
        if nblocks == 1:
            return None
        return self._cached_splits(A, nblocks, self.R // bpr)

    def pass_splits(self, A: CSR, passes: int) -> Optional[torch.Tensor]:
        """Split points of A's rows into `passes` equal column ranges of the whole operand (cached on A)."""
        if passes == 1:
            return None
        return self._cached_splits(A, passes, -(-self.n // passes))

    # The phases of a layer; forward() runs them in order.  Tests that
    # emulate several ranks in one process interleave them across shards.
    def transform(self, li: int, H: torch.Tensor) -> None:
        """This rank's rows of H . W (and H . W_self for SAGE) into the gather buffer."""
        L = self.layers[li]
        fo = L.W.shape[1]
        r = self.comm.rank
        self._mark(li, "gemm", "start")
        if self.pex is not None and self.peer_layers[li]:
            self.full[li] = buf = self.pex.next_epoch(li)
            if H.stride(1) != 1 or H.stride(0) % 4 or H.data_ptr() % 16:
                # the tensor-core GEMM reads H with TMA: 16-byte aligned rows
                if self.hpad[li] is None or self.hpad[li].shape[0] != H.shape[0]:
                    self.hpad[li] = torch.zeros((H.shape[0], _pad4(H.shape[1])), dtype=torch.float32,
                                                device=H.device)
                self.hpad[li][:, :H.shape[1]] = H
                H = self.hpad[li][:, :H.shape[1]]
            outs, flags = self.pex.peer_targets(li, r * self.R * buf.shape[1])
            ops.gemm_peers(H, L.W, buf[r * self.R:r * self.R + self.rows, :fo], outs, flags, cols_padded=True,
                           row_scale=self.scale if self._scaled(li) else None)
        elif L.kind == "sage":  # W_neigh and W_self in one pass over H (FAST: one tensor-core GEMM)
            ops.gemm_pair(H, L.W, L.W_self, self.full[li][r * self.R:r * self.R + self.rows, :fo],
                          self.selfs[li][:, :fo], mode=self.mode, cols_padded=True)
        else:  # the gather buffer's rows are padded to 16 bytes
            ops.matmul(H, L.W, out=self.full[li][r * self.R:r * self.R + self.rows, :fo], mode=self.mode,
                       row_scale=self.scale if self._scaled(li) else None, cols_padded=True)
        if L.kind == "sage" and self.pex is not None and self.peer_layers[li]:
            ops.matmul(H, L.W_self, out=self.selfs[li][:, :fo], mode=self.mode, cols_padded=True)
        self._mark(li, "gemm", "end")

    def exchange(self, li: int) -> None:
        """Every rank's rows into this rank's gather buffer: the wait for the
        peers' tiles (peer exchange) or an NCCL all-gather."""
        self._mark(li, "exchange", "start")
        if self.pex is not None and self.peer_layers[li]:
            self.pex.wait(li)
        else:
            self.comm.all_gather_rows(self.full[li], self.R)
        self._mark(li, "exchange", "end")

    def close(self) -> None:
        """Unmap the peers' exchange memory (call before the process group ends)."""
        if self.pex is not None:
            self.pex.close()

    def _pass(self, li: int, A: CSR, lo, hi, carry: bool, last: bool) -> torch.Tensor:
        self._join_prep()
        L = self.layers[li]
        fo = L.W.shape[1]
        B = self.full[li][:self.n, :fo]
        if self._scaled(li):
            return ops.gcn_aggregate(A, B, self._self_rows(li), self.scale, bias=L.b, act=L.act, out=self.outs[li],
                                     seg_begin=lo, seg_end=hi, carry=carry, last=last)
        if L.kind == "gcn":
            if lo is None:
                return ops.spmm(A, B, bias=L.b, act=L.act, out=self.outs[li])
            return ops.spmm_segment(A, B, lo, hi, self.outs[li], carry, last, bias=L.b, act=L.act)
        if lo is None:
            return ops.sage_mean_combine(A, B, self.selfs[li][:, :fo], bias=L.b, act=L.act, out=self.outs[li])
        return ops.sage_mean_combine_segment(A, B, self.selfs[li][:, :fo], lo, hi, self.outs[li], carry, last,
                                             bias=L.b, act=L.act)

    def _join_prep(self) -> None:
        """The current stream waits for _normalise's side-stream work (once)."""
        if self._prep_ready is not None:
            torch.cuda.current_stream().wait_event(self._prep_ready)
            self._prep_ready = None

    def aggregate(self, li: int, A_gcn: Optional[CSR], A_raw: Optional[CSR]) -> torch.Tensor:
        """Single pass over the whole (already exchanged) operand."""
        A = A_gcn if self.layers[li].kind == "gcn" else A_raw
        self._mark(li, "gather", "start")
        H = self._pass(li, A, None, None, False, True)
        self._mark(li, "gather", "end")
        return H

    def exchange_and_aggregate(self, li: int, A_gcn: Optional[CSR], A_raw: Optional[CSR]) -> torch.Tensor:
        """The exchange, then the gather: passes over column ranges in increasing
        order (one all-gather first), or -- pipelined -- one pass per rank block
        as soon as that block has arrived."""
        A = A_gcn if self.layers[li].kind == "gcn" else A_raw
        if not self.pipe[li]:
            self.exchange(li)
            sp = self.pass_splits(A, self.passes[li])
            if sp is None:
                return self.aggregate(li, A_gcn, A_raw)
            self._mark(li, "gather", "start")
            nb = self.passes[li]
            for q in range(nb):
                H = self._pass(li, A, sp[q], sp[q + 1], q > 0, q == nb - 1)
            self._mark(li, "gather", "end")
            return H
        bpr = self.bprs[li]
        sp = self.splits(A, bpr)
        if sp is None:
            self.exchange(li)
            return self.aggregate(li, A_gcn, A_raw)
        nblocks = self.comm.world * bpr
        self._mark(li, "gather", "start")
        works = [self.comm.broadcast_rows(self.full[li], self.R, src) for src in range(self.comm.world)]
        H = None
        for q in range(nblocks):
            src = q // bpr
            if works[src] is not None and src != self.comm.rank:
                works[src].wait()
                works[src] = None
            H = self._pass(li, A, sp[q], sp[q + 1], q > 0, q == nblocks - 1)
        for w in works:
            if w is not None:
                w.wait()
        self._mark(li, "gather", "end")
        return H

    def forward_from_host(self, h_rp: torch.Tensor, h_ci: torch.Tensor, h_v: Optional[torch.Tensor],
                          h_X: torch.Tensor, h_out: torch.Tensor, bufs: dict,
                          feature_blocks: int = 8, out_chunks: int = 2) -> torch.Tensor:
        """The whole call from host inputs: raw CSR rows + feature rows (pinned
        host tensors of this rank) in, logits (pinned host tensor) out.

        ``h_v = None`` is an unweighted graph: every stored value is 1.0 (what
        edge_list_to_csr and from_edge_index produce), written on the device
        instead of crossing PCIe.  Uploads are queued first on a copy stream
        (CSR, then the features in row blocks); gcn_norm runs as soon as the
        CSR is in, while the features stream; on one GPU the first layer's
        GEMM and exact gather pass for feature block q start when block q has
        landed.  Feature rows whose width is not a multiple of 4 land in a
        contiguous buffer and are repacked on the device to the 16-byte row
        stride the tensor-core GEMM reads (a pitched host-to-device copy of
        2,408-byte rows is slower than the repack).  The last layer's gather,
        when it is one pass, runs in ``out_chunks`` row chunks, each with its
        own longest-rows-first schedule, and each chunk's logits go back to
        the host while the next chunk gathers.  ``bufs`` holds the device
        buffers across calls (filled on first use).
        """
        dev = self.device
        cur = torch.cuda.current_stream()
        cp = bufs.get("stream")
        if cp is None:
            cp = bufs["stream"] = torch.cuda.Stream(device=dev)
            bufs["rp"] = torch.empty_like(h_rp, device=dev)
            bufs["ci"] = torch.empty_like(h_ci, device=dev)
            bufs["v"] = torch.empty(h_ci.shape, dtype=torch.float32, device=dev)
            bufs["X"] = torch.zeros((self.rows, _pad4(h_X.shape[1])), dtype=torch.float32, device=dev)
            if h_X.shape[1] % 4:
                bufs["X_landing"] = torch.empty((self.rows, h_X.shape[1]), dtype=torch.float32, device=dev)
            bufs["dis"] = torch.zeros(self.R * self.comm.world, dtype=torch.float32, device=dev)
        d_rp, d_ci, d_v, d_X = bufs["rp"], bufs["ci"], bufs["v"], bufs["X"][:, :h_X.shape[1]]
        landing = bufs.get("X_landing")
        x_dst = d_X if landing is None else landing
        single = self.comm.world == 1 and self.layers[0].kind == "gcn"
        nb = max(1, feature_blocks) if single else 1
        width = (self.rows + nb - 1) // nb
        x_ready = []
        cp.wait_stream(cur)
        with torch.cuda.stream(cp):
            d_rp.copy_(h_rp, non_blocking=True)
            d_ci.copy_(h_ci, non_blocking=True)
            if h_v is not None:
                d_v.copy_(h_v, non_blocking=True)
            csr_ready = torch.cuda.Event()
            csr_ready.record(cp)
            for q in range(nb):
                a, b = q * width, min(self.rows, (q + 1) * width)
                if a < b:
                    x_dst[a:b].copy_(h_X[a:b], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(cp)
                x_ready.append(ev)
        if h_v is None:  # on the compute stream, while the uploads run
            d_v.fill_(1.0)
        cur.wait_event(csr_ready)
        A = CSR(self.rows, self.n, d_rp, d_ci, d_v)
        A_gcn = self._normalise(A, bufs["dis"], scratch=True)
        self._join_prep()
        if single and nb > 1:
            # Layer 1 per feature block: GEMM of block q's rows, then the gather
            # pass over the columns of block q (exact: passes in column order).
            L = self.layers[0]
            fo = L.W.shape[1]
            sp = ops.column_splits(A_gcn, nb, width)
            B = self.full[0][:self.n, :fo]
            for q in range(nb):
                a, b = q * width, min(self.rows, (q + 1) * width)
                cur.wait_event(x_ready[q])
                if a < b:
                    if landing is not None:
                        d_X[a:b].copy_(landing[a:b])
                    ops.matmul(d_X[a:b], L.W, out=self.full[0][a:b, :fo], mode=self.mode,
                               row_scale=self.scale[a:b] if self._scaled(0) else None, cols_padded=True)
                if self._scaled(0):
                    ops.gcn_aggregate(A_gcn, B, self._self_rows(0), self.scale, bias=L.b, act=L.act,
                                      out=self.outs[0], seg_begin=sp[q], seg_end=sp[q + 1], carry=q > 0,
                                      last=q == nb - 1)
                else:
                    ops.spmm_segment(A_gcn, B, sp[q], sp[q + 1], self.outs[0], q > 0, q == nb - 1, bias=L.b,
                                     act=L.act)
            H = self.outs[0]
            first = 1
        else:
            for ev in x_ready:
                cur.wait_event(ev)
            if landing is not None:
                d_X.copy_(landing)
            H, first = d_X, 0
        last = len(self.layers) - 1
        for li in range(first, last):
            self.transform(li, H)
            H = self.exchange_and_aggregate(li, A_gcn, A)
        if first > last:
            ops.log_softmax_(H)
            h_out.copy_(H, non_blocking=True)
        elif self.pipe[last] or self.pass_splits(A_gcn if self.layers[last].kind == "gcn" else A,
                                                 self.passes[last]) is not None or out_chunks <= 1:
            self.transform(last, H)
            H = self.exchange_and_aggregate(last, A_gcn, A)
            ops.log_softmax_(H)
            h_out.copy_(H, non_blocking=True)
        else:
            self.transform(last, H)
            self.exchange(last)
            self._chunked_last_layer(A_gcn, A, h_out, cp, out_chunks)
        cur.synchronize()
        self.scale = None
        return h_out

    def _normalise(self, A: CSR, dis_all: torch.Tensor, scratch: bool = False) -> Optional[CSR]:
        """What Model::forward does to the raw adjacency rows before the GCN
        layers (src/model.cpp:365-381), with a longest-first row schedule:
        EXACT -- the normalised copy, bit for bit; FAST -- the raw rows plus
        this rank's 1/sqrt(deg) (self.scale), for the factored layers.
        None when no layer is a GCN layer.  ``scratch``: the schedule and split
        points go into buffers the model rewrites every call (a forward that does
        not keep the returned CSR); otherwise they are the CSR's own."""
        if not any(L.kind == "gcn" for L in self.layers):
            self.scale = None
            return None
        if self.mode == "fast":
            As = CSR(A.n_rows, A.n_cols, A.row_ptr, A.col_ind, A.values, A.order, A.validated)
            if not As.validated:
                ops.csr_validate(As)  # Tensor::sparse_csr's checks, once, before any kernel reads As
                As.validated = True
            if not scratch:
                if As.order is None:
                    As.order = ops.degree_order(As)
                self.scale = ops.gcn_norm_scale(As, out=self.scale_buf[:A.n_rows])
                A.validated = True
                return As
            # The row schedule and the column-pass split points run on a side
            # stream beside the scale and the first GEMM, which need neither;
            # the first gather joins them (_join_prep).  They go into buffers
            # the model keeps: the side stream starts after all earlier work
            # of the current stream (the previous forward's reads of them),
            # and no per-call allocation crosses streams (freed blocks of
            # another stream are reusable only once the GPU has caught up,
            # which made the allocator grow, and synchronise, while the host
            # ran ahead).
            # High priority: its blocks are dispatched ahead of the scale
            # kernel's, so it is done before the GEMM (a persistent kernel
            # holding every SM's shared memory until its last tile) starts.
            cur = torch.cuda.current_stream()
            side = self._prep_stream
            if side is None:
                side = self._prep_stream = torch.cuda.Stream(device=self.device, priority=-1)
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                if As.order is None:
                    if self._order_buf is None or self._order_buf.numel() < As.n_rows:
                        self._order_buf = torch.empty(max(As.n_rows, 1), dtype=torch.int32, device=self.device)
                    As.order = ops.degree_order(As, out=self._order_buf[:As.n_rows])
                if not self.pipeline:
                    for li, L in enumerate(self.layers):
                        p = self.passes[li]
                        if L.kind != "gcn" or p == 1:
                            continue
                        buf = self._split_bufs.get(p)
                        if buf is None or buf.shape[1] != As.n_rows:
                            buf = self._split_bufs[p] = torch.empty((p + 1, As.n_rows), dtype=torch.int32,
                                                                     device=self.device)
                        cache = As.__dict__.setdefault("_splits", {})
                        key = (p, -(-self.n // p))
                        if key not in cache:
                            cache[key] = ops.column_splits(As, p, key[1], out=buf)
            self._prep_ready = torch.cuda.Event()
            self._prep_ready.record(side)
            self.scale = ops.gcn_norm_scale(As, out=self.scale_buf[:A.n_rows])
            A.validated = True  # same arrays: checked once
            return As
        self.scale = None
        return gcn_norm_rows_scheduled(A, self.row0, self.R, self.comm, dis_all)

    def prepare(self, A_raw: CSR, dis_all: Optional[torch.Tensor] = None, scratch: bool = False):
        """The per-graph part of Model::forward for this rank's raw adjacency
        rows: (A for the GCN layers, A for the SAGE layers, this rank's GCN
        scale or None) -- see _normalise."""
        if dis_all is None and self.mode != "fast":
            dis_all = torch.zeros(self.R * self.comm.world, dtype=torch.float32, device=self.device)
        A_gcn = self._normalise(A_raw, dis_all, scratch)
        scale, self.scale = self.scale, None
        A_sage = A_raw
        if A_gcn is not None and self.mode == "fast":
            A_sage = A_gcn  # the same raw rows, scheduled
        elif A_raw.order is None and any(L.kind == "sage" for L in self.layers):
            A_sage = CSR(A_raw.n_rows, A_raw.n_cols, A_raw.row_ptr, A_raw.col_ind, A_raw.values,
                         ops.degree_order(A_raw), A_raw.validated)
        return A_gcn, A_sage, scale

    def forward_prepared(self, prepared, X: torch.Tensor, log_softmax: bool = True) -> torch.Tensor:
        """The layers (and log_softmax) on a graph prepared by prepare()."""
        A_gcn, A_sage, scale = prepared
        self.scale = scale
        try:
            return self.forward(A_gcn, A_sage, X, log_softmax)
        finally:
            self.scale = None

    def forward_model(self, A_raw: CSR, X: torch.Tensor, log_softmax: bool = True,
                      dis_all: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Model::forward on this rank's raw adjacency rows (no self-loops) and
        feature rows in HBM: normalisation, the layers, log_softmax."""
        return self.forward_prepared(self.prepare(A_raw, dis_all, scratch=True), X, log_softmax)

    def _chunked_last_layer(self, A_gcn: Optional[CSR], A_raw: CSR, h_out: torch.Tensor,
                            cp: torch.cuda.Stream, chunks: int) -> None:
        """The last layer's single-pass gather over row chunks (row-offset
        views of the CSR, each with its own degree order), log_softmax per
        chunk, and each chunk's logits copied out on `cp` while the next
        chunk gathers.  Per row the same arithmetic as one launch."""
        li = len(self.layers) - 1
        L = self.layers[li]
        fo = L.W.shape[1]
        A = A_gcn if L.kind == "gcn" else A_raw
        B = self.full[li][:self.n, :fo]
        cur = torch.cuda.current_stream()
        step = max(1, -(-self.rows // chunks))  # a rank may own no rows
        for a in range(0, self.rows, step):
            b = min(self.rows, a + step)
            # rows [a, b) of a checked CSR (its row_ptr slice indexes the same arrays)
            Ak = CSR(b - a, A.n_cols, A.row_ptr[a:b + 1], A.col_ind, A.values, validated=A.validated)
            Ak.order = ops.degree_order(Ak)
            out = self.outs[li][a:b]
            if self._scaled(li):
                ops.gcn_aggregate(Ak, B, self._self_rows(li, a, b), self.scale[a:b], bias=L.b, act=L.act, out=out)
            elif L.kind == "gcn":
                ops.spmm(Ak, B, bias=L.b, act=L.act, out=out)
            else:
                ops.sage_mean_combine(Ak, B, self.selfs[li][a:b, :fo], bias=L.b, act=L.act, out=out)
            ops.log_softmax_(out)
            done = torch.cuda.Event()
            done.record(cur)
            cp.wait_event(done)
            with torch.cuda.stream(cp):
                h_out[a:b].copy_(out, non_blocking=True)
        cur.wait_stream(cp)

    def forward(self, A_gcn: Optional[CSR], A_raw: Optional[CSR], X: torch.Tensor,
                log_softmax: bool = True) -> torch.Tensor:
        H = X
        for li in range(len(self.layers)):
            self.transform(li, H)
            H = self.exchange_and_aggregate(li, A_gcn, A_raw)
        if log_softmax:
            ops.log_softmax_(H)
        return H
