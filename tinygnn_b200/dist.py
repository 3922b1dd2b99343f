"""Row-partitioned GCN / SAGE forward over several GPUs (one process per GPU).

Partitioning (1-D, by rows): with P ranks and N nodes, rank r owns global
rows [r*R, min(N, (r+1)*R)) where R = ceil(N/P) -- its rows of the
adjacency (global column ids) and of the features.  Every per-layer exchange
is one NCCL all-gather of the transformed rows into a (P*R) x F buffer whose
row j is global node j, so gathers index it with the global column ids
directly (no remapping).  Hubs are never split across ranks.

Per GCN layer on rank r (src/layers.cpp:286-339 per block of rows):
  1. HW[rR : rR + rows] = H_r . W          (exact GEMM, this rank's rows)
  2. all-gather HW over the ranks           (torch.distributed, NCCL)
  3. H'_r = act(A_norm[r-rows] . HW + b)    (gather kernel, fused epilogue)
gcn_norm of a row block (src/layers.cpp:158-208): self-loops and degrees are
row-local; the column scale needs every node's 1/sqrt(deg), which one
all-gather of the degree vector provides -- bit-identical to the
single-GPU gcn_norm.

SAGE (transform-first, mean): Tn_r = H_r . W_neigh is all-gathered,
Ts_r = H_r . W_self stays local, H'_r = act(mean_j Tn[j] + Ts_r[i] + b).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from . import ops
from .ops import CSR


def row_block(n: int, world: int, rank: int) -> Tuple[int, int, int]:
    """(R, row0, row1): the equal-size row block of ``rank``."""
    R = (n + world - 1) // world
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
    """The exchange step: all-gather of equal row blocks (NCCL), or nothing at P=1."""

    def __init__(self, world: int, rank: int, group=None):
        self.world, self.rank, self.group = world, rank, group

    def all_gather_rows(self, full: torch.Tensor, R: int) -> None:
        """In-place all-gather: rank r's rows [rR, rR+R) of ``full`` go to every rank."""
        if self.world == 1:
            return
        mine = full[self.rank * R:(self.rank + 1) * R]
        dist.all_gather_into_tensor(full, mine, group=self.group)


def gcn_norm_rows(A: CSR, row0: int, R: int, comm: Comm, dis_all: Optional[torch.Tensor] = None) -> CSR:
    """gcn_norm of this rank's row block (global columns), bit-identical to the
    rows of the single-GPU gcn_norm."""
    asl = ops.add_self_loops_rows(A, row0)
    if dis_all is None:
        dis_all = torch.zeros(R * comm.world, dtype=torch.float32, device=A.row_ptr.device)
    mine = dis_all[comm.rank * R:comm.rank * R + A.n_rows]
    ops.degree_inv_sqrt(asl, out=mine)
    comm.all_gather_rows(dis_all.view(-1, 1), R)
    return ops.scale_sym_(asl, mine, dis_all)


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
    """

    def __init__(self, layers: List[Layer], n: int, comm: Comm, device, mode: str = "exact"):
        self.layers, self.n, self.comm, self.device, self.mode = layers, n, comm, device, mode
        self.R, self.row0, self.row1 = row_block(n, comm.world, comm.rank)
        self.rows = self.row1 - self.row0
        P = comm.world
        self.full = []   # gathered operand per layer: (P*R) x pad4(F_out)
        self.outs = []
        self.selfs = []
        for L in layers:
            fo = L.W.shape[1]
            self.full.append(torch.zeros((P * self.R, _pad4(fo)), dtype=torch.float32, device=device))
            self.outs.append(torch.empty((self.rows, fo), dtype=torch.float32, device=device))
            self.selfs.append(torch.empty((self.rows, _pad4(fo)), dtype=torch.float32, device=device)
                              if L.kind == "sage" else None)
        self.timing = None  # optional hook: (layer index, "gather"|"gemm", start|end) -> None

    def _mark(self, li: int, what: str, edge: str) -> None:
        if self.timing is not None:
            self.timing(li, what, edge)

    # The three phases of a layer; forward() runs them in order.  Tests that
    # emulate several ranks in one process interleave them across shards.
    def transform(self, li: int, H: torch.Tensor) -> None:
        """This rank's rows of H . W (and H . W_self for SAGE) into the gather buffer."""
        L = self.layers[li]
        fo = L.W.shape[1]
        r = self.comm.rank
        self._mark(li, "gemm", "start")
        ops.matmul(H, L.W, out=self.full[li][r * self.R:r * self.R + self.rows, :fo], mode=self.mode)
        if L.kind == "sage":
            ops.matmul(H, L.W_self, out=self.selfs[li][:, :fo], mode=self.mode)
        self._mark(li, "gemm", "end")

    def exchange(self, li: int) -> None:
        self.comm.all_gather_rows(self.full[li], self.R)

    def aggregate(self, li: int, A_gcn: Optional[CSR], A_raw: Optional[CSR]) -> torch.Tensor:
        L = self.layers[li]
        fo = L.W.shape[1]
        B = self.full[li][:self.n, :fo]
        self._mark(li, "gather", "start")
        if L.kind == "gcn":
            H = ops.spmm(A_gcn, B, bias=L.b, act=L.act, out=self.outs[li])
        else:
            H = ops.sage_mean_combine(A_raw, B, self.selfs[li][:, :fo], bias=L.b, act=L.act, out=self.outs[li])
        self._mark(li, "gather", "end")
        return H

    def forward(self, A_gcn: Optional[CSR], A_raw: Optional[CSR], X: torch.Tensor,
                log_softmax: bool = True) -> torch.Tensor:
        H = X
        for li in range(len(self.layers)):
            self.transform(li, H)
            self.exchange(li)
            H = self.aggregate(li, A_gcn, A_raw)
        if log_softmax:
            ops.log_softmax_(H)
        return H
