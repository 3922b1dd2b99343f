"""Torch-tensor front end of the C ABI (device-pointer level).

Every function here calls one ``tg_*`` entry point of
libtinygnn_b200.so on torch's current CUDA stream; torch only provides the
device memory.  Dense operands are 2-D float32 CUDA tensors with unit column
stride (any row stride); CSR operands are :class:`CSR`.

Names and semantics follow TinyGNN's operator API (include/tinygnn/ops.hpp,
include/tinygnn/layers.hpp, include/tinygnn/graph_loader.hpp).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import _lib
from ._lib import check, lib

ACT = {None: _lib.ACT_NONE, "none": _lib.ACT_NONE, "relu": _lib.ACT_RELU, "elu": _lib.ACT_ELU,
       "leaky_relu": _lib.ACT_LEAKY_RELU, "sigmoid": _lib.ACT_SIGMOID, "tanh": _lib.ACT_TANH,
       "gelu": _lib.ACT_GELU}
MODE = {"exact": _lib.MODE_EXACT, "fast": _lib.MODE_FAST}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _p(t: Optional[torch.Tensor]):
    return None if t is None else C.c_void_p(t.data_ptr())


def _dense(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dim() != 2 or t.dtype != torch.float32 or not t.is_cuda:
        raise ValueError(f"{name} must be a 2-D float32 CUDA tensor")
    if t.stride(1) != 1 and t.numel() > 0:
        t = t.contiguous()
    return t


def _ld(t: torch.Tensor) -> int:
    return max(t.stride(0), t.shape[1]) if t.dim() == 2 else 1


def _ord(A, row_order):
    return row_order if row_order is not None else getattr(A, "order", None)


def _vec(t: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    if t is None:
        return None
    return t.reshape(-1).to(torch.float32).contiguous()


@dataclass
class CSR:
    """Device CSR matrix: int32 row_ptr[n_rows+1], col_ind[nnz], float32 values[nnz].

    values may be None: an unweighted CSR (every entry 1.0, no array), which
    spmm / spmm_segment, gcn_norm_scale, gcn_aggregate and the FAST GCN
    forward take as they take an array of ones, bit for bit, without reading
    one; every other operation needs the values array."""

    n_rows: int
    n_cols: int
    row_ptr: torch.Tensor
    col_ind: torch.Tensor
    values: Optional[torch.Tensor]
    # Optional row schedule (int32 permutation, longest rows first) reused by
    # every gather over this matrix; without it large gathers compute one.
    order: Optional[torch.Tensor] = None
    # The library checks every CSR it is given (Tensor::sparse_csr's checks,
    # on the device) before reading through it; a CSR that passed once, or
    # that the library built, is marked and not checked again.
    validated: bool = False

    @property
    def nnz(self) -> int:
        return int(self.col_ind.numel())

    def with_degree_order(self) -> "CSR":
        """Compute and keep the longest-rows-first schedule."""
        self.order = degree_order(self)
        return self

    @classmethod
    def from_numpy(cls, row_ptr, col_ind, values=None, n_cols=None, device="cuda") -> "CSR":
        rp = torch.as_tensor(np.ascontiguousarray(row_ptr, dtype=np.int32), device=device)
        ci = torch.as_tensor(np.ascontiguousarray(col_ind, dtype=np.int32), device=device)
        if values is None:
            v = torch.ones(ci.numel(), dtype=torch.float32, device=device)
        else:
            v = torch.as_tensor(np.ascontiguousarray(values, dtype=np.float32), device=device)
        n = rp.numel() - 1
        return cls(n, n if n_cols is None else int(n_cols), rp, ci, v)

    def numpy(self):
        v = (np.ones(self.nnz, np.float32) if self.values is None else self.values.cpu().numpy())
        return (self.row_ptr.cpu().numpy(), self.col_ind.cpu().numpy(), v)


def _csr_call(csrs, fn, *args) -> None:
    """Call a C-ABI entry point that reads the CSRs ``csrs``.  The library
    checks a caller's CSR on every call unless the thread turns the checks
    off (tg_set_csr_checks); here they run once per CSR object: calls on CSRs
    already checked (or built by the library) turn them off around the call."""
    trusted = all(c.validated for c in csrs)
    prev = lib.tg_set_csr_checks(0) if trusted else None
    try:
        check(fn(*args))
    finally:
        if prev is not None:
            lib.tg_set_csr_checks(prev)
    if not trusted:
        for c in csrs:
            c.validated = True


# ── dense ops ────────────────────────────────────────────────────────────────
def matmul(A: torch.Tensor, B: torch.Tensor, bias=None, act=None, alpha: float = 0.0,
           out: Optional[torch.Tensor] = None, mode: str = "exact",
           row_scale: Optional[torch.Tensor] = None, cols_padded: bool = False) -> torch.Tensor:
    """C = act(A . B + bias)  (TinyGNN matmul, src/ops.cpp:70); with
    ``row_scale``, C = act(diag(row_scale) . (A . B) + bias).  ``cols_padded``:
    out's rows have room up to round_up(N, 4) columns, which FAST mode may
    write (act(0)) to store rows 16 bytes at a time."""
    A, B = _dense(A, "A"), _dense(B, "B")
    if A.shape[1] != B.shape[0]:
        raise _lib.InvalidArgument(
            _lib.INVALID_ARGUMENT,
            f"matmul: dimension mismatch — A is ({A.shape[0]}×{A.shape[1]}) but B is "
            f"({B.shape[0]}×{B.shape[1]}). Required: A.cols() == B.rows() (both = {A.shape[1]} vs {B.shape[0]}).")
    M, K = A.shape
    N = B.shape[1]
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=A.device)
    b = _vec(bias)
    if row_scale is not None:
        check(lib.tg_gemm_rowscale_f32(M, N, K, _p(A), _ld(A), _p(B), _ld(B), _p(out), _ld(out), _p(row_scale),
                                       _p(b), ACT[act], alpha, MODE[mode] | (FLAG_C_COLS_PADDED if cols_padded else 0),
                                       _stream()))
        return out
    check(lib.tg_gemm_f32(M, N, K, _p(A), _ld(A), _p(B), _ld(B), _p(out), _ld(out), _p(b), ACT[act], alpha,
                          MODE[mode] | (FLAG_C_COLS_PADDED if cols_padded else 0), _stream()))
    return out


def gemm_pair(A: torch.Tensor, B1: torch.Tensor, B2: torch.Tensor, out1: torch.Tensor, out2: torch.Tensor,
              mode: str = "fast", cols_padded: bool = False):
    """out1 = A . B1, out2 = A . B2 (one tensor-core pass over A in FAST mode);
    ``cols_padded`` as in matmul, for both outputs."""
    A, B1, B2 = _dense(A, "A"), _dense(B1, "B1").contiguous(), _dense(B2, "B2").contiguous()
    M, K = A.shape
    N = B1.shape[1]
    check(lib.tg_gemm_pair_f32(M, N, K, _p(A), _ld(A), _p(B1), _p(B2), N, _p(out1), _ld(out1), _p(out2), _ld(out2),
                               MODE[mode] | (FLAG_C_COLS_PADDED if cols_padded else 0), _stream()))
    return out1, out2


def gemm_cat(A1: torch.Tensor, A2: torch.Tensor, B1: torch.Tensor, B2: torch.Tensor, bias=None, act=None,
             alpha: float = 0.0, out: Optional[torch.Tensor] = None, mode: str = "fast") -> torch.Tensor:
    """C = act([A1 | A2] . [B1; B2] + bias) without forming the concatenation."""
    A1, A2 = _dense(A1, "A1"), _dense(A2, "A2")
    B1, B2 = _dense(B1, "B1"), _dense(B2, "B2")
    M, K1 = A1.shape
    K2, N = A2.shape[1], B1.shape[1]
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=A1.device)
    b = _vec(bias)
    check(lib.tg_gemm_cat_f32(M, N, K1, _p(A1), _ld(A1), K2, _p(A2), _ld(A2), _p(B1), _ld(B1), _p(B2), _ld(B2),
                              _p(out), _ld(out), _p(b), ACT[act], alpha, MODE[mode], _stream()))
    return out


def gemm_dual(A1, A2, B1, B2, bias=None, act=None, out=None) -> torch.Tensor:
    """C = interleaved A1.B1 + A2.B2 (SAGE's fused dual GEMV order)."""
    A1, A2, B1, B2 = _dense(A1, "A1"), _dense(A2, "A2"), _dense(B1, "B1"), _dense(B2, "B2")
    M, K = A1.shape
    N = B1.shape[1]
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=A1.device)
    b = _vec(bias)
    check(lib.tg_gemm_dual_f32(M, N, K, _p(A1), _ld(A1), _p(A2), _ld(A2), _p(B1), _p(B2), _ld(B1), _p(out),
                               _ld(out), _p(b), ACT[act], 0.0, _stream()))
    return out


def activation_(X: torch.Tensor, kind: str, alpha: float = 0.0) -> torch.Tensor:
    """In-place activation (src/ops.cpp:328-482)."""
    X = _dense(X, "X")
    check(lib.tg_activation_f32(ACT[kind], alpha, _p(X), X.shape[0], X.shape[1], _ld(X), _stream()))
    return X


def relu_(X):
    return activation_(X, "relu")


def leaky_relu_(X, alpha: float = 0.01):
    return activation_(X, "leaky_relu", alpha)


def elu_(X, alpha: float = 1.0):
    return activation_(X, "elu", alpha)


def sigmoid_(X):
    return activation_(X, "sigmoid")


def tanh_(X):
    return activation_(X, "tanh")


def gelu_(X):
    return activation_(X, "gelu")


def softmax_(X: torch.Tensor) -> torch.Tensor:
    X = _dense(X, "X")
    check(lib.tg_softmax_rows_f32(_p(X), X.shape[0], X.shape[1], _ld(X), _stream()))
    return X


def log_softmax_(X: torch.Tensor) -> torch.Tensor:
    X = _dense(X, "X")
    check(lib.tg_log_softmax_rows_f32(_p(X), X.shape[0], X.shape[1], _ld(X), _stream()))
    return X


def add_bias_(X: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    X = _dense(X, "X")
    b = _vec(bias)
    if b.numel() != X.shape[1]:
        raise _lib.InvalidArgument(
            _lib.INVALID_ARGUMENT,
            f"add_bias: bias must be shape (1×{X.shape[1]}) to match X columns, but got (1×{b.numel()}).")
    check(lib.tg_add_bias_f32(_p(X), X.shape[0], X.shape[1], _ld(X), _p(b), _stream()))
    return X


# ── sparse ops ───────────────────────────────────────────────────────────────
FLAG_B_ROWS_PADDED = 0x100
FLAG_C_COLS_PADDED = 0x200


def _padded(t: torch.Tensor) -> bool:
    """True when every row of the 2-D view t is readable up to its row stride."""
    if t.dim() != 2 or t.shape[0] == 0:
        return False
    storage_elems = t.untyped_storage().nbytes() // t.element_size()
    last_row_end = t.storage_offset() + (t.shape[0] - 1) * t.stride(0) + t.stride(0)
    return t.stride(0) % 4 == 0 and last_row_end <= storage_elems


def spmm(A: CSR, B: torch.Tensor, bias=None, act=None, alpha: float = 0.0, row_order=None,
         out: Optional[torch.Tensor] = None, mode: str = "exact") -> torch.Tensor:
    """C = act(A . B + bias)  (TinyGNN spmm, src/ops.cpp:198)."""
    B = _dense(B, "B")
    if A.n_cols != B.shape[0]:
        raise _lib.InvalidArgument(
            _lib.INVALID_ARGUMENT,
            f"spmm: dimension mismatch — A is ({A.n_rows}×{A.n_cols}, SparseCSR) but B is "
            f"({B.shape[0]}×{B.shape[1]}, Dense). Required: A.cols() == B.rows() ({A.n_cols} vs {B.shape[0]}).")
    F = B.shape[1]
    if out is None:
        out = torch.empty((A.n_rows, F), dtype=torch.float32, device=B.device)
    b = _vec(bias)
    flags = MODE[mode] | (FLAG_B_ROWS_PADDED if _padded(B) else 0)
    _csr_call((A,), lib.tg_spmm_f32, A.n_rows, A.n_cols, A.nnz, _p(A.row_ptr), _p(A.col_ind), _p(A.values), _p(B), F,
                          _ld(B), _p(out), _ld(out), _p(b), ACT[act], alpha, _p(_ord(A, row_order)), flags,
                          _stream())
    return out


def column_splits(A: CSR, nblocks: int, width: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """(nblocks+1) x n_rows split points of sorted rows at column multiples of `width`."""
    if out is None:
        out = torch.empty((nblocks + 1, A.n_rows), dtype=torch.int32, device=A.row_ptr.device)
    _csr_call((A,), lib.tg_csr_column_splits, A.n_rows, _p(A.row_ptr), _p(A.col_ind), nblocks, width, _p(out), _stream())
    return out


def spmm_segment(A: CSR, B: torch.Tensor, seg_begin: torch.Tensor, seg_end: torch.Tensor, out: torch.Tensor,
                 carry: bool, last: bool, bias=None, act=None, alpha: float = 0.0, row_order=None) -> torch.Tensor:
    """One column-block pass of spmm (see tg_spmm_segment_f32)."""
    B = _dense(B, "B")
    b = _vec(bias)
    flags = FLAG_B_ROWS_PADDED if _padded(B) else 0
    _csr_call((A,), lib.tg_spmm_segment_f32, A.n_rows, A.n_cols, _p(A.row_ptr), _p(A.col_ind), _p(A.values), _p(seg_begin),
                                  _p(seg_end), _p(B), B.shape[1], _ld(B), _p(out), _ld(out), _p(b), ACT[act], alpha,
                                  _p(_ord(A, row_order)), int(carry), int(last), flags, _stream())
    return out


def sage_mean_combine_segment(A: CSR, Tn: torch.Tensor, Ts: torch.Tensor, seg_begin, seg_end, out, carry: bool,
                              last: bool, bias=None, act=None, row_order=None) -> torch.Tensor:
    """One column-block pass of the transform-first SAGE-mean combine."""
    Tn, Ts = _dense(Tn, "Tn"), _dense(Ts, "Ts")
    b = _vec(bias)
    flags = FLAG_B_ROWS_PADDED if _padded(Tn) else 0
    _csr_call((A,), lib.tg_sage_mean_combine_segment_f32, A.n_rows, A.n_cols, _p(A.row_ptr), _p(A.col_ind), _p(seg_begin),
                                               _p(seg_end), _p(Tn), Tn.shape[1], _ld(Tn), _p(Ts), _ld(Ts), _p(b),
                                               ACT[act], _p(out), _ld(out), _p(_ord(A, row_order)), int(carry),
                                               int(last), flags, _stream())
    return out


def sage_mean_combine(A: CSR, Tn: torch.Tensor, Ts: torch.Tensor, bias=None, act=None, row_order=None,
                      out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[i] = act(mean_j Tn[j] + Ts[i] + bias): transform-first SAGE mean."""
    Tn, Ts = _dense(Tn, "Tn"), _dense(Ts, "Ts")
    F = Tn.shape[1]
    if out is None:
        out = torch.empty((A.n_rows, F), dtype=torch.float32, device=Tn.device)
    b = _vec(bias)
    flags = FLAG_B_ROWS_PADDED if _padded(Tn) else 0
    _csr_call((A,), lib.tg_sage_mean_combine_f32, A.n_rows, A.n_cols, A.nnz, _p(A.row_ptr), _p(A.col_ind), _p(Tn), F,
                                       _ld(Tn), _p(Ts), _ld(Ts), _p(b), ACT[act], _p(out), _ld(out),
                                       _p(_ord(A, row_order)), flags, _stream())
    return out


def degree_order(A: CSR, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Rows by decreasing stored length (a schedule for the gather kernels)."""
    if out is None:
        out = torch.empty(A.n_rows, dtype=torch.int32, device=A.row_ptr.device)
    check(lib.tg_csr_degree_order(A.n_rows, _p(A.row_ptr), _p(out), _stream()))
    return out


def sage_aggregate(A: CSR, H: torch.Tensor, aggregator: str = "mean") -> torch.Tensor:
    H = _dense(H, "H")
    out = torch.empty((A.n_rows, H.shape[1]), dtype=torch.float32, device=H.device)
    _csr_call((A,), lib.tg_sage_aggregate_f32, A.n_rows, A.n_cols, A.nnz, _p(A.row_ptr), _p(A.col_ind), _p(H), H.shape[1],
                                    _ld(H), _p(out), _ld(out), _lib.AGG_MAX if aggregator == "max" else
                                    _lib.AGG_MEAN, _stream())
    return out


def sage_max_aggregate(A: CSR, H: torch.Tensor) -> torch.Tensor:
    """sage_max_aggregate (src/layers.cpp:359)."""
    H = _dense(H, "H")
    if A.n_cols != H.shape[0]:
        raise _lib.InvalidArgument(_lib.INVALID_ARGUMENT,
                                   f"sage_max_aggregate: A.cols() ({A.n_cols}) != H.rows() ({H.shape[0]}).")
    out = torch.empty((A.n_rows, H.shape[1]), dtype=torch.float32, device=H.device)
    _csr_call((A,), lib.tg_sage_max_aggregate_f32, A.n_rows, A.n_cols, A.nnz, _p(A.row_ptr), _p(A.col_ind), _p(H),
                                        H.shape[1], _ld(H), _p(out), _ld(out), _stream())
    return out


def edge_softmax(A: CSR) -> CSR:
    """edge_softmax (src/layers.cpp:768): same structure, row-softmaxed values."""
    v = torch.zeros_like(A.values)
    _csr_call((A,), lib.tg_edge_softmax_f32, A.n_rows, A.nnz, _p(A.row_ptr), _p(A.values), _p(v), _stream())
    return CSR(A.n_rows, A.n_cols, A.row_ptr.clone(), A.col_ind.clone(), v, validated=True)


# ── graph construction ───────────────────────────────────────────────────────
def edge_list_to_csr(src: torch.Tensor, dst: torch.Tensor, num_nodes: int) -> CSR:
    """GraphLoader::edge_list_to_csr (src/graph_loader.cpp:211)."""
    src = src.to(torch.int32).contiguous()
    dst = dst.to(torch.int32).contiguous()
    E = src.numel()
    dev = src.device
    rp = torch.empty(num_nodes + 1, dtype=torch.int32, device=dev)
    ci = torch.empty(max(E, 1), dtype=torch.int32, device=dev)
    v = torch.empty(max(E, 1), dtype=torch.float32, device=dev)
    check(lib.tg_edge_list_to_csr(num_nodes, E, _p(src), _p(dst), _p(rp), _p(ci), _p(v), _stream()))
    return CSR(num_nodes, num_nodes, rp, ci[:E], v[:E], validated=True)


def _csr_expand(fn, A: CSR) -> CSR:
    N = A.n_rows
    if A.n_rows != A.n_cols:
        name = "gcn_norm" if fn is lib.tg_gcn_norm_f32 else "add_self_loops"
        raise _lib.InvalidArgument(_lib.INVALID_ARGUMENT,
                                   f"{name}: A must be square — got ({A.n_rows}×{A.n_cols}).")
    cap = A.nnz + N
    dev = A.row_ptr.device
    rp = torch.empty(N + 1, dtype=torch.int32, device=dev)
    ci = torch.empty(max(cap, 1), dtype=torch.int32, device=dev)
    v = torch.empty(max(cap, 1), dtype=torch.float32, device=dev)
    nnz = C.c_int64(0)
    _csr_call((A,), fn, N, A.nnz, _p(A.row_ptr), _p(A.col_ind), _p(A.values), _p(rp), _p(ci), _p(v), C.byref(nnz),
              _stream())
    return CSR(N, N, rp, ci[:nnz.value], v[:nnz.value], validated=True)


def add_self_loops(A: CSR) -> CSR:
    """add_self_loops (src/layers.cpp:71)."""
    return _csr_expand(lib.tg_add_self_loops_f32, A)


def gcn_norm(A: CSR) -> CSR:
    """gcn_norm (src/layers.cpp:158): D^-1/2 (A + I) D^-1/2."""
    return _csr_expand(lib.tg_gcn_norm_f32, A)


def add_self_loops_rows(A: CSR, row_offset: int) -> CSR:
    """add_self_loops of a row block (global rows row_offset.., global columns)."""
    N = A.n_rows
    cap = A.nnz + N
    dev = A.row_ptr.device
    rp = torch.empty(N + 1, dtype=torch.int32, device=dev)
    ci = torch.empty(max(cap, 1), dtype=torch.int32, device=dev)
    v = torch.empty(max(cap, 1), dtype=torch.float32, device=dev)
    nnz = C.c_int64(0)
    _csr_call((A,), lib.tg_add_self_loops_rows_f32, N, row_offset, A.nnz, _p(A.row_ptr), _p(A.col_ind), _p(A.values), _p(rp),
                                         _p(ci), _p(v), C.byref(nnz), _stream())
    return CSR(N, A.n_cols, rp, ci[:nnz.value], v[:nnz.value], validated=True)


def degree_inv_sqrt(A: CSR, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """dis[i] = 1/sqrtf(sum of row i's values) (0 for non-positive sums)."""
    if out is None:
        out = torch.empty(A.n_rows, dtype=torch.float32, device=A.row_ptr.device)
    _csr_call((A,), lib.tg_csr_degree_inv_sqrt_f32, A.n_rows, _p(A.row_ptr), _p(A.values), _p(out), _stream())
    return out


def scale_sym_(A: CSR, dis_row: torch.Tensor, dis_col: torch.Tensor) -> CSR:
    """values = (values * dis_row[i]) * dis_col[j], in place."""
    _csr_call((A,), lib.tg_csr_scale_sym_f32, A.n_rows, _p(A.row_ptr), _p(A.col_ind), _p(A.values), _p(dis_row),
                                   _p(dis_col), _stream())
    return A


def gcn_norm_rows_degrees(A: CSR, row_offset: int, dis_out: torch.Tensor, row_order=None):
    """Pass 1 of gcn_norm on a row block: (row_ptr of the self-looped block,
    per-row insertion offsets); 1/sqrt(deg) into ``dis_out`` (float32[n_rows]).
    ``row_order`` (or A's own schedule) only orders the work."""
    N = A.n_rows
    dev = A.row_ptr.device
    rp = torch.empty(N + 1, dtype=torch.int32, device=dev)
    ins = torch.empty(max(N, 1), dtype=torch.int32, device=dev)
    _csr_call((A,), lib.tg_gcn_norm_rows_degrees_f32, N, row_offset, A.nnz, _p(A.row_ptr), _p(A.col_ind), _p(A.values),
                                           _p(_ord(A, row_order)), _p(rp), _p(ins), _p(dis_out), _stream())
    return rp, ins


def gcn_norm_rows_fill(A: CSR, row_offset: int, rp_out: torch.Tensor, insert: torch.Tensor, dis_row: torch.Tensor,
                       dis_col: torch.Tensor, row_order=None) -> CSR:
    """Pass 2 of gcn_norm on a row block: the self-looped rows, values scaled
    (v * dis_row[i]) * dis_col[j] (global columns).  The result keeps A's row
    schedule: its rows have the same lengths, plus one where a diagonal was
    inserted."""
    N = A.n_rows
    cap = A.nnz + N
    dev = A.row_ptr.device
    order = _ord(A, row_order)
    ci = torch.empty(max(cap, 1), dtype=torch.int32, device=dev)
    v = torch.empty(max(cap, 1), dtype=torch.float32, device=dev)
    _csr_call((A,), lib.tg_gcn_norm_rows_fill_f32, N, row_offset, dis_col.numel(), _p(A.row_ptr), _p(A.col_ind),
              _p(A.values), _p(order), _p(rp_out), _p(insert), _p(dis_row), _p(dis_col), _p(ci), _p(v), _stream())
    nnz = int(rp_out[N].item()) if N else 0  # after both passes are queued
    return CSR(N, A.n_cols, rp_out, ci[:nnz], v[:nnz], order, validated=True)


def gcn_norm_scale(A: CSR, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """FAST gcn_norm as per-row factors: dis[i] = 1/sqrt(sum of row i's values + 1)."""
    if out is None:
        out = torch.empty(A.n_rows, dtype=torch.float32, device=A.row_ptr.device)
    nnz = A.nnz
    _csr_call((A,), lib.tg_gcn_norm_scale_f32, A.n_rows, nnz, _p(A.row_ptr), _p(A.values), _p(out), _stream())
    return out


def gcn_aggregate(A: CSR, Hs: torch.Tensor, Hs_self: torch.Tensor, dis: torch.Tensor, bias=None, act=None,
                  out: Optional[torch.Tensor] = None, seg_begin=None, seg_end=None, carry: bool = False,
                  last: bool = True, row_order=None) -> torch.Tensor:
    """out_i = act(dis[i] * (sum_j a_ij Hs[j] + Hs_self[i]) + bias): the GCN
    aggregation of D^-1/2 (A + I) D^-1/2 without a normalised copy of A
    (Hs = diag(dis) . HW over all nodes).  Optional column-block pass."""
    Hs, Hs_self = _dense(Hs, "Hs"), _dense(Hs_self, "Hs_self")
    F = Hs.shape[1]
    if out is None:
        out = torch.empty((A.n_rows, F), dtype=torch.float32, device=Hs.device)
    b = _vec(bias)
    flags = FLAG_B_ROWS_PADDED if _padded(Hs) else 0
    _csr_call((A,), lib.tg_gcn_aggregate_f32, A.n_rows, A.n_cols, A.nnz, _p(A.row_ptr), _p(A.col_ind), _p(A.values),
              _p(Hs), F, _ld(Hs), _p(Hs_self), _ld(Hs_self), _p(dis), _p(b), ACT[act], _p(out), _ld(out),
              _p(_ord(A, row_order)), _p(seg_begin), _p(seg_end), int(carry), int(last), flags, _stream())
    return out


def csr_validate(A: CSR) -> None:
    """Tensor::sparse_csr's checks (src/tensor.cpp:46-86) on device arrays."""
    check(lib.tg_csr_validate(A.n_rows, A.n_cols, A.nnz, _p(A.row_ptr), _p(A.col_ind), _stream()))


# ── layers ───────────────────────────────────────────────────────────────────
def gcn_layer(A_norm: CSR, H: torch.Tensor, W: torch.Tensor, bias=None, act="relu", row_order=None,
              out=None, mode: str = "exact") -> torch.Tensor:
    """GCNLayer::forward (src/layers.cpp:286)."""
    H, W = _dense(H, "H"), _dense(W, "W").contiguous()
    N, F_out = A_norm.n_rows, W.shape[1]
    if out is None:
        out = torch.empty((N, F_out), dtype=torch.float32, device=H.device)
    b = _vec(bias)
    _csr_call((A_norm,), lib.tg_gcn_layer_f32, N, A_norm.nnz, _p(A_norm.row_ptr), _p(A_norm.col_ind), _p(A_norm.values), _p(H),
                               _ld(H), W.shape[0], F_out, _p(W), _p(b), ACT[act], _p(out), _ld(out),
                               _p(_ord(A_norm, row_order)), MODE[mode], _stream())
    return out


def sage_layer(A: CSR, H: torch.Tensor, W_neigh: torch.Tensor, W_self: torch.Tensor, bias=None,
               aggregator: str = "mean", act="relu", row_order=None, out=None, mode: str = "exact"):
    """SAGELayer::forward (src/layers.cpp:538)."""
    H = _dense(H, "H")
    Wn, Ws = _dense(W_neigh, "W_neigh").contiguous(), _dense(W_self, "W_self").contiguous()
    N, F_out = A.n_rows, Wn.shape[1]
    if out is None:
        out = torch.empty((N, F_out), dtype=torch.float32, device=H.device)
    b = _vec(bias)
    _csr_call((A,), lib.tg_sage_layer_f32, N, A.nnz, _p(A.row_ptr), _p(A.col_ind), _p(H), _ld(H), Wn.shape[0], F_out,
                                _p(Wn), _p(Ws), _p(b), _lib.AGG_MAX if aggregator == "max" else _lib.AGG_MEAN,
                                ACT[act], _p(out), _ld(out), _p(_ord(A, row_order)), MODE[mode], _stream())
    return out


def gat_layer(A_sl: CSR, H: torch.Tensor, W: torch.Tensor, a_left: torch.Tensor, a_right: torch.Tensor,
              heads: int = 1, bias=None, negative_slope: float = 0.2, concat: bool = True, act=None,
              row_order=None, out=None, mode: str = "exact") -> torch.Tensor:
    """Multi-head GATLayer::forward + head concat/average (src/layers.cpp:945, src/model.cpp:403).

    W is F_in x (heads*F_out) with head h in columns [h*F_out, (h+1)*F_out);
    a_left / a_right / bias are heads x F_out.
    """
    H, W = _dense(H, "H"), _dense(W, "W").contiguous()
    F_out = W.shape[1] // heads
    al, ar, b = _vec(a_left), _vec(a_right), _vec(bias)
    N = A_sl.n_rows
    if out is None:
        out = torch.empty((N, heads * F_out if concat else F_out), dtype=torch.float32, device=H.device)
    _csr_call((A_sl,), lib.tg_gat_layer_f32, N, A_sl.nnz, _p(A_sl.row_ptr), _p(A_sl.col_ind), _p(H), _ld(H), W.shape[0], heads,
                               F_out, _p(W), _p(al), _p(ar), _p(b), negative_slope, int(concat), ACT[act],
                               _p(out), _ld(out), _p(_ord(A_sl, row_order)), MODE[mode], _stream())
    return out


def take_device_error() -> None:
    """Raise if a tensor-core GEMM pipeline wait timed out since the last call."""
    check(lib.tg_take_device_error(_stream()))


# ── Fused GEMM -> exchange over NVLink ──────────────────────────────────────
def ipc_get_handle(t: torch.Tensor):
    """(handle bytes, offset): a CUDA IPC handle of the allocation holding t, and t's offset in it."""
    h = C.create_string_buffer(64)
    off = C.c_int64()
    check(lib.tg_ipc_get_handle(_p(t), h, C.byref(off)))
    return h.raw, off.value


def ipc_open_handle(handle: bytes) -> int:
    """Map another process's allocation; returns its base address here."""
    base = C.c_void_p()
    check(lib.tg_ipc_open_handle(C.create_string_buffer(handle, 64), C.byref(base)))
    return base.value


def ipc_close_handle(base: int) -> None:
    check(lib.tg_ipc_close_handle(C.c_void_p(base)))


def gemm_peers(A: torch.Tensor, B: torch.Tensor, out: torch.Tensor, peer_out, peer_flags, bias=None, act=None,
               alpha: float = 0.0, cols_padded: bool = False, row_scale=None) -> torch.Tensor:
    """out = act(A . B + bias) on the tensor cores (rows scaled by
    ``row_scale`` before the bias when given), every row also stored at
    the same offset of each peer_out[p] (device addresses of other GPUs'
    copies, same leading dimension); after each 128-row tile the counter at
    peer_flags[p] is incremented (release, system scope)."""
    A, B = _dense(A, "A"), _dense(B, "B")
    M, K = A.shape
    N = B.shape[1]
    n = len(peer_out)
    pc = (C.c_void_p * max(1, n))(*peer_out)
    pf = (C.c_void_p * max(1, n))(*peer_flags)
    b = _vec(bias)
    check(lib.tg_gemm_peers_f32(M, N, K, _p(A), _ld(A), _p(B), _ld(B), _p(out), _ld(out), _p(b), ACT[act], alpha,
                                _p(row_scale), n, pc, pf, FLAG_C_COLS_PADDED if cols_padded else 0, _stream()))
    return out


def wait_flags(flags: torch.Tensor, targets, timeout_ns: int = 2_000_000_000) -> None:
    """Device-side wait (in stream order) until flags[i] >= targets[i] for every i (0 = skip)."""
    n = len(targets)
    t = (C.c_uint64 * max(1, n))(*targets)
    check(lib.tg_wait_flags(_p(flags), t, n, int(timeout_ns), _stream()))
