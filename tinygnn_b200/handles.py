"""Python side of the handle C ABI (tg_tensor_* / tg_model_*).

TinyGNN's drop-in Tensor and Model driven through the C ABI with host
buffers, as a caller binding C would: tensors uploaded from host arrays
(numpy or torch CPU tensors; pinned memory uploads at full PCIe rate), a
Model built layer by layer with named weights, forward, logits downloaded
into a host array.  Every call completes before it returns.
"""
from __future__ import annotations

import ctypes as C
from typing import Dict, Optional

import numpy as np

from . import _lib
from ._lib import check, lib


def _ptr(a) -> Optional[int]:
    """Host address of a C-contiguous numpy array or torch CPU tensor (None passes NULL)."""
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data


class HTensor:
    """A tg_tensor: TinyGNN's Tensor in device memory, owned by this object."""

    def __init__(self, handle: C.c_void_p):
        self.h = handle

    @classmethod
    def dense(cls, host, rows: int, cols: int, ld: Optional[int] = None) -> "HTensor":
        h = C.c_void_p()
        check(lib.tg_tensor_create_dense(rows, cols, _ptr(host), cols if ld is None else ld, C.byref(h)))
        return cls(h)

    @classmethod
    def csr(cls, rows: int, cols: int, row_ptr, col_ind, values=None) -> "HTensor":
        """From host row_ptr / col_ind (int32) and values (float32; None = all 1.0)."""
        nnz = int(row_ptr[rows]) if rows else 0
        h = C.c_void_p()
        check(lib.tg_tensor_create_csr(rows, cols, nnz, _ptr(row_ptr), _ptr(col_ind), _ptr(values), C.byref(h)))
        return cls(h)

    def shape(self):
        r, c, n = C.c_int64(), C.c_int64(), C.c_int64()
        f = C.c_int32()
        check(lib.tg_tensor_shape(self.h, C.byref(r), C.byref(c), C.byref(n), C.byref(f)))
        return r.value, c.value, n.value, bool(f.value)

    def download(self, out=None):
        """The values into ``out`` (a host float32 rows x cols array or tensor) or a new numpy array."""
        rows, cols, _, _ = self.shape()
        if out is None:
            out = np.empty((rows, cols), np.float32)
        check(lib.tg_tensor_download(self.h, _ptr(out), cols))
        return out

    def upload(self, host) -> "HTensor":
        """New values from the host, shape and structure kept: a dense tensor's
        rows (host rows x cols, C-contiguous), or a CSR tensor's nnz values."""
        ld = host.shape[1] if len(host.shape) == 2 else 0
        check(lib.tg_tensor_upload(self.h, _ptr(host), ld))
        return self

    def free(self) -> None:
        if self.h:
            lib.tg_tensor_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class HModel:
    """A tg_model: TinyGNN's Model (add_*_layer, load_weights, forward)."""

    POST = {None: 0, "none": 0, "relu": 1, "elu": 2}

    def __init__(self):
        self.h = C.c_void_p()
        check(lib.tg_model_create(C.byref(self.h)))

    @staticmethod
    def _act(a):
        return _lib.ACT_RELU if a == "relu" else _lib.ACT_NONE

    def add_gcn(self, fin: int, fout: int, bias: bool = True, act="relu", post=None) -> "HModel":
        check(lib.tg_model_add_gcn(self.h, fin, fout, int(bias), self._act(act), self.POST[post]))
        return self

    def add_sage(self, fin: int, fout: int, agg: str = "mean", bias: bool = True, act="relu", post=None) -> "HModel":
        check(lib.tg_model_add_sage(self.h, fin, fout, _lib.AGG_MAX if agg == "max" else _lib.AGG_MEAN, int(bias),
                                    self._act(act), self.POST[post]))
        return self

    def add_gat(self, fin: int, fout: int, heads: int = 1, concat: bool = True, slope: float = 0.2,
                bias: bool = True, act=None, post=None) -> "HModel":
        check(lib.tg_model_add_gat(self.h, fin, fout, heads, int(concat), slope, int(bias), self._act(act),
                                   self.POST[post]))
        return self

    def load_weights(self, weights: Dict[str, np.ndarray]) -> None:
        names = list(weights)
        arrs = [np.ascontiguousarray(weights[k], dtype=np.float32) for k in names]
        arrs = [a.reshape(1, -1) if a.ndim == 1 else a for a in arrs]
        n = len(names)
        cn = (C.c_char_p * n)(*[k.encode() for k in names])
        cd = (C.c_void_p * n)(*[a.ctypes.data for a in arrs])
        cr = (C.c_int64 * n)(*[a.shape[0] for a in arrs])
        cc = (C.c_int64 * n)(*[a.shape[1] for a in arrs])
        check(lib.tg_model_load_weights(self.h, n, cn, cd, cr, cc))

    def load_weights_file(self, path: str) -> None:
        check(lib.tg_model_load_weights_file(self.h, path.encode()))

    def forward(self, adjacency: HTensor, features: HTensor) -> HTensor:
        out = C.c_void_p()
        check(lib.tg_model_forward(self.h, adjacency.h, features.h, C.byref(out)))
        return HTensor(out)

    def forward_host(self, row_ptr, col_ind, values, features, feature_cols: int, out, out_cols: int):
        """Model::forward from host arrays in one call (tg_model_forward_host):
        the raw adjacency's CSR arrays (values None: unweighted) and the
        features (rows x >= feature_cols, C-contiguous) in; the last layer's
        output written into ``out`` (rows x >= out_cols).  Uploads overlap
        the compute; pinned torch tensors copy at full PCIe rate."""
        n = len(row_ptr) - 1
        nnz = int(row_ptr[n]) if n else 0
        ld_f = features.shape[1] if len(features.shape) == 2 else feature_cols
        ld_o = out.shape[1] if len(out.shape) == 2 else out_cols
        check(lib.tg_model_forward_host(self.h, n, nnz, _ptr(row_ptr), _ptr(col_ind), _ptr(values), _ptr(features),
                                        feature_cols, ld_f, _ptr(out), out_cols, ld_o))
        return out

    def capture(self, adjacency: HTensor, features: HTensor) -> "HGraph":
        """forward(adjacency, features) recorded as a CUDA graph (tg_model_capture)."""
        g = C.c_void_p()
        check(lib.tg_model_capture(self.h, adjacency.h, features.h, C.byref(g)))
        return HGraph(g, (adjacency, features))

    def free(self) -> None:
        if self.h:
            lib.tg_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class HGraph:
    """A tg_graph: a captured Model::forward, replayed on its input tensors."""

    def __init__(self, handle: C.c_void_p, inputs):
        self.h = handle
        self._inputs = inputs  # the graph reads their device memory: keep them alive

    def replay(self) -> "HGraph":
        check(lib.tg_graph_replay(self.h))
        return self

    def download(self, out):
        """The output into ``out`` (a host float32 rows x cols array or tensor)."""
        check(lib.tg_graph_download(self.h, _ptr(out), out.shape[1]))
        return out

    def free(self) -> None:
        if self.h:
            lib.tg_graph_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def set_fast_math(fast: bool) -> bool:
    """FAST (True) or EXACT arithmetic for the handle / C++ APIs; returns the previous setting."""
    return bool(lib.tg_set_fast_math(int(fast)))


def partition_rows(world: int, rank: int, n: int, row_ptr=None):
    """(row_begin, row_end, entry_begin, entry_end) of rank's equal row block
    (entries None without row_ptr) -- tg_dist_partition_csr."""
    vals = [C.c_int64() for _ in range(4)]
    rp = None if row_ptr is None else np.ascontiguousarray(row_ptr, dtype=np.int32)
    outs = [C.byref(v) for v in vals[:2]] + ([None, None] if rp is None else [C.byref(v) for v in vals[2:]])
    check(lib.tg_dist_partition_csr(world, rank, n, None if rp is None else rp.ctypes.data, *outs))
    rb, re_, eb, ee = (v.value for v in vals)
    return (rb, re_, eb, ee) if rp is not None else (rb, re_, None, None)


class HDist:
    """A tg_dist: this process's rank of the row-partitioned forward (NCCL)."""

    def __init__(self, world: int, rank: int, device: int, id_path: str, timeout_ms: int = 60000):
        self.h = C.c_void_p()
        self.world, self.rank = world, rank
        check(lib.tg_dist_init(world, rank, device, id_path.encode(), timeout_ms, C.byref(self.h)))

    def forward(self, model: HModel, n: int, adjacency_rows: HTensor, feature_rows: HTensor) -> HTensor:
        out = C.c_void_p()
        check(lib.tg_dist_forward(self.h, model.h, n, adjacency_rows.h, feature_rows.h, C.byref(out)))
        return HTensor(out)

    def finalize(self) -> None:
        if self.h:
            h, self.h = self.h, None
            check(lib.tg_dist_finalize(h))
