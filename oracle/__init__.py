"""TEST INFRASTRUCTURE ONLY -- the parity checker for the CUDA path.

Two CPU implementations of the TinyGNN hot path, both behind numpy-in /
numpy-out functions with identical signatures:

* ``port`` -- oracle/tg_oracle.c, a plain-C restatement of the reference
  algorithms (each function cites the reference lines it follows).
* ``ref``  -- oracle/_ref/libtinygnn_ref.so, the reference library itself,
  compiled from its own sources by oracle/Makefile (None when not built).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline and
reference legs may import this package.  The product (``tinygnn_b200``)
never does: it has no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(_HERE, "_build", "libtg_oracle.so")
REF_SO = os.path.join(_HERE, "_ref", "libtinygnn_ref.so")

_i64, _i32, _f32, _vp = C.c_int64, C.c_int, C.c_float, C.c_void_p


def build(quiet: bool = True, target: str = "all") -> None:
    """Build the oracle libraries (the reference one only where its sources
    exist), serialised across processes by a lock file."""
    import fcntl
    import subprocess

    os.makedirs(os.path.join(_HERE, "_build"), exist_ok=True)
    with open(os.path.join(_HERE, "_build", ".build.lock"), "w") as lk:
        fcntl.flock(lk, fcntl.LOCK_EX)
        try:
            subprocess.run(["make", "-C", _HERE, "-j8", target], check=True,
                           stdout=subprocess.DEVNULL if quiet else None)
        finally:
            fcntl.flock(lk, fcntl.LOCK_UN)


def _p(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(_vp)


def _f(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _i(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


class OracleError(RuntimeError):
    """Raised when the reference library rejects an input."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code  # 1 invalid_argument, 2 out_of_range, 3 other


ACT = {"relu": 0, "leaky_relu": 1, "elu": 2, "sigmoid": 3, "tanh": 4,
       "gelu": 5, "softmax": 6, "log_softmax": 7}


class _Port:
    """Numpy wrappers over the C restatement."""

    name = "port"

    def __init__(self, path: str):
        L = self.lib = C.CDLL(path)
        L.orc_matmul.argtypes = [_i64, _i64, _i64, _vp, _vp, _vp]
        L.orc_spmm.argtypes = [_i64, _vp, _vp, _vp, _vp, _i64, _vp]
        L.orc_activation.argtypes = [_i32, _f32, _vp, _i64, _i64]
        L.orc_activation.restype = _i32
        L.orc_add_bias.argtypes = [_vp, _i64, _i64, _vp]
        for fn in (L.orc_add_self_loops, L.orc_gcn_norm):
            fn.argtypes = [_i64, _vp, _vp, _vp, _vp, _vp, _vp]
            fn.restype = _i64
        L.orc_edge_list_to_csr.argtypes = [_i64, _i64, _vp, _vp, _vp, _vp, _vp]
        L.orc_edge_list_to_csr.restype = _i64
        L.orc_edge_softmax.argtypes = [_i64, _vp, _vp, _vp]
        L.orc_sage_max_aggregate.argtypes = [_i64, _vp, _vp, _vp, _i64, _vp]
        L.orc_gcn_layer.argtypes = [_i64, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _i32, _vp]
        L.orc_sage_layer.argtypes = [_i64, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _i32, _i32, _vp]
        L.orc_gat_layer.argtypes = [_i64, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _f32, _i32, _vp]
        L.orc_max_threads.restype = _i32
        L.orc_set_num_threads.argtypes = [_i32]

    def max_threads(self) -> int:
        return self.lib.orc_max_threads()

    def set_num_threads(self, n: int) -> None:
        self.lib.orc_set_num_threads(n)

    def matmul(self, A, B):
        A, B = _f(A), _f(B)
        M, K = A.shape
        N = B.shape[1]
        out = np.empty((M, N), np.float32)
        self.lib.orc_matmul(M, K, N, _p(A), _p(B), _p(out))
        return out

    def spmm(self, rp, ci, v, B):
        rp, ci, v, B = _i(rp), _i(ci), _f(v), _f(B)
        M = rp.size - 1
        out = np.empty((M, B.shape[1]), np.float32)
        self.lib.orc_spmm(M, _p(rp), _p(ci), _p(v), _p(B), B.shape[1], _p(out))
        return out

    def activation(self, kind, X, alpha=0.0):
        X = np.array(X, dtype=np.float32, copy=True, order="C")
        rows, cols = X.shape
        if self.lib.orc_activation(ACT[kind], alpha, _p(X), rows, cols):
            raise OracleError(1, f"{kind}: tensor has 0 columns")
        return X

    def add_bias(self, X, b):
        X = np.array(X, dtype=np.float32, copy=True, order="C")
        b = _f(b).reshape(-1)
        self.lib.orc_add_bias(_p(X), X.shape[0], X.shape[1], _p(b))
        return X

    def _csr_out(self, fn, rp, ci, v):
        rp, ci, v = _i(rp), _i(ci), _f(v)
        N = rp.size - 1
        cap = ci.size + N
        rpo = np.empty(N + 1, np.int32)
        cio = np.empty(max(cap, 1), np.int32)
        vo = np.empty(max(cap, 1), np.float32)
        nnz = fn(N, _p(rp), _p(ci), _p(v), _p(rpo), _p(cio), _p(vo))
        return rpo, cio[:nnz].copy(), vo[:nnz].copy()

    def add_self_loops(self, rp, ci, v):
        return self._csr_out(self.lib.orc_add_self_loops, rp, ci, v)

    def gcn_norm(self, rp, ci, v):
        return self._csr_out(self.lib.orc_gcn_norm, rp, ci, v)

    def edge_list_to_csr(self, src, dst, num_nodes):
        src, dst = _i(src), _i(dst)
        E = src.size
        rp = np.empty(num_nodes + 1, np.int32)
        ci = np.empty(max(E, 1), np.int32)
        v = np.empty(max(E, 1), np.float32)
        bad = self.lib.orc_edge_list_to_csr(num_nodes, E, _p(src), _p(dst), _p(rp), _p(ci), _p(v))
        if bad >= 0:
            raise OracleError(1, f"edge[{bad}] out of range [0, {num_nodes})")
        return rp, ci[:E].copy(), v[:E].copy()

    def edge_softmax(self, rp, ci, v):
        rp, v = _i(rp), _f(v)
        out = np.zeros_like(v)
        self.lib.orc_edge_softmax(rp.size - 1, _p(rp), _p(v), _p(out))
        return out

    def sage_max_aggregate(self, rp, ci, v, H):
        rp, ci, H = _i(rp), _i(ci), _f(H)
        N = rp.size - 1
        out = np.empty((N, H.shape[1]), np.float32)
        self.lib.orc_sage_max_aggregate(N, _p(rp), _p(ci), _p(H), H.shape[1], _p(out))
        return out

    def gcn_layer(self, rp, ci, v, H, W, bias=None, relu=True):
        rp, ci, v, H, W = _i(rp), _i(ci), _f(v), _f(H), _f(W)
        b = None if bias is None else _f(bias).reshape(-1)
        N = rp.size - 1
        out = np.empty((N, W.shape[1]), np.float32)
        self.lib.orc_gcn_layer(N, _p(rp), _p(ci), _p(v), _p(H), W.shape[0], W.shape[1],
                               _p(W), _p(b), int(relu), _p(out))
        return out

    def sage_layer(self, rp, ci, v, H, Wn, Ws, bias=None, agg="mean", relu=True):
        rp, ci, H, Wn, Ws = _i(rp), _i(ci), _f(H), _f(Wn), _f(Ws)
        b = None if bias is None else _f(bias).reshape(-1)
        N = rp.size - 1
        out = np.empty((N, Wn.shape[1]), np.float32)
        self.lib.orc_sage_layer(N, _p(rp), _p(ci), _p(H), Wn.shape[0], Wn.shape[1], _p(Wn),
                                _p(Ws), _p(b), int(agg == "max"), int(relu), _p(out))
        return out

    def gat_layer(self, rp, ci, v, H, W, a_l, a_r, bias=None, slope=0.2, relu=False):
        rp, ci, H, W = _i(rp), _i(ci), _f(H), _f(W)
        al, ar = _f(a_l).reshape(-1), _f(a_r).reshape(-1)
        b = None if bias is None else _f(bias).reshape(-1)
        N = rp.size - 1
        out = np.empty((N, W.shape[1]), np.float32)
        self.lib.orc_gat_layer(N, _p(rp), _p(ci), _p(H), W.shape[0], W.shape[1], _p(W),
                               _p(al), _p(ar), _p(b), slope, int(relu), _p(out))
        return out


class _Ref:
    """Numpy wrappers over the reference library (same signatures as _Port)."""

    name = "ref"

    def __init__(self, path: str):
        L = self.lib = C.CDLL(path)
        L.ref_last_error.restype = C.c_char_p
        L.ref_set_num_threads.argtypes = [_i32]
        L.ref_get_max_threads.restype = _i32
        L.ref_matmul.argtypes = [_i64, _i64, _i64, _vp, _vp, _vp]
        L.ref_spmm.argtypes = [_i64, _i64, _i64, _vp, _vp, _vp, _vp, _i64, _vp]
        L.ref_activation.argtypes = [_i32, _f32, _vp, _i64, _i64]
        L.ref_add_bias.argtypes = [_vp, _i64, _i64, _vp, _i64, _i64]
        for fn in (L.ref_add_self_loops, L.ref_gcn_norm):
            fn.argtypes = [_i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, C.POINTER(_i64)]
        L.ref_edge_softmax.argtypes = [_i64, _i64, _i64, _vp, _vp, _vp, _vp]
        L.ref_sage_max_aggregate.argtypes = [_i64, _i64, _i64, _vp, _vp, _vp, _vp, _i64, _vp]
        L.ref_edge_list_to_csr.argtypes = [_i64, _i64, _vp, _vp, _vp, _vp, _vp]
        L.ref_gcn_layer.argtypes = [_i64, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _i32, _vp]
        L.ref_sage_layer.argtypes = [_i64, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp,
                                     _i32, _i32, _vp]
        L.ref_gat_layer.argtypes = [_i64, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp,
                                    _vp, _f32, _i32, _vp]
        L.ref_model_create.restype = _vp
        L.ref_model_free.argtypes = [_vp]
        L.ref_model_add_gcn.argtypes = [_vp, _i64, _i64, _i32, _i32, _i32]
        L.ref_model_add_sage.argtypes = [_vp, _i64, _i64, _i32, _i32, _i32, _i32]
        L.ref_model_add_gat.argtypes = [_vp, _i64, _i64, _i64, _i32, _f32, _i32, _i32, _i32]
        L.ref_model_set_tensor.argtypes = [_vp, C.c_char_p, _vp, _i64, _i64]
        L.ref_model_load.argtypes = [_vp]
        L.ref_model_load_file.argtypes = [_vp, C.c_char_p]
        L.ref_model_forward.argtypes = [_vp, _i64, _i64, _vp, _vp, _vp, _vp, _i64, _vp]
        L.ref_tensor_csr.argtypes = [_i64, _i64, _vp, _vp, _vp]
        L.ref_tensor_csr.restype = _vp
        L.ref_tensor_dense.argtypes = [_i64, _i64, _vp]
        L.ref_tensor_dense.restype = _vp
        L.ref_tensor_free.argtypes = [_vp]
        L.ref_model_forward_tensors.argtypes = [_vp, _vp, _vp, _vp, _i32]
        L.ref_spmm_tensors.argtypes = [_vp, _vp, _vp]
        L.ref_stack_create.restype = _vp
        L.ref_stack_free.argtypes = [_vp]
        L.ref_stack_add_gcn.argtypes = [_vp, _i64, _i64, _i32, _i32, _vp, _vp]
        L.ref_stack_add_sage.argtypes = [_vp, _i64, _i64, _i32, _i32, _i32, _vp, _vp, _vp]
        L.ref_gcn_norm_tensor.argtypes = [_vp]
        L.ref_gcn_norm_tensor.restype = _vp
        L.ref_stack_forward_tensors.argtypes = [_vp, _vp, _vp, _vp, _i32, _vp]

    def _chk(self, rc: int) -> None:
        if rc:
            raise OracleError(rc, self.lib.ref_last_error().decode())

    def set_num_threads(self, n: int) -> None:
        self.lib.ref_set_num_threads(n)

    def max_threads(self) -> int:
        return self.lib.ref_get_max_threads()

    def matmul(self, A, B):
        A, B = _f(A), _f(B)
        if A.shape[1] != B.shape[0]:
            raise OracleError(1, "matmul: dimension mismatch")
        out = np.empty((A.shape[0], B.shape[1]), np.float32)
        self._chk(self.lib.ref_matmul(A.shape[0], A.shape[1], B.shape[1], _p(A), _p(B), _p(out)))
        return out

    def spmm(self, rp, ci, v, B, n_cols=None):
        rp, ci, v, B = _i(rp), _i(ci), _f(v), _f(B)
        M = rp.size - 1
        K = B.shape[0] if n_cols is None else n_cols
        out = np.empty((M, B.shape[1]), np.float32)
        self._chk(self.lib.ref_spmm(M, K, ci.size, _p(rp), _p(ci), _p(v), _p(B), B.shape[1], _p(out)))
        return out

    def activation(self, kind, X, alpha=0.0):
        X = np.array(X, dtype=np.float32, copy=True, order="C")
        self._chk(self.lib.ref_activation(ACT[kind], alpha, _p(X), X.shape[0], X.shape[1]))
        return X

    def add_bias(self, X, b):
        X = np.array(X, dtype=np.float32, copy=True, order="C")
        b = _f(b)
        b2 = b.reshape(1, -1) if b.ndim == 1 else b
        self._chk(self.lib.ref_add_bias(_p(X), X.shape[0], X.shape[1], _p(b2), b2.shape[0], b2.shape[1]))
        return X

    def _csr_out(self, fn, rp, ci, v):
        rp, ci, v = _i(rp), _i(ci), _f(v)
        N = rp.size - 1
        cap = _i64(ci.size + N)
        rpo = np.empty(N + 1, np.int32)
        cio = np.empty(max(cap.value, 1), np.int32)
        vo = np.empty(max(cap.value, 1), np.float32)
        self._chk(fn(N, ci.size, _p(rp), _p(ci), _p(v), _p(rpo), _p(cio), _p(vo), C.byref(cap)))
        return rpo, cio[:cap.value].copy(), vo[:cap.value].copy()

    def add_self_loops(self, rp, ci, v):
        return self._csr_out(self.lib.ref_add_self_loops, rp, ci, v)

    def gcn_norm(self, rp, ci, v):
        return self._csr_out(self.lib.ref_gcn_norm, rp, ci, v)

    def edge_list_to_csr(self, src, dst, num_nodes):
        src, dst = _i(src), _i(dst)
        E = src.size
        rp = np.empty(num_nodes + 1, np.int32)
        ci = np.empty(max(E, 1), np.int32)
        v = np.empty(max(E, 1), np.float32)
        self._chk(self.lib.ref_edge_list_to_csr(num_nodes, E, _p(src), _p(dst), _p(rp), _p(ci), _p(v)))
        return rp, ci[:E].copy(), v[:E].copy()

    def edge_softmax(self, rp, ci, v, n_cols=None):
        rp, ci, v = _i(rp), _i(ci), _f(v)
        N = rp.size - 1
        out = np.zeros_like(v)
        self._chk(self.lib.ref_edge_softmax(N, N if n_cols is None else n_cols, v.size,
                                            _p(rp), _p(ci), _p(v), _p(out)))
        return out

    def sage_max_aggregate(self, rp, ci, v, H):
        rp, ci, v, H = _i(rp), _i(ci), _f(v), _f(H)
        N = rp.size - 1
        out = np.empty((N, H.shape[1]), np.float32)
        self._chk(self.lib.ref_sage_max_aggregate(N, H.shape[0], ci.size, _p(rp), _p(ci), _p(v),
                                                  _p(H), H.shape[1], _p(out)))
        return out

    def gcn_layer(self, rp, ci, v, H, W, bias=None, relu=True):
        rp, ci, v, H, W = _i(rp), _i(ci), _f(v), _f(H), _f(W)
        b = None if bias is None else _f(bias).reshape(-1)
        N = rp.size - 1
        out = np.empty((N, W.shape[1]), np.float32)
        self._chk(self.lib.ref_gcn_layer(N, ci.size, _p(rp), _p(ci), _p(v), _p(H), W.shape[0],
                                         W.shape[1], _p(W), _p(b), int(relu), _p(out)))
        return out

    def sage_layer(self, rp, ci, v, H, Wn, Ws, bias=None, agg="mean", relu=True):
        rp, ci, v, H, Wn, Ws = _i(rp), _i(ci), _f(v), _f(H), _f(Wn), _f(Ws)
        b = None if bias is None else _f(bias).reshape(-1)
        N = rp.size - 1
        out = np.empty((N, Wn.shape[1]), np.float32)
        self._chk(self.lib.ref_sage_layer(N, ci.size, _p(rp), _p(ci), _p(v), _p(H), Wn.shape[0],
                                          Wn.shape[1], _p(Wn), _p(Ws), _p(b), int(agg == "max"),
                                          int(relu), _p(out)))
        return out

    def gat_layer(self, rp, ci, v, H, W, a_l, a_r, bias=None, slope=0.2, relu=False):
        rp, ci, v, H, W = _i(rp), _i(ci), _f(v), _f(H), _f(W)
        al, ar = _f(a_l).reshape(-1), _f(a_r).reshape(-1)
        b = None if bias is None else _f(bias).reshape(-1)
        N = rp.size - 1
        out = np.empty((N, W.shape[1]), np.float32)
        self._chk(self.lib.ref_gat_layer(N, ci.size, _p(rp), _p(ci), _p(v), _p(H), W.shape[0],
                                         W.shape[1], _p(W), _p(al), _p(ar), _p(b), slope,
                                         int(relu), _p(out)))
        return out

    def model(self, spec, weights):
        """A reference ``Model`` built from a layer spec and named weights."""
        return RefModel(self, spec, weights)

    def stack(self, spec, weights):
        """The same GCN / SAGE layers as reference layer objects (RefStack)."""
        return RefStack(self, spec, weights)


class RefModel:
    """The reference ``Model`` (src/model.cpp) driven through the shim.

    ``spec`` is a list of dicts: {"type": "gcn"|"sage"|"gat", "in", "out",
    "bias", "act", "post", "agg", "heads", "concat", "slope"}; ``weights``
    maps the reference's tensor names (model.cpp:258-305) to arrays.
    """

    POST = {None: 0, "none": 0, "relu": 1, "elu": 2}

    def __init__(self, ref: _Ref, spec, weights):
        self.ref, self.lib = ref, ref.lib
        self.h = self.lib.ref_model_create()
        for L in spec:
            act = 1 if L.get("act") == "relu" else 0
            post = self.POST[L.get("post")]
            bias = int(L.get("bias", True))
            if L["type"] == "gcn":
                rc = self.lib.ref_model_add_gcn(self.h, L["in"], L["out"], bias, act, post)
            elif L["type"] == "sage":
                rc = self.lib.ref_model_add_sage(self.h, L["in"], L["out"],
                                                 int(L.get("agg", "mean") == "max"), bias, act, post)
            else:
                rc = self.lib.ref_model_add_gat(self.h, L["in"], L["out"], L.get("heads", 1),
                                                int(L.get("concat", True)), L.get("slope", 0.2),
                                                bias, act, post)
            ref._chk(rc)
        for name, arr in weights.items():
            a = _f(arr)
            a2 = a.reshape(1, -1) if a.ndim == 1 else a
            ref._chk(self.lib.ref_model_set_tensor(self.h, name.encode(), _p(a2), a2.shape[0],
                                                   a2.shape[1]))
        ref._chk(self.lib.ref_model_load(self.h))
        self.out_cols = None
        last = spec[-1]
        self.out_cols = last["out"] * (last.get("heads", 1) if last["type"] == "gat" and
                                       last.get("concat", True) else 1)

    def forward(self, rp, ci, v, X):
        rp, ci, v, X = _i(rp), _i(ci), _f(v), _f(X)
        N = rp.size - 1
        out = np.empty((N, self.out_cols), np.float32)
        self.ref._chk(self.lib.ref_model_forward(self.h, N, ci.size, _p(rp), _p(ci), _p(v),
                                                 _p(X), X.shape[1], _p(out)))
        return out

    def __del__(self):
        try:
            self.lib.ref_model_free(self.h)
        except Exception:
            pass


class RefStack:
    """The reference's GCNLayer / SAGELayer objects of a GCN or SAGE ``spec``
    (as for :class:`RefModel`), run on pre-built Tensors: ``forward`` takes
    the normalised adjacency (GCN) and the raw one (SAGE) prepared once --
    the layer forwards of Model::forward without its per-call gcn_norm."""

    def __init__(self, ref: _Ref, spec, weights):
        self.ref, self.lib = ref, ref.lib
        self.h = self.lib.ref_stack_create()
        self._keep = []
        for li, L in enumerate(spec):
            act = 1 if L.get("act") == "relu" else 0
            post = RefModel.POST[L.get("post")]
            b = _f(weights[f"layer{li}.bias"]).reshape(-1) if L.get("bias", True) else None
            self._keep.append(b)
            if L["type"] == "gcn":
                W = _f(weights[f"layer{li}.weight"])
                self._keep.append(W)
                rc = self.lib.ref_stack_add_gcn(self.h, L["in"], L["out"], act, post, _p(W), _p(b))
            elif L["type"] == "sage":
                Wn, Ws = _f(weights[f"layer{li}.weight_neigh"]), _f(weights[f"layer{li}.weight_self"])
                self._keep += [Wn, Ws]
                rc = self.lib.ref_stack_add_sage(self.h, L["in"], L["out"], int(L.get("agg", "mean") == "max"),
                                                 act, post, _p(Wn), _p(Ws), _p(b))
            else:
                raise ValueError("RefStack: GCN and SAGE layers only")
            ref._chk(rc)
        self.out_cols = spec[-1]["out"]

    def gcn_norm_tensor(self, A):
        t = self.lib.ref_gcn_norm_tensor(A)
        if not t:
            raise OracleError(3, self.lib.ref_last_error().decode())
        return t

    def forward_tensors(self, A_norm, A_raw, X, log_softmax=True, rows=None):
        out = None if rows is None else np.empty((rows, self.out_cols), np.float32)
        self.ref._chk(self.lib.ref_stack_forward_tensors(self.h, A_norm, A_raw, X, int(log_softmax), _p(out)))
        return out

    def __del__(self):
        try:
            self.lib.ref_stack_free(self.h)
        except Exception:
            pass


def model_forward(impl, spec, weights, rp, ci, v, X):
    """Model::forward (src/model.cpp:359-439) composed from ``impl``'s layers.

    gcn_norm(A) for GCN layers and add_self_loops(A) for GAT layers are built
    once per call (365-381); layers run in order; a multi-head GAT layer runs
    each head and concatenates (312-332) or averages (335-354) them; then the
    post activation (426-435).  ``spec``/``weights`` as in :class:`RefModel`.
    """
    need_gcn = any(L["type"] == "gcn" for L in spec)
    need_sl = any(L["type"] == "gat" for L in spec)
    A_gcn = impl.gcn_norm(rp, ci, v) if need_gcn else None
    A_sl = impl.add_self_loops(rp, ci, v) if need_sl else None
    H = _f(X)
    for li, L in enumerate(spec):
        pre = f"layer{li}"
        relu = L.get("act") == "relu"
        bias = L.get("bias", True)
        if L["type"] == "gcn":
            H = impl.gcn_layer(*A_gcn, H, weights[f"{pre}.weight"],
                               weights[f"{pre}.bias"] if bias else None, relu)
        elif L["type"] == "sage":
            H = impl.sage_layer(rp, ci, v, H, weights[f"{pre}.weight_neigh"], weights[f"{pre}.weight_self"],
                                weights[f"{pre}.bias"] if bias else None, L.get("agg", "mean"), relu)
        else:
            heads = []
            for h in range(L.get("heads", 1)):
                hp = f"{pre}.head{h}"
                heads.append(impl.gat_layer(*A_sl, H, weights[f"{hp}.weight"], weights[f"{hp}.attn_left"],
                                            weights[f"{hp}.attn_right"],
                                            weights[f"{hp}.bias"] if bias else None,
                                            L.get("slope", 0.2), relu))
            if len(heads) == 1:
                H = heads[0]
            elif L.get("concat", True):
                H = np.ascontiguousarray(np.concatenate(heads, axis=1))
            else:
                acc = np.zeros_like(heads[0])
                for t in heads:
                    acc = (acc + t).astype(np.float32)
                H = (acc * np.float32(1.0 / len(heads))).astype(np.float32)
        post = L.get("post")
        if post == "relu":
            H = impl.activation("relu", H)
        elif post == "elu":
            H = impl.activation("elu", H, 1.0)
    return H


def _load(cls, path):
    return cls(path) if os.path.exists(path) else None


if not os.path.exists(PORT_SO):  # a fresh checkout: the C restatement builds anywhere gcc is
    build(target="oracle")
port = _load(_Port, PORT_SO)
ref = _load(_Ref, REF_SO)
