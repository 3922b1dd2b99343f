"""ctypes binding of the C ABI declared in include/tinygnn_b200.h.

The shared library lives in-tree at tinygnn_b200/lib/libtinygnn_b200.so and
is built by ``python tinygnn_b200/build.py`` (nvcc, sm_100a).  When it is
missing, importing this module builds it (``build.ensure_built``); where it
is missing and cannot be built (no nvcc), the import raises: the package
has no CPU path.
"""
from __future__ import annotations

import ctypes as C

from . import build as _build

LIB_PATH = _build.ensure_built()

lib = C.CDLL(LIB_PATH)

i64, i32, f32, vp, u64 = C.c_int64, C.c_int32, C.c_float, C.c_void_p, C.c_uint64
P64 = C.POINTER(C.c_int64)

# status codes (tg_status)
OK, INVALID_ARGUMENT, OUT_OF_RANGE, RUNTIME, CUDA, NCCL, TIMEOUT, DEVICE_CHECK, NO_DEVICE = range(9)
# activations (tg_activation)
ACT_NONE, ACT_RELU, ACT_ELU, ACT_LEAKY_RELU, ACT_SIGMOID, ACT_TANH, ACT_GELU = range(7)
AGG_MEAN, AGG_MAX = 0, 1
MODE_EXACT, MODE_FAST = 0, 1

# name -> (restype, argtypes); the exact list of entry points in the header.
SIGNATURES = {
    "tg_last_error_message": (C.c_char_p, []),
    "tg_version": (C.c_char_p, []),
    "tg_abi_version": (i32, []),
    "tg_device_count": (i32, []),
    "tg_kernel_launch_count": (u64, []),
    "tg_gemm_f32": (i32, [i64, i64, i64, vp, i64, vp, i64, vp, i64, vp, i32, f32, i32, vp]),
    "tg_gemm_pair_f32": (i32, [i64, i64, i64, vp, i64, vp, vp, i64, vp, i64, vp, i64, i32, vp]),
    "tg_gemm_cat_f32": (i32, [i64, i64, i64, vp, i64, i64, vp, i64, vp, i64, vp, i64, vp, i64, vp, i32, f32, i32, vp]),
    "tg_gemm_rowscale_f32": (i32, [i64, i64, i64, vp, i64, vp, i64, vp, i64, vp, vp, i32, f32, i32, vp]),
    "tg_gcn_norm_scale_f32": (i32, [i64, i64, vp, vp, vp, vp]),
    "tg_gcn_aggregate_f32": (i32, [i64, i64, i64, vp, vp, vp, vp, i64, i64, vp, i64, vp, vp, i32, vp, i64, vp, vp, vp,
                                   i32, i32, i32, vp]),
    "tg_gemm_dual_f32": (i32, [i64, i64, i64, vp, i64, vp, i64, vp, vp, i64, vp, i64, vp, i32, f32, vp]),
    "tg_activation_f32": (i32, [i32, f32, vp, i64, i64, i64, vp]),
    "tg_softmax_rows_f32": (i32, [vp, i64, i64, i64, vp]),
    "tg_log_softmax_rows_f32": (i32, [vp, i64, i64, i64, vp]),
    "tg_add_bias_f32": (i32, [vp, i64, i64, i64, vp, vp]),
    "tg_spmm_f32": (i32, [i64, i64, i64, vp, vp, vp, vp, i64, i64, vp, i64, vp, i32, f32, vp, i32, vp]),
    "tg_csr_degree_order": (i32, [i64, vp, vp, vp]),
    "tg_csr_column_splits": (i32, [i64, vp, vp, i32, i64, vp, vp]),
    "tg_spmm_segment_f32": (i32, [i64, i64, vp, vp, vp, vp, vp, vp, i64, i64, vp, i64, vp, i32, f32, vp, i32, i32,
                                  i32, vp]),
    "tg_sage_mean_combine_segment_f32": (i32, [i64, i64, vp, vp, vp, vp, vp, i64, i64, vp, i64, vp, i32, vp, i64,
                                               vp, i32, i32, i32, vp]),
    "tg_sage_aggregate_f32": (i32, [i64, i64, i64, vp, vp, vp, i64, i64, vp, i64, i32, vp]),
    "tg_sage_max_aggregate_f32": (i32, [i64, i64, i64, vp, vp, vp, i64, i64, vp, i64, vp]),
    "tg_sage_mean_combine_f32": (i32, [i64, i64, i64, vp, vp, vp, i64, i64, vp, i64, vp, i32, vp, i64, vp, i32,
                                       vp]),
    "tg_edge_softmax_f32": (i32, [i64, i64, vp, vp, vp, vp]),
    "tg_edge_list_to_csr": (i32, [i64, i64, vp, vp, vp, vp, vp, vp]),
    "tg_add_self_loops_f32": (i32, [i64, i64, vp, vp, vp, vp, vp, vp, P64, vp]),
    "tg_gcn_norm_f32": (i32, [i64, i64, vp, vp, vp, vp, vp, vp, P64, vp]),
    "tg_csr_validate": (i32, [i64, i64, i64, vp, vp, vp]),
    "tg_add_self_loops_rows_f32": (i32, [i64, i64, i64, vp, vp, vp, vp, vp, vp, P64, vp]),
    "tg_csr_degree_inv_sqrt_f32": (i32, [i64, vp, vp, vp, vp]),
    "tg_csr_scale_sym_f32": (i32, [i64, vp, vp, vp, vp, vp, vp]),
    "tg_gcn_norm_rows_degrees_f32": (i32, [i64, i64, i64, vp, vp, vp, vp, vp, vp, vp, vp]),
    "tg_gcn_norm_rows_fill_f32": (i32, [i64, i64, i64, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp]),
    "tg_set_csr_checks": (i32, [i32]),
    "tg_tensor_create_dense": (i32, [i64, i64, vp, i64, C.POINTER(vp)]),
    "tg_tensor_create_csr": (i32, [i64, i64, i64, vp, vp, vp, C.POINTER(vp)]),
    "tg_tensor_download": (i32, [vp, vp, i64]),
    "tg_tensor_upload": (i32, [vp, vp, i64]),
    "tg_tensor_shape": (i32, [vp, P64, P64, P64, C.POINTER(i32)]),
    "tg_tensor_free": (None, [vp]),
    "tg_model_create": (i32, [C.POINTER(vp)]),
    "tg_model_add_gcn": (i32, [vp, i64, i64, i32, i32, i32]),
    "tg_model_add_sage": (i32, [vp, i64, i64, i32, i32, i32, i32]),
    "tg_model_add_gat": (i32, [vp, i64, i64, i64, i32, f32, i32, i32, i32]),
    "tg_model_load_weights_file": (i32, [vp, C.c_char_p]),
    "tg_model_load_weights": (i32, [vp, i32, C.POINTER(C.c_char_p), C.POINTER(vp), P64, P64]),
    "tg_model_forward": (i32, [vp, vp, vp, C.POINTER(vp)]),
    "tg_model_forward_host": (i32, [vp, i64, i64, vp, vp, vp, vp, i64, i64, vp, i64, i64]),
    "tg_model_free": (None, [vp]),
    "tg_model_capture": (i32, [vp, vp, vp, C.POINTER(vp)]),
    "tg_graph_replay": (i32, [vp]),
    "tg_graph_download": (i32, [vp, vp, i64]),
    "tg_graph_free": (None, [vp]),
    "tg_set_fast_math": (i32, [i32]),
    "tg_dist_partition_csr": (i32, [i32, i32, i64, vp, P64, P64, P64, P64]),
    "tg_dist_init": (i32, [i32, i32, i32, C.c_char_p, i32, C.POINTER(vp)]),
    "tg_dist_forward": (i32, [vp, vp, i64, vp, vp, C.POINTER(vp)]),
    "tg_dist_finalize": (i32, [vp]),
    "tg_gcn_layer_f32": (i32, [i64, i64, vp, vp, vp, vp, i64, i64, i64, vp, vp, i32, vp, i64, vp, i32, vp]),
    "tg_sage_layer_f32": (i32, [i64, i64, vp, vp, vp, i64, i64, i64, vp, vp, vp, i32, i32, vp, i64, vp, i32, vp]),
    "tg_gat_layer_f32": (i32, [i64, i64, vp, vp, vp, i64, i64, i64, i64, vp, vp, vp, vp, f32, i32, i32, vp, i64,
                               vp, i32, vp]),
    "tg_take_device_error": (i32, [vp]),
    "tg_ipc_get_handle": (i32, [vp, vp, P64]),
    "tg_ipc_open_handle": (i32, [vp, C.POINTER(vp)]),
    "tg_ipc_close_handle": (i32, [vp]),
    "tg_gemm_peers_f32": (i32, [i64, i64, i64, vp, i64, vp, i64, vp, i64, vp, i32, f32, vp, i32, C.POINTER(vp),
                                C.POINTER(vp), i32, vp]),
    "tg_wait_flags": (i32, [vp, C.POINTER(u64), i32, i64, vp]),
    "tg_gcn_layer_noalloc_f32": (i32, [i64, i64, vp, vp, vp, vp, i64, i64, i64, vp, vp, i32, vp, i64, vp, vp]),
}

for _name, (_res, _args) in SIGNATURES.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


class TinyGNNError(RuntimeError):
    """A non-OK tg_status; ``status`` is the code."""

    def __init__(self, status: int, msg: str):
        super().__init__(msg)
        self.status = status


class InvalidArgument(TinyGNNError, ValueError):
    """std::invalid_argument in the reference."""


class OutOfRange(TinyGNNError, IndexError):
    """std::out_of_range in the reference."""


def last_error() -> str:
    return lib.tg_last_error_message().decode("utf-8", "replace")


def check(status: int) -> None:
    """Raise the Python exception matching a tg_status."""
    if status == OK:
        return
    msg = last_error()
    if status == INVALID_ARGUMENT:
        raise InvalidArgument(status, msg)
    if status == OUT_OF_RANGE:
        raise OutOfRange(status, msg)
    raise TinyGNNError(status, msg)


def launches() -> int:
    """Kernels this library has launched so far in this process."""
    return int(lib.tg_kernel_launch_count())
