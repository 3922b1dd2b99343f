"""tinygnn_b200 -- a B200-native GNN inference engine with TinyGNN's API.

The compute path is libtinygnn_b200.so (hand-written sm_100a CUDA kernels
behind the C ABI in include/tinygnn_b200.h).  This package is its Python
host side: ctypes bindings (``_lib``), torch-tensor front ends of every
entry point (``ops``), seeded synthetic inputs (``synth``) and the
row-partitioned multi-GPU driver (``dist``).  Importing it without the
built library raises: there is no CPU fallback.
"""
from . import _lib
from ._lib import InvalidArgument, OutOfRange, TinyGNNError, launches
from .ops import (CSR, add_bias_, add_self_loops, csr_validate, degree_order, edge_list_to_csr,
                  edge_softmax, elu_, gat_layer, gcn_layer, gcn_norm, gelu_, leaky_relu_, log_softmax_,
                  matmul, relu_, sage_aggregate, sage_layer, sage_max_aggregate, sigmoid_, softmax_,
                  spmm, tanh_)

__version__ = "0.1.0"


def version() -> str:
    return _lib.lib.tg_version().decode()


def device_count() -> int:
    return int(_lib.lib.tg_device_count())
