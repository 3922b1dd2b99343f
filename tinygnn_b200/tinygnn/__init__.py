"""TinyGNN's Python API, running on the B200.

The names, argument names, defaults and errors of TinyGNN's ``tinygnn``
package (python/tinygnn/__init__.py, re-exporting python/tinygnn_ext.cpp),
bound to this library's C++ API, so a TinyGNN user switches by changing the
import::

    import tinygnn_b200.tinygnn as tinygnn

    X = tinygnn.Tensor.from_numpy(features)            # copied into HBM
    A = tinygnn.Tensor.from_scipy_csr(adj)            # raw adjacency
    model = tinygnn.Model()
    model.add_gcn_layer(1433, 16)
    model.add_gcn_layer(16, 7, act=tinygnn.Activation.NONE)
    model.load_weights("weights_gcn.bin")
    logits = model.forward(A, X).to_numpy()

Every op runs on the current CUDA device (sm_100a kernels); tensors stay in
device memory between calls and are copied to the host only by
``to_numpy`` / ``*_numpy`` / ``at``.  Importing this package loads
libtinygnn_b200.so and the module over it, building both when they are
missing; where they cannot be built the import raises, never a CPU path.
"""
from __future__ import annotations

from .. import build as _build

_build.ensure_built(pymodule=True)

try:
    from ._core import (
        Activation,
        CoraData,
        GATLayer,
        GCNLayer,
        GraphData,
        GraphLoader,
        Model,
        SAGELayer,
        StorageFormat,
        Tensor,
        WeightFile,
        add_bias,
        add_self_loops,
        edge_softmax,
        elu_inplace,
        fast_math,
        gcn_norm,
        gelu_inplace,
        get_max_threads,
        leaky_relu_inplace,
        load_cora_binary,
        load_weight_file,
        log_softmax_inplace,
        matmul,
        relu_inplace,
        sage_max_aggregate,
        set_fast_math,
        set_num_threads,
        sigmoid_inplace,
        softmax_inplace,
        spmm,
        tanh_inplace,
    )
except ImportError as e:  # pragma: no cover - exercised only without a build
    raise ImportError("tinygnn_b200.tinygnn: the native module is not built "
                      "(run tinygnn_b200/build.py): " + str(e)) from e

__version__ = "0.1.5"

__all__ = [
    "StorageFormat",
    "Activation",
    "Tensor",
    "matmul",
    "spmm",
    "relu_inplace",
    "leaky_relu_inplace",
    "elu_inplace",
    "sigmoid_inplace",
    "tanh_inplace",
    "gelu_inplace",
    "softmax_inplace",
    "log_softmax_inplace",
    "add_bias",
    "add_self_loops",
    "gcn_norm",
    "edge_softmax",
    "sage_max_aggregate",
    "GCNLayer",
    "SAGELayer",
    "GATLayer",
    "Model",
    "CoraData",
    "WeightFile",
    "load_cora_binary",
    "load_weight_file",
    "GraphData",
    "GraphLoader",
    "set_num_threads",
    "get_max_threads",
    "set_fast_math",
    "fast_math",
]
