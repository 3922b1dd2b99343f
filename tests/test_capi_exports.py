"""The C-ABI library loads and exports every entry point the headers declare (CPU)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, "include")


def declared_symbols():
    names = set()
    for fn in os.listdir(INCLUDE):
        if fn.endswith(".h"):
            src = open(os.path.join(INCLUDE, fn)).read()
            names |= set(re.findall(r"TG_API\s+[\w\s\*]+?\b(tg_\w+)\s*\(", src))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "tg_spmm_f32" in names and "tg_gemm_f32" in names and len(names) >= 20


def test_library_exports_every_declared_symbol():
    from tinygnn_b200 import _lib
    missing = [n for n in declared_symbols() if not hasattr(_lib.lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_python_binding_covers_every_declared_symbol():
    from tinygnn_b200 import _lib
    unbound = [n for n in declared_symbols() if n not in _lib.SIGNATURES]
    assert not unbound, f"declared but not bound in _lib.SIGNATURES: {unbound}"


def test_library_metadata_calls():
    from tinygnn_b200 import _lib
    assert _lib.lib.tg_abi_version() == 2
    assert b"sm_100a" in _lib.lib.tg_version()
    assert _lib.lib.tg_device_count() >= 0


def test_library_is_built_for_sm100a_only():
    """The fatbin targets sm_100a (reads the ELF section names only)."""
    from tinygnn_b200 import _lib
    data = open(_lib.LIB_PATH, "rb").read()
    assert b".nv_fatbin" in data


def test_no_cpu_fallback_when_library_missing(tmp_path, monkeypatch):
    """Importing the package without the built library, where nvcc is not
    there to build it, fails loudly."""
    import importlib
    import shutil
    import sys
    from tinygnn_b200 import _lib, build
    hidden = {_lib.LIB_PATH, build.NVCC}
    monkeypatch.setattr(os.path, "exists", lambda p, _e=os.path.exists: False if p in hidden else _e(p))
    monkeypatch.setattr(shutil, "which", lambda *a, **k: None)
    saved = {k: sys.modules.pop(k) for k in list(sys.modules) if k.startswith("tinygnn_b200")}
    try:
        with pytest.raises(ImportError):
            importlib.import_module("tinygnn_b200._lib")
    finally:
        for k in list(sys.modules):
            if k.startswith("tinygnn_b200"):
                del sys.modules[k]
        sys.modules.update(saved)


def test_compute_call_without_device_reports_no_device():
    """On a host without a GPU the status is TG_ERR_NO_DEVICE, never a CPU result."""
    from tinygnn_b200 import _lib
    if _lib.lib.tg_device_count() > 0:
        pytest.skip("a device is present")
    st = _lib.lib.tg_gemm_f32(1, 1, 1, None, 1, None, 1, None, 1, None, 0, 0.0, 0, None)
    assert st == _lib.NO_DEVICE
    assert "no CUDA device" in _lib.last_error()


def test_handle_calls_without_device_report_no_device():
    """The handle C ABI (tg_tensor_* / tg_model_*) has no CPU path either."""
    import ctypes as C
    from tinygnn_b200 import _lib
    if _lib.lib.tg_device_count() > 0:
        pytest.skip("a device is present")
    h = C.c_void_p()
    rp = (C.c_int32 * 2)(0, 0)
    assert _lib.lib.tg_tensor_create_csr(1, 1, 0, C.cast(rp, C.c_void_p), None, None, C.byref(h)) == _lib.NO_DEVICE
    assert _lib.lib.tg_tensor_create_dense(2, 2, None, 2, C.byref(h)) == _lib.NO_DEVICE
    assert "no CUDA device" in _lib.last_error()
    m = C.c_void_p()
    assert _lib.lib.tg_model_create(C.byref(m)) == _lib.OK  # host-side object
    assert _lib.lib.tg_model_add_gcn(m, 4, 2, 1, _lib.ACT_RELU, 0) == _lib.OK
    assert _lib.lib.tg_model_add_gcn(m, 0, 2, 1, _lib.ACT_RELU, 0) == _lib.INVALID_ARGUMENT
    assert _lib.lib.tg_model_forward_host(m, 1, 0, C.cast(rp, C.c_void_p), None, None, None, 4, 4, None, 2,
                                          2) == _lib.NO_DEVICE
    _lib.lib.tg_model_free(m)


def test_dist_partition_csr_rows_and_entries():
    """tg_dist_partition_csr: equal row blocks of ceil(n / world) rows and
    their entry ranges (host only, no device needed)."""
    import numpy as np
    from tinygnn_b200.handles import partition_rows
    rp = np.array([0, 2, 2, 5, 9, 9, 12, 13], np.int32)  # n = 7
    blocks = [partition_rows(3, r, 7, rp) for r in range(3)]
    assert blocks == [(0, 3, 0, 5), (3, 6, 5, 12), (6, 7, 12, 13)]
    assert partition_rows(4, 2, 5) == (4, 5, None, None)      # R = 2: rank 2 holds the last row
    assert partition_rows(4, 3, 5)[:2] == (5, 5)              # ... and rank 3 none
    from tinygnn_b200 import _lib
    assert _lib.lib.tg_dist_partition_csr(2, 2, 5, None, None, None, None, None) == _lib.INVALID_ARGUMENT


def test_dist_init_without_device_reports_no_device(tmp_path):
    import ctypes as C
    from tinygnn_b200 import _lib
    if _lib.lib.tg_device_count() > 0:
        pytest.skip("a device is present")
    h = C.c_void_p()
    st = _lib.lib.tg_dist_init(1, 0, 0, str(tmp_path / "id").encode(), 1000, C.byref(h))
    assert st == _lib.NO_DEVICE
