"""The build works from a clean checkout (CPU): the tracked files alone,
copied to a fresh directory with nothing built, give the native library,
the Python module and the oracle through ``__graft_entry__.build()`` --
the first thing that runs on a fresh machine."""
import os
import shutil
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _tracked_files():
    r = subprocess.run(["git", "-C", ROOT, "ls-files", "-z"], capture_output=True, check=True)
    return [p for p in r.stdout.decode().split("\0") if p]


def test_build_from_clean_checkout(tmp_path):
    if not os.path.isdir(os.path.join(ROOT, ".git")):
        import pytest
        pytest.skip("not a git checkout")
    dst = tmp_path / "repo"
    for rel in _tracked_files():
        src = os.path.join(ROOT, rel)
        if not os.path.isfile(src):
            continue  # tracked but deleted in the working tree
        os.makedirs(dst / os.path.dirname(rel), exist_ok=True)
        shutil.copy2(src, dst / rel)
    assert not (dst / "tinygnn_b200" / "lib").exists()
    code = ("import sys; sys.path.insert(0, '.'); import __graft_entry__ as g; g.build(); "
            "import tinygnn_b200, oracle; print(tinygnn_b200.version()); "
            "assert oracle.port is not None")
    r = subprocess.run([sys.executable, "-c", code], cwd=dst, capture_output=True, text=True, timeout=900,
                       env={k: v for k, v in os.environ.items() if k != "PYTHONPATH"})
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert (dst / "tinygnn_b200" / "lib" / "libtinygnn_b200.so").exists()
    assert (dst / "oracle" / "_build" / "libtg_oracle.so").exists()
    assert any(p.startswith("_core") for p in os.listdir(dst / "tinygnn_b200" / "tinygnn"))
    assert "sm_100a" in r.stdout
