"""Shared test helpers: fixtures, tolerances, small graph builders."""
from __future__ import annotations

import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")

# fp32 tolerance for results that are not bit-exact by construction
# (|gpu - ref| <= ATOL + RTOL * |ref|).
ATOL = 1e-5
RTOL = 1e-4


class Golden:
    """Access to golden_ref.npz as golden[case][array]."""

    def __init__(self, path: str):
        self.z = np.load(path)
        self.cases = sorted({k.split("/")[0] for k in self.z.files})

    def __getitem__(self, case):
        prefix = case + "/"
        return {k[len(prefix):]: self.z[k] for k in self.z.files if k.startswith(prefix)}

    def matching(self, prefix):
        return [c for c in self.cases if c.startswith(prefix)]


def load_golden() -> Golden:
    return Golden(os.path.join(GOLDEN, "golden_ref.npz"))


def load_known_answers():
    with open(os.path.join(GOLDEN, "known_answers.json")) as f:
        return json.load(f)


def bits_equal(a, b) -> bool:
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    if a.shape != b.shape or a.dtype != b.dtype:
        return False
    if a.dtype == np.float32:
        return np.array_equal(a.view(np.uint32), b.view(np.uint32))
    return np.array_equal(a, b)


def assert_bits_equal(a, b, what=""):
    a, b = np.asarray(a), np.asarray(b)
    if bits_equal(a, b):
        return
    msg = f"{what}: not bit-identical"
    if a.shape == b.shape and a.dtype == np.float32:
        d = np.abs(a.astype(np.float64) - b.astype(np.float64))
        i = np.unravel_index(np.argmax(d), d.shape)
        msg += f"; {np.count_nonzero(a.view(np.uint32) != b.view(np.uint32))} differ, max |d| {d.max():.3g} at {i}"
    else:
        msg += f"; shapes {a.shape} {b.shape} dtypes {a.dtype} {b.dtype}"
    raise AssertionError(msg)


def assert_close(a, ref, what="", atol=ATOL, rtol=RTOL):
    a = np.asarray(a, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert a.shape == ref.shape, f"{what}: shape {a.shape} vs {ref.shape}"
    bad = np.abs(a - ref) > atol + rtol * np.abs(ref)
    if bad.any():
        i = np.argwhere(bad)[0]
        raise AssertionError(f"{what}: {bad.sum()} elements outside |d| <= {atol} + {rtol}|ref|; "
                             f"first at {tuple(i)}: {a[tuple(i)]} vs {ref[tuple(i)]}")


def undirected_csr(n, pairs):
    """make_undirected_csr of the reference tests."""
    src = [u for u, v in pairs] + [v for u, v in pairs]
    dst = [v for u, v in pairs] + [u for u, v in pairs]
    order = sorted(range(len(src)), key=lambda k: (src[k], dst[k]))
    rp = np.zeros(n + 1, np.int32)
    for k in order:
        rp[src[k] + 1] += 1
    rp = np.cumsum(rp).astype(np.int32)
    return rp, np.array([dst[k] for k in order], np.int32), np.ones(len(order), np.float32)


def rand_csr(rng, n, m, deg, weighted=True, diag=True, empty_frac=0.0):
    """Random deduplicated row-sorted CSR (numpy)."""
    e = n * deg
    s = rng.integers(0, n, e)
    d = rng.integers(0, m, e)
    if not diag:
        keep = s != d
        s, d = s[keep], d[keep]
    if empty_frac > 0:
        empty = rng.random(n) < empty_frac
        keep = ~empty[s]
        s, d = s[keep], d[keep]
    key = np.unique(s.astype(np.int64) * m + d)
    s, d = (key // m).astype(np.int32), (key % m).astype(np.int32)
    rp = np.zeros(n + 1, np.int64)
    np.add.at(rp, s + 1, 1)
    rp = np.cumsum(rp).astype(np.int32)
    v = (rng.random(d.size) + 0.05).astype(np.float32) if weighted else np.ones(d.size, np.float32)
    return rp, d, v


def powerlaw_csr(rng, n, deg, alpha=1.2, weighted=True, diag=True):
    """Heavy-tailed random CSR: row lengths ~ Zipf, columns uniform."""
    w = (np.arange(n) + 1.0) ** (-1.0 / alpha)
    w = w / w.sum()
    e = n * deg
    s = rng.choice(n, size=e, p=w)
    d = rng.integers(0, n, e)
    if not diag:
        keep = s != d
        s, d = s[keep], d[keep]
    key = np.unique(s.astype(np.int64) * n + d)
    s, d = (key // n).astype(np.int32), (key % n).astype(np.int32)
    perm = rng.permutation(n).astype(np.int32)
    s, d = perm[s], perm[d]
    key = np.sort(s.astype(np.int64) * n + d)
    s, d = (key // n).astype(np.int32), (key % n).astype(np.int32)
    rp = np.zeros(n + 1, np.int64)
    np.add.at(rp, s + 1, 1)
    rp = np.cumsum(rp).astype(np.int32)
    v = (rng.random(d.size) + 0.05).astype(np.float32) if weighted else np.ones(d.size, np.float32)
    return rp, d, v


def assert_sage_fast_close(got, ref, rp, ci, H, Wn, Ws, what=""):
    """A FAST-mode SAGE layer (its products on the tensor cores, 3xTF32):
    a reordered fp32 sum of 2 F_in terms per output, held to
    |d| <= ATOL + RTOL * sum_k |a_k||b_k| -- the magnitude its rounding acts
    on (|mean| and |max| of the aggregate are bounded by the largest |h| of
    the row's neighbours).  An elementwise bound on |ref| cannot hold at
    cancelling elements for any reordering; logits are checked elementwise
    by the model tests."""
    n, fi = H.shape
    absH = np.abs(H).astype(np.float64)
    seg = np.repeat(np.arange(n), np.diff(rp))
    agg_abs = np.zeros((n, fi))
    np.maximum.at(agg_abs, seg, absH[ci])
    mag = agg_abs @ np.abs(Wn).astype(np.float64) + absH @ np.abs(Ws).astype(np.float64)
    err = np.abs(np.asarray(got, np.float64) - np.asarray(ref, np.float64))
    bad = err > ATOL + RTOL * mag
    assert not bad.any(), f"{what}: {bad.sum()} outside |d| <= {ATOL} + {RTOL} sum|a||b|; max err {err.max():.3g}"
