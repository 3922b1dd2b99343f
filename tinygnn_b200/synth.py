"""Seeded synthetic graphs and features with the shapes of the benchmark configs.

The real datasets (Cora, Reddit) are not available offline; these seeded
generators stand in for them with their published shapes:

* ``cora_like``   -- 2,708 nodes, preferential attachment (m=2) trimmed to
  5,278 undirected pairs = 10,556 directed entries; 1,433 binary features
  with ~1.27% ones, row-normalised.
* ``rmat``        -- R-MAT (a, b, c, d) = (.57, .19, .19, .05), duplicates
  removed; optionally symmetrised / transposed / without self pairs.
* ``chung_lu``    -- 232,965 nodes, Zipf weights (i+1)^-0.3, self pairs
  rejected, drawing until exactly E unique directed edges; node ids
  permuted.  Mean degree ~492 with a heavy tail (Reddit-shaped).

Randomness is a counter-based hash (SplitMix64 finalizer) over int64
tensors, so integer outputs (graphs) are identical on CPU and GPU for the
same seed; float features use Box-Muller on the device that generates them.
torch is used only as the array engine here.
"""
from __future__ import annotations

import math
from typing import Optional

import numpy as np
import torch

_M1 = 0xBF58476D1CE4E5B9 - (1 << 64)
_M2 = 0x94D049BB133111EB - (1 << 64)
_GOLD = 0x9E3779B97F4A7C15 - (1 << 64)


def _lsr(x: torch.Tensor, k: int) -> torch.Tensor:
    return (x >> k) & ((1 << (64 - k)) - 1)


def hash64(idx: torch.Tensor, seed: int, stream: int = 0) -> torch.Tensor:
    """SplitMix64 of (seed, stream, idx): int64 tensor of pseudo-random bits."""
    base = (seed * 0x2545F4914F6CDD1D + stream * 0x632BE59BD9B4E019) & ((1 << 64) - 1)
    if base >= 1 << 63:
        base -= 1 << 64
    x = idx.to(torch.int64) * _GOLD + base
    x = x ^ _lsr(x, 30)
    x = x * _M1
    x = x ^ _lsr(x, 27)
    x = x * _M2
    return x ^ _lsr(x, 31)


def uniform(n: int, seed: int, stream: int = 0, device="cpu", offset: int = 0) -> torch.Tensor:
    """float32 in [0, 1) with 24 random bits (exactly representable)."""
    h = hash64(torch.arange(offset, offset + n, device=device), seed, stream)
    return _lsr(h, 40).to(torch.float32) * (1.0 / (1 << 24))


def normal(shape, seed: int, stream: int = 0, device="cpu") -> torch.Tensor:
    """float32 N(0, 1) by Box-Muller."""
    n = int(np.prod(shape))
    m = (n + 1) // 2
    idx = torch.arange(m, device=device)
    u1 = (_lsr(hash64(idx, seed, 2 * stream + 1), 11).to(torch.float64) + 1.0) * (1.0 / (1 << 53))  # (0, 1]
    u2 = _lsr(hash64(idx, seed, 2 * stream + 2), 11).to(torch.float64) * (1.0 / (1 << 53))
    r = torch.sqrt(-2.0 * torch.log(u1))
    z = torch.cat([r * torch.cos(2 * math.pi * u2), r * torch.sin(2 * math.pi * u2)])[:n]
    return z.to(torch.float32).reshape(shape)


def normal_rows(row0: int, rows: int, cols: int, seed: int, stream: int = 0, device="cpu") -> torch.Tensor:
    """Rows [row0, row0 + rows) of a seeded N(0, 1) matrix with ``cols`` columns.

    Element (i, j) depends only on (seed, i*cols + j), so any row block of
    the global matrix is the same whichever process generates it.
    """
    idx = torch.arange(row0 * cols, (row0 + rows) * cols, device=device)
    u1 = (_lsr(hash64(idx, seed, 2 * stream + 1), 11).to(torch.float64) + 1.0) * (1.0 / (1 << 53))
    u2 = _lsr(hash64(idx, seed, 2 * stream + 2), 11).to(torch.float64) * (1.0 / (1 << 53))
    z = torch.sqrt(-2.0 * torch.log(u1)) * torch.cos(2 * math.pi * u2)
    return z.to(torch.float32).reshape(rows, cols)


def glorot(fan_in: int, fan_out: int, seed: int, stream: int = 0, device="cpu") -> torch.Tensor:
    """Glorot-uniform fan_in x fan_out weight."""
    r = math.sqrt(6.0 / (fan_in + fan_out))
    u = uniform(fan_in * fan_out, seed, stream, device)
    return ((u * 2.0 - 1.0) * r).to(torch.float32).reshape(fan_in, fan_out)


def _first_unique(keys: torch.Tensor, limit: Optional[int]) -> torch.Tensor:
    """Unique keys in order of first appearance, truncated to ``limit``."""
    sk, perm = torch.sort(keys, stable=True)
    first = torch.ones_like(sk, dtype=torch.bool)
    first[1:] = sk[1:] != sk[:-1]
    uk, upos = sk[first], perm[first]
    if limit is not None and uk.numel() > limit:
        order = torch.argsort(upos)[:limit]
        uk = uk[order]
    return uk


def csr_from_keys(keys: torch.Tensor, n_rows: int, n_cols: int):
    """Row-sorted CSR (int32 row_ptr, col_ind) from unique row*n_cols+col keys."""
    keys = torch.sort(keys).values
    rows = torch.div(keys, n_cols, rounding_mode="floor")
    cols = keys - rows * n_cols
    counts = torch.bincount(rows, minlength=n_rows)
    rp = torch.zeros(n_rows + 1, dtype=torch.int64, device=keys.device)
    rp[1:] = torch.cumsum(counts, 0)
    return rp.to(torch.int32), cols.to(torch.int32)


def rmat_edges(scale: int, draws: int, seed: int, device="cpu", abcd=(0.57, 0.19, 0.19, 0.05),
               chunk: int = 1 << 24):
    """Raw R-MAT (src, dst) draws as int64 tensors."""
    a, b, c, _ = abcd
    srcs, dsts = [], []
    for off in range(0, draws, chunk):
        n = min(chunk, draws - off)
        s = torch.zeros(n, dtype=torch.int64, device=device)
        d = torch.zeros(n, dtype=torch.int64, device=device)
        for lvl in range(scale):
            u = uniform(n, seed, 1000 + lvl, device, offset=off)
            down = u >= (a + b)                                   # quadrant c or d: src bit
            right = ((u >= a) & (u < a + b)) | (u >= a + b + c)   # quadrant b or d: dst bit
            s = (s << 1) | down.to(torch.int64)
            d = (d << 1) | right.to(torch.int64)
        srcs.append(s)
        dsts.append(d)
    return torch.cat(srcs), torch.cat(dsts)


def rmat_csr(scale: int, draws: int, seed: int, device="cpu", symmetric=False, transpose=False,
             no_self=False, values_seed: Optional[int] = None):
    """R-MAT graph as a deduplicated row-sorted CSR; values U(0,1] when values_seed is given."""
    N = 1 << scale
    s, d = rmat_edges(scale, draws, seed, device)
    if transpose:
        s, d = d, s
    if symmetric:
        s, d = torch.cat([s, d]), torch.cat([d, s])
    if no_self:
        keep = s != d
        s, d = s[keep], d[keep]
    keys = torch.unique(s * N + d)
    rp, ci = csr_from_keys(keys, N, N)
    if values_seed is None:
        v = torch.ones(ci.numel(), dtype=torch.float32, device=device)
    else:
        v = 1.0 - uniform(ci.numel(), values_seed, 7, device)  # (0, 1]
    return N, rp, ci, v


def _alias_table(w: np.ndarray):
    """Walker alias table for probabilities proportional to w (float64)."""
    n = w.size
    p = w * (n / w.sum())
    prob = np.zeros(n)
    alias = np.zeros(n, dtype=np.int64)
    small = [i for i in range(n) if p[i] < 1.0]
    large = [i for i in range(n) if p[i] >= 1.0]
    p = p.copy()
    while small and large:
        s, l = small.pop(), large.pop()
        prob[s] = p[s]
        alias[s] = l
        p[l] = (p[l] + p[s]) - 1.0
        (small if p[l] < 1.0 else large).append(l)
    for i in large + small:
        prob[i] = 1.0
        alias[i] = i
    return prob, alias


def chung_lu_csr(n: int, edges: int, seed: int, exponent: float = 0.3, device="cpu"):
    """Chung-Lu directed graph with Zipf weights: exactly ``edges`` unique
    (src != dst) pairs, taken in draw order; node ids then permuted."""
    w = (np.arange(n, dtype=np.float64) + 1.0) ** (-exponent)
    prob, alias = _alias_table(w)
    prob_t = torch.as_tensor(prob, dtype=torch.float64, device=device)
    alias_t = torch.as_tensor(alias, dtype=torch.int64, device=device)

    def draw(count: int, offset: int, stream: int) -> torch.Tensor:
        idx = torch.arange(offset, offset + count, device=device)
        h = hash64(idx, seed, stream)
        col = _lsr(h, 1) % n
        u = _lsr(hash64(idx, seed, stream + 1), 11).to(torch.float64) * (1.0 / (1 << 53))
        return torch.where(u < prob_t[col], col, alias_t[col])

    # The draw sequence is a pure function of (seed, index), so growing it
    # and re-reading it from the start selects exactly the first `edges`
    # unique pairs in draw order.
    drawn = int(edges * 1.1) + 1024
    while True:
        s = draw(drawn, 0, 11)
        d = draw(drawn, 0, 13)
        k = s * n + d
        k = k[s != d]
        del s, d
        n_unique = int(torch.unique(k).numel())
        if n_unique >= edges:
            break
        drawn = int(drawn * (edges / max(n_unique, 1)) * 1.03) + 1024
    keys = _first_unique(k, edges)
    del k
    # Seeded node permutation.
    perm = torch.argsort(hash64(torch.arange(n, device=device), seed, 17))
    src = perm[torch.div(keys, n, rounding_mode="floor")]
    dst = perm[keys % n]
    rp, ci = csr_from_keys(src * n + dst, n, n)
    return n, rp, ci, torch.ones(ci.numel(), dtype=torch.float32, device=device)


def cora_like(seed: int = 1, n: int = 2708, pairs: int = 5278, feats: int = 1433, p_one: float = 0.0127,
              device="cpu"):
    """Cora-shaped graph (undirected, stored both ways) and row-normalised binary features."""
    # Preferential attachment (m = 2) with hash-driven choices, sequential.
    rng_u = uniform(4 * n, seed, 21).numpy().astype(np.float64)
    ends: list = [0, 1]
    pair_set = {(0, 1)}
    order = [(0, 1)]
    t = 0
    for v in range(2, n):
        chosen = set()
        while len(chosen) < 2 and len(chosen) < v:
            u = rng_u[t % rng_u.size]
            t += 1
            chosen.add(ends[int(u * len(ends))])
        for c in sorted(chosen):
            key = (min(c, v), max(c, v))
            if key not in pair_set:
                pair_set.add(key)
                order.append(key)
            ends += [c, v]
    order = order[:pairs]
    src = np.array([a for a, b in order] + [b for a, b in order], dtype=np.int64)
    dst = np.array([b for a, b in order] + [a for a, b in order], dtype=np.int64)
    keys = torch.as_tensor(np.unique(src * n + dst), device=device)
    rp, ci = csr_from_keys(keys, n, n)
    u = uniform(n * feats, seed + 1, 22, device).reshape(n, feats)
    X = (u < p_one).to(torch.float32)
    rs = X.sum(1, keepdim=True)
    X = torch.where(rs > 0, X / torch.where(rs > 0, rs, torch.ones_like(rs)), X)
    return n, rp, ci, torch.ones(ci.numel(), dtype=torch.float32, device=device), X
