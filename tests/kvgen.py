"""Deterministic synthetic inputs shared by the oracle, the golden fixtures and
the GPU parity tests.

The generator is splitmix64 + Box-Muller written out in numpy, so the same
seed gives the same bits on every machine and numpy version (the golden
fixtures only store seeds and results, not the multi-MB inputs).
"""
from __future__ import annotations

import numpy as np

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def splitmix64(seed: int, n: int) -> np.ndarray:
    """n successive splitmix64 outputs for a stream starting at `seed`."""
    with np.errstate(over="ignore"):
        idx = np.arange(1, n + 1, dtype=np.uint64)
        z = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) + idx * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return z


def uniform(seed: int, n: int) -> np.ndarray:
    """n doubles in (0, 1)."""
    u = splitmix64(seed, n) >> np.uint64(11)
    return (u.astype(np.float64) + 0.5) * (1.0 / 9007199254740992.0)


def normal(seed: int, shape, dtype=np.float32) -> np.ndarray:
    """N(0,1) via Box-Muller, rounded to `dtype` (round to nearest)."""
    n = int(np.prod(shape))
    m = (n + 1) // 2
    u = uniform(seed, 2 * m)
    r = np.sqrt(-2.0 * np.log(u[:m]))
    th = 2.0 * np.pi * u[m:]
    z = np.concatenate([r * np.cos(th), r * np.sin(th)])[:n]
    return z.reshape(shape).astype(dtype)


def randint(seed: int, n: int, lo: int, hi: int) -> np.ndarray:
    """n integers uniform in [lo, hi] (inclusive)."""
    span = hi - lo + 1
    return (lo + np.floor(uniform(seed, n) * span)).astype(np.int64)


def permutation(seed: int, n: int) -> np.ndarray:
    """Fisher-Yates shuffle of range(n) driven by splitmix64."""
    p = np.arange(n, dtype=np.int64)
    u = uniform(seed, n)
    for i in range(n - 1, 0, -1):
        j = int(u[i] * (i + 1))
        p[i], p[j] = p[j], p[i]
    return p


def zipf_pages(seed: int, n: int, num_pages: int, s: float = 1.1) -> np.ndarray:
    """n page ids drawn Zipf(s) over [0, num_pages) (rank r has weight r^-s)."""
    w = 1.0 / np.power(np.arange(1, num_pages + 1, dtype=np.float64), s)
    cdf = np.cumsum(w)
    cdf /= cdf[-1]
    return np.searchsorted(cdf, uniform(seed, n), side="right").clip(0, num_pages - 1)


def paged_layout(seq_lens, page_tokens: int, extra_tokens: int, seed: int | None):
    """Block tables for sequences of the given lengths (plus room for
    `extra_tokens` appended later).  Physical ids are a seeded permutation of
    the pool (None: sequential).  Returns (block_table [B][max_pages], num_pages)."""
    seq_lens = np.asarray(seq_lens, dtype=np.int64)
    need = (seq_lens + extra_tokens + page_tokens - 1) // page_tokens
    num_pages = int(need.sum())
    max_pages = int(need.max()) if need.size else 1
    phys = np.arange(num_pages) if seed is None else permutation(seed, num_pages)
    bt = np.full((seq_lens.size, max_pages), -1, dtype=np.int32)
    off = 0
    for s, n in enumerate(need):
        bt[s, :n] = phys[off:off + n]
        off += n
    return bt, num_pages
