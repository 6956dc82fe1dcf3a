"""Seeded synthetic stand-ins for the benchmark configurations.

The reference measures on public datasets (Covertype, Credit-G) that are not available
here; these generators reproduce the configurations' shapes, feature types and value
distributions from a recorded numpy seed. Each returns float32 row-major x and y.
"""
from __future__ import annotations

import numpy as np


def c1(n: int = 100_000, n_test: int = 0, seed: int = 0):
    """100k x 28 ~ N(0,1); y ~ Bernoulli(sigmoid(w.x + 0.5*x0*x1)), w ~ N(0,1)."""
    rng = np.random.default_rng(seed)
    m = n + n_test
    x = rng.standard_normal((m, 28), dtype=np.float32)
    w = rng.standard_normal(28)
    logit = x.astype(np.float64) @ w + 0.5 * x[:, 0].astype(np.float64) * x[:, 1]
    y = (rng.random(m) < 1.0 / (1.0 + np.exp(-logit))).astype(np.float32)
    return _split(x, y, n)


def c2(n: int = 1_000_000, n_test: int = 0, seed: int = 0):
    """1M x 54 (Covertype-shaped): 10 U[0,1], 34 integer-valued 0..360, 10 binary;
    7-class label = argmax of random linear scores + noise, reduced one-vs-rest to
    class index 1 (the reference's Covertype target, scripts/dataset_bench.py)."""
    rng = np.random.default_rng(seed)
    m = n + n_test
    x = np.empty((m, 54), dtype=np.float32)
    x[:, :10] = rng.random((m, 10), dtype=np.float32)
    x[:, 10:44] = rng.integers(0, 361, size=(m, 34)).astype(np.float32)
    x[:, 44:] = rng.integers(0, 2, size=(m, 10)).astype(np.float32)
    z = (x - x.mean(axis=0)) / (x.std(axis=0) + 1e-6)
    w = rng.standard_normal((54, 7)).astype(np.float32)
    scores = z @ w + rng.standard_normal((m, 7), dtype=np.float32) * 2.0
    y = (np.argmax(scores, axis=1) == 1).astype(np.float32)
    return _split(x, y, n)


def c3(n: int = 50_000, n_test: int = 0, seed: int = 0):
    """50k x 20 (Credit-G-shaped): 7 N(0,1) + 13 categorical codes with Zipf(1.2)
    cardinalities in 2..50; label from per-category random effects + a linear term.
    Use with categorical = 7..19, unique_bins = 1, monotone = [1]."""
    rng = np.random.default_rng(seed)
    m = n + n_test
    x = np.empty((m, 20), dtype=np.float32)
    x[:, :7] = rng.standard_normal((m, 7), dtype=np.float32)
    logit = 0.8 * x[:, 0].astype(np.float64) + 0.3 * x[:, 1] - 0.2 * x[:, 2]
    for c in range(13):
        card = int(rng.integers(2, 51))
        p = 1.0 / np.arange(1, card + 1) ** 1.2
        p /= p.sum()
        codes = rng.choice(card, size=m, p=p)
        x[:, 7 + c] = codes.astype(np.float32)
        logit += rng.standard_normal(card)[codes] * 0.5
    y = (rng.random(m) < 1.0 / (1.0 + np.exp(-logit))).astype(np.float32)
    return _split(x, y, n)


def c4(n: int = 10_000_000, n_test: int = 0, seed: int = 0, nf: int = 100):
    """10M x 100 ~ N(0,1); y = sum of 10 random depth-3 step functions + N(0, 0.1)."""
    rng = np.random.default_rng(seed)
    m = n + n_test
    x = rng.standard_normal((m, nf), dtype=np.float32)
    y = np.zeros(m, dtype=np.float32)
    for _ in range(10):
        fs = rng.integers(0, nf, size=3)
        ts = rng.standard_normal(3).astype(np.float32) * 0.5
        vals = rng.standard_normal(8).astype(np.float32)
        idx = ((x[:, fs[0]] > ts[0]).astype(np.int64) * 4 + (x[:, fs[1]] > ts[1]) * 2 +
               (x[:, fs[2]] > ts[2]))
        y += vals[idx]
    y += rng.normal(0.0, 0.1, size=m).astype(np.float32)
    return _split(x, y, n)


def c5_model(n_trees: int = 500, depth: int = 6, nf: int = 54, seed: int = 0):
    """Random oblivious model: per (tree, level) feature ~U[0,nf), bin threshold ~U[0,255),
    leaves ~N(0, 0.1). Returns (feat u32, thr_bin u16, leafval f32)."""
    rng = np.random.default_rng(seed)
    feat = rng.integers(0, nf, size=n_trees * depth).astype(np.uint32)
    thr_bin = rng.integers(0, 255, size=n_trees * depth).astype(np.uint16)
    leafval = rng.normal(0.0, 0.1, size=n_trees << depth).astype(np.float32)
    return feat, thr_bin, leafval


def c5_bins(n: int, nf: int = 54, seed: int = 1, ld: int | None = None):
    """u8 bins ~U[0,255], feature-major [nf][ld] (ld >= n, padding zero)."""
    rng = np.random.default_rng(seed)
    ld = n if ld is None else ld
    b = np.zeros((nf, ld), dtype=np.uint8)
    b[:, :n] = rng.integers(0, 256, size=(nf, n), dtype=np.uint8)
    return b


def _split(x, y, n):
    return x[:n], y[:n], x[n:], y[n:]
