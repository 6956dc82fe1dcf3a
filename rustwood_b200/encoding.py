"""Categorical target encoding kept from the reference host code (src/encoding.rs).

Training rows are encoded out-of-fold (K folds by row index modulo K) with smoothed
category means; test rows use the full-train maps, unseen codes the global mean.
This is host preprocessing that runs before binning; it is not on the GPU path.
"""
from __future__ import annotations

import numpy as np

HASH_SALT = 0x0041_4456_5052_4F50  # src/encoding.rs:27
_M64 = (1 << 64) - 1


def _codes(col: np.ndarray) -> np.ndarray:
    """f32::round (half away from zero) then a saturating `as i64` cast; NaN -> 0."""
    r = np.where(col >= 0, np.floor(col.astype(np.float64) + 0.5),
                 np.ceil(col.astype(np.float64) - 0.5))
    r = np.where(np.isnan(r), 0.0, r)
    r = np.clip(r, -9.223372036854775808e18, 9.223372036854775807e18)
    out = np.empty(r.shape, dtype=np.int64)
    big = r >= 9.223372036854775807e18
    out[~big] = r[~big].astype(np.int64)
    out[big] = np.iinfo(np.int64).max
    return out


def key_of(col: np.ndarray, hash_buckets: int) -> np.ndarray:
    """src/encoding.rs:29-40: category code, optionally folded by the hashing trick."""
    c = _codes(col)
    if hash_buckets == 0:
        return c
    x = (c.astype(np.uint64) ^ np.uint64(HASH_SALT)) * np.uint64(0x9E37_79B9_7F4A_7C15)
    x ^= x >> np.uint64(29)
    x = x * np.uint64(0xBF58_476D_1CE4_E5B9)
    x ^= x >> np.uint64(32)
    return (x % np.uint64(hash_buckets)).astype(np.int64)


def fit_transform_train(x: np.ndarray, y: np.ndarray, categorical: list[int], smoothing: float,
                        k_folds: int = 5, hash_buckets: int = 0):
    """src/encoding.rs:44-95. Encodes x (row-major, float32) in place; returns
    (encoders, gmean) with encoders[i] a dict code -> float32 value."""
    n = x.shape[0]
    k = max(k_folds, 2)
    a = float(smoothing)
    gmean = np.float32(np.sum(y.astype(np.float64)) / n)
    gm = float(gmean)
    folds = np.arange(n) % k
    encoders = []
    for c in categorical:
        keys = key_of(x[:, c], hash_buckets)
        uniq, inv = np.unique(keys, return_inverse=True)
        sums = np.zeros((len(uniq), k))
        cnts = np.zeros((len(uniq), k), dtype=np.uint64)
        # per-fold sums accumulate in row order (f64), as the reference's loop does
        for i in range(n):
            sums[inv[i], folds[i]] += float(y[i])
            cnts[inv[i], folds[i]] += 1
        tot_s = np.zeros(len(uniq))
        for j in range(k):
            tot_s = tot_s + sums[:, j]
        tot_c = cnts.sum(axis=1)
        full = {int(key): np.float32((tot_s[u] + a * gm) / (float(tot_c[u]) + a))
                for u, key in enumerate(uniq)}
        s = tot_s[inv] - sums[inv, folds]
        cnt = tot_c[inv].astype(np.float64) - cnts[inv, folds].astype(np.float64)
        enc = np.where(cnt > 0.0, ((s + a * gm) / np.where(cnt > 0, cnt + a, 1.0)), 0.0)
        x[:, c] = np.where(cnt > 0.0, enc.astype(np.float32), gmean)
        encoders.append(full)
    return encoders, gmean


def transform(x: np.ndarray, categorical: list[int], encoders, gmean: float,
              hash_buckets: int = 0) -> None:
    """src/encoding.rs:99-115 (in place)."""
    for ci, c in enumerate(categorical):
        keys = key_of(x[:, c], hash_buckets)
        m = encoders[ci]
        x[:, c] = np.array([m.get(int(kk), np.float32(gmean)) for kk in keys], dtype=np.float32)
