"""Generates the golden fixtures in this directory from the pure-Python restatement
(tests/pyref.py) of rustwood's CPU trainer.

The reference ships no golden vectors and cannot be built here, so these fixtures pin
the C oracle and the GPU path to an independent restatement on small seeded inputs.
Run: python tests/golden/make_golden.py  (writes tests/golden/*.npz)
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
import pyref  # noqa: E402
import ctypes  # noqa: E402

_libm = ctypes.CDLL("libm.so.6")
_libm.logf.argtypes = [ctypes.c_float]
_libm.logf.restype = ctypes.c_float


def _logf(v: float) -> float:
    return _libm.logf(v)

CASES = [
    # name, seed, n, nf, n_bins, unique, trees, depth, lr, objective, exact, n_threads, subsample
    ("logistic_exact", 11, 160, 4, 8, False, 3, 3, 0.3, "logistic", True, 1, 1.0),
    ("logistic_ref_nt3", 12, 140, 3, 6, False, 3, 3, 0.2, "logistic", False, 3, 1.0),
    ("l2_exact_unique", 13, 120, 3, 8, True, 2, 3, 0.1, "l2", True, 1, 1.0),
    ("l2_ref_nt2", 14, 130, 4, 5, False, 3, 2, 0.5, "l2", False, 2, 1.0),
    ("logistic_exact_stride", 15, 150, 3, 7, False, 3, 3, 0.3, "logistic", True, 1, 0.5),
]


def make(case):
    name, seed, n, nf, nb, uniq, trees, depth, lr, obj, exact, nt, sub = case
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n, nf)).astype(np.float32)
    x[:, 0] = np.round(x[:, 0] * 2)  # ties
    if obj == "logistic":
        y = (rng.random(n) < 1 / (1 + np.exp(-x[:, 1]))).astype(np.float32)
    else:
        y = (x[:, 1] * 2 + rng.normal(0, 0.3, n)).astype(np.float32)
    s = np.float32(0)
    for v in y:
        s = np.float32(s + v)
    mean = np.float32(s / np.float32(n))
    mean = min(max(mean, np.float32(1e-6)), np.float32(1 - 1e-6))
    # booster.rs:201-205: Rust f32::ln is glibc logf
    base = np.float32(_logf(float(np.float32(mean / np.float32(1 - mean))))) \
        if obj == "logistic" else mean
    cuts = pyref.boundaries(x, nb, unique=uniq)
    fit = pyref.train(x, y, cuts, base, n_trees=trees, depth=depth, n_bins=nb, learning_rate=lr,
                      objective=obj, exact=exact, n_threads=nt, subsample=sub)
    pred = pyref.predict(x, fit["feat"], fit["thr"], fit["leafval"], base, trees, depth)
    np.savez(os.path.join(HERE, name + ".npz"), x=x, y=y, cuts=cuts, base=np.float32(base),
             params=np.array([nb, int(uniq), trees, depth, lr, obj == "l2", int(exact), nt, sub],
                             dtype=np.float64),
             pred=pred, **fit)


if __name__ == "__main__":
    for c in CASES:
        make(c)
        print("wrote", c[0])
