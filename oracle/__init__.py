"""ctypes wrapper of the CPU oracle (oracle.c) -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm use
this package, as the checker or as the timed CPU baseline; the product never imports it.
The restatement's scope, modes and pinning status are described in oracle.h.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liborc.so")


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


class _Params(C.Structure):
    _fields_ = [
        ("n_trees", C.c_uint32), ("depth", C.c_uint32), ("n_bins", C.c_uint32),
        ("learning_rate", C.c_float), ("lambda_", C.c_float), ("min_child_h", C.c_float),
        ("subsample", C.c_float), ("colsample", C.c_float), ("goss_top", C.c_float),
        ("goss_other", C.c_float), ("objective", C.c_int32), ("subtract", C.c_int32),
        ("monotone", C.POINTER(C.c_int32)), ("n_monotone", C.c_uint32), ("exact", C.c_int32),
        ("n_threads", C.c_int32), ("leafvar", C.POINTER(C.c_float)),
    ]


class _Trace(C.Structure):
    _fields_ = [("level_hist", C.c_void_p * 16), ("e_g", C.c_int32), ("e_h", C.c_int32),
                ("split_f", C.c_uint32 * 16), ("split_b", C.c_uint32 * 16),
                ("loop_seconds", C.c_double), ("trace_trees", C.c_uint32),
                ("tree_g", C.c_void_p), ("tree_h", C.c_void_p), ("tree_leaf", C.c_void_p)]


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) or any(
                os.path.getmtime(os.path.join(HERE, f)) > os.path.getmtime(LIB_PATH)
                for f in ("oracle.c", "oracle.h") if os.path.exists(LIB_PATH)):
            build()
        L = C.CDLL(LIB_PATH)
        vp, u64, u32, i32, f32 = C.c_void_p, C.c_uint64, C.c_uint32, C.c_int32, C.c_float
        L.orc_default_threads.restype = C.c_int
        L.orc_compute_boundaries.argtypes = [vp, u64, u32, u32, u64, C.c_int, vp]
        L.orc_bin_rowmajor.argtypes = [vp, u64, u32, vp, u32, vp]
        L.orc_base_score.argtypes = [vp, u64, C.c_int]
        L.orc_base_score.restype = f32
        L.orc_train.argtypes = [C.POINTER(_Params), vp, vp, u64, u32, vp, f32, vp, vp, vp, vp, vp,
                                vp, C.POINTER(_Trace)]
        L.orc_train.restype = C.c_int
        L.orc_predict.argtypes = [vp, u64, u32, u32, u32, vp, vp, vp, f32, vp]
        L.orc_level_hist_exact.argtypes = [vp, u64, u32, u32, vp, vp, vp, C.c_int, C.c_int, u32,
                                           C.c_int, vp]
        for m in ("auc", "logloss", "rmse", "mae", "r2", "accuracy"):
            fn = getattr(L, "orc_" + m)
            fn.argtypes = [vp, vp, u64]
            fn.restype = C.c_double
        L.orc_target_encode.argtypes = [vp, u64, u32, vp, vp, u32, f32, u32, u64, vp]
        L.orc_rw_expf.argtypes = [f32]
        L.orc_rw_expf.restype = f32
        _lib = L
    return _lib


def _p(a):
    return None if a is None else C.c_void_p(a.ctypes.data)


def default_threads() -> int:
    return lib().orc_default_threads()


def compute_boundaries(x, n_bins, sample=200_000, unique=False):
    x = np.ascontiguousarray(x, np.float32)
    n, nf = x.shape
    out = np.empty(nf * (n_bins - 1), np.float32)
    lib().orc_compute_boundaries(_p(x), n, nf, n_bins, sample, int(unique), _p(out))
    return out


def bin_rowmajor(x, cuts, n_bins):
    x = np.ascontiguousarray(x, np.float32)
    cuts = np.ascontiguousarray(cuts, np.float32)
    n, nf = x.shape
    out = np.empty((n, nf), np.uint8)
    lib().orc_bin_rowmajor(_p(x), n, nf, _p(cuts), n_bins, _p(out))
    return out


def base_score(y, objective="logistic"):
    y = np.ascontiguousarray(y, np.float32)
    return float(lib().orc_base_score(_p(y), len(y), 0 if objective == "logistic" else 1))


class OracleFit:
    pass


def train(x, y, cuts, base, *, n_trees, depth, n_bins, learning_rate=0.1, lambda_=1.0,
          min_child_h=1e-3, subsample=1.0, colsample=1.0, goss_top=0.0, goss_other=0.1,
          objective="logistic", subtract=True, monotone=(), exact=True, n_threads=0,
          trace_levels=False, trace_trees=0, pgbm=False) -> OracleFit:
    """orc_train: exact=True is oracle_exact (the GPU's arithmetic), False is oracle_ref
    (faithful src/cpu.rs with n_threads rayon chunks). trace_trees > 0 records the first
    trees' g, h ([k][n] f32, 0 outside the sample) and final leaves ([k][n] u16)."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.ascontiguousarray(y, np.float32)
    cuts = np.ascontiguousarray(cuts, np.float32)
    n, nf = x.shape
    p = _Params()
    p.n_trees, p.depth, p.n_bins = n_trees, depth, n_bins
    p.learning_rate, p.lambda_, p.min_child_h = learning_rate, lambda_, min_child_h
    p.subsample, p.colsample, p.goss_top, p.goss_other = subsample, colsample, goss_top, goss_other
    p.objective = 0 if objective == "logistic" else 1
    p.subtract = int(subtract)
    mono = np.ascontiguousarray(monotone, np.int32)
    p.monotone = mono.ctypes.data_as(C.POINTER(C.c_int32)) if len(mono) else None
    p.n_monotone = len(mono)
    p.exact, p.n_threads = int(exact), n_threads
    r = OracleFit()
    r.feat = np.zeros(n_trees * depth, np.uint32)
    r.thr = np.zeros(n_trees * depth, np.float32)
    r.thr_bin = np.zeros(n_trees * depth, np.uint32)
    r.leafval = np.zeros(n_trees << depth, np.float32)
    r.fi_gain = np.zeros(nf, np.float32)
    r.fi_count = np.zeros(nf, np.float32)
    r.leafvar = None
    if pgbm:  # PGBM leaf variances (exact mode only)
        if not exact:
            raise ValueError("pgbm leaf variances are computed in exact mode only")
        r.leafvar = np.zeros(n_trees << depth, np.float32)
        p.leafvar = r.leafvar.ctypes.data_as(C.POINTER(C.c_float))
    tr = _Trace()
    hists = []
    if trace_levels:
        for d in range(min(depth, 16)):
            h = np.zeros(((1 << d), nf, n_bins, 2), np.int64)
            hists.append(h)
            tr.level_hist[d] = h.ctypes.data
    k = min(int(trace_trees), n_trees)
    if k:
        r.tree_g = np.zeros((k, n), np.float32)
        r.tree_h = np.zeros((k, n), np.float32)
        r.tree_leaf = np.zeros((k, n), np.uint16)
        tr.trace_trees = k
        tr.tree_g, tr.tree_h = r.tree_g.ctypes.data, r.tree_h.ctypes.data
        tr.tree_leaf = r.tree_leaf.ctypes.data
    rc = lib().orc_train(C.byref(p), _p(x), _p(y), n, nf, _p(cuts), base, _p(r.feat), _p(r.thr),
                         _p(r.thr_bin), _p(r.leafval), _p(r.fi_gain), _p(r.fi_count),
                         C.byref(tr))
    if rc != 0:
        raise ValueError(f"orc_train rejected its arguments ({rc})")
    r.level_hist = hists
    r.e_g, r.e_h = tr.e_g, tr.e_h
    r.split_f = list(tr.split_f)[:depth]
    r.split_b = list(tr.split_b)[:depth]
    r.loop_seconds = tr.loop_seconds
    return r


def predict(x, feat, thr, leafval, base, n_trees, depth):
    x = np.ascontiguousarray(x, np.float32)
    n, nf = x.shape
    out = np.empty(n, np.float32)
    lib().orc_predict(_p(x), n, nf, n_trees, depth, _p(np.ascontiguousarray(feat, np.uint32)),
                      _p(np.ascontiguousarray(thr, np.float32)),
                      _p(np.ascontiguousarray(leafval, np.float32)), base, _p(out))
    return out


def level_hist_exact(bins_rowmajor, node, g, h, e_g, e_h, groups, odd_only, n_bins):
    b = np.ascontiguousarray(bins_rowmajor, np.uint8)
    n, nf = b.shape
    out = np.zeros((groups, nf, n_bins, 2), np.int64)
    lib().orc_level_hist_exact(_p(b), n, nf, n_bins, _p(np.ascontiguousarray(node, np.int32)),
                               _p(np.ascontiguousarray(g, np.float32)),
                               _p(np.ascontiguousarray(h, np.float32)), e_g, e_h, groups,
                               int(odd_only), _p(out))
    return out


def metric(name, s, y):
    s = np.ascontiguousarray(s, np.float32)
    y = np.ascontiguousarray(y, np.float32)
    return float(getattr(lib(), "orc_" + name)(_p(s), _p(y), len(s)))


def target_encode(x, y, categorical, smoothing=10.0, k_folds=5, hash_buckets=0):
    x = np.array(x, np.float32, order="C", copy=True)
    y = np.ascontiguousarray(y, np.float32)
    cat = np.ascontiguousarray(categorical, np.uint32)
    gm = C.c_float()
    n, nf = x.shape
    lib().orc_target_encode(_p(x), n, nf, _p(y), _p(cat), len(cat), smoothing, k_folds,
                            hash_buckets, C.byref(gm))
    return x, gm.value


def rw_expf(x: float) -> float:
    return float(lib().orc_rw_expf(x))
