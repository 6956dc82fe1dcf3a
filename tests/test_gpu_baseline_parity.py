"""GPU parity at the benchmark configurations, through the C ABI.

Against oracle_exact (the same arithmetic as the CUDA path): every output bit-exact at
full size -- C1 (100k x 28, 200 trees), C2 (1M x 54, 200 trees, the benchmark fit),
C3 (50k x 20, target encoding + monotone, 200 trees) and C4's first 20 trees
(4M x 100 here, 16 bins 4-bit, depth 8, GOSS; 10M rows are the benchmark's size).

Against oracle_ref (src/cpu.rs as written: f32 histograms, f64 gains and leaf sums):
  - the split sequences are compared slot by slot; the report gives the count of equal
    slots and the first slot that differs;
  - the common prefix (the trees before the first differing slot) has leaf values and
    margins within 1e-5 relative (leaf sums come from the unquantised g/h on both sides),
    as the normwise relative error max|a - b| / max|b| per tree (leaves) and over all
    held-out rows (margins). The only difference left between the two trainers is the
    exponential (glibc expf against the shared correctly rounded one, 1 ulp apart on a
    few hundred rows per tree from the third tree on), and a leaf whose value is a
    near-total cancellation of its rows' gradients amplifies it elementwise; the
    elementwise maximum and the count of bit-identical leaf values are reported too;
  - held-out AUC and logloss within 1e-4;
  - teacher forcing: cpu.rs's own g, h and node assignment at every level of its fit are
    fed to the GPU's level step (the production k_hist/k_gain/k_best kernels); where
    the GPU picks another split than cpu.rs, the exact gain gap between the two picks
    must lie below the arithmetic noise bound: the error that 17-bit quantisation
    (<= 2^-(e+1) per row) and cpu.rs's own f32 histogram cells (<= (k + 1 + log2 nt) u
    sum|x| for a cell of k rows in one thread chunk, u = 2^-24; a sibling cell adds its
    parent's and the built cell's errors) can put into the two gains, propagated to
    first order, plus the whole node term wherever a child's hessian sum lies within its
    error of min_child_h.
Set RW_PARITY_REPORT=<path> to have the agreement figures written there as JSON.
"""
import ctypes as C
import json
import math
import os

import numpy as np
import pytest

import oracle
import rustwood_b200 as rb
from rustwood_b200 import _native as N
from rustwood_b200 import synth
from rustwood_b200.booster import Dataset, fit_dataset, train_params

pytestmark = pytest.mark.gpu

U32 = np.uint32


def _report(name, d):
    print(f"\n[{name}] " + json.dumps(d))
    path = os.environ.get("RW_PARITY_REPORT")
    if path:
        rep = json.load(open(path)) if os.path.exists(path) else {}
        rep[name] = d
        json.dump(rep, open(path, "w"), indent=1)


CONFIGS = {
    "c1": dict(data=lambda: synth.c1(100_000, 20_000, seed=0),
               cfg=dict(n_trees=200, depth=6, n_bins=255, learning_rate=0.2)),
    "c2": dict(data=lambda: synth.c2(1_000_000, 100_000, seed=0),
               cfg=dict(n_trees=200, depth=6, n_bins=255, learning_rate=0.3)),
    "c3": dict(data=lambda: synth.c3(50_000, 10_000, seed=0),
               cfg=dict(n_trees=200, depth=6, n_bins=255, categorical=list(range(7, 20)),
                        unique_bins=True, monotone=[1])),
    "c4_first20_4M": dict(data=lambda: synth.c4(4_000_000, 100_000, seed=0, nf=100),
                          cfg=dict(n_trees=20, depth=8, n_bins=16, pack4=True, goss_top=0.2,
                                   goss_other=0.1, objective="l2")),
}

_cache = {}


def _prepared(name, ctx):
    """Data, encoded features, cut table, base score and the GPU fit of one config."""
    if name in _cache:
        return _cache[name]
    case = CONFIGS[name]
    x, y, xt, yt = case["data"]()
    cfg = rb.Config(**case["cfg"])
    b = rb.Booster(cfg, ctx)
    xe, cuts, base = b.prepare(x, y)
    if cfg.categorical:
        xte = np.array(xt, np.float32, order="C", copy=True)
        from rustwood_b200 import encoding
        encoding.transform(xte, cfg.categorical, b.encoders, b.gmean, cfg.cat_hash_buckets)
    else:
        xte = xt
    ds = Dataset(ctx, xe, y, cuts, cfg.n_bins, cfg.pack4)
    r = fit_dataset(ds, cfg, base)
    ds.close()
    _cache.clear()  # keep one configuration's data alive at a time
    _cache[name] = (xe, y, xte, yt, cfg, cuts, base, r)
    return _cache[name]


def _oracle(xe, y, cuts, base, cfg, exact, **kw):
    return oracle.train(xe, y, cuts, base, n_trees=cfg.n_trees, depth=cfg.depth,
                        n_bins=cfg.n_bins, learning_rate=cfg.learning_rate, lambda_=cfg.lambda_,
                        min_child_h=cfg.min_child_h, subsample=cfg.subsample,
                        colsample=cfg.colsample, goss_top=cfg.goss_top,
                        goss_other=cfg.goss_other, objective=cfg.objective,
                        subtract=cfg.subtract, monotone=cfg.monotone, exact=exact, **kw)


@pytest.mark.parametrize("name", list(CONFIGS))
def test_full_size_fit_matches_oracle_exact(ctx, name):
    xe, y, xte, yt, cfg, cuts, base, r = _prepared(name, ctx)
    o = _oracle(xe, y, cuts, base, cfg, True)
    np.testing.assert_array_equal(r.feat, o.feat)
    np.testing.assert_array_equal(r.thr_bin.astype(U32), o.thr_bin)
    for k in ("thr", "leafval", "fi_gain", "fi_count"):
        np.testing.assert_array_equal(getattr(r, k).view(U32), getattr(o, k).view(U32),
                                      err_msg=k)
    # the held-out margins of the GPU scorer, bit-exact with predict_cpu
    b = rb.Booster(cfg.replace(categorical=[]), ctx)
    b.n_features, b.base_score = xe.shape[1], np.float32(base)
    b._take(r)
    got = b.predict(xte)
    want = oracle.predict(xte, o.feat, o.thr, o.leafval, base, cfg.n_trees, cfg.depth)
    np.testing.assert_array_equal(got.view(U32), want.view(U32))
    _report(f"exact_{name}", {"slots": int(r.feat.size), "bit_exact": True,
                               "rows": int(len(y)), "trees": cfg.n_trees})


def _rel(a, b, floor=0.0):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.abs(a - b) / np.maximum(np.maximum(np.abs(b), floor), 1e-300)


def _leaf_rel(a, b, n_leaves):
    """Normwise relative leaf-value error of each tree: max|a - b| / max|b|."""
    a = np.asarray(a, np.float64).reshape(-1, n_leaves)
    b = np.asarray(b, np.float64).reshape(-1, n_leaves)
    return np.abs(a - b).max(axis=1) / np.maximum(np.abs(b).max(axis=1), 1e-300)


@pytest.mark.parametrize("name", ["c1", "c2"])
def test_full_size_agreement_with_faithful_cpu_rs(ctx, name):
    xe, y, xte, yt, cfg, cuts, base, r = _prepared(name, ctx)
    o = _oracle(xe, y, cuts, base, cfg, False, n_threads=oracle.default_threads())
    D, T, NL = cfg.depth, cfg.n_trees, 1 << cfg.depth
    same = (r.feat == o.feat) & (r.thr_bin.astype(U32) == o.thr_bin)
    diff = np.nonzero(~same)[0]
    first = int(diff[0]) if len(diff) else T * D
    t0 = first // D  # trees fully before the first differing slot
    lv_rel = float(_leaf_rel(r.leafval[:t0 * NL], o.leafval[:t0 * NL], NL).max()) if t0 else 0.0
    lv_raw = float(_rel(r.leafval[:t0 * NL], o.leafval[:t0 * NL]).max()) if t0 else 0.0
    lv_bits = int((r.leafval[:t0 * NL].view(U32) == o.leafval[:t0 * NL].view(U32)).sum())
    pg = oracle.predict(xte, r.feat, r.thr, r.leafval, base, t0, D) if t0 else None
    po = oracle.predict(xte, o.feat, o.thr, o.leafval, base, t0, D) if t0 else None
    m_rel = float(np.abs(pg - po).max() / max(np.abs(po).max(), 1e-300)) if t0 else 0.0
    m_raw = float(_rel(pg, po).max()) if t0 else 0.0
    full_g = oracle.predict(xte, r.feat, r.thr, r.leafval, base, T, D)
    full_o = oracle.predict(xte, o.feat, o.thr, o.leafval, base, T, D)
    d_auc = abs(oracle.metric("auc", full_g, yt) - oracle.metric("auc", full_o, yt))
    d_ll = abs(oracle.metric("logloss", full_g, yt) - oracle.metric("logloss", full_o, yt))
    rep = {"slots": T * D, "equal_slots": int(same.sum()),
           "first_differing_slot": None if first == T * D else
           {"tree": first // D, "level": first % D},
           "common_prefix_trees": t0, "leafval_max_rel": lv_rel, "leafval_max_rel_raw": lv_raw,
           "leafval_bit_identical": lv_bits, "leafvals": t0 * NL,
           "margin_max_rel": m_rel, "margin_max_rel_raw": m_raw,
           "auc_gap": d_auc, "logloss_gap": d_ll, "cpu_threads": oracle.default_threads()}
    _report(f"faithful_{name}", rep)
    assert lv_rel <= 1e-5 and m_rel <= 1e-5, rep
    assert d_auc < 1e-4 and d_ll < 1e-4, rep


# ---- teacher forcing -------------------------------------------------------------------

def _f32_cell_error(col, leaf, a, depth, level, nb, nt):
    """Per (node, bin) bound of the error of cpu.rs's f32 histogram cell at `level`
    (src/cpu.rs:17-62, 210-232) for row weights a >= 0 (|g| or h): a cell built from k
    rows of one thread's chunk carries <= (k + 1) u sum|x|, the rayon reduce of nt
    chunks <= ceil(log2 nt) u sum|x| more; a sibling cell = parent - built adds both
    cells' errors plus one rounding (<= u sum|x|)."""
    u = 2.0 ** -24
    lg = math.ceil(math.log2(max(nt, 1)))
    err = None
    for j in range(level + 1):
        nn = 1 << j
        nd = leaf >> (depth - j)
        key = nd.astype(np.int64) * nb + col
        cnt = np.bincount(key, minlength=nn * nb).reshape(nn, nb)
        A = np.bincount(key, weights=a, minlength=nn * nb).reshape(nn, nb)
        direct = (np.ceil(cnt / nt) + lg + 1) * u * A
        if j == 0:
            err = direct
            continue
        new = np.empty_like(direct)
        new[1::2] = direct[1::2]  # the odd child is built
        new[0::2] = err + direct[1::2] + u * A[0::2]  # the even child: parent - odd
        err = new
    return err


def _gain_and_bounds(col, leaf, g, h, b, depth, level, nb, lam, mc, e_g, e_h, nt):
    """Exact gain of split (col <= b goes left) at `level` from f64 sums, and first-order
    bounds of the error 17-bit quantisation (bq: <= 2^-(e+1) per row) and cpu.rs's f32
    histograms (bf: _f32_cell_error over the side's cells) put into it; a node whose
    child hessian sum lies within its error of min_child_h adds its whole term (its
    validity may flip)."""
    n_nodes = 1 << level
    nd = leaf >> (depth - level)
    key = nd.astype(np.int64) * nb + col
    cnt = np.bincount(key, minlength=n_nodes * nb).reshape(n_nodes, nb).astype(np.float64)
    Gc = np.bincount(key, weights=g, minlength=n_nodes * nb).reshape(n_nodes, nb)
    Hc = np.bincount(key, weights=h, minlength=n_nodes * nb).reshape(n_nodes, nb)
    eG = _f32_cell_error(col, leaf, np.abs(g), depth, level, nb, nt)
    eH = _f32_cell_error(col, leaf, h, depth, level, nb, nt)
    qg, qh = 2.0 ** -(e_g + 1), 2.0 ** -(e_h + 1)
    L = slice(0, b + 1)
    R = slice(b + 1, nb)
    T = slice(0, nb)
    gain, bq, bf = 0.0, 0.0, 0.0
    for k in range(n_nodes):
        sides = []
        for sl in (L, R, T):
            sides.append((cnt[k, sl].sum(), Gc[k, sl].sum(), Hc[k, sl].sum(),
                          eG[k, sl].sum(), eH[k, sl].sum()))
        node_term = sum((1, 1, -1)[i] * G * G / (H + lam) for i, (_, G, H, _, _) in
                        enumerate(sides))
        sens = [(2 * abs(G) / (H + lam), G * G / (H + lam) ** 2) for _, G, H, _, _ in sides]
        dq = sum(sg * n * qg + sh * n * qh for (n, _, _, _, _), (sg, sh) in zip(sides, sens))
        df = sum(sg * eg + sh * eh for (_, _, _, eg, eh), (sg, sh) in zip(sides, sens))
        (nL, _, HL, _, eHL), (nR, _, HR, _, eHR) = sides[0], sides[1]
        if HL >= mc and HR >= mc:
            gain += node_term
            bq += dq
            bf += df
        near_q = abs(HL - mc) <= nL * qh or abs(HR - mc) <= nR * qh
        near_f = abs(HL - mc) <= eHL or abs(HR - mc) <= eHR
        if near_q:  # a child's hessian within its error of min_child_h: validity may flip
            bq += abs(node_term)
        if near_f:
            bf += abs(node_term)
    return gain, bq, bf


def _qexp(m):
    if m == 0:
        return 0
    return max(-126, min(100, 17 - int(np.frexp(np.float32(m))[1])))


@pytest.mark.parametrize("name,trees", [("c1", 200), ("c2", 20)])
def test_teacher_forced_gpu_level_step(ctx, name, trees):
    xe, y, xte, yt, cfg, cuts, base, r = _prepared(name, ctx)
    nt = oracle.default_threads()
    o = _oracle(xe, y, cuts, base, cfg.replace(n_trees=trees), False, n_threads=nt,
                trace_trees=trees)
    n, nf = xe.shape
    D = cfg.depth
    bins = oracle.bin_rowmajor(xe, cuts, cfg.n_bins)
    ds = Dataset(ctx, xe, y, cuts, cfg.n_bins)
    p = train_params(cfg)
    gains = np.zeros(nf, np.float64)
    gbins = np.zeros(nf, np.uint32)
    chosen = np.zeros(2, np.uint32)
    agree, worst, disagreements = 0, 0.0, []
    try:
        for t in range(trees):
            g = np.ascontiguousarray(o.tree_g[t])
            h = np.ascontiguousarray(o.tree_h[t])
            leaf = o.tree_leaf[t].astype(np.int32)
            for d in range(D):
                nd = np.ascontiguousarray(leaf >> (D - d), np.int32)
                ctx.check(N.lib.rw_debug_level_step(ds.h, C.byref(p), N.ptr(nd), N.ptr(g),
                                                    N.ptr(h), 1 << d, t, N.ptr(gains),
                                                    N.ptr(gbins), N.ptr(chosen)))
                k = t * D + d
                ref = (int(o.feat[k]), int(o.thr_bin[k]))
                gpu = (int(chosen[0]), int(chosen[1]))
                if gpu == ref:
                    agree += 1
                    continue
                e_g, e_h = _qexp(np.abs(g).max()), _qexp(h.max())
                g64, h64 = g.astype(np.float64), h.astype(np.float64)
                args = (leaf, g64, h64)
                ga, qa, fa = _gain_and_bounds(bins[:, ref[0]], *args, ref[1], D, d, cfg.n_bins,
                                              cfg.lambda_, cfg.min_child_h, e_g, e_h, nt)
                gb, qb, fb = _gain_and_bounds(bins[:, gpu[0]], *args, gpu[1], D, d, cfg.n_bins,
                                              cfg.lambda_, cfg.min_child_h, e_g, e_h, nt)
                bound = qa + qb + fa + fb
                gap = abs(ga - gb)
                worst = max(worst, gap / bound if bound > 0 else math.inf)
                disagreements.append({"tree": t, "level": d, "cpu_rs": ref, "gpu": gpu,
                                      "exact_gain_cpu_rs": ga, "exact_gain_gpu": gb,
                                      "gap": gap, "bound_q17": qa + qb, "bound_f32": fa + fb})
    finally:
        ds.close()
    rep = {"levels": trees * D, "agree": agree, "disagree": len(disagreements),
           "max_gap_over_bound": worst, "cpu_threads": nt,
           "disagreements": disagreements[:20]}
    _report(f"teacher_forced_{name}", rep)
    assert worst <= 1.0, rep
