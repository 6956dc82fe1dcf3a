"""The CPU oracle against the golden fixtures, the pure-Python restatement and the
reference's own self-checks restated as known-answer tests (CPU only)."""
import ctypes
import glob
import os
import sys

import numpy as np
import pytest

import oracle

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import pyref  # noqa: E402

GOLDEN = sorted(glob.glob(os.path.join(HERE, "golden", "*.npz")))


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p) for p in GOLDEN])
def test_oracle_matches_golden(path):
    z = np.load(path)
    nb, uniq, trees, depth, lr, is_l2, exact, nt, sub = z["params"]
    nb, trees, depth, nt = int(nb), int(trees), int(depth), int(nt)
    cuts = oracle.compute_boundaries(z["x"], nb, unique=bool(uniq))
    np.testing.assert_array_equal(cuts.view(np.uint32), z["cuts"].view(np.uint32))
    obj = "l2" if is_l2 else "logistic"
    assert np.float32(oracle.base_score(z["y"], obj)) == z["base"]
    r = oracle.train(z["x"], z["y"], cuts, float(z["base"]), n_trees=trees, depth=depth,
                     n_bins=nb, learning_rate=float(lr), objective=obj, exact=bool(exact),
                     n_threads=nt, subsample=float(sub))
    for k in ("feat", "thr_bin"):
        np.testing.assert_array_equal(getattr(r, k), z[k])
    for k in ("thr", "leafval", "fi_gain", "fi_count"):
        np.testing.assert_array_equal(getattr(r, k).view(np.uint32), z[k].view(np.uint32))
    p = oracle.predict(z["x"], r.feat, r.thr, r.leafval, float(z["base"]), trees, depth)
    np.testing.assert_array_equal(p.view(np.uint32), z["pred"].view(np.uint32))


@pytest.mark.parametrize("exact,nt,obj,subtract", [
    (True, 1, "logistic", True), (False, 1, "logistic", True), (False, 4, "logistic", True),
    (False, 3, "l2", False), (True, 2, "l2", False),
])
def test_oracle_matches_python_restatement(exact, nt, obj, subtract):
    rng = np.random.default_rng(17 + nt)
    n, nf, nb = 120, 3, 7
    x = rng.standard_normal((n, nf)).astype(np.float32)
    y = ((rng.random(n) < 0.5) if obj == "logistic" else rng.standard_normal(n)).astype(np.float32)
    cuts = pyref.boundaries(x, nb)
    base = np.float32(oracle.base_score(y, obj))
    a = pyref.train(x, y, cuts, base, n_trees=2, depth=3, n_bins=nb, learning_rate=0.3,
                    objective=obj, exact=exact, n_threads=nt, subtract=subtract)
    b = oracle.train(x, y, cuts, float(base), n_trees=2, depth=3, n_bins=nb, learning_rate=0.3,
                     objective=obj, exact=exact, n_threads=nt, subtract=subtract)
    for k in ("feat", "thr_bin", "thr", "leafval", "fi_gain", "fi_count"):
        np.testing.assert_array_equal(a[k].view(np.uint32), getattr(b, k).view(np.uint32))


@pytest.mark.parametrize("obj,subsample", [("logistic", 1.0), ("l2", 0.5)])
def test_pgbm_leaf_variances_match_python_restatement(obj, subsample):
    """PGBM leaf variances (gpu_kernels.rs:1015-1080) from exact sums: the C oracle and the
    Python restatement agree bit for bit, and the margins' leaf values are unchanged."""
    rng = np.random.default_rng(5)
    n, nf, nb = 300, 3, 9
    x = rng.standard_normal((n, nf)).astype(np.float32)
    y = ((rng.random(n) < 0.4) if obj == "logistic" else 3 * rng.standard_normal(n)).astype(np.float32)
    cuts = pyref.boundaries(x, nb)
    base = np.float32(oracle.base_score(y, obj))
    kw = dict(n_trees=3, depth=3, n_bins=nb, learning_rate=0.3, objective=obj, subsample=subsample)
    a = pyref.train(x, y, cuts, base, exact=True, pgbm=True, **kw)
    b = oracle.train(x, y, cuts, float(base), exact=True, pgbm=True, **kw)
    c = oracle.train(x, y, cuts, float(base), exact=True, **kw)
    np.testing.assert_array_equal(a["leafvar"].view(np.uint32), b.leafvar.view(np.uint32))
    np.testing.assert_array_equal(b.leafval.view(np.uint32), c.leafval.view(np.uint32))
    assert (b.leafvar >= 0).all() and (b.leafvar > 0).any()


def test_kat_shared_memory_spike():
    """src/main.rs:27-47: 256 rows with bins i % 16 and unit weight give 16 per bin."""
    n = 256
    bins = (np.arange(n) % 16).astype(np.uint8).reshape(n, 1)
    node = np.zeros(n, np.int32)
    g = np.ones(n, np.float32)
    h = np.ones(n, np.float32)
    hist = oracle.level_hist_exact(bins, node, g, h, 0, 0, 1, False, 16)
    assert (hist[0, 0, :, 0] == 16).all() and (hist[0, 0, :, 1] == 16).all()


def test_kat_bin_split_equivalence():
    """src/gpu_kernels.rs:497-498: with bin = #{cut < v}, `bin > t` <=> `v > cut[t]`."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((5000, 3)).astype(np.float32)
    x[:, 1] = np.round(x[:, 1])
    cuts = oracle.compute_boundaries(x, 32)
    bins = oracle.bin_rowmajor(x, cuts, 32)
    c = cuts.reshape(3, 31)
    for f in range(3):
        for t in range(31):
            np.testing.assert_array_equal(bins[:, f] > t, x[:, f] > c[f, t])


def test_exact_and_faithful_modes_agree_on_clear_splits():
    from rustwood_b200 import synth
    x, y, xt, yt = synth.c1(20_000, 5_000, seed=2)
    cuts = oracle.compute_boundaries(x, 255)
    base = oracle.base_score(y)
    a = oracle.train(x, y, cuts, base, n_trees=15, depth=6, n_bins=255, learning_rate=0.2,
                     exact=True, n_threads=4)
    b = oracle.train(x, y, cuts, base, n_trees=15, depth=6, n_bins=255, learning_rate=0.2,
                     exact=False, n_threads=8)
    np.testing.assert_array_equal(a.feat, b.feat)
    np.testing.assert_array_equal(a.thr_bin, b.thr_bin)
    # Leaf sums come from the unquantised g/h in both modes (exact integers in a wide
    # fixed point against f64 accumulation), so the leaf values agree to the north-star
    # bound of 1e-5 relative with no absolute slack (measured: 2e-7; the remaining
    # differences come from glibc expf and the shared exponential differing by 1 ulp).
    np.testing.assert_allclose(a.leafval, b.leafval, rtol=1e-5, atol=0)
    pa = oracle.predict(xt, a.feat, a.thr, a.leafval, base, 15, 6)
    pb = oracle.predict(xt, b.feat, b.thr, b.leafval, base, 15, 6)
    assert abs(oracle.metric("auc", pa, yt) - oracle.metric("auc", pb, yt)) < 1e-4
    assert abs(oracle.metric("logloss", pa, yt) - oracle.metric("logloss", pb, yt)) < 1e-4


def test_exact_mode_is_thread_count_invariant():
    from rustwood_b200 import synth
    x, y, _, _ = synth.c1(8_000, seed=4)
    cuts = oracle.compute_boundaries(x, 64)
    base = oracle.base_score(y)
    runs = [oracle.train(x, y, cuts, base, n_trees=6, depth=5, n_bins=64, exact=True,
                         n_threads=nt) for nt in (1, 3, 8)]
    for r in runs[1:]:
        np.testing.assert_array_equal(r.leafval.view(np.uint32), runs[0].leafval.view(np.uint32))


def _correctly_rounded_expf(v: np.float32) -> np.float32:
    from decimal import Decimal, getcontext
    getcontext().prec = 60
    e = Decimal(float(v)).exp()
    f = np.float32(float(e))
    cands = [np.nextafter(f, np.float32(-np.inf)), f, np.nextafter(f, np.float32(np.inf))]
    return min(cands, key=lambda c: abs(Decimal(float(c)) - e))


def test_rw_expf_error_against_glibc():
    """The shared exponential is within 1 ulp of glibc expf over the logistic link's
    input range, and wherever the two differ it is the correctly rounded one (glibc's
    expf is not correctly rounded everywhere)."""
    libm = ctypes.CDLL("libm.so.6")
    libm.expf.argtypes = [ctypes.c_float]
    libm.expf.restype = ctypes.c_float
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.uniform(-104, 89, 20_000), rng.normal(0, 2, 20_000),
                         np.linspace(-1e-3, 1e-3, 2_001)]).astype(np.float32)
    worst, same = 0, 0
    for v in xs:
        a = np.float32(oracle.rw_expf(float(v)))
        b = np.float32(libm.expf(float(v)))
        if not np.isfinite(b) or b == 0:
            assert a == b
            continue
        d = abs(int(a.view(np.int32)) - int(b.view(np.int32)))
        worst = max(worst, d)
        same += d == 0
        if d:
            assert a == _correctly_rounded_expf(v), float(v)
    assert worst <= 1
    assert same / len(xs) > 0.998
    for v in rng.uniform(-104, 89, 300).astype(np.float32):
        assert np.float32(oracle.rw_expf(float(v))) == _correctly_rounded_expf(v)
    assert oracle.rw_expf(0.0) == 1.0


def test_rw_expf_python_and_c_agree():
    rng = np.random.default_rng(1)
    for v in rng.uniform(-100, 88, 3000).astype(np.float32):
        assert np.float32(oracle.rw_expf(float(v))).view(np.uint32) == \
            pyref.rw_expf(np.float32(v)).view(np.uint32)


def test_metrics_match_definitions():
    rng = np.random.default_rng(3)
    s = rng.normal(size=2000).astype(np.float32)
    s[::10] = s[1::10]  # ties
    y = (rng.random(2000) < 0.4).astype(np.float32)
    from sklearn.metrics import roc_auc_score
    assert abs(oracle.metric("auc", s, y) - roc_auc_score(y, s)) < 1e-12
    p = np.clip(1 / (1 + np.exp(-s.astype(np.float64))), 1e-7, 1 - 1e-7)
    ll = -np.mean(y * np.log(p) + (1 - y) * np.log(1 - p))
    assert abs(oracle.metric("logloss", s, y) - ll) < 1e-12
    assert abs(oracle.metric("rmse", s, y) - np.sqrt(np.mean((s - y.astype(np.float64)) ** 2))) < 1e-9
    assert abs(oracle.metric("accuracy", s, y) - np.mean((s > 0) == (y > 0.5))) < 1e-12


def test_target_encoding_product_matches_oracle():
    from rustwood_b200 import encoding, synth
    x, y, _, _ = synth.c3(5_000, seed=1)
    cats = list(range(7, 20))
    for hb in (0, 7):
        xo, gmo = oracle.target_encode(x, y, cats, 10.0, 5, hb)
        xp = x.copy()
        _, gmp = encoding.fit_transform_train(xp, y, cats, 10.0, 5, hb)
        assert np.float32(gmp) == np.float32(gmo)
        np.testing.assert_array_equal(xp.view(np.uint32), xo.view(np.uint32))


def _exact_level_choice(bins, node, qscale, g, h, n_nodes, nb, lam, mc):
    """cpu.rs's split choice for one level (src/cpu.rs:235-271: gains summed in node
    order, lowest flat (f, b) among the maxima) from exact fixed-point histograms."""
    e_g, e_h = qscale
    hist = oracle.level_hist_exact(bins, node, g, h, e_g, e_h, n_nodes, False, nb)
    cs = np.cumsum(hist, axis=2)
    pg = cs[..., 0].astype(np.float64) * 2.0 ** -e_g
    ph = cs[..., 1].astype(np.float64) * 2.0 ** -e_h
    nb1 = nb - 1
    gain = np.zeros((hist.shape[1], nb1))
    for nd in range(n_nodes):
        gt, ht = pg[nd, :, nb1:], ph[nd, :, nb1:]
        parent = gt * gt / (ht + lam)
        gl, hl = pg[nd, :, :nb1], ph[nd, :, :nb1]
        gr, hr = gt - gl, ht - hl
        valid = ((hl >= mc) & (hr >= mc)).astype(np.float64)
        with np.errstate(divide="ignore", invalid="ignore"):
            gain += valid * (gl * gl / (hl + lam) + gr * gr / (hr + lam) - parent)
    flat = int(np.argmax(gain.reshape(-1)))
    return flat // nb1, flat % nb1, gain


@pytest.mark.parametrize("shape", ["c1_64bins", "c2_255bins"])
def test_teacher_forced_exact_levels_choose_cpu_rs_splits(shape):
    """Teacher forcing: at every level of every tree of a faithful cpu.rs fit (oracle_ref,
    f32 histograms), the exact fixed-point level step -- the arithmetic the CUDA path
    matches bit for bit -- is fed the faithful model's own gradients and must choose the
    same split, or one whose gain is within a near-tie (relative gap < 1e-4) of it."""
    import shard_protocol as sp
    from rustwood_b200 import synth
    if shape == "c1_64bins":
        x, y, _, _ = synth.c1(20_000, seed=5)
        nb, T, D, lr = 64, 12, 6, 0.2
    else:  # C2-shaped: integer-valued and binary features, many tied bins
        x, y, _, _ = synth.c2(30_000, seed=6)
        nb, T, D, lr = 255, 10, 6, 0.3
    lam, mc = 1.0, float(np.float32(1e-3))
    cuts = oracle.compute_boundaries(x, nb)
    base = oracle.base_score(y)
    ref = oracle.train(x, y, cuts, base, n_trees=T, depth=D, n_bins=nb, learning_rate=lr,
                       exact=False, n_threads=4)
    bins = oracle.bin_rowmajor(x, cuts, nb)
    feat = ref.feat.reshape(T, D)
    tbin = ref.thr_bin.reshape(T, D)
    nl = 1 << D
    pred = np.full(len(y), np.float32(base), np.float32)
    checked = near_ties = 0
    for t in range(T):
        p = (np.float32(1.0) / (np.float32(1.0) + np.exp(-pred))).astype(np.float32)
        g = (p - y).astype(np.float32)
        h = np.maximum((p * (np.float32(1.0) - p)).astype(np.float32), np.float32(1e-6))
        qs = (sp.qscale_exp(int(sp.f32_bits(np.abs(g)).max())),
              sp.qscale_exp(int(sp.f32_bits(h).max())))
        node = np.zeros(len(y), np.int64)
        for d in range(D):
            f, b, gain = _exact_level_choice(bins, node.astype(np.int32), qs, g, h, 1 << d,
                                             nb, lam, mc)
            fr, br = int(feat[t, d]), int(tbin[t, d])
            checked += 1
            if (f, b) != (fr, br):
                best, theirs = gain[f, b], gain[fr, br]
                assert best - theirs <= 1e-4 * max(abs(best), 1e-12), (t, d, best, theirs)
                near_ties += 1
            node = node * 2 + (bins[:, fr] > br)  # follow the faithful tree
        pred = (pred + ref.leafval[t * nl:(t + 1) * nl][node]).astype(np.float32)
    assert checked == T * D
    assert near_ties <= checked // 10


def test_fixed_point_scale_bounds():
    """The round's scale keeps every |q| within 2^17 (so 8192 rows sum exactly in a 32-bit
    shared cell: 2^13 * 2^17 = 2^30) and uses the range: the largest |q| is at least 2^16.
    Restated from rw_expf.h (rw_qscale_exp, rw_quantize) in tests/shard_protocol.py."""
    import shard_protocol as sp
    rng = np.random.default_rng(9)
    for mag in (1e-30, 1e-8, 1e-3, 0.25, 1.0, 3.0, 1e6, 1e30, 3.4e38):
        x = (rng.uniform(-1.0, 1.0, 4097) * mag).astype(np.float32)
        x[0] = np.float32(mag)  # make the maximum exact
        e = sp.qscale_exp(int(sp.f32_bits(np.abs(x)).max()))
        q = sp.quantize(x, e)
        top = int(np.abs(q).max())
        assert top <= 1 << sp.QBITS, (mag, top)
        if -126 < e < 100:  # not clamped at the exponent limits
            assert top >= 1 << (sp.QBITS - 1), (mag, top)
    assert (8192 << sp.QBITS) <= 1 << 30
