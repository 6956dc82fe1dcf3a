"""GPU parity against the oracle, through the C ABI.

Bar: integer/index outputs (bins, histograms, chosen (feature, threshold) sequences,
leaf indices) bit-exact; floating outputs (leaf values, thresholds, feature importance,
margins) bit-exact as well, because the CUDA path and oracle_exact share one
arithmetic definition (fixed-point histograms, f64 gains, the same exponential).
"""
import numpy as np
import pytest

import oracle
import rustwood_b200 as rb
from rustwood_b200 import _native as N
from rustwood_b200 import synth
from rustwood_b200.booster import Dataset, fit_dataset

pytestmark = pytest.mark.gpu


def _exact_fit(x, y, cfg, ctx, **kw):
    cuts = rb.compute_boundaries(x, cfg.n_bins, cfg.bin_sample, cfg.unique_bins)
    base = rb.base_score(y, cfg.objective)
    ds = Dataset(ctx, x, y, cuts, cfg.n_bins, cfg.pack4)
    r = fit_dataset(ds, cfg, base)
    ds.close()
    o = oracle.train(x, y, cuts, base, n_trees=cfg.n_trees, depth=cfg.depth, n_bins=cfg.n_bins,
                     learning_rate=cfg.learning_rate, lambda_=cfg.lambda_,
                     min_child_h=cfg.min_child_h, subsample=cfg.subsample,
                     colsample=cfg.colsample, goss_top=cfg.goss_top, goss_other=cfg.goss_other,
                     objective=cfg.objective, subtract=cfg.subtract, monotone=cfg.monotone,
                     exact=True, n_threads=4)
    return r, o, cuts, base


def _assert_same_model(r, o):
    np.testing.assert_array_equal(r.feat, o.feat)
    np.testing.assert_array_equal(r.thr_bin.astype(np.uint32), o.thr_bin)
    np.testing.assert_array_equal(r.thr.view(np.uint32), o.thr.view(np.uint32))
    np.testing.assert_array_equal(r.leafval.view(np.uint32), o.leafval.view(np.uint32))
    np.testing.assert_array_equal(r.fi_count, o.fi_count)
    np.testing.assert_array_equal(r.fi_gain.view(np.uint32), o.fi_gain.view(np.uint32))


def test_expf_device_matches_host(ctx):
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.uniform(-110, 95, 200_000), rng.normal(0, 3, 100_000),
                        [0.0, -0.0, 88.7, 88.73, -103.9, -104.0, np.inf, -np.inf, np.nan]]
                       ).astype(np.float32)
    out_rw = np.empty_like(x)
    out_cu = np.empty_like(x)
    ctx.check(N.lib.rw_debug_expf(ctx.h, N.ptr(x), len(x), N.ptr(out_rw), N.ptr(out_cu)))
    host = np.array([oracle.rw_expf(float(v)) for v in x], dtype=np.float32)
    np.testing.assert_array_equal(out_rw.view(np.uint32), host.view(np.uint32))
    # CUDA expf is documented within 2 ulp; the shared routine must sit within that band.
    fin = np.isfinite(out_cu) & np.isfinite(out_rw) & (out_cu > 0)
    ulp = np.abs(out_rw[fin].view(np.int32).astype(np.int64) -
                 out_cu[fin].view(np.int32).astype(np.int64))
    assert ulp.max() <= 2


@pytest.mark.parametrize("case", ["c1", "c2", "c3_unique", "nan_inf"])
def test_binning_matches_oracle(ctx, case):
    if case == "c1":
        x, y, _, _ = synth.c1(30_011)
        nb, uniq = 255, False
    elif case == "c2":
        x, y, _, _ = synth.c2(20_000)
        nb, uniq = 255, False
    elif case == "c3_unique":
        x, y, _, _ = synth.c3(10_000)
        nb, uniq = 64, True
    else:
        x, y, _, _ = synth.c1(5_003)
        x = x.copy()
        x[::7, 3] = np.nan
        x[::11, 5] = np.inf
        x[::13, 6] = -np.inf
        nb, uniq = 16, False
    cuts = rb.compute_boundaries(np.nan_to_num(x, nan=0.0), nb, 200_000, uniq)
    ds = Dataset(ctx, x, y, cuts, nb)
    got = ds.bins()
    ds.close()
    want = oracle.bin_rowmajor(x, cuts, nb).T
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("nf,nb,groups,odd,packed", [
    (28, 255, 1, 0, False), (54, 255, 16, 1, False), (3, 255, 4, 1, False),
    (100, 16, 64, 1, True), (1, 2, 1, 0, False), (33, 256, 8, 0, False), (20, 64, 2, 1, False),
])
def test_level_hist_matches_oracle(ctx, nf, nb, groups, odd, packed):
    rng = np.random.default_rng(nf * 1000 + groups)
    n = 40_003
    x = rng.standard_normal((n, nf)).astype(np.float32)
    x[:, 0] = np.round(x[:, 0])  # heavy ties -> hot bins
    y = np.zeros(n, np.float32)
    cuts = rb.compute_boundaries(x, nb)
    ds = Dataset(ctx, x, y, cuts, nb, pack4=packed)
    span = groups * (2 if odd else 1)
    node = rng.integers(0, span, n).astype(np.int32)
    node[rng.random(n) < 0.1] = -1
    g = rng.normal(0, 1, n).astype(np.float32)
    h = rng.uniform(1e-6, 0.25, n).astype(np.float32)
    # scales as the trainer picks them (|q| <= 2^RW_QBITS, RW_QBITS = 17)
    e_g = 17 - int(np.frexp(np.abs(g).max())[1])
    e_h = 17 - int(np.frexp(h.max())[1])
    got = np.zeros((groups, nf, nb, 2), np.int64)
    ctx.check(N.lib.rw_debug_level_hist(ds.h, N.ptr(node), N.ptr(g), N.ptr(h), e_g, e_h, groups,
                                        odd, N.ptr(got)))
    ds.close()
    want = oracle.level_hist_exact(oracle.bin_rowmajor(x, cuts, nb), node, g, h, e_g, e_h, groups,
                                   odd, nb)
    np.testing.assert_array_equal(got, want)


def test_large_pageable_inputs_upload_exactly(ctx):
    """Pageable host inputs of 32 MiB and more take the library's staged upload (pinned
    slots filled by several host threads, chunks not a multiple of the slot): the binned
    dataset and the margins equal the host restatements bit for bit."""
    x, y, _, _ = synth.c2(170_003)  # 36.7 MB of f32 rows
    cuts = rb.compute_boundaries(x, 255)
    cfg = rb.Config(n_trees=3, depth=4, n_bins=255)
    base = rb.base_score(y, cfg.objective)
    ds = Dataset(ctx, x, y, cuts, 255)
    try:
        np.testing.assert_array_equal(ds.bins(), oracle.bin_rowmajor(x, cuts, 255).T)
        r = fit_dataset(ds, cfg, base)
    finally:
        ds.close()
    b = rb.Booster(cfg, ctx)
    b.n_features, b.base_score = x.shape[1], np.float32(base)
    b._take(r)
    want = oracle.predict(x, r.feat, r.thr, r.leafval, base, cfg.n_trees, cfg.depth)
    np.testing.assert_array_equal(b.predict(x).view(np.uint32), want.view(np.uint32))


CASES = {
    "c1": dict(data=lambda: synth.c1(30_000), cfg=dict(n_trees=25, depth=6, n_bins=255,
                                                         learning_rate=0.2)),
    "c2": dict(data=lambda: synth.c2(40_000), cfg=dict(n_trees=12, depth=6, n_bins=255,
                                                         learning_rate=0.3)),
    "c3": dict(data=lambda: synth.c3(20_000), cfg=dict(n_trees=20, depth=6, n_bins=255,
                                                         categorical=list(range(7, 20)),
                                                         unique_bins=True, monotone=[1])),
    "l2_goss_pack4_d8": dict(data=lambda: synth.c4(30_000, nf=24),
                             cfg=dict(n_trees=10, depth=8, n_bins=16, pack4=True,
                                      goss_top=0.2, goss_other=0.1, objective="l2")),
    "subsample_colsample": dict(data=lambda: synth.c1(20_000),
                                cfg=dict(n_trees=10, depth=5, n_bins=128, subsample=0.5,
                                         colsample=0.6)),
    "no_subtract_d3": dict(data=lambda: synth.c1(15_000),
                           cfg=dict(n_trees=8, depth=3, n_bins=64, subtract=False)),
    "depth1_l2": dict(data=lambda: synth.c4(10_000, nf=7),
                      cfg=dict(n_trees=15, depth=1, n_bins=255, objective="l2")),
    "depth12_small": dict(data=lambda: synth.c1(6_000),
                          cfg=dict(n_trees=2, depth=12, n_bins=32)),
    "goss_logistic": dict(data=lambda: synth.c1(25_000),
                          cfg=dict(n_trees=8, depth=6, n_bins=255, goss_top=0.3,
                                   goss_other=0.2)),
}


@pytest.mark.parametrize("name", list(CASES))
def test_fit_matches_oracle_exact(ctx, name):
    case = CASES[name]
    x, y, _, _ = case["data"]()
    cfg = rb.Config(**case["cfg"])
    if cfg.categorical:
        b = rb.Booster(cfg, ctx)
        x, _, _ = b.prepare(x, y)
        cfg = cfg.replace(categorical=[])
    r, o, cuts, base = _exact_fit(x, y, cfg, ctx)
    _assert_same_model(r, o)
    # scoring: GPU f32 and u8 scorers vs predict_cpu, bit-exact
    b = rb.Booster(cfg, ctx)
    b.n_features, b.base_score = x.shape[1], base
    b._take(r)
    want = oracle.predict(x, r.feat, r.thr, r.leafval, base, cfg.n_trees, cfg.depth)
    got = b.predict(x)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    bins = oracle.bin_rowmajor(x, cuts, cfg.n_bins).T
    if cfg.depth <= 12:
        got_u8 = b.predict_bins(bins)
        np.testing.assert_array_equal(got_u8.view(np.uint32), want.view(np.uint32))


def test_predict_u8_random_model(ctx):
    feat, thr_bin, leafval = synth.c5_model(n_trees=500, depth=6, nf=54, seed=3)
    n = 20_011
    bins = synth.c5_bins(n, 54, seed=4)
    # raw-threshold twin of the same model: thr = cut[f][t] on a synthetic cut table
    cuts = np.sort(np.random.default_rng(5).standard_normal((54, 255)).astype(np.float32), axis=1)
    thr = cuts[feat, thr_bin]
    x = np.empty((n, 54), np.float32)
    for f in range(54):  # bin b holds (cut[b-1], cut[b]]: take cut[b], or above the last cut
        x[:, f] = np.where(bins[f] < 255, cuts[f, np.minimum(bins[f], 254)], cuts[f, 254] + 1.0)
    np.testing.assert_array_equal(oracle.bin_rowmajor(x, cuts.ravel(), 256).T, bins)
    want = oracle.predict(x, feat, thr, leafval, 0.25, 500, 6)
    b = rb.Booster(rb.Config(n_trees=500, depth=6), ctx)
    b.n_features, b.base_score = 54, np.float32(0.25)
    b.feat, b.thr, b.thr_bin, b.leafval = feat, thr, thr_bin, leafval
    got = b.predict_bins(bins)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    got32 = b.predict(x)
    np.testing.assert_array_equal(got32.view(np.uint32), want.view(np.uint32))


def _raw_twin(bins, feat, thr_bin, nf, seed):
    """Raw f32 rows and thresholds that bin to `bins` against a synthetic cut table."""
    cuts = np.sort(np.random.default_rng(seed).standard_normal((nf, 255)).astype(np.float32),
                   axis=1)
    x = np.empty((bins.shape[1], nf), np.float32)
    for f in range(nf):
        x[:, f] = np.where(bins[f] < 255, cuts[f, np.minimum(bins[f], 254)], cuts[f, 254] + 1.0)
    return x, cuts[feat, thr_bin]


@pytest.mark.parametrize("depth,trees,nf,n", [
    (1, 7, 3, 12289), (4, 100, 20, 16385), (6, 500, 54, 12289), (8, 1200, 10, 17000),
    (10, 50, 30, 15000), (6, 64, 120, 14000), (6, 500, 54, 16388), (3, 33, 5, 13316),
    (6, 251, 54, 16384), (7, 300, 64, 20488),
])
def test_predict_u8_shapes(ctx, depth, trees, nf, n):
    """The u8 scorers for batches above 12288 rows (tiled shared-memory kernel for depth <=
    8 with tree chunks, the older byte-SIMD kernel for wide rows, the scalar kernel for
    depth > 8 or a row stride not a multiple of 4) against predict_cpu on the
    raw-threshold twin of the same model."""
    feat, thr_bin, leafval = synth.c5_model(n_trees=trees, depth=depth, nf=nf, seed=depth)
    bins = synth.c5_bins(n, nf, seed=depth + 1)
    x, thr = _raw_twin(bins, feat, thr_bin, nf, seed=depth + 2)
    want = oracle.predict(x, feat, thr, leafval, -0.5, trees, depth)
    b = rb.Booster(rb.Config(n_trees=trees, depth=depth), ctx)
    b.n_features, b.base_score = nf, np.float32(-0.5)
    b.feat, b.thr, b.thr_bin, b.leafval = feat, thr, thr_bin, leafval
    got = b.predict_bins(bins)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("depth,trees,nf,n", [
    (1, 1, 1, 1), (6, 500, 54, 1), (6, 500, 54, 1000), (12, 40, 9, 37), (9, 3000, 16, 300),
    (4, 100, 20, 4097), (6, 500, 54, 12288), (2, 12289, 4, 64),
])
def test_small_batch_scoring(ctx, depth, trees, nf, n):
    """Batches of at most 12288 rows (one CTA per row, its threads on different trees, the
    leaf values added in tree order by one thread) against predict_cpu, through both
    host-buffer entry points (u8 bins and raw f32 rows). 3000 trees put several trees on
    each thread; 12,289 trees exceed the kernel's 48 KB of leaf values and take the
    chunked scorers instead."""
    feat, thr_bin, leafval = synth.c5_model(n_trees=trees, depth=depth, nf=nf, seed=depth + 20)
    bins = synth.c5_bins(n, nf, seed=depth + 21)
    x, thr = _raw_twin(bins, feat, thr_bin, nf, seed=depth + 22)
    want = oracle.predict(x, feat, thr, leafval, 0.75, trees, depth)
    b = rb.Booster(rb.Config(n_trees=trees, depth=depth), ctx)
    b.n_features, b.base_score = nf, np.float32(0.75)
    b.feat, b.thr, b.thr_bin, b.leafval = feat, thr, thr_bin, leafval
    got = b.predict_bins(bins)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    got32 = b.predict(x)
    np.testing.assert_array_equal(got32.view(np.uint32), want.view(np.uint32))


def test_tiled_scorer_alternating_model_sizes(ctx):
    """The tiled u8 scorer's shared-memory size follows the model: scoring a large model,
    then a small one, then the large one again must not leave the kernel's limit at the
    small size (each call bit-exact against predict_cpu)."""
    n, nf = 13_000, 54
    bins = synth.c5_bins(n, nf, seed=31)
    for trees in (500, 20, 500, 120):
        feat, thr_bin, leafval = synth.c5_model(n_trees=trees, depth=6, nf=nf, seed=trees)
        x, thr = _raw_twin(bins, feat, thr_bin, nf, seed=32)
        want = oracle.predict(x, feat, thr, leafval, 0.0, trees, 6)
        b = rb.Booster(rb.Config(n_trees=trees, depth=6), ctx)
        b.n_features, b.base_score = nf, np.float32(0.0)
        b.feat, b.thr, b.thr_bin, b.leafval = feat, thr, thr_bin, leafval
        got = b.predict_bins(bins)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def test_fit_vs_faithful_cpu_rs(ctx):
    """Against oracle_ref (faithful cpu.rs, f32 histograms, glibc expf): identical splits
    except at near-ties, and test metrics within 1e-4."""
    x, y, xt, yt = synth.c1(30_000, 10_000, seed=7)
    cfg = rb.Config(n_trees=40, depth=6, n_bins=255, learning_rate=0.2)
    b = rb.Booster(cfg, ctx)
    b.fit(x, y)
    cuts = rb.compute_boundaries(x, 255)
    base = rb.base_score(y, "logistic")
    o = oracle.train(x, y, cuts, base, n_trees=40, depth=6, n_bins=255, learning_rate=0.2,
                     exact=False, n_threads=8)
    agree = np.mean(b.feat == o.feat)
    pg = b.predict(xt)
    po = oracle.predict(xt, o.feat, o.thr, o.leafval, base, 40, 6)
    assert abs(oracle.metric("auc", pg, yt) - oracle.metric("auc", po, yt)) < 1e-4
    assert abs(oracle.metric("logloss", pg, yt) - oracle.metric("logloss", po, yt)) < 1e-4
    assert agree > 0.9


def test_errors_are_reported(ctx):
    # depth 13 passes the host mirror and the parameter struct; the library rejects it
    cfg = rb.Config(n_trees=1, depth=13, n_bins=256)
    rb.train_params(cfg)
    x, y, _, _ = synth.c1(1000)
    cuts = rb.compute_boundaries(x, 256)
    ds = Dataset(ctx, x, y, cuts, 256)
    with pytest.raises(N.RwError) as ei:
        fit_dataset(ds, cfg, 0.0)
    assert ei.value.code == -1 and "depth" in str(ei.value)
    ds.close()
    x, y, _, _ = synth.c1(1000)
    cuts = rb.compute_boundaries(x, 64)
    ds = Dataset(ctx, x, y, cuts, 64)
    with pytest.raises(N.RwError) as ei:
        fit_dataset(ds, rb.Config(n_trees=1, depth=4, n_bins=32), 0.0)
    assert ei.value.code == -1
    with pytest.raises(N.RwError) as ei:
        fit_dataset(ds, rb.Config(n_trees=1, depth=4, n_bins=64, clamp_hessian=0.5), 0.0)
    assert ei.value.code == -5
    ds.close()
