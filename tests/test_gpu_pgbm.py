"""PGBM leaf variances and predict_std on the GPU, through the C ABI.

The reference computes the variances on its GPU path only (gpu_kernels.rs:1015-1080: per
leaf the f32-atomic sums of g, h and g*g, then lr^2 * max(S2/H - (G/H)^2, 0) when H > 1)
and sums them per row over the trees for predict_std (gpu_kernels.rs:1084-1120,
booster.rs:559-577). Here the three sums are exact wide-fixed-point integers evaluated in
f64, the same definition as oracle_exact's, so the bar is bit-exact.
"""
import numpy as np
import pytest

import oracle
import rustwood_b200 as rb
from rustwood_b200 import synth
from rustwood_b200.booster import Dataset, fit_dataset

pytestmark = pytest.mark.gpu

CASES = {
    "logistic_d6": dict(data=lambda: synth.c1(30_000), cfg=dict(n_trees=12, depth=6, n_bins=255,
                                                                learning_rate=0.2)),
    "l2_goss_pack4_d8": dict(data=lambda: synth.c4(30_000, nf=24),
                             cfg=dict(n_trees=6, depth=8, n_bins=16, pack4=True, goss_top=0.2,
                                      goss_other=0.1, objective="l2")),
    "l2_subsample_d4": dict(data=lambda: synth.c4(20_000, nf=9),
                            cfg=dict(n_trees=8, depth=4, n_bins=64, subsample=0.5,
                                     objective="l2")),
}


@pytest.mark.parametrize("name", list(CASES))
def test_pgbm_fit_and_predict_std_match_oracle(ctx, name):
    case = CASES[name]
    x, y, _, _ = case["data"]()
    cfg = rb.Config(pgbm=True, **case["cfg"])
    cuts = rb.compute_boundaries(x, cfg.n_bins, cfg.bin_sample, cfg.unique_bins)
    base = rb.base_score(y, cfg.objective)
    ds = Dataset(ctx, x, y, cuts, cfg.n_bins, cfg.pack4)
    r = fit_dataset(ds, cfg, base)
    plain = fit_dataset(ds, cfg.replace(pgbm=False), base)
    ds.close()
    o = oracle.train(x, y, cuts, base, n_trees=cfg.n_trees, depth=cfg.depth, n_bins=cfg.n_bins,
                     learning_rate=cfg.learning_rate, lambda_=cfg.lambda_,
                     min_child_h=cfg.min_child_h, subsample=cfg.subsample,
                     goss_top=cfg.goss_top, goss_other=cfg.goss_other,
                     objective=cfg.objective, exact=True, n_threads=4, pgbm=True)
    np.testing.assert_array_equal(r.feat, o.feat)
    np.testing.assert_array_equal(r.leafval.view(np.uint32), o.leafval.view(np.uint32))
    np.testing.assert_array_equal(r.leafvar.view(np.uint32), o.leafvar.view(np.uint32))
    assert (r.leafvar > 0).any()
    # the variances leave the model itself unchanged
    np.testing.assert_array_equal(plain.leafval.view(np.uint32), r.leafval.view(np.uint32))
    assert len(plain.leafvar) == 0
    # predict_std: per row sqrt(max(sum over trees of leafvar, 0)), summed in tree order in f32
    b = rb.Booster(cfg, ctx)
    b.n_features, b.base_score = x.shape[1], base
    b._take(r)
    xt = x[:5000]
    var = oracle.predict(xt, r.feat, r.thr, r.leafvar, 0.0, cfg.n_trees, cfg.depth)
    want = np.sqrt(np.maximum(var, np.float32(0.0)))
    got = b.predict_std(xt)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def test_predict_std_needs_variances(ctx):
    x, y, _, _ = synth.c1(2_000)
    cfg = rb.Config(n_trees=2, depth=3, n_bins=32)
    b = rb.Booster(cfg, ctx)
    b.fit(x, y)
    with pytest.raises(RuntimeError):
        b.predict_std(x)
