"""Categorical target encoding on the GPU (rw_target_encode) against the sequential f64
restatement of src/encoding.rs:44-95 (oracle.target_encode) and the host encoder.

The GPU sums labels as exact fixed-point integers in any order; the reference sums them
in f64 in row order. The two agree bit for bit wherever the reference's sums are exact,
which is what these cases use: 0/1 labels (C3) and small integer labels.
"""
import numpy as np
import pytest

import oracle
import rustwood_b200 as rb
from rustwood_b200 import _native as N
from rustwood_b200 import encoding, synth
from rustwood_b200.booster import target_encode_gpu

pytestmark = pytest.mark.gpu

CATS = list(range(7, 20))


@pytest.mark.parametrize("hash_buckets,label", [(0, "binary"), (7, "binary"), (0, "int"),
                                                (1000, "int")])
def test_gpu_target_encoding_matches_reference_order(ctx, hash_buckets, label):
    x, y, _, _ = synth.c3(50_003, seed=2)
    if label == "int":  # small integer labels: every f64 partial sum is exact
        y = np.floor(np.random.default_rng(3).random(len(y)) * 9 - 4).astype(np.float32)
    x = np.ascontiguousarray(x, np.float32)
    # negative and NaN codes in one feature (NaN rounds to code 0 like `as i64`)
    x[::97, 8] = -3.0
    x[::101, 9] = np.nan
    want_x, want_gm = oracle.target_encode(x, y, CATS, 10.0, 5, hash_buckets)
    host_x = x.copy()
    host_enc, host_gm = encoding.fit_transform_train(host_x, y, CATS, 10.0, 5, hash_buckets)
    got_x = x.copy()
    got_enc, got_gm = target_encode_gpu(ctx, got_x, y, CATS, 10.0, 5, hash_buckets)
    assert np.float32(got_gm) == np.float32(want_gm) == np.float32(host_gm)
    np.testing.assert_array_equal(got_x.view(np.uint32), want_x.view(np.uint32))
    assert len(got_enc) == len(host_enc)
    for g, h in zip(got_enc, host_enc):
        assert g.keys() == h.keys()
        for k in h:
            assert np.float32(g[k]).view(np.uint32) == np.float32(h[k]).view(np.uint32), k


def test_gpu_target_encoding_refuses_wide_key_ranges(ctx):
    x, y, _, _ = synth.c3(2_000, seed=4)
    x = np.ascontiguousarray(x, np.float32)
    x[::3, 7] = 3.0e9  # codes 0 .. 3e9: too many keys for the dense tables
    with pytest.raises(N.RwError) as ei:
        target_encode_gpu(ctx, x.copy(), y, CATS, 10.0, 5, 0)
    assert ei.value.code == N.RW_ERR_UNSUPPORTED
    # Booster.prepare falls back to the host encoder, with the host encoder's result
    cfg = rb.Config(n_trees=2, depth=3, n_bins=32, categorical=CATS)
    b = rb.Booster(cfg, ctx)
    xe, _, _ = b.prepare(x, y)
    want = x.copy()
    encoding.fit_transform_train(want, y, CATS, cfg.te_smoothing, 5, 0)
    np.testing.assert_array_equal(xe.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("hash_buckets", [0, 7])
def test_gpu_transform_matches_host_transform(ctx, hash_buckets):
    """encoding::transform on the GPU (rw_target_transform) equals the host transform for
    seen, unseen (beyond and inside the training range), negative and NaN codes."""
    from rustwood_b200.booster import target_transform_gpu
    x, y, xt, _ = synth.c3(20_000, n_test=6_007, seed=5)
    x = np.ascontiguousarray(x, np.float32)
    enc, gm = target_encode_gpu(ctx, x.copy(), y, CATS, 10.0, 5, hash_buckets)
    xt = np.ascontiguousarray(xt, np.float32)
    xt[::5, 7] = 77.0    # unseen, above the training codes
    xt[::7, 8] = -2.0    # unseen, below
    xt[::11, 9] = np.nan
    want = xt.copy()
    encoding.transform(want, CATS, enc, gm, hash_buckets)
    got = xt.copy()
    assert target_transform_gpu(ctx, got, CATS, enc, gm, hash_buckets)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    # too many slots for the dense tables: nothing is touched, the caller falls back
    untouched = xt.copy()
    assert not target_transform_gpu(ctx, untouched, CATS, enc, gm, hash_buckets, max_slots=4)
    np.testing.assert_array_equal(untouched.view(np.uint32), xt.view(np.uint32))


def test_booster_categorical_fit_and_predict_use_the_gpu_encoder(ctx):
    x, y, xt, _ = synth.c3(20_000, n_test=3_000, seed=6)
    cfg = rb.Config(n_trees=15, depth=5, n_bins=64, categorical=CATS)
    b = rb.Booster(cfg, ctx)
    b.fit(x, y)
    got = b.predict(xt)
    xe = np.array(xt, np.float32, order="C", copy=True)
    encoding.transform(xe, CATS, b.encoders, b.gmean, cfg.cat_hash_buckets)
    want = oracle.predict(xe, b.feat, b.thr, b.leafval, b.base_score, cfg.n_trees, cfg.depth)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
