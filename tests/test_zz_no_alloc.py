"""rw_predict_f32_noalloc: scoring for callers that cannot allocate device memory.

A serving process whose device memory is owned by another allocator, or a path that
must not pay cudaMalloc's implicit synchronisation, scores through this entry point,
which only uses the library's fixed 16 MiB staging array. Its margins must equal the
allocating entry point rw_predict_f32 bit-for-bit (the tolerance every scoring test in
this suite uses), on two calls in a row that reuse the same array.

The file name sorts last so a run that stops at the first failure has already run
every other test; it also passes on its own in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

from rustwood_b200 import _native as N
from rustwood_b200 import synth

pytestmark = pytest.mark.gpu


def _model(n_trees, depth, nf, seed):
    feat, _, leafval = synth.c5_model(n_trees, depth, nf, seed=seed)
    thr = np.random.default_rng(seed + 1).standard_normal(n_trees * depth).astype(np.float32)
    m = N.Model()
    m.n_trees, m.depth, m.n_features, m.base_score = n_trees, depth, nf, 0.125
    m.feat = feat.ctypes.data_as(C.POINTER(C.c_uint32))
    m.thr = thr.ctypes.data_as(C.POINTER(C.c_float))
    m.leafval = leafval.ctypes.data_as(C.POINTER(C.c_float))
    return m, (feat, thr, leafval)


def _score(fn, ctx, m, x):
    out = np.empty(x.shape[0], np.float32)
    ctx.check(fn(ctx.h, C.byref(m), N.ptr(x), x.shape[0], x.shape[1], N.ptr(out)))
    return out


def test_noalloc_scores_match_rw_predict_f32_twice_in_a_row():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from rustwood_b200 import Context
    ctx = Context(0)
    try:
        # call 1: 500-tree depth-6 model, more rows than one staging batch holds
        m1, keep1 = _model(500, 6, 54, seed=3)
        x1 = np.random.default_rng(10).standard_normal((400_003, 54)).astype(np.float32)
        want1 = _score(N.lib.rw_predict_f32, ctx, m1, x1)
        got1 = _score(N.lib.rw_predict_f32_noalloc, ctx, m1, x1)
        np.testing.assert_array_equal(got1.view(np.uint32), want1.view(np.uint32))
        # call 2: a different model and input reuse the same staging array
        m2, keep2 = _model(37, 8, 20, seed=7)
        x2 = np.random.default_rng(11).standard_normal((12_345, 20)).astype(np.float32)
        want2 = _score(N.lib.rw_predict_f32, ctx, m2, x2)
        got2 = _score(N.lib.rw_predict_f32_noalloc, ctx, m2, x2)
        np.testing.assert_array_equal(got2.view(np.uint32), want2.view(np.uint32))
        # the defining property: after the first call has loaded everything, further calls
        # leave the device's free memory unchanged (nothing allocated, nothing freed)
        free0 = torch.cuda.mem_get_info(0)[0]
        for _ in range(3):
            _score(N.lib.rw_predict_f32_noalloc, ctx, m1, x1)
            _score(N.lib.rw_predict_f32_noalloc, ctx, m2, x2)
        assert torch.cuda.mem_get_info(0)[0] == free0
        # a model without trees scores base_score, as rw_predict_f32 does (also with no
        # features)
        for nf0 in (5, 0):
            m0 = N.Model()
            m0.n_trees, m0.depth, m0.n_features, m0.base_score = 0, 6, nf0, -0.75
            x0 = np.zeros((1000, nf0), np.float32)
            want0 = _score(N.lib.rw_predict_f32, ctx, m0, x0)
            got0 = _score(N.lib.rw_predict_f32_noalloc, ctx, m0, x0)
            np.testing.assert_array_equal(got0, want0)
            assert (got0 == np.float32(-0.75)).all()
        # a model beyond the 4 MiB staging limit is rejected with a clear error
        m3, keep3 = _model(300, 12, 8, seed=9)
        with pytest.raises(N.RwError) as ei:
            _score(N.lib.rw_predict_f32_noalloc, ctx, m3, x2[:, :8].copy())
        assert ei.value.code == -1 and "4 MiB" in str(ei.value)
    finally:
        ctx.close()
