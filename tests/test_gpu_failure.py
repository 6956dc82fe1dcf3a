"""Failure detection on one GPU, with no fault: bounded device-side waits on peer ranks.

Every wait of a peer exchange is bounded by %globaltimer; when it expires the kernel
sets the error word and returns, later exchanges skip their waits, and the host reports
RW_ERR_TIMEOUT. Here rank 1 is a local buffer that nothing ever runs for, so its signal
never comes (or comes with its error bit set): the waits must end by themselves within
their limit, the error word must say why, and a fit on such a context must return an
error instead of waiting. No wait here can run longer than its limit (<= 50 ms).
"""
import ctypes as C
import time

import numpy as np
import pytest

from rustwood_b200 import _native as N
from rustwood_b200 import synth

pytestmark = pytest.mark.gpu


def _wait(ctx, mode, timeout_ms=50):
    err = C.c_int32(-1)
    ms = C.c_float(0)
    ctx.check(N.lib.rw_debug_peer_wait(ctx.h, mode, timeout_ms, C.byref(err), C.byref(ms)))
    return err.value, ms.value


def test_peer_wait_expires_and_reports(ctx):
    err, ms = _wait(ctx, 0, 50)  # rank 1 never signals
    assert err == 2
    assert 45.0 <= ms < 2000.0  # waited for its limit, then returned


def test_peer_error_bit_reaches_this_rank(ctx):
    err, ms = _wait(ctx, 1, 50)  # rank 1 signalled with its error bit
    assert err == 3
    assert ms < 45.0


def test_wait_after_an_expired_one_is_skipped(ctx):
    err, ms = _wait(ctx, 2, 50)  # this rank's error word already says a wait expired
    assert err == 2
    assert ms < 45.0


def test_normal_signal_passes(ctx):
    err, ms = _wait(ctx, 3, 50)
    assert err == 0
    assert ms < 45.0


def test_fit_with_a_rank_that_never_arrives_returns_timeout():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from rustwood_b200 import Config, base_score, compute_boundaries
    from rustwood_b200.booster import Dataset, fit_dataset
    h = C.c_void_p()
    N.check(N.lib.rw_debug_lonely_rank_ctx(0, 50, C.byref(h)))

    class Ctx:  # the Context interface Dataset and fit_dataset use
        pass
    ctx = Ctx()
    ctx.h = h
    ctx.check = lambda code: N.check(code, h)
    try:
        x, y, _, _ = synth.c1(20_000, seed=1)
        cuts = compute_boundaries(x, 32)
        ds = Dataset(ctx, x, y, cuts, 32)
        cfg = Config(n_trees=3, depth=4, n_bins=32)
        t0 = time.perf_counter()
        with pytest.raises(N.RwError) as ei:
            fit_dataset(ds, cfg, base_score(y, "logistic"))
        elapsed = time.perf_counter() - t0
        assert ei.value.code == -6, str(ei.value)  # RW_ERR_TIMEOUT
        assert "peer" in str(ei.value)
        # the first expired wait ends every later one at once: far below one limit per wait
        assert elapsed < 5.0
        assert N.lib.rw_ctx_peer_failed(h) == 1
        # the context refuses further exchanges instead of waiting again
        with pytest.raises(N.RwError) as ei2:
            fit_dataset(ds, cfg, base_score(y, "logistic"))
        assert "timed out" in str(ei2.value)
        ds.close()
    finally:
        N.lib.rw_ctx_destroy(h)
