"""compute_boundaries (src/data.rs:86-146) on the GPU against the host restatement
(rw_compute_boundaries, itself checked against the oracle on the CPU): the cut tables
must be bit-identical -- quantile and unique modes, heavy ties, -0.0 next to +0.0, sample
strides 1..10, 2..256 bins -- and a fit whose cut table comes from the GPU equals the
fit from the host table.
"""
import ctypes as C

import numpy as np
import pytest

import rustwood_b200 as rb
from rustwood_b200 import _native as N
from rustwood_b200 import synth

pytestmark = pytest.mark.gpu


def _gpu_cuts(ctx, x, n_bins, sample, unique):
    import torch
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda(ctx.gpu)
    out = np.empty(x.shape[1] * (n_bins - 1), np.float32)
    ctx.check(N.lib.rw_compute_boundaries_device(ctx.h, C.c_void_p(xd.data_ptr()), x.shape[0],
                                                 x.shape[1], n_bins, sample, int(unique),
                                                 N.ptr(out)))
    return out


def _signed_zeros(rng, n, nf):
    x = np.round(rng.standard_normal((n, nf)) * 1.5).astype(np.float32)  # ties, many zeros
    z = x == 0
    x[z & (rng.random((n, nf)) < 0.5)] = np.float32(-0.0)
    return x


CASES = {
    "c1_100k": lambda: synth.c1(100_000)[0],
    "c2_1M_stride5": lambda: synth.c2(1_000_000)[0],
    "c4_2M_stride10": lambda: synth.c4(2_000_000, nf=30)[0],
    "signed_zeros": lambda: _signed_zeros(np.random.default_rng(3), 50_000, 6),
    "tiny": lambda: np.random.default_rng(4).standard_normal((3, 2)).astype(np.float32),
    "constant": lambda: np.full((1000, 3), 2.5, np.float32),
}


_DATA = {}


@pytest.mark.parametrize("n_bins", [2, 16, 255, 256])
@pytest.mark.parametrize("unique", [False, True])
@pytest.mark.parametrize("case", list(CASES))
def test_gpu_cut_table_matches_host(ctx, case, n_bins, unique):
    if case not in _DATA:
        _DATA.clear()
        _DATA[case] = CASES[case]()
    x = _DATA[case]
    for sample in (200_000, 7_777):
        want = rb.compute_boundaries(x, n_bins, sample, unique)
        got = _gpu_cuts(ctx, x, n_bins, sample, unique)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32),
                                      err_msg=f"{case} bins={n_bins} sample={sample}")


def test_fit_with_gpu_boundaries_equals_host_cut_fit(ctx):
    from rustwood_b200.booster import train_params
    x, y, _, _ = synth.c2(300_000, seed=5)
    cfg = rb.Config(n_trees=10, depth=6, n_bins=255, learning_rate=0.3)
    base = rb.base_score(y, "logistic")
    T, D, nf = cfg.n_trees, cfg.depth, x.shape[1]

    def outs():
        return dict(feat=np.zeros(T * D, np.uint32), thr=np.zeros(T * D, np.float32),
                    thr_bin=np.zeros(T * D, np.uint16), leafval=np.zeros(T << D, np.float32),
                    fi_gain=np.zeros(nf, np.float32), fi_count=np.zeros(nf, np.float32))
    p = train_params(cfg)
    a, b = outs(), outs()
    cuts = rb.compute_boundaries(x, 255)
    ctx.check(N.lib.rw_fit(ctx.h, C.byref(p), N.ptr(x), N.ptr(y), len(y), nf, N.ptr(cuts), base,
                           *(N.ptr(a[k]) for k in ("feat", "thr", "thr_bin", "leafval")), None,
                           N.ptr(a["fi_gain"]), N.ptr(a["fi_count"]), None))
    gcuts = np.zeros_like(cuts)
    ctx.check(N.lib.rw_fit_with_boundaries(ctx.h, C.byref(p), N.ptr(x), N.ptr(y), len(y), nf,
                                           200_000, 0, base, N.ptr(gcuts),
                                           *(N.ptr(b[k]) for k in ("feat", "thr", "thr_bin",
                                                                    "leafval")),
                                           None, N.ptr(b["fi_gain"]), N.ptr(b["fi_count"]), None))
    np.testing.assert_array_equal(gcuts.view(np.uint32), cuts.view(np.uint32))
    for k in a:
        np.testing.assert_array_equal(a[k].view(a[k].dtype), b[k], err_msg=k)
