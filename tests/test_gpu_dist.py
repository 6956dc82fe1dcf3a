"""Multi-GPU training and scoring through the C ABI, at 2, 4 and 8 ranks.

Two ways in:
  - one process per GPU (rw_ctx_create_rank): each rank builds its contiguous row shard
    with rw_dataset_create (n_global, row_offset) and runs rw_fit_dataset;
  - one process for all GPUs (rw_ctx_create with n_gpus > 1, what rustwood's
    single-process Booster binds): rw_fit takes the whole dataset and the library runs
    one rank per GPU on its own host thread.
Either way the library all-reduces the int64 histograms, the fixed-point scale maxima,
the GOSS digit counts and the per-tree leaf sums, over NVLink peer memory by default
(one-shot exchange at 2 ranks, two-shot above) and over NCCL with RW_PEER_EXCHANGE=0
(one case). Every rank's model must be bit-identical to the single-process exact oracle
on all rows (the bar of the 1-GPU parity tests), with ragged shards too. A case needs as
many GPUs as ranks and is skipped otherwise.
"""
import ctypes as C
import multiprocessing as mp
import os
import tempfile

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

KEYS = ("feat", "thr", "leafval", "fi_gain", "fi_count")
WORLDS = (2, 4, 8)


def _n_gpus() -> int:
    try:
        import torch
        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:
        return 0


def _case_data(case):
    from rustwood_b200 import synth
    if case["data"] == "c1":
        x, y, _, _ = synth.c1(case["n"], seed=case["seed"])
    else:
        x, y, _, _ = synth.c4(case["n"], seed=case["seed"], nf=20)
    return np.ascontiguousarray(x, np.float32), np.ascontiguousarray(y, np.float32)


def _cfg(case):
    from rustwood_b200 import Config
    return Config(n_trees=case["trees"], depth=case["depth"], n_bins=case["nb"],
                  learning_rate=0.2, objective=case["objective"], pack4=case.get("pack4", False),
                  goss_top=case.get("goss_top", 0.0), goss_other=case.get("goss_other", 0.1),
                  subsample=case.get("subsample", 1.0))


def _bounds(n, world, seed):
    """Ragged contiguous shards: world - 1 random cut points (each shard non-empty)."""
    rng = np.random.default_rng(seed)
    cuts = np.sort(rng.choice(np.arange(1, n), world - 1, replace=False))
    return [0] + [int(c) for c in cuts] + [n]


def _oracle(case, x, y, cuts, base, pgbm=False):
    cfg = _cfg(case)
    return oracle.train(x, y, cuts, base, n_trees=cfg.n_trees, depth=cfg.depth,
                        n_bins=cfg.n_bins, learning_rate=cfg.learning_rate, lambda_=cfg.lambda_,
                        min_child_h=cfg.min_child_h, subsample=cfg.subsample,
                        goss_top=cfg.goss_top, goss_other=cfg.goss_other,
                        objective=cfg.objective, exact=True, n_threads=4, pgbm=pgbm)


def _assert_model(m, o, who):
    np.testing.assert_array_equal(np.asarray(m["thr_bin"]).astype(np.uint32), o.thr_bin,
                                  err_msg=who)
    for k in KEYS:
        got = np.asarray(m[k])
        np.testing.assert_array_equal(got.view(np.uint32),
                                      getattr(o, k).astype(got.dtype).view(np.uint32),
                                      err_msg=f"{who} {k}")


def _rank_main(rank, world, q, case, bounds, cuts, base, out_dir):
    os.environ["RW_PEER_EXCHANGE"] = case.get("peer", "1")
    from rustwood_b200 import Context
    from rustwood_b200.booster import Dataset, fit_dataset
    if rank == 0:
        uid = Context.nccl_unique_id()
        for _ in range(world - 1):
            q.put(uid)
    else:
        uid = q.get(timeout=120)
    ctx = Context(rank, rank, world, uid)
    x, y = _case_data(case)
    lo, hi = bounds[rank], bounds[rank + 1]
    ds = Dataset(ctx, x[lo:hi], y[lo:hi], cuts, case["nb"], case.get("pack4", False),
                 n_global=len(y), row_offset=lo)
    r = fit_dataset(ds, _cfg(case), base)
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), feat=r.feat, thr=r.thr,
             thr_bin=r.thr_bin, leafval=r.leafval, fi_gain=r.fi_gain, fi_count=r.fi_count)
    ds.close()
    ctx.close()


CASES = [
    dict(id="c1_logistic", data="c1", n=200_003, seed=3, nb=255, trees=6, depth=6,
         objective="logistic"),
    dict(id="c4_goss_pack4", data="c4", n=300_000, seed=5, nb=16, trees=4, depth=8,
         objective="l2", pack4=True, goss_top=0.2, goss_other=0.1),
    dict(id="c1_subsample", data="c1", n=150_000, seed=7, nb=64, trees=5, depth=5,
         objective="logistic", subsample=0.5),
    dict(id="c1_nccl_transport", data="c1", n=120_001, seed=9, nb=255, trees=4, depth=6,
         objective="logistic", peer="0"),
]


@pytest.mark.parametrize("world", WORLDS)
@pytest.mark.parametrize("case", CASES, ids=[c["id"] for c in CASES])
def test_process_per_gpu_fit_matches_oracle_exact(case, world):
    if _n_gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    from rustwood_b200 import base_score, compute_boundaries
    x, y = _case_data(case)
    n = len(y)
    bounds = _bounds(n, world, case["seed"] + world)
    cfg = _cfg(case)
    cuts = compute_boundaries(x, cfg.n_bins)
    base = base_score(y, cfg.objective)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as out_dir:
        procs = [ctx.Process(target=_rank_main,
                             args=(r, world, q, case, bounds, cuts, base, out_dir))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        models = [dict(np.load(os.path.join(out_dir, f"rank{r}.npz"))) for r in range(world)]
    o = _oracle(case, x, y, cuts, base)
    for r, m in enumerate(models):
        _assert_model(m, o, f"rank {r}")


def _in_process_main(world, case, q):
    """One process, one context over `world` GPUs: rw_fit on the whole dataset, then
    scoring sharded over the GPUs (f32, u8 and the no-allocation entry point)."""
    try:
        os.environ["RW_PEER_EXCHANGE"] = case.get("peer", "1")
        import rustwood_b200 as rb
        from rustwood_b200 import _native as N
        from rustwood_b200.booster import train_params
        x, y = _case_data(case)
        n, nf = x.shape
        cfg = _cfg(case)
        cuts = rb.compute_boundaries(x, cfg.n_bins)
        base = rb.base_score(y, cfg.objective)
        ctx = rb.Context.multi(range(world))
        T, D = cfg.n_trees, cfg.depth
        out = dict(feat=np.zeros(T * D, np.uint32), thr=np.zeros(T * D, np.float32),
                   thr_bin=np.zeros(T * D, np.uint16), leafval=np.zeros(T << D, np.float32),
                   leafvar=np.zeros(T << D, np.float32),  # PGBM variances (every rank)
                   fi_gain=np.zeros(nf, np.float32), fi_count=np.zeros(nf, np.float32))
        p = train_params(cfg)
        p.pack4 = int(case.get("pack4", False))
        ctx.check(N.lib.rw_fit(ctx.h, C.byref(p), N.ptr(x), N.ptr(y), n, nf, N.ptr(cuts),
                               float(base),
                               *(N.ptr(out[k]) for k in ("feat", "thr", "thr_bin", "leafval",
                                                         "leafvar")),
                               N.ptr(out["fi_gain"]), N.ptr(out["fi_count"]), None))
        # scoring through the same context (row shards over the GPUs)
        b = rb.Booster(cfg, ctx)
        b.n_features, b.base_score = nf, np.float32(base)
        b.feat, b.thr, b.thr_bin, b.leafval = out["feat"], out["thr"], out["thr_bin"], out["leafval"]
        xs = np.ascontiguousarray(x[:50_007])
        margins = b.predict(xs)
        bins = oracle.bin_rowmajor(xs, cuts, cfg.n_bins).T.copy()
        margins_u8 = b.predict_bins(bins)
        m, keep = b.model()
        margins_na = np.empty(len(xs), np.float32)
        ctx.check(N.lib.rw_predict_f32_noalloc(ctx.h, C.byref(m), N.ptr(xs), len(xs), nf,
                                               N.ptr(margins_na)))
        ctx.close()
        q.put(("ok", dict(out, cuts=cuts, base=np.float32(base), margins=margins,
                          margins_u8=margins_u8, margins_na=margins_na)))
    except Exception as e:  # reported to the test process
        q.put(("error", repr(e)))


IN_PROCESS_CASES = [CASES[0], CASES[1], CASES[3]]


@pytest.mark.parametrize("world", WORLDS)
@pytest.mark.parametrize("case", IN_PROCESS_CASES, ids=[c["id"] for c in IN_PROCESS_CASES])
def test_one_context_over_several_gpus_matches_oracle_exact(case, world):
    """rw_ctx_create(gpu_ids, world): the single-process Booster trains and scores on
    several GPUs and gets the 1-GPU oracle_exact model bit for bit, PGBM leaf variances
    included (their g^2 sums take a second exchange)."""
    if _n_gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_in_process_main, args=(world, case, q))
    p.start()
    try:
        status, res = q.get(timeout=600)
    finally:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            p.join()
    assert status == "ok", res
    x, y = _case_data(case)
    o = _oracle(case, x, y, res["cuts"], float(res["base"]), pgbm=True)
    _assert_model(res, o, f"{world}-GPU context")
    np.testing.assert_array_equal(res["leafvar"].view(np.uint32), o.leafvar.view(np.uint32))
    cfg = _cfg(case)
    want = oracle.predict(np.ascontiguousarray(x[:50_007]), o.feat, o.thr, o.leafval,
                          float(res["base"]), cfg.n_trees, cfg.depth)
    for k in ("margins", "margins_u8", "margins_na"):
        np.testing.assert_array_equal(res[k].view(np.uint32), want.view(np.uint32), err_msg=k)
