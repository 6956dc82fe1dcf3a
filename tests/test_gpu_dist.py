"""Multi-GPU training through the C ABI: one process per GPU, NCCL inside librwgpu.

Each rank builds its contiguous row shard with rw_dataset_create (n_global, row_offset)
on its own GPU and runs rw_fit_dataset; the library all-reduces the int64 histograms,
the fixed-point scale maxima and the GOSS digit counts, over NVLink peer memory by
default and over NCCL with RW_PEER_EXCHANGE=0 (one case). Every rank's model must be
bit-identical to the single-process exact oracle on all rows (the same bar as the
1-GPU parity tests), for ragged shards too. Needs at least 2 GPUs; skipped otherwise.
"""
import multiprocessing as mp
import os
import tempfile

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

KEYS = ("feat", "thr", "leafval", "fi_gain", "fi_count")


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
         objective="logistic", split=(0.37,)),
    dict(id="c4_goss_pack4", data="c4", n=300_000, seed=5, nb=16, trees=4, depth=8,
         objective="l2", pack4=True, goss_top=0.2, goss_other=0.1, split=(0.5,)),
    dict(id="c1_subsample", data="c1", n=150_000, seed=7, nb=64, trees=5, depth=5,
         objective="logistic", subsample=0.5, split=(0.5,)),
    dict(id="c1_nccl_transport", data="c1", n=120_001, seed=9, nb=255, trees=4, depth=6,
         objective="logistic", split=(0.61,), peer="0"),
]


@pytest.mark.parametrize("case", CASES, ids=[c["id"] for c in CASES])
def test_two_gpu_fit_matches_oracle_exact(case):
    if _n_gpus() < 2:
        pytest.skip("needs 2 GPUs")
    from rustwood_b200 import base_score, compute_boundaries
    world = 2
    x, y = _case_data(case)
    n = len(y)
    bounds = [0] + [int(f * n) for f in case["split"]] + [n]
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
    o = oracle.train(x, y, cuts, base, n_trees=cfg.n_trees, depth=cfg.depth, n_bins=cfg.n_bins,
                     learning_rate=cfg.learning_rate, lambda_=cfg.lambda_,
                     min_child_h=cfg.min_child_h, subsample=cfg.subsample,
                     goss_top=cfg.goss_top, goss_other=cfg.goss_other,
                     objective=cfg.objective, exact=True, n_threads=4)
    for r, m in enumerate(models):
        np.testing.assert_array_equal(m["thr_bin"].astype(np.uint32), o.thr_bin,
                                      err_msg=f"rank {r}")
        for k in KEYS:
            np.testing.assert_array_equal(m[k].view(np.uint32),
                                          getattr(o, k).astype(m[k].dtype).view(np.uint32),
                                          err_msg=f"rank {r} {k}")
