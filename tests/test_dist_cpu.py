"""The multi-GPU exchange protocol on CPU ranks (gloo, world_size 2 and 3).

Each rank trains on a contiguous row shard with tests/shard_protocol.py, which restates
the collectives librwgpu issues over NCCL (all-reduce of the fixed-point scale maxima,
of the GOSS radix-select digit counts, of every level's int64 histogram and of the leaf
sums). The models of all ranks must be bit-identical to each other and to the
single-process exact oracle on the concatenated rows, including ragged shards, stride
subsampling, GOSS and both objectives. A rank that leaves between steps makes the
survivor's next exchange fail with an error within the group timeout.
"""
import multiprocessing as mp
import os
import socket
import sys
import tempfile

import numpy as np
import pytest

import oracle

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import shard_protocol as sp  # noqa: E402

KEYS = ("feat", "thr_bin", "thr", "leafval", "fi_gain", "fi_count")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data(n, nf, nb, seed, objective):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n, nf)).astype(np.float32)
    x[:, 1] = np.round(x[:, 1] * 2)  # ties in one feature
    if objective == "logistic":
        y = (rng.random(n) < 1 / (1 + np.exp(-(x[:, 0] + 0.5 * x[:, 2])))).astype(np.float32)
    else:
        y = (np.sin(x[:, 0]) + 0.3 * x[:, 2] + 0.1 * rng.standard_normal(n)).astype(np.float32)
    cuts = oracle.compute_boundaries(x, nb)
    return x, y, cuts


def _rank_main(rank, world, port, bounds, case, out_dir):
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        x, y, cuts = _data(case["n"], case["nf"], case["nb"], case["seed"], case["objective"])
        base = oracle.base_score(y, case["objective"])
        lo, hi = bounds[rank], bounds[rank + 1]
        bins = oracle.bin_rowmajor(x[lo:hi], cuts, case["nb"])
        m = sp.train_shard(bins, y[lo:hi], cuts, base, row_offset=lo, n_global=case["n"],
                           n_trees=case["trees"], depth=case["depth"], n_bins=case["nb"],
                           learning_rate=0.3, objective=case["objective"],
                           subsample=case.get("subsample", 1.0),
                           goss_top=case.get("goss_top", 0.0),
                           goss_other=case.get("goss_other", 0.1),
                           subtract=case.get("subtract", True), ex=sp.Exchange(dist),
                           expf=oracle.rw_expf)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **m)
    finally:
        dist.destroy_process_group()


CASES = [
    dict(id="l2_ragged_2ranks", n=3001, nf=4, nb=32, seed=1, objective="l2", trees=4, depth=4,
         bounds=[0, 1187, 3001]),
    dict(id="logistic_3ranks_subsample", n=2400, nf=3, nb=16, seed=2, objective="logistic",
         trees=3, depth=3, bounds=[0, 700, 1500, 2400], subsample=0.5),
    dict(id="goss_2ranks", n=4000, nf=4, nb=64, seed=3, objective="l2", trees=4, depth=5,
         bounds=[0, 2000, 4000], goss_top=0.2, goss_other=0.1),
    dict(id="no_subtract_2ranks", n=1500, nf=3, nb=8, seed=4, objective="l2", trees=2, depth=3,
         bounds=[0, 3, 1500], subtract=False),
]


@pytest.mark.parametrize("case", CASES, ids=[c["id"] for c in CASES])
def test_sharded_protocol_matches_single_process_oracle(case):
    world = len(case["bounds"]) - 1
    ctx = mp.get_context("spawn")
    with tempfile.TemporaryDirectory() as out_dir:
        port = _free_port()
        procs = [ctx.Process(target=_rank_main,
                             args=(r, world, port, case["bounds"], case, out_dir))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=240)
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        models = [dict(np.load(os.path.join(out_dir, f"rank{r}.npz"))) for r in range(world)]

    x, y, cuts = _data(case["n"], case["nf"], case["nb"], case["seed"], case["objective"])
    base = oracle.base_score(y, case["objective"])
    want = oracle.train(x, y, cuts, base, n_trees=case["trees"], depth=case["depth"],
                        n_bins=case["nb"], learning_rate=0.3, objective=case["objective"],
                        subsample=case.get("subsample", 1.0), goss_top=case.get("goss_top", 0.0),
                        goss_other=case.get("goss_other", 0.1),
                        subtract=case.get("subtract", True), exact=True, n_threads=2)
    for r, m in enumerate(models):
        for k in KEYS:
            np.testing.assert_array_equal(
                m[k].view(np.uint32), getattr(want, k).astype(m[k].dtype).view(np.uint32),
                err_msg=f"rank {r} {k}")


def test_radix_select_matches_sorted_order():
    """The distributed k-th largest |g| (one process, no exchange) equals sorting."""
    rng = np.random.default_rng(5)
    g = rng.standard_normal(5000).astype(np.float32)
    g[::7] = g[1::7][: len(g[::7])]  # duplicates
    g[:3] = 0.0
    srt = np.sort(np.abs(g))[::-1]
    for k in (0, 1, 17, 999, 4096, 4999):
        bits = sp.kth_largest_abs_bits(g, k, sp.Exchange())
        assert np.array([bits], np.uint32).view(np.float32)[0] == srt[k]


def _failing_rank_main(rank, world, port, out_dir):
    """Rank 1 leaves right after joining (between steps, nothing in flight); rank 0 runs
    the protocol and must get an error from its next collective instead of waiting."""
    import datetime
    import time

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)
    case = CASES[0]
    x, y, cuts = _data(case["n"], case["nf"], case["nb"], case["seed"], case["objective"])
    base = oracle.base_score(y, case["objective"])
    bins = oracle.bin_rowmajor(x[:1000], cuts, case["nb"])
    t0 = time.monotonic()
    try:
        sp.train_shard(bins, y[:1000], cuts, base, row_offset=0, n_global=case["n"],
                       n_trees=2, depth=3, n_bins=case["nb"], ex=sp.Exchange(dist),
                       expf=oracle.rw_expf)
        status = "completed"
    except Exception as e:  # the collective reports the lost rank
        status = "error: " + type(e).__name__
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(f"{status}\n{time.monotonic() - t0:.3f}\n")
    os._exit(0)


def test_lost_rank_is_reported_not_waited_for():
    """A rank that exits between steps: the surviving rank's next exchange fails within
    the process group's timeout and the failure reaches the caller as an exception."""
    world = 2
    ctx = mp.get_context("spawn")
    with tempfile.TemporaryDirectory() as out_dir:
        port = _free_port()
        procs = [ctx.Process(target=_failing_rank_main, args=(r, world, port, out_dir))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join()
        assert procs[1].exitcode == 3
        assert procs[0].exitcode == 0, procs[0].exitcode
        status, seconds = open(os.path.join(out_dir, "rank0.txt")).read().splitlines()[:2]
    assert status.startswith("error"), status
    assert float(seconds) < 60.0
