"""The `--serve` worker (src/main.rs:344-416) and loaded-model scoring.

CPU: the dataset files round-trip, and a bad request is answered with an ERROR line
without touching a GPU. GPU: one worker process serves a fit (saving a .rwood model) and
then a load + predict of that model on the same resident context; the dumped margins are
bit-identical to predict_cpu on the loaded model and to the oracle_exact fit's. A loaded
model also scores pre-binned rows once its cut table gives back the bin thresholds.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _data(tmp_path, n=4000, nt=1000):
    from rustwood_b200 import serve, synth
    x, y, xt, yt = synth.c1(n, nt, seed=11)
    d = str(tmp_path / "data")
    serve.write_dataset(d, x, y, xt, yt)
    return d, x, y, xt, yt


def test_dataset_files_round_trip(tmp_path):
    from rustwood_b200 import serve
    d, x, y, xt, yt = _data(tmp_path)
    ds = serve.load_dataset(d)
    assert (ds["n_train"], ds["n_test"], ds["n_features"]) == (4000, 1000, 28)
    for k, a in (("x_train", x), ("y_train", y), ("x_test", xt), ("y_test", yt)):
        np.testing.assert_array_equal(ds[k], a)


def test_bad_requests_answer_errors_without_a_gpu(tmp_path):
    from rustwood_b200 import serve
    d, *_ = _data(tmp_path)
    w = serve.Worker([0])
    assert w.handle(["--data", d, "--no-such-flag", "1"]).startswith("ERROR args")
    assert w.handle(["--data", str(tmp_path / "missing")]).startswith("ERROR data")
    assert w.handle(["--data", d, "--trees"]).startswith("ERROR args")
    assert w.ctx is None  # nothing above needed the GPU


@pytest.mark.gpu
def test_worker_fits_then_scores_the_saved_model(tmp_path):
    import oracle
    import rustwood_b200 as rb
    d, x, y, xt, yt = _data(tmp_path)
    model = str(tmp_path / "m.rwood")
    dump = str(tmp_path / "pred.bin")
    fit = ["--data", d, "--trees", "12", "--depth", "5", "--bins", "64", "--lr", "0.2",
           "--save-model", model]
    pred = ["--data", d, "--load-model", model, "--dump-pred", dump]
    bad = ["--data", d, "--load-model", str(tmp_path / "nope.rwood")]
    lines = "\t".join(fit) + "\n" + "\t".join(pred) + "\n" + "\t".join(bad) + "\nQUIT\n"
    out = subprocess.run([sys.executable, "-m", "rustwood_b200.serve", "--gpu", "0"],
                         input=lines, capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr
    replies = [r.strip() for r in out.stdout.split("__END__") if r.strip()]
    assert len(replies) == 3, out.stdout
    assert replies[0].startswith("OK train_s="), replies[0]
    assert replies[1] == "OK n=1000", replies[1]
    assert replies[2].startswith("ERROR load"), replies[2]
    got = np.fromfile(dump, dtype="<f4")
    b = rb.Booster.load_model(model)
    want = oracle.predict(xt, b.feat, b.thr, b.leafval, float(b.base_score), 12, 5)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    # the saved model is the exact oracle's fit of the same data
    cuts = rb.compute_boundaries(x, 64)
    base = rb.base_score(y, "logistic")
    o = oracle.train(x, y, cuts, base, n_trees=12, depth=5, n_bins=64, learning_rate=0.2,
                     exact=True, n_threads=4)
    np.testing.assert_array_equal(b.feat, o.feat)
    np.testing.assert_array_equal(b.leafval.view(np.uint32), o.leafval.view(np.uint32))
    # a loaded model (raw thresholds only) scores binned rows once its cut table is known
    b.set_cut_table(cuts, 64)
    np.testing.assert_array_equal(b.thr_bin.astype(np.uint32), o.thr_bin)
    got_u8 = b.predict_bins(oracle.bin_rowmajor(xt, cuts, 64).T.copy())
    np.testing.assert_array_equal(got_u8.view(np.uint32), want.view(np.uint32))
    b.ctx.close()


def test_launcher_speaks_the_wrappers_protocol_without_a_gpu(tmp_path):
    """rustwood_b200/rustwood as the reference's Python wrapper runs it (RUSTWOOD_BIN):
    `--serve 1` answers every stdin line with a reply and __END__ and stops at QUIT; a
    one-shot command line answers once, exit status 1 for a failed request and 2 for a bad
    command line. Requests that fail before the GPU is needed run without one."""
    exe = os.path.join(ROOT, "rustwood_b200", "rustwood")
    env = dict(os.environ, RUSTWOOD_PYTHON=sys.executable)
    missing = str(tmp_path / "missing")
    lines = "--data\t" + missing + "\n--trees\nQUIT\n"
    out = subprocess.run([exe, "--serve", "1"], input=lines, capture_output=True, text=True,
                         timeout=300, env=env)
    assert out.returncode == 0, out.stderr
    replies = [r.strip() for r in out.stdout.split("__END__") if r.strip()]
    assert len(replies) == 2, out.stdout
    assert replies[0].startswith("ERROR data") and replies[1].startswith("ERROR args")
    one = subprocess.run([exe, "--data", missing, "--trees", "5", "--device", "gpu"],
                         capture_output=True, text=True, timeout=300, env=env)
    assert one.returncode == 1 and one.stdout.startswith("ERROR data"), one.stdout + one.stderr
    bad = subprocess.run([exe, "--no-such-flag", "1"], capture_output=True, text=True,
                         timeout=300, env=env)
    assert bad.returncode == 2 and bad.stdout.startswith("ERROR args"), bad.stdout


def test_thr_bins_reject_a_foreign_cut_table():
    import rustwood_b200 as rb
    from rustwood_b200 import _native as N
    b = rb.Booster(rb.Config(n_trees=1, depth=2, n_bins=4))
    b.n_features = 2
    b.feat = np.array([0, 1], np.uint32)
    b.thr = np.array([0.5, 2.0], np.float32)
    b.leafval = np.zeros(4, np.float32)
    cuts = np.array([0.1, 0.5, 0.9, 1.0, 2.0, 3.0], np.float32)  # [2][3]
    b.set_cut_table(cuts, 4)
    np.testing.assert_array_equal(b.thr_bin, [1, 1])
    with pytest.raises(N.RwError):
        b.set_cut_table(np.array([0.1, 0.6, 0.9, 1.0, 2.0, 3.0], np.float32), 4)
