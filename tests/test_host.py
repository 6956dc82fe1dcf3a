"""Host-side mirror of the reference API: Config token parser (src/config.rs) and the
.rwood v1 model format (src/booster.rs:797-878). CPU only."""
import struct

import numpy as np
import pytest

import rustwood_b200 as rb
from rustwood_b200 import Booster, Config


def test_config_defaults_match_reference():
    c = Config()
    assert (c.n_trees, c.depth, c.learning_rate, c.n_bins, c.lambda_) == (500, 6, 0.1, 256, 1.0)
    assert c.subtract and c.replicas == 64 and c.bin_sample == 200_000
    assert c.objective == "logistic" and c.device == "gpu"


def test_config_tokens():
    c = Config.from_tokens(["--trees", "200", "--depth", "8", "--bins", "16", "--pack4", "1",
                            "--goss-top", "0.2", "--goss-other", "0.1", "--objective", "reg",
                            "--monotone", "1,0,-1", "--categorical", "7,8", "--device", "cuda",
                            "--smem-hist", "true", "--replicas", "8", "--unique-bins", "0"])
    assert (c.n_trees, c.depth, c.n_bins, c.pack4) == (200, 8, 16, True)
    assert c.objective == "l2" and c.monotone == [1, 0, -1] and c.categorical == [7, 8]
    assert c.smem_hist and c.replicas == 8 and not c.unique_bins and c.device == "gpu"


@pytest.mark.parametrize("toks,msg", [
    (["--bogus", "1"], "unknown flag"), (["--trees"], "missing value"),
    (["--bins", "300"], "n_bins"), (["--depth", "13"], "depth"),
    (["--objective", "poisson"], "objective"), (["--device", "tpu"], "device"),
])
def test_config_errors(toks, msg):
    with pytest.raises(ValueError, match=msg):
        Config.from_tokens(toks)


def _toy_booster(categorical=()):
    cfg = Config(n_trees=3, depth=2, categorical=list(categorical), cat_hash_buckets=5)
    b = Booster(cfg)
    b.n_features, b.base_score, b.gmean = 4, np.float32(-0.25), np.float32(0.4)
    b.feat = np.array([0, 1, 2, 3, 0, 1], np.uint32)
    b.thr = np.linspace(-1, 1, 6).astype(np.float32)
    b.leafval = np.arange(12, dtype=np.float32) / 7
    b.encoders = [{3: np.float32(0.5), -2: np.float32(0.1)}] if categorical else []
    return b


def test_rwood_layout_and_roundtrip(tmp_path):
    b = _toy_booster(categorical=[2])
    path = str(tmp_path / "m.rwood")
    b.save_model(path)
    raw = open(path, "rb").read()
    assert raw[:4] == b"RWD1"
    ver, nf, nt, depth, logistic = struct.unpack_from("<5I", raw, 4)
    assert (ver, nf, nt, depth, logistic) == (1, 4, 3, 2, 1)
    base, gmean, hb = struct.unpack_from("<ffQ", raw, 24)
    assert np.float32(base) == np.float32(-0.25) and hb == 5
    # header 40 + categorical list 8 + three length-prefixed arrays + encoder maps
    assert len(raw) == 40 + 8 + (4 + 24) + (4 + 24) + (4 + 48) + 4 + 4 + 2 * 12
    c = Booster.load_model(path)
    np.testing.assert_array_equal(c.feat, b.feat)
    np.testing.assert_array_equal(c.thr.view(np.uint32), b.thr.view(np.uint32))
    np.testing.assert_array_equal(c.leafval.view(np.uint32), b.leafval.view(np.uint32))
    assert c.cfg.categorical == [2] and c.encoders[0][3] == np.float32(0.5)
    assert c.cfg.n_trees == 3 and c.cfg.depth == 2 and c.n_features == 4


def test_rwood_rejects_other_files(tmp_path):
    p = tmp_path / "x.bin"
    p.write_bytes(b"NOPE" + bytes(40))
    with pytest.raises(ValueError):
        Booster.load_model(str(p))


def test_cpu_device_is_not_reimplemented():
    with pytest.raises(NotImplementedError):
        Booster(Config(device="cpu"))
