"""The CPU side of bench.py: the reference arm's JSON line and the scoring baseline.

The reference arm times the oracle's restatement of src/cpu.rs on host cores and must
print one JSON line with the keys the driver reads; the scoring baseline restates
predict_cpu on a C5 sample. Both run here at tiny sizes (no GPU needed).
"""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_contract_line():
    out = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--rows",
         "20000", "--trees", "4", "--steps", "2", "--warmup", "1"],
        capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
              "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference"
    assert d["higher_is_better"] is False
    assert d["value"] > 0 and d["cpu_baseline"]["value"] == d["value"]
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    # every step is one whole fit: the timed steps are the printed ones, nothing scaled
    assert len(d["step_seconds"]) == 2
    assert abs(sum(d["step_seconds"]) / 2 - d["value"]) < 1e-12


def test_reference_arm_config_equals_gpu_arm_config():
    sys.path.insert(0, ROOT)
    import bench

    class A:
        rows, trees = 1_000_000, 200
    assert bench.bench_config(A) == bench.bench_config(A)
    cfg = bench.bench_config(A)
    assert cfg["rows"] == 1_000_000 and cfg["trees"] == 200 and cfg["depth"] == 6


def test_reference_arm_does_not_load_the_gpu_library():
    """The reference arm times the CPU restatement alone: its process maps liborc.so and
    never librwgpu.so (the seeded generator is loaded by file path, not via the package)."""
    code = (
        "import sys; sys.argv=['bench.py','--impl','reference','--rows','5000','--trees','2',"
        "'--steps','1','--warmup','0']; sys.path.insert(0, %r); import bench; bench.main(); "
        "maps=open('/proc/self/maps').read(); "
        "assert 'liborc.so' in maps, 'oracle not loaded'; "
        "assert 'librwgpu' not in maps, 'GPU library mapped'; "
        "assert 'rustwood_b200' not in sys.modules" % ROOT)
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr


def test_predict_cpu_baseline_small_sample():
    sys.path.insert(0, ROOT)
    import bench
    r = bench.predict_cpu_baseline(rows=2000)
    assert r["rows_per_s"] > 0
    assert r["cores"] == 1 and r["kind"] == "port"
    assert r["row_split"]["rows_per_s"] > 0 and r["row_split"]["threads"] >= 1


def test_c4_cpu_baseline_small_sample():
    sys.path.insert(0, ROOT)
    import bench
    r = bench.c4_cpu_baseline(trees=2, sample_rows=20_000, full_rows=200_000)
    assert r["seconds_sample"] > 0 and r["kind"] == "port" and r["cores"] >= 1
    assert abs(r["seconds_full_rows_extrapolated"] - 10 * r["seconds_sample"]) < 1e-9
