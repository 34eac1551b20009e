"""The benchmark's output contract, checked on the CPU through its reference arm (the CPU
algorithm of the path on the host threads): one JSON line on stdout with the fields a driver
reads, for a short run on two streams."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_json_line_with_the_contract_fields():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0", "--streams", "2"], cwd=ROOT, capture_output=True, text=True, timeout=600,
                         env={**os.environ, "WORLD_SIZE": "1", "RANK": "0", "LOCAL_RANK": "0"})
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1, out.stdout
    r = json.loads(lines[0])
    assert r["impl"] == "reference"
    assert r["unit"] == "active tubelets/s" and r["value"] > 0
    assert r["n_gpus"] == 1 and r["steps"] == 1 and r["warmup"] == 0
    assert r["higher_is_better"] is True and r["scaling"] == "weak" and r["vs_baseline"] is None
    assert r["data"] == "synthetic" and r["dtype"] == "f32"
    assert "workload" in r["config"] and r["ms_per_step"] > 0
    cb = r["cpu_baseline"]
    assert cb["value"] == r["value"] and cb["unit"] == r["unit"] and cb["cores"] >= 1
    assert cb["kind"] in ("port", "reference") and cb["sample"]
    e2e = r["e2e"]
    assert e2e["value"] == r["value"] and e2e["unit"] == r["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_cpu_rows_time_the_oracle_for_each_row():
    sys.path.insert(0, ROOT)
    import bench

    rows = bench.cpu_rows(2, budget_s=0.01)
    assert set(rows) == {"patch_diff_select", "feature_memory_assign_latest", "feature_memory_update_ema",
                         "rgba_patch_diff_scores", "gather_gemm_vitg_batch"}
    for r in rows.values():
        assert r["cpu_ms"] > 0 and r["cpu_sample"]
