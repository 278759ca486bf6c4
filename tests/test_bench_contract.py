"""bench.py's reference arm on the CPU: one JSON line with the keys the benchmark contract needs.

`bench.py --impl reference` times the CPU restatement of the reference's token loop on the host
cores (the reference itself needs WebGPU and a JS runtime). Its line is compared with the CUDA
arm's line, so it must carry the same metric, unit and config shape plus its own cpu_baseline
and e2e objects.
"""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    env = dict(os.environ, OMP_NUM_THREADS=os.environ.get("OMP_NUM_THREADS", "4"))
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "2",
                        "--warmup", "1"], capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    sys.path.insert(0, ROOT)
    import bench
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == bench.UNIT == "tok/s"
    assert d["steps"] == 2 and d["n_gpus"] == 1
    assert d["warmup"] == 3  # at least three warm-up steps, whatever is asked (the timing rules)
    assert d["higher_is_better"] is True and d["scaling"] in ("weak", "strong")
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert isinstance(d["config"], dict) and "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
