"""bench.py's reference arm (the reference's own CPU path for the decode chain,
timed on the host) runs without a GPU and prints the contract's JSON line:
the same metric, unit, direction and workload as the GPU arm, plus the
reference-arm fields (impl, cpu_baseline, an e2e object with no host-device
copies)."""
import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "2", "--warmup", "1"],
                       capture_output=True, text=True, timeout=600, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    sys.path.insert(0, REPO)
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(REPO, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == "tok/s" and line["higher_is_better"] is True
    assert line["config"]["workload"] == bench.CONFIG["workload"]
    assert line["steps"] == 2 and line["warmup"] == 1 and line["value"] > 0
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"] and cb["value"] == line["value"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
