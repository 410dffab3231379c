"""bench.py's reference arm runs on the host cores only (the oracle port, no GPU) and prints
the one JSON line of the benchmark contract: the same metric, unit and direction as the
GPU arm, "impl": "reference", a cpu_baseline describing the run and an e2e record with no
host-device traffic."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args):
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                         timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    return json.loads(lines[0])


def test_reference_arm_prints_the_contract_line():
    d = _run("--impl", "reference", "--workload", "0", "--steps", "2", "--warmup", "1")
    assert d["impl"] == "reference"
    assert d["metric"].startswith("certified input regions/sec")
    assert d["unit"] == "regions/s" and d["higher_is_better"] is True
    assert d["steps"] == 2 and d["warmup"] == 1 and d["n_gpus"] == 1
    assert d["value"] > 0 and d["ms_per_step"] > 0
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert d["config"]["workload"] and d["config"]["certifier"] == "deeppoly"


def test_reference_arm_other_certifier():
    d = _run("--impl", "reference", "--workload", "0", "--certifier", "ibp", "--steps", "1", "--warmup", "0")
    assert d["impl"] == "reference" and d["config"]["certifier"] == "ibp" and d["value"] > 0
