"""bench.py's reference arm runs on the CPU alone: it times the oracle (the C
restatement of the reference's CPU operators) on a bounded ResNet-50 sample and
prints one JSON line with the fields the driver reads.  Under torchrun only
rank 0 prints; the other ranks exit 0 without work."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_bench(env_extra):
    env = dict(os.environ, **env_extra)
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0"], capture_output=True, text=True, timeout=600, cwd=ROOT, env=env)
    assert r.returncode == 0, r.stderr[-3000:]
    return r.stdout.strip()


def test_reference_arm_json_line():
    out = run_bench({})
    d = json.loads(out.splitlines()[-1])
    assert d["impl"] == "reference"
    assert d["metric"].startswith("ResNet-50") and d["unit"] == "images/s" and d["value"] > 0
    assert d["higher_is_better"] is True and d["config"]["workload"] == "resnet50_v1.5_b256"
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    # the line describes what ran: the sample batch and the measured time of one pass over it
    n = d["config"]["global_batch"]
    assert n == d["config"]["per_step_batch"] == d["cpu_baseline"]["cores"]
    assert abs(d["ms_per_step"] - 1000.0 * n / d["value"]) <= 1e-6 * d["ms_per_step"]


def test_reference_arm_silent_on_other_ranks():
    assert run_bench({"RANK": "1", "WORLD_SIZE": "2"}) == ""
