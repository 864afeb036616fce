"""bench.py's reference arm on the host cores: the line the driver pairs with
the GPU arm's, from the reference engine's own C attention (oracle/_ref), and
the rank rule under torchrun (rank 0 alone prints; other ranks exit 0 without
work). The GPU arm itself needs a B200 and is exercised by the bench runs."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench(*args, rank="0", timeout=300):
    env = dict(os.environ, RANK=rank)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=timeout)


def test_reference_arm_other_ranks_do_no_work():
    r = _bench("--impl", "reference", "--gpus", "2", rank="1", timeout=60)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == ""


def test_reference_arm_prints_one_paired_line():
    r = _bench("--impl", "reference", "--steps", "1", "--warmup", "0")
    assert r.returncode == 0, r.stderr
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["metric"].startswith("decode tok/s (config 2") and d["config"]["workload"] == "config2-decode"
    assert d["value"] > 0 and d["n_gpus"] == 1
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["value"] == d["value"] and cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["prefill"]["value"] > 0 and d["prefill"]["metric"].startswith("prefill tok/s (config 3")
