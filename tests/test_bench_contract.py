"""The bench.py JSON contract on CPU: the reference arm (`--impl reference`,
the oracle port timed on the host cores) prints one JSON line with the keys
the harness reads, under the same metric and unit as the GPU arm."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--config", "1",
                        "--steps", "1", "--warmup", "3"], capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["steps"] == 1 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert d["value"] > 0 and d["unit"] == "GB/s" and d["metric"] == "decode attn HBM GB/s"
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_cfg5_tokens_must_be_a_positive_multiple_of_64():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--config", "5", "--cfg5-tokens", "100"],
                       capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 2 and "--cfg5-tokens must be a positive multiple of 64" in r.stderr
