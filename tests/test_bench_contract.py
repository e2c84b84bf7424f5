"""bench.py's JSON line contract, checked on the arm that runs without a GPU: the reference arm
(`--impl reference`) times the oracle port of the reference CPU path on the host cores and prints
one line with the same metric / unit / config keys as the device arm, plus impl, cpu_baseline and
e2e."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _reference_line(*args):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", *args],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-3000:]
    lines = [l for l in r.stdout.splitlines() if l.strip().startswith("{")]
    assert len(lines) == 1, r.stdout
    return json.loads(lines[0])


def test_reference_arm_single_linear_line():
    line = _reference_line("--workload", "single", "--steps", "1", "--warmup", "0")
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["unit"] == "GB/s" and line["value"] > 0
    assert line["config"]["workload"] == "single Linear" and (line["config"]["M"], line["config"]["N"],
                                                              line["config"]["K"]) == (16, 1536, 576)
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0


def test_reference_arm_linear_sweep_line_names_the_device_metric():
    line = _reference_line("--workload", "linear", "--shapes", "k,v", "--steps", "1", "--warmup", "0")
    assert line["metric"].startswith("decode GEMV GB/s at M=1") and line["unit"] == "GB/s"
    assert line["config"]["shapes"] == ["k", "v"] and line["value"] > 0
