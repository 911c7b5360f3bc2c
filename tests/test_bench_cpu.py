"""The reference arm of bench.py (the oracle port of flame's CPU decode on
the host cores; no GPU) prints the one JSON line its contract asks for: the
repo arm's metric, unit and workload, a cpu_baseline describing the run, and
an e2e block with no host-device bytes."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"].startswith("decode tok/s (7B-shape int4 g128, bs1, ctx 2048)")
    assert d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 0
    cfg = d["config"]
    assert cfg["workload"] == "7b_int4_decode" and cfg["batch"] == 1 and cfg["ctx"] == 2048
    assert (cfg["n_layer"], cfg["d_model"], cfg["heads"], cfg["head_dim"], cfg["ffn"], cfg["vocab"]) == \
        (32, 4096, 32, 128, 11008, 32000)
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
