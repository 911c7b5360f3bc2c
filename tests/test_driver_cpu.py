"""The command-line driver (hexa-lang_b200/driver/forge_generate.c) without a
GPU: it builds against the public headers only, prints its usage, rejects bad
usage with status 2, and reports the library's error with status 1 when no
device is there (no compute runs)."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "hexa-lang_b200", "forge_generate")
MODEL = ["--layers", "1", "--dim", "256", "--heads", "4", "--kv-heads", "2", "--head-dim", "64", "--ffn", "512",
         "--vocab", "1000"]


@pytest.fixture(scope="module")
def driver(forge):
    if not os.path.exists(BIN):
        subprocess.run(["make", "-C", os.path.join(ROOT, "hexa-lang_b200", "csrc"), "../forge_generate"], check=True,
                       capture_output=True)
    return BIN


def test_usage(driver):
    r = subprocess.run([driver, "--help"], capture_output=True, text=True)
    assert r.returncode == 0 and r.stdout.startswith("usage: forge_generate")
    for bad in ([], MODEL, MODEL + ["--gen", "4"], MODEL + ["--synthetic", "1", "--gen", "4"],
                MODEL + ["--bogus", "--synthetic", "1", "--gen", "4", "5"]):
        r = subprocess.run([driver] + bad, capture_output=True, text=True)
        assert r.returncode == 2, (bad, r.stderr)


def test_library_error_without_gpu(driver):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    r = subprocess.run([driver] + MODEL + ["--synthetic", "1", "--gen", "4", "5", "6"], capture_output=True, text=True)
    assert r.returncode == 1 and "forge_generate: create:" in r.stderr and r.stdout == ""


def test_check_mode(driver, tmp_path):
    """--check validates a checkpoint against the model options without a GPU."""
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from test_safetensors_cpu import _llama, write_st
    cfg = (1, 256, 4, 2, 64, 512, 1000)
    good = str(tmp_path / "good.safetensors")
    write_st(good, _llama(cfg, False))
    r = subprocess.run([driver, "--check", "--weights", good] + MODEL, capture_output=True, text=True)
    assert r.returncode == 0 and r.stdout.startswith("ok: 1 file"), r.stderr
    bad = str(tmp_path / "bad.safetensors")
    write_st(bad, _llama(cfg, False, drop=("model.norm.weight",)))
    r = subprocess.run([driver, "--check", "--weights", bad] + MODEL, capture_output=True, text=True)
    assert r.returncode == 1 and "model.norm.weight missing" in r.stderr
    assert subprocess.run([driver, "--check"] + MODEL, capture_output=True).returncode == 2
