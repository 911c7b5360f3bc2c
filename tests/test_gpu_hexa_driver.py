"""The hexa-side decode driver (hexa-lang_b200/hexa/forge_greedy.hexa) on the
B200: its forge_b200_generate tokens (prompt prefilled in one pass) and its
stepwise tokens (flame's loop, one forge_b200_decode_step per token, as in
self/ml/gpu_generate.hexa) agree, and both equal ForgeModel.generate on the
same synthetic int4 model (2 layers, d 256, 4 / 2 heads of 64, SwiGLU 512,
vocabulary 1000, seed 1234, std 0.02)."""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "hexa-lang_b200", "hexa", "forge_greedy")
PROMPT = [3, 17, 5, 99, 42]


def test_hexa_driver_matches_python_generate(forge, cuda):
    if not os.path.exists(BIN):
        subprocess.run(["make", "-C", os.path.join(ROOT, "hexa-lang_b200", "csrc"), "../hexa/forge_greedy"],
                       check=True, capture_output=True)
    r = subprocess.run([BIN], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = r.stdout.strip().splitlines()
    assert lines[-1] == "match", r.stdout
    gen = [int(t) for t in lines[0].split()[1:]]
    step = [int(t) for t in lines[1].split()[1:]]
    assert lines[0].startswith("generate") and lines[1].startswith("stepwise")
    m = forge.ForgeModel(2, 256, 4, 2, 64, 512, 1000, weight_kind=forge.FORGE_WEIGHT_Q4_G128, max_batch=1,
                         max_ctx=32)
    m.init_synthetic(1234, 0.02)
    want = m.generate([PROMPT], 16)[0].tolist()
    m.close()
    assert gen == want and step == want
