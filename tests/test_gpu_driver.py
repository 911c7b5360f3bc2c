"""The command-line driver on the B200: greedy output equals
ForgeModel.generate on the same synthetic weights, sampled output equals
the prompt fed through decode_step followed by decode_step_sampled."""
import os
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "hexa-lang_b200", "forge_generate")
CFG = (2, 256, 4, 2, 64, 512, 1000)
MODEL = ["--layers", "2", "--dim", "256", "--heads", "4", "--kv-heads", "2", "--head-dim", "64", "--ffn", "512",
         "--vocab", "1000", "--ctx", "32"]
PROMPT = [5, 17, 99]


def _run(args):
    r = subprocess.run([BIN] + MODEL + args + [str(t) for t in PROMPT], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    return [int(x) for x in r.stdout.split()]


def test_driver_greedy_and_sampled(forge, cuda):
    if not os.path.exists(BIN):
        pytest.skip("driver not built")
    m = forge.ForgeModel(*CFG, max_batch=1, max_ctx=32)
    m.init_synthetic(7, 0.02)
    want = m.generate([PROMPT], 8)[0].tolist()
    assert _run(["--synthetic", "7", "--gen", "8"]) == want
    m.reset()
    for t in PROMPT[:-1]:
        m.step([t])
    state = np.array([1234], np.int64)
    cur, want_s = PROMPT[-1], []
    for _ in range(8):
        cur = int(m.step_sampled([cur], state, 0.8, 20, 0.9)[0])
        want_s.append(cur)
    m.close()
    got = _run(["--synthetic", "7", "--gen", "8", "--temperature", "0.8", "--top-k", "20", "--top-p", "0.9",
                "--seed", "1234"])
    assert got == want_s
