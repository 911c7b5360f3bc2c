"""Decode parity at the full model shapes of the benchmark, through the C ABI,
against the oracle (a float64 restatement of flame's decoder with a KV
cache, given the same weights):

  7B-shape int4 g128: 32 layers, d 4096, 32 x 128 MHA, SwiGLU 11008,
                      vocab 32000, int4 group-128 weights with bf16 scales,
                      bf16 embeddings and untied head
  1B-shape bf16 GQA:  16 layers, d 2048, 32 query / 8 KV heads x 64,
                      SwiGLU 8192, vocab 32000, bf16 weights

Weights are the seeded synthetic N(0, 0.02) tensors (seed 1234), generated
on the device by forge_b200_init_synthetic and bit for bit on the host by
the oracle (the same counter-based generator; the oracle quantises each int4
matrix as it is generated). A 16-token prompt (uniform ids, seed 5678) is
followed by 32 greedy steps:

  * step by step, the engine is fed the oracle's token sequence and every
    step's logits are compared with the oracle's (max |dlogit| within 5e-2
    for int4, 2e-2 for bf16), and the engine's argmax
    must equal the oracle's at each of the 32 generated positions; the
    oracle's top-2 margin is printed next to the logit error;
  * free-running, forge_b200_generate from the same prompt must return the
    oracle's 32 tokens exactly.
"""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SHAPES = {
    "7b_int4": dict(n_layer=32, d=4096, n_head=32, n_kv=32, hd=128, ffn=11008, vocab=32000, q4=True, tol=5e-2),
    "1b_bf16": dict(n_layer=16, d=2048, n_head=32, n_kv=8, hd=64, ffn=8192, vocab=32000, q4=False, tol=2e-2),
}
N_PROMPT, N_GEN = 16, 32


@pytest.mark.parametrize("name", list(SHAPES))
def test_full_shape_greedy_matches_oracle(forge, oracle, cuda, name):
    c = SHAPES[name]
    t0 = time.time()
    om = oracle.OracleModel(c["n_layer"], c["d"], c["n_head"], c["n_kv"], c["hd"], c["ffn"], c["vocab"],
                            q4=c["q4"], tied=False, seed=1234, std=0.02, keep_bf16=not c["q4"])
    t_or = time.time() - t0
    lmax = N_PROMPT + N_GEN
    fm = forge.ForgeModel(c["n_layer"], c["d"], c["n_head"], c["n_kv"], c["hd"], c["ffn"], c["vocab"],
                          weight_kind=forge.FORGE_WEIGHT_Q4_G128 if c["q4"] else forge.FORGE_WEIGHT_BF16,
                          tied_head=False, max_batch=1, max_ctx=lmax)
    fm.init_synthetic(1234, 0.02)
    prompt = np.random.default_rng(5678).integers(0, c["vocab"], N_PROMPT).astype(np.int32)

    kc, vc = om.new_cache(1, lmax)
    seq = [int(t) for t in prompt]
    fm.reset()
    worst, min_margin, rows = 0.0, np.inf, []
    for p in range(N_PROMPT + N_GEN - 1):
        nxt, lg = fm.step([seq[p]], want_logits=True)
        ref_lg, ref_am = om.decode_step(kc, vc, [seq[p]], [p], oracle.OR_KV_BF16)
        err = float(np.abs(lg[0] - ref_lg[0]).max())
        worst = max(worst, err)
        assert err < c["tol"], f"position {p}: max |dlogit| {err}"
        if p >= N_PROMPT - 1:
            top2 = np.sort(ref_lg[0])[-2:]
            margin = float(top2[1] - top2[0])
            min_margin = min(min_margin, margin)
            rows.append((p, int(ref_am[0]), int(nxt[0]), margin, err))
            assert nxt[0] == ref_am[0], f"position {p}: argmax {nxt[0]} vs oracle {ref_am[0]} (margin {margin}, err {err})"
            seq.append(int(ref_am[0]))
    print(f"\n{name}: oracle build {t_or:.0f} s; max |dlogit| {worst:.3g}; min top-2 margin {min_margin:.3g}")
    for p, a, b, m, e in rows:
        print(f"  pos {p:2d} token {a:5d} engine {b:5d} margin {m:.4f} |dlogit| {e:.2e}")

    got = fm.generate(prompt, N_GEN)[0]
    assert [int(t) for t in got] == seq[N_PROMPT:], f"free-running tokens differ:\n{list(got)}\n{seq[N_PROMPT:]}"
    fm.close()
