"""Whole-model decode parity on the B200 against the oracle: the KV-cache
decode step (logits, argmax, KV cache contents) and greedy generation, for
bf16 and int4-g128 weights, MHA and GQA, batch 1/3/8. The library is driven
only through its C ABI (forge_b200_*)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["fused", "graph"])
def path(request, monkeypatch):
    """Both decode paths: the persistent one-kernel step and the captured
    multi-kernel graph (FORGE_DECODE_PATH is read at handle creation)."""
    monkeypatch.setenv("FORGE_DECODE_PATH", request.param)
    return request.param

CONFIGS = {
    # the reference's CPU-runnable shape: 4L d256 4x64 MHA ffn688 V4096
    "tiny_bf16": dict(n_layer=4, d=256, n_head=4, n_kv=4, hd=64, ffn=688, vocab=4096, q4=False, tied=True),
    # 1B-style GQA (4 q heads per kv head), scaled down
    "gqa_bf16": dict(n_layer=2, d=512, n_head=8, n_kv=2, hd=64, ffn=1024, vocab=2048, q4=False, tied=False),
    # 7B-style MHA hd128 with int4 group-128 weights, scaled down
    "mha_q4": dict(n_layer=2, d=512, n_head=4, n_kv=4, hd=128, ffn=1280, vocab=2048, q4=True, tied=False),
}


def _models(oracle, forge, cfg, max_batch, max_ctx, act_mode=0, seed=1234):
    om = oracle.OracleModel(cfg["n_layer"], cfg["d"], cfg["n_head"], cfg["n_kv"], cfg["hd"], cfg["ffn"],
                            cfg["vocab"], q4=cfg["q4"], tied=cfg["tied"], seed=seed, std=0.02)
    fm = forge.ForgeModel(cfg["n_layer"], cfg["d"], cfg["n_head"], cfg["n_kv"], cfg["hd"], cfg["ffn"],
                          cfg["vocab"], weight_kind=forge.FORGE_WEIGHT_Q4_G128 if cfg["q4"] else forge.FORGE_WEIGHT_BF16,
                          tied_head=cfg["tied"], max_batch=max_batch, max_ctx=max_ctx, act_mode=act_mode)
    return om, fm


@pytest.mark.parametrize("name", list(CONFIGS))
def test_synthetic_init_matches_upload(forge, oracle, cuda, name, path):
    """Device-side synthetic init == uploading the oracle's weights (same logits)."""
    cfg = CONFIGS[name]
    om, fa = _models(oracle, forge, cfg, 1, 64)
    fa.init_synthetic(1234, 0.02)
    fb = forge.ForgeModel(cfg["n_layer"], cfg["d"], cfg["n_head"], cfg["n_kv"], cfg["hd"], cfg["ffn"], cfg["vocab"],
                          weight_kind=forge.FORGE_WEIGHT_Q4_G128 if cfg["q4"] else forge.FORGE_WEIGHT_BF16,
                          tied_head=cfg["tied"], max_batch=1, max_ctx=64)
    _upload(om, fb, cfg)
    for t in [3, 17, 1000 % cfg["vocab"]]:
        na, la = fa.step([t], want_logits=True)
        nb, lb = fb.step([t], want_logits=True)
        assert np.array_equal(la, lb) and np.array_equal(na, nb)
    fa.close(); fb.close()


def _upload(om, fm, cfg):
    for l in range(cfg["n_layer"]):
        w = [om.bf16[(l, n)] for n in ("wq", "wk", "wv", "wo", "wg", "wu", "wd")]
        fm.load_layer(l, *w, om.gains[(l, "g1")], om.gains[(l, "g2")])
    fm.load_embedding(om.bf16["emb"], om.gains["gF"], None if cfg["tied"] else om.bf16["head"])


@pytest.mark.parametrize("name", list(CONFIGS))
@pytest.mark.parametrize("batch", [1, 3, 8])
def test_decode_steps_match_oracle(forge, oracle, cuda, name, batch, path):
    cfg = CONFIGS[name]
    lmax = 48
    # bf16-weight models round GEMV inputs to bf16 above 4 sequences; int4
    # models always use hi/lo int8 activations (no oracle rounding)
    act_bf16 = batch > 4 and not cfg["q4"]
    om, fm = _models(oracle, forge, cfg, batch, lmax)
    _upload(om, fm, cfg)
    if path == "graph":
        assert not fm.uses_fused_step(batch)
    elif batch <= 4:
        assert fm.uses_fused_step(batch), "the fused step must fit at this size"
    kc, vc = om.new_cache(batch, lmax)
    rng = np.random.default_rng(5678 + batch)
    flags = oracle.OR_KV_BF16 | (oracle.OR_ACT_BF16 if act_bf16 else 0)
    # The device rounds K/V (and, in bf16-activation mode, GEMV inputs) to
    # bf16 from fp32 values that differ from the oracle's f64 values in the
    # last bits; values sitting on a rounding tie then round one bf16 ulp
    # apart, which moves logits by up to a few 1e-3 (logit std ~0.3-0.45).
    # Bounds: max |dlogit| 5e-3 exact-activation mode, 1e-2 bf16 mode — both
    # inside the 2e-2 (bf16) / 5e-2 (int4) gates — and a median below 2e-4
    # (exact activations) or 1e-3 (bf16 activations).
    tol = 5e-3 if not act_bf16 else 1e-2
    med_tol = (8e-4 if cfg["q4"] else 2e-4) if not act_bf16 else 1.5e-3
    fm.reset()
    worst = 0.0
    for p in range(20):
        tok = rng.integers(0, cfg["vocab"], batch)
        nxt, lg = fm.step(tok, want_logits=True)
        ref_lg, ref_am = om.decode_step(kc, vc, tok, [p] * batch, flags)
        err = np.abs(lg - ref_lg).max()
        worst = max(worst, err)
        assert err < tol, f"step {p}: max |dlogit| {err}"
        assert np.median(np.abs(lg - ref_lg)) < med_tol
        for b in range(batch):
            top2 = np.sort(ref_lg[b])[-2:]
            if top2[1] - top2[0] > 10 * tol:
                assert nxt[b] == ref_am[b], f"step {p} seq {b}: argmax {nxt[b]} vs {ref_am[b]}"
    # KV cache contents (bf16) of the last layer, first sequence
    c = cfg
    k, v = fm.get_kv(c["n_layer"] - 1, 0, c["n_kv"], lmax, c["hd"])
    kr = oracle.f32_to_bf16(kc[c["n_layer"] - 1, 0])
    vr = oracle.f32_to_bf16(vc[c["n_layer"] - 1, 0])
    kd = np.abs(oracle.bf16_to_f32(k[:, :20]) - oracle.bf16_to_f32(kr[:, :20])).max()
    vd = np.abs(oracle.bf16_to_f32(v[:, :20]) - oracle.bf16_to_f32(vr[:, :20])).max()
    assert kd < 2e-2 and vd < 2e-2, (kd, vd)
    fm.close()


@pytest.mark.parametrize("name", list(CONFIGS))
def test_greedy_32_tokens_match_oracle(forge, oracle, cuda, name, path):
    cfg = CONFIGS[name]
    om, fm = _models(oracle, forge, cfg, 1, 64)
    _upload(om, fm, cfg)
    prompt = np.random.default_rng(5678).integers(0, cfg["vocab"], 16).astype(np.int32)
    ref, margins = om.greedy(prompt, 32)
    got = fm.generate(prompt, 32)[0]
    print(f"{name}: min top-2 margin {margins.min():.4g}")
    assert np.array_equal(got, ref), f"tokens differ:\n{got}\n{ref}\nmargins {margins}"
    fm.close()


@pytest.mark.parametrize("name", ["tiny_bf16", "mha_q4"])
def test_fused_and_graph_paths_agree(forge, oracle, cuda, name, monkeypatch):
    """Same tokens, same logits (to fp32 reordering) from both step paths."""
    cfg = CONFIGS[name]
    outs = []
    for p in ("fused", "graph"):
        monkeypatch.setenv("FORGE_DECODE_PATH", p)
        om, fm = _models(oracle, forge, cfg, 2, 40)
        _upload(om, fm, cfg)
        fm.reset()
        lgs = []
        for t in ([1, 2], [3, 4], [5, 6], [7, 8]):
            _, lg = fm.step(t, want_logits=True)
            lgs.append(lg)
        outs.append(np.array(lgs))
        fm.close()
    assert np.abs(outs[0] - outs[1]).max() < 2e-3


def _handoff_runs(oracle, forge, batch, monkeypatch, settings):
    cfg = CONFIGS["mha_q4"]
    monkeypatch.setenv("FORGE_DECODE_PATH", "graph")
    runs = []
    for env in settings:
        for k, v in env.items():
            monkeypatch.setenv(k, v)
        _, fm = _models(oracle, forge, cfg, batch, 64)
        fm.init_synthetic(1234, 0.02)
        fm.fill_kv_synthetic(5, 20, 0.5)
        toks = np.arange(batch, dtype=np.int32) * 37 + 3
        lgs, tks = [], []
        for _ in range(6):
            toks, lg = fm.step(toks, want_logits=True)
            lgs.append(lg)
            tks.append(toks.copy())
        fm.close()
        runs.append((np.stack(lgs), np.stack(tks)))
    return runs


@pytest.mark.parametrize("batch", [1, 2, 4])
def test_context_handoff_bit_identical(forge, oracle, cuda, batch, monkeypatch):
    """int4, head dim 128, up to 4 sequences: the flash-decode merge hands
    each head's context to the O projection already staged (int8 hi/lo
    groups, scales, column sums), and a small kernel stages the SwiGLU output
    for the down projection; both GEMVs copy the block instead of staging.
    The bytes equal the staging's, so logits and tokens are bit-identical
    with the handoffs off (FORGE_PREQUANT=0, read at handle creation). The
    residual-stream handoff, which is not bit-identical, is off in both."""
    runs = _handoff_runs(oracle, forge, batch, monkeypatch,
                         [dict(FORGE_PREQUANT="1", FORGE_PREQUANT_NORM="0"), dict(FORGE_PREQUANT="0")])
    assert np.array_equal(runs[0][0], runs[1][0])


@pytest.mark.parametrize("batch", [1, 2, 4])
def test_residual_handoff_close_to_staging(forge, oracle, cuda, batch, monkeypatch):
    """The residual stream staged for the next RMSNorm GEMV (QKV after down,
    gate/up after O) as codes of gain * x plus per-group sums of squares, the
    GEMV folding its RMSNorm factor into the group scales: same tokens as
    the GEMVs staging x themselves, logits within 2e-3 of the logit scale
    (the reordered RMSNorm sum moves QKV outputs in the last bits, which can
    round a cached K/V value one bf16 step apart)."""
    on, off = _handoff_runs(oracle, forge, batch, monkeypatch,
                            [dict(FORGE_PREQUANT="1", FORGE_PREQUANT_NORM="1"), dict(FORGE_PREQUANT="0")])
    assert np.array_equal(on[1], off[1])
    scale = np.abs(off[0]).max()
    assert np.abs(on[0] - off[0]).max() <= 2e-3 * scale, np.abs(on[0] - off[0]).max() / scale
