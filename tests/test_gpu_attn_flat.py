"""The small-batch flash-decode of the engine (attn_flat.cu: key tiles of all
(sequence, KV head) pairs cut into one range per SM, per-warp online
softmax, ticketed merge of the partials) against a float64 softmax(QK^T)V,
through the engine's block-level attention entry (forge_b200_attention) on
a cache written with forge_b200_set_kv. Cases cover the 7B shape (MHA, head
dim 128, context 2048), the 1B shape (GQA 4:1, head dim 64), positions on
and beside tile boundaries, position 0, uneven batches, and the same call
on the per-(sequence, head, split) kernel (FORGE_ATTN=split)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CASES = [
    # B, H, Hkv, hd, lmax, positions
    (1, 32, 32, 128, 2304, [2047]),                        # 7B bs1, ctx 2048
    (1, 32, 8, 64, 1152, [1024]),                          # 1B bs1 (GQA 4:1)
    (3, 32, 8, 64, 1100, [1023, 5, 0]),
    (4, 8, 2, 128, 2048, [100, 31, 32, 1999]),             # GQA 4:1, hd 128, tile edges
    (8, 32, 32, 128, 600, [0, 1, 31, 32, 63, 64, 511, 599]),
    (2, 16, 2, 64, 700, [63, 64]),                         # GQA 8:1
    # several tiles per CTA with a 6-slot ring (4 or more query heads per KV
    # head): warps run ahead of the ring's refills
    (8, 32, 8, 64, 1500, [1400, 1450, 1499, 1300, 1472, 1024, 1408, 1399]),  # 1B bs8
    (8, 16, 2, 64, 4200, [4100, 4000, 4199, 3000, 4150, 4096, 2047, 4111]),  # GQA 8:1
    (4, 8, 2, 128, 4100, [4000, 4095, 3333, 4096]),       # GQA 4:1, hd 128
]


def _run(forge, oracle, cuda, B, H, Hkv, hd, lmax, pos, monkeypatch, impl):
    import torch
    monkeypatch.setenv("FORGE_ATTN", impl)
    d = H * hd
    fm = forge.ForgeModel(1, d, H, Hkv, hd, 256, 256, weight_kind=forge.FORGE_WEIGHT_BF16, max_batch=B,
                          max_ctx=lmax)
    fm.init_synthetic(1234, 0.02)
    rng = np.random.default_rng(B * 7919 + H * 31 + hd + lmax)
    Kf = np.zeros((B, Hkv, lmax, hd))
    Vf = np.zeros((B, Hkv, lmax, hd))
    for b in range(B):
        n = pos[b] + 1
        kb = oracle.f32_to_bf16(rng.standard_normal((Hkv, n, hd)).astype(np.float32) * 0.5)
        vb = oracle.f32_to_bf16(rng.standard_normal((Hkv, n, hd)).astype(np.float32))
        fm.set_kv(0, b, kb, vb)
        Kf[b, :, :n] = oracle.bf16_to_f32(kb)
        Vf[b, :, :n] = oracle.bf16_to_f32(vb)
    fm.set_positions(np.asarray(pos, np.int32))
    q = rng.standard_normal((B, H * hd)).astype(np.float32)
    qd = torch.from_numpy(q).to(cuda)
    ctx = torch.full((B, H * hd), float("nan"), device=cuda)
    G = H // Hkv
    ref = np.zeros((B, H * hd))
    for b in range(B):
        n = pos[b] + 1
        for h in range(H):
            s = Kf[b, h // G, :n] @ q[b, h * hd:(h + 1) * hd].astype(np.float64) / np.sqrt(hd)
            p = np.exp(s - s.max())
            ref[b, h * hd:(h + 1) * hd] = (p / p.sum()) @ Vf[b, h // G, :n]
    outs = []
    for rep in range(2):  # the second call starts from the counters the first left behind
        fm.attention(0, B, qd, ctx)
        fm.sync()
        outs.append(ctx.cpu().numpy())
    fm.close()
    return ref, outs


@pytest.mark.parametrize("B,H,Hkv,hd,lmax,pos", CASES)
def test_flat_attention_matches_f64(forge, oracle, cuda, monkeypatch, B, H, Hkv, hd, lmax, pos):
    ref, outs = _run(forge, oracle, cuda, B, H, Hkv, hd, lmax, pos, monkeypatch, "flat")
    tol = 2e-5 * max(1.0, np.abs(ref).max())
    for got in outs:
        assert np.isfinite(got).all()
        assert np.abs(got - ref).max() < tol, np.abs(got - ref).max()
    assert np.array_equal(outs[0], outs[1])  # same plan, same order: same bits


@pytest.mark.parametrize("B,H,Hkv,hd,lmax,pos", CASES[:3])
def test_flat_and_split_attention_agree(forge, oracle, cuda, monkeypatch, B, H, Hkv, hd, lmax, pos):
    ref, flat = _run(forge, oracle, cuda, B, H, Hkv, hd, lmax, pos, monkeypatch, "flat")
    _, split = _run(forge, oracle, cuda, B, H, Hkv, hd, lmax, pos, monkeypatch, "split")
    assert np.abs(flat[0] - split[0]).max() < 2e-5 * max(1.0, np.abs(ref).max())
