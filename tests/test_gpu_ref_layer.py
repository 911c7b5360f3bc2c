"""One decoder layer of the engine against the reference's own f64 decode
check `cpu_ref` (tool/decode_eager_baseline.cu:160-198) on its own inputs:
GPT-2-small shape (768 = 12 heads x 64, ffn 3072, RMSNorm eps 1e-5 with
non-unit gains, no RoPE) at cache lengths 1, 17 and 256. The reference
outputs are committed fixtures (tests/golden/cpu_ref_decode_layer.npz); the
inputs come from the oracle's restatement of the check's LCG.

The engine stores weights and the KV cache in bf16 where the check keeps
fp32, so against the reference the bar is the bf16 tolerance of 2e-2 max
abs; against the oracle given the same bf16-rounded weights and cache the
bar is 1e-4 of the output scale."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "cpu_ref_decode_layer.npz")


@pytest.mark.parametrize("L", [1, 17, 256])
def test_engine_layer_matches_reference_cpu_ref(forge, oracle, cuda, L):
    import torch
    F = forge
    D, NH, HD, FF = oracle.REF_D, oracle.REF_NH, oracle.REF_HD, oracle.REF_FF
    inp = oracle.ref_inputs(L)
    bf = {k: oracle.f32_to_bf16(inp[k]) for k in ("Wq", "Wk", "Wv", "Wo", "Wg", "Wu", "Wd", "Kc", "Vc")}
    m = F.ForgeModel(1, D, NH, NH, HD, FF, 64, tied_head=True, max_batch=1, max_ctx=L + 1, rms_eps=1e-5,
                     rope_theta=0.0)
    m.load_layer(0, bf["Wq"], bf["Wk"], bf["Wv"], bf["Wo"], bf["Wg"], bf["Wu"], bf["Wd"],
                 np.ascontiguousarray(inp["g1"], np.float32), np.ascontiguousarray(inp["g2"], np.float32))
    m.load_embedding(oracle.fill_normal_bf16(64 * D, 1, 0, 0.02), np.ones(D, np.float32))
    kc = np.ascontiguousarray(bf["Kc"].reshape(L, NH, HD).transpose(1, 0, 2))
    vc = np.ascontiguousarray(bf["Vc"].reshape(L, NH, HD).transpose(1, 0, 2))
    m.set_kv(0, 0, kc, vc)
    m.set_positions([L])
    x = torch.from_numpy(inp["x"].reshape(1, D).copy()).to(cuda)
    q = torch.empty((1, D), device=cuda)
    ctx = torch.empty((1, D), device=cuda)
    h = x.clone()
    torch.cuda.synchronize()
    m.qkv_rope(0, 1, x, q)
    m.attention(0, 1, q, ctx)
    m.o_proj(0, 1, ctx, h)
    m.mlp(0, 1, h, h)
    m.sync()
    got = h.cpu().numpy()[0].astype(np.float64)
    gold = np.load(GOLD)[f"L{L}"]
    assert np.abs(got - gold).max() <= 2e-2, np.abs(got - gold).max()
    # the same bf16 weights and cache through the oracle (appended row rounded to bf16)
    rin = dict(inp)
    for k in bf:
        rin[k] = oracle.bf16_to_f32(bf[k])
    ref = oracle.ref_layer_via_oracle(rin, L, flags=oracle.OR_NO_ROPE | oracle.OR_KV_BF16)
    assert np.abs(got - ref).max() <= 1e-4 * np.abs(ref).max(), np.abs(got - ref).max()
    m.close()
