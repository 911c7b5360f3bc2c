"""Llama-layout safetensors checkpoints through forge_b200_load_safetensors on
the B200: a model loaded from the files (two shards, a mix of BF16, F32 and
F16 tensors) must decode with the same logits, bit for bit, as the same
weights uploaded through forge_b200_load_layer / _load_embedding; a missing
or mis-shaped tensor is rejected with its name."""
import json
import struct

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CONFIGS = {
    "gqa_bf16_untied": dict(n_layer=2, d=256, n_head=4, n_kv=2, hd=64, ffn=512, vocab=1000, q4=False, tied=False),
    "mha_q4_tied": dict(n_layer=2, d=256, n_head=2, n_kv=2, hd=128, ffn=768, vocab=512, q4=True, tied=True),
}


def _write(path, tensors):
    hdr, blobs, off = {}, [], 0
    for name, dt, shape, data in tensors:
        hdr[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + len(data)]}
        blobs.append(data)
        off += len(data)
    h = json.dumps(hdr).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"".join(blobs))


def _checkpoint(om, cfg, tmp_path, drop=None, reshape=None):
    """The oracle model's weights under Llama names; 2-D weights alternate
    BF16 / F32 (bf16 values widened exactly); the second norm of each layer
    is stored as F16 when its gains are F16 values, the others as F32."""
    names = {"wq": "self_attn.q_proj", "wk": "self_attn.k_proj", "wv": "self_attn.v_proj", "wo": "self_attn.o_proj",
             "wg": "mlp.gate_proj", "wu": "mlp.up_proj", "wd": "mlp.down_proj"}
    d, q, kv, f = cfg["d"], cfg["n_head"] * cfg["hd"], cfg["n_kv"] * cfg["hd"], cfg["ffn"]
    shapes = {"wq": (q, d), "wk": (kv, d), "wv": (kv, d), "wo": (d, q), "wg": (f, d), "wu": (f, d), "wd": (d, f)}
    ts, k = [], 0

    def mat(name, bits, shape):
        nonlocal k
        k += 1
        if reshape == name:
            shape = (shape[0] + 16, shape[1])
            bits = np.zeros(shape[0] * shape[1], np.uint16)
        if k % 2:
            ts.append((name, "BF16", shape, np.ascontiguousarray(bits, np.uint16).tobytes()))
        else:
            f32 = (np.asarray(bits, np.uint32) << 16).view(np.float32)
            ts.append((name, "F32", shape, f32.tobytes()))

    def gain(name, g):
        g = np.asarray(g, np.float32)
        if np.all(g == np.float16(g).astype(np.float32)) and "post_attention" in name:
            ts.append((name, "F16", g.shape, g.astype(np.float16).tobytes()))
        else:
            ts.append((name, "F32", g.shape, g.tobytes()))

    for l in range(cfg["n_layer"]):
        pre = f"model.layers.{l}."
        for w, hf in names.items():
            mat(pre + hf + ".weight", om.bf16[(l, w)], shapes[w])
        gain(pre + "input_layernorm.weight", om.gains[(l, "g1")])
        gain(pre + "post_attention_layernorm.weight", om.gains[(l, "g2")])
    mat("model.embed_tokens.weight", om.bf16["emb"], (cfg["vocab"], d))
    gain("model.norm.weight", om.gains["gF"])
    if not cfg["tied"]:
        mat("lm_head.weight", om.bf16["head"], (cfg["vocab"], d))
    ts = [t for t in ts if t[0] != drop]
    half = len(ts) // 2
    paths = [str(tmp_path / "model-00001-of-00002.safetensors"), str(tmp_path / "model-00002-of-00002.safetensors")]
    _write(paths[0], ts[:half])
    _write(paths[1], ts[half:])
    return paths


def _pair(oracle, forge, cfg):
    om = oracle.OracleModel(cfg["n_layer"], cfg["d"], cfg["n_head"], cfg["n_kv"], cfg["hd"], cfg["ffn"],
                            cfg["vocab"], q4=cfg["q4"], tied=cfg["tied"], seed=99, std=0.03)
    mk = lambda: forge.ForgeModel(cfg["n_layer"], cfg["d"], cfg["n_head"], cfg["n_kv"], cfg["hd"], cfg["ffn"],
                                  cfg["vocab"], tied_head=cfg["tied"], max_batch=2, max_ctx=32,
                                  weight_kind=forge.FORGE_WEIGHT_Q4_G128 if cfg["q4"] else forge.FORGE_WEIGHT_BF16)
    return om, mk


@pytest.mark.parametrize("name", list(CONFIGS))
def test_safetensors_load_matches_upload(forge, oracle, cuda, tmp_path, name):
    cfg = CONFIGS[name]
    om, mk = _pair(oracle, forge, cfg)
    fa, fb = mk(), mk()
    fa.load_safetensors(_checkpoint(om, cfg, tmp_path))
    for l in range(cfg["n_layer"]):
        w = [om.bf16[(l, n)] for n in ("wq", "wk", "wv", "wo", "wg", "wu", "wd")]
        fb.load_layer(l, *w, om.gains[(l, "g1")], om.gains[(l, "g2")])
    fb.load_embedding(om.bf16["emb"], om.gains["gF"], None if cfg["tied"] else om.bf16["head"])
    toks = np.array([3, 77], np.int32)
    for _ in range(5):
        na, la = fa.step(toks, want_logits=True)
        nb, lb = fb.step(toks, want_logits=True)
        assert np.array_equal(la, lb) and np.array_equal(na, nb)
        toks = na
    fa.close(); fb.close()


def test_safetensors_load_rejects_bad_checkpoints(forge, oracle, cuda, tmp_path):
    cfg = CONFIGS["gqa_bf16_untied"]
    om, mk = _pair(oracle, forge, cfg)
    m = mk()
    (tmp_path / "a").mkdir()
    (tmp_path / "b").mkdir()
    with pytest.raises(forge.ForgeError, match="model.layers.1.mlp.up_proj.weight missing"):
        m.load_safetensors(_checkpoint(om, cfg, tmp_path / "a", drop="model.layers.1.mlp.up_proj.weight"))
    with pytest.raises(forge.ForgeError, match=r"self_attn.k_proj.weight has shape \[144, 256\]"):
        m.load_safetensors(_checkpoint(om, cfg, tmp_path / "b", reshape="model.layers.0.self_attn.k_proj.weight"))
    m.close()
