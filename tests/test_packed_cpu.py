"""Packed-argument entries (forge_b200_create_packed,
forge_b200_decode_step_sampled_packed, forge_b200_desc_from_packed) for FFIs
that pass at most six integer arguments and write 8-byte fields — the
convention of hxflash_attn_fwd_packed (self/ml/hxflash.hexa:40-62). On CPU:
the field layout decodes into ForgeModelDesc, out-of-range fields are
rejected, and the entries fail cleanly without a device."""
import ctypes as C
import struct

import pytest


def create_block(result_addr=0, **kw):
    f = dict(n_layer=32, d_model=4096, n_head=32, n_kv_head=8, head_dim=128, ffn=11008, vocab=32000,
             rms_eps=1e-5, rope_theta=500000.0, weight_kind=1, tied_head=0, max_batch=4, max_ctx=2048, act_mode=0,
             device=0)
    f.update(kw)
    b = struct.pack("<7q2d6qq", f["n_layer"], f["d_model"], f["n_head"], f["n_kv_head"], f["head_dim"], f["ffn"],
                    f["vocab"], f["rms_eps"], f["rope_theta"], f["weight_kind"], f["tied_head"], f["max_batch"],
                    f["max_ctx"], f["act_mode"], f["device"], result_addr)
    assert len(b) == 128
    return C.create_string_buffer(b, 128)


def test_desc_from_packed(forge):
    d = forge.ForgeModelDesc()
    buf = create_block()
    assert forge.lib().forge_b200_desc_from_packed(buf, C.byref(d)) == 0
    assert (d.n_layer, d.d_model, d.n_head, d.n_kv_head, d.head_dim, d.ffn, d.vocab) == (32, 4096, 32, 8, 128, 11008,
                                                                                      32000)
    assert d.rms_eps == pytest.approx(1e-5) and d.rope_theta == 500000.0
    assert (d.weight_kind, d.tied_head, d.max_batch, d.max_ctx, d.act_mode, d.tp_rank, d.tp_size) == (1, 0, 4, 2048, 0,
                                                                                                     0, 1)
    assert forge.lib().forge_b200_desc_from_packed(create_block(vocab=1 << 40), C.byref(d)) != 0
    assert "out of range" in forge.lib().forge_b200_last_error().decode()


def test_packed_entries_fail_cleanly_without_device(forge):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    L = forge.lib()
    h = C.c_void_p()
    assert L.forge_b200_create_packed(create_block(C.addressof(h), n_layer=1, d_model=256, n_head=4, n_kv_head=2,
                                                   head_dim=64, ffn=512, vocab=1000)) != 0
    assert h.value is None
    assert L.forge_b200_create_packed(create_block(0)) != 0  # no result address
    step = C.create_string_buffer(struct.pack("<qqqqdqdq", 0, 1, 0, 0, 0.7, 40, 0.9, 0), 64)
    assert L.forge_b200_decode_step_sampled_packed(step) != 0
    assert "null handle" in L.forge_b200_last_error().decode()
