"""The safetensors reader (forge_st_*, host code in libforge_b200.so) on CPU.

test_mmap_views follows self/test_safetensors_mmap.hexa (dummy file of an F32
[3] and a BF16 [2, 2] tensor: count, header end, names in header order,
dtype / byte count / shape, byte accessor with 0 out of range, adjacent
views, total bytes, null view for a missing name, close, null handle for a
missing file); test_builtin_contract follows tmp_stmmap_smoke.hexa (56-byte
header, t0 = [1, 2, 3, 4]: data offset 64, size 80, read_f32 / read_bytes at
the data offset, re-open after close, two opens byte-equal). The remaining
tests cover random files against Python's json / struct reading of the same
bytes, the dtype conversions against the oracle's round-to-nearest-even and
exact rational rounding, and malformed files (each rejected with a message).
"""
import json
import os
import struct
from fractions import Fraction

import numpy as np
import pytest


def write_st(path, tensors, metadata=None, pad_to=None, raw_header=None):
    """tensors: list of (name, dtype, shape, bytes); offsets laid out in order."""
    hdr, blobs, off = {}, [], 0
    if metadata is not None:
        hdr["__metadata__"] = metadata
    for name, dt, shape, data in tensors:
        hdr[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + len(data)]}
        blobs.append(data)
        off += len(data)
    h = raw_header if raw_header is not None else json.dumps(hdr, separators=(",", ":")).encode()
    if pad_to:
        h = h + b" " * (pad_to - len(h))
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"".join(blobs))
    return 8 + len(h)


def test_mmap_views(forge, tmp_path):
    p = str(tmp_path / "dummy.safetensors")
    t0 = bytes([10, 11, 12, 20, 21, 22, 30, 31, 32, 40, 41, 42])
    t1 = bytes([50, 51, 60, 61, 70, 71, 80, 81])
    header_end = write_st(p, [("t0", "F32", [3], t0), ("t1", "BF16", [2, 2], t1)])
    st = forge.Safetensors(p)
    assert len(st) == 2
    assert st.data_offset == header_end
    assert st.names() == ["t0", "t1"]
    v0, v1 = st.find("t0"), st.find("t1")
    assert forge.ST_DTYPES[v0.dtype] == "F32" and v0.nbytes == 12 and v0.ndim == 1 and v0.shape[0] == 3
    assert forge.ST_DTYPES[v1.dtype] == "BF16" and v1.nbytes == 8 and (v1.ndim, v1.shape[0], v1.shape[1]) == (2, 2, 2)
    L = forge.lib()
    u8 = lambda v, i: L.forge_st_view_u8(forge.C.byref(v), i)
    assert (u8(v0, 0), u8(v0, 1), u8(v0, 11)) == (10, 11, 42)
    assert u8(v0, 12) == 0 and u8(v0, -1) == 0
    assert (u8(v1, 0), u8(v1, 7)) == (50, 81)
    assert v0.offset >= header_end and v0.offset < st.size
    assert v1.data == v0.data + 12 and v1.offset == v0.offset + 12
    assert st.total_bytes == 20
    assert st.find("__nope__") is None
    assert st.close() >= 0
    with pytest.raises(forge.ForgeError, match="cannot open"):
        forge.Safetensors(str(tmp_path / "does_not_exist.bin"))
    assert L.forge_st_close(None) == 0


def test_builtin_contract(forge, tmp_path):
    p = str(tmp_path / "fixture.safetensors")
    data = np.array([1, 2, 3, 4], np.float32).tobytes()
    write_st(p, [("t0", "F32", [4], data)], pad_to=56)
    st = forge.Safetensors(p)
    hdr = st.header()
    assert len(hdr) == 56 and b"{" in hdr and b"t0" in hdr and b"F32" in hdr
    assert st.data_offset == 64 and st.size == 80
    assert st.read_f32(64, 4).tolist() == [1.0, 2.0, 3.0, 4.0]
    assert st.read_bytes(64, 4) == bytes([0, 0, 0x80, 0x3F])
    st.close()
    st2 = forge.Safetensors(p)
    st3 = forge.Safetensors(p)
    assert st2.header() == st3.header() == hdr and st2.data_offset == st3.data_offset == 64
    with pytest.raises(forge.ForgeError, match="outside the file"):
        st2.read_f32(64, 5)
    with pytest.raises(forge.ForgeError, match="outside the file"):
        st2.read_bytes(-1, 2)
    assert st2.read_bf16_to_f32(64 + 2, 1).tolist() == [1.0]  # upper half of 1.0f


NP = {"F16": np.float16, "F32": np.float32, "F64": np.float64, "I8": np.int8, "U8": np.uint8, "I16": np.int16,
      "U16": np.uint16, "I32": np.int32, "U32": np.uint32, "I64": np.int64, "U64": np.uint64, "BOOL": np.bool_}


def test_random_files_match_python_reading(forge, tmp_path):
    rng = np.random.default_rng(7)
    for trial in range(6):
        tensors = []
        for k in range(int(rng.integers(1, 12))):
            dt = rng.choice(["F16", "F32", "F64", "BF16", "I8", "U8", "I16", "U16", "I32", "U32", "I64", "U64",
                             "BOOL", "F8_E4M3", "F8_E5M2"])
            shape = [int(s) for s in rng.integers(0, 5, size=int(rng.integers(0, 4)))]
            esz = {"BF16": 2, "F8_E4M3": 1, "F8_E5M2": 1}.get(dt) or np.dtype(NP[dt]).itemsize
            n = int(np.prod(shape, dtype=np.int64))
            name = f"model.layers.{k}.wéight \"q\"/{trial}"
            tensors.append((name, str(dt), shape, rng.integers(0, 256, size=n * esz, dtype=np.uint8).tobytes()))
        p = str(tmp_path / f"r{trial}.safetensors")
        meta = {"format": "pt", "note": "tab\there ☃"} if trial % 2 else None
        write_st(p, tensors, metadata=meta, pad_to=None if trial % 3 else 4096)
        raw = open(p, "rb").read()
        hl = struct.unpack("<Q", raw[:8])[0]
        hdr = json.loads(raw[8:8 + hl])
        st = forge.Safetensors(p)
        names = [k for k in hdr if k != "__metadata__"]
        assert st.names() == names
        assert st.total_bytes == sum(len(t[3]) for t in tensors)
        for name, dt, shape, data in tensors:
            v = st.find(name)
            assert forge.ST_DTYPES[v.dtype] == dt and v.ndim == len(shape)
            assert [v.shape[i] for i in range(v.ndim)] == shape
            assert v.offset == 8 + hl + hdr[name]["data_offsets"][0]
            assert st.read_bytes(v.offset, v.nbytes) == data
            assert forge.C.string_at(v.data, v.nbytes) == data if v.nbytes else True
        if meta:
            assert st.metadata("format") == "pt" and st.metadata("note") == meta["note"]
        assert st.metadata("absent") is None
        st.close()


def _bf16_nearest_even(x: float) -> int:
    """Exact round-to-nearest-even of a finite double to bf16 bits (Fractions)."""
    if x == 0:
        return 0x8000 if np.signbit(x) else 0
    sign = 0x8000 if x < 0 else 0
    ax = Fraction(abs(x))
    def val(b):  # b: 15-bit magnitude; 0x7F80 stands for 2^128 (rounding as if the range went on)
        if b >= 0x7F80:
            return Fraction(2) ** 128
        return Fraction(float(np.array([b << 16], np.uint32).view(np.float32)[0]))
    with np.errstate(over="ignore"):
        t = int(np.array([abs(x)], np.float32).view(np.uint32)[0]) >> 16  # near the answer
    best = None
    for b in range(max(t - 2, 0), min(t + 3, 0x7F81)):
        d = abs(val(b) - ax)
        if best is None or d < best[0] or (d == best[0] and b % 2 == 0):
            best = (d, b)
    return sign | min(best[1], 0x7F80)


def test_conversions(forge, oracle, tmp_path):
    rng = np.random.default_rng(3)
    f32 = np.concatenate([rng.standard_normal(4000).astype(np.float32) * np.float32(10) ** rng.integers(-40, 38, 4000),
                          np.array([0.0, -0.0, np.inf, -np.inf, 3.4e38, -3.4e38, 1e-45, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8],
                                   np.float32)]).astype(np.float32)
    f16 = np.concatenate([rng.standard_normal(3000).astype(np.float16),
                          np.array([0, -0.0, 6e-8, -6e-8, 65504, np.inf, -np.inf], np.float16)])
    f16_bits = np.concatenate([f16.view(np.uint16), np.arange(0, 65536, 97, dtype=np.uint16)])
    f16 = f16_bits.view(np.float16)
    f16 = f16[~np.isnan(f16)]
    f64 = np.concatenate([rng.standard_normal(2000) * 10.0 ** rng.integers(-40, 38, 2000),
                          np.array([1.0 + 2 ** -8, 1.0 + 2 ** -8 + 2 ** -40, 1.0 + 2 ** -8 - 2 ** -40,
                                    1.0 + 3 * 2 ** -8, (1.0 + 2 ** -8) * (1 + 2 ** -30), 3.4e38, 3.5e38, 1e300,
                                    -1e300, 1e-300, 2.0 ** -133, 2.0 ** -134 * 3])])
    bf = rng.integers(0, 65536, 3000, dtype=np.uint16)
    bf = bf[(bf & 0x7F80) != 0x7F80]  # no NaN / inf patterns in the value checks
    p = str(tmp_path / "conv.safetensors")
    write_st(p, [("f32", "F32", [f32.size], f32.tobytes()), ("f16", "F16", [f16.size], f16.tobytes()),
                 ("f64", "F64", [f64.size], f64.tobytes()), ("bf", "BF16", [bf.size], bf.tobytes()),
                 ("i8", "I8", [4], b"\x01\x02\x03\x04")])
    st = forge.Safetensors(p)
    # F32 -> bf16 equals the oracle's round to nearest even
    assert np.array_equal(st.to_bf16(st.find("f32")), oracle.f32_to_bf16(f32))
    # F16 -> f32 exact, F16 -> bf16 = RNE of that
    assert np.array_equal(st.to_f32(st.find("f16")).view(np.uint32), f16.astype(np.float32).view(np.uint32))
    assert np.array_equal(st.to_bf16(st.find("f16")), oracle.f32_to_bf16(f16.astype(np.float32)))
    # F64 -> bf16: one rounding, checked exactly
    got = st.to_bf16(st.find("f64"))
    want = np.array([_bf16_nearest_even(float(x)) for x in f64], np.uint16)
    assert np.array_equal(got, want), np.nonzero(got != want)
    # BF16 passes through; to_f32 widens exactly
    assert np.array_equal(st.to_bf16(st.find("bf")), bf)
    assert np.array_equal(st.to_f32(st.find("bf")).view(np.uint32), bf.astype(np.uint32) << 16)
    with pytest.raises(forge.ForgeError, match="not a floating-point"):
        st.to_bf16(st.find("i8"))


BAD = [
    ("short", None, "shorter than"),
    ("hlen", "hlen", "past the end"),
    ("huge", "huge", "100 MB limit"),
    ("notjson", b"[1, 2]", "not a JSON object"),
    ("badjson", b'{"a": {"dtype": "F32", "shape": [1], "data_offsets": [0, 4]', "expected"),
    ("dtype", b'{"a": {"dtype": "F31", "shape": [1], "data_offsets": [0, 4]}}', "unknown dtype"),
    ("count", b'{"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 4]}}', "byte count"),
    ("range", b'{"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}}', "outside the data region"),
    ("order", b'{"a": {"dtype": "F32", "shape": [0], "data_offsets": [4, 0]}}', "outside the data region"),
    ("neg", b'{"a": {"dtype": "F32", "shape": [-1], "data_offsets": [0, 4]}}', "bad shape"),
    ("frac", b'{"a": {"dtype": "F32", "shape": [1.0], "data_offsets": [0, 4]}}', "fraction"),
    ("dup", b'{"a": {"dtype": "U8", "shape": [1], "data_offsets": [0, 1]}, '
            b'"a": {"dtype": "U8", "shape": [1], "data_offsets": [1, 2]}}', "duplicate"),
    ("missing", b'{"a": {"dtype": "F32", "shape": [1]}}', "needs dtype"),
    ("trail", b'{"a": {"dtype": "F32", "shape": [1], "data_offsets": [0, 4]}} x', "trailing"),
    ("meta", b'{"__metadata__": {"k": 1}}', "expected a string"),
    ("esc", b'{"a\\q": {"dtype": "F32", "shape": [1], "data_offsets": [0, 4]}}', "bad escape"),
]


@pytest.mark.parametrize("case,header,msg", BAD, ids=[b[0] for b in BAD])
def test_malformed_files_are_rejected(forge, tmp_path, case, header, msg):
    p = str(tmp_path / f"{case}.safetensors")
    if case == "short":
        open(p, "wb").write(b"\x01\x02\x03")
    elif case == "hlen":
        open(p, "wb").write(struct.pack("<Q", 1000) + b"{}")
    elif case == "huge":
        with open(p, "wb") as f:  # a sparse file past the 100 MB header limit
            f.write(struct.pack("<Q", 100000001) + b"{")
            f.truncate(8 + 100000001)
    else:
        open(p, "wb").write(struct.pack("<Q", len(header)) + header + b"\0" * 4)
    with pytest.raises(forge.ForgeError, match=msg):
        forge.Safetensors(p)


def test_empty_header_and_escaped_names(forge, tmp_path):
    p = str(tmp_path / "empty.safetensors")
    write_st(p, [], raw_header=b"{}")
    st = forge.Safetensors(p)
    assert len(st) == 0 and st.total_bytes == 0 and st.data_offset == 10
    p2 = str(tmp_path / "esc.safetensors")
    write_st(p2, [("x", "U8", [1], b"\x07")],
             raw_header=b'{"\\u00e9\\ud83d\\ude00\\n\\"": {"dtype": "U8", "shape": [1], "data_offsets": [0, 1]}}')
    st2 = forge.Safetensors(p2)
    assert st2.names() == ["é\U0001F600\n\""]


def _llama(cfg, tied, dtype="BF16", drop=(), reshape=None, int_name=None):
    """Tensors of the Llama layout for cfg, zero-filled (shapes are what matter)."""
    L, d, H, Hkv, hd, F, V = cfg
    shapes = {}
    for l in range(L):
        p = f"model.layers.{l}."
        shapes.update({p + "self_attn.q_proj.weight": (H * hd, d), p + "self_attn.k_proj.weight": (Hkv * hd, d),
                       p + "self_attn.v_proj.weight": (Hkv * hd, d), p + "self_attn.o_proj.weight": (d, H * hd),
                       p + "mlp.gate_proj.weight": (F, d), p + "mlp.up_proj.weight": (F, d),
                       p + "mlp.down_proj.weight": (d, F), p + "input_layernorm.weight": (d,),
                       p + "post_attention_layernorm.weight": (d,)})
    shapes.update({"model.embed_tokens.weight": (V, d), "model.norm.weight": (d,)})
    if not tied:
        shapes["lm_head.weight"] = (V, d)
    out = []
    for name, shp in shapes.items():
        if name in drop:
            continue
        if name == reshape:
            shp = (shp[0] + 1,) + shp[1:]
        dt = "I32" if name == int_name else dtype
        esz = {"BF16": 2, "F16": 2, "F32": 4, "F64": 8, "I32": 4}[dt]
        out.append((name, dt, list(shp), bytes(int(np.prod(shp)) * esz)))
    return out


def test_check_llama_checkpoint(forge, tmp_path):
    cfg = (2, 128, 4, 2, 32, 256, 300)
    L = forge.lib()

    def check(tensors, tied=False, split=2, sub="c"):
        d = tmp_path / sub
        d.mkdir(exist_ok=True)
        paths = []
        for k in range(split):
            p = str(d / f"model-{k}.safetensors")
            write_st(p, tensors[k::split])
            paths.append(p)
        desc = forge.ForgeModelDesc(n_layer=cfg[0], d_model=cfg[1], n_head=cfg[2], n_kv_head=cfg[3],
                                    head_dim=cfg[4], ffn=cfg[5], vocab=cfg[6], tied_head=int(tied))
        arr = (forge.C.c_char_p * len(paths))(*[p.encode() for p in paths])
        rc = L.forge_safetensors_check_llama(forge.C.byref(desc), len(paths), arr)
        return rc, L.forge_b200_last_error().decode()

    assert check(_llama(cfg, False), sub="ok")[0] == 0
    assert check(_llama(cfg, True), tied=True, sub="tied")[0] == 0
    assert check(_llama(cfg, False) + [("extra.bias", "F32", [3], bytes(12))], sub="extra")[0] == 0  # extras ignored
    for dt in ("F16", "F32", "F64"):
        assert check(_llama(cfg, False, dtype=dt), split=1, sub=dt)[0] == 0
    rc, msg = check(_llama(cfg, True), tied=False, sub="nohead")
    assert rc != 0 and "lm_head.weight missing" in msg
    rc, msg = check(_llama(cfg, False, drop=("model.layers.1.mlp.down_proj.weight",)), sub="drop")
    assert rc != 0 and "model.layers.1.mlp.down_proj.weight missing" in msg
    rc, msg = check(_llama(cfg, False, reshape="model.layers.0.self_attn.k_proj.weight"), sub="shape")
    assert rc != 0 and "self_attn.k_proj.weight has shape [65, 128], expected [64, 128]" in msg
    rc, msg = check(_llama(cfg, False, int_name="model.norm.weight"), sub="int")
    assert rc != 0 and "model.norm.weight is not a floating-point tensor" in msg
    t = _llama(cfg, False)
    rc, msg = check(t + [t[0]], split=2, sub="dup")  # the same name in both shards
    assert rc != 0 and "appears in two files" in msg
