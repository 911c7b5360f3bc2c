"""The .clm int4 checkpoint reader (forge_clm_*) on CPU.

test_roundtrip_reference_blocks replays the F-CLM-CKPT-ROUNDTRIP check of
stdlib/flame/clm_ckpt.hexa:95-160: the six conv-MoE blocks of its main()
(flame LCG weights, seeds 2/4/14/16/12/20, scale 0.2, quantised by
nn_int4_quant_fwd — both through the oracle's restatements) are written in
the .clm layout of save_block (clm_ckpt.hexa:47-61) and read back: every
int4 level exact and every fp32 scale byte-identical. The other tests cover
odd element counts (the pad nibble), the group-128 conversion and malformed
files."""
import ctypes as C
import struct

import numpy as np
import pytest


def quantise(oracle, w, cout, rest):
    L = oracle.lib()
    wq = np.zeros(cout * rest)
    scale = np.zeros(cout)
    q = np.zeros(cout * rest)
    mask = np.zeros(cout * rest)
    L.or_int4_quant_fwd(oracle.P(w), oracle.P(wq), oracle.P(scale), oracle.P(q), oracle.P(mask), cout, rest)
    return q.astype(np.int64), scale


def save_block(q, scale, cout, rest):
    """clm_ckpt.hexa:47-61: dims, (q+8) nibbles (pad 8), fp32-le scales."""
    out = bytearray(struct.pack("<II", cout, rest))
    n = cout * rest
    for i in range(0, n, 2):
        lo = (int(q[i]) + 8) & 0xF
        hi = (int(q[i + 1]) + 8) & 0xF if i + 1 < n else 8
        out.append(lo + hi * 16)
    out += np.asarray(scale, np.float32).tobytes()
    return bytes(out)


def write_clm(path, blocks):
    with open(path, "wb") as f:
        f.write(b"CLM\x01" + bytes([len(blocks)]) + b"".join(save_block(*b) for b in blocks))


def test_roundtrip_reference_blocks(forge, oracle, tmp_path):
    d, E, V, K = 8, 2, 256, 3
    seeds = [2, 4, 14, 16, 12, 20]
    couts = [d, d, d, d, E, V]
    rests = [d * K, d * K, d * K, d * K, d, d]
    blocks = []
    for seed, cout, rest in zip(seeds, couts, rests):
        w = np.zeros(cout * rest)
        oracle.lib().or_flame_fill_lcg(oracle.P(w), cout * rest, seed, 0.2)
        q, s = quantise(oracle, w, cout, rest)
        assert q.min() >= -7 and q.max() <= 7
        blocks.append((q, s, cout, rest))
    p = str(tmp_path / "clm_ckpt_smoke.clm")
    write_clm(p, blocks)
    c = forge.Clm(p)
    assert len(c) == 6
    for i, (q, s, cout, rest) in enumerate(blocks):
        b = c.block(i)
        assert (b.cout, b.rest) == (cout, rest)
        ql, sl = c.levels(i)
        assert np.array_equal(ql.ravel().astype(np.int64), q)
        assert sl.tobytes() == np.asarray(s, np.float32).tobytes()
    c.close()


def test_odd_count_and_q4g128(forge, oracle, tmp_path):
    rng = np.random.default_rng(1)
    blocks = []
    for cout, rest in [(3, 5), (16, 256), (5, 384)]:
        w = rng.standard_normal(cout * rest)
        q, s = quantise(oracle, w, cout, rest)
        blocks.append((q, s, cout, rest))
    # a bf16-exact scale row, so the conversion is exact for that row
    blocks[1][1][0] = 0.0625
    p = str(tmp_path / "m.clm")
    write_clm(p, blocks)
    c = forge.Clm(p)
    q0, _ = c.levels(0)
    assert np.array_equal(q0.ravel().astype(np.int64), blocks[0][0])  # 15 levels, one pad nibble
    with pytest.raises(forge.ForgeError, match="multiple of 128"):
        c.to_q4g128(0)
    for i in (1, 2):
        q, s, cout, rest = blocks[i]
        codes, sc = c.to_q4g128(i)
        assert np.array_equal(codes.ravel().astype(np.int64), q + 7)
        want = oracle.f32_to_bf16(np.asarray(s, np.float32))
        assert np.array_equal(sc, np.repeat(want[:, None], rest // 128, axis=1))
    assert c.to_q4g128(1)[1][0, 0] == oracle.f32_to_bf16(np.float32([0.0625]))[0]


def test_level_minus_8_and_malformed(forge, tmp_path):
    p = str(tmp_path / "m8.clm")
    q = np.zeros(128, np.int64)
    q[5] = -8
    write_clm(p, [(q, np.ones(1), 1, 128)])
    c = forge.Clm(p)
    assert c.levels(0)[0][0, 5] == -8
    with pytest.raises(forge.ForgeError, match="level -8"):
        c.to_q4g128(0)
    good = open(p, "rb").read()
    for name, data, msg in [("magic", b"CLX\x01" + good[4:], "magic"), ("short", good[:-3], "truncated"),
                            ("trail", good + b"\0", "trailing"), ("hdr", good[:7], "truncated")]:
        bp = str(tmp_path / f"{name}.clm")
        open(bp, "wb").write(data)
        with pytest.raises(forge.ForgeError, match=msg):
            forge.Clm(bp)
    with pytest.raises(forge.ForgeError, match="cannot open"):
        forge.Clm(str(tmp_path / "missing.clm"))
