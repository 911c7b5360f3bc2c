"""The dispatch entries and descriptors on the B200, through the C ABI:
v1 PURE_BF16 families on HexaFarrBf16 slots (against numpy restatements of
the reference kernels' arithmetic), v2 GEMV / FLASH_DECODE on packed-weight
and KV-cache descriptors (against the per-op entries and the oracle), and
the engine's block-level families chained into a decode step (bit-identical
to forge_b200_decode_step)."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def bf16_farr(forge, a_bf16):
    L = forge.lib()
    a = np.ascontiguousarray(a_bf16, np.uint16).ravel()
    f = L.hexa_farr_bf16_alloc(len(a))
    C.memmove(f.contents.h_buf, a.ctypes.data, a.nbytes)
    return f


def bf16_of(forge, f):
    L = forge.lib()
    forge.check(L.hexa_farr_bf16_to_host(f), "to_host")
    n = f.contents.len
    return np.ctypeslib.as_array(C.cast(f.contents.h_buf, C.POINTER(C.c_uint16)), shape=(n,)).copy()


def f32_farr(forge, a, i32=False):
    L = forge.lib()
    a = np.ascontiguousarray(a, np.int32 if i32 else np.float32).ravel()
    f = (L.hexa_farr_i32_alloc if i32 else L.hexa_farr_f32_alloc)(len(a))
    C.memmove(f.contents.h_buf, a.ctypes.data, a.nbytes)
    return f


def f32_of(forge, f, i32=False):
    L = forge.lib()
    forge.check((L.hexa_farr_i32_to_host if i32 else L.hexa_farr_f32_to_host)(f), "to_host")
    n = f.contents.len
    t = C.c_int32 if i32 else C.c_float
    return np.ctypeslib.as_array(C.cast(f.contents.h_buf, C.POINTER(t)), shape=(n,)).copy()


def dispatch(forge, fam, prec, shape, ins, outs, v2=False):
    L = forge.lib()
    s = forge.ForgeShapeInfo(*shape)
    a, b = forge.forge_args(*ins), forge.forge_args(*outs)
    f = L.forge_tier_dispatch_v2 if v2 else L.forge_tier_dispatch_v1
    return f(fam, C.byref(s), 0, prec, 0, C.byref(a), C.byref(b))


def test_v1_matmul_known_answer(forge, cuda):
    F = forge
    A = bf16_farr(F, np.array([0x3F80, 0x4000, 0x4040, 0x4080, 0x40A0, 0x40C0], np.uint16))   # 1..6
    B = bf16_farr(F, np.array([0x40E0, 0x4100, 0x4110, 0x4120, 0x4130, 0x4140], np.uint16))   # 7..12
    Cc = F.lib().hexa_farr_bf16_alloc(4)
    rc = dispatch(F, F.FORGE_KERNEL_MATMUL, F.FORGE_PREC_PURE_BF16, (2, 2, 3, 0), (A, B), (Cc,))
    assert rc == F.FORGE_OK
    import oracle
    got = oracle.bf16_to_f32(bf16_of(F, Cc))
    assert np.array_equal(got, [58, 64, 139, 154])
    for f in (A, B, Cc):
        F.lib().hexa_farr_bf16_free(f)


@pytest.mark.parametrize("M,K,N", [(1, 4096, 1024), (7, 300, 130), (96, 128, 200)])
def test_v1_matmul(forge, oracle, cuda, M, K, N):
    F = forge
    rng = np.random.default_rng(M + K + N)
    a = oracle.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    b = oracle.f32_to_bf16((rng.standard_normal((K, N)) * 0.05).astype(np.float32))
    A, B, Cc = bf16_farr(F, a), bf16_farr(F, b), F.lib().hexa_farr_bf16_alloc(M * N)
    assert dispatch(F, F.FORGE_KERNEL_MATMUL, F.FORGE_PREC_PURE_BF16, (M, N, K, 0), (A, B), (Cc,)) == 0
    got = oracle.bf16_to_f32(bf16_of(F, Cc)).reshape(M, N).astype(np.float64)
    ref = oracle.bf16_to_f32(a).astype(np.float64) @ oracle.bf16_to_f32(b).astype(np.float64)
    # fp32 accumulation then one bf16 rounding (2^-9 relative)
    assert np.all(np.abs(got - ref) <= 2 ** -8 * np.abs(ref) + 1e-5 * np.abs(ref).max())
    for f in (A, B, Cc):
        F.lib().hexa_farr_bf16_free(f)


def test_v1_ffn(forge, oracle, cuda):
    F = forge
    M, D, FD = 4, 256, 512
    rng = np.random.default_rng(5)
    x = oracle.f32_to_bf16(rng.standard_normal((M, D)).astype(np.float32))
    w1 = oracle.f32_to_bf16((rng.standard_normal((D, FD)) * 0.06).astype(np.float32))
    w2 = oracle.f32_to_bf16((rng.standard_normal((FD, D)) * 0.06).astype(np.float32))
    X, W1, W2, Y = bf16_farr(F, x), bf16_farr(F, w1), bf16_farr(F, w2), F.lib().hexa_farr_bf16_alloc(M * D)
    assert dispatch(F, F.FORGE_KERNEL_FFN_FUSED, F.FORGE_PREC_PURE_BF16, (M, FD, D, 0), (X, W1, W2), (Y,)) == 0
    got = oracle.bf16_to_f32(bf16_of(F, Y)).reshape(M, D).astype(np.float64)
    f = lambda a: oracle.bf16_to_f32(a).astype(np.float64)
    h = f(oracle.f32_to_bf16((f(x) @ f(w1)).astype(np.float32)))        # H = bf16(X W1)
    hs = f(oracle.f32_to_bf16((h / (1 + np.exp(-h))).astype(np.float32)))  # in-place SiLU, bf16
    ref = hs @ f(w2)
    assert np.abs(got - ref).max() <= 2e-2 * np.abs(ref).max()
    for a in (X, W1, W2, Y):
        F.lib().hexa_farr_bf16_free(a)


def test_v1_rmsnorm_silu_rope(forge, oracle, cuda):
    F = forge
    rng = np.random.default_rng(9)
    T, d = 5, 768
    x = oracle.f32_to_bf16(rng.standard_normal((T, d)).astype(np.float32))
    g = oracle.f32_to_bf16((1 + 0.1 * rng.standard_normal(d)).astype(np.float32))
    X, G = bf16_farr(F, x), bf16_farr(F, g)
    Y, XN, I = (F.lib().hexa_farr_bf16_alloc(n) for n in (T * d, T * d, T))
    assert dispatch(F, F.FORGE_KERNEL_RMSNORM_MH, F.FORGE_PREC_PURE_BF16, (T, 0, d, 0), (X, G), (Y, XN, I)) == 0
    xf = oracle.bf16_to_f32(x).astype(np.float64)
    inv = 1 / np.sqrt((xf ** 2).mean(1, keepdims=True) + 1e-6)
    ref = oracle.bf16_to_f32(g) * xf * inv
    got = oracle.bf16_to_f32(bf16_of(F, Y)).reshape(T, d)
    assert np.all(np.abs(got - ref) <= 2 ** -7 * np.abs(ref) + 1e-6)
    assert np.all(np.abs(oracle.bf16_to_f32(bf16_of(F, I)) - inv[:, 0]) <= 2 ** -7 * inv[:, 0])
    # SILU_GATE: (a * sigmoid(a)) * b
    a = oracle.f32_to_bf16(rng.standard_normal(1000).astype(np.float32) * 3)
    b = oracle.f32_to_bf16(rng.standard_normal(1000).astype(np.float32))
    A, B, O = bf16_farr(F, a), bf16_farr(F, b), F.lib().hexa_farr_bf16_alloc(1000)
    assert dispatch(F, F.FORGE_KERNEL_SILU_GATE, F.FORGE_PREC_PURE_BF16, (10, 100, 0, 0), (A, B), (O,)) == 0
    af, bf = oracle.bf16_to_f32(a).astype(np.float64), oracle.bf16_to_f32(b).astype(np.float64)
    ref = af / (1 + np.exp(-af)) * bf
    got = oracle.bf16_to_f32(bf16_of(F, O))
    assert np.all(np.abs(got - ref) <= 2 ** -7 * np.abs(ref) + 1e-7)
    # ROPE_MH: two fp32 roundings then bf16: bit-exact against numpy float32
    T, nh, hd = 3, 4, 64
    xr = oracle.f32_to_bf16(rng.standard_normal((T, nh, hd)).astype(np.float32))
    ang = np.arange(T)[:, None] * (10000.0 ** (-np.arange(hd // 2) * 2.0 / hd))[None]
    cos = oracle.f32_to_bf16(np.concatenate([np.cos(ang)] * 2, 1).astype(np.float32))
    sin = oracle.f32_to_bf16(np.concatenate([np.sin(ang)] * 2, 1).astype(np.float32))
    Xr, Cs, Sn, Yr = bf16_farr(F, xr), bf16_farr(F, cos), bf16_farr(F, sin), F.lib().hexa_farr_bf16_alloc(T * nh * hd)
    assert dispatch(F, F.FORGE_KERNEL_ROPE_MH, F.FORGE_PREC_PURE_BF16, (T, nh, hd, 0), (Xr, Cs, Sn), (Yr,)) == 0
    xv = oracle.bf16_to_f32(xr)
    rh = np.concatenate([-xv[..., hd // 2:], xv[..., :hd // 2]], -1)
    cv, sv = oracle.bf16_to_f32(cos)[:, None, :], oracle.bf16_to_f32(sin)[:, None, :]
    ref = oracle.f32_to_bf16((xv * cv).astype(np.float32) + (rh * sv).astype(np.float32))
    assert np.array_equal(bf16_of(F, Yr), ref.ravel())


@pytest.mark.parametrize("q4", [True, False])
def test_v2_gemv_descriptors(forge, oracle, cuda, q4):
    F = forge
    L = F.lib()
    N, K, B = 1024, 2048, 3
    w = oracle.fill_normal_bf16(N * K, 3, 77, 0.02).reshape(N, K)
    Wl = bf16_farr(F, w)
    W = L.hexa_farr_w_alloc(F.HEXA_FARR_W_Q4_G128 if q4 else F.HEXA_FARR_W_BF16, N, K)
    F.check(L.hexa_farr_w_pack(W, Wl), "pack")
    x = np.random.default_rng(1).standard_normal((B, K)).astype(np.float32)
    X, Y = f32_farr(F, x), L.hexa_farr_f32_alloc(B * N)
    fam = F.FORGE_KERNEL_GEMV_W4A16_G128 if q4 else F.FORGE_KERNEL_GEMV_BF16
    prec = F.FORGE_PREC_W4A16_G128_BF16 if q4 else F.FORGE_PREC_PURE_BF16
    assert dispatch(F, fam, prec, (B, N, K, 0), (W, X), (Y,), v2=True) == 0
    got = f32_of(F, Y).reshape(B, N).astype(np.float64)
    if q4:
        codes = np.empty((N, K // 2), np.uint8)
        scales = np.empty((N, K // 128), np.uint16)
        F.check(L.hexa_farr_q4_unpack(W, codes.ctypes.data, scales.ctypes.data), "unpack")
        c_ref, s_ref = oracle.q4g_quantize(w)
        assert np.array_equal(codes, c_ref) and np.array_equal(scales, s_ref)
        Wf = oracle.q4g_dequant(c_ref, s_ref, K)
    else:
        Wf = oracle.bf16_to_f32(w)
    ref = x.astype(np.float64) @ Wf.astype(np.float64).T
    assert np.abs(got - ref).max() / np.abs(ref).max() < 6e-5
    L.hexa_farr_bf16_free(Wl)
    L.hexa_farr_w_free(W)
    L.hexa_farr_f32_free(X)
    L.hexa_farr_f32_free(Y)


def test_v2_flash_decode_kv_descriptor(forge, oracle, cuda):
    F = forge
    L = F.lib()
    nl, B, Hkv, lmax, hd, H = 2, 2, 2, 700, 128, 8
    kv = L.hexa_kv_alloc(nl, B, Hkv, lmax, hd)
    assert kv
    rng = np.random.default_rng(2)
    K = oracle.f32_to_bf16(rng.standard_normal((nl, B, Hkv, lmax, hd)).astype(np.float32) * 0.5)
    V = oracle.f32_to_bf16(rng.standard_normal((nl, B, Hkv, lmax, hd)).astype(np.float32))
    for l in range(nl):
        for b in range(B):
            k = np.ascontiguousarray(K[l, b])
            v = np.ascontiguousarray(V[l, b])
            F.check(L.hexa_kv_write(kv, l, b, k.ctypes.data, v.ctypes.data, lmax), "kv write")
    pos = np.array([699, 5], np.int32)
    F.check(L.hexa_kv_set_positions(kv, pos.ctypes.data, B), "positions")
    q = rng.standard_normal((B, H * hd)).astype(np.float32)
    Q, O = f32_farr(F, q), L.hexa_farr_f32_alloc(B * H * hd)
    layer = 1
    assert dispatch(F, F.FORGE_KERNEL_FLASH_DECODE, F.FORGE_PREC_PURE_BF16, (B, H, hd, 0),
                    (Q, kv, layer), (O,), v2=True) == 0
    got = f32_of(F, O).reshape(B, H * hd)
    Kf, Vf = oracle.bf16_to_f32(K[layer]).astype(np.float64), oracle.bf16_to_f32(V[layer]).astype(np.float64)
    G = H // Hkv
    for b in range(B):
        for h in range(H):
            s = Kf[b, h // G, :pos[b] + 1] @ q[b, h * hd:(h + 1) * hd] / np.sqrt(hd)
            p = np.exp(s - s.max())
            ref = p / p.sum() @ Vf[b, h // G, :pos[b] + 1]
            assert np.abs(got[b, h * hd:(h + 1) * hd] - ref).max() < 2e-5 * max(1, np.abs(ref).max())
    # a device-side bad position (written past the host check) is reported by
    # the per-op error word, not by the allocation-free entry's own word
    import torch
    F.check(L.forge_ops_check(), "clean before")
    L.forge_flash_decode_noalloc_status()

    class _Pos:  # the descriptor's device positions as a torch view
        __cuda_array_interface__ = {"shape": (B,), "typestr": "<i4", "data": (kv.contents.d_pos, False),
                                    "version": 3}
    torch.as_tensor(_Pos(), device="cuda")[1] = lmax
    assert dispatch(F, F.FORGE_KERNEL_FLASH_DECODE, F.FORGE_PREC_PURE_BF16, (B, H, hd, 0),
                    (Q, kv, layer), (O,), v2=True) == 0
    torch.cuda.synchronize()
    assert L.forge_flash_decode_noalloc_status() == 0
    assert L.forge_ops_check() != 0
    assert L.forge_ops_check() == 0
    L.hexa_kv_free(kv)
    L.hexa_farr_f32_free(Q)
    L.hexa_farr_f32_free(O)


@pytest.mark.parametrize("q4", [False, True])
def test_block_entries_chain_equals_decode_step(forge, cuda, q4, monkeypatch):
    """embed -> per layer (qkv_rope, attention, o_proj, mlp) -> lm_head through
    the block-level entries gives the decode step's logits bit for bit, and
    the DECODE_STEP / LMHEAD_ARGMAX dispatch families agree with both. The
    step's residual-stream handoff (int4), which changes the last bits of
    the RMSNorm GEMVs, is off here (FORGE_PREQUANT_NORM=0); its other
    handoffs are bit-identical to the staging."""
    import torch
    monkeypatch.setenv("FORGE_PREQUANT_NORM", "0")
    F = forge
    L = F.lib()
    nl, d, H, Hkv, hd, ffn, V = (2, 256, 8, 2, 64, 512, 1000) if not q4 else (2, 256, 4, 4, 64, 512, 1000)
    B, P0 = 3, 20
    m = F.ForgeModel(nl, d, H, Hkv, hd, ffn, V, weight_kind=F.FORGE_WEIGHT_Q4_G128 if q4 else F.FORGE_WEIGHT_BF16,
                     max_batch=4, max_ctx=64)
    m.init_synthetic(1234, 0.05)
    m.fill_kv_synthetic(7, P0, 0.5)
    tok = np.array([5, 17, 900], np.int32)
    nxt, lg = m.step(tok, want_logits=True)

    m.set_positions([P0] * B)
    x = torch.empty((B, d), device=cuda)
    q = torch.empty((B, H * hd), device=cuda)
    ctx = torch.empty((B, H * hd), device=cuda)
    tokd = torch.from_numpy(tok).to(cuda)
    out_tok = torch.empty(B, dtype=torch.int32, device=cuda)
    logits = torch.empty((B, V), device=cuda)
    torch.cuda.synchronize()
    m.embed(B, tokd, x)
    for layer in range(nl):
        m.qkv_rope(layer, B, x, q)
        m.attention(layer, B, q, ctx)
        m.o_proj(layer, B, ctx, x)
        m.mlp(layer, B, x, x)
    m.lm_head(B, x, out_tok, logits)
    m.sync()
    assert np.array_equal(logits.cpu().numpy(), lg)
    assert np.array_equal(out_tok.cpu().numpy(), nxt)

    # DECODE_STEP family on host int32 descriptors, from the same state
    m.set_positions([P0] * B)
    T, N, LG = f32_farr(F, tok, i32=True), L.hexa_farr_i32_alloc(B), L.hexa_farr_f32_alloc(B * V)
    prec = F.FORGE_PREC_W4A16_G128_BF16 if q4 else F.FORGE_PREC_PURE_BF16
    h = m.h.value
    assert dispatch(F, F.FORGE_KERNEL_DECODE_STEP, prec, (B, 0, 0, B), (h, T), (N, LG), v2=True) == 0
    got_n = np.ctypeslib.as_array(C.cast(N.contents.h_buf, C.POINTER(C.c_int32)), shape=(B,)).copy()
    got_l = np.ctypeslib.as_array(C.cast(LG.contents.h_buf, C.POINTER(C.c_float)), shape=(B * V,)).copy()
    assert np.array_equal(got_n, nxt) and np.array_equal(got_l.reshape(B, V), lg)

    # LMHEAD_ARGMAX family on the chained hidden state
    X = L.hexa_farr_f32_alloc(B * d)
    xh = np.ascontiguousarray(x.cpu().numpy())  # kept alive for the copy
    C.memmove(X.contents.h_buf, xh.ctypes.data, B * d * 4)
    TK = L.hexa_farr_i32_alloc(B)
    assert dispatch(F, F.FORGE_KERNEL_LMHEAD_ARGMAX, prec, (B, 0, 0, B), (h, X), (TK,), v2=True) == 0
    m.sync()
    assert np.array_equal(f32_of(F, TK, i32=True), nxt)
    for f in (T, N, TK):
        L.hexa_farr_i32_free(f)
    for f in (LG, X):
        L.hexa_farr_f32_free(f)
    m.close()


@pytest.mark.parametrize("B", [1, 4])
def test_block_entries_with_context_handoff(forge, cuda, B, monkeypatch):
    """Head dim 128, int4, up to 4 sequences: the decode step hands the
    staged context from the flash-decode merge to the O projection (and the
    staged SwiGLU output to the down projection); the block-level chain
    (which stages the inputs it is given) still equals the step bit for bit,
    and o_proj on a context of the caller's own after an attention call uses
    that context, not the step's handoff block. The residual-stream handoff,
    not bit-identical, is off (FORGE_PREQUANT_NORM=0)."""
    import torch
    monkeypatch.setenv("FORGE_PREQUANT_NORM", "0")
    F = forge
    nl, d, H, Hkv, hd, ffn, V, P0 = 2, 512, 4, 4, 128, 1024, 1000, 20
    m = F.ForgeModel(nl, d, H, Hkv, hd, ffn, V, weight_kind=F.FORGE_WEIGHT_Q4_G128, max_batch=4, max_ctx=64)
    m.init_synthetic(99, 0.05)
    m.fill_kv_synthetic(3, P0, 0.5)
    tok = (np.arange(B, dtype=np.int32) * 211 + 5) % V
    nxt, lg = m.step(tok, want_logits=True)
    m.set_positions([P0] * B)
    x = torch.empty((B, d), device=cuda)
    q = torch.empty((B, H * hd), device=cuda)
    ctx = torch.empty((B, H * hd), device=cuda)
    out_tok = torch.empty(B, dtype=torch.int32, device=cuda)
    logits = torch.empty((B, V), device=cuda)
    torch.cuda.synchronize()
    m.embed(B, torch.from_numpy(tok).to(cuda), x)
    for layer in range(nl):
        m.qkv_rope(layer, B, x, q)
        m.attention(layer, B, q, ctx)
        m.o_proj(layer, B, ctx, x)
        m.mlp(layer, B, x, x)
    m.lm_head(B, x, out_tok, logits)
    m.sync()
    assert np.array_equal(logits.cpu().numpy(), lg) and np.array_equal(out_tok.cpu().numpy(), nxt)

    # a context of the caller's own, right after an attention call
    own = torch.randn((B, H * hd), device=cuda) * 0.3
    x0 = torch.randn((B, d), device=cuda)
    x1, x2 = x0.clone(), x0.clone()
    m.attention(0, B, q, ctx)
    m.o_proj(0, B, own, x1)
    m.sync()
    m2 = F.ForgeModel(nl, d, H, Hkv, hd, ffn, V, weight_kind=F.FORGE_WEIGHT_Q4_G128, max_batch=4, max_ctx=64)
    m2.init_synthetic(99, 0.05)
    m2.o_proj(0, B, own, x2)
    m2.sync()
    assert torch.equal(x1, x2)
    m.close(); m2.close()
