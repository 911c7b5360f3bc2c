"""Per-op parity on the B200: device weight generation, int4 quantisation and
packing (bit-exact against the oracle), decode GEMVs and split-K flash-decode
(against f64 oracle arithmetic). All calls go through libforge_b200.so."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _dev_bf16(torch, a, dev):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev)


def test_fill_normal_bit_exact(forge, oracle, cuda):
    import torch
    n = 1 << 17
    for seed, off in [(1234, 0), (1234, (5 << 40) + 17), (7, 99)]:
        d = torch.empty(n, dtype=torch.int16, device=cuda)
        forge.check(forge.lib().forge_fill_normal_bf16(d.data_ptr(), n, seed, off, 0.02, 0), "fill")
        torch.cuda.synchronize()
        host = oracle.fill_normal_bf16(n, seed, off, 0.02)
        got = d.cpu().numpy().view(np.uint16)
        assert np.array_equal(got, host), f"mismatches: {(got != host).sum()}"
    vals = oracle.bf16_to_f32(host)
    assert abs(vals.mean()) < 1e-3 and abs(vals.std() - 0.02) < 1e-3


@pytest.mark.parametrize("rows,K", [(16, 128), (48, 1024), (64, 11008)])
def test_q4_quantize_bit_exact(forge, oracle, cuda, rows, K):
    import torch
    w = oracle.fill_normal_bf16(rows * K, 99, 3, 0.05).reshape(rows, K)
    w[0, :128] = 0                      # all-zero group -> scale 1 sentinel
    w[1, :] = oracle.f32_to_bf16(np.linspace(-3, 3, K, dtype=np.float32))  # wide group
    wd = _dev_bf16(torch, w, cuda)
    codes, scales, tiles, stiles = forge.q4_pack(wd)
    torch.cuda.synchronize()
    c_ref, s_ref = oracle.q4g_quantize(w)
    assert np.array_equal(codes.cpu().numpy(), c_ref)
    assert np.array_equal(scales.cpu().numpy().view(np.uint16), s_ref)
    # the packed tile layout round-trips to the logical codes/scales
    c2 = torch.empty_like(codes)
    s2 = torch.empty_like(scales)
    forge.check(forge.lib().forge_q4_unpack_tiles(tiles.data_ptr(), stiles.data_ptr(), rows, K, 128,
                                                  c2.data_ptr(), s2.data_ptr(), 0), "unpack")
    torch.cuda.synchronize()
    assert np.array_equal(c2.cpu().numpy(), c_ref)
    assert np.array_equal(s2.cpu().numpy().view(np.uint16), s_ref)


def _gemv_ref(Wf, X, act_bf16, oracle):
    x = X.astype(np.float64)
    if act_bf16:
        x = oracle.bf16_to_f32(oracle.f32_to_bf16(X)).astype(np.float64)
    return x @ Wf.astype(np.float64).T


@pytest.mark.parametrize("wkind", ["q4", "bf16"])
@pytest.mark.parametrize("N,K", [(16, 128), (4096, 4096), (1376, 4096), (4096, 11008), (32000, 256)])
@pytest.mark.parametrize("batch,exact", [(1, 1), (3, 1), (8, 0), (5, 1)])
def test_gemv(forge, oracle, cuda, wkind, N, K, batch, exact):
    import torch
    if wkind == "bf16" and K % 16:
        pytest.skip("shape")
    rng = np.random.default_rng(N * 7 + K + batch)
    w = oracle.fill_normal_bf16(N * K, 5, N + K, 0.02).reshape(N, K)
    X = rng.standard_normal((batch, K)).astype(np.float32)
    wd = _dev_bf16(torch, w, cuda)
    xd = torch.from_numpy(X).to(cuda)
    yd = torch.full((batch, N), float("nan"), dtype=torch.float32, device=cuda)
    if wkind == "q4":
        codes, scales, tiles, stiles = forge.q4_pack(wd)
        Wf = oracle.q4g_dequant(codes.cpu().numpy(), scales.cpu().numpy().view(np.uint16), K)
        rc = forge.lib().forge_gemv_w4a16_g128(tiles.data_ptr(), stiles.data_ptr(), N, K, xd.data_ptr(),
                                               batch, yd.data_ptr(), exact, 0)
    else:
        tiles = forge.bf16_pack(wd)
        Wf = oracle.bf16_to_f32(w)
        rc = forge.lib().forge_gemv_bf16(tiles.data_ptr(), N, K, xd.data_ptr(), batch, yd.data_ptr(), exact, 0)
    forge.check(rc, "gemv")
    torch.cuda.synchronize()
    forge.check(forge.lib().forge_ops_check(), "gemv error word")
    y = yd.cpu().numpy().astype(np.float64)
    # bf16 weights: exact mode splits every activation into hi/lo bf16 (~16
    # bits each), bf16 mode is compared against bf16-rounded activations.
    # int4 weights always run the int8 tensor-core path with hi/lo int8
    # activations per 128-group (~2^-16 of the group maximum).
    act_bf16 = wkind == "bf16" and not exact
    ref = _gemv_ref(Wf, X, act_bf16, oracle)
    scale = np.abs(ref).max() + 1e-12
    err = np.abs(y - ref).max() / scale
    assert err < (6e-5 if wkind == "q4" else 2e-5), f"rel err {err}"


@pytest.mark.parametrize("B,H,Hkv,hd,lmax,pos", [
    (1, 4, 4, 64, 300, [200]),
    (2, 8, 2, 64, 1100, [1023, 5]),
    (1, 32, 32, 128, 2304, [2047]),
    (3, 4, 1, 128, 600, [0, 599, 77]),
    (4, 16, 4, 128, 4200, [4100, 3000, 17, 1]),
])
def test_flash_decode(forge, oracle, cuda, B, H, Hkv, hd, lmax, pos):
    import torch
    rng = np.random.default_rng(B * 1000 + H + lmax)
    q = rng.standard_normal((B, H * hd)).astype(np.float32)
    K = rng.standard_normal((B, Hkv, lmax, hd)).astype(np.float32) * 0.5
    V = rng.standard_normal((B, Hkv, lmax, hd)).astype(np.float32)
    Kb, Vb = oracle.f32_to_bf16(K), oracle.f32_to_bf16(V)
    Kf, Vf = oracle.bf16_to_f32(Kb).astype(np.float64), oracle.bf16_to_f32(Vb).astype(np.float64)
    ref = np.zeros((B, H * hd))
    G = H // Hkv
    for b in range(B):
        L = pos[b] + 1
        for h in range(H):
            kv = h // G
            s = Kf[b, kv, :L] @ q[b, h * hd:(h + 1) * hd].astype(np.float64) / np.sqrt(hd)
            p = np.exp(s - s.max())
            ref[b, h * hd:(h + 1) * hd] = (p / p.sum()) @ Vf[b, kv, :L]
    ws_bytes = forge.lib().forge_flash_decode_workspace_bytes(B, H, Hkv, hd, lmax)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=cuda)
    qd = torch.from_numpy(q).to(cuda)
    kd = torch.from_numpy(Kb.view(np.int16)).to(cuda)
    vd = torch.from_numpy(Vb.view(np.int16)).to(cuda)
    pd = torch.tensor(pos, dtype=torch.int32, device=cuda)
    out = torch.full((B, H * hd), float("nan"), device=cuda)
    for rep in range(2):  # second call reuses the workspace (counters must be back at zero)
        forge.check(forge.lib().forge_flash_decode(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), pd.data_ptr(),
                                                   B, H, Hkv, hd, lmax, out.data_ptr(), ws.data_ptr(), 0), "fd")
        torch.cuda.synchronize()
        forge.check(forge.lib().forge_ops_check(), "fd error word")
        got = out.cpu().numpy()
        assert np.abs(got - ref).max() < 2e-5 * max(1.0, np.abs(ref).max()), np.abs(got - ref).max()


# K 384 / 1408 / 128: odd group counts and a single group (the tensor-core
# path works on pairs of groups)
@pytest.mark.parametrize("N,K", [(4096, 4096), (4096, 11008), (22016, 4096), (1376, 4096), (48, 256), (1024, 384),
                                 (4096, 1408), (48, 128)])
@pytest.mark.parametrize("batch", [5, 8, 17, 32, 37])
def test_gemv_int4_batched_matches_small_batch(forge, oracle, cuda, N, K, batch):
    """Above 4 sequences the int4 GEMV streams the weights once for up to 32
    sequences (activations quantised once into a global scratch): on the
    register-fragment kernel (bit-identical to the small-batch path) or, for
    chunks of >= 24 sequences, on the tensor cores (tcgen05 kind::i8), whose
    integer products are the same and whose fp32 sums over groups run in
    another order, so results agree to a few ulps of the partial sums
    (bound: 1e-5 of the largest output)."""
    import torch
    rng = np.random.default_rng(N + K + batch)
    w = oracle.fill_normal_bf16(N * K, 9, N * 3 + K, 0.02).reshape(N, K)
    X = (rng.standard_normal((batch, K)) * rng.uniform(0.1, 4.0, (batch, 1))).astype(np.float32)
    _, _, tiles, stiles = forge.q4_pack(_dev_bf16(torch, w, cuda))
    xd = torch.from_numpy(X).to(cuda)
    lib = forge.lib()
    yb = torch.full((batch, N), float("nan"), device=cuda)
    forge.check(lib.forge_gemv_w4a16_g128(tiles.data_ptr(), stiles.data_ptr(), N, K, xd.data_ptr(), batch,
                                          yb.data_ptr(), 1, 0), "batched")
    ys = torch.full((batch, N), float("nan"), device=cuda)
    for b0 in range(0, batch, 4):
        nb = min(4, batch - b0)
        forge.check(lib.forge_gemv_w4a16_g128(tiles.data_ptr(), stiles.data_ptr(), N, K, xd[b0:].data_ptr(), nb,
                                              ys[b0:].data_ptr(), 1, 0), "grouped")
    torch.cuda.synchronize()
    forge.check(lib.forge_ops_check(), "error word")
    assert not torch.isnan(yb).any()
    err = (yb - ys).abs().max().item()
    assert err <= 1e-5 * ys.abs().max().item(), err


def test_gemv_int4_batched_tensor_core_every_batch(cuda):
    """The tensor-core int4 path (tcgen05 kind::i8) normally takes chunks of
    >= 24 sequences; with FORGE_GEMV_TC_MIN_SEQ=1 it takes every batched
    chunk, so its N = 16 / 32 / 48 shapes and split tiles are checked against
    the small-batch path too (in a child process: the threshold is read once)."""
    import os
    import subprocess
    import sys
    env = dict(os.environ, FORGE_GEMV_TC_MIN_SEQ="1")
    here = os.path.dirname(os.path.abspath(__file__))
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", os.path.join(here, "test_gpu_ops.py"), "-k",
                        "int4_batched_matches_small_batch"], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


@pytest.mark.parametrize("N,K", [(2048, 2048), (32000, 2048), (8192, 688)])
@pytest.mark.parametrize("batch", [5, 9, 16, 32, 33])
def test_gemv_bf16_batched_bit_identical(forge, oracle, cuda, N, K, batch):
    """bf16 weights with bf16 activations above 4 sequences: one weight stream
    per 32 sequences, the same bits as the small-batch path on slices of 4."""
    import torch
    if K % 16:
        pytest.skip("shape")
    rng = np.random.default_rng(N + K + batch)
    w = oracle.fill_normal_bf16(N * K, 4, N + 7 * K, 0.02).reshape(N, K)
    X = rng.standard_normal((batch, K)).astype(np.float32)
    tiles = forge.bf16_pack(_dev_bf16(torch, w, cuda))
    xd = torch.from_numpy(X).to(cuda)
    lib = forge.lib()
    yb = torch.full((batch, N), float("nan"), device=cuda)
    forge.check(lib.forge_gemv_bf16(tiles.data_ptr(), N, K, xd.data_ptr(), batch, yb.data_ptr(), 0, 0), "batched")
    ys = torch.full((batch, N), float("nan"), device=cuda)
    for b0 in range(0, batch, 4):
        nb = min(4, batch - b0)
        forge.check(lib.forge_gemv_bf16(tiles.data_ptr(), N, K, xd[b0:].data_ptr(), nb, ys[b0:].data_ptr(), 0, 0),
                    "grouped")
    torch.cuda.synchronize()
    forge.check(lib.forge_ops_check(), "error word")
    assert torch.equal(yb.view(torch.int32), ys.view(torch.int32))
