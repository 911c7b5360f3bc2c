"""The training-side forge families on the B200 (train.cu, float64) against
the oracle's restatement of the reference kernels
(self/cuda/runtime_cuda_emit.hexa), through the C ABI. The kernels keep the
reference's order of operations per output, so RoPE, AdamW, the SiLU gate
(flame's series exp) and attention forward / backward (GQA, causal, P kept)
must equal the oracle bit for bit; RMSNorm's row reductions are block trees
(last-bit differences, bound 1e-14 relative) and SiLU / its derivative use
the device's exp against libm's (bound 4e-15 relative)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def P(a):
    return a.ctypes.data


def _dev(torch, cuda, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def test_elementwise_families(forge, oracle, cuda):
    import torch
    L, O = forge.lib(), oracle.lib()
    rng = np.random.default_rng(11)
    n = 100003
    w = rng.standard_normal(n)
    m = rng.standard_normal(n) * 0.1
    v = rng.random(n) * 0.01
    g = rng.standard_normal(n)
    args = (1e-3, 0.9, 0.999, 1e-8, 0.01, 7)
    ow, om, ov = np.empty(n), m.copy(), v.copy()
    O.or_train_adamw(P(w), P(om), P(ov), P(g), n, *args, P(ow))
    dw, dm, dv, dg = (_dev(torch, cuda, a) for a in (w, m, v, g))
    forge.check(L.forge_train_adamw_step(dw.data_ptr(), dm.data_ptr(), dv.data_ptr(), dg.data_ptr(), n, *args,
                                         dw.data_ptr(), 0), "adamw in place")
    torch.cuda.synchronize()
    assert np.array_equal(dw.cpu().numpy(), ow) and np.array_equal(dm.cpu().numpy(), om)
    assert np.array_equal(dv.cpu().numpy(), ov)

    T, nh, hd = 37, 6, 64
    ang = rng.uniform(0, 6.3, (T, hd // 2))
    c = np.concatenate([np.cos(ang)] * 2, 1)
    s = np.concatenate([np.sin(ang)] * 2, 1)
    x = rng.standard_normal((T, nh, hd))
    for bwd in (0, 1):
        ref = np.empty_like(x)
        O.or_train_rope(P(x), P(c), P(s), T, nh, hd, bwd, P(ref))
        dx, dc, ds = (_dev(torch, cuda, a) for a in (x, c, s))
        out = torch.empty_like(dx)
        forge.check(L.forge_train_rope(dx.data_ptr(), dc.data_ptr(), ds.data_ptr(), T, nh, hd, bwd, out.data_ptr(), 0),
                    "rope")
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), ref), bwd

    a = rng.standard_normal(n) * 6
    b = rng.standard_normal(n)
    da, db = _dev(torch, cuda, a), _dev(torch, cuda, b)
    for mode in (0, 1, 2):
        ref = np.empty(n)
        O.or_train_silu(P(a), P(b), n, mode, P(ref))
        out = torch.empty_like(da)
        forge.check(L.forge_train_silu(da.data_ptr(), db.data_ptr(), n, mode, out.data_ptr(), 0), "silu")
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        if mode == 2:
            assert np.array_equal(got, ref)
        else:
            # the device's exp against libm's, and the compiler's contraction of
            # s * (1 + x * (1 - s)): a few ulp
            assert np.abs(got - ref).max() <= 4e-15 * max(1.0, np.abs(ref).max())


@pytest.mark.parametrize("R,C", [(7, 768), (3, 4096), (129, 100)])
def test_rmsnorm_rows_and_bwd(forge, oracle, cuda, R, C):
    import torch
    L, O = forge.lib(), oracle.lib()
    rng = np.random.default_rng(R * C)
    x = rng.standard_normal((R, C))
    dy = rng.standard_normal((R, C))
    ref, refb = np.empty_like(x), np.empty_like(x)
    O.or_train_rmsnorm_rows(P(x), R, C, 1e-5, P(ref))
    O.or_train_rmsnorm_bwd_rows(P(x), P(dy), R, C, P(refb))
    dx, ddy = _dev(torch, cuda, x), _dev(torch, cuda, dy)
    y, gx = torch.empty_like(dx), torch.empty_like(dx)
    forge.check(L.forge_train_rmsnorm_rows(dx.data_ptr(), R, C, 1e-5, y.data_ptr(), 0), "rmsnorm")
    forge.check(L.forge_train_rmsnorm_bwd_rows(dx.data_ptr(), ddy.data_ptr(), R, C, gx.data_ptr(), 0), "rmsnorm bwd")
    torch.cuda.synchronize()
    assert np.abs(y.cpu().numpy() - ref).max() <= 1e-14 * np.abs(ref).max()
    assert np.abs(gx.cpu().numpy() - refb).max() <= 1e-13 * np.abs(refb).max()


@pytest.mark.parametrize("T,nh,nkv,hd", [(1, 2, 2, 8), (33, 4, 4, 64), (70, 8, 2, 64), (48, 4, 1, 128)])
def test_attention_fwd_bwd_bit_exact(forge, oracle, cuda, T, nh, nkv, hd):
    import torch
    L, O = forge.lib(), oracle.lib()
    rng = np.random.default_rng(T + nh + hd)
    q = rng.standard_normal((T, nh, hd))
    k = rng.standard_normal((T, nkv, hd))
    v = rng.standard_normal((T, nkv, hd))
    dctx = rng.standard_normal((T, nh * hd))
    p, ctx = np.empty((nh, T, T)), np.empty((T, nh * hd))
    O.or_train_attn_fwd(P(q), P(k), P(v), T, nh, nkv, hd, P(p), P(ctx))
    dq, dk, dv = np.empty_like(q), np.empty_like(k), np.empty_like(v)
    O.or_train_attn_bwd(P(q), P(k), P(v), P(p), P(dctx), T, nh, nkv, hd, P(dq), P(dk), P(dv))
    Q, K, V, D = (_dev(torch, cuda, a) for a in (q, k, v, dctx))
    Pd = torch.empty((nh, T, T), dtype=torch.float64, device=cuda)
    Cd = torch.empty((T, nh * hd), dtype=torch.float64, device=cuda)
    forge.check(L.forge_train_attn_fwd(Q.data_ptr(), K.data_ptr(), V.data_ptr(), T, nh, nkv, hd, Pd.data_ptr(),
                                       Cd.data_ptr(), 0), "attn fwd")
    dQ, dK, dV = torch.empty_like(Q), torch.empty_like(K), torch.empty_like(V)
    scratch = torch.empty((nh, T, T), dtype=torch.float64, device=cuda)
    forge.check(L.forge_train_attn_bwd(Q.data_ptr(), K.data_ptr(), V.data_ptr(), Pd.data_ptr(), D.data_ptr(), T, nh,
                                       nkv, hd, dQ.data_ptr(), dK.data_ptr(), dV.data_ptr(), scratch.data_ptr(), 0),
                "attn bwd")
    torch.cuda.synchronize()
    assert np.array_equal(Pd.cpu().numpy(), p) and np.array_equal(Cd.cpu().numpy(), ctx)
    assert np.array_equal(dQ.cpu().numpy(), dq)
    assert np.array_equal(dK.cpu().numpy(), dk) and np.array_equal(dV.cpu().numpy(), dv)
