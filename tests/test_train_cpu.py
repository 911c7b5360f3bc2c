"""The oracle's restatement of the training-side forge families (float64,
self/cuda/runtime_cuda_emit.hexa) checked on the CPU against mathematics:
flame's series exp against libm, backward kernels against finite
differences of their forward kernels, RoPE as an orthogonal map whose
backward is its transpose, and one AdamW step worked by hand."""
import math

import numpy as np
import pytest


def P(a):
    return a.ctypes.data


def test_dt_exp_close_to_libm(oracle):
    L = oracle.lib()
    for x in np.linspace(-30, 30, 241):
        assert abs(L.or_dt_exp(float(x)) - math.exp(x)) <= 1e-13 * math.exp(x)
    assert L.or_dt_exp(0.0) == 1.0
    assert abs(L.or_attn_scale(64) - 0.125) < 1e-16 and abs(L.or_attn_scale(128) - 1 / math.sqrt(128)) < 1e-16


def _rms(oracle, x, C):
    y = np.empty_like(x)
    oracle.lib().or_train_rmsnorm_rows(P(x), x.size // C, C, 1e-6, P(y))
    return y


def test_rmsnorm_bwd_is_the_vjp(oracle):
    rng = np.random.default_rng(1)
    R, C = 3, 40
    x = rng.standard_normal((R, C))
    dy = rng.standard_normal((R, C))
    dx = np.empty_like(x)
    oracle.lib().or_train_rmsnorm_bwd_rows(P(x), P(dy), R, C, P(dx))
    h = 1e-6
    for r, c in [(0, 0), (1, 17), (2, 39)]:
        xp, xm = x.copy(), x.copy()
        xp[r, c] += h
        xm[r, c] -= h
        num = ((_rms(oracle, xp, C) - _rms(oracle, xm, C)) * dy).sum() / (2 * h)
        assert abs(num - dx[r, c]) < 1e-7, (num, dx[r, c])


def test_rope_orthogonal_and_bwd_is_transpose(oracle):
    L = oracle.lib()
    rng = np.random.default_rng(2)
    T, nh, hd = 5, 3, 8
    ang = rng.uniform(0, 2 * np.pi, (T, hd // 2))
    c = np.concatenate([np.cos(ang), np.cos(ang)], 1).copy()
    s = np.concatenate([np.sin(ang), np.sin(ang)], 1).copy()
    x = rng.standard_normal((T, nh, hd))
    y = rng.standard_normal((T, nh, hd))
    rx, rty = np.empty_like(x), np.empty_like(y)
    L.or_train_rope(P(x), P(c), P(s), T, nh, hd, 0, P(rx))
    L.or_train_rope(P(y), P(c), P(s), T, nh, hd, 1, P(rty))
    assert abs(np.linalg.norm(rx) - np.linalg.norm(x)) < 1e-12            # R^T R = I
    assert abs((rx * y).sum() - (x * rty).sum()) < 1e-12                  # <Rx, y> = <x, R^T y>


def test_adamw_one_step_by_hand(oracle):
    w = np.array([1.0, -2.0, 0.5])
    m = np.array([0.1, 0.0, -0.2])
    v = np.array([0.01, 0.0, 0.04])
    g = np.array([0.3, -0.1, 0.0])
    out = np.empty(3)
    lr, b1, b2, eps, wd, t = 1e-3, 0.9, 0.999, 1e-8, 0.01, 3
    mm, vv = m.copy(), v.copy()
    oracle.lib().or_train_adamw(P(w), P(mm), P(vv), P(g), 3, lr, b1, b2, eps, wd, t, P(out))
    em = b1 * m + (1 - b1) * g
    ev = b2 * v + (1 - b2) * g * g
    ew = w - lr * wd * w - lr * (em / (1 - b1 ** t)) / (np.sqrt(ev / (1 - b2 ** t)) + eps)
    assert np.allclose(mm, em, rtol=0, atol=1e-15) and np.allclose(vv, ev, rtol=0, atol=1e-15)
    assert np.allclose(out, ew, rtol=1e-14, atol=0)


def test_attention_bwd_is_the_vjp(oracle):
    L = oracle.lib()
    rng = np.random.default_rng(3)
    T, nh, nkv, hd = 4, 4, 2, 8
    q = rng.standard_normal((T, nh, hd))
    k = rng.standard_normal((T, nkv, hd))
    v = rng.standard_normal((T, nkv, hd))
    dctx = rng.standard_normal((T, nh * hd))

    def fwd(q, k, v):
        p = np.empty((nh, T, T))
        ctx = np.empty((T, nh * hd))
        L.or_train_attn_fwd(P(q), P(k), P(v), T, nh, nkv, hd, P(p), P(ctx))
        return p, ctx

    p, ctx = fwd(q, k, v)
    # causal softmax rows sum to one, zero above the diagonal
    assert np.allclose(p.sum(-1), 1.0) and np.all(p[:, np.triu_indices(T, 1)[0], np.triu_indices(T, 1)[1]] == 0)
    dq, dk, dv = np.empty_like(q), np.empty_like(k), np.empty_like(v)
    L.or_train_attn_bwd(P(q), P(k), P(v), P(p), P(dctx), T, nh, nkv, hd, P(dq), P(dk), P(dv))
    h = 1e-6
    for arr, grad, idx in [(q, dq, (2, 3, 5)), (k, dk, (1, 1, 0)), (v, dv, (0, 0, 7)), (k, dk, (3, 0, 2))]:
        a, b = arr.copy(), arr.copy()
        a[idx] += h
        b[idx] -= h
        args_a = [a if arr is x else x for x in (q, k, v)]
        args_b = [b if arr is x else x for x in (q, k, v)]
        num = ((fwd(*args_a)[1] - fwd(*args_b)[1]) * dctx).sum() / (2 * h)
        assert abs(num - grad[idx]) < 1e-6, (idx, num, grad[idx])
