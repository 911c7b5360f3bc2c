"""The sampler oracle (or_sample_token, a C restatement of
self/ml/gpu_sampler.hexa) against a second, line-by-line Python
transcription of the same hexa code (Python floats are f64 like hexa's,
np.float32 stands for write_f32, ints wrap at 64 bits as the compiled
runtime's int64 does). The reference has no sampler tests or golden vectors,
so this pins the restatement to the hexa text, not to reference outputs."""
import math

import numpy as np
import pytest

M64 = (1 << 64) - 1


def _s64(v):
    v &= M64
    return v - (1 << 64) if v >> 63 else v


def _tdiv(a, b):  # C division: truncation toward zero
    q = abs(a) // abs(b)
    return q if (a >= 0) == (b >= 0) else -q


def _rand(state):  # gpu_sampler.hexa:57-65
    x = state
    x = _s64(x ^ _s64(x * 8192))
    x = _s64(x ^ _tdiv(x, 131072))
    x = _s64(x ^ _s64(x * 32))
    if x < 0:
        x = _s64(0 - x)
    r = math.fmod(x, 1000000) if x < 0 else x % 1000000
    return x, float(int(r)) / 1000000.0


f32 = lambda v: float(np.float32(v))


def _sample(logits, temperature, top_k, top_p, state):  # gpu_sampler.hexa:89-277
    vocab = len(logits)
    host = [float(v) for v in np.asarray(logits, np.float32)]
    if temperature <= 0.0:
        best_i, best_v = 0, host[0]
        for i in range(1, vocab):
            if host[i] > best_v:
                best_v, best_i = host[i], i
        return best_i, state, None
    inv_t = 1.0 / temperature
    host = [f32(v * inv_t) for v in host]
    mx = host[0]
    for v in host[1:]:
        if v > mx:
            mx = v
    sum_e = 0.0
    for i in range(vocab):
        e = math.exp(host[i] - mx)
        host[i] = f32(e)
        sum_e = sum_e + e
    inv_sum = 1.0 / sum_e
    host = [f32(v * inv_sum) for v in host]
    if 0 < top_k < vocab:
        sb = list(host)
        for j in range(top_k):
            best = j
            for m in range(j + 1, vocab):
                if sb[m] > sb[best]:
                    best = m
            if best != j:
                sb[j], sb[best] = sb[best], sb[j]
        thr = sb[top_k - 1]
        sum_k = 0.0
        for i in range(vocab):
            if host[i] < thr:
                host[i] = 0.0
            else:
                sum_k = sum_k + host[i]
        if sum_k > 0.0:
            inv_k = 1.0 / sum_k
            host = [f32(v * inv_k) for v in host]
    if 0.0 < top_p < 1.0:
        idx = [i for i in range(vocab) if host[i] > 0.0]
        val = [host[i] for i in idx]
        nn = len(idx)
        for ii in range(nn):
            best = ii
            for jj in range(ii + 1, nn):
                if val[jj] > val[best]:
                    best = jj
            if best != ii:
                idx[ii], idx[best] = idx[best], idx[ii]
                val[ii], val[best] = val[best], val[ii]
        host = [0.0] * vocab
        cum = sum_p = 0.0
        done = False
        for i in range(nn):
            if not done:
                host[idx[i]] = f32(val[i])
                sum_p = sum_p + val[i]
                cum = cum + val[i]
                if cum >= top_p:
                    done = True
        if sum_p > 0.0:
            inv_p = 1.0 / sum_p
            host = [f32(v * inv_p) for v in host]
    state, r = _rand(state)
    cum, chosen = 0.0, vocab - 1
    for i in range(vocab):
        cum = cum + host[i]
        if cum > r:
            chosen = i
            break
    return chosen, state, np.array(host, np.float32)


def test_rng_sequence_matches_transcription(oracle):
    import ctypes as C
    for seed in (2463534242, 42, 1, 123456789, (1 << 62) + 12345):
        s_py, st = seed, C.c_int64(seed)
        for _ in range(200):
            s_py, r_py = _rand(s_py)
            r_c = oracle.lib().or_sampler_rand(C.byref(st))
            assert st.value == s_py and r_c == r_py


CASES = [(0.0, 0, 1.0), (0.7, 40, 0.9), (1.0, 0, 1.0), (0.5, 5, 1.0), (1.3, 0, 0.8), (0.9, 17, 0.5), (2.0, 200, 0.95)]


@pytest.mark.parametrize("temperature,top_k,top_p", CASES)
def test_sampler_matches_transcription(oracle, temperature, top_k, top_p):
    rng = np.random.default_rng(11)
    state = 42
    for trial in range(12):
        V = int(rng.integers(2, 300))
        logits = (rng.standard_normal(V) * rng.uniform(0.5, 6)).astype(np.float32)
        if trial % 4 == 3:  # ties
            logits = np.round(logits).astype(np.float32)
        t_c, s_c, p_c = oracle.sample_token(logits, temperature, top_k, top_p, state)
        t_p, s_p, p_p = _sample(logits, temperature, top_k, top_p, state)
        assert (t_c, s_c) == (t_p, s_p)
        if p_p is not None:
            assert np.array_equal(p_c, p_p)
        state = s_c


def test_sampler_edge_cases(oracle):
    # greedy: first maximum
    assert oracle.sample_token(np.array([1, 3, 3, 2], np.float32), 0.0, 0, 1.0, 7)[:2] == (1, 7)
    # a single allowed token (top_k 1) is always drawn; the state still advances
    t, s, p = oracle.sample_token(np.array([0.1, 2.0, -1.0], np.float32), 1.0, 1, 1.0, 42)
    assert t == 1 and s != 42 and p.tolist() == [0.0, 1.0, 0.0]
    # top-k ties keep every entry equal to the k-th largest
    _, _, p = oracle.sample_token(np.array([1, 1, 1, 0], np.float32), 1.0, 2, 1.0, 42)
    assert (p[:3] > 0).all() and p[3] == 0
