"""The device sampler (forge_sample, and forge_b200_decode_step_sampled in the
decode engine) against the oracle's restatement of
self/ml/gpu_sampler.hexa: the same tokens and RNG states for every row and
configuration, the final distribution equal up to f32 rounding flips (the
device sums in parallel, the reference left to right, both in f64)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# (temperature, top_k, top_p): greedy, gpu_sampler_default, plain, top-k
# only, top-p only, both, wide top-k
CASES = [(0.0, 0, 1.0), (0.7, 40, 0.9), (1.0, 0, 1.0), (0.5, 5, 1.0), (1.3, 0, 0.8), (0.9, 17, 0.5),
         (2.0, 1000, 0.95)]


def _run(forge, torch, logits, t, k, p, states):
    dev = torch.device("cuda:0")
    B, V = logits.shape
    lg = torch.from_numpy(logits).to(dev)
    st = torch.from_numpy(states.copy()).to(dev)
    probs = torch.zeros(B, V, dtype=torch.float32, device=dev)
    tok = torch.zeros(B, dtype=torch.int32, device=dev)
    forge.check(forge.lib().forge_sample(lg.data_ptr(), V, B, V, t, k, p, st.data_ptr(), probs.data_ptr(),
                                         tok.data_ptr(), None), "forge_sample")
    torch.cuda.synchronize()
    return tok.cpu().numpy(), st.cpu().numpy(), probs.cpu().numpy()


@pytest.mark.parametrize("V", [1000, 32000])
@pytest.mark.parametrize("case", CASES, ids=[f"t{c[0]}_k{c[1]}_p{c[2]}" for c in CASES])
def test_sampler_matches_oracle(forge, oracle, cuda, V, case):
    import torch
    t, k, p = case
    rng = np.random.default_rng(V + int(100 * t) + k)
    B = 8
    states = np.array([42, 2463534242, 7, 123456789, 99, 1 << 40, 5, 31337], np.int64)
    for trial in range(3):
        logits = (rng.standard_normal((B, V)) * rng.uniform(1, 8, (B, 1))).astype(np.float32)
        tok, st, probs = _run(forge, torch, logits, t, k, p, states)
        for b in range(B):
            ot, os_, op = oracle.sample_token(logits[b], t, k, p, int(states[b]))
            assert tok[b] == ot, (trial, b, tok[b], ot)
            if t > 0:
                assert st[b] == os_
                assert np.abs(probs[b] - op).max() <= 1e-6 * op.max(), np.abs(probs[b] - op).max()
        states = st if t > 0 else states


def test_sampler_ties_and_edges(forge, oracle, cuda):
    """Integer logits (many equal probabilities): top-k keeps every entry equal
    to the k-th largest, greedy takes the first maximum."""
    import torch
    rng = np.random.default_rng(5)
    B, V = 4, 4096
    logits = np.round(rng.standard_normal((B, V)) * 2).astype(np.float32)
    states = np.array([1, 2, 3, 4], np.int64)
    for t, k in [(0.0, 0), (1.0, 3), (0.8, 50), (1.0, 0)]:
        tok, st, probs = _run(forge, torch, logits, t, k, 1.0, states)
        for b in range(B):
            ot, os_, op = oracle.sample_token(logits[b], t, k, 1.0, int(states[b]))
            assert tok[b] == ot
            if t > 0:
                assert st[b] == os_ and np.abs(probs[b] - op).max() <= 1e-6 * op.max()


def test_engine_sampled_step(forge, oracle, cuda):
    """decode_step_sampled draws from the step's own logits."""
    m = forge.ForgeModel(2, 256, 4, 2, 64, 512, 3000, weight_kind=forge.FORGE_WEIGHT_BF16, max_batch=3, max_ctx=16)
    m.init_synthetic(7, 0.05)
    toks = np.array([5, 60, 700], np.int32)
    for t, k, p in [(0.7, 40, 0.9), (1.0, 0, 1.0), (0.0, 0, 1.0)]:
        m.reset()
        _, lg = m.step(toks, want_logits=True)
        m.reset()
        states = np.array([42, 43, 44], np.int64)
        want = [oracle.sample_token(lg[b], t, k, p, int(states[b]))[:2] for b in range(3)]
        nxt = m.step_sampled(toks, states, t, k, p)
        assert [int(x) for x in nxt] == [w[0] for w in want]
        if t > 0:
            assert [int(s) for s in states] == [w[1] for w in want]
    m.close()
