"""The allocation-free flash-decode entry, for callers that cannot allocate
device memory (their device memory belongs to another allocator, they run
during stream capture, or their memory budget is fixed).

forge_flash_decode_noalloc takes the same inputs and outputs as
forge_flash_decode but keeps its scratch in a fixed library-owned device
array instead of a caller workspace. Checked through the C ABI against the
workspace entry on two calls in a row (the array keeps the previous call's
contents), for the clean rejection of shapes above its fixed size, and for
its error word: a position outside the cache is reported once by
forge_flash_decode_noalloc_status (and by no other error word) and then
reads clean. This file is collected last so that a failure here leaves
every other test run.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _inputs(oracle, B, H, Hkv, hd, lmax, pos, seed):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, H * hd)).astype(np.float32)
    Kb = oracle.f32_to_bf16(rng.standard_normal((B, Hkv, lmax, hd)).astype(np.float32) * 0.5)
    Vb = oracle.f32_to_bf16(rng.standard_normal((B, Hkv, lmax, hd)).astype(np.float32))
    return q, Kb, Vb, np.asarray(pos, np.int32)


@pytest.mark.parametrize("B,H,Hkv,hd,lmax,pos", [
    (1, 32, 32, 128, 2304, [2047]),
    (2, 8, 2, 64, 1100, [1023, 5]),
    (4, 16, 4, 128, 4200, [4100, 3000, 17, 1]),
])
def test_noalloc_matches_workspace_entry(forge, oracle, cuda, B, H, Hkv, hd, lmax, pos):
    import torch
    lib = forge.lib()
    need = lib.forge_flash_decode_workspace_bytes(B, H, Hkv, hd, lmax)
    assert 0 < need <= lib.forge_flash_decode_noalloc_capacity()
    q, Kb, Vb, p = _inputs(oracle, B, H, Hkv, hd, lmax, pos, seed=B * 31 + H)
    qd = torch.from_numpy(q).to(cuda)
    kd = torch.from_numpy(Kb.view(np.int16)).to(cuda)
    vd = torch.from_numpy(Vb.view(np.int16)).to(cuda)
    pd = torch.from_numpy(p).to(cuda)
    stream = torch.cuda.current_stream().cuda_stream

    ws = torch.zeros(need, dtype=torch.uint8, device=cuda)
    ref = torch.full((B, H * hd), float("nan"), device=cuda)
    forge.check(lib.forge_flash_decode(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), pd.data_ptr(), B, H, Hkv, hd,
                                       lmax, ref.data_ptr(), ws.data_ptr(), stream), "workspace entry")
    torch.cuda.synchronize()
    forge.check(lib.forge_ops_check(), "workspace entry error word")
    ref_h = ref.cpu().numpy()
    assert np.isfinite(ref_h).all()

    for call in range(2):  # the second call starts from the first call's scratch contents
        out = torch.full((B, H * hd), float("nan"), device=cuda)
        forge.check(lib.forge_flash_decode_noalloc(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), pd.data_ptr(), B, H,
                                                   Hkv, hd, lmax, out.data_ptr(), stream), f"no-alloc call {call}")
        torch.cuda.synchronize()
        forge.check(lib.forge_flash_decode_noalloc_status(), f"no-alloc call {call} error word")
        got = out.cpu().numpy()
        # same kernel and split plan: the tolerance of the flash-decode tests
        assert np.abs(got - ref_h).max() <= 2e-5 * max(1.0, np.abs(ref_h).max()), (call, np.abs(got - ref_h).max())


def test_noalloc_rejects_shapes_above_capacity(forge, cuda):
    import torch
    lib = forge.lib()
    B, H, Hkv, hd, lmax = 256, 64, 64, 128, 8192
    assert lib.forge_flash_decode_workspace_bytes(B, H, Hkv, hd, lmax) > lib.forge_flash_decode_noalloc_capacity()
    tiny = torch.zeros(16, dtype=torch.float32, device=cuda)
    rc = lib.forge_flash_decode_noalloc(tiny.data_ptr(), tiny.data_ptr(), tiny.data_ptr(), tiny.data_ptr(), B, H, Hkv,
                                        hd, lmax, tiny.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc != 0
    assert b"scratch bytes" in lib.forge_b200_last_error()


def test_noalloc_error_word_reports_once_and_clears(forge, oracle, cuda):
    """A position outside the cache: the kernel's bounds check skips the
    sequence and records the error in the entry's own word; the status call
    returns the failure once, then reads clean. The per-op error word of the
    rest of the library does not see it."""
    import torch
    lib = forge.lib()
    B, H, Hkv, hd, lmax = 2, 8, 2, 64, 256
    q, Kb, Vb, _ = _inputs(oracle, B, H, Hkv, hd, lmax, [0, 0], seed=11)
    qd = torch.from_numpy(q).to(cuda)
    kd = torch.from_numpy(Kb.view(np.int16)).to(cuda)
    vd = torch.from_numpy(Vb.view(np.int16)).to(cuda)
    stream = torch.cuda.current_stream().cuda_stream
    torch.cuda.synchronize()
    lib.forge_ops_check()                   # start from clean words
    lib.forge_flash_decode_noalloc_status()
    bad = torch.tensor([10, lmax], dtype=torch.int32, device=cuda)  # sequence 1 past the cache
    out = torch.zeros((B, H * hd), device=cuda)
    forge.check(lib.forge_flash_decode_noalloc(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), bad.data_ptr(), B, H,
                                               Hkv, hd, lmax, out.data_ptr(), stream), "launch")
    assert lib.forge_flash_decode_noalloc_status() != 0
    assert b"error word" in lib.forge_b200_last_error()
    assert lib.forge_flash_decode_noalloc_status() == 0   # cleared by the read
    assert lib.forge_ops_check() == 0                     # never reported elsewhere
    good = torch.tensor([10, 200], dtype=torch.int32, device=cuda)
    forge.check(lib.forge_flash_decode_noalloc(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), good.data_ptr(), B, H,
                                               Hkv, hd, lmax, out.data_ptr(), stream), "launch after the error")
    forge.check(lib.forge_flash_decode_noalloc_status(), "clean call after the error")
