"""Paged flash-decode on the B200 (forge_flash_decode_paged): pages handed out
by the host allocator (interleaved across sequences, some released and
re-used, so each sequence's pages are scattered over the pool) hold the same
K/V rows as a contiguous cache; the paged result must equal forge_flash_decode
on the contiguous cache bit for bit. A page id outside the pool sets the
error word."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _pool(forge, rng, B, max_pages, num_pages):
    a = forge.PagedKv(num_pages, 16, 64)
    for j in range(max_pages):
        for b in rng.permutation(B):
            a.alloc_page(int(b))
        if j % 3 == 1:  # a released page goes to the next allocation
            t = a.page_table(int(B - 1))
            a.release_page(int(B - 1), t[-1])
            a.alloc_page(int(B - 1))
    return np.array([a.page_table(b) for b in range(B)], np.int32)


@pytest.mark.parametrize("hd,H,Hkv,pt,pos", [(128, 8, 2, 16, [0, 100, 255, 17]), (64, 4, 4, 32, [31, 32, 200, 255]),
                                             (128, 32, 8, 16, [2047, 1500, 16, 1023])])
def test_paged_equals_contiguous(forge, oracle, cuda, hd, H, Hkv, pt, pos):
    import torch
    rng = np.random.default_rng(hd + H + pt)
    B = len(pos)
    lmax = max(pos) + 1
    lmax = (lmax + pt - 1) // pt * pt
    max_pages = lmax // pt
    num_pages = B * max_pages + 7
    table = _pool(forge, rng, B, max_pages, num_pages)
    assert sorted(set(table.ravel().tolist())) == sorted(table.ravel().tolist())  # no page twice
    K = oracle.f32_to_bf16((rng.standard_normal((B, Hkv, lmax, hd)) * 0.5).astype(np.float32))
    V = oracle.f32_to_bf16(rng.standard_normal((B, Hkv, lmax, hd)).astype(np.float32))
    kpool = np.zeros((num_pages, Hkv, pt, hd), np.uint16)
    vpool = np.zeros_like(kpool)
    for b in range(B):
        for j in range(max_pages):
            kpool[table[b, j]] = K[b, :, j * pt:(j + 1) * pt]
            vpool[table[b, j]] = V[b, :, j * pt:(j + 1) * pt]
    q = rng.standard_normal((B, H * hd)).astype(np.float32)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(cuda)
    qd, kd, vd, kp, vp = torch.from_numpy(q).to(cuda), dev(K), dev(V), dev(kpool), dev(vpool)
    td = torch.from_numpy(table).to(cuda)
    pd = torch.tensor(pos, dtype=torch.int32, device=cuda)
    ws_bytes = forge.lib().forge_flash_decode_workspace_bytes(B, H, Hkv, hd, lmax)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=cuda)
    out_c = torch.full((B, H * hd), float("nan"), device=cuda)
    out_p = torch.full((B, H * hd), float("nan"), device=cuda)
    L = forge.lib()
    forge.check(L.forge_flash_decode(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), pd.data_ptr(), B, H, Hkv, hd, lmax,
                                     out_c.data_ptr(), ws.data_ptr(), None), "contiguous")
    forge.check(L.forge_flash_decode_paged(qd.data_ptr(), kp.data_ptr(), vp.data_ptr(), num_pages, td.data_ptr(),
                                           max_pages, pt, pd.data_ptr(), B, H, Hkv, hd, out_p.data_ptr(),
                                           ws.data_ptr(), None), "paged")
    torch.cuda.synchronize()
    forge.check(L.forge_ops_check(), "error word")
    assert torch.equal(out_c, out_p)
    assert not torch.isnan(out_p).any()

    # a page id outside the pool: the error word is set, the sequence is not written
    bad = table.copy()
    bad[1, 0] = num_pages + 5
    out_b = torch.full((B, H * hd), float("nan"), device=cuda)
    forge.check(L.forge_flash_decode_paged(qd.data_ptr(), kp.data_ptr(), vp.data_ptr(), num_pages,
                                           torch.from_numpy(bad).to(cuda).data_ptr(), max_pages, pt, pd.data_ptr(), B,
                                           H, Hkv, hd, out_b.data_ptr(), ws.data_ptr(), None), "paged bad")
    torch.cuda.synchronize()
    with pytest.raises(forge.ForgeError, match="error word"):
        forge.check(L.forge_ops_check(), "error word")
    assert torch.isnan(out_b[1]).all()
    assert torch.equal(out_b[0], out_c[0]) and torch.equal(out_b[2], out_c[2])
