"""Flash-attention prefill on the tcgen05 tensor cores against a PyTorch
fp32 reference of the same op: O = softmax(Q K^T / sqrt(hd) + causal mask) V
(head dim 128 and 64)
(nn_attn_core_fwd, stdlib/flame/nn_lib.hexa:221-278), bf16 inputs ~ N(0, 1).

Tolerance: the kernel rounds P to bf16 before P V and O to bf16 on output,
so against the fp32 reference the bar is max |err| <= 2e-2 and mean |err| <=
2e-3. The first case is a single CTA, so a broken kernel fails in one short
launch before the larger grids run."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ref(torch, q, k, v, causal):
    qf, kf, vf = q.float(), k.float(), v.float()
    s = qf @ kf.transpose(-1, -2) / np.sqrt(q.shape[-1])
    if causal:
        S = q.shape[-2]
        mask = torch.triu(torch.ones(S, S, dtype=torch.bool, device=q.device), 1)
        s = s.masked_fill(mask, float("-inf"))
    return torch.softmax(s, -1) @ vf


@pytest.mark.parametrize("B,H,S,causal,hd", [
    (1, 1, 128, True, 128),
    (1, 1, 128, False, 128),
    (1, 2, 256, True, 128),
    (1, 2, 512, False, 128),
    (2, 3, 1024, True, 128),
    (1, 1, 128, True, 64),
    (1, 2, 384, False, 64),
    (2, 4, 1024, True, 64),
])
def test_flash_prefill(forge, cuda, B, H, S, causal, hd):
    import torch
    g = torch.Generator(device=cuda).manual_seed(B * 100 + H * 10 + S + causal + hd)
    q, k, v = (torch.randn(B, H, S, hd, generator=g, device=cuda).to(torch.bfloat16) for _ in range(3))
    o = torch.full_like(q, float("nan"))
    torch.cuda.synchronize()
    forge.check(forge.lib().forge_flash_prefill(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B, H, S, hd,
                                                int(causal), torch.cuda.current_stream().cuda_stream), "prefill")
    torch.cuda.synchronize()
    forge.check(forge.lib().forge_ops_check(), "prefill error word")
    ref = _ref(torch, q, k, v, causal)
    err = (o.float() - ref).abs()
    assert torch.isfinite(o.float()).all()
    assert err.max().item() <= 2e-2, err.max().item()
    assert err.mean().item() <= 2e-3, err.mean().item()


def test_flash_prefill_dispatch_family(forge, cuda):
    """FLASH_PREFILL through forge_tier_dispatch_v2 on HexaFarrBf16 slots."""
    import ctypes as C
    import torch
    F = forge
    L = F.lib()
    B, H, S = 1, 2, 256
    g = torch.Generator().manual_seed(5)
    arrs = [torch.randn(B, H, S, 128, generator=g).to(torch.bfloat16) for _ in range(3)]
    descs = []
    for a in arrs:
        d = L.hexa_farr_bf16_alloc(a.numel())
        C.memmove(d.contents.h_buf, a.view(torch.int16).numpy().ctypes.data, a.numel() * 2)
        descs.append(d)
    out = L.hexa_farr_bf16_alloc(B * H * S * 128)
    shape = F.ForgeShapeInfo(B, H, 128, S)
    ins, outs = F.forge_args(*descs, 1), F.forge_args(out)
    rc = L.forge_tier_dispatch_v2(F.FORGE_KERNEL_FLASH_PREFILL, C.byref(shape), 0, F.FORGE_PREC_PURE_BF16, 0,
                                  C.byref(ins), C.byref(outs))
    assert rc == F.FORGE_OK
    F.check(L.hexa_farr_bf16_to_host(out), "to_host")
    got = np.ctypeslib.as_array(C.cast(out.contents.h_buf, C.POINTER(C.c_uint16)), shape=(B * H * S * 128,))
    o = torch.from_numpy(got.astype(np.int32) << 16).view(torch.float32).reshape(B, H, S, 128)
    ref = _ref(torch, *[a.to(cuda) for a in arrs], True).cpu()
    assert (o - ref).abs().max().item() <= 2e-2
    for d in descs + [out]:
        L.hexa_farr_bf16_free(d)


def test_flash_prefill_benchmark_shape(forge, cuda):
    """The benchmark's prefill (B 8, H 32, S 4096, head dim 128, causal): the
    whole launch runs; eight (batch, head) pairs spread over the grid are
    compared with the fp32 reference row by row (every query row of 4096),
    plus a B 1, H 4 launch at the same length checked in full."""
    import torch
    for B, H, pairs in ((1, 4, [(0, h) for h in range(4)]),
                        (8, 32, [(0, 0), (1, 31), (2, 7), (3, 16), (4, 3), (5, 28), (6, 12), (7, 21)])):
        S = 4096
        g = torch.Generator(device=cuda).manual_seed(4096 + B)
        q, k, v = (torch.randn(B, H, S, 128, generator=g, device=cuda).to(torch.bfloat16) for _ in range(3))
        o = torch.full_like(q, float("nan"))
        torch.cuda.synchronize()
        forge.check(forge.lib().forge_flash_prefill(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B, H, S,
                                                    128, 1, torch.cuda.current_stream().cuda_stream), "prefill")
        torch.cuda.synchronize()
        forge.check(forge.lib().forge_ops_check(), "prefill error word")
        assert torch.isfinite(o.float()).all()
        for b, h in pairs:
            ref = _ref(torch, q[b:b + 1, h:h + 1], k[b:b + 1, h:h + 1], v[b:b + 1, h:h + 1], True)
            err = (o[b:b + 1, h:h + 1].float() - ref).abs()
            assert err.max().item() <= 2e-2, (B, H, b, h, err.max().item())
            assert err.mean().item() <= 2e-3, (B, H, b, h, err.mean().item())
        del q, k, v, o
