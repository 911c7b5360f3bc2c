"""Tensor-parallel decode on two B200s against the same model on one GPU:
the sharded model (heads, FFN groups and vocabulary split, NCCL all-reduce
after the O and down projections, max all-reduce of the argmax keys) must give
the single-GPU logits up to summation order and the same greedy tokens.
Runs as two spawned rank processes, with the residual all-reduce through
peer memory (the default) and through NCCL; skipped with fewer than two
GPUs. Up to 4 sequences the peer exchange either runs inside the O / down
GEMV's epilogue (FORGE_TP_FUSED_RESID=1), which must give the bits of the
GEMV + separate all-reduce, or as its own kernel that also stages the next
RMSNorm GEMV's input (int4 weights; FORGE_PREQUANT=0 turns it off)."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CONFIGS = {
    "gqa_q4": dict(cfg=(2, 256, 8, 4, 64, 768, 1000), q4=True),
    "gqa_bf16": dict(cfg=(2, 256, 4, 2, 64, 512, 500), q4=False),
}
PROMPT = [[3, 17, 5, 99], [8, 2, 64, 1]]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(fb, model_kw, tp_kw, device):
    m = fb.ForgeModel(*model_kw["cfg"], weight_kind=fb.FORGE_WEIGHT_Q4_G128 if model_kw["q4"] else fb.FORGE_WEIGHT_BF16,
                      max_batch=2, max_ctx=64, device=device, **tp_kw)
    m.init_synthetic(1234, 0.05)
    gen = m.generate(PROMPT, 12)
    m.reset()
    toks, lgs = np.array([3, 8], np.int32), []
    for _ in range(6):
        toks, lg = m.step(toks, want_logits=True)
        lgs.append(lg)
    m.close()
    return gen, np.stack(lgs)


def _rank_main(rank, world, port, name, ar, q, fused="1", prequant="1"):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "hexa-lang_b200"))
    import datetime
    import torch
    import torch.distributed as dist
    import forge_b200 as fb
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), FORGE_TP_ALLREDUCE=ar, FORGE_TP_FUSED_RESID=fused,
                      FORGE_PREQUANT=prequant)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        obj = [fb.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        gen, lgs = _run(fb, CONFIGS[name], dict(tp_rank=rank, tp_size=world, nccl_id=obj[0]), rank)
        q.put((rank, gen, lgs, None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, None, repr(e)))
    finally:
        dist.destroy_process_group()


def _tp2(name, ar, fused="1", prequant="1"):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, name, ar, q, fused, prequant)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        rank, gen, lgs, err = q.get(timeout=300)
        res[rank] = (gen, lgs, err)
    for p in procs:
        p.join(timeout=120)
    return res


@pytest.mark.parametrize("ar", ["peer", "nccl", "peer_handoff"])
@pytest.mark.parametrize("name", list(CONFIGS))
def test_tp2_matches_single_gpu(forge, cuda, name, ar):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ref_gen, ref_lgs = _run(forge, CONFIGS[name], {}, 0)
    # peer_handoff: the all-reduce kernel (not the fused epilogue), which
    # stages the next GEMV's input for int4 weights
    res = _tp2(name, "peer", "0") if ar == "peer_handoff" else _tp2(name, ar)
    for rank in (0, 1):
        gen, lgs, err = res[rank]
        assert err is None, err
        # every rank ends with the same tokens and the full (gathered) logits
        assert np.array_equal(gen, ref_gen), (rank, gen, ref_gen)
        scale = np.abs(ref_lgs).max()
        assert np.abs(lgs - ref_lgs).max() <= 2e-3 * scale, np.abs(lgs - ref_lgs).max()
    assert np.array_equal(res[0][1], res[1][1])


@pytest.mark.parametrize("name", list(CONFIGS))
def test_tp2_fused_residual_same_bits(cuda, name):
    """The exchange inside the GEMV epilogue against GEMV + one-shot all-reduce."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    fused, plain = _tp2(name, "peer", "1", "0"), _tp2(name, "peer", "0", "0")
    for rank in (0, 1):
        assert fused[rank][2] is None and plain[rank][2] is None, (fused[rank][2], plain[rank][2])
        assert np.array_equal(fused[rank][0], plain[rank][0])
        assert np.array_equal(fused[rank][1], plain[rank][1])


def test_tp2_handoff_close_to_staging(cuda):
    """int4: the all-reduce's staged input (codes of gain * x, the RMSNorm
    factor from per-group sums of squares folded into the scales) against
    the GEMVs staging x themselves: same greedy tokens, logits within the
    reordering of the RMSNorm sum and the fold of its factor."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    on, off = _tp2("gqa_q4", "peer", "0", "1"), _tp2("gqa_q4", "peer", "0", "0")
    for rank in (0, 1):
        assert on[rank][2] is None and off[rank][2] is None, (on[rank][2], off[rank][2])
        assert np.array_equal(on[rank][0], off[rank][0])
        scale = np.abs(off[rank][1]).max()
        assert np.abs(on[rank][1] - off[rank][1]).max() <= 1e-3 * scale
    assert np.array_equal(on[0][1], on[1][1])
