"""Host side of the tensor-parallel mode without a GPU: the shard plan every
rank derives on its own (FFN in whole 128-row groups for int4 — 7B's 11008 =
86 groups and 13B's 13824 = 108 groups do not divide by 8, so the slices
are uneven, the first ranks taking one group more — heads evenly, vocabulary in equal 16-row slices), and its
agreement across processes: two `gloo` ranks share rank 0's NCCL unique id
the way bench.py does and check that their shards tile the model exactly."""
import os
import socket

import pytest


def _plan(fb, n, gran, size):
    return [fb.tp_split(n, gran, r, size) for r in range(size)]


@pytest.mark.parametrize("n,gran", [(11008, 128), (13824, 128), (8192, 128), (688, 16), (4096, 16)])
@pytest.mark.parametrize("size", [1, 2, 4, 8])
def test_split_tiles_exactly(forge, n, gran, size):
    plan = _plan(forge, n, gran, size)
    pos = 0
    for off, ln in plan:
        assert off == pos and ln > 0 and ln % gran == 0
        pos += ln
    assert pos == n
    lens = [ln for _, ln in plan]
    assert max(lens) - min(lens) <= gran          # balanced to one unit
    assert lens == sorted(lens, reverse=True)      # the first ranks take the extra units


def test_split_rejects_empty_or_misaligned(forge):
    with pytest.raises(forge.ForgeError):
        forge.tp_split(256, 128, 2, 4)             # 2 groups over 4 ranks
    with pytest.raises(forge.ForgeError):
        forge.tp_split(1000, 128, 0, 2)            # not whole groups


def test_unique_id_is_fresh(forge):
    a, b = forge.tp_unique_id(), forge.tp_unique_id()
    assert len(a) == 128 and len(b) == 128 and a != b


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "hexa-lang_b200"))
    import datetime
    import torch.distributed as dist
    import forge_b200 as fb
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        obj = [fb.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        mine = {"id": obj[0], "ffn": fb.tp_split(11008, 128, rank, world), "ffn13": fb.tp_split(13824, 128, rank, world)}
        got = [None] * world
        dist.all_gather_object(got, mine)
        q.put((rank, got))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_agree_on_the_shard_plan():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in (0, 1):
        got = res[rank]
        assert got[0]["id"] == got[1]["id"] and len(got[0]["id"]) == 128   # one communicator id
        for key, n in (("ffn", 11008), ("ffn13", 13824)):
            (o0, l0), (o1, l1) = got[0][key], got[1][key]
            assert o0 == 0 and o1 == l0 and l0 + l1 == n
