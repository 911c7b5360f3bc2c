"""Failure detection on the host, without a GPU (two processes on CPU):

  * a tensor-parallel rank that leaves between steps is found by the
    heartbeat of the next step (forge_b200.tp_heartbeat over a shared
    key-value store) before anything of that step is launched, and the
    error names the missing rank;
  * a gloo rank that exits before a collective: the surviving rank's
    collective (the host-side reductions the tensor-parallel bench uses for
    its timings) ends with an error instead of waiting for ever.
"""
import multiprocessing as mp
import os
import socket
import sys
import time

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _hb_rank(rank, port, q):
    sys.path.insert(0, os.path.join(ROOT, "hexa-lang_b200"))
    import datetime
    import torch.distributed as dist
    import forge_b200 as fb
    store = dist.TCPStore("127.0.0.1", port, 2, rank == 0, timeout=datetime.timedelta(seconds=30))
    try:
        fb.tp_heartbeat(store, rank, 2, 0, timeout_s=10.0)   # step 0: both ranks present
        if rank == 1:
            q.put((1, "left", 0.0))
            return                                             # rank 1 leaves between steps
        time.sleep(0.5)
        t0 = time.time()
        try:
            fb.tp_heartbeat(store, rank, 2, 1, timeout_s=2.0)
            q.put((0, "no error", time.time() - t0))
        except fb.ForgeError as e:
            q.put((0, str(e), time.time() - t0))
    except Exception as e:  # reported to the parent
        q.put((rank, "unexpected: " + repr(e), 0.0))


def test_heartbeat_finds_a_rank_that_left():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_hb_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (msg, dt)) for r, msg, dt in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
    msg, dt = res[0]
    assert "rank(s) [1] missed the heartbeat of step 1" in msg, msg
    assert dt < 10.0


def _gloo_rank(rank, port, q):
    import datetime
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)                                  # no clean shutdown: the process is gone
    time.sleep(1.0)
    t0 = time.time()
    try:
        t = torch.ones(4)
        dist.all_reduce(t)
        q.put((0, "no error", time.time() - t0))
    except Exception as e:
        q.put((0, type(e).__name__ + ": " + str(e)[:200], time.time() - t0))


def test_gloo_collective_with_a_departed_rank_fails():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    rank, msg, dt = q.get(timeout=120)               # only the surviving rank reports
    for p in procs:
        p.join(timeout=60)
    assert msg != "no error", msg
    assert dt < 30.0, dt


def test_bad_nccl_unique_id_is_refused_before_any_nccl_call(forge):
    """An all-zero id (never written by forge_b200_tp_unique_id) and a rank
    outside 0..tp_size-1 are refused before the device or NCCL is touched,
    so no rank is left waiting in NCCL's bootstrap; a well-formed id gets as
    far as the device check (no GPU here)."""
    import ctypes as C
    fb = forge
    d = fb.ForgeModelDesc(2, 256, 4, 4, 64, 512, 1000, 1e-5, 10000.0, 0, 0, 1, 64, 0, 2, 0)
    h = C.c_void_p()
    zero = (C.c_ubyte * 128)()
    rc = fb.lib().forge_b200_create_tp(C.byref(d), 0, zero, C.byref(h))
    assert rc == fb.FORGE_INVALID_ARGS and b"empty NCCL unique id" in fb.lib().forge_b200_last_error()
    d.tp_rank = 2
    some = (C.c_ubyte * 128)(*([7] * 128))
    rc = fb.lib().forge_b200_create_tp(C.byref(d), 0, some, C.byref(h))
    assert rc == fb.FORGE_INVALID_ARGS and b"rank 2 outside 0..1" in fb.lib().forge_b200_last_error()
    import torch
    if not torch.cuda.is_available():
        d.tp_rank = 0
        rc = fb.lib().forge_b200_create_tp(C.byref(d), 0, some, C.byref(h))
        assert rc != 0 and b"unique id" not in fb.lib().forge_b200_last_error()
