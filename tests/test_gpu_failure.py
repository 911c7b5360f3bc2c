"""Failure detection on the GPU without a fault: a bounded wait that runs
out. The tensor-parallel peer exchange is run as rank 0 of two ranks whose
other rank never comes (forge_tp_selftest_absent_peer: both ranks' buffers
in this process, nothing raises rank 1's flags). The kernel's flag wait
must give up after its limit (50 ms here), set the error bit and return;
the context must stay usable, and the engine must keep working after it."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_peer_wait_runs_out_and_the_context_survives(forge, cuda):
    L = forge.lib()
    for T, n in ((2, 4096), (8, 40000)):
        bits, ms = C.c_uint32(0), C.c_double(0.0)
        forge.check(L.forge_tp_selftest_absent_peer(T, n, 50_000_000, C.byref(bits), C.byref(ms)), "self-test")
        assert bits.value & 2, bits.value          # FORGE_DEVERR_COUNTER_TIMEOUT
        assert 40.0 <= ms.value < 1000.0, ms.value  # gave up after ~50 ms, not the 2 s default
    # the engine still runs on this device
    m = forge.ForgeModel(2, 256, 4, 2, 64, 512, 1000, weight_kind=forge.FORGE_WEIGHT_Q4_G128, max_batch=1, max_ctx=16)
    m.init_synthetic(1234, 0.02)
    m.reset()
    nxt = m.step([5])
    assert 0 <= int(nxt[0]) < 1000
    m.close()


def test_selftest_rejects_bad_arguments(forge, cuda):
    L = forge.lib()
    bits, ms = C.c_uint32(0), C.c_double(0.0)
    assert L.forge_tp_selftest_absent_peer(1, 4096, 50_000_000, C.byref(bits), C.byref(ms)) != 0   # one rank
    assert L.forge_tp_selftest_absent_peer(2, 4096, 1000, C.byref(bits), C.byref(ms)) != 0         # limit < 1 ms
