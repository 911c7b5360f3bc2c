"""Continuous batching (include/forge_serve.h) without a GPU: the native
scheduler in its books-only mode (no engine) against the oracle's restatement
of self/ml/continuous_batching.hexa (oracle/cb2.py) over seeded random
operation sequences — every request record, stats, throughput, the queue head
and the per-phase counts after every operation — plus the cases of the
reference's self/test_continuous_batching.hexa (T1-T14, written for its
earlier create_scheduler / run_iteration API) restated on this one, and the
argument checks."""
import random

import pytest

import cb2

PHASES = range(6)


def _compare(sv, o, rids):
    assert sv.stats() == cb2.stats(o)
    assert sv.throughput() == cb2.throughput(o)  # the averages: one IEEE division each side
    assert sv.peek_queue() == cb2.peek_queue(o)
    for rid in rids:
        assert sv.find_request(rid) == cb2.find_request(o, rid), rid
    for ph in PHASES:
        assert sv.count_by_phase(ph) == cb2.count_by_phase(o, ph)


@pytest.mark.parametrize("seed", range(12))
def test_random_operations_match_the_oracle(forge, seed):
    rng = random.Random(seed)
    max_batch, kv = rng.choice([(1, 30), (2, 40), (4, 64), (8, 200), (3, 25)])
    sv = forge.ForgeServe(None, max_batch, kv)
    o = cb2.create(max_batch, kv)
    rids = []
    for _ in range(160):
        op = rng.random()
        if op < 0.3:
            rid = rng.randrange(40)  # ids may repeat, as in the hexa module
            pl, mg, pr = rng.randint(0, 18), rng.randint(1, 9), rng.randint(0, 3)
            dl = 0 if rng.random() < 0.5 else o["step"] + rng.randint(-2, 12)
            sv.add_request(rid, pl, mg, pr, dl)
            o = cb2.add_request(o, rid, pl, mg, pr, dl)
            rids.append(rid)
        elif op < 0.7:
            t = o["step"] + rng.randint(0, 3)
            assert sv.run_step(t) == 0
            o = cb2.run_step(o, t)
        elif op < 0.76 and rids:
            rid = rng.choice(rids)
            sv.preempt(rid)
            o = cb2.preempt(o, rid)
        elif op < 0.84 and rids:
            rid = rng.choice(rids)
            sv.swap_out(rid)
            o = cb2.swap_out(o, rid)
        elif op < 0.92 and rids:
            rid = rng.choice(rids)
            sv.swap_in(rid)
            o = cb2.swap_in(o, rid)
        elif op < 0.95:
            t = o["step"] + rng.randint(0, 10)
            sv.check_deadlines(t)
            o = cb2.check_deadlines(o, t)
        elif op < 0.98:
            need = rng.randint(0, kv)
            sv.preempt_for_room(need)
            o = cb2.preempt_for_room(o, need)
        else:
            n = rng.randint(1, 6)
            sv.run_until_done(n)
            o = cb2.run_until_done(o, n)
        _compare(sv, o, set(rids))
    sv.run_until_done(500)
    o = cb2.run_until_done(o, 500)
    _compare(sv, o, set(rids))
    sv.close()


def test_return_codes(forge):
    sv = forge.ForgeServe(None, 2, 10)
    assert sv.peek_queue() == {} and sv.find_request(7) == {}
    assert sv.preempt(7) == 1 and sv.swap_out(7) == 1 and sv.swap_in(7) == 1
    sv.add_request(7, 4, 3, 0, 0)
    assert sv.run_step(0) == 0 and sv.swap_out(7) == 0
    sv.add_request(8, 8, 3, 0, 0)
    assert sv.run_step(1) == 0
    assert sv.swap_in(7) == 1  # needs 4 + 1 slots, 10 - 9 free
    with pytest.raises(RuntimeError):
        sv.add_request(9, -1, 3, 0, 0)
    with pytest.raises(RuntimeError):
        forge.ForgeServe(None, 0, 10)
    sv.close()


def test_deadline_boost_reorders_the_queue(forge):
    """cb2_check_deadlines: within 20% of the deadline → priority + 100 (every
    call), queue re-sorted by priority, FIFO within a priority."""
    sv = forge.ForgeServe(None, 1, 1000)
    o = cb2.create(1, 1000)
    for rid, pr, dl in ((1, 5, 0), (2, 1, 10), (3, 1, 0), (4, 5, 50)):
        sv.add_request(rid, 2, 20, pr, dl)
        o = cb2.add_request(o, rid, 2, 20, pr, dl)
    for t in (0, 7, 8, 9, 9, 45):
        sv.check_deadlines(t)
        o = cb2.check_deadlines(o, t)
        _compare(sv, o, [1, 2, 3, 4])
    assert sv.peek_queue()["req_id"] == 2 and sv.find_request(2)["priority"] == 301  # boosted at t 8, 9, 9
    assert sv.find_request(4)["priority"] == 105
    sv.close()


# ---- the reference's test_continuous_batching.hexa cases (T1-T14) on this API ----

def test_reference_cases_t1_t14(forge):
    # T1-T4: creation and enqueueing (FIFO at one priority; ids as given)
    s = forge.ForgeServe(None, 4, 1 << 20)
    s.add_request(0, 5, 3, 0, 0)
    assert s.stats()["queue_size"] == 1
    s.add_request(1, 5, 5, 0, 0)
    assert s.peek_queue()["req_id"] == 0 and s.peek_queue()["max_gen"] == 3
    assert s.find_request(1)["max_gen"] == 5
    # T5-T6: one iteration moves pending to running and generates tokens
    s.run_step(0)
    st = s.stats()
    assert st["running_count"] >= 1 and st["total_tokens"] > 0
    s.close()
    # T7-T8: run until done completes all (max_batch 2, three requests)
    s = forge.ForgeServe(None, 2, 1 << 20)
    for rid, n in ((0, 3), (1, 2), (2, 4)):
        s.add_request(rid, 5, n, 0, 0)
    s.run_until_done(100)
    assert s.stats()["completed_count"] == 3
    assert all(s.find_request(r)["tokens_generated"] >= 1 for r in range(3))
    assert [s.find_request(r)["tokens_generated"] for r in range(3)] == [3, 2, 4]
    s.close()
    # T9-T11: max_batch limits the running set; the rest wait
    s = forge.ForgeServe(None, 2, 1 << 20)
    for rid in range(4):
        s.add_request(rid, 1, 10, 0, 0)
    s.run_step(0)
    st = s.stats()
    assert st["running_count"] <= 2 and st["queue_size"] >= 1
    s.close()
    # T13: an empty scheduler's iteration generates nothing
    s = forge.ForgeServe(None, 4, 1 << 20)
    s.run_step(0)
    assert s.stats()["total_tokens"] == 0
    s.close()
    # T14: a single request completes in max_gen iterations
    s = forge.ForgeServe(None, 1, 1 << 20)
    s.add_request(0, 6, 2, 0, 0)
    s.run_until_done(50)
    st = s.stats()
    assert st["completed_count"] == 1 and st["step"] == 2
    s.close()
