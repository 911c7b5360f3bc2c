"""Test infrastructure (the oracle): a plain-Python restatement of the cb2
continuous-batching scheduler of hexa-lang's self/ml/continuous_batching.hexa,
used only by tests/ to check the library's native scheduler
(hexa-lang_b200/csrc/serve.cu) in its books-only mode. Nothing in the product
imports this module.

Each function follows the hexa function named in its docstring (line numbers
of continuous_batching.hexa). The hexa code is written as value updates
(`let mut s2 = s; s2["k"] = v`); this restatement copies where it does, so
every read of `s` sees the state before the update. (hexa-lang's compiled
runtime updates a map in place, so `s` and `s2` share one table; the only
place where that changes a result is cb2_decode_phase's
`len(new_completed) - len(s["completed"])`, which would then always be 0 and
leave total_requests_done and the averages at 0. Both this restatement and
the library count the completed requests.)

Parity is unpinned: the reference has no tests or vectors for cb2_* (its
self/test_continuous_batching.hexa exercises the earlier create_scheduler /
run_iteration API, whose cases tests/test_serve_cpu.py restates).
"""
from __future__ import annotations

import copy

QUEUED, PREFILL, DECODE, PREEMPTED, SWAPPED, DONE = range(6)  # :36-41


def new_request(req_id, prompt_len, max_gen, priority, deadline):  # :46
    return {"req_id": req_id, "prompt_len": prompt_len, "max_gen": max_gen, "priority": priority,
            "deadline": deadline, "phase": QUEUED, "tokens_generated": 0, "kv_slots_used": 0,
            "enqueue_time": 0, "start_time": 0, "finish_time": 0, "was_preempted": 0, "preempt_count": 0}


def new_tracker():  # :74
    return {k: 0 for k in ("total_tokens", "total_requests_done", "total_preemptions", "total_swaps_out",
                           "total_swaps_in", "total_latency", "total_wait_time", "max_latency", "max_wait_time")}


def create(max_batch, max_kv_slots):  # :91
    return {"max_batch": max_batch, "max_kv_slots": max_kv_slots, "queue": [], "running": [], "swapped": [],
            "completed": [], "kv_used": 0, "step": 0, "tracker": new_tracker()}


def insert_sorted(queue, req):  # :111
    result, inserted = [], False
    for q in queue:
        if not inserted and req["priority"] > q["priority"]:
            result.append(req)
            inserted = True
        result.append(q)
    if not inserted:
        result.append(req)
    return result


def add_request(s, req_id, prompt_len, max_gen, priority, deadline):  # :134
    req = new_request(req_id, prompt_len, max_gen, priority, deadline)
    req["enqueue_time"] = s["step"]
    s2 = copy.deepcopy(s)
    s2["queue"] = insert_sorted(s2["queue"], req)
    return s2


def peek_queue(s):  # :152
    return dict(s["queue"][0]) if s["queue"] else {}


def kv_free(s):  # :176
    return s["max_kv_slots"] - s["kv_used"]


def find_preempt_victim(running):  # :196
    n = len(running)
    if n == 0:
        return -1
    vi, vp, vg = 0, running[0]["priority"], running[0]["tokens_generated"]
    for i in range(1, n):
        r = running[i]
        if r["priority"] < vp:
            vi, vp, vg = i, r["priority"], r["tokens_generated"]
        if r["priority"] == vp and r["tokens_generated"] > vg:
            vi, vg = i, r["tokens_generated"]
    return vi


def preempt_at(s, idx):  # :224
    s = copy.deepcopy(s)
    running = s["running"]
    if idx < 0 or idx >= len(running):
        return s
    victim = running[idx]
    freed = victim["kv_slots_used"]
    new_running = [r for i, r in enumerate(running) if i != idx]
    victim["phase"] = PREEMPTED
    victim["was_preempted"] = 1
    victim["preempt_count"] += 1
    kv_used = s["kv_used"]
    s["running"] = new_running
    s["kv_used"] = kv_used - freed
    s["queue"] = insert_sorted(s["queue"], victim)
    s["tracker"]["total_preemptions"] += 1
    return s


def preempt(s, rid):  # :255
    for i, r in enumerate(s["running"]):
        if r["req_id"] == rid:
            return preempt_at(s, i)
    return s


def swap_out(s, rid):  # :270
    found = -1
    for i, r in enumerate(s["running"]):
        if r["req_id"] == rid:
            found = i
    if found < 0:
        return s
    s = copy.deepcopy(s)
    victim = s["running"][found]
    kv_size = victim["kv_slots_used"]
    victim["phase"] = SWAPPED
    victim["kv_slots_used"] = 0
    s["running"] = [r for i, r in enumerate(s["running"]) if i != found]
    s["swapped"] = s["swapped"] + [victim]
    s["kv_used"] -= kv_size
    s["tracker"]["total_swaps_out"] += 1
    return s


def swap_in(s, rid):  # :306
    found = -1
    for i, r in enumerate(s["swapped"]):
        if r["req_id"] == rid:
            found = i
    if found < 0:
        return s
    restored = s["swapped"][found]
    needed = restored["prompt_len"] + restored["tokens_generated"]
    if kv_free(s) < needed:
        return s
    s = copy.deepcopy(s)
    restored = s["swapped"][found]
    restored["phase"] = DECODE
    restored["kv_slots_used"] = needed
    s["swapped"] = [r for i, r in enumerate(s["swapped"]) if i != found]
    s["running"] = s["running"] + [restored]
    s["kv_used"] += needed
    s["tracker"]["total_swaps_in"] += 1
    return s


def _boost(r, cur_time):
    if r["deadline"] > 0:
        remaining = r["deadline"] - cur_time
        if remaining >= 0:
            budget = r["deadline"] - r["enqueue_time"]
            if budget > 0 and float(remaining) / float(budget) <= 0.2:
                r["priority"] += 100


def check_deadlines(s, cur_time):  # :341
    s = copy.deepcopy(s)
    for r in s["queue"]:
        _boost(r, cur_time)
    for r in s["running"]:
        _boost(r, cur_time)
    q = []
    for r in s["queue"]:
        q = insert_sorted(q, r)
    s["queue"] = q
    return s


def admit(s):  # :398
    s = copy.deepcopy(s)
    while s["queue"] and len(s["running"]) < s["max_batch"]:
        head = s["queue"][0]
        needed = head["prompt_len"]
        if needed > kv_free(s):
            break
        s["queue"] = s["queue"][1:]
        head["phase"] = PREFILL
        head["kv_slots_used"] = needed
        head["start_time"] = s["step"]
        s["running"] = s["running"] + [head]
        s["kv_used"] += needed
    return s


def prefill_phase(s):  # :437
    s = copy.deepcopy(s)
    for r in s["running"]:
        if r["phase"] == PREFILL:
            r["phase"] = DECODE
    return s


def decode_phase(s):  # :456
    s2 = copy.deepcopy(s)
    t = s2["tracker"]
    new_running, new_completed = [], list(s2["completed"])
    tokens = freed = lat_add = wait_add = 0
    max_lat, max_wait = t["max_latency"], t["max_wait_time"]
    for r in s2["running"]:
        if r["phase"] == DECODE:
            r["tokens_generated"] += 1
            r["kv_slots_used"] += 1
            tokens += 1
            if r["tokens_generated"] >= r["max_gen"]:
                r["phase"] = DONE
                r["finish_time"] = s["step"]
                latency = r["finish_time"] - r["enqueue_time"]
                wait = r["start_time"] - r["enqueue_time"]
                lat_add += latency
                wait_add += wait
                max_lat = max(max_lat, latency)
                max_wait = max(max_wait, wait)
                freed += r["kv_slots_used"]
                new_completed.append(r)
            else:
                new_running.append(r)
        else:
            new_running.append(r)
    s2["running"] = new_running
    s2["completed"] = new_completed
    s2["kv_used"] = s["kv_used"] - freed + tokens
    t["total_tokens"] += tokens
    t["total_requests_done"] += len(new_completed) - len(s["completed"])
    t["total_latency"] += lat_add
    t["total_wait_time"] += wait_add
    t["max_latency"] = max_lat
    t["max_wait_time"] = max_wait
    return s2


def preemption_pass(s):  # :511
    safety = 0
    while s["kv_used"] > s["max_kv_slots"]:
        if safety > 100 or not s["running"]:
            return s
        v = find_preempt_victim(s["running"])
        if v < 0:
            return s
        s = preempt_at(s, v)
        safety += 1
    return s


def run_step(s, cur_time):  # :530
    s = check_deadlines(s, cur_time)
    s = admit(s)
    s = prefill_phase(s)
    s = decode_phase(s)
    s = preemption_pass(s)
    s["step"] += 1
    return s


def run_until_done(s, max_steps):  # :543
    for _ in range(max_steps):
        if not s["queue"] and not s["running"] and not s["swapped"]:
            return s
        s = run_step(s, s["step"])
    return s


def stats(s):  # :573
    t = s["tracker"]
    return {"queue_size": len(s["queue"]), "running_count": len(s["running"]), "swapped_count": len(s["swapped"]),
            "completed_count": len(s["completed"]), "kv_used": s["kv_used"], "kv_free": kv_free(s),
            "step": s["step"], "total_tokens": t["total_tokens"], "total_preemptions": t["total_preemptions"]}


def throughput(s):  # :588
    t, steps = s["tracker"], s["step"]
    done = t["total_requests_done"]
    return {"tokens_per_step": float(t["total_tokens"]) / float(steps) if steps > 0 else 0.0,
            "avg_latency": float(t["total_latency"]) / float(done) if done > 0 else 0.0,
            "avg_wait_time": float(t["total_wait_time"]) / float(done) if done > 0 else 0.0,
            "max_latency": t["max_latency"], "max_wait_time": t["max_wait_time"], "total_tokens": t["total_tokens"],
            "total_preemptions": t["total_preemptions"], "total_swaps_out": t["total_swaps_out"],
            "total_swaps_in": t["total_swaps_in"], "total_requests_done": done}


def find_request(s, rid):  # :621
    for key in ("running", "queue", "swapped", "completed"):
        for r in s[key]:
            if r["req_id"] == rid:
                return dict(r)
    return {}


def count_by_phase(s, phase):  # :645
    return sum(r["phase"] == phase for r in s["running"]) + sum(r["phase"] == phase for r in s["queue"])


def preempt_for_room(s, needed):  # :662
    safety = 0
    while kv_free(s) < needed:
        if safety > 100 or not s["running"]:
            return s
        v = find_preempt_victim(s["running"])
        if v < 0:
            return s
        s = preempt_at(s, v)
        safety += 1
    return s
