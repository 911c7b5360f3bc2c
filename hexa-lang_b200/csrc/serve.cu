// Continuous batching over the engine: the cb2 scheduler of hexa-lang's
// self/ml/continuous_batching.hexa with real model passes (one ragged
// forge_b200_forward_rows pass per iteration). Host code only; the contract
// and the line references are in include/forge_serve.h.
#include <chrono>
#include <cstring>
#include <vector>

#include "forge_internal.h"
#include "forge_serve.h"

namespace {

struct Req {
    ForgeServeRequest r{};
    std::vector<int32_t> toks;     // prompt, then the generated tokens
    int slot = -1;                 // engine sequence slot while running
    int64_t n_cached = 0;          // leading tokens whose K/V are in the slot
    std::vector<uint16_t> swap_kv; // [L][2][Hkv][n_cached][hd] while swapped out
};

}  // namespace

struct ForgeServe {
    ForgeB200* eng = nullptr;
    ForgeModelDesc desc{};
    int64_t max_batch = 0, max_kv_slots = 0;
    int32_t eos = -1;
    std::vector<Req> reqs;  // every request ever added; the lists hold indices
    std::vector<int> queue, running, swapped, completed;
    int64_t kv_used = 0, step = 0;
    // tracker (cb2_new_tracker)
    int64_t total_tokens = 0, total_requests_done = 0, total_preemptions = 0, total_swaps_out = 0,
            total_swaps_in = 0, total_latency = 0, total_wait_time = 0, max_latency = 0, max_wait_time = 0;
    std::vector<int> free_slots;  // LIFO
    double engine_ms = 0;
    int64_t engine_rows = 0, engine_passes = 0;
};

namespace {

int64_t kv_free(const ForgeServe* s) { return s->max_kv_slots - s->kv_used; }

// cb2_insert_sorted: before the first entry of strictly lower priority
void insert_sorted(ForgeServe* s, std::vector<int>& q, int idx) {
    const int64_t p = s->reqs[idx].r.priority;
    size_t i = 0;
    while (i < q.size() && !(p > s->reqs[q[i]].r.priority)) ++i;
    q.insert(q.begin() + i, idx);
}

int take_slot(ForgeServe* s) {
    if (s->free_slots.empty()) return -1;
    const int v = s->free_slots.back();
    s->free_slots.pop_back();
    return v;
}

void give_slot(ForgeServe* s, Req& q) {
    if (q.slot >= 0) s->free_slots.push_back(q.slot);
    q.slot = -1;
}

// cb2_find_preempt_victim: lowest priority, then most tokens generated
int find_victim(const ForgeServe* s) {
    const auto& run = s->running;
    if (run.empty()) return -1;
    int vi = 0;
    int64_t vp = s->reqs[run[0]].r.priority, vg = s->reqs[run[0]].r.tokens_generated;
    for (size_t i = 1; i < run.size(); ++i) {
        const ForgeServeRequest& r = s->reqs[run[i]].r;
        if (r.priority < vp) {
            vi = (int)i;
            vp = r.priority;
            vg = r.tokens_generated;
        }
        if (r.priority == vp && r.tokens_generated > vg) {
            vi = (int)i;
            vg = r.tokens_generated;
        }
    }
    return vi;
}

// cb2_preempt_at; the request's slot and cache are given up
void preempt_at(ForgeServe* s, int i) {
    if (i < 0 || i >= (int)s->running.size()) return;
    const int idx = s->running[i];
    Req& q = s->reqs[idx];
    const int64_t freed = q.r.kv_slots_used;
    s->running.erase(s->running.begin() + i);
    q.r.phase = FORGE_CB_PREEMPTED;
    q.r.was_preempted = 1;
    q.r.preempt_count += 1;
    give_slot(s, q);
    q.n_cached = 0;
    s->kv_used -= freed;
    insert_sorted(s, s->queue, idx);
    s->total_preemptions += 1;
}

// cb2_check_deadlines' boost of one request
void boost(ForgeServeRequest& r, int64_t cur_time) {
    if (r.deadline > 0) {
        const int64_t remaining = r.deadline - cur_time;
        if (remaining >= 0) {
            const int64_t budget = r.deadline - r.enqueue_time;
            if (budget > 0 && (double)remaining / (double)budget <= 0.2) r.priority += 100;
        }
    }
}

void check_deadlines(ForgeServe* s, int64_t cur_time) {
    for (int idx : s->queue) boost(s->reqs[idx].r, cur_time);
    for (int idx : s->running) boost(s->reqs[idx].r, cur_time);
    std::vector<int> sorted;
    for (int idx : s->queue) insert_sorted(s, sorted, idx);
    s->queue.swap(sorted);
}

// cb2_admit; with an engine each admitted request takes a sequence slot
// (running < max_batch <= the engine's slots, so one is always free)
void admit(ForgeServe* s) {
    while (!s->queue.empty() && (int64_t)s->running.size() < s->max_batch) {
        const int idx = s->queue.front();
        Req& q = s->reqs[idx];
        const int64_t needed = q.r.prompt_len;
        if (needed > kv_free(s)) break;
        s->queue.erase(s->queue.begin());
        q.r.phase = FORGE_CB_PREFILL;
        q.r.kv_slots_used = needed;
        q.r.start_time = s->step;
        if (s->eng) {
            q.slot = take_slot(s);
            q.n_cached = 0;
        }
        s->running.push_back(idx);
        s->kv_used += needed;
    }
}

// One engine pass: every running request's uncached tokens as rows, the
// argmax of its last row appended to its tokens.
int engine_pass(ForgeServe* s) {
    if (!s->eng || s->running.empty()) return 0;
    std::vector<int32_t> tok, pos, seq, out_rows;
    for (int idx : s->running) {
        Req& q = s->reqs[idx];
        if (q.slot < 0) return forge_fail(-1, "forge_serve: running request %lld has no slot", (long long)q.r.req_id);
        for (int64_t p = q.n_cached; p < (int64_t)q.toks.size(); ++p) {
            tok.push_back(q.toks[p]);
            pos.push_back((int32_t)p);
            seq.push_back(q.slot);
        }
        out_rows.push_back((int32_t)tok.size() - 1);
    }
    std::vector<int32_t> next(out_rows.size());
    const int exact = s->desc.act_mode == 2 ? 0 : 1;
    const auto t0 = std::chrono::steady_clock::now();
    const int rc = forge_b200_forward_rows(s->eng, (int)tok.size(), tok.data(), pos.data(), seq.data(),
                                           (int)out_rows.size(), out_rows.data(), exact, next.data(), nullptr);
    s->engine_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    if (rc) return -1;
    s->engine_rows += (int64_t)tok.size();
    s->engine_passes += 1;
    for (size_t i = 0; i < s->running.size(); ++i) {
        Req& q = s->reqs[s->running[i]];
        q.n_cached = (int64_t)q.toks.size();
        q.toks.push_back(next[i]);
    }
    return 0;
}

// cb2_prefill_phase + cb2_decode_phase (the pass runs between them)
int prefill_decode(ForgeServe* s) {
    for (int idx : s->running)
        if (s->reqs[idx].r.phase == FORGE_CB_PREFILL) s->reqs[idx].r.phase = FORGE_CB_DECODE;
    if (int rc = engine_pass(s)) return rc;
    std::vector<int> keep;
    int64_t tokens = 0, freed = 0, done = 0;
    for (int idx : s->running) {
        Req& q = s->reqs[idx];
        ForgeServeRequest& r = q.r;
        if (r.phase != FORGE_CB_DECODE) {
            keep.push_back(idx);
            continue;
        }
        r.tokens_generated += 1;
        r.kv_slots_used += 1;
        tokens += 1;
        const bool eos = s->eng && s->eos >= 0 && q.toks.back() == s->eos;
        if (r.tokens_generated >= r.max_gen || eos) {
            r.phase = FORGE_CB_DONE;
            r.finish_time = s->step;
            const int64_t latency = r.finish_time - r.enqueue_time, wait = r.start_time - r.enqueue_time;
            s->total_latency += latency;
            s->total_wait_time += wait;
            if (latency > s->max_latency) s->max_latency = latency;
            if (wait > s->max_wait_time) s->max_wait_time = wait;
            freed += r.kv_slots_used;
            give_slot(s, q);
            s->completed.push_back(idx);
            done += 1;
        } else {
            keep.push_back(idx);
        }
    }
    s->running.swap(keep);
    s->kv_used = s->kv_used - freed + tokens;
    s->total_tokens += tokens;
    s->total_requests_done += done;
    return 0;
}

// cb2_preemption_pass
void preemption_pass(ForgeServe* s) {
    int safety = 0;
    while (s->kv_used > s->max_kv_slots) {
        if (safety > 100) return;
        if (s->running.empty()) return;
        const int v = find_victim(s);
        if (v < 0) return;
        preempt_at(s, v);
        ++safety;
    }
}

const Req* find_req(const ForgeServe* s, int64_t rid) {
    for (const auto* list : {&s->running, &s->queue, &s->swapped, &s->completed})
        for (int idx : *list)
            if (s->reqs[idx].r.req_id == rid) return &s->reqs[idx];
    return nullptr;
}

// the last index of rid in a list (cb2_swap_out / cb2_swap_in keep looping)
int last_index(const ForgeServe* s, const std::vector<int>& list, int64_t rid) {
    int found = -1;
    for (size_t i = 0; i < list.size(); ++i)
        if (s->reqs[list[i]].r.req_id == rid) found = (int)i;
    return found;
}

size_t kv_floats_per_pos(const ForgeServe* s) { return (size_t)s->desc.n_kv_head * s->desc.head_dim; }

}  // namespace

FORGE_API int forge_serve_create(ForgeB200* engine, int max_batch, int64_t max_kv_slots, ForgeServe** out) {
    if (!out || max_batch <= 0 || max_kv_slots < 0) return forge_fail(FORGE_INVALID_ARGS, "forge_serve_create: bad arguments");
    *out = nullptr;
    ForgeModelDesc d{};
    if (engine) {
        if (forge_b200_get_desc(engine, &d)) return FORGE_INVALID_ARGS;
        if (d.tp_size != 1)
            return forge_fail(FORGE_INVALID_ARGS, "forge_serve_create: tensor-parallel handles are not supported");
        if (max_batch > d.max_batch)
            return forge_fail(FORGE_INVALID_ARGS, "forge_serve_create: max_batch %d above the engine's %d", max_batch,
                              d.max_batch);
    }
    ForgeServe* s = new ForgeServe();
    s->eng = engine;
    s->desc = d;
    s->max_batch = max_batch;
    s->max_kv_slots = max_kv_slots;
    if (engine)
        for (int i = d.max_batch - 1; i >= 0; --i) s->free_slots.push_back(i);
    *out = s;
    return 0;
}

FORGE_API int forge_serve_destroy(ForgeServe* s) {
    delete s;
    return 0;
}

FORGE_API int forge_serve_set_eos(ForgeServe* s, int32_t eos) {
    if (!s) return forge_fail(FORGE_INVALID_ARGS, "forge_serve_set_eos: null handle");
    s->eos = eos;
    return 0;
}

FORGE_API int forge_serve_add_request(ForgeServe* s, int64_t req_id, const int32_t* prompt, int64_t prompt_len,
                                      int64_t max_gen, int64_t priority, int64_t deadline) {
    if (!s || prompt_len < 0 || max_gen < 0) return forge_fail(FORGE_INVALID_ARGS, "forge_serve_add_request: bad arguments");
    if (s->eng) {
        if (!prompt || prompt_len < 1 || max_gen < 1)
            return forge_fail(FORGE_INVALID_ARGS, "forge_serve_add_request: an engine request needs a prompt and max_gen >= 1");
        if (prompt_len + max_gen - 1 > s->desc.max_ctx)
            return forge_fail(FORGE_INVALID_ARGS, "forge_serve_add_request: %lld prompt + %lld generated tokens exceed the context %d",
                              (long long)prompt_len, (long long)max_gen, s->desc.max_ctx);
        for (int64_t i = 0; i < prompt_len; ++i)
            if (prompt[i] < 0 || prompt[i] >= s->desc.vocab)
                return forge_fail(FORGE_INVALID_ARGS, "forge_serve_add_request: token %d outside the vocabulary", prompt[i]);
    }
    Req q;
    q.r.req_id = req_id;
    q.r.prompt_len = prompt_len;
    q.r.max_gen = max_gen;
    q.r.priority = priority;
    q.r.deadline = deadline;
    q.r.phase = FORGE_CB_QUEUED;
    q.r.enqueue_time = s->step;
    if (prompt) q.toks.assign(prompt, prompt + prompt_len);
    s->reqs.push_back(std::move(q));
    insert_sorted(s, s->queue, (int)s->reqs.size() - 1);
    return 0;
}

FORGE_API int forge_serve_run_step(ForgeServe* s, int64_t cur_time) {
    if (!s) return forge_fail(FORGE_INVALID_ARGS, "forge_serve_run_step: null handle");
    check_deadlines(s, cur_time);
    admit(s);
    if (int rc = prefill_decode(s)) return rc;
    preemption_pass(s);
    s->step += 1;
    return 0;
}

FORGE_API int forge_serve_run_until_done(ForgeServe* s, int64_t max_steps) {
    if (!s) return forge_fail(FORGE_INVALID_ARGS, "forge_serve_run_until_done: null handle");
    for (int64_t i = 0; i < max_steps; ++i) {
        if (s->queue.empty() && s->running.empty() && s->swapped.empty()) return 0;
        if (int rc = forge_serve_run_step(s, s->step)) return rc;
    }
    return 0;
}

FORGE_API int forge_serve_check_deadlines(ForgeServe* s, int64_t cur_time) {
    if (!s) return forge_fail(FORGE_INVALID_ARGS, "forge_serve_check_deadlines: null handle");
    check_deadlines(s, cur_time);
    return 0;
}

FORGE_API int forge_serve_preempt(ForgeServe* s, int64_t req_id) {
    if (!s) return forge_fail(FORGE_INVALID_ARGS, "forge_serve_preempt: null handle");
    for (size_t i = 0; i < s->running.size(); ++i)
        if (s->reqs[s->running[i]].r.req_id == req_id) {
            preempt_at(s, (int)i);
            return 0;
        }
    return 1;
}

FORGE_API int forge_serve_preempt_for_room(ForgeServe* s, int64_t needed) {
    if (!s) return forge_fail(FORGE_INVALID_ARGS, "forge_serve_preempt_for_room: null handle");
    int safety = 0;
    while (kv_free(s) < needed) {
        if (safety > 100) return 0;
        if (s->running.empty()) return 0;
        const int v = find_victim(s);
        if (v < 0) return 0;
        preempt_at(s, v);
        ++safety;
    }
    return 0;
}

FORGE_API int forge_serve_swap_out(ForgeServe* s, int64_t req_id) {
    if (!s) return forge_fail(FORGE_INVALID_ARGS, "forge_serve_swap_out: null handle");
    const int i = last_index(s, s->running, req_id);
    if (i < 0) return 1;
    const int idx = s->running[i];
    Req& q = s->reqs[idx];
    if (s->eng && q.slot >= 0 && q.n_cached > 0) {
        const size_t per = kv_floats_per_pos(s) * (size_t)q.n_cached;  // one layer's K (or V)
        q.swap_kv.resize(2 * per * (size_t)s->desc.n_layer);
        for (int l = 0; l < s->desc.n_layer; ++l) {
            uint16_t* base = q.swap_kv.data() + 2 * per * (size_t)l;
            if (forge_b200_get_kv_rows(s->eng, l, q.slot, base, base + per, (int)q.n_cached)) return -1;
        }
    }
    const int64_t kv_size = q.r.kv_slots_used;
    q.r.phase = FORGE_CB_SWAPPED;
    q.r.kv_slots_used = 0;
    give_slot(s, q);
    s->running.erase(s->running.begin() + i);
    s->swapped.push_back(idx);
    s->kv_used -= kv_size;
    s->total_swaps_out += 1;
    return 0;
}

FORGE_API int forge_serve_swap_in(ForgeServe* s, int64_t req_id) {
    if (!s) return forge_fail(FORGE_INVALID_ARGS, "forge_serve_swap_in: null handle");
    const int i = last_index(s, s->swapped, req_id);
    if (i < 0) return 1;
    const int idx = s->swapped[i];
    Req& q = s->reqs[idx];
    const int64_t needed = q.r.prompt_len + q.r.tokens_generated;
    if (kv_free(s) < needed) return 1;
    if (s->eng) {
        if (s->free_slots.empty()) return 1;
        q.slot = take_slot(s);
        if (q.n_cached > 0) {
            const size_t per = kv_floats_per_pos(s) * (size_t)q.n_cached;
            for (int l = 0; l < s->desc.n_layer; ++l) {
                const uint16_t* base = q.swap_kv.data() + 2 * per * (size_t)l;
                if (forge_b200_set_kv(s->eng, l, q.slot, base, base + per, (int)q.n_cached)) {
                    give_slot(s, q);
                    return -1;
                }
            }
        }
        std::vector<uint16_t>().swap(q.swap_kv);
    }
    q.r.phase = FORGE_CB_DECODE;
    q.r.kv_slots_used = needed;
    s->swapped.erase(s->swapped.begin() + i);
    s->running.push_back(idx);
    s->kv_used += needed;
    s->total_swaps_in += 1;
    return 0;
}

FORGE_API int forge_serve_peek_queue(const ForgeServe* s, ForgeServeRequest* out) {
    if (!s || !out) return forge_fail(FORGE_INVALID_ARGS, "forge_serve_peek_queue: null argument");
    if (s->queue.empty()) return 1;
    *out = s->reqs[s->queue.front()].r;
    return 0;
}

FORGE_API int forge_serve_find_request(const ForgeServe* s, int64_t req_id, ForgeServeRequest* out) {
    if (!s || !out) return forge_fail(FORGE_INVALID_ARGS, "forge_serve_find_request: null argument");
    const Req* q = find_req(s, req_id);
    if (!q) return 1;
    *out = q->r;
    return 0;
}

FORGE_API int64_t forge_serve_count_by_phase(const ForgeServe* s, int64_t phase) {
    if (!s) return forge_fail(FORGE_INVALID_ARGS, "forge_serve_count_by_phase: null handle");
    int64_t n = 0;
    for (int idx : s->running) n += s->reqs[idx].r.phase == phase;
    for (int idx : s->queue) n += s->reqs[idx].r.phase == phase;
    return n;
}

FORGE_API int forge_serve_stats(const ForgeServe* s, ForgeServeStats* out) {
    if (!s || !out) return forge_fail(FORGE_INVALID_ARGS, "forge_serve_stats: null argument");
    out->queue_size = (int64_t)s->queue.size();
    out->running_count = (int64_t)s->running.size();
    out->swapped_count = (int64_t)s->swapped.size();
    out->completed_count = (int64_t)s->completed.size();
    out->kv_used = s->kv_used;
    out->kv_free = kv_free(s);
    out->step = s->step;
    out->total_tokens = s->total_tokens;
    out->total_preemptions = s->total_preemptions;
    return 0;
}

FORGE_API int forge_serve_throughput(const ForgeServe* s, ForgeServeThroughput* out) {
    if (!s || !out) return forge_fail(FORGE_INVALID_ARGS, "forge_serve_throughput: null argument");
    out->tokens_per_step = s->step > 0 ? (double)s->total_tokens / (double)s->step : 0.0;
    out->avg_latency = s->total_requests_done > 0 ? (double)s->total_latency / (double)s->total_requests_done : 0.0;
    out->avg_wait_time = s->total_requests_done > 0 ? (double)s->total_wait_time / (double)s->total_requests_done : 0.0;
    out->max_latency = s->max_latency;
    out->max_wait_time = s->max_wait_time;
    out->total_tokens = s->total_tokens;
    out->total_preemptions = s->total_preemptions;
    out->total_swaps_out = s->total_swaps_out;
    out->total_swaps_in = s->total_swaps_in;
    out->total_requests_done = s->total_requests_done;
    return 0;
}

FORGE_API int forge_serve_output(const ForgeServe* s, int64_t req_id, int32_t* tokens, int64_t cap, int64_t* n) {
    if (!s || !n || cap < 0 || (cap > 0 && !tokens)) return forge_fail(FORGE_INVALID_ARGS, "forge_serve_output: bad arguments");
    const Req* q = find_req(s, req_id);
    if (!q) return 1;
    const int64_t gen = (int64_t)q->toks.size() - q->r.prompt_len;
    *n = gen > 0 ? gen : 0;
    for (int64_t i = 0; i < *n && i < cap; ++i) tokens[i] = q->toks[q->r.prompt_len + i];
    return 0;
}

FORGE_API int forge_serve_engine_time(const ForgeServe* s, double* ms, int64_t* rows, int64_t* passes) {
    if (!s) return forge_fail(FORGE_INVALID_ARGS, "forge_serve_engine_time: null handle");
    if (ms) *ms = s->engine_ms;
    if (rows) *rows = s->engine_rows;
    if (passes) *passes = s->engine_passes;
    return 0;
}
