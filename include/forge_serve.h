/* forge_serve.h — continuous batching over the forge_b200 engine.
 *
 * The scheduler contract of hexa-lang's self/ml/continuous_batching.hexa
 * (cb2_*): a priority queue (higher priority first, FIFO within a priority),
 * an iteration that runs deadline boosts → admission → prefill → decode →
 * preemption, preemption of the lowest-priority / longest-running request
 * when the KV budget is over-committed, KV swap out to host memory and back,
 * SLA deadline boosts and a throughput tracker. Every scheduling decision
 * and every counter follows the hexa functions (line numbers in that file:
 * cb2_insert_sorted:111, cb2_add_request:134, cb2_find_preempt_victim:196,
 * cb2_preempt_at:224, cb2_preempt:255, cb2_swap_out:270, cb2_swap_in:306,
 * cb2_check_deadlines:341, cb2_admit:398, cb2_prefill_phase:437,
 * cb2_decode_phase:456, cb2_preemption_pass:511, cb2_run_step:530,
 * cb2_run_until_done:543, cb2_stats:573, cb2_throughput:588,
 * cb2_find_request:621, cb2_count_by_phase:645, cb2_preempt_for_room:662).
 *
 * The hexa module only keeps the books; here each iteration also runs the
 * model. With an engine handle, every admitted request owns one sequence
 * slot of the engine's KV cache, and one forge_b200_forward_rows pass per
 * iteration carries the whole prompt of each newly admitted request (its
 * prompt and the tokens generated so far, after a preemption) together with
 * one row for every decoding request; each running request's next token is
 * the argmax at its last row (greedy). A preempted request gives up its slot
 * and its cache (recomputed when it is admitted again); a swapped-out one
 * has its cache rows copied to host memory and back into a free slot on
 * swap-in. Without an engine (NULL) the scheduler keeps the books alone,
 * exactly as the hexa module does, and produces no tokens.
 *
 * Functions return 0 when done, 1 when the state is unchanged (the request
 * was not found, the KV budget or, with an engine, a free sequence slot is
 * missing: the hexa functions return the state as it was), FORGE_INVALID_ARGS
 * (-4) for bad arguments and -1 when an engine pass failed (the iteration's
 * books are then left as they were before its decode phase).
 * Handles are not thread-safe. */
#ifndef FORGE_SERVE_H
#define FORGE_SERVE_H
#include <stdint.h>

#include "forge_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ForgeServe ForgeServe;

/* request phases (cb2_phase_*) */
enum {
    FORGE_CB_QUEUED = 0,
    FORGE_CB_PREFILL = 1,
    FORGE_CB_DECODE = 2,
    FORGE_CB_PREEMPTED = 3,
    FORGE_CB_SWAPPED = 4,
    FORGE_CB_DONE = 5
};

/* cb2_new_request's fields */
typedef struct ForgeServeRequest {
    int64_t req_id, prompt_len, max_gen, priority, deadline, phase, tokens_generated, kv_slots_used;
    int64_t enqueue_time, start_time, finish_time, was_preempted, preempt_count;
} ForgeServeRequest;

/* cb2_stats */
typedef struct ForgeServeStats {
    int64_t queue_size, running_count, swapped_count, completed_count, kv_used, kv_free, step;
    int64_t total_tokens, total_preemptions;
} ForgeServeStats;

/* cb2_throughput (the three averages are doubles, the rest counts) */
typedef struct ForgeServeThroughput {
    double tokens_per_step, avg_latency, avg_wait_time;
    int64_t max_latency, max_wait_time, total_tokens, total_preemptions, total_swaps_out, total_swaps_in;
    int64_t total_requests_done;
} ForgeServeThroughput;

/* cb2_create(max_batch, max_kv_slots). engine may be NULL (books only);
 * otherwise max_batch must not exceed the engine's max_batch, and the
 * engine must be a single-GPU handle with weights loaded. */
int forge_serve_create(ForgeB200* engine, int max_batch, int64_t max_kv_slots, ForgeServe** out);
int forge_serve_destroy(ForgeServe* s);
/* A token id that ends a request early (as the v1 scheduler's EOS check);
 * -1 (the default) for none. */
int forge_serve_set_eos(ForgeServe* s, int32_t eos);
/* cb2_add_request / cb2_add_mid_generation. prompt [prompt_len] token ids;
 * with an engine it is required and prompt_len + max_gen - 1 must fit the
 * engine's context; without one it may be NULL. */
int forge_serve_add_request(ForgeServe* s, int64_t req_id, const int32_t* prompt, int64_t prompt_len,
                            int64_t max_gen, int64_t priority, int64_t deadline);
int forge_serve_run_step(ForgeServe* s, int64_t cur_time);          /* cb2_run_step */
int forge_serve_run_until_done(ForgeServe* s, int64_t max_steps);   /* cb2_run_until_done */
int forge_serve_check_deadlines(ForgeServe* s, int64_t cur_time);   /* cb2_check_deadlines */
int forge_serve_preempt(ForgeServe* s, int64_t req_id);             /* cb2_preempt */
int forge_serve_preempt_for_room(ForgeServe* s, int64_t needed);    /* cb2_preempt_for_room */
int forge_serve_swap_out(ForgeServe* s, int64_t req_id);            /* cb2_swap_out */
int forge_serve_swap_in(ForgeServe* s, int64_t req_id);             /* cb2_swap_in */
/* cb2_peek_queue / cb2_find_request: 1 when the queue is empty / the id
 * is nowhere */
int forge_serve_peek_queue(const ForgeServe* s, ForgeServeRequest* out);
int forge_serve_find_request(const ForgeServe* s, int64_t req_id, ForgeServeRequest* out);
int64_t forge_serve_count_by_phase(const ForgeServe* s, int64_t phase);  /* cb2_count_by_phase */
int forge_serve_stats(const ForgeServe* s, ForgeServeStats* out);
int forge_serve_throughput(const ForgeServe* s, ForgeServeThroughput* out);
/* The tokens a request has generated so far (the request cb2_find_request
 * would return): up to cap of them into tokens, their count into *n. */
int forge_serve_output(const ForgeServe* s, int64_t req_id, int32_t* tokens, int64_t cap, int64_t* n);
/* Time spent in engine passes (ms, host clock around the synchronous
 * forge_b200_forward_rows calls) and the rows they carried. */
int forge_serve_engine_time(const ForgeServe* s, double* ms, int64_t* rows, int64_t* passes);

#ifdef __cplusplus
}
#endif
#endif
