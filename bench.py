"""Decode throughput of the flame->forge hot path on B200.

Headline workload: 7B-shape int4 weight-only decode — 32 layers, d_model
4096, 32 heads x 128 (MHA), SwiGLU ffn 11008, vocab 32000, linear weights
int4 group-128 with bf16 scales, bf16 embeddings and LM head, batch 1, KV
context 2048 (synthetic N(0, 0.5) bf16 cache), greedy steps. Weights are
synthetic N(0, 0.02) generated on the device. A step is one greedy decode
step for every sequence; value = tokens/s over K timed steps (max over
ranks). Every step streams ~4.7 GB of weights+KV, far above the 126 MB L2,
so no flush is needed between steps. With N > 1 processes the same model is
split tensor-parallel over the N GPUs.

batch_sweep: the 7B shape at batch 8 and 32, the 1B-shape bf16 GQA model
(16 layers, d 2048, 32/8 heads x 64, ffn 8192, context 1024) at batch 1, 8
and 32 and, at N > 1, the 13B-shape int4 model (40 layers, d 5120, 40 x 128,
ffn 13824, batch 64, context 4096; at N = 1 its 221.6 GB do not fit one
B200 and the entry says so). tp_parity (N > 1): greedy tokens and logits of
the tensor-parallel engine against one GPU.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl forge|reference]

--impl reference times the CPU path (the oracle restatement of flame's
decode, OpenMP over all host cores) on a bounded sample of the headline
workload; its line also carries the reference's own single-layer decode
check (cpu_ref, one core) where it was built.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "hexa-lang_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

WORKLOADS = {
    "7b_int4_decode": dict(n_layer=32, d=4096, n_head=32, n_kv=32, hd=128, ffn=11008, vocab=32000, q4=True, ctx=2048),
    "1b_bf16_decode": dict(n_layer=16, d=2048, n_head=32, n_kv=8, hd=64, ffn=8192, vocab=32000, q4=False, ctx=1024),
    "13b_int4_tp_decode": dict(n_layer=40, d=5120, n_head=40, n_kv=40, hd=128, ffn=13824, vocab=32000, q4=True,
                               ctx=4096),
}
MODEL = WORKLOADS["7b_int4_decode"]
CTX = MODEL["ctx"]
HBM_BYTES = 183359 * 2**20  # one B200 (nvidia-smi total)


def config_of(world, batch):
    """The headline workload's config dict (both arms print the same one)."""
    m = MODEL
    return {"workload": "7b_int4_decode", "n_layer": m["n_layer"], "d_model": m["d"], "heads": m["n_head"],
            "head_dim": m["hd"], "ffn": m["ffn"], "vocab": m["vocab"], "batch": batch, "ctx": CTX,
            "parallelism": f"tp{world}" if world > 1 else "single",
            "l2": "inputs larger than L2 (4.7 GB streamed per step)"}
# dram__bytes_read.sum + dram__bytes_write.sum of one k_gemv launch (int4
# gate/up 22016 x 4096, batch 1) from an ncu capture of this kernel alone
# (46.56 MB read + 0.05 MB written).
GEMV_TRAFFIC = 46558720 + 51968


def _tc_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"])
    except Exception:
        return 1590.0


TC_PEAK = _tc_peak()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks sampled every 200 ms while the timed region runs."""

    def __init__(self, index):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if len(r) > 8 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) > 8 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows if len(r) > 8 for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
        pg = dist
    return world, rank, local, pg


def max_over_ranks(pg, v):
    if pg is None:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


def barrier(pg):
    if pg is not None:
        pg.barrier()


def time_dominant_gemv(fb, torch, dev, K=4096, N=2 * 11008, copies=4, reps=20, batch=1):
    """The 7B gate/up int4 GEMV (N=22016 rows, K=4096; under tensor
    parallelism this rank's row shard) via the per-op C-ABI entry for `batch`
    sequences (above 4: the batched paths, whose call includes the
    activation-quantising launch), rotating over `copies` weight sets (more
    than L2 in total) so every launch streams from HBM. Returns (avg ms per
    call, algorithmic bytes)."""
    lib = fb.lib()
    copies = max(copies, -(-4 * 2**27 // max(1, N * K // 2)))  # > 512 MB in total
    ws = []
    for c in range(copies):
        w = torch.empty((N, K), dtype=torch.int16, device=dev)
        fb.check(lib.forge_fill_normal_bf16(w.data_ptr(), N * K, 77, c << 40, 0.02, 0), "fill")
        ws.append(fb.q4_pack(w)[2:])
        del w
    x = torch.randn(batch, K, device=dev)
    y = torch.empty(batch, N, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    for i in range(6):
        t, s = ws[i % copies]
        fb.check(lib.forge_gemv_w4a16_g128(t.data_ptr(), s.data_ptr(), N, K, x.data_ptr(), batch, y.data_ptr(), 1,
                                           stream), "gemv")
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(reps):
        t, s = ws[i % copies]
        lib.forge_gemv_w4a16_g128(t.data_ptr(), s.data_ptr(), N, K, x.data_ptr(), batch, y.data_ptr(), 1, stream)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    nbytes = lib.forge_q4_tile_bytes(N, K) + lib.forge_q4_scale_tile_bytes(N, K, 128) + batch * (4 * K + 4 * N)
    return ms, nbytes


def time_prefill(fb, torch, dev, B=8, H=32, S=4096, reps=10, hd=128):
    """Causal flash-attention prefill on the tcgen05 kernel: bf16 Q/K/V
    ~N(0,1) [B][H][S][hd] (805 MB at hd 128, larger than L2). Algorithmic
    FLOPs: 4 * B * H * S^2 * hd / 2 (causal half)."""
    q, k, v = (torch.randn(B, H, S, hd, device=dev).to(torch.bfloat16) for _ in range(3))
    o = torch.empty_like(q)
    lib = fb.lib()
    stream = torch.cuda.current_stream().cuda_stream
    run = lambda: lib.forge_flash_prefill(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B, H, S, hd, 1,
                                          stream)
    for _ in range(3):
        fb.check(run(), "prefill")
    torch.cuda.synchronize()
    fb.check(lib.forge_ops_check(), "prefill error word")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    flops = 4.0 * B * H * S * S * hd / 2
    return {"workload": f"flash prefill B{B} H{H} S{S} hd{hd} causal bf16", "ms": ms, "tflops": flops / ms / 1e9,
            "peak_tflops": TC_PEAK, "frac": flops / ms / 1e9 / TC_PEAK, "peak_kind": "measured bf16 burst",
            "launches": reps}


def time_model_prefill(fb, torch, local, n_prompt=2048, batch=1, reps=3):
    """Model-level prompt prefill (forge_b200_prefill) of the 7B int4 model:
    batch x n_prompt positions through all 32 layers in one pass (K/V
    written), then the LM head of the last position; wall clock around the
    synchronous call, best of reps. Weight bytes per 32-row chunk of the
    batched GEMVs are the floor of this path: tokens/s and the implied
    weight-stream rate are reported."""
    import numpy as np
    m = MODEL
    fm = fb.ForgeModel(m["n_layer"], m["d"], m["n_head"], m["n_kv"], m["hd"], m["ffn"], m["vocab"],
                       weight_kind=fb.FORGE_WEIGHT_Q4_G128, max_batch=batch, max_ctx=n_prompt + 8, device=local)
    fm.init_synthetic(1234, 0.02)
    prompt = np.random.default_rng(3).integers(0, m["vocab"], (batch, n_prompt)).astype(np.int32)
    fm.prefill(prompt)  # buffers, batched paths
    best = 1e9
    for _ in range(reps):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        fm.prefill(prompt)
        best = min(best, time.perf_counter() - t0)
    wbytes = fm.step_bytes(1, 0)
    fm.close()
    rows = batch * n_prompt
    chunks = -(-rows // 32)
    return {"workload": f"7b_int4 prompt prefill B{batch} x {n_prompt}", "ms": best * 1e3,
            "value": rows / best, "unit": "prompt tok/s (wall clock, synchronous call)",
            "weight_passes": chunks, "weight_gbs": chunks * wbytes / best / 1e9}


def all_cores():
    """Host threads for the CPU legs: every core the process may run on
    (torchrun sets OMP_NUM_THREADS=1 for its workers; the CPU legs run on
    one rank only, so they take the whole host)."""
    try:
        n = len(os.sched_getaffinity(0))
    except Exception:
        n = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(n)
    return n


def cpu_sample(batch, ctx, reps=2):
    """Oracle decode of the same 7B int4 shape on the host cores: one layer and
    the LM head are timed and the step extrapolated to 32 layers."""
    import oracle as orc
    m = MODEL
    res = {}
    for nl in (0, 1):
        om = orc.OracleModel(nl, m["d"], m["n_head"], m["n_kv"], m["hd"], m["ffn"], m["vocab"], q4=True, tied=False)
        kc, vc = om.new_cache(batch, ctx + 1)
        kc[...] = 0.1
        vc[...] = 0.1
        ts = []
        for r in range(reps):
            t0 = time.perf_counter()
            om.decode_step(kc, vc, [1] * batch, [ctx] * batch)
            ts.append(time.perf_counter() - t0)
        res[nl] = min(ts)
        del om, kc, vc
    t_layer = max(res[1] - res[0], 1e-9)
    t_step = m["n_layer"] * t_layer + res[0]
    out = {"value": batch / t_step, "unit": "tok/s", "cores": orc.lib().or_num_threads(), "kind": "port",
           "sample": f"oracle decode of 1 layer + LM head of the 7B int4 shape at ctx {ctx}, batch {batch}, "
                     f"best of {reps}; step = 32 x layer ({t_layer*1e3:.1f} ms) + head ({res[0]*1e3:.1f} ms)"}
    ref = cpu_ref_sample()
    if ref:
        out["reference_cpu_ref"] = ref
    return out


def cpu_ref_sample(lengths=(256, 1024, 2048)):
    """The reference's own f64 single-layer decode check, cpu_ref
    (tool/decode_eager_baseline.cu:160-198: d 768, 12 x 64 MHA, ffn 3072,
    single thread), built from the reference source into oracle/_ref where
    the reference tree was present; ms per layer at the given cache lengths."""
    import numpy as np
    import oracle as orc
    R = orc.ref_lib()
    if R is None:
        return None
    keys = ("x", "g1", "g2", "Wq", "Wk", "Wv", "Wo", "Wg", "Wu", "Wd", "Kc", "Vc")
    res = {}
    for L in lengths:
        inp = orc.ref_inputs(L)
        bufs = [np.ascontiguousarray(inp[k]) for k in keys]
        y = np.empty(orc.REF_D, np.float64)
        ts = []
        for _ in range(2):
            t0 = time.perf_counter()
            R.ref_cpu_ref(*[b.ctypes.data for b in bufs], L, y.ctypes.data)
            ts.append(time.perf_counter() - t0)
        res[str(L)] = min(ts) * 1e3
    return {"unit": "ms per layer", "cores": 1, "kind": "reference",
            "shape": "d 768, 12 x 64 MHA, ffn 3072, f64 (the reference's fixed check shape)", "ms_by_ctx": res}


def run_reference(args, world, rank):
    if rank != 0:
        return
    cores = all_cores()
    sample = cpu_sample(args.batch, CTX, reps=max(1, min(args.steps, 2)))
    sample["cores"] = cores
    v = sample["value"]
    print(json.dumps({
        "impl": "reference", "metric": "decode tok/s (7B-shape int4 g128, bs%d, ctx %d)" % (args.batch, CTX),
        "value": v, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "dtype": "int4 weights / f64 compute", "data": "synthetic",
        "config": config_of(world, args.batch),
        "cpu_baseline": sample, "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def tp_id(fb, pg, rank):
    """NCCL unique id made on rank 0 and shared over the host process group."""
    obj = [fb.tp_unique_id() if rank == 0 else None]
    pg.broadcast_object_list(obj, src=0)
    return obj[0]


def model_bytes(m, B, ctx):
    """Weights + KV cache of a workload on one GPU (for the does-not-fit check)."""
    lin = m["n_layer"] * ((m["n_head"] + 2 * m["n_kv"]) * m["hd"] * m["d"] + m["n_head"] * m["hd"] * m["d"] +
                          3 * m["ffn"] * m["d"])
    w = lin * (0.5 + 2 / 128) if m["q4"] else lin * 2
    kv = 2 * m["n_layer"] * B * m["n_kv"] * m["hd"] * 2 * (ctx + 64)
    return w + 2 * m["vocab"] * m["d"] * 2 + kv


def run_decode(fb, torch, pg, local, world, rank, B, K, W, name="7b_int4_decode", e2e=True):
    """K timed greedy steps of workload `name` at batch B (device-resident
    tokens), then K steps through the host C-ABI call (e2e). With N > 1
    processes the model is split tensor-parallel over the N GPUs (one
    all-reduce after the O and after the down projection)."""
    m = WORKLOADS[name]
    ctx = m["ctx"]
    lmax = ctx + W + 2 * K + 8
    tp = dict(tp_rank=rank, tp_size=world, nccl_id=tp_id(fb, pg, rank)) if world > 1 else {}
    fm = fb.ForgeModel(m["n_layer"], m["d"], m["n_head"], m["n_kv"], m["hd"], m["ffn"], m["vocab"],
                       weight_kind=fb.FORGE_WEIGHT_Q4_G128 if m["q4"] else fb.FORGE_WEIGHT_BF16, tied_head=False,
                       max_batch=B, max_ctx=lmax, device=local, **tp)
    fm.init_synthetic(1234, 0.02)
    fm.fill_kv_synthetic(99, ctx, 0.5)
    # warm-up (graph capture + replays)
    fm.decode_device(B, W)
    fm.sync()
    ctx_mid = ctx + W + K // 2
    stream = torch.cuda.ExternalStream(fm.stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(pg)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e0.record(stream)
        fm.decode_device(B, K)
        e1.record(stream)
        fm.sync()
    barrier(pg)
    ms = e0.elapsed_time(e1) / K
    ms = max_over_ranks(pg, ms)
    value = B / (ms / 1e3)  # the N ranks decode the same B sequences together
    out = {"workload": name, "batch": B, "ctx": ctx, "value": value, "unit": "tok/s", "ms_per_step": ms,
           "clocks": clk.summary()}
    if e2e:
        # end to end through the host C-ABI call: H2D tokens, step, D2H next tokens
        toks = [1] * B
        for _ in range(3):
            toks = fm.step(toks)
        torch.cuda.synchronize()
        barrier(pg)
        t0 = time.perf_counter()
        e2 = torch.cuda.Event(enable_timing=True)
        e3 = torch.cuda.Event(enable_timing=True)
        e2.record(stream)
        for _ in range(K):
            toks = fm.step(toks)
        e3.record(stream)
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) / K * 1e3
        e2e_ms = max(e2.elapsed_time(e3) / K, wall)
        e2e_ms = max_over_ranks(pg, e2e_ms)
        out["e2e"] = {"value": B / (e2e_ms / 1e3), "unit": "tok/s", "h2d_bytes_per_step": 4 * B,
                      "d2h_bytes_per_step": 4 * B, "ms_per_step": e2e_ms}
    # this rank's shard bytes; the whole job streams world x that
    rank_bytes = fm.step_bytes(B, ctx_mid)
    total = max_over_ranks(pg, rank_bytes) * world
    peak, peak_kind = peaks()
    gbs = total / (ms / 1e3) / 1e9
    out["hbm_roofline_step"] = {"bytes_per_step": total, "achieved_gbs": gbs, "peak_gbs": peak * world,
                                "frac": gbs / (peak * world), "per_gpu_frac": gbs / world / peak,
                                "peak_kind": peak_kind, "frac_of_8tbs_nominal": gbs / world / 8000.0}
    out["gpu_launches"] = fm.launches_per_step(B) * K
    fm.close()
    return out


def run_serve(fb, torch, local, n_req=64, max_batch=32, seed=5):
    """Continuous batching (forge_serve over the 7B int4 model): n_req
    requests with prompts of 64-512 tokens and 32-128 generated tokens, half
    queued at the start and the rest arriving 4 per iteration, max_batch
    running at once, a KV budget that never preempts. Wall clock (host) around
    the whole run: scheduling, one ragged engine pass per iteration (prompt
    rows of the admitted requests + one row per decoding request), H2D of the
    rows and D2H of the next tokens. Tokens generated / second."""
    import numpy as np
    m = MODEL
    fm = fb.ForgeModel(m["n_layer"], m["d"], m["n_head"], m["n_kv"], m["hd"], m["ffn"], m["vocab"],
                       weight_kind=fb.FORGE_WEIGHT_Q4_G128, max_batch=max_batch, max_ctx=640, device=local)
    fm.init_synthetic(1234, 0.02)
    rng = np.random.default_rng(seed)
    reqs = [(rng.integers(0, m["vocab"], int(rng.integers(64, 513))).astype(np.int32), int(rng.integers(32, 129)))
            for _ in range(n_req)]

    def one_run(rs):
        sv = fb.ForgeServe(fm, max_batch, max_batch * 640)
        pending = list(enumerate(rs))
        for rid, (p, g) in pending[:len(rs) // 2]:
            sv.add_request(rid, max_gen=g, prompt=p)
        pending = pending[len(rs) // 2:]
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        step = 0
        while True:
            for rid, (p, g) in pending[:4]:
                sv.add_request(rid, max_gen=g, prompt=p)
            pending = pending[4:]
            st = sv.stats()
            if not pending and st["queue_size"] == 0 and st["running_count"] == 0:
                break
            sv.run_step(step)
            step += 1
        wall = time.perf_counter() - t0
        out = sv.throughput(), sv.engine_time(), wall, step
        sv.close()
        return out

    one_run(reqs[:8])  # warm-up: buffers and the batched paths
    thr, (eng_ms, rows, passes), wall, steps = one_run(reqs)
    fm.close()
    gen = sum(g for _, g in reqs)
    assert thr["total_tokens"] == gen
    return {"workload": "7b_int4 continuous batching (forge_serve)", "requests": n_req, "max_batch": max_batch,
            "prompt_tokens": int(sum(len(p) for p, _ in reqs)), "generated_tokens": gen,
            "value": gen / wall, "unit": "generated tok/s (wall clock)", "wall_s": wall, "iterations": steps,
            "engine_ms": eng_ms, "engine_rows": rows, "engine_passes": passes,
            "tokens_per_step": thr["tokens_per_step"], "avg_latency_steps": thr["avg_latency"],
            "avg_wait_steps": thr["avg_wait_time"]}


def tp_parity(fb, torch, pg, local, world, rank):
    """Greedy tokens and logits of the tensor-parallel engine against one GPU
    (rank 0) with the same seeded weights: a small GQA int4 model (2 layers,
    d 512, 8/2 heads x 64, ffn 1536, vocab 2000; 6 logit steps at batch 2 and
    32 greedy tokens), and the first 8 greedy tokens of the 7B shape."""
    import numpy as np
    cases = [("small_gqa_int4", dict(cfg=(2, 512, 8, 2, 64, 1536, 2000), std=0.05, n_gen=32, batch=2, steps=6)),
             ("7b_int4", dict(cfg=(32, 4096, 32, 32, 128, 11008, 32000), std=0.02, n_gen=8, batch=1, steps=0))]
    prompts = np.array([[3, 17, 5, 99], [8, 2, 64, 1]], np.int32)
    res = {"ok": True, "n_ranks": world}

    def run(cfg, kw, tp):
        B = kw["batch"]
        fm = fb.ForgeModel(*cfg, weight_kind=fb.FORGE_WEIGHT_Q4_G128, max_batch=B, max_ctx=64, device=local, **tp)
        fm.init_synthetic(1234, kw["std"])
        gen = fm.generate(prompts[:B], kw["n_gen"])
        fm.reset()
        toks, lgs = prompts[:B, 0].copy(), []
        for _ in range(kw["steps"]):
            toks, lg = fm.step(toks, want_logits=True)
            lgs.append(lg)
        fm.close()
        return gen, (np.stack(lgs) if lgs else None)

    for name, kw in cases:
        gen, lgs = run(kw["cfg"], kw, dict(tp_rank=rank, tp_size=world, nccl_id=tp_id(fb, pg, rank)))
        ok_local = 1.0
        entry = {}
        if rank == 0:
            rg, rl = run(kw["cfg"], kw, {})
            tok_ok = bool(np.array_equal(gen, rg))
            entry = {"tokens_equal": tok_ok, "n_tokens": int(gen.size)}
            if lgs is not None:
                scale = float(np.abs(rl).max())
                err = float(np.abs(lgs - rl).max())
                entry.update(max_abs_logit_err=err, logit_scale=scale, bound=2e-3 * scale)
                tok_ok = tok_ok and err <= 2e-3 * scale
            ok_local = 1.0 if tok_ok else 0.0
            res[name] = entry
        ok_all = -max_over_ranks(pg, -ok_local)
        res["ok"] = res["ok"] and ok_all > 0.5
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", default="forge", choices=["forge", "reference"])
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="headline workload only")
    ap.add_argument("--only-gemv", action="store_true", help="run only the dominant GEMV (for profiling)")
    ap.add_argument("--only-prefill", action="store_true", help="run only the flash prefill (for profiling)")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-serve", action="store_true")
    ap.add_argument("--only-serve", action="store_true", help="run only the continuous-batching workload")
    ap.add_argument("--only-step", default=None, metavar="WORKLOAD",
                    help="run only --warmup + --steps decode steps of WORKLOAD at --batch (for profiling)")
    ap.add_argument("--ctx", type=int, default=None, help="KV context of --only-step (default: the workload's)")
    ap.add_argument("--layers", type=int, default=None, help="layers of --only-step (default: the workload's)")
    args = ap.parse_args()
    world, rank, local, pg = dist_setup()
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    import torch
    import forge_b200 as fb
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.only_gemv:
        # the dominant kernel alone, for profiling: a few launches of the 7B
        # gate/up int4 GEMV (22016 x 4096) over several weight copies, for
        # --batch sequences (32: the tensor-core path)
        ms, nbytes = time_dominant_gemv(fb, torch, dev, reps=3 if args.batch == 1 else 20, batch=args.batch)
        print(json.dumps({"kernel": f"int4 gemv 22016x4096 batch {args.batch}", "ms": ms, "bytes": nbytes,
                          "gbs": nbytes / ms / 1e6}))
        return
    if args.only_prefill:
        print(json.dumps(time_prefill(fb, torch, dev, B=4, H=16, S=4096, reps=2)))
        return
    if args.only_serve:
        print(json.dumps(run_serve(fb, torch, local)))
        print(json.dumps(time_model_prefill(fb, torch, local)))
        return
    if args.only_step:
        m = WORKLOADS[args.only_step]
        ctx = args.ctx or m["ctx"]
        fm = fb.ForgeModel(args.layers or m["n_layer"], m["d"], m["n_head"], m["n_kv"], m["hd"], m["ffn"], m["vocab"],
                           weight_kind=fb.FORGE_WEIGHT_Q4_G128 if m["q4"] else fb.FORGE_WEIGHT_BF16,
                           max_batch=args.batch, max_ctx=ctx + args.warmup + args.steps + 8, device=local)
        fm.init_synthetic(1234, 0.02)
        fm.fill_kv_synthetic(99, ctx, 0.5)
        fm.decode_device(args.batch, args.warmup)
        fm.sync()
        t0 = time.perf_counter()
        fm.decode_device(args.batch, args.steps)
        fm.sync()
        print(json.dumps({"workload": args.only_step, "layers": args.layers or m["n_layer"], "batch": args.batch,
                          "ctx": ctx, "steps": args.steps,
                          "ms_per_step_wall": (time.perf_counter() - t0) * 1e3 / max(1, args.steps),
                          "launches_per_step": fm.launches_per_step(args.batch)}))
        fm.close()
        return
    B, K, W = args.batch, args.steps, max(3, args.warmup)
    r = run_decode(fb, torch, pg, local, world, rank, B, K, W)
    sweep = []
    if not args.no_sweep:
        K2 = max(3, K // 4)
        plan = [("7b_int4_decode", b) for b in (8, 32) if b != B]
        plan += [("1b_bf16_decode", b) for b in (1, 8, 32)]
        plan.append(("13b_int4_tp_decode", 64))
        for name, b2 in plan:
            m = WORKLOADS[name]
            if model_bytes(m, b2, m["ctx"]) / world > 0.95 * HBM_BYTES:
                sweep.append({"workload": name, "batch": b2, "ctx": m["ctx"], "value": None,
                              "unavailable": f"does not fit: {model_bytes(m, b2, m['ctx']) / 1e9:.1f} GB of weights "
                                             f"and KV cache over {world} GPU(s) of {HBM_BYTES / 1e9:.0f} GB"})
                continue
            r2 = run_decode(fb, torch, pg, local, world, rank, b2, K2, W, name=name, e2e=False)
            sweep.append({k: r2[k] for k in ("workload", "batch", "ctx", "value", "unit", "ms_per_step",
                                             "hbm_roofline_step", "gpu_launches")})
    parity = tp_parity(fb, torch, pg, local, world, rank) if world > 1 else None
    peak, peak_kind = peaks()
    # the dominant kernel: gate/up GEMV (at N > 1 this rank's row shard)
    rows = 2 * (fb.tp_split(MODEL["ffn"], 128, rank, world)[1] if world > 1 else MODEL["ffn"])
    gemv_ms, gemv_bytes = time_dominant_gemv(fb, torch, dev, N=rows)
    gemv_ms = max_over_ranks(pg, gemv_ms)
    achieved = gemv_bytes / (gemv_ms / 1e3) / 1e9
    prefill = None if (args.no_prefill or world > 1) else time_prefill(fb, torch, dev)
    if prefill is not None:
        prefill["hd64"] = time_prefill(fb, torch, dev, hd=64)
    serve = None if (args.no_serve or world > 1) else run_serve(fb, torch, local)
    model_prefill = None if (args.no_prefill or world > 1) else time_model_prefill(fb, torch, local)
    if rank != 0:
        return
    cpu = None
    if not args.no_cpu and world == 1:
        cores = all_cores()
        cpu = cpu_sample(B, CTX)
        cpu["cores"] = cores
    out = {
        "metric": "decode tok/s (7B-shape int4 g128, bs%d, ctx %d)" % (B, CTX),
        "value": r["value"], "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": r["ms_per_step"], "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "int4 weights (g128 bf16 scales), bf16 KV/head, fp32 accumulate",
        "data": "synthetic",
        "config": config_of(world, B),
        "hbm_roofline_step": r["hbm_roofline_step"],
        "roofline": {"bound": "hbm", "kernel": f"k_gemv<int4, gate/up {rows}x4096>", "achieved": achieved,
                     "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": GEMV_TRAFFIC if world == 1 else None,
                     "peak_kind": peak_kind, "launch_ms": gemv_ms, "bytes_per_launch": gemv_bytes},
        "e2e": r["e2e"],
        "gpu_launches": r["gpu_launches"],
        "clocks": r["clocks"],
        "batch_sweep": sweep,
        "tp_parity": parity,
        "prefill": prefill,
        "serve": serve,
        "model_prefill": model_prefill,
        "cpu_baseline": cpu,
    }
    print(json.dumps(out))


if __name__ == "__main__":
    main()
