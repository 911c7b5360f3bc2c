"""Decode throughput of the flame->forge hot path on B200.

Workload (default): 7B-shape int4 weight-only decode — 32 layers, d_model
4096, 32 heads x 128 (MHA), SwiGLU ffn 11008, vocab 32000, linear weights
int4 group-128 with bf16 scales, bf16 embeddings and LM head, batch 1, KV
context 2048 (synthetic N(0, 0.5) bf16 cache), greedy steps. Weights are
synthetic N(0, 0.02) generated on the device. A step is one greedy decode
step for every sequence; value = tokens/s over K timed steps (max over
ranks). Every step streams ~3.9 GB of weights+KV, far above the 126 MB L2,
so no flush is needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl forge|reference]

--impl reference times the CPU path (the oracle restatement of flame's
decode, OpenMP over the host cores) on a bounded sample of the same workload.
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

MODEL = dict(n_layer=32, d=4096, n_head=32, n_kv=32, hd=128, ffn=11008, vocab=32000)
CTX = 2048
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
    """The 7B gate/up int4 GEMV (N=22016, K=4096) via the per-op C-ABI entry
    for `batch` sequences (above 4: the batched paths, whose call includes the
    activation-quantising launch), rotating over `copies` weight sets
    (copies x 45 MB > L2) so every launch streams from HBM. Returns (avg ms
    per call, algorithmic bytes)."""
    lib = fb.lib()
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


def time_prefill(fb, torch, dev, B=8, H=32, S=4096, reps=10):
    """Causal flash-attention prefill on the tcgen05 kernel: bf16 Q/K/V
    ~N(0,1) [B][H][S][128] (805 MB, larger than L2). Algorithmic FLOPs:
    4 * B * H * S^2 * hd / 2 (causal half)."""
    q, k, v = (torch.randn(B, H, S, 128, device=dev).to(torch.bfloat16) for _ in range(3))
    o = torch.empty_like(q)
    lib = fb.lib()
    stream = torch.cuda.current_stream().cuda_stream
    run = lambda: lib.forge_flash_prefill(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B, H, S, 128, 1,
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
    flops = 4.0 * B * H * S * S * 128 / 2
    return {"workload": f"flash prefill B{B} H{H} S{S} hd128 causal bf16", "ms": ms, "tflops": flops / ms / 1e9,
            "peak_tflops": TC_PEAK, "frac": flops / ms / 1e9 / TC_PEAK, "peak_kind": "measured bf16 burst",
            "launches": reps}


def cpu_sample(batch, ctx, reps=2):
    """Oracle decode of the same 7B int4 shape on the host cores: one layer and
    the LM head are timed and the step extrapolated to 32 layers."""
    import numpy as np
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
    return {"value": batch / t_step, "unit": "tok/s", "cores": orc.lib().or_num_threads(), "kind": "port",
            "sample": f"oracle decode of 1 layer + LM head of the 7B int4 shape at ctx {ctx}, batch {batch}, "
                      f"best of {reps}; step = 32 x layer ({t_layer*1e3:.1f} ms) + head ({res[0]*1e3:.1f} ms)"}


def run_reference(args, world, rank):
    if rank != 0:
        return
    sample = cpu_sample(args.batch, CTX, reps=max(1, min(args.steps, 2)))
    v = sample["value"]
    print(json.dumps({
        "impl": "reference", "metric": "decode tok/s (7B-shape int4 g128, bs%d, ctx %d)" % (args.batch, CTX),
        "value": v, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "dtype": "int4 weights / f64 compute", "data": "synthetic",
        "config": {"workload": "7b_int4_decode", "batch": args.batch, "ctx": CTX},
        "cpu_baseline": sample, "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def tp_id(fb, pg, rank):
    """NCCL unique id made on rank 0 and shared over the host process group."""
    obj = [fb.tp_unique_id() if rank == 0 else None]
    pg.broadcast_object_list(obj, src=0)
    return obj[0]


def run_decode(fb, torch, pg, local, world, rank, B, K, W):
    """K timed greedy steps of the 7B int4 model at batch B (device-resident
    tokens), then K steps through the host C-ABI call (e2e). With N > 1
    processes the model is split tensor-parallel over the N GPUs (one NCCL
    all-reduce after the O and after the down projection)."""
    m = MODEL
    lmax = CTX + W + 2 * K + 8
    tp = dict(tp_rank=rank, tp_size=world, nccl_id=tp_id(fb, pg, rank)) if world > 1 else {}
    fm = fb.ForgeModel(m["n_layer"], m["d"], m["n_head"], m["n_kv"], m["hd"], m["ffn"], m["vocab"],
                       weight_kind=fb.FORGE_WEIGHT_Q4_G128, tied_head=False, max_batch=B, max_ctx=lmax,
                       device=local, **tp)
    fm.init_synthetic(1234, 0.02)
    fm.fill_kv_synthetic(99, CTX, 0.5)
    # warm-up (graph capture + replays)
    fm.decode_device(B, W)
    fm.sync()
    ctx_mid = CTX + W + K // 2
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
    # end-to-end through the host C-ABI call: H2D tokens, step, D2H next tokens
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
    step_bytes = fm.step_bytes(B, ctx_mid) * world  # every rank streams its shard
    launches = fm.launches_per_step(B) * K
    peak, peak_kind = peaks()
    step_gbs = step_bytes / (ms / 1e3) / 1e9
    fm.close()
    return {
        "batch": B, "value": value, "ms_per_step": ms, "clocks": clk.summary(),
        "hbm_roofline_step": {"bytes_per_step": step_bytes, "achieved_gbs": step_gbs, "peak_gbs": peak,
                              "frac": step_gbs / peak, "peak_kind": peak_kind,
                              "frac_of_8tbs_nominal": step_gbs / 8000.0},
        "e2e": {"value": B / (e2e_ms / 1e3), "unit": "tok/s", "h2d_bytes_per_step": 4 * B,
                "d2h_bytes_per_step": 4 * B, "ms_per_step": e2e_ms},
        "gpu_launches": launches,
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", default="forge", choices=["forge", "reference"])
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--also-batch", type=int, nargs="*", default=[32],
                    help="further batch sizes measured after the main one (reported under batch_sweep)")
    ap.add_argument("--only-gemv", action="store_true", help="run only the dominant GEMV (for profiling)")
    ap.add_argument("--only-prefill", action="store_true", help="run only the flash prefill (for profiling)")
    ap.add_argument("--no-prefill", action="store_true")
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
        # gate/up int4 GEMV (22016 x 4096) over 4 weight copies (180 MB), for
        # --batch sequences (32: the tensor-core path)
        ms, nbytes = time_dominant_gemv(fb, torch, dev, reps=3 if args.batch == 1 else 20, batch=args.batch)
        print(json.dumps({"kernel": f"int4 gemv 22016x4096 batch {args.batch}", "ms": ms, "bytes": nbytes,
                          "gbs": nbytes / ms / 1e6}))
        return
    if args.only_prefill:
        print(json.dumps(time_prefill(fb, torch, dev, B=4, H=16, S=4096, reps=2)))
        return
    B, K, W = args.batch, args.steps, max(3, args.warmup)
    r = run_decode(fb, torch, pg, local, world, rank, B, K, W)
    extra = []
    for B2 in args.also_batch:
        if B2 != B:
            r2 = run_decode(fb, torch, pg, local, world, rank, B2, max(3, K // 4), W)
            extra.append({k: r2[k] for k in ("batch", "value", "ms_per_step", "hbm_roofline_step", "e2e", "gpu_launches")})
    peak, peak_kind = peaks()
    gemv_ms, gemv_bytes = time_dominant_gemv(fb, torch, dev)
    achieved = gemv_bytes / (gemv_ms / 1e3) / 1e9
    prefill = None if args.no_prefill else time_prefill(fb, torch, dev)
    if rank != 0:
        return
    cpu = None if args.no_cpu else cpu_sample(B, CTX)
    B = r["batch"]
    out = {
        "metric": "decode tok/s (7B-shape int4 g128, bs%d, ctx %d)" % (B, CTX),
        "value": r["value"], "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": r["ms_per_step"], "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "int4 weights (g128 bf16 scales), bf16 KV/head, fp32 accumulate",
        "data": "synthetic",
        "config": {"workload": "7b_int4_decode", "n_layer": 32, "d_model": 4096, "heads": 32, "head_dim": 128,
                   "ffn": 11008, "vocab": 32000, "batch": B, "ctx": CTX,
                   "parallelism": f"tp{world}" if world > 1 else "single",
                   "l2": "inputs larger than L2 (3.9 GB streamed per step)"},
        "hbm_roofline_step": r["hbm_roofline_step"],
        "roofline": {"bound": "hbm", "kernel": "k_gemv<int4, gate/up 22016x4096>", "achieved": achieved,
                     "peak": peak, "unit": "GB/s", "frac": achieved / peak, "traffic": GEMV_TRAFFIC,
                     "peak_kind": peak_kind, "launch_ms": gemv_ms, "bytes_per_launch": gemv_bytes},
        "e2e": r["e2e"],
        "gpu_launches": r["gpu_launches"],
        "clocks": r["clocks"],
        "batch_sweep": extra,
        "prefill": prefill,
        "cpu_baseline": cpu,
    }
    print(json.dumps(out))


if __name__ == "__main__":
    main()
