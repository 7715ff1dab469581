#!/usr/bin/env python
"""Decode throughput of Minima's token loop on B200 (one process per GPU).

Headline workload (per GPU; weak scaling across GPUs): the Minima default
decoder (config.h defaults: V=30000, D=128, 8 layers, 4 heads / 2 KV heads,
FFN 512; 5,808,256 fp32 parameters) with seeded model_init_config weights
(seed 1), max_seq 512, batch 4 x (prompt of 128 uniform non-special ids, then
256 greedy tokens) — the reference's training shape as prefill followed by
decode.  One step = one generate_with_options call for the batch (prefill +
decode, one device launch for the token loop).  metric = generated tokens /
second.

* value: device-resident inputs (mc_generate with MC_DEVICE_POINTERS), timed
  with CUDA events on the session's stream, L2 flushed (256 MiB write)
  before every timed step and excluded from the timing.
* e2e:   the drop-in generate_batch_with_options with host buffers (prompt
  upload and id download inside the timed region), host wall clock.
* roofline: algorithmic bytes of the token-loop launch (weights read once
  per token step + KV cache reads/appends) / its CUDA-event duration,
  against the measured HBM copy bandwidth; roofline_l2 gives the same
  numerator against an L2 read bandwidth measured in the same process
  (the 23 MB model is L2-resident after the first token step).
* cpu_baseline: the reference's own generate() (oracle/_ref, built from its
  unmodified C files), one thread, on a bounded sample.
* configs: the other decode workloads of the scope, measured in the same
  run (unless --no-extra): config 1 (B=1 latency), config 3 (118M fp32, B=64,
  T=0.8 top-k 40), config 4 per GPU (411M bf16, 32 sequences per GPU, the
  tensor-core batched decode) and config 5 (prompt 1900; 8 sequences split
  over the ranks).
--impl reference runs the reference's CPU implementation instead (the
reference arm): that process loads only oracle/ libraries.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WL = dict(vocab=30000, dim=128, n_layers=8, n_heads=4, ffn_dim=512, max_seq=512, seed=1,
          batch=4, prompt=128, new_tokens=256)
WORKLOAD_NAME = ("minima-default-5.8M fp32: 4 seq x (prefill 128 random ids + 256 greedy), "
                 "seed 1, max_seq 512")
METRIC = "decode tokens/s (generated ids per second, prefill included)"
UNIT = "tokens/s"
FALLBACK_HBM_GBS = 6650.0
L2_NOTE = "flushed (256 MiB write) before each timed step, outside the timing"

# The other decode workloads of the scope.  "batch" is per GPU except for
# config 5, whose 8 sequences are split over the ranks (strong scaling).
# decode/prefill select the kernels (MINIMA_CUDA_DECODE / _PREFILL).
EXTRA = {
    "c1": dict(name="config 1: default 5.8M fp32, B=1, prompt 32, 128 greedy, seed 0",
               vocab=30000, dim=128, n_layers=8, n_heads=4, ffn_dim=512, max_seq=512, seed=0,
               batch=1, prompt=32, new_tokens=128, bf16=False, decode="", prefill="",
               sampling=dict(top_k=1), prompt_seed=100, flush=True),
    "c3": dict(name="config 3: 12L/768/12H/F3072/V16384 fp32, B=64/GPU, prompt 256, "
                    "512 tokens T=0.8 top-k 40, seed 2",
               vocab=16384, dim=768, n_layers=12, n_heads=12, ffn_dim=3072, max_seq=1024, seed=2,
               batch=64, prompt=256, new_tokens=512, bf16=False, decode="tcgen05",
               prefill="tcgen05", sampling=dict(temperature=0.8, top_k=40), prompt_seed=2000,
               flush=False),
    "c4": dict(name="config 4 per GPU: 24L/1024/16H/F4096/V32768 bf16, 32 seq/GPU, prompt 512, "
                    "256 greedy, seed 3",
               vocab=32768, dim=1024, n_layers=24, n_heads=16, ffn_dim=4096, max_seq=2048, seed=3,
               batch=32, prompt=512, new_tokens=256, bf16=True, decode="tcgen05",
               prefill="tcgen05", sampling=dict(top_k=1), prompt_seed=3000, flush=False),
    "c5": dict(name="config 5: same 24L/1024 bf16 model, 8 seq split over the GPUs, prompt 1900, "
                    "148 greedy",
               vocab=32768, dim=1024, n_layers=24, n_heads=16, ffn_dim=4096, max_seq=2048, seed=3,
               batch=8, prompt=1900, new_tokens=148, bf16=True, decode="tcgen05",
               prefill="tcgen05", sampling=dict(top_k=1), prompt_seed=5000, flush=False,
               split=True),
}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="measure the headline workload only (no config 1/3/4/5 fields)")
    ap.add_argument("--extra-steps", type=int, default=3)
    ap.add_argument("--extra-warmup", type=int, default=2)
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def workload_config(world):
    """The `config` object both arms print (same keys, same values)."""
    return {"workload": WORKLOAD_NAME, "global_batch": WL["batch"] * world,
            "seq_len": WL["prompt"] + WL["new_tokens"], "parallelism": f"dp{world}",
            "l2": L2_NOTE, "per_gpu_batch": WL["batch"]}


def prompt_ids(n, vocab, seed):
    """Uniform non-special ids in [4, vocab-1] from rng_int (util.c:29-33),
    through this repository's host library (native arm)."""
    import ctypes as C
    import numpy as np
    import minima_b200 as M
    host = M.libs()[0]
    r = M.Rng()
    host.rng_seed(C.byref(r), seed)
    return np.array([host.rng_int(C.byref(r), 4, vocab - 1) for _ in range(n)], dtype=np.uint16)


def workload_prompts(first_seq, count, draw=None):
    """Prompts of global sequences first_seq .. first_seq+count-1: sequence g
    gets prompt seed 1000 + g and RNG state g + 1, whichever rank runs it."""
    import numpy as np
    draw = draw or prompt_ids
    prompts = np.stack([draw(WL["prompt"], WL["vocab"], 1000 + g)
                        for g in range(first_seq, first_seq + count)])
    rng = [g + 1 for g in range(first_seq, first_seq + count)]
    return prompts, rng


def max_over_ranks(pg, values, device):
    """Element-wise MAX of per-rank timings (the slowest rank sets the time)."""
    import torch
    t = torch.tensor(values, dtype=torch.float64, device=device)
    if pg is not None:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return [float(v) for v in t]


def whole_job_rate(world, tokens_per_rank, max_seconds):
    """Aggregate generated tokens/s over all ranks (weak scaling: every rank
    decodes its own, disjoint sequences)."""
    return world * tokens_per_rank / max_seconds


def kv_heads(H):
    K = H // 2 if H > 1 else 1
    while H % K:
        K -= 1
    return K


def algorithmic_bytes(P, nnew, B, t0=0, weight_bytes_per=4, wl=None):
    """Bytes the token-loop launch must move for positions t0..T-1: every
    token step reads the layer weights, steps that produce logits read the
    tied lm_head, and every active sequence reads its K/V rows 0..t and
    appends row t (fp32)."""
    wl = wl or WL
    V, D, L, H, F = wl["vocab"], wl["dim"], wl["n_layers"], wl["n_heads"], wl["ffn_dim"]
    K = kv_heads(H)
    hd = D // H
    kvd = K * hd
    Q = D + 2 * kvd
    w_layers = L * (Q * D + D * D + 3 * F * D) * weight_bytes_per + 2 * L * D * 4
    w_head = V * D * weight_bytes_per + D * 4
    total = 0
    T = P + nnew - 1
    for t in range(t0, T):
        total += w_layers
        if t >= P - 1:
            total += w_head
        total += B * (L * 2 * (t + 1) * kvd * 4 + D * weight_bytes_per)
    return total


def profiled_traffic(kernel_name):
    """DRAM bytes per launch of `kernel_name` from the ncu summaries under
    profiles/ (one *_traffic.json per captured kernel); None when that kernel
    has no capture."""
    import glob
    for tf in sorted(glob.glob(os.path.join(ROOT, "profiles", "*_traffic.json"))):
        with open(tf) as fh:
            rec = json.load(fh)
        if rec.get("kernel", "").split("<")[0] == (kernel_name or "").split("<")[0]:
            return rec.get("dram_bytes_per_launch")
    return None


def measured_hbm():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def measure_l2_read_gbs(dev, mib=24, reps=200):
    """Read bandwidth of an L2-resident buffer (the size of the default
    model's weights): the best of a sum reduction and a copy over `mib` MiB,
    repeated `reps` times back to back, CUDA events on the current stream."""
    import torch
    n = mib * (1 << 20) // 4
    a = torch.rand(n, device=dev)
    b = torch.empty_like(a)
    out = torch.empty(1, device=dev)
    best = 0.0
    for kind in ("sum", "copy"):
        for _ in range(10):
            torch.sum(a, dim=0, keepdim=True, out=out) if kind == "sum" else b.copy_(a)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            torch.sum(a, dim=0, keepdim=True, out=out) if kind == "sum" else b.copy_(a)
        e1.record()
        torch.cuda.synchronize()
        s = e0.elapsed_time(e1) / 1e3
        moved = reps * n * 4 * (1 if kind == "sum" else 2)
        best = max(best, moved / s / 1e9)
    del a, b
    return best


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(gpu_index), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [[c.strip() for c in l.split(",")] for l in out.splitlines() if l.strip()]
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        if not sm:
            return None
        maxc = float(rows[0][2])
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v == "Active"})
        loaded = [s for s in sm if s > 0.5 * maxc] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": maxc, "reasons": reasons,
                "samples": len(sm)}


def reference_model(O):
    dims = O.Dims(WL["vocab"], WL["dim"], WL["n_layers"], WL["n_heads"], WL["ffn_dim"],
                  WL["max_seq"])
    if O.ref_available():
        return O.RefModel(dims, WL["seed"]), "reference", O.ref_random_prompt
    return O.OrcModel(dims, WL["seed"]), "port", O.random_prompt


def cpu_baseline(steps_budget_s=20.0):
    """The reference's generate() (oracle/_ref) on one host core, on the
    whole batch of one step (4 sequences back to back)."""
    from oracle import oracle as O
    model, kind, draw = reference_model(O)
    prompts, rng = workload_prompts(0, WL["batch"], draw)
    opts = O.make_options(top_k=1, max_new_tokens=WL["new_tokens"])
    toks, t0 = 0, time.perf_counter()
    n_seq = 0
    for b in range(WL["batch"]):
        ids = model.generate(prompts[b], WL["max_seq"], WL["max_seq"], opts, rng[b])[0]
        toks += len(ids) - WL["prompt"]
        n_seq += 1
        if time.perf_counter() - t0 > steps_budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": toks / dt, "unit": UNIT, "cores": 1, "kind": kind,
            "sample": f"{n_seq} of the step's sequences (prompt {WL['prompt']} + "
                      f"{WL['new_tokens']} greedy), reference generate(), gcc -O2, 1 thread, "
                      f"{dt:.1f} s"}


def reference_arm(args):
    """The reference's own generate() on the host cores, for the whole job's
    sequences (every rank's batch), one thread per sequence.  Runs on rank 0
    alone; loads oracle/ libraries only (no minima_b200 import)."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from concurrent.futures import ThreadPoolExecutor
    from oracle import oracle as O
    model, kind, draw = reference_model(O)
    n_seq = WL["batch"] * world
    threads = min(n_seq, os.cpu_count() or 1)
    prompts, rng = workload_prompts(0, n_seq, draw)
    opts = O.make_options(top_k=1, max_new_tokens=WL["new_tokens"])

    def one(b):
        return len(model.generate(prompts[b], WL["max_seq"], WL["max_seq"], opts, rng[b])[0])

    times, toks = [], 0
    with ThreadPoolExecutor(threads) as ex:
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            n = sum(ex.map(one, range(n_seq)))
            dt = time.perf_counter() - t0
            if i >= args.warmup:
                times.append(dt)
                toks += n - n_seq * WL["prompt"]
    total = sum(times)
    value = toks / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": workload_config(world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": f"each step: the job's {n_seq} sequences, one per thread "
                                   f"({threads} threads, nproc {os.cpu_count()}), reference "
                                   "generate() built with gcc -O2"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def decode_step_bytes(cfg, P, N, B):
    """Algorithmic bytes of the N decode steps t = P-1 .. P+N-2 of B
    sequences: per step the weights (layers + tied lm_head), per sequence
    its K/V rows 0..t of every layer (fp32) plus the appended row."""
    w = 2 if cfg["bf16"] else 4
    return algorithmic_bytes(P, N, B, t0=P - 1, weight_bytes_per=w, wl=cfg)


def run_extra(key, cfg, rank, world, dev, pg, steps, warmup, hm_cache):
    """One config of EXTRA on this rank; returns its JSON object (rank 0)."""
    import numpy as np
    import torch
    import minima_b200 as M
    B = cfg["batch"]
    first = rank * B
    if cfg.get("split"):
        B = max(1, cfg["batch"] // world)
        first = rank * B
    P, N = cfg["prompt"], cfg["new_tokens"]
    mkey = (cfg["vocab"], cfg["dim"], cfg["n_layers"], cfg["n_heads"], cfg["ffn_dim"],
            cfg["max_seq"], cfg["seed"], cfg["bf16"])
    if mkey not in hm_cache:
        hm_cache.clear()
        hm = M.HostModel(*mkey[:7], bf16=cfg["bf16"])
        dm = M.DeviceModel(hm, M.MC_WEIGHTS_BF16 if cfg["bf16"] else M.MC_WEIGHTS_F32, device=dev.index)
        hm_cache[mkey] = (hm, dm)
    hm, dm = hm_cache[mkey]
    saved = {k: os.environ.get(k) for k in ("MINIMA_CUDA_DECODE", "MINIMA_CUDA_PREFILL")}
    for k, v in (("MINIMA_CUDA_DECODE", cfg["decode"]), ("MINIMA_CUDA_PREFILL", cfg["prefill"])):
        if v:
            os.environ[k] = v
        else:
            os.environ.pop(k, None)
    try:
        cap = P + N
        sess = M.Session(dm, B, cap)
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    prompts = np.stack([prompt_ids(P, cfg["vocab"], cfg["prompt_seed"] + g)
                        for g in range(first, first + B)])
    rng = np.array([g + 1 for g in range(first, first + B)], dtype=np.uint64)
    prompts_d = torch.from_numpy(prompts.view(np.int16).copy()).to(dev)
    out_d = torch.zeros((B, cap), dtype=torch.int16, device=dev)
    rng0 = torch.tensor(rng.view(np.int64), device=dev)
    rng_d = rng0.clone()
    counts_d = torch.zeros(B, dtype=torch.int32, device=dev)
    opts = M.options(max_new_tokens=N, **cfg["sampling"])
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev) if cfg["flush"] else None
    stream = torch.cuda.ExternalStream(sess.stream_handle(), device=dev)
    call_ms, dec_ns, step_us, tokens = [], [], [], 0
    with torch.cuda.stream(stream):
        for i in range(warmup + steps):
            if flush is not None:
                flush.zero_()
            rng_d.copy_(rng0)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            sess.generate_device(prompts_d.data_ptr(), P, [P] * B, out_d.data_ptr(), cap, opts,
                                 rng_d.data_ptr(), counts_d.data_ptr())
            e1.record(stream)
            torch.cuda.synchronize()
            if i < warmup:
                continue
            call_ms.append(e0.elapsed_time(e1))
            tokens += int((counts_d - P).sum().item())
            st = sess.last_step_times_ns().astype(np.int64)
            d = np.diff(st[P - 1:P + N])           # the N decode steps
            dec_ns.append(int(d.sum()))
            step_us.extend((d / 1e3).tolist())
    kernel = sess.last_kernel_name()
    pf_pos, pf_ms = sess.last_prefill()
    sess.close()
    t_call, t_dec = max_over_ranks(pg, [sum(call_ms), sum(dec_ns) / 1e9], dev)
    if rank != 0:
        return None
    seqs = B * world
    algo = decode_step_bytes(cfg, P, N, B)      # per call, per rank
    peak, src = measured_hbm()
    achieved = algo * steps / t_dec / 1e9
    return {
        "workload": cfg["name"], "n_gpus": world, "sequences": seqs, "per_gpu_batch": B,
        "scaling": "strong" if cfg.get("split") else "weak",
        "dtype": "bf16 weights, f32 math" if cfg["bf16"] else "f32",
        "kernel": kernel, "steps": steps, "warmup": warmup,
        "l2": L2_NOTE if cfg["flush"] else "weights larger than L2 (not flushed)",
        "tokens_per_s": whole_job_rate(world, tokens / steps, t_call / 1e3 / steps),
        "decode_tokens_per_s": world * B * N * steps / t_dec,
        "ms_per_call": t_call / steps, "prefill_ms": pf_ms, "prefill_positions": pf_pos,
        "p50_token_us": float(np.median(step_us)), "p99_token_us": float(np.percentile(step_us, 99)),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": None,
                     "algorithmic_bytes_per_call": algo,
                     "peak_source": f"{src} HBM copy bandwidth",
                     "what": "decode steps only (weights + K/V rows read + appended per step)"},
    }


def native_arm(args):
    import numpy as np
    import torch
    import minima_b200 as M

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    os.environ["MINIMA_CUDA_DEVICE"] = str(local)   # the drop-in's device (e2e leg)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        pg = dist
    B, P, N = WL["batch"], WL["prompt"], WL["new_tokens"]
    hm = M.HostModel(WL["vocab"], WL["dim"], WL["n_layers"], WL["n_heads"], WL["ffn_dim"],
                     WL["max_seq"], seed=WL["seed"])
    dm = M.DeviceModel(hm, device=local)
    sess = M.Session(dm, B, WL["max_seq"])
    prompts, rng = workload_prompts(rank * B, B)
    out_cap = WL["max_seq"]
    dev = torch.device("cuda", local)
    prompts_d = torch.from_numpy(prompts.view(np.int16).copy()).to(dev)
    out_d = torch.zeros((B, out_cap), dtype=torch.int16, device=dev)
    rng0 = torch.tensor(np.array(rng, dtype=np.uint64).view(np.int64), device=dev)
    rng_d = rng0.clone()
    counts_d = torch.zeros(B, dtype=torch.int32, device=dev)
    fpos_d = torch.zeros(B, dtype=torch.int32, device=dev)
    opts = M.options(top_k=1, max_new_tokens=N)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)  # 256 MiB > L2
    stream = torch.cuda.ExternalStream(sess.stream_handle(), device=dev)

    def step():
        sess.generate_device(prompts_d.data_ptr(), P, [P] * B, out_d.data_ptr(), out_cap, opts,
                             rng_d.data_ptr(), counts_d.data_ptr(), fpos_d.data_ptr())

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            rng_d.copy_(rng0)
            step()
        torch.cuda.synchronize()
        if pg:
            pg.barrier()
        torch.cuda.synchronize()
        clocks = ClockSampler(local)
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        kernel_ms, launches, tokens = [], 0, 0
        for i in range(args.steps):
            flush.zero_()
            rng_d.copy_(rng0)
            starts[i].record(stream)
            step()
            ends[i].record(stream)
            kernel_ms.append(sess.last_kernel_ms())
            launches += sess.last_launch_count()
            tokens += int((counts_d - P).sum().item())
        torch.cuda.synchronize()
        if pg:
            pg.barrier()
        torch.cuda.synchronize()
        clk = clocks.stop()
    kernel_name = sess.last_kernel_name()
    prefill_pos, prefill_ms = sess.last_prefill()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = sum(step_ms)
    stamps = sess.last_step_times_ns().astype(np.int64)
    # stamps[t] for the positions the token loop ran (t >= prefill_pos)
    tok_us = np.diff(stamps[prefill_pos:]) / 1e3
    dec_us = tok_us[max(0, P - 1 - prefill_pos):]
    pre_us = tok_us[:max(0, P - 1 - prefill_pos)]
    got = out_d.cpu().numpy().view(np.uint16)

    # ---- end to end through the drop-in generate.h with host buffers
    tok = M.make_tokenizer(WL["vocab"])
    caches = M.Caches(hm, B, WL["max_seq"])
    e2e_times, e2e_tokens = [], 0
    for i in range(args.warmup + args.steps):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        ok, out, counts, _ = M.generate_batch(hm, tok, caches, prompts, [P] * B, out_cap, opts, rng)
        dt = time.perf_counter() - t0
        if not ok:
            raise RuntimeError("generate_batch_with_options failed: " + M.last_error())
        if i >= args.warmup:
            e2e_times.append(dt)
            e2e_tokens += int((counts - P).sum())
    assert np.array_equal(out[:, :P + N], got[:, :P + N]), "e2e and device-resident runs differ"

    # ---- max over ranks
    total_ms, e2e_s = max_over_ranks(pg, [total_ms, sum(e2e_times)], dev)
    value = whole_job_rate(world, tokens, total_ms / 1e3)
    e2e_value = whole_job_rate(world, e2e_tokens, e2e_s)
    kms = statistics.mean(kernel_ms) - prefill_ms     # the token loop's own time
    l2_gbs = measure_l2_read_gbs(dev)
    sess.close()

    # ---- the other decode workloads (every rank takes the same steps)
    extras = {}
    if not args.no_extra:
        cache = {}
        for key, cfg in EXTRA.items():
            if cfg.get("split") and cfg["batch"] % world:
                continue
            extras[key] = run_extra(key, cfg, rank, world, dev, pg, args.extra_steps,
                                    args.extra_warmup, cache)
        cache.clear()

    if rank == 0:
        algo = algorithmic_bytes(P, N, B, t0=prefill_pos)
        peak, peak_src = measured_hbm()
        achieved = algo / (kms / 1e3) / 1e9
        traffic = profiled_traffic(kernel_name)
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": workload_config(world),
            "p50_token_us": float(np.median(dec_us)), "p99_token_us": float(np.percentile(dec_us, 99)),
            "p50_prefill_token_us": float(np.median(pre_us)) if len(pre_us) else None,
            "prefill": {"positions": prefill_pos, "ms": prefill_ms,
                        "kind": "batched (all sequences' positions in one pass)"},
            "token_steps_per_launch": P + N - 1 - prefill_pos,
            "e2e": {"value": e2e_value, "unit": UNIT,
                    "h2d_bytes_per_step": B * P * 2 + B * 32,
                    "d2h_bytes_per_step": B * 32 + B * (P + N) * 2 + 4},
            "gpu_launches": launches,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "kernel": kernel_name,
                         "algorithmic_bytes_per_launch": algo, "kernel_ms": kms,
                         "peak_source": f"{peak_src} HBM copy bandwidth"},
            "roofline_l2": {"bound": "l2", "achieved": achieved, "peak": l2_gbs, "unit": "GB/s",
                            "frac": achieved / l2_gbs,
                            "peak_source": "L2 read bandwidth measured in this run: best of a "
                                           "sum and a copy over a 24 MiB L2-resident buffer"},
            "clocks": clk,
            "configs": extras,
        }
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()
        pg.destroy_process_group()


def main():
    args = parse_args()
    if args.impl == "reference":
        reference_arm(args)
    else:
        native_arm(args)


if __name__ == "__main__":
    main()
