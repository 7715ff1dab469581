"""Throughput of the tcgen05 GEMM (mc_gemm) on one GPU.

    python -m minima_b200.gemm_bench --m 4096 --n 4096 --k 4096 --kind tf32

Prints one JSON line: shape, kind, kernel milliseconds (CUDA events around
the launch, median of --iters after --warmup), TFLOP/s and the fraction of
the measured dense bf16 GEMM peak (MEASURED_PEAKS.json; tf32 runs at half
the bf16 rate on B200, so its own ceiling is half that figure).  Operands
are seeded random; every call uploads them, which is outside the timing.
"""
import argparse
import json
import os
import statistics

import numpy as np

import minima_b200 as M

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def bf16_bits(x):
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint16)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", type=int, default=4096)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--kind", choices=["tf32", "bf16"], default="bf16")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args()
    rng = np.random.default_rng(0)
    a = rng.standard_normal((args.m, args.k), dtype=np.float32)
    b = rng.standard_normal((args.n, args.k), dtype=np.float32)
    kind = M.MC_GEMM_TF32 if args.kind == "tf32" else M.MC_GEMM_BF16
    if kind == M.MC_GEMM_BF16:
        a, b = bf16_bits(a), bf16_bits(b)
    times = []
    for i in range(args.warmup + args.iters):
        _, ms = M.gemm(a, b, kind)
        if i >= args.warmup:
            times.append(ms)
    ms = statistics.median(times)
    tflops = 2.0 * args.m * args.n * args.k / (ms * 1e-3) / 1e12
    peak = None
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            peak = json.load(fh).get("bf16_tflops")
    except (OSError, ValueError):
        pass
    print(json.dumps({"m": args.m, "n": args.n, "k": args.k, "kind": args.kind, "ms": ms,
                      "tflops": tflops, "bf16_peak_tflops": peak,
                      "frac_of_bf16_peak": tflops / peak if peak else None}), flush=True)


if __name__ == "__main__":
    main()
