"""Batched-prefill time with the CUDA-core fp32 GEMMs and with the tcgen05
GEMMs (kind::tf32 for fp32 weights, kind::f16 with --bf16), on a seeded
random-init Minima-architecture model.

    python -m minima_b200.prefill_bench --dim 768 --layers 12 --heads 12 --ffn 3072 \\
        --vocab 16384 --batch 64 --prompt 256

Each arm creates its session with MINIMA_CUDA_PREFILL unset / =tcgen05 and
runs generate_with_options with one new token per sequence; the prefill
device time comes from mc_last_prefill (CUDA events around the prefill
kernels).  Prints one JSON line per arm: milliseconds (median of --iters
after --warmup) and the GEMM TFLOP/s implied by the layer FLOPs.
"""
import argparse
import json
import os
import statistics

import numpy as np

import minima_b200 as M


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--vocab", type=int, default=16384)
    ap.add_argument("--dim", type=int, default=768)
    ap.add_argument("--layers", type=int, default=12)
    ap.add_argument("--heads", type=int, default=12)
    ap.add_argument("--ffn", type=int, default=3072)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=256)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--bf16", action="store_true", help="bf16 weights (tensor-core arm: kind::f16)")
    args = ap.parse_args()
    cap = args.prompt + 8
    hm = M.HostModel(args.vocab, args.dim, args.layers, args.heads, args.ffn, cap, seed=2, bf16=args.bf16)
    dm = M.DeviceModel(hm, M.MC_WEIGHTS_BF16 if args.bf16 else M.MC_WEIGHTS_F32)
    # non-special ids (generate.c:567 rejects none of them), seeded
    prompts = np.random.default_rng(1000).integers(4, args.vocab, (args.batch, args.prompt), dtype=np.uint16)
    opts = M.options(top_k=1, max_new_tokens=1)
    K = M.kv_head_count(args.heads)
    hd = args.dim // args.heads
    Q = args.dim + 2 * K * hd
    rows = args.batch * (args.prompt - 1)
    flops = 2.0 * rows * args.layers * (Q * args.dim + args.dim * args.dim + 3 * args.ffn * args.dim)
    arms = ("cuda_cores", "tcgen05_bf16" if args.bf16 else "tcgen05_tf32")
    for arm in arms:
        if arm != "cuda_cores":
            os.environ["MINIMA_CUDA_PREFILL"] = "tcgen05"
        else:
            os.environ.pop("MINIMA_CUDA_PREFILL", None)
        sess = M.Session(dm, args.batch, cap)
        times = []
        for i in range(args.warmup + args.iters):
            sess.generate(prompts, [args.prompt] * args.batch, cap, opts,
                          list(range(1, args.batch + 1)))
            pos, ms = sess.last_prefill()
            if i >= args.warmup:
                times.append(ms)
        ms = statistics.median(times)
        print(json.dumps({"arm": arm, "positions": pos, "rows": rows, "prefill_ms": ms,
                          "gemm_tflops": flops / (ms * 1e-3) / 1e12}), flush=True)
        sess.close()


if __name__ == "__main__":
    main()
