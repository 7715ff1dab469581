"""Decode-step time of a batch on one GPU, with the token loop the session
picks by default (grid-barrier / cluster loop) and with the batched decode on
tcgen05 tensor-core GEMMs (MINIMA_CUDA_DECODE=tcgen05), on a seeded
random-init Minima-architecture model.

    python -m minima_b200.decode_bench --dim 768 --layers 12 --heads 12 --ffn 3072 \\
        --vocab 16384 --batch 64 --prompt 256 --new 32

Each arm runs generate_with_options for the batch (prompts of --prompt
seeded non-special ids, --new tokens, greedy unless --top-k/--temperature
say otherwise; sequence b is seeded b + 1); the per-step device time comes
from the %globaltimer stamps the kernels write at each step start
(mc_last_step_times), median over the decode steps after the first 8 (the
first half when there are fewer than 16) of the last of --iters calls.
Prints one JSON line per arm: step microseconds (p50, min), generated
tokens/s of the decode steps, and the algorithmic bytes per step (layer
weights + lm_head + the K/V rows read at the middle step) over the p50 step
time.
"""
import argparse
import json
import os

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
    ap.add_argument("--new", type=int, default=32)
    ap.add_argument("--iters", type=int, default=2)
    ap.add_argument("--bf16", action="store_true", help="bf16 weights (tensor-core arm: kind::f16)")
    ap.add_argument("--arms", default="default,tcgen05")
    ap.add_argument("--temperature", type=float, default=1.0)
    ap.add_argument("--top-k", type=int, default=1, help="1 = greedy; config 3 samples with T=0.8, k=40")
    args = ap.parse_args()
    cap = args.prompt + args.new + 8
    hm = M.HostModel(args.vocab, args.dim, args.layers, args.heads, args.ffn, cap, seed=2, bf16=args.bf16)
    dm = M.DeviceModel(hm, M.MC_WEIGHTS_BF16 if args.bf16 else M.MC_WEIGHTS_F32)
    prompts = np.random.default_rng(5).integers(4, args.vocab, (args.batch, args.prompt), dtype=np.uint16)
    opts = M.options(temperature=args.temperature, top_k=args.top_k, max_new_tokens=args.new)
    K = M.kv_head_count(args.heads)
    hd = args.dim // args.heads
    Q = args.dim + 2 * K * hd
    w = 2 if args.bf16 else 4
    weights = (args.layers * (Q * args.dim + args.dim * args.dim + 3 * args.ffn * args.dim)
               + args.vocab * args.dim) * w
    t_mid = args.prompt + args.new // 2        # the mean position of the decode steps
    kv = args.batch * args.layers * 2 * t_mid * K * hd * 4
    for arm in args.arms.split(","):
        if arm == "tcgen05":
            os.environ["MINIMA_CUDA_DECODE"] = "tcgen05"
        else:
            os.environ.pop("MINIMA_CUDA_DECODE", None)
        sess = M.Session(dm, args.batch, cap)
        for _ in range(args.iters):
            sess.generate(prompts, [args.prompt] * args.batch, cap, opts, list(range(1, args.batch + 1)))
        st = sess.last_step_times_ns().astype(np.int64)
        st = st[st > 0]                       # decode steps (prefilled positions have none)
        d = np.diff(st)[min(8, len(st) // 2):] / 1e3
        p50 = float(np.median(d))
        print(json.dumps({"arm": arm, "batch": args.batch, "kernel": sess.last_kernel_name(),
                          "step_us_p50": p50, "step_us_min": float(d.min()),
                          "tok_per_s": args.batch / (p50 * 1e-6),
                          "bytes_per_step": weights + kv,
                          "gbs_p50": (weights + kv) / (p50 * 1e-6) / 1e9}), flush=True)
        sess.close()


if __name__ == "__main__":
    main()
