"""Generate the golden vectors under tests/golden/ from the Minima reference.

Runs the reference's own decode path (oracle/_ref/libminima_ref.so, built by
oracle/Makefile from the reference's unmodified C files) on seeded weights
and synthetic prompts, and stores the outputs as small fixtures so that the
oracle restatement and the GPU path can be pinned to the reference on
machines without the reference sources.  Also records the C struct layouts
of the reference's headers that the drop-in must match.

Usage (needs the reference sources and a built oracle/_ref):
    python tests/golden/make_golden.py --ref <directory of the Minima sources>
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

# (name, dims, weight seed, prompt len, prompt seed, rng state, options, logit positions)
CASES = [
    ("c1_greedy", O.Dims(30000, 128, 8, 4, 512, 512), 0, 32, 7, 42,
     dict(top_k=1, max_new_tokens=128), [0, 31]),
    ("small_sampled", O.Dims(512, 64, 2, 4, 128, 128), 5, 12, 8, 1234,
     dict(temperature=0.8, top_k=40, top_p=0.9, repetition_penalty=1.1, min_p=0.02,
          frequency_penalty=0.2, presence_penalty=0.1, no_repeat_ngram_size=2,
          max_new_tokens=48), [11]),
    ("small_stop", O.Dims(512, 64, 2, 4, 128, 128), 5, 6, 9, 77,
     dict(temperature=1.0, top_k=256, max_new_tokens=40, min_new_tokens=3, stop=[300]), [5]),
    ("kat_dims", O.Dims(260, 8, 1, 2, 16, 32), 1234, 2, 10, 5678,
     dict(temperature=1.0, top_k=256, max_new_tokens=20), [1]),
    ("odd_heads", O.Dims(300, 42, 3, 7, 60, 64), 21, 10, 11, 3,
     dict(temperature=0.7, top_k=10, max_new_tokens=30), [9]),
]

LAYOUT_TYPES = {
    "ModelConfig": ["vocab_size", "dim", "n_layers", "n_heads", "ffn_dim", "max_seq"],
    "ArenaBudget": ["limit", "committed", "external_committed", "peak", "failed", "lock"],
    "Arena": ["base", "size", "used", "peak", "committed", "page_size", "budget"],
    "Model": ["vocab_size", "dim", "n_layers", "n_heads", "n_kv_heads", "head_dim", "kv_dim",
              "qkv_dim", "ffn_dim", "max_seq", "tok_emb", "attn_qkv", "attn_proj", "ffn_up",
              "ffn_gate", "ffn_down", "rms1_scale", "rms2_scale", "rms_final_scale",
              "weight_bytes", "memory_budget"],
    "Rng": ["state"],
    "KVCache": ["max_seq", "n_layers", "n_heads", "n_kv_heads", "head_dim", "dim", "kv_dim",
                "k_cache", "v_cache", "pos"],
    "GenerationOptions": ["temperature", "top_p", "repetition_penalty", "min_p",
                          "frequency_penalty", "presence_penalty", "top_k", "max_new_tokens",
                          "min_new_tokens", "no_repeat_ngram_size", "stop_sequence_ids",
                          "stop_sequence_len"],
    "Tokenizer": ["vocab_size", "n_merges", "memory_budget", "token_str", "token_len", "merges",
                  "merge_rank_index", "merge_rank_capacity"],
    "Activations": ["x", "x_norm", "qkv", "attn_out", "ffn_buf", "up_buf", "gate_buf",
                    "resid_attn", "resid_ffn", "logits", "dx", "dx_tmp", "dx_norm", "dattn",
                    "dqkv", "dffn", "dup", "dgate", "attention_scores"],
}


def layout_program(headers):
    lines = ["#include <stdio.h>", "#include <stddef.h>"]
    lines += [f'#include "{h}"' for h in headers]
    lines.append("int main(void) {")
    lines.append('  printf("{");')
    first = True
    for t, fields in LAYOUT_TYPES.items():
        sep = "" if first else ","
        first = False
        lines.append(f'  printf("{sep}\\"{t}\\": {{\\"__sizeof__\\": %zu", sizeof({t}));')
        for f in fields:
            lines.append(f'  printf(", \\"{f}\\": %zu", offsetof({t}, {f}));')
        lines.append('  printf("}");')
    lines.append('  printf("}\\n");')
    lines.append("  return 0;")
    lines.append("}")
    return "\n".join(lines)


def struct_layout(include_dirs, headers, defines=()):
    """sizeof/offsetof of LAYOUT_TYPES as seen through `headers`."""
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "layout.c")
        exe = os.path.join(d, "layout")
        with open(src, "w") as fh:
            fh.write(layout_program(headers))
        cmd = ["gcc", "-std=c11", "-w", "-D_GNU_SOURCE"] + [f"-D{x}" for x in defines]
        cmd += [f"-I{i}" for i in include_dirs] + ["-o", exe, src]
        subprocess.run(cmd, check=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    return json.loads(out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="directory of the Minima sources")
    args = ap.parse_args()
    if not O.ref_available():
        sys.exit("oracle/_ref/libminima_ref.so is not built (make -C oracle)")
    for name, dims, seed, plen, pseed, rng, kw, positions in CASES:
        ref = O.RefModel(dims, seed)
        prompt = O.random_prompt(plen, dims.vocab, pseed)
        opts = O.make_options(**kw)
        ids, st, pos = ref.generate(prompt, 512, dims.max_seq, opts, rng)
        logits = ref.forward_logits(ids[:max(positions) + 1])[positions]
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), prompt=prompt, ids=ids,
                            rng_state=np.uint64(st), final_pos=np.int32(pos),
                            positions=np.array(positions, np.int32),
                            logits=logits.astype(np.float32),
                            dims=np.array([dims.vocab, dims.dim, dims.n_layers, dims.n_heads,
                                           dims.ffn_dim, dims.max_seq], np.int32),
                            seed=np.uint64(seed), rng_in=np.uint64(rng),
                            options=json.dumps(kw))
        print(name, len(ids), st, pos)
    compat = os.path.join(ROOT, "oracle", "compat")
    layout = struct_layout([compat, args.ref], ["generate.h", "forward.h"])
    with open(os.path.join(HERE, "struct_layout.json"), "w") as fh:
        json.dump(layout, fh, indent=1, sort_keys=True)
    print("layout", {k: v["__sizeof__"] for k, v in layout.items()})


if __name__ == "__main__":
    main()
