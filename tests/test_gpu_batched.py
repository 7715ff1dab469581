"""GPU: the batched decode step on tcgen05 (MINIMA_CUDA_DECODE=tcgen05) —
every matrix product of a step is one batch-wide tensor-core GEMM.

Bounds (tensor-core path): the logits each sampler saw stay within
BD_ATOL + BD_RTOL |ref| of the oracle's for the same sequence, over the
steps where the generated ids agree with the oracle's (kind::tf32 for fp32
weights; kind::f16 with bf16 activations for bf16 weights, against the
oracle with the same bf16 weights and fp32 activations).
"""
import numpy as np
import pytest

import minima_b200 as M
from oracle import oracle as O

pytestmark = pytest.mark.gpu

DIMS = O.Dims(4096, 128, 2, 4, 512, 256)
BD_ATOL, BD_RTOL = 1e-2, 1e-2


def run(monkeypatch, bf16, batch, steps, dims=DIMS, lens=None, cap=128, **kw):
    monkeypatch.setenv("MINIMA_CUDA_DECODE", "tcgen05")
    hm = M.HostModel(dims.vocab, dims.dim, dims.n_layers, dims.n_heads, dims.ffn_dim, dims.max_seq,
                     seed=21, bf16=bf16)
    orc = O.OrcModel(dims, 21, bf16=bf16)
    if lens is None:
        lens = [20 + (b * 7) % 23 for b in range(batch)]      # ragged prompts
    prompts = np.zeros((batch, max(lens)), dtype=np.uint16)
    for b, n in enumerate(lens):
        prompts[b, :n] = O.random_prompt(n, dims.vocab, 300 + b)
    sess = M.Session(M.DeviceModel(hm, M.MC_WEIGHTS_BF16 if bf16 else M.MC_WEIGHTS_F32), batch, cap)
    opts = M.options(max_new_tokens=steps, **kw)
    out, counts, st, _, trace = sess.generate(prompts, lens, cap, opts, list(range(1, batch + 1)),
                                              trace_steps=steps)
    assert sess.last_kernel_name() == "mc::tc_gemm_kernel"
    worst, agree = 0.0, []
    for b in range(batch):
        ids, _, _, ref_tr = orc.generate(prompts[b, :lens[b]], cap, cap, O.make_options(max_new_tokens=steps, **kw),
                                         b + 1, trace_steps=steps)
        got = out[b, lens[b]:counts[b]]
        want = ids[lens[b]:]
        n = 0
        while n < min(len(got), len(want)) and got[n] == want[n]:
            n += 1
        agree.append(n)
        for s in range(min(n + 1, steps)):
            g, w = trace[b, s].astype(np.float64), ref_tr[s].astype(np.float64)
            fin = np.isfinite(w)
            assert np.array_equal(np.isfinite(g), fin)
            err = np.abs(g[fin] - w[fin])
            ratio = (err / (BD_ATOL + BD_RTOL * np.abs(w[fin]))).max()
            worst = max(worst, ratio)
            assert ratio <= 1.0, f"seq {b} step {s}: max |err| {err.max():.3e}"
    return worst, agree


@pytest.mark.parametrize("bf16", [False, True])
def test_batched_greedy_matches_oracle(gpu, monkeypatch, bf16):
    worst, agree = run(monkeypatch, bf16, 40, 12, top_k=1)
    print(f"bf16={bf16}: worst err/bound {worst:.3f}, ids agree {sum(a == 12 for a in agree)}/40")
    assert sum(a == 12 for a in agree) >= 36


def test_batched_sampled_runs(gpu, monkeypatch):
    worst, agree = run(monkeypatch, False, 33, 8, temperature=0.8, top_k=40, top_p=0.9)
    print(f"sampled: worst err/bound {worst:.3f}")


def test_batched_two_sequence_tiles(gpu, monkeypatch):
    """80 sequences: the decode GEMMs run two 64-sequence tiles."""
    worst, agree = run(monkeypatch, False, 80, 6, top_k=1)
    print(f"B=80: worst err/bound {worst:.3f}")
    assert sum(a == 6 for a in agree) >= 72


def test_batched_penalties_and_bans(gpu, monkeypatch):
    """Greedy with repetition/frequency/presence penalties and n-gram bans:
    the lm_head epilogue's transformed values (generate.c:438-460)."""
    worst, agree = run(monkeypatch, False, 36, 10, top_k=1, repetition_penalty=1.3,
                       frequency_penalty=0.5, presence_penalty=0.2, no_repeat_ngram_size=2)
    print(f"penalties: worst err/bound {worst:.3f}")
    assert sum(a == 10 for a in agree) >= 32


def test_batched_head_dim_64_key_splits(gpu, monkeypatch):
    """head_dim 64 (the lane-per-key attention kernel's HD = 64 build) with
    ~300-key contexts over 24 sequences: too few (sequence, KV head) pairs
    to fill the GPU, so each pair's keys are split and merged."""
    dims = O.Dims(4096, 256, 2, 4, 512, 512)
    lens = [280 + (b * 5) % 31 for b in range(24)]
    worst, agree = run(monkeypatch, False, 24, 6, dims=dims, lens=lens, cap=512, top_k=1)
    print(f"hd=64 splits: worst err/bound {worst:.3f}")
    assert sum(a == 6 for a in agree) >= 21


def test_batched_wide_query_groups(gpu, monkeypatch):
    """7 heads share one KV head (G = 7 > the lane-per-key kernel's limit):
    the shared-memory tile attention kernel."""
    dims = O.Dims(4096, 224, 2, 7, 512, 256)
    worst, agree = run(monkeypatch, False, 33, 6, dims=dims, top_k=1)
    print(f"G=7: worst err/bound {worst:.3f}")
    assert sum(a == 6 for a in agree) >= 30
