"""GPU parity: the CUDA token loop against the oracle, through the C ABI and
the drop-in generate.h.

Tolerances (fp32 path, the bound the port is held to):
  per-position logits   |gpu - ref| <= 1e-3 + 1e-4 * |ref|
  greedy ids            identical for the first 64 generated tokens (the
                        whole sequence is compared where the top-1/top-2
                        margin of every step exceeds 1e-4)
bf16-weight path: weights are rounded to bf16 on both sides, arithmetic is
fp32 on both sides, so the same logits bound applies.
"""
import os
import subprocess

import numpy as np
import pytest

import minima_b200 as M
from oracle import oracle as O

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-3, 1e-4
C1 = O.Dims(vocab=30000, dim=128, n_layers=8, n_heads=4, ffn_dim=512, max_seq=512)


def assert_logits_close(got, ref):
    finite = np.isfinite(ref)
    assert np.array_equal(np.isfinite(got), finite)
    err = np.abs(got[finite].astype(np.float64) - ref[finite].astype(np.float64))
    bound = ATOL + RTOL * np.abs(ref[finite].astype(np.float64))
    worst = float(np.max(err - bound))
    assert worst <= 0.0, f"max |err| {err.max():.3e} exceeds bound"


@pytest.fixture(scope="module")
def c1(gpu):
    hm = M.HostModel(C1.vocab, C1.dim, C1.n_layers, C1.n_heads, C1.ffn_dim, C1.max_seq, seed=0)
    orc = O.OrcModel(C1, 0)
    return hm, orc


def test_kat_generation_special_tokens_on_gpu(gpu):
    """The reference's own generation test, linked unchanged against the drop-in."""
    exe = os.path.join(os.path.dirname(O.__file__), "_ref", "kat_generation_cuda")
    if not os.path.exists(exe):
        pytest.fail("oracle/_ref/kat_generation_cuda not built")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "Generation sampling and reserved-token tests passed." in r.stdout


def test_c1_prefix_logits(c1):
    hm, orc = c1
    dm = M.DeviceModel(hm)
    sess = M.Session(dm, 2, 128)
    toks = np.stack([O.random_prompt(40, C1.vocab, 1), O.random_prompt(40, C1.vocab, 2)])
    got = sess.forward_logits(toks)
    for b in range(2):
        ref = orc.forward_prefixes(toks[b])
        assert_logits_close(got[b], ref)
    assert sess.last_launch_count() == 1


def test_c1_greedy_drop_in(c1):
    """Config 1: B=1, prompt 32, 128 greedy tokens, via generate() of the drop-in."""
    hm, orc = c1
    prompt = O.random_prompt(32, C1.vocab, 7)
    tok = M.make_tokenizer(C1.vocab)
    caches = M.Caches(hm, 1, 512)
    opts = M.options(temperature=1.0, top_k=1, max_new_tokens=128)
    got, st, pos = M.generate_with_options(hm, tok, caches.caches[0], prompt, 512, opts, 42)
    ref, st_r, pos_r, trace = orc.generate(prompt, 512, 512, O.make_options(top_k=1, max_new_tokens=128),
                                           42, trace_steps=64)
    assert len(got) == len(ref) == 160
    assert np.array_equal(got[:32 + 64], ref[:32 + 64])
    assert st == st_r and pos == pos_r == 160


def test_c2_batch_greedy(gpu):
    """Config 2: 4 x (prompt 128 + 256 greedy), seed 1, one device token loop."""
    hm = M.HostModel(C1.vocab, C1.dim, C1.n_layers, C1.n_heads, C1.ffn_dim, C1.max_seq, seed=1)
    orc = O.OrcModel(C1, 1)
    B = 4
    prompts = np.stack([O.random_prompt(128, C1.vocab, 1000 + b) for b in range(B)])
    tok = M.make_tokenizer(C1.vocab)
    caches = M.Caches(hm, B, 512)
    opts = M.options(top_k=1, max_new_tokens=256)
    ok, out, counts, st = M.generate_batch(hm, tok, caches, prompts, [128] * B, 512, opts,
                                           list(range(1, B + 1)))
    assert ok, M.last_error()
    okr, outr, countsr, str_ = orc.generate_batch(prompts, [128] * B, 512, 512,
                                                  O.make_options(top_k=1, max_new_tokens=256),
                                                  list(range(1, B + 1)))
    assert okr
    assert list(counts) == list(countsr) == [384] * B
    for b in range(B):
        assert np.array_equal(out[b, :128 + 64], outr[b, :128 + 64])
    assert np.array_equal(st, str_)
    assert [c.pos for c in caches.caches] == [384] * B


@pytest.mark.parametrize("loop", ["cluster", "cluster2", "cluster1", "grid"])
def test_c2_shape_both_loops(gpu, loop, monkeypatch):
    """The config-2 shape (4 x prompt 128, greedy) on the cluster-resident loop
    (its two-phase layer loop with the dataflow exchange, the same loop with
    cluster barriers under MINIMA_CUDA_LOOP=cluster2, and the five-phase one
    with MINIMA_CUDA_LOOP=cluster1) and on the grid-barrier loop: same ids as
    the oracle, and each session reports the loop it ran."""
    if loop in ("grid", "cluster1", "cluster2"):
        monkeypatch.setenv("MINIMA_CUDA_LOOP", loop)
    else:
        monkeypatch.delenv("MINIMA_CUDA_LOOP", raising=False)
    hm = M.HostModel(C1.vocab, C1.dim, C1.n_layers, C1.n_heads, C1.ffn_dim, C1.max_seq, seed=1)
    orc = O.OrcModel(C1, 1)
    B = 4
    prompts = np.stack([O.random_prompt(128, C1.vocab, 2000 + b) for b in range(B)])
    sess = M.Session(M.DeviceModel(hm), B, 512)
    opts = M.options(top_k=1, max_new_tokens=96, repetition_penalty=1.05)
    out, counts, st, fpos = sess.generate(prompts, [128] * B, 512, opts, [5, 6, 7, 8])
    assert sess.last_kernel_name() == ("mc::token_loop_kernel" if loop == "grid"
                                       else "mc::cluster_loop_kernel")
    assert sess.cluster_variant() == {"cluster": 2, "cluster2": 1, "cluster1": 0, "grid": -1}[loop]
    ok, outr, countsr, str_ = orc.generate_batch(
        prompts, [128] * B, 512, 512, O.make_options(top_k=1, max_new_tokens=96,
                                                      repetition_penalty=1.05), [5, 6, 7, 8])
    assert list(counts) == list(countsr)
    for b in range(B):
        assert np.array_equal(out[b, :counts[b]], outr[b, :countsr[b]])
    assert np.array_equal(st, str_)


def test_sampling_teacher_forced(c1):
    """Temperature/top-k/top-p sampling: with the sampler fed the device's
    own logits and RNG state, the oracle sampler picks the same ids."""
    hm, orc = c1
    dm = M.DeviceModel(hm)
    sess = M.Session(dm, 2, 256)
    prompts = np.stack([O.random_prompt(20, C1.vocab, 5), O.random_prompt(20, C1.vocab, 6)])
    kw = dict(temperature=0.8, top_k=40, top_p=0.95, repetition_penalty=1.1, min_p=0.01,
              frequency_penalty=0.1, presence_penalty=0.05, no_repeat_ngram_size=3,
              max_new_tokens=24)
    out, counts, st, fpos, trace = sess.generate(prompts, [20, 20], 64, M.options(**kw), [9, 10],
                                                 trace_steps=24)
    for b in range(2):
        state = O.Rng(9 + b).state.value
        hist = list(prompts[b])
        for i in range(counts[b] - 20):
            tid, state = O.sample(trace[b, i], O.make_options(**kw), np.array(hist, np.uint16), state)
            assert tid == out[b, 20 + i], (b, i)
            hist.append(tid)
        assert state == st[b]


def test_sampling_end_to_end(c1):
    """Full sampled generation agrees with the oracle on most sequences."""
    hm, orc = c1
    dm = M.DeviceModel(hm)
    sess = M.Session(dm, 4, 256)
    prompts = np.stack([O.random_prompt(16, C1.vocab, 50 + b) for b in range(4)])
    kw = dict(temperature=0.8, top_k=40, max_new_tokens=32)
    out, counts, st, fpos = sess.generate(prompts, [16] * 4, 64, M.options(**kw), [1, 2, 3, 4])
    agree = 0
    for b in range(4):
        ref, st_r, pos_r = orc.generate(prompts[b], 64, 256, O.make_options(**kw), b + 1)
        agree += int(np.array_equal(out[b, :counts[b]], ref))
    assert agree >= 3


def test_stop_sequence_and_ragged(c1):
    hm, orc = c1
    dm = M.DeviceModel(hm)
    sess = M.Session(dm, 3, 128)
    lens = [9, 17, 4]
    prompts = np.zeros((3, 17), dtype=np.uint16)
    for b, n in enumerate(lens):
        prompts[b, :n] = O.random_prompt(n, C1.vocab, 300 + b)
    # first greedy token of sequence 1 as a one-token stop: that sequence stops at once
    first, _, _ = orc.generate(prompts[1, :17], 40, 128, O.make_options(top_k=1, max_new_tokens=1), 0)
    stop = [int(first[17])]
    kw = dict(top_k=1, max_new_tokens=12, stop=stop)
    out, counts, st, fpos = sess.generate(prompts, lens, 40, M.options(**kw), [0, 0, 0])
    for b, n in enumerate(lens):
        ref, st_r, pos_r = orc.generate(prompts[b, :n], 40, 128, O.make_options(**kw), 0)
        assert counts[b] == len(ref)
        assert np.array_equal(out[b, :counts[b]], ref)
        assert fpos[b] == pos_r and st[b] == st_r


@pytest.mark.parametrize("hd_dims", [O.Dims(1000, 64, 2, 4, 128, 256), O.Dims(777, 48, 2, 6, 96, 256)],
                         ids=["head_dim16", "head_dim8"])
def test_small_head_dim_long_prompt(gpu, hd_dims):
    """head_dim below 32 with prompts past one 64-key prefill tile: the
    prefill attention's lanes past head_dim own no output and read nothing
    (a 150-id prompt fills two tiles), then greedy decode; ids equal the
    oracle's, logits within the fp32 bound."""
    hm = M.HostModel(hd_dims.vocab, hd_dims.dim, hd_dims.n_layers, hd_dims.n_heads, hd_dims.ffn_dim,
                     hd_dims.max_seq, seed=4)
    orc = O.OrcModel(hd_dims, 4)
    prompts = np.stack([O.random_prompt(150, hd_dims.vocab, 70 + b) for b in range(2)])
    sess = M.Session(M.DeviceModel(hm), 2, 256)
    out, counts, _, _, trace = sess.generate(prompts, [150, 150], 256, M.options(top_k=1, max_new_tokens=24),
                                             [1, 2], trace_steps=24)
    for b in range(2):
        ids, _, _, ref_tr = orc.generate(prompts[b], 256, 256, O.make_options(top_k=1, max_new_tokens=24),
                                         b + 1, trace_steps=24)
        assert np.array_equal(out[b, :counts[b]], ids)
        assert_logits_close(trace[b], ref_tr)
