"""GPU parity for the larger Minima-architecture decoders (oracle: the lifted
CPU restatement, pinned to the reference on the configurations it accepts).

The model dimensions are the full ones of each configuration; batch, prompt
and generated lengths are cut so that the CPU oracle finishes in seconds.
Size-independent properties cover the full lengths:
  * batched prefill + token loop == token-by-token loop (two independent
    device paths) at long context;
  * greedy decode is deterministic and identical between the grid-barrier
    and cluster loops.
Tolerance (fp32 arithmetic, fp32 or bf16-rounded weights on both sides):
|gpu - ref| <= 1e-3 + 1e-4 |ref| per logit.
"""
import numpy as np
import pytest

import minima_b200 as M
from oracle import oracle as O

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-3, 1e-4


def close(got, ref):
    """allclose with infinities (masked ids) required to match exactly."""
    got = got.astype(np.float64)
    ref = ref.astype(np.float64)
    fin = np.isfinite(ref)
    if not np.array_equal(np.isfinite(got), fin) or not np.array_equal(got[~fin], ref[~fin]):
        return False, float("inf")
    err = np.abs(got[fin] - ref[fin])
    ok = err <= ATOL + RTOL * np.abs(ref[fin])
    return bool(ok.all()), float(err.max()) if err.size else 0.0


def host_model(d, seed, bf16=False):
    return M.HostModel(d.vocab, d.dim, d.n_layers, d.n_heads, d.ffn_dim, d.max_seq, seed=seed,
                       bf16=bf16)


# config 3: 12 layers, d768, 12 heads (6 KV heads), FFN 3072, V16384, ctx 1024, fp32
C3 = O.Dims(16384, 768, 12, 12, 3072, 1024)
# configs 4/5: 24 layers, d1024, 16 heads (8 KV heads), FFN 4096, V32768, ctx 2048, bf16 weights
C4 = O.Dims(32768, 1024, 24, 16, 4096, 2048)
C4_L2 = O.Dims(32768, 1024, 2, 16, 4096, 2048)   # same layer shapes, 2 of the 24 layers


@pytest.fixture(scope="module")
def c3(gpu):
    return host_model(C3, 2), O.OrcModel(C3, 2)


def test_c3_prefix_logits(c3):
    hm, orc = c3
    sess = M.Session(M.DeviceModel(hm), 1, 64)
    toks = O.random_prompt(12, C3.vocab, 31)[None, :]
    got = sess.forward_logits(toks)[0]
    ok, err = close(got, orc.forward_prefixes(toks[0]))
    assert ok, err


def test_c3_temperature_sampling_teacher_forced(c3):
    """Config 3 sampling (T=0.8, top-k 40, per-sequence RNG): ids equal the
    oracle sampler's on the device's own logits and RNG states."""
    hm, orc = c3
    sess = M.Session(M.DeviceModel(hm), 2, 64)
    prompts = np.stack([O.random_prompt(16, C3.vocab, 40 + b) for b in range(2)])
    kw = dict(temperature=0.8, top_k=40, max_new_tokens=8)
    out, counts, st, fpos, trace = sess.generate(prompts, [16, 16], 64, M.options(**kw),
                                                 [100, 101], trace_steps=8)
    for b in range(2):
        state, hist = 100 + b, list(prompts[b])
        for i in range(8):
            tid, state = O.sample(trace[b, i], O.make_options(**kw), np.array(hist, np.uint16), state)
            assert tid == out[b, 16 + i]
            hist.append(tid)
        assert state == st[b]
        # and the logits the sampler saw are the oracle's
        ref, st_r, pos_r, rtrace = orc.generate(prompts[b], 64, 64, O.make_options(**kw), 100 + b,
                                                trace_steps=8)
        if np.array_equal(out[b, :counts[b]], ref):
            for i in range(8):
                ok, err = close(trace[b, i], rtrace[i])
                assert ok, (b, i, err)


@pytest.fixture(scope="module")
def c4l2(gpu):
    return host_model(C4_L2, 3, bf16=True), O.OrcModel(C4_L2, 3, bf16=True)


def test_c4_bf16_weights_logits_and_greedy(c4l2):
    """bf16 weights (RNE from the fp32 init), fp32 arithmetic, layer shapes of
    config 4: per-position logits and greedy ids against the oracle."""
    hm, orc = c4l2
    dm = M.DeviceModel(hm, dtype=M.MC_WEIGHTS_BF16)
    sess = M.Session(dm, 2, 128)
    toks = O.random_prompt(10, C4_L2.vocab, 50)[None, :]
    ok, err = close(sess.forward_logits(toks)[0], orc.forward_prefixes(toks[0]))
    assert ok, err
    prompts = np.stack([O.random_prompt(24, C4_L2.vocab, 60 + b) for b in range(2)])
    out, counts, st, fpos = sess.generate(prompts, [24, 24], 64, M.options(top_k=1, max_new_tokens=12),
                                          [7, 8])
    for b in range(2):
        ref, _, _ = orc.generate(prompts[b], 64, 128, O.make_options(top_k=1, max_new_tokens=12), 7 + b)
        assert np.array_equal(out[b, :counts[b]], ref)


def test_c4_full_depth_bf16_short(gpu):
    """All 24 layers of config 4 (bf16 weights): a short greedy run equals the oracle."""
    hm = host_model(C4, 3, bf16=True)
    orc = O.OrcModel(C4, 3, bf16=True)
    sess = M.Session(M.DeviceModel(hm, dtype=M.MC_WEIGHTS_BF16), 1, 64)
    prompt = O.random_prompt(6, C4.vocab, 70)
    out, counts, st, fpos = sess.generate(prompt[None, :], [6], 16, M.options(top_k=1, max_new_tokens=4), [9])
    ref, _, _ = orc.generate(prompt, 16, 64, O.make_options(top_k=1, max_new_tokens=4), 9)
    assert np.array_equal(out[0, :counts[0]], ref)


def test_long_context_prefill_matches_token_loop(c4l2):
    """Config-5 regime (prompt 1900, KV near 2048): logits of the last prompt
    position from batched prefill + token loop equal those of the pure
    token-by-token loop, and the first greedy ids agree."""
    hm, _ = c4l2
    dm = M.DeviceModel(hm, dtype=M.MC_WEIGHTS_BF16)
    sess = M.Session(dm, 2, 2048)
    P = 1900
    prompts = np.stack([O.random_prompt(P, C4_L2.vocab, 80 + b) for b in range(2)])
    opts = M.options(top_k=1, max_new_tokens=148)
    out, counts, st, fpos, trace = sess.generate(prompts, [P, P], 2048, opts, [1, 2], trace_steps=1)
    assert sess.last_prefill()[0] == P - 1
    assert list(counts) == [2048, 2048] and list(fpos) == [2048, 2048]
    tl = sess.forward_logits(prompts)       # token-by-token through the grid loop
    for b in range(2):
        ref = tl[b, P - 1].copy()
        ref[:4] = -np.inf
        ok, err = close(trace[b, 0], ref)
        assert ok, (b, err)


def test_long_context_oracle_at_moderate_length(c4l2):
    hm, orc = c4l2
    sess = M.Session(M.DeviceModel(hm, dtype=M.MC_WEIGHTS_BF16), 1, 512)
    prompt = O.random_prompt(300, C4_L2.vocab, 90)
    out, counts, st, fpos, trace = sess.generate(prompt[None, :], [300], 512,
                                                 M.options(top_k=1, max_new_tokens=2), [3],
                                                 trace_steps=2)
    ref, _, _, rtrace = orc.generate(prompt, 512, 512, O.make_options(top_k=1, max_new_tokens=2), 3,
                                     trace_steps=2)
    ok, err = close(trace[0, 0], rtrace[0])
    assert ok, err
    assert np.array_equal(out[0, :counts[0]], ref)


@pytest.mark.parametrize("loop", ["cluster", "cluster1", "grid"])
def test_long_context_against_oracle_at_full_length(gpu, monkeypatch, loop):
    """The config-5 context length (prompt 1900, 4 greedy steps) on a 2-layer
    model of the default widths, against the oracle at full length: the
    batched prefill attends over up to 1899 keys, and each token loop over
    1900-1903 (the cluster loop's two-phase layers in eight K/V tiles, the
    keys past the first tile on the unit's second CTA; its five-phase layers
    with keys split over CTAs; the grid loop's split-K attention).  Logits of
    every step within the bound while the ids agree; a divergence only where
    the oracle's top-1/top-2 margin is within twice the bound."""
    for var in ("MINIMA_CUDA_LOOP", "MINIMA_CUDA_DECODE", "MINIMA_CUDA_PREFILL"):
        monkeypatch.delenv(var, raising=False)
    if loop != "cluster":
        monkeypatch.setenv("MINIMA_CUDA_LOOP", loop)
    d = O.Dims(4096, 128, 2, 4, 512, 2048)
    hm = host_model(d, 21)
    orc = O.OrcModel(d, 21)
    sess = M.Session(M.DeviceModel(hm), 1, 2048)
    prompt = O.random_prompt(1900, d.vocab, 95)
    steps = 4
    out, counts, st, fpos, trace = sess.generate(prompt[None, :], [1900], 2048,
                                                 M.options(top_k=1, max_new_tokens=steps), [5],
                                                 trace_steps=steps)
    assert sess.last_kernel_name() == ("mc::token_loop_kernel" if loop == "grid" else "mc::cluster_loop_kernel")
    assert sess.cluster_variant() == {"cluster": 2, "cluster1": 0, "grid": -1}[loop]
    ref, _, _, rtr = orc.generate(prompt, 2048, 2048, O.make_options(top_k=1, max_new_tokens=steps), 5,
                                  trace_steps=steps)
    got = out[0, 1900:counts[0]]
    want = ref[1900:]
    for s_ in range(steps):
        ok, err = close(trace[0, s_], rtr[s_])
        assert ok, (s_, err)
        if got[s_] != want[s_]:
            w = np.sort(rtr[s_][np.isfinite(rtr[s_])])
            margin = float(w[-1] - w[-2])
            assert margin <= 2 * (ATOL + RTOL * abs(float(w[-1]))), (s_, margin)
            break
