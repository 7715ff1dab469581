"""GPU: the paged KV cache (mc_session_create_paged).

A paged session holds a pool of pages of page_len positions; each call
gives every sequence the pages its positions need, handed out from the top
of the pool down, so a sequence's consecutive pages are never adjacent in
memory and every kernel must follow the page table.  The sessions here
have fewer pages than batch x max_seq / page_len (mixed lengths: one long
sequence and several short ones, the shape of config 5's stress case), and
each of the device loops must give the oracle's ids, with the sampler's
logits within the path's bound:
  * the cluster-resident loop (greedy, fp32) and the grid-barrier loop:
    1e-3 + 1e-4 |ref|;
  * the batched tensor-core decode (MINIMA_CUDA_DECODE=tcgen05):
    1e-2 + 1e-2 |ref|;
  * mc_model_forward (batched prefill kernels + lm_head) on a paged
    session: the oracle's per-prefix logits within 1e-3 + 1e-4 |ref|.
A pool too small for a call's sequences is refused with MC_ERR_NOMEM and
leaves the session usable.
"""
import numpy as np
import pytest

import minima_b200 as M
from oracle import oracle as O

pytestmark = pytest.mark.gpu

DIMS = O.Dims(4096, 128, 2, 4, 512, 512)


def ragged_prompts(lens, vocab, seed):
    prompts = np.zeros((len(lens), max(lens)), dtype=np.uint16)
    for b, n in enumerate(lens):
        prompts[b, :n] = O.random_prompt(n, vocab, seed + b)
    return prompts


def check(out, counts, trace, orc, prompts, lens, cap, kw, rng, steps, atol, rtol, min_agree):
    worst = 0.0
    for b, n in enumerate(lens):
        ids, _, _, rtr = orc.generate(prompts[b, :n], cap, cap, O.make_options(**kw), rng[b],
                                      trace_steps=steps)
        got = out[b, :counts[b]]
        agree = 0
        while agree < min(len(got), len(ids)) - n and got[n + agree] == ids[n + agree]:
            agree += 1
        assert agree >= min(min_agree, len(ids) - n), (b, agree)
        for s in range(min(agree + 1, steps, len(ids) - n)):
            w = rtr[s].astype(np.float64)
            fin = np.isfinite(w)
            g = trace[b, s].astype(np.float64)
            assert np.array_equal(np.isfinite(g), fin)
            worst = max(worst, float((np.abs(g[fin] - w[fin]) / (atol + rtol * np.abs(w[fin]))).max()))
    assert worst <= 1.0, worst
    return worst


@pytest.mark.parametrize("loop,page_len", [("cluster", 64), ("cluster2", 64), ("cluster1", 64),
                                           ("grid", 64), ("grid", 128), ("tcgen05", 64)])
def test_paged_sessions_match_oracle(gpu, monkeypatch, loop, page_len):
    monkeypatch.delenv("MINIMA_CUDA_LOOP", raising=False)
    monkeypatch.delenv("MINIMA_CUDA_DECODE", raising=False)
    if loop in ("grid", "cluster1", "cluster2"):
        monkeypatch.setenv("MINIMA_CUDA_LOOP", loop)
    if loop == "tcgen05":
        monkeypatch.setenv("MINIMA_CUDA_DECODE", "tcgen05")
    hm = M.HostModel(DIMS.vocab, DIMS.dim, DIMS.n_layers, DIMS.n_heads, DIMS.ffn_dim, DIMS.max_seq,
                     seed=31)
    orc = O.OrcModel(DIMS, 31)
    lens = [300, 20, 45, 9]                     # one long sequence, three short ones
    B, cap, new = len(lens), 512, 24
    need = sum(-(-(n + new - 1) // page_len) for n in lens)
    sess = M.Session(M.DeviceModel(hm), B, cap, page_len=page_len, n_pages=need)
    assert need < B * cap // page_len            # the pool is smaller than a dense cache
    prompts = ragged_prompts(lens, DIMS.vocab, 500)
    kw = dict(top_k=1, max_new_tokens=new)
    rng = [3, 4, 5, 6]
    for _ in range(2):                            # the pool is reused call after call
        out, counts, st, fpos, trace = sess.generate(prompts, lens, cap, M.options(**kw), rng,
                                                     trace_steps=new)
    expected = {"cluster": "mc::cluster_loop_kernel", "cluster2": "mc::cluster_loop_kernel",
                "cluster1": "mc::cluster_loop_kernel", "grid": "mc::token_loop_kernel",
                "tcgen05": "mc::tc_gemm_kernel"}[loop]
    assert sess.last_kernel_name() == expected
    atol, rtol = (1e-2, 1e-2) if loop == "tcgen05" else (1e-3, 1e-4)
    worst = check(out, counts, trace, orc, prompts, lens, cap, kw, rng, new, atol, rtol,
                  0 if loop == "tcgen05" else new)
    print(f"{loop} page_len {page_len}: {need} pages, worst err/bound {worst:.3f}")


def test_paged_pool_too_small_is_refused(gpu):
    hm = M.HostModel(DIMS.vocab, DIMS.dim, DIMS.n_layers, DIMS.n_heads, DIMS.ffn_dim, DIMS.max_seq,
                     seed=31)
    orc = O.OrcModel(DIMS, 31)
    sess = M.Session(M.DeviceModel(hm), 2, 512, page_len=64, n_pages=3)
    prompts = ragged_prompts([100, 40], DIMS.vocab, 900)
    with pytest.raises(M.MinimaCudaError) as err:
        sess.generate(prompts, [100, 40], 512, M.options(top_k=1, max_new_tokens=40), [1, 2])
    assert "status 3" in str(err.value)          # MC_ERR_NOMEM
    # a call that fits runs on the same session
    out, counts, _, _ = sess.generate(prompts[:, :40], [40, 40], 512, M.options(top_k=1, max_new_tokens=20),
                                      [1, 2])
    for b in range(2):
        ref, _, _ = orc.generate(prompts[b, :40], 512, 512, O.make_options(top_k=1, max_new_tokens=20), b + 1)
        assert np.array_equal(out[b, :counts[b]], ref)


def test_paged_model_forward_matches_oracle(gpu):
    hm = M.HostModel(DIMS.vocab, DIMS.dim, DIMS.n_layers, DIMS.n_heads, DIMS.ffn_dim, DIMS.max_seq,
                     seed=32)
    orc = O.OrcModel(DIMS, 32)
    seq = 200
    sess = M.Session(M.DeviceModel(hm), 2, 256, page_len=64, n_pages=8)
    toks = np.stack([O.random_prompt(seq, DIMS.vocab, 40), O.random_prompt(seq, DIMS.vocab, 41)])
    got = sess.model_forward(toks)
    for b in range(2):
        ref = orc.forward_prefixes(toks[b])
        err = np.abs(got[b].astype(np.float64) - ref)
        assert (err <= 1e-3 + 1e-4 * np.abs(ref)).all(), float(err.max())
