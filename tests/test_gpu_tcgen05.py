"""GPU: the tcgen05 tensor-core GEMM (mc_gemm: TMA-fed tiles, tcgen05.mma,
TMEM accumulator) and the batched prefill that runs on it when
MINIMA_CUDA_PREFILL=tcgen05.

Bounds of the tensor-core path (looser than the fp32 path by design):
  kind::tf32   |C - ref| <= 2^-9 * (|A| . |B|^T) + 1e-6   (operands carry
               10-bit mantissas, products accumulate in fp32)
  kind::f16    |C - ref| <= 1e-5 * (|A| . |B|^T) + 1e-6   (bf16 operands are
               exact, so only the fp32 accumulation rounds)
  prefill      decode-step logits after a tf32 prefill: |gpu - ref| <=
               TC_ATOL + TC_RTOL * |ref| against the fp32 oracle (measured
               max |err| 3.8e-4 on this model); after a bf16 (kind::f16)
               prefill, TC16_ATOL + TC16_RTOL * |ref| against the oracle with
               the same bf16 weights and fp32 activations (measured 7.1e-4).
"""
import numpy as np
import pytest

import minima_b200 as M
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TC_ATOL, TC_RTOL = 2e-3, 2e-3
TC16_ATOL, TC16_RTOL = 5e-3, 5e-3


def to_bf16_bits(x):
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint16)


def from_bf16_bits(b):
    return (b.astype(np.uint32) << 16).view(np.float32)


@pytest.mark.parametrize("m,n,k", [(128, 128, 32), (300, 200, 96), (77, 130, 40), (1024, 768, 768)])
def test_tf32_gemm(gpu, m, n, k):
    rng = np.random.default_rng(m * 7 + n + k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((n, k)).astype(np.float32)
    c, ms = M.gemm(a, b, M.MC_GEMM_TF32)
    ref = a.astype(np.float64) @ b.astype(np.float64).T
    bound = 2.0 ** -9 * (np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64).T) + 1e-6
    err = np.abs(c - ref)
    assert np.all(err <= bound), f"max err {err.max():.3e}, worst ratio {(err / bound).max():.2f}"
    assert ms > 0.0


@pytest.mark.parametrize("m,n,k", [(128, 128, 64), (300, 200, 96), (77, 130, 40)])
def test_bf16_gemm(gpu, m, n, k):
    rng = np.random.default_rng(m + n * 3 + k)
    a16 = to_bf16_bits(rng.standard_normal((m, k)))
    b16 = to_bf16_bits(rng.standard_normal((n, k)))
    a, b = from_bf16_bits(a16).astype(np.float64), from_bf16_bits(b16).astype(np.float64)
    c, _ = M.gemm(a16, b16, M.MC_GEMM_BF16)
    ref = a @ b.T
    bound = 1e-5 * (np.abs(a) @ np.abs(b).T) + 1e-6
    err = np.abs(c - ref)
    assert np.all(err <= bound), f"max err {err.max():.3e}"


def test_gemm_rejects_misaligned_k(gpu):
    a = np.zeros((8, 6), np.float32)
    with pytest.raises(M.MinimaCudaError):
        M.gemm(a, a, M.MC_GEMM_TF32)


def test_tcgen05_prefill_logits(gpu, monkeypatch):
    """Prompt positions prefilled on the tensor cores, then decoded by the
    token loop: the decode logits stay within the tensor-core bound of the
    fp32 oracle and differ from the fp32 prefill's (the path really ran)."""
    dims = O.Dims(4096, 128, 2, 4, 512, 256)
    hm = M.HostModel(dims.vocab, dims.dim, dims.n_layers, dims.n_heads, dims.ffn_dim, dims.max_seq,
                     seed=11)
    orc = O.OrcModel(dims, 11)
    prompts = np.stack([O.random_prompt(150, dims.vocab, 20 + b) for b in range(2)])
    opts = M.options(top_k=1, max_new_tokens=8)
    steps = 8

    def run(tc):
        if tc:
            monkeypatch.setenv("MINIMA_CUDA_PREFILL", "tcgen05")
        else:
            monkeypatch.delenv("MINIMA_CUDA_PREFILL", raising=False)
        sess = M.Session(M.DeviceModel(hm), 2, 256)
        out, counts, _, _, trace = sess.generate(prompts, [150, 150], 256, opts, [1, 2],
                                                 trace_steps=steps)
        assert sess.last_prefill()[0] == 149
        return out, counts, trace

    out_tc, counts_tc, tr_tc = run(True)
    out_f, counts_f, tr_f = run(False)
    assert not np.array_equal(tr_tc, tr_f)
    for b in range(2):
        ref_ids, _, _, ref_tr = orc.generate(prompts[b], 256, 256, O.make_options(top_k=1, max_new_tokens=8),
                                             b + 1, trace_steps=steps)
        got, want = tr_tc[b].astype(np.float64), ref_tr.astype(np.float64)
        finite = np.isfinite(want)
        assert np.array_equal(np.isfinite(got), finite)
        err = np.abs(got[finite] - want[finite])
        bound = TC_ATOL + TC_RTOL * np.abs(want[finite])
        assert np.all(err <= bound), f"max err {err.max():.3e}"
        assert np.array_equal(out_f[b, :counts_f[b]], ref_ids)


def test_tcgen05_prefill_longer_than_a_pass(gpu, monkeypatch):
    """Few sequences with long prompts: the tensor-core prefill takes up to
    1024 positions per pass (2 sequences: 1024, then the rest), and the
    decode logits after it stay within the tensor-core bound of the fp32
    oracle."""
    dims = O.Dims(4096, 128, 2, 4, 512, 1536)
    hm = M.HostModel(dims.vocab, dims.dim, dims.n_layers, dims.n_heads, dims.ffn_dim, dims.max_seq,
                     seed=13)
    orc = O.OrcModel(dims, 13)
    P, steps = 1300, 4
    prompts = np.stack([O.random_prompt(P, dims.vocab, 40 + b) for b in range(2)])
    monkeypatch.setenv("MINIMA_CUDA_PREFILL", "tcgen05")
    sess = M.Session(M.DeviceModel(hm), 2, 1536)
    _, _, _, _, tr = sess.generate(prompts, [P, P], 1536, M.options(top_k=1, max_new_tokens=steps), [1, 2],
                                   trace_steps=steps)
    assert sess.last_prefill()[0] == P - 1
    for b in range(2):
        _, _, _, ref_tr = orc.generate(prompts[b], 1536, 1536, O.make_options(top_k=1, max_new_tokens=steps),
                                       b + 1, trace_steps=steps)
        got, want = tr[b, 0].astype(np.float64), ref_tr[0].astype(np.float64)
        finite = np.isfinite(want)
        assert np.array_equal(np.isfinite(got), finite)
        err = np.abs(got[finite] - want[finite])
        bound = TC_ATOL + TC_RTOL * np.abs(want[finite])
        assert np.all(err <= bound), f"max err {err.max():.3e}"


def test_tcgen05_bf16_prefill_logits(gpu, monkeypatch):
    """bf16 weights: the prefill GEMMs run as kind::f16 on bf16 copies of the
    activations; decode logits against the oracle with the same bf16-rounded
    weights and fp32 activations stay within TC16_ATOL + TC16_RTOL |ref|."""
    dims = O.Dims(4096, 128, 2, 4, 512, 256)
    hm = M.HostModel(dims.vocab, dims.dim, dims.n_layers, dims.n_heads, dims.ffn_dim, dims.max_seq,
                     seed=12, bf16=True)
    orc = O.OrcModel(dims, 12, bf16=True)
    prompts = np.stack([O.random_prompt(150, dims.vocab, 30 + b) for b in range(2)])
    monkeypatch.setenv("MINIMA_CUDA_PREFILL", "tcgen05")
    sess = M.Session(M.DeviceModel(hm, M.MC_WEIGHTS_BF16), 2, 256)
    _, _, _, _, tr = sess.generate(prompts, [150, 150], 256, M.options(top_k=1, max_new_tokens=8),
                                   [1, 2], trace_steps=8)
    assert sess.last_prefill()[0] == 149
    for b in range(2):
        _, _, _, ref_tr = orc.generate(prompts[b], 256, 256, O.make_options(top_k=1, max_new_tokens=8),
                                       b + 1, trace_steps=8)
        got, want = tr[b].astype(np.float64), ref_tr.astype(np.float64)
        finite = np.isfinite(want)
        assert np.array_equal(np.isfinite(got), finite)
        err = np.abs(got[finite] - want[finite])
        bound = TC16_ATOL + TC16_RTOL * np.abs(want[finite])
        assert np.all(err <= bound), f"max err {err.max():.3e}"
