"""GPU: mc_generate_static, the entry point that allocates no device memory.

Some callers cannot call cudaMalloc at all — real-time hosts that must not
take its cost (or the device-wide wait of a later cudaFree) mid-session, hosts
that hand out device memory only from their own pre-carved pool, plugins
that must not grow the device footprint once the host application is up.  mc_generate_static serves them: they pass their
own device buffers for weights, prompts and outputs, and the KV cache and
work buffers come from a fixed static array inside the library.

This file is collected last on purpose (pytest orders files by name), so
that a run stopping at the first failure has already run every other test.
Each test checks the static entry point's output against mc_generate's on a
session that runs the same grid-barrier token loop (MINIMA_CUDA_LOOP=grid),
on two calls in a row: ids, counts and RNG states identical (greedy and
seeded sampling are deterministic, and no step of these cases is a near-tie
of the fp32 logits); it passes alone in a fresh process and after the other
tests.  A last case makes the loop's grid barrier wait for an arrival that
never comes (MINIMA_CUDA_TEST_STALL=1, 50 ms deadline): the call returns
MC_ERR_TIMEOUT and the next call is correct again.
"""
import ctypes as C

import numpy as np
import pytest

import minima_b200 as M
from oracle import oracle as O

pytestmark = pytest.mark.gpu

MC_ERR_INVALID = 1
MC_ERR_TIMEOUT = 4


def _lib():
    cuda = M.libs()[1]
    vp = C.c_void_p
    cuda.mc_generate_static.restype = C.c_int
    cuda.mc_generate_static.argtypes = [C.POINTER(M.ModelDesc), C.c_int, vp, C.c_int,
                                        C.POINTER(C.c_int), vp, C.c_int,
                                        C.POINTER(M.GenerationOptions), vp, vp, C.c_int, vp]
    return cuda


def _device_weights(hm, torch):
    """The nine weight arrays copied into caller-owned device buffers."""
    ts = [torch.from_numpy(np.ascontiguousarray(t)).cuda() for t in hm.tensors()]
    m = hm.model
    f = lambda t: C.cast(C.c_void_p(t.data_ptr()), C.POINTER(C.c_float))
    desc = M.ModelDesc(m.vocab_size, m.dim, m.n_layers, m.n_heads, m.n_kv_heads, m.head_dim,
                       m.kv_dim, m.qkv_dim, m.ffn_dim, m.max_seq, *[f(t) for t in ts])
    return desc, ts


@pytest.mark.parametrize("kw", [
    dict(top_k=1, max_new_tokens=64),
    dict(temperature=0.8, top_k=40, top_p=0.95, repetition_penalty=1.2,
         frequency_penalty=0.3, no_repeat_ngram_size=2, max_new_tokens=48),
])
def test_static_entry_point_matches_generate_twice(gpu, kw, monkeypatch):
    import torch
    cuda = _lib()
    monkeypatch.setenv("MINIMA_CUDA_LOOP", "grid")
    # the reference's default model (config.h) at batch 4 and max_seq 512
    hm = M.HostModel(30000, 128, 8, 4, 512, 512, seed=1)
    B, P, cap, out_cap = 4, 32, 512, 128
    prompts = np.stack([O.random_prompt(P, 30000, 700 + b) for b in range(B)])
    rng0 = np.arange(11, 11 + B, dtype=np.uint64)
    opts = M.options(**kw)

    # the existing entry point
    sess = M.Session(M.DeviceModel(hm), B, cap)
    ref_out, ref_counts, ref_rng, _ = sess.generate(prompts, [P] * B, out_cap, opts, rng0)
    assert sess.last_kernel_name() == "mc::token_loop_kernel"
    sess.close()

    desc, keep = _device_weights(hm, torch)
    prompts_d = torch.from_numpy(prompts.view(np.int16).copy()).cuda()
    lens = (C.c_int * B)(*([P] * B))
    free_after_first = None
    for call in range(2):
        out_d = torch.full((B, out_cap), -1, dtype=torch.int16, device="cuda")
        rng_d = torch.from_numpy(rng0.view(np.int64).copy()).cuda()
        counts_d = torch.zeros(B, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        st = cuda.mc_generate_static(C.byref(desc), B, prompts_d.data_ptr(), P, lens,
                                     out_d.data_ptr(), out_cap, C.byref(opts), rng_d.data_ptr(),
                                     counts_d.data_ptr(), cap, None)
        assert st == 0, cuda.mc_last_error().decode()
        torch.cuda.synchronize()
        free_after = torch.cuda.mem_get_info()[0]
        if call == 1:
            # no device memory taken by the second call
            assert free_after == free_before == free_after_first
        free_after_first = free_after
        counts = counts_d.cpu().numpy()
        out = out_d.cpu().numpy().view(np.uint16)
        assert list(counts) == list(ref_counts), call
        for b in range(B):
            assert np.array_equal(out[b, :counts[b]], ref_out[b, :counts[b]]), (call, b)
        assert np.array_equal(rng_d.cpu().numpy().view(np.uint64), ref_rng), call


def test_static_entry_point_rejects_oversize(gpu):
    import torch
    cuda = _lib()
    hm = M.HostModel(30000, 128, 8, 4, 512, 512, seed=1)
    desc, keep = _device_weights(hm, torch)
    B, P = 64, 8
    prompts_d = torch.zeros((B, P), dtype=torch.int16, device="cuda") + 5
    out_d = torch.zeros((B, 64), dtype=torch.int16, device="cuda")
    rng_d = torch.ones(B, dtype=torch.int64, device="cuda")
    counts_d = torch.zeros(B, dtype=torch.int32, device="cuda")
    lens = (C.c_int * B)(*([P] * B))
    # 64 sequences x 512 positions of KV cache do not fit the static array
    st = cuda.mc_generate_static(C.byref(desc), B, prompts_d.data_ptr(), P, lens,
                                 out_d.data_ptr(), 64, C.byref(M.options(max_new_tokens=4)),
                                 rng_d.data_ptr(), counts_d.data_ptr(), 512, None)
    assert st == MC_ERR_INVALID
    assert "scratch" in cuda.mc_last_error().decode()
    assert int(counts_d.sum()) == 0


def test_static_entry_point_wait_deadline(gpu, monkeypatch):
    """A grid barrier that can never complete ends the static call with
    MC_ERR_TIMEOUT (no fault, no hang); the next call is correct."""
    import torch
    cuda = _lib()
    hm = M.HostModel(4096, 128, 2, 4, 512, 128, seed=4)
    orc = O.OrcModel(O.Dims(4096, 128, 2, 4, 512, 128), 4)
    desc, keep = _device_weights(hm, torch)
    B, P, out_cap = 2, 8, 32
    prompts = np.stack([O.random_prompt(P, 4096, 10 + b) for b in range(B)])
    prompts_d = torch.from_numpy(prompts.view(np.int16).copy()).cuda()
    lens = (C.c_int * B)(*([P] * B))
    opts = M.options(top_k=1, max_new_tokens=6)

    def call():
        out_d = torch.zeros((B, out_cap), dtype=torch.int16, device="cuda")
        rng_d = torch.tensor([1, 2], dtype=torch.int64, device="cuda")
        counts_d = torch.zeros(B, dtype=torch.int32, device="cuda")
        st = cuda.mc_generate_static(C.byref(desc), B, prompts_d.data_ptr(), P, lens,
                                     out_d.data_ptr(), out_cap, C.byref(opts), rng_d.data_ptr(),
                                     counts_d.data_ptr(), 128, None)
        torch.cuda.synchronize()
        return st, out_d.cpu().numpy().view(np.uint16), counts_d.cpu().numpy()

    monkeypatch.setenv("MINIMA_CUDA_TEST_STALL", "1")
    monkeypatch.setenv("MINIMA_CUDA_WAIT_NS", str(50_000_000))   # 50 ms
    st, _, _ = call()
    assert st == MC_ERR_TIMEOUT, cuda.mc_last_error().decode()
    monkeypatch.delenv("MINIMA_CUDA_TEST_STALL")
    monkeypatch.delenv("MINIMA_CUDA_WAIT_NS")
    st, out, counts = call()
    assert st == 0, cuda.mc_last_error().decode()
    for b in range(B):
        ref, _, _ = orc.generate(prompts[b], out_cap, 128, O.make_options(top_k=1, max_new_tokens=6), b + 1)
        assert np.array_equal(out[b, :counts[b]], ref)
