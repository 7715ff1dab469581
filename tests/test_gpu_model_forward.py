"""GPU: mc_model_forward — the batched causal forward (model_forward,
forward.c:176-274) at every position, against the oracle's per-prefix
logits (forward_one, generate.c:76-194; bit-identical to model_forward in
the reference).

Bounds: fp32 CUDA-core path |gpu - ref| <= 1e-3 + 1e-4 |ref| (the fp32
bound of the decode path); tcgen05 path (MINIMA_CUDA_PREFILL=tcgen05,
kind::tf32 GEMMs) |gpu - ref| <= 2e-2 + 2e-2 |ref|.
"""
import numpy as np
import pytest

import minima_b200 as M
from oracle import oracle as O

pytestmark = pytest.mark.gpu

DIMS = O.Dims(4096, 128, 2, 4, 512, 512)


def check(got, want, atol, rtol):
    got, want = got.astype(np.float64), want.astype(np.float64)
    err = np.abs(got - want)
    bound = atol + rtol * np.abs(want)
    assert np.all(err <= bound), f"max |err| {err.max():.3e}, worst ratio {(err / bound).max():.2f}"


@pytest.fixture(scope="module")
def model(gpu):
    hm = M.HostModel(DIMS.vocab, DIMS.dim, DIMS.n_layers, DIMS.n_heads, DIMS.ffn_dim, DIMS.max_seq,
                     seed=13)
    return hm, O.OrcModel(DIMS, 13)


@pytest.mark.parametrize("tc", [False, True])
def test_model_forward_matches_per_prefix_logits(model, monkeypatch, tc):
    hm, orc = model
    if tc:
        monkeypatch.setenv("MINIMA_CUDA_PREFILL", "tcgen05")
    else:
        monkeypatch.delenv("MINIMA_CUDA_PREFILL", raising=False)
    # 300 positions: two chunks of the batched path, ragged last chunk
    toks = np.stack([O.random_prompt(300, DIMS.vocab, 40 + b) for b in range(3)])
    sess = M.Session(M.DeviceModel(hm), 3, 512)
    got = sess.model_forward(toks)
    for b in range(3):
        want = orc.forward_prefixes(toks[b])
        if tc:
            check(got[b], want, 2e-2, 2e-2)
        else:
            check(got[b], want, 1e-3, 1e-4)


def test_model_forward_rejects_ids_outside_the_vocabulary(model):
    hm, _ = model
    sess = M.Session(M.DeviceModel(hm), 1, 64)
    toks = np.array([[5, 6, DIMS.vocab]], dtype=np.uint16)
    with pytest.raises(M.MinimaCudaError):
        sess.model_forward(toks)
