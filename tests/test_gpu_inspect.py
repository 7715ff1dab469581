"""GPU: the next-token statistics behind generation_inspect_next_tokens
(generate.c:291-388), computed on the device by mc_next_token_stats, against
the same statistics of the oracle's logits computed here in double
precision with the reference's definitions: ids 0..3 excluded, maximum,
softmax denominator, entropy in bits, the top-n ids by logit with ties to
the lower id, and the cumulative top-1/5/10 masses.

Bounds: the device logits are within the fp32 bound of the oracle's
(1e-3 + 1e-4 |ref|), so the top-n ids must be identical wherever the
oracle's consecutive top logits differ by more than twice that bound, and
probabilities, entropy and masses agree to 1e-3 relative.
"""
import ctypes as C

import numpy as np
import pytest

import minima_b200 as M
from oracle import oracle as O

pytestmark = pytest.mark.gpu


class TokenStats(C.Structure):
    _fields_ = [("status", C.c_int), ("found", C.c_int), ("ids", C.c_int * 20),
                ("logits", C.c_float * 20), ("probability", C.c_double * 20),
                ("max_logit", C.c_double), ("denominator", C.c_double),
                ("entropy_bits", C.c_double), ("top1_mass", C.c_double),
                ("top5_mass", C.c_double), ("top10_mass", C.c_double)]


def host_stats(logits, top_n):
    v = logits.astype(np.float64)[4:]
    m = v.max()
    e = np.exp(v - m)
    denom = e.sum()
    p = e / denom
    ent = -np.sum(p[p > 0] * (np.log(p[p > 0]) / np.log(2.0)))
    order = np.lexsort((np.arange(len(v)), -logits[4:]))[:top_n]   # logit desc, id asc
    return order + 4, p[order], ent, m, denom


@pytest.mark.parametrize("dims,seed,n,top_n", [
    (O.Dims(30000, 128, 8, 4, 512, 512), 0, 40, 20),
    (O.Dims(4096, 128, 2, 4, 512, 128), 4, 7, 5),
    (O.Dims(260, 32, 1, 2, 64, 64), 9, 5, 20),       # the smallest vocabulary config.h allows
])
def test_next_token_stats_match_oracle(gpu, dims, seed, n, top_n):
    cuda = M.libs()[1]
    cuda.mc_next_token_stats.argtypes = [C.c_void_p, C.POINTER(C.c_uint16), C.c_int, C.c_int,
                                         C.POINTER(TokenStats)]
    hm = M.HostModel(dims.vocab, dims.dim, dims.n_layers, dims.n_heads, dims.ffn_dim, dims.max_seq,
                     seed=seed)
    orc = O.OrcModel(dims, seed)
    sess = M.Session(M.DeviceModel(hm), 1, dims.max_seq)
    toks = O.random_prompt(n, dims.vocab, 50 + seed)
    st = TokenStats()
    arr = (C.c_uint16 * n)(*[int(t) for t in toks])
    assert cuda.mc_next_token_stats(sess.h, arr, n, top_n, C.byref(st)) == 0, M.last_error()
    assert st.status == 0
    ref_logits = orc.forward_prefixes(toks)[-1]
    ids, probs, ent, m, denom = host_stats(ref_logits, top_n)
    assert st.found == len(ids) == top_n
    got_ids = list(st.ids[:st.found])
    srt = np.sort(ref_logits[4:].astype(np.float64))[::-1]
    for i in range(st.found):
        # an id may only differ where the oracle's neighbouring logits are within the bound
        gap = min(srt[i - 1] - srt[i] if i > 0 else np.inf, srt[i] - srt[i + 1] if i + 1 < len(srt) else np.inf)
        if gap > 2 * (1e-3 + 1e-4 * abs(srt[i])):
            assert got_ids[i] == ids[i], (i, got_ids, list(ids))
    assert np.allclose(st.probability[:st.found], probs, rtol=1e-3, atol=1e-9)
    assert st.entropy_bits == pytest.approx(ent, rel=1e-3)
    assert st.max_logit == pytest.approx(m, abs=1e-3 + 1e-4 * abs(m))
    cum = np.cumsum(probs)
    assert st.top1_mass == pytest.approx(cum[0], rel=1e-3)
    assert st.top5_mass == (pytest.approx(cum[4], rel=1e-3) if st.found >= 5 else 0.0)
    assert st.top10_mass == (pytest.approx(cum[9], rel=1e-3) if st.found >= 10 else 0.0)
