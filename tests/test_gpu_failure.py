"""GPU: a device-side wait that can never complete ends with MC_ERR_TIMEOUT
and leaves the context usable.

No fault, trap or endless loop is involved: MINIMA_CUDA_TEST_STALL=1 makes
every wait expect one arrival more than there are participants (the grid
barrier of the grid loop; the layer cluster's wait on the head CTAs of the
cluster loop), MINIMA_CUDA_WAIT_NS shortens the deadline, and the kernel
unwinds with the status word set.  The next call, without the hook, must
produce the reference's output.
"""
import numpy as np
import pytest

import minima_b200 as M
from oracle import oracle as O

pytestmark = pytest.mark.gpu

DIMS = O.Dims(4096, 128, 2, 4, 512, 128)


@pytest.mark.parametrize("loop", ["grid", "cluster", "cluster2", "cluster1"])
def test_wait_deadline_reports_timeout_and_recovers(gpu, loop, monkeypatch):
    if loop in ("grid", "cluster1", "cluster2"):
        monkeypatch.setenv("MINIMA_CUDA_LOOP", loop)
    else:
        monkeypatch.delenv("MINIMA_CUDA_LOOP", raising=False)
    hm = M.HostModel(DIMS.vocab, DIMS.dim, DIMS.n_layers, DIMS.n_heads, DIMS.ffn_dim, DIMS.max_seq,
                     seed=4)
    orc = O.OrcModel(DIMS, 4)
    sess = M.Session(M.DeviceModel(hm), 2, 128)
    prompts = np.stack([O.random_prompt(8, DIMS.vocab, 10 + b) for b in range(2)])
    opts = M.options(top_k=1, max_new_tokens=6)
    monkeypatch.setenv("MINIMA_CUDA_TEST_STALL", "1")
    monkeypatch.setenv("MINIMA_CUDA_WAIT_NS", str(50_000_000))   # 50 ms
    with pytest.raises(M.MinimaCudaError) as err:
        sess.generate(prompts, [8, 8], 32, opts, [1, 2])
    assert "status 4" in str(err.value)                        # MC_ERR_TIMEOUT
    monkeypatch.delenv("MINIMA_CUDA_TEST_STALL")
    monkeypatch.delenv("MINIMA_CUDA_WAIT_NS")
    out, counts, st, fpos = sess.generate(prompts, [8, 8], 32, opts, [1, 2])
    for b in range(2):
        ref, _, _ = orc.generate(prompts[b], 32, 128, O.make_options(top_k=1, max_new_tokens=6), b + 1)
        assert np.array_equal(out[b, :counts[b]], ref)
    expected = "mc::token_loop_kernel" if loop == "grid" else "mc::cluster_loop_kernel"
    assert sess.last_kernel_name() == expected
    assert sess.cluster_variant() == {"cluster": 2, "cluster2": 1, "cluster1": 0, "grid": -1}[loop]
