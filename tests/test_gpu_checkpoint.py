"""GPU: mc_model_load_checkpoint against the reference's checkpoint_save /
checkpoint_load (checkpoint.c:154-426).

The reference writes the files (weights moved off their seeded values so
that only a faithful load can reproduce them); the model streamed to the
device must then generate exactly what the reference generates from the
same weights, and the loader must reject what checkpoint_load rejects.
"""
import struct

import numpy as np
import pytest

import minima_b200 as M
from oracle import oracle as O

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")]

DIMS = O.Dims(1000, 64, 2, 4, 128, 64)
HASH = 0xABC


def round_bf16(a):
    """Round-to-nearest-even to bf16, kept in fp32 (finite inputs)."""
    u = a.astype(np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


@pytest.fixture(scope="module")
def ckpt(gpu, tmp_path_factory):
    ref = O.RefModel(DIMS, 9)
    t = ref.tensors()
    t[0] *= 1.5
    t[3] += 0.01
    t[7] *= 0.9
    d = tmp_path_factory.mktemp("ckpt")
    paths = {}
    for opt in (0, 1):
        p = str(d / f"w{opt}.ckpt")
        assert ref.checkpoint_save(p, optimizer=opt, moment_fill=0.25, tokenizer_hash=HASH)
        paths[opt] = p
    yield ref, paths
    ref.close()


def generate(dm, prompts, opts, seeds, cap=64):
    sess = M.Session(dm, len(prompts), cap)
    out, counts, st, _ = sess.generate(np.stack(prompts), [len(p) for p in prompts], cap, opts,
                                       seeds)
    return [out[b, :counts[b]].copy() for b in range(len(prompts))], st


@pytest.mark.parametrize("optimizer", [0, 1])
def test_loaded_model_generates_like_the_reference(ckpt, optimizer):
    ref, paths = ckpt
    dm = M.DeviceModel.from_checkpoint(paths[optimizer], tokenizer_hash=HASH)
    assert dm.info["n_params"] == ref.param_count() and dm.info["optimizer_type"] == optimizer
    prompts = [O.random_prompt(12, DIMS.vocab, s) for s in (1, 2)]
    for kw in (dict(top_k=1, max_new_tokens=20),
               dict(temperature=0.8, top_k=40, top_p=0.9, max_new_tokens=20)):
        got, st = generate(dm, prompts, M.options(**kw), [3, 4])
        for b in range(2):
            want, want_st, _ = ref.generate(prompts[b], 64, 64, O.make_options(**kw), b + 3)
            assert np.array_equal(got[b], want), kw
            assert st[b] == want_st


def test_bf16_load_rounds_on_the_device(ckpt):
    ref, paths = ckpt
    dm = M.DeviceModel.from_checkpoint(paths[0], dtype=M.MC_WEIGHTS_BF16, tokenizer_hash=HASH)
    orc = O.OrcModel(DIMS, 0)
    for src, dst in zip(ref.tensors(), orc.tensors()):
        dst[...] = src
    for i in range(6):                       # matrices in bf16, norm scales stay fp32
        orc.tensors()[i][...] = round_bf16(ref.tensors()[i])
    prompts = [O.random_prompt(10, DIMS.vocab, s) for s in (5, 6)]
    got, _ = generate(dm, prompts, M.options(top_k=1, max_new_tokens=24), [1, 2])
    for b in range(2):
        want, _, _ = orc.generate(prompts[b], 64, 64, O.make_options(top_k=1, max_new_tokens=24),
                                  b + 1)
        assert np.array_equal(got[b], want)


def test_loader_rejects_what_the_reference_rejects(ckpt, tmp_path):
    ref, paths = ckpt
    good = open(paths[0], "rb").read()
    cases = {
        "nan weight": (116 + 4 * 123, float("nan")),
        "inf norm scale": (116 + 4 * (ref.param_count() - 1), float("inf")),
        "nan moment": (len(good) - 4, float("nan")),
    }
    for name, (off, val) in cases.items():
        bad = bytearray(good)
        struct.pack_into("<f", bad, off, val)
        p = str(tmp_path / "bad.ckpt")
        open(p, "wb").write(bad)
        assert ref.checkpoint_load(p) is None, name
        with pytest.raises(M.MinimaCudaError, match="non-finite"):
            M.DeviceModel.from_checkpoint(p, tokenizer_hash=HASH)
    with pytest.raises(M.MinimaCudaError, match="tokenizer"):
        M.DeviceModel.from_checkpoint(paths[0], tokenizer_hash=HASH + 1)
    # any fingerprint when asked, and the device is still usable after the failures
    dm = M.DeviceModel.from_checkpoint(paths[0])
    assert dm.info["tokenizer_hash"] == HASH
