"""CPU: the checkpoint reader's header and length checks against the
reference's own checkpoint_save / checkpoint_load (checkpoint.c:154-426).

Files are written by the reference (oracle/_ref); corrupted variants are
derived from them byte by byte.  For every variant, mc_checkpoint_inspect
must accept exactly when the reference's checkpoint_load accepts (the
non-finite-value check needs the arrays and runs on the device: see
test_gpu_checkpoint.py).
"""
import os
import struct

import numpy as np
import pytest

import minima_b200 as M
from oracle import oracle as O

pytestmark = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built here")

DIMS = O.Dims(1000, 64, 2, 4, 128, 64)

# byte offsets of the header fields (checkpoint.c:183-200, written back to back)
OFF = {"magic": 0, "version": 8, "dims": 12, "params": 36, "step": 44, "rng": 52, "tok": 60,
       "lr": 68, "beta1": 72, "beta2": 76, "eps": 80, "wd": 84, "base_lr": 88, "total": 92,
       "warmup": 100, "sched": 108, "opt": 112}


@pytest.fixture(scope="module")
def ref():
    r = O.RefModel(DIMS, 5)
    yield r
    r.close()


def saved(ref, path, optimizer=0, **kw):
    assert ref.checkpoint_save(path, optimizer=optimizer, **kw)
    return bytearray(open(path, "rb").read())


def patched(data, off, fmt, value):
    d = bytearray(data)
    struct.pack_into("<" + fmt, d, off, value)
    return d


def both_verdicts(ref, path, data, optimizer=0):
    with open(path, "wb") as fh:
        fh.write(data)
    try:
        info = M.checkpoint_inspect(path)
    except M.MinimaCudaError:
        info = None
    return info, ref.checkpoint_load(path, optimizer=optimizer)


@pytest.mark.parametrize("optimizer", [0, 1])
def test_inspect_reads_the_reference_header(ref, tmp_path, optimizer):
    path = str(tmp_path / "a.ckpt")
    saved(ref, path, optimizer=optimizer, step=3, total_steps=10, rng_state=77,
          tokenizer_hash=0x1234)
    info = M.checkpoint_inspect(path)
    assert info["version"] == 5 and info["header_bytes"] == 116
    assert (info["vocab_size"], info["dim"], info["n_layers"], info["n_heads"], info["ffn_dim"],
            info["max_seq"]) == (DIMS.vocab, DIMS.dim, DIMS.n_layers, DIMS.n_heads, DIMS.ffn_dim,
                                 DIMS.max_seq)
    assert info["n_params"] == ref.param_count()
    assert (info["step"], info["rng_state"], info["tokenizer_hash"]) == (3, 77, 0x1234)
    assert info["optimizer_type"] == optimizer
    assert info["schedule_total_steps"] == 10 and info["schedule_type"] == 0
    assert np.float32(info["lr"]) == np.float32(1e-3) and np.float32(info["beta2"]) == np.float32(0.95)
    # model arrays + m (+ v for AdamW), nothing after them
    assert info["file_bytes"] == os.path.getsize(path)
    assert info["file_bytes"] == 116 + 4 * ref.param_count() * (3 if optimizer == 0 else 2)
    assert ref.checkpoint_load(path, optimizer=optimizer) == (77, 3)


def test_version4_header_is_accepted_like_the_reference(ref, tmp_path):
    path = str(tmp_path / "v5.ckpt")
    v5 = saved(ref, path)
    v4 = bytearray(b"MINIMA04") + struct.pack("<I", 4) + v5[12:112] + v5[116:]
    info, verdict = both_verdicts(ref, str(tmp_path / "v4.ckpt"), v4)
    assert verdict == (77, 3)
    assert info is not None and info["version"] == 4 and info["header_bytes"] == 112
    assert info["optimizer_type"] == 0 and info["file_bytes"] == len(v4)


def test_zero_rng_state_restores_the_default_seed(ref, tmp_path):
    path = str(tmp_path / "r.ckpt")
    saved(ref, path, rng_state=0)
    assert ref.checkpoint_load(path)[0] == 0x123456789ABCDEF0
    assert M.checkpoint_inspect(path)["rng_state"] == 0x123456789ABCDEF0


CORRUPTIONS = {
    "magic": lambda d: patched(d, OFF["magic"], "8s", b"MINIMA03"),
    "version": lambda d: patched(d, OFF["version"], "I", 6),
    "v4 magic, v5 version": lambda d: patched(d, OFF["magic"], "8s", b"MINIMA04"),
    "truncated": lambda d: d[:-4],
    "trailing byte": lambda d: d + b"\0",
    "header only": lambda d: d[:116],
    "param count": lambda d: patched(d, OFF["params"], "Q", struct.unpack_from("<Q", d, 36)[0] + 1),
    "vocab": lambda d: patched(d, OFF["dims"], "I", DIMS.vocab + 1),
    "negative step": lambda d: patched(d, OFF["step"], "q", -1),
    "step past total": lambda d: patched(d, OFF["step"], "q", 11),
    "lr nan": lambda d: patched(d, OFF["lr"], "f", float("nan")),
    "beta1 one": lambda d: patched(d, OFF["beta1"], "f", 1.0),
    "beta2 negative": lambda d: patched(d, OFF["beta2"], "f", -0.5),
    "eps zero": lambda d: patched(d, OFF["eps"], "f", 0.0),
    "weight decay inf": lambda d: patched(d, OFF["wd"], "f", float("inf")),
    "base lr zero": lambda d: patched(d, OFF["base_lr"], "f", 0.0),
    "total zero": lambda d: patched(d, OFF["total"], "q", 0),
    "warmup at total": lambda d: patched(d, OFF["warmup"], "q", 10),
    "schedule type": lambda d: patched(d, OFF["sched"], "i", 2),
    "optimizer type": lambda d: patched(d, OFF["opt"], "i", 7),
}


@pytest.mark.parametrize("name", sorted(CORRUPTIONS))
def test_header_rejections_match_the_reference(ref, tmp_path, name):
    good = saved(ref, str(tmp_path / "good.ckpt"), step=3, total_steps=10)
    info, verdict = both_verdicts(ref, str(tmp_path / "bad.ckpt"), CORRUPTIONS[name](good))
    assert verdict is None, "the reference accepts this variant"
    assert info is None, "mc_checkpoint_inspect accepts a file the reference rejects"


def test_non_finite_values_pass_the_header_check_only(ref, tmp_path):
    """A NaN among the arrays is invisible to the header checks; the
    reference rejects the file after reading it, and so does the device
    loader (GPU test)."""
    good = saved(ref, str(tmp_path / "good.ckpt"))
    bad = patched(good, 116 + 4 * 10, "f", float("nan"))
    info, verdict = both_verdicts(ref, str(tmp_path / "nan.ckpt"), bad)
    assert verdict is None
    assert info is not None


def test_inspect_missing_file(tmp_path):
    with pytest.raises(M.MinimaCudaError):
        M.checkpoint_inspect(str(tmp_path / "absent.ckpt"))
