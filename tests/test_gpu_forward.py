"""GPU: the drop-in forward.h (libminima_forward.so) against the reference's
forward.c, each under the reference's own backward.c.

* The reference's tests/attention_workspace_test.c, linked unchanged over
  the drop-in (oracle/_ref/attention_workspace_cuda): forward on the
  device, backward on the host, sequences 1, 32 and 512.
* tests/forward_e2e_main.c built twice (oracle/_ref/forward_e2e_ref over
  forward.c, oracle/_ref/forward_e2e_cuda over the drop-in): logits and
  every cache model_forward fills, then the gradients model_backward
  derives from those caches, array by array.  Bounds: caches and logits
  |gpu - ref| <= 1e-3 + 1e-4 |ref| (the fp32 bound); gradients, which sum
  many products of cached values, |gpu - ref| <= 1e-4 max|ref| + 1e-3 |ref|
  per array.  One case spans two 256-position chunks of the device forward.
"""
import ctypes as C
import os
import subprocess

import numpy as np
import pytest

import minima_b200 as M
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REF_DIR = os.path.join(os.path.dirname(O.__file__), "_ref")
CACHES = ("x", "x_norm", "qkv", "attn_out", "ffn_buf", "up_buf", "gate_buf", "resid_attn",
          "resid_ffn", "logits")
GRADS = ("d_tok_emb", "d_attn_qkv", "d_attn_proj", "d_ffn_up", "d_ffn_gate", "d_ffn_down",
         "d_rms1_scale", "d_rms2_scale", "d_rms_final_scale")


def _exe(name):
    path = os.path.join(REF_DIR, name)
    if not os.path.exists(path):
        pytest.fail(f"oracle/_ref/{name} not built (make -C oracle forward_e2e)")
    return path


def _read(path):
    out = []
    with open(path, "rb") as fh:
        while True:
            head = fh.read(8)
            if not head:
                break
            n = int(np.frombuffer(head, np.uint64)[0])
            out.append(np.frombuffer(fh.read(4 * n), np.float32).astype(np.float64))
    return dict(zip(CACHES + GRADS, out))


def test_attention_workspace_test_on_drop_in(gpu):
    r = subprocess.run([_exe("attention_workspace_cuda")], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "Attention arena workspace regression passed." in r.stdout


@pytest.mark.parametrize("args", [
    # vocab dim layers heads ffn max_seq batch seq seed
    (2048, 64, 2, 2, 128, 128, 2, 64, 5),
    (30000, 128, 2, 4, 512, 512, 1, 300, 7),     # default widths, two prefill chunks
    (4096, 96, 3, 6, 256, 256, 3, 40, 9),        # head_dim 16, three KV heads
])
def test_model_forward_and_backward_match_reference(gpu, tmp_path, args):
    files = {}
    for side in ("ref", "cuda"):
        out = str(tmp_path / f"{side}.bin")
        r = subprocess.run([_exe(f"forward_e2e_{side}"), out, *map(str, args)], capture_output=True,
                           text=True, timeout=600)
        assert r.returncode == 0, side + ": " + r.stdout + r.stderr
        files[side] = _read(out)
    ref, got = files["ref"], files["cuda"]
    assert list(got) == list(ref) == list(CACHES + GRADS)
    report = []
    for name in CACHES + GRADS:
        g, w = got[name], ref[name]
        assert g.shape == w.shape, name
        assert np.isfinite(g).all(), name
        if name in CACHES:
            bound = 1e-3 + 1e-4 * np.abs(w)
        else:
            bound = 1e-4 * np.abs(w).max() + 1e-3 * np.abs(w)
        ratio = float((np.abs(g - w) / np.maximum(bound, 1e-30)).max())
        report.append(f"{name} {ratio:.3f}")
        assert ratio <= 1.0, f"{name}: err/bound {ratio:.3f}"
    print("err/bound per array:", ", ".join(report))


def test_generation_check_kv_cache_on_device(gpu, capsys):
    """generation_check_kv_cache of the drop-in (generate.c:202-265): the
    device token loop position by position against the device batched
    forward, printed and judged as the reference does (main.c:1177-1179
    calls it with tolerance 1e-4)."""
    host, _, gen = M.libs()
    dims = O.Dims(30000, 128, 8, 4, 512, 512)
    hm = M.HostModel(dims.vocab, dims.dim, dims.n_layers, dims.n_heads, dims.ffn_dim, dims.max_seq, seed=0)
    caches = M.Caches(hm, 1, 512)
    arena = M.Arena()
    assert host.arena_init(C.byref(arena), 64 << 20)
    toks = O.random_prompt(96, dims.vocab, 11)
    arr = (C.c_uint16 * len(toks))(*[int(t) for t in toks])
    gen.generation_check_kv_cache.restype = C.c_bool
    gen.generation_check_kv_cache.argtypes = [C.POINTER(M.Model), C.POINTER(M.KVCache),
                                              C.POINTER(M.Arena), C.POINTER(C.c_uint16), C.c_int,
                                              C.c_float]
    ok = gen.generation_check_kv_cache(C.byref(hm.model), C.byref(caches.caches[0]), C.byref(arena),
                                       arr, len(toks), 1e-4)
    assert ok, M.last_error()
    assert caches.caches[0].pos == len(toks)
    host.arena_free(C.byref(arena))
