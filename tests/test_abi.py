"""CPU: the C-ABI boundary and the drop-in's host-side logic.

No compute call reaches the device here: only library loading, exported
symbols, struct layouts, and the argument checks / early returns that
generate.c performs before any forward pass (generate.c:526-560).
"""
import ctypes as C
import json
import os
import re
import subprocess
import tempfile

import numpy as np
import pytest

import minima_b200 as M
from oracle import oracle as O
from tests.golden.make_golden import struct_layout

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INC = os.path.join(ROOT, "include")


def declared_functions(header):
    """Function names declared at top level of a C header."""
    src = open(os.path.join(INC, header)).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    src = re.sub(r"//[^\n]*", "", src)
    src = "\n".join(l for l in src.splitlines() if not l.strip().startswith("#"))
    names = set()
    for stmt in src.split(";"):
        stmt = " ".join(stmt.split())
        if stmt.startswith("typedef") or "{" in stmt or "}" in stmt and "(" not in stmt:
            stmt = stmt.split("}")[-1]
        m = re.match(r"^(?:extern \"C\" \{ )?[A-Za-z_][\w\s\*]*?\b([A-Za-z_]\w*)\s*\(", stmt.strip())
        if m and not stmt.strip().startswith("typedef"):
            names.add(m.group(1))
    return names


def test_libraries_export_every_declared_symbol():
    host, cuda, gen = M.libs()
    cuda_decl = declared_functions("minima_cuda.h")
    gen_decl = declared_functions("minima_generate.h")
    assert {"mc_init", "mc_generate", "mc_forward_logits"} <= cuda_decl
    assert {"generate", "generate_ex", "generate_with_options", "kvcache_init",
            "generation_check_kv_cache", "generate_batch_with_options"} <= gen_decl
    for name in cuda_decl:
        assert hasattr(cuda, name), name
    for name in gen_decl:
        assert hasattr(gen, name), name
    assert set(M.CUDA_SYMBOLS) <= cuda_decl
    assert set(M.GENERATE_SYMBOLS) <= gen_decl
    fwd = M.forward_lib()
    fwd_decl = declared_functions("minima_forward.h")
    assert fwd_decl == set(M.FORWARD_SYMBOLS)
    for name in fwd_decl:
        assert hasattr(fwd, name), name


def test_forward_drop_in_exports_match_reference_forward_h():
    """libminima_forward.so defines every function of the reference's
    forward.h:43-57, and the scalar helpers compute what forward.c does."""
    out = subprocess.run(["nm", "-D", "--defined-only", M.LIB_FWD], capture_output=True, text=True,
                         check=True).stdout
    for name in M.FORWARD_SYMBOLS:
        assert re.search(rf"\bT {name}\b", out), name
    fwd = M.forward_lib()
    for v in (-3.5, -0.25, 0.0, 0.7, 12.0):
        want = np.float32(v) / (np.float32(1) + np.exp(np.float64(-v)).astype(np.float32))
        assert abs(np.float32(fwd.silu(v)) - want) <= 2 * np.spacing(np.float32(abs(want)))


def test_exports_match_reference_generate_h():
    """The drop-in defines every function of the reference's generate.h."""
    for name in ("kvcache_init", "kvcache_reset", "generation_check_kv_cache",
                 "generation_inspect_next_tokens", "generate", "generate_with_options",
                 "generate_ex"):
        out = subprocess.run(["nm", "-D", "--defined-only", M.LIB_GEN], capture_output=True,
                             text=True, check=True).stdout
        assert re.search(rf"\bT {name}\b", out), name


def test_struct_layouts_match_reference():
    """The restated types in include/minima_generate.h have the reference's
    sizes and field offsets (fixture from the reference headers)."""
    golden = json.load(open(os.path.join(ROOT, "tests", "golden", "struct_layout.json")))
    mine = struct_layout([INC], ["minima_generate.h"])
    assert mine == golden
    # and the ctypes mirror agrees too
    for name, cls in [("Model", M.Model), ("KVCache", M.KVCache), ("Arena", M.Arena),
                      ("GenerationOptions", M.GenerationOptions), ("Rng", M.Rng),
                      ("Tokenizer", M.Tokenizer), ("ModelConfig", M.ModelConfig)]:
        assert C.sizeof(cls) == golden[name]["__sizeof__"], name
        for f, off in golden[name].items():
            if f != "__sizeof__":
                assert getattr(cls, f).offset == off, (name, f)


def test_host_init_matches_oracle_and_reference():
    dims = O.Dims(30000, 128, 8, 4, 512, 512)
    hm = M.HostModel(*[getattr(dims, k) for k in ("vocab", "dim", "n_layers", "n_heads",
                                                  "ffn_dim", "max_seq")], seed=1)
    orc = O.OrcModel(dims, 1)
    for a, b in zip(hm.tensors(), orc.tensors()):
        assert np.array_equal(a, b)
    assert hm.param_count() == 5_808_256
    if O.ref_available():
        ref = O.RefModel(dims, 1)
        for a, b in zip(hm.tensors(), ref.tensors()):
            assert np.array_equal(a, b)
        assert ref.param_count() == 5_808_256


def test_host_init_bf16_rounding_matches_oracle():
    dims = O.Dims(1024, 64, 2, 4, 256, 64)
    hm = M.HostModel(1024, 64, 2, 4, 256, 64, seed=3, bf16=True)
    orc = O.OrcModel(dims, 3, bf16=True)
    for a, b in zip(hm.tensors(), orc.tensors()):
        assert np.array_equal(a, b)
    assert np.all((hm.tensors()[0].view(np.uint32) & 0xFFFF) == 0)


def test_lifted_envelope_accepts_large_configs():
    # 24L/d1024 model of the bf16 configuration is accepted by model_init_config
    c = M.ModelConfig(32768, 1024, 24, 16, 4096, 2048)
    host, _, _ = M.libs()
    assert host.model_config_validate(C.byref(c))
    c.dim = 1000  # not divisible by 16 heads
    assert not host.model_config_validate(C.byref(c))


@pytest.fixture(scope="module")
def small():
    hm = M.HostModel(300, 32, 2, 4, 64, 96, seed=4)
    tok = M.make_tokenizer(300)
    caches = M.Caches(hm, 1, 96)
    return hm, tok, caches


def test_drop_in_rejects_invalid_options_without_device(small):
    hm, tok, caches = small
    prompt = O.random_prompt(5, 300, 1)
    bad = [dict(temperature=0.0), dict(temperature=float("nan")), dict(top_p=0.0),
           dict(top_p=1.01), dict(repetition_penalty=0.5), dict(min_p=-0.1), dict(min_p=1.1),
           dict(frequency_penalty=2.5), dict(presence_penalty=-2.5),
           dict(no_repeat_ngram_size=-1), dict(no_repeat_ngram_size=17),
           dict(min_new_tokens=3, max_new_tokens=2), dict(max_new_tokens=-1)]
    for kw in bad:
        kw = dict(dict(max_new_tokens=4), **kw)
        ids, st, pos = M.generate_with_options(hm, tok, caches.caches[0], prompt, 50,
                                               M.options(**kw), 7)
        assert len(ids) == 0 and st == 7, kw


def test_drop_in_zero_budget_copies_prompt(small):
    """generate.c:553-560: n_new <= 0 returns the prompt, cache untouched,
    before prompt ids are even checked."""
    hm, tok, caches = small
    cache = caches.caches[0]
    cache.pos = 17
    prompt = np.array([5, 6, 299, 1000], np.uint16)   # 1000 >= vocab: not checked here
    ids, st, pos = M.generate_with_options(hm, tok, cache, prompt, 4, M.options(max_new_tokens=9), 3)
    assert list(ids) == [5, 6, 299, 1000] and st == 3 and pos == 17
    ids, st, pos = M.generate_with_options(hm, tok, cache, prompt[:2], 10,
                                           M.options(max_new_tokens=0), 3)
    assert list(ids) == [5, 6] and pos == 17


def test_drop_in_rejects_bad_ids_and_shapes(small):
    hm, tok, caches = small
    cache = caches.caches[0]
    opts = M.options(max_new_tokens=4)
    assert len(M.generate_with_options(hm, tok, cache, [5, 300], 50, opts, 1)[0]) == 0
    stop_bad = M.options(max_new_tokens=4, stop=[300])
    assert len(M.generate_with_options(hm, tok, cache, [5, 6], 50, stop_bad, 1)[0]) == 0
    # prompt longer than out_cap / cache
    assert len(M.generate_with_options(hm, tok, cache, list(range(4, 60)), 50, opts, 1)[0]) == 0
    tok2 = M.make_tokenizer(299)   # tokenizer/model vocab mismatch (generate.c:550)
    assert len(M.generate_with_options(hm, tok2, cache, [5, 6], 50, opts, 1)[0]) == 0


def test_kvcache_init_contract(small):
    hm, _, _ = small
    host, _, gen = M.libs()
    arena = M.Arena()
    assert host.arena_init(C.byref(arena), 1 << 20)
    kc = M.KVCache()
    assert gen.kvcache_init(C.byref(kc), C.byref(arena), C.byref(hm.model), 96)
    assert (kc.max_seq, kc.n_layers, kc.kv_dim, kc.pos) == (96, 2, 16, 0)
    assert kc.k_cache and kc.v_cache
    assert not gen.kvcache_init(C.byref(kc), C.byref(arena), C.byref(hm.model), 97)  # > max_seq
    assert not gen.kvcache_init(C.byref(kc), C.byref(arena), C.byref(hm.model), 0)
    kc.pos = 5
    gen.kvcache_reset(C.byref(kc))
    assert kc.pos == 0
    host.arena_free(C.byref(arena))
