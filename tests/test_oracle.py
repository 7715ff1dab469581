"""CPU: the oracle pinned to the Minima reference.

* against the committed golden vectors (tests/golden/*.npz, produced by
  tests/golden/make_golden.py from the reference's own C code) — these run
  everywhere;
* against the live reference build (oracle/_ref) where it exists — bit-for-bit
  on weights, per-prefix logits, generated ids, RNG state and cache position;
* the reference's own generation test (tests/generation_special_tokens_test.c)
  built against the reference generate.c.
"""
import glob
import json
import os
import subprocess

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz")))
need_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built here")


def load_case(path):
    z = np.load(path)
    dims = O.Dims(*[int(v) for v in z["dims"]])
    kw = json.loads(str(z["options"]))
    return z, dims, kw


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_oracle_matches_golden(path):
    z, dims, kw = load_case(path)
    orc = O.OrcModel(dims, int(z["seed"]))
    prompt = z["prompt"]
    assert np.array_equal(prompt, O.random_prompt(len(prompt), dims.vocab, _prompt_seed(path)))
    ids, st, pos = orc.generate(prompt, 512, dims.max_seq, O.make_options(**kw), int(z["rng_in"]))
    assert np.array_equal(ids, z["ids"])
    assert st == int(z["rng_state"])
    assert pos == int(z["final_pos"])
    positions = list(z["positions"])
    logits = orc.forward_prefixes(ids[:max(positions) + 1])[positions]
    assert np.array_equal(logits, z["logits"])  # bit-exact


def _prompt_seed(path):
    from tests.golden.make_golden import CASES
    name = os.path.basename(path)[:-4]
    return [c for c in CASES if c[0] == name][0][4]


@need_ref
@pytest.mark.parametrize("dims,seed", [
    (O.Dims(30000, 128, 8, 4, 512, 512), 0),
    (O.Dims(260, 8, 1, 2, 16, 32), 1234),
    (O.Dims(1000, 96, 3, 6, 200, 64), 3),
    (O.Dims(777, 30, 2, 5, 50, 40), 9),
])
def test_oracle_weights_and_logits_bitexact(dims, seed):
    ref = O.RefModel(dims, seed)
    orc = O.OrcModel(dims, seed)
    for a, b, name in zip(ref.tensors(), orc.tensors(), O.TENSOR_NAMES):
        assert np.array_equal(a, b), name
    n = min(dims.max_seq, 24)
    toks = O.random_prompt(n, dims.vocab, seed + 1)
    assert np.array_equal(ref.forward_logits(toks), orc.forward_prefixes(toks))


SAMPLING_CASES = [
    dict(top_k=1, max_new_tokens=40),
    dict(temperature=0.8, top_k=40, max_new_tokens=40),
    dict(temperature=1.3, top_k=256, top_p=0.7, max_new_tokens=40),
    dict(temperature=0.9, top_k=50, repetition_penalty=1.3, frequency_penalty=0.5,
         presence_penalty=-0.4, max_new_tokens=40),
    dict(temperature=1.0, top_k=100, min_p=0.05, no_repeat_ngram_size=3, max_new_tokens=40),
    dict(temperature=1.0, top_k=8, no_repeat_ngram_size=1, max_new_tokens=40),
    dict(temperature=0.5, top_k=20, stop=[7, 8], min_new_tokens=2, max_new_tokens=40),
    dict(top_k=1, max_new_tokens=0),
]


@need_ref
@pytest.mark.parametrize("kw", SAMPLING_CASES)
def test_oracle_generate_bitexact(kw):
    dims = O.Dims(300, 32, 2, 4, 64, 96)
    ref = O.RefModel(dims, 17)
    orc = O.OrcModel(dims, 17)
    for s in range(3):
        prompt = O.random_prompt(5 + 7 * s, dims.vocab, 40 + s)
        a = ref.generate(prompt, 80, 96, O.make_options(**kw), 1000 + s)
        b = orc.generate(prompt, 80, 96, O.make_options(**kw), 1000 + s)
        assert np.array_equal(a[0], b[0]) and a[1:] == b[1:]


@need_ref
def test_oracle_rejects_what_reference_rejects():
    dims = O.Dims(300, 32, 2, 4, 64, 96)
    ref = O.RefModel(dims, 1)
    orc = O.OrcModel(dims, 1)
    prompt = O.random_prompt(4, dims.vocab, 1)
    bad = [dict(temperature=0.0), dict(top_p=0.0), dict(top_p=1.5), dict(repetition_penalty=0.9),
           dict(min_p=1.5), dict(frequency_penalty=3.0), dict(presence_penalty=-3.0),
           dict(no_repeat_ngram_size=17), dict(min_new_tokens=5, max_new_tokens=4),
           dict(max_new_tokens=-1), dict(stop=[300], max_new_tokens=3)]
    for kw in bad:
        kw = dict(dict(max_new_tokens=4), **kw)
        assert ref.generate(prompt, 80, 96, O.make_options(**kw), 1)[0].size == 0, kw
        assert orc.generate(prompt, 80, 96, O.make_options(**kw), 1)[0].size == 0, kw


@need_ref
def test_reference_kv_cache_parity_check():
    """generation_check_kv_cache (main.c:1177-1179): incremental == full forward."""
    ref = O.RefModel(O.Dims(1000, 64, 2, 4, 128, 64), 2)
    assert ref.check_kv_cache(O.random_prompt(48, 1000, 3), 1e-4)


def test_reference_kat_binary():
    exe = os.path.join(os.path.dirname(O.__file__), "_ref", "kat_generation_ref")
    if not os.path.exists(exe):
        pytest.skip("reference KAT not built here")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert "Generation sampling and reserved-token tests passed." in r.stdout


def test_rng_known_values():
    """xorshift64* (util.c:11-27): seed 0 maps to 0x123456789abcdef0."""
    r = O.Rng(0)
    assert r.state.value == 0x123456789ABCDEF0
    x = 0x123456789ABCDEF0
    x ^= x >> 12
    x ^= (x << 25) & 0xFFFFFFFFFFFFFFFF
    x ^= x >> 27
    assert r.u64() == (x * 0x2545F4914F6CDD1D) & 0xFFFFFFFFFFFFFFFF


def test_sampler_tie_order_replay():
    """Ties: the streaming replace-min keeps insertion-order quirks
    (generate.c:447-468); with all logits equal the result is still a pure
    function of the RNG draw."""
    logits = np.zeros(300, np.float32)
    logits[:4] = -np.inf
    opts = O.make_options(top_k=256)
    ids = {O.sample(logits, opts, np.zeros(0, np.uint16), s)[0] for s in range(1, 40)}
    assert all(i >= 4 for i in ids) and len(ids) > 5


_ISOLATION_PROBE = r"""
import ctypes as C, sys
sys.path.insert(0, sys.argv[1])
import minima_b200 as M
M.libs()                       # the repo's host library, loaded RTLD_GLOBAL first
from oracle import oracle as O
lib = O._load_ref()
# config.h:9-14 caps dim at 512: the reference's own model_config_validate
# must reject dim 768 however the process was set up.
h = lib.refsh_model_create(1000, 768, 1, 12, 1024, 64, 1)
print("NULL" if not h else "ACCEPTED")
"""


def test_reference_library_is_not_interposed():
    """The reference build keeps its own model_config_validate /
    model_init_config / rng_* / arena_* even in a process that loaded this
    repository's host library with RTLD_GLOBAL before it (the reference arm of
    the benchmark and several tests run in such processes)."""
    import subprocess
    import sys
    if not O.ref_available():
        pytest.skip("oracle/_ref not built")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _ISOLATION_PROBE, root], capture_output=True,
                       text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip().splitlines()[-1] == "NULL"


def test_reference_prompts_equal_oracle_prompts():
    """The reference's rng_int (util.c:29-33) and the restatement's give the
    same prompt ids, so the reference arm can draw its prompts without the
    product libraries."""
    if not O.ref_available():
        pytest.skip("oracle/_ref not built")
    for seed in (1000, 1003, 7):
        assert np.array_equal(O.ref_random_prompt(128, 30000, seed),
                              O.random_prompt(128, 30000, seed))
