"""Oracle for the Minima decode path — TEST INFRASTRUCTURE ONLY.

Two CPU implementations, both used strictly as checkers:

* ``RefModel``  — the Minima reference itself (its unmodified forward.c,
  generate.c, model.c, arena.c, util.c, tokenizer.c compiled by
  ``oracle/Makefile`` into ``oracle/_ref/libminima_ref.so``), driven through
  its public API (``model_init_config``, ``generate_with_options``,
  ``model_forward``) by ``oracle/ref_shim.c``.  It only accepts the
  reference's envelope (config.h:7-14, generate.c:14-22).
* ``OrcModel``  — ``oracle/minima_oracle.c``, a restatement of the same
  arithmetic in the same order with the envelope lifted, pinned bit-for-bit
  against ``RefModel`` by ``tests/test_oracle.py``.

Only tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
import this module.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_LIB = os.path.join(HERE, "_ref", "libminima_ref.so")
ORC_LIB = os.path.join(HERE, "liboracle.so")

TENSOR_NAMES = ("tok_emb", "attn_qkv", "attn_proj", "ffn_up", "ffn_gate",
                "ffn_down", "rms1_scale", "rms2_scale", "rms_final_scale")


class GenerationOptions(C.Structure):
    """Field-for-field the reference's GenerationOptions (generate.h:50-63)."""
    _fields_ = [
        ("temperature", C.c_float),
        ("top_p", C.c_float),
        ("repetition_penalty", C.c_float),
        ("min_p", C.c_float),
        ("frequency_penalty", C.c_float),
        ("presence_penalty", C.c_float),
        ("top_k", C.c_int),
        ("max_new_tokens", C.c_int),
        ("min_new_tokens", C.c_int),
        ("no_repeat_ngram_size", C.c_int),
        ("stop_sequence_ids", C.POINTER(C.c_uint16)),
        ("stop_sequence_len", C.c_int),
    ]


def make_options(temperature=1.0, top_k=1, top_p=1.0, repetition_penalty=1.0,
                 min_p=0.0, frequency_penalty=0.0, presence_penalty=0.0,
                 max_new_tokens=0, min_new_tokens=0, no_repeat_ngram_size=0,
                 stop=None):
    """GenerationOptions with generate_ex's defaults (generate.c:604-625).

    The stop array is kept alive on the returned object."""
    o = GenerationOptions()
    o.temperature = temperature
    o.top_p = top_p
    o.repetition_penalty = repetition_penalty
    o.min_p = min_p
    o.frequency_penalty = frequency_penalty
    o.presence_penalty = presence_penalty
    o.top_k = top_k
    o.max_new_tokens = max_new_tokens
    o.min_new_tokens = min_new_tokens
    o.no_repeat_ngram_size = no_repeat_ngram_size
    if stop:
        arr = (C.c_uint16 * len(stop))(*stop)
        o._stop_keepalive = arr
        o.stop_sequence_ids = C.cast(arr, C.POINTER(C.c_uint16))
        o.stop_sequence_len = len(stop)
    else:
        o.stop_sequence_ids = None
        o.stop_sequence_len = 0
    return o


def kv_head_count(n_heads: int) -> int:
    """model_kv_head_count (model.c:34-40)."""
    if n_heads <= 1:
        return 1
    for kv in range(n_heads // 2, 0, -1):
        if n_heads % kv == 0:
            return kv
    return 1


@dataclass(frozen=True)
class Dims:
    vocab: int
    dim: int
    n_layers: int
    n_heads: int
    ffn_dim: int
    max_seq: int

    @property
    def n_kv_heads(self):
        return kv_head_count(self.n_heads)

    @property
    def head_dim(self):
        return self.dim // self.n_heads

    @property
    def kv_dim(self):
        return self.n_kv_heads * self.head_dim

    @property
    def qkv_dim(self):
        return self.dim + 2 * self.kv_dim

    def tensor_shapes(self):
        V, D, L, F, Q = self.vocab, self.dim, self.n_layers, self.ffn_dim, self.qkv_dim
        return [(V, D), (L, Q, D), (L, D, D), (L, F, D), (L, F, D), (L, D, F),
                (L, D), (L, D), (D,)]


_u16p = C.POINTER(C.c_uint16)
_f32p = C.POINTER(C.c_float)
_u64p = C.POINTER(C.c_uint64)
_intp = C.POINTER(C.c_int)


def _u16(a):
    a = np.ascontiguousarray(a, dtype=np.uint16)
    return a, a.ctypes.data_as(_u16p)


_ref_lib = None
_orc_lib = None


def ref_available() -> bool:
    return os.path.exists(REF_LIB)


def _load_ref():
    global _ref_lib
    if _ref_lib is None:
        lib = C.CDLL(REF_LIB)
        lib.refsh_model_create.restype = C.c_void_p
        lib.refsh_model_create.argtypes = [C.c_int] * 6 + [C.c_uint64]
        lib.refsh_model_free.argtypes = [C.c_void_p]
        lib.refsh_tensor.restype = _f32p
        lib.refsh_tensor.argtypes = [C.c_void_p, C.c_int, C.POINTER(C.c_size_t)]
        lib.refsh_param_count.restype = C.c_size_t
        lib.refsh_param_count.argtypes = [C.c_void_p]
        lib.refsh_generate.restype = C.c_int
        lib.refsh_generate.argtypes = [C.c_void_p, _u16p, C.c_int, _u16p, C.c_int,
                                       C.c_int, C.POINTER(GenerationOptions), _u64p, _intp]
        lib.refsh_forward_logits.restype = C.c_int
        lib.refsh_forward_logits.argtypes = [C.c_void_p, _u16p, C.c_int, _f32p]
        lib.refsh_check_kv_cache.restype = C.c_int
        lib.refsh_check_kv_cache.argtypes = [C.c_void_p, _u16p, C.c_int, C.c_float]
        lib.refsh_checkpoint_save.restype = C.c_int
        lib.refsh_checkpoint_save.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.c_int64,
                                              C.c_int64, C.c_uint64, C.c_uint64, C.c_float]
        lib.refsh_checkpoint_load.restype = C.c_int
        lib.refsh_checkpoint_load.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.c_uint64,
                                              _u64p, C.POINTER(C.c_int64)]
        lib.rng_seed.argtypes = [C.c_void_p, C.c_uint64]
        lib.rng_u64.restype = C.c_uint64
        lib.rng_u64.argtypes = [C.c_void_p]
        lib.rng_int.restype = C.c_int
        lib.rng_int.argtypes = [C.c_void_p, C.c_int, C.c_int]
        _ref_lib = lib
    return _ref_lib


def _load_orc():
    global _orc_lib
    if _orc_lib is None:
        lib = C.CDLL(ORC_LIB)
        lib.orc_model_create.restype = C.c_void_p
        lib.orc_model_create.argtypes = [C.c_int] * 6 + [C.c_uint64, C.c_int]
        lib.orc_model_free.argtypes = [C.c_void_p]
        lib.orc_model_tensor.restype = _f32p
        lib.orc_model_tensor.argtypes = [C.c_void_p, C.c_int, C.POINTER(C.c_size_t)]
        lib.orc_forward_prefixes.restype = C.c_int
        lib.orc_forward_prefixes.argtypes = [C.c_void_p, _u16p, C.c_int, _f32p]
        lib.orc_sample.restype = C.c_int
        lib.orc_sample.argtypes = [_f32p, C.c_int, C.POINTER(GenerationOptions),
                                   _u16p, C.c_int, _u64p]
        lib.orc_generate.restype = C.c_int
        lib.orc_generate.argtypes = [C.c_void_p, _u16p, C.c_int, _u16p, C.c_int, C.c_int,
                                     C.POINTER(GenerationOptions), _u64p, _f32p, C.c_int,
                                     _intp]
        lib.orc_generate_batch.restype = C.c_int
        lib.orc_generate_batch.argtypes = [C.c_void_p, C.c_int, _u16p, C.c_int, _intp,
                                           _u16p, C.c_int, C.c_int,
                                           C.POINTER(GenerationOptions), _u64p, _intp,
                                           C.c_int]
        lib.orc_rng_seed.restype = C.c_uint64
        lib.orc_rng_seed.argtypes = [C.c_uint64]
        lib.orc_rng_u64.restype = C.c_uint64
        lib.orc_rng_u64.argtypes = [_u64p]
        lib.orc_rng_f32.restype = C.c_float
        lib.orc_rng_f32.argtypes = [_u64p]
        lib.orc_rng_int.restype = C.c_int
        lib.orc_rng_int.argtypes = [_u64p, C.c_int, C.c_int]
        _orc_lib = lib
    return _orc_lib


class Rng:
    """xorshift64* (util.c:11-27) on the oracle side."""

    def __init__(self, seed: int):
        self.state = C.c_uint64(_load_orc().orc_rng_seed(seed))

    def u64(self):
        return _load_orc().orc_rng_u64(C.byref(self.state))

    def f32(self):
        return _load_orc().orc_rng_f32(C.byref(self.state))

    def int(self, lo, hi):
        return _load_orc().orc_rng_int(C.byref(self.state), lo, hi)


def random_prompt(n: int, vocab: int, seed: int) -> np.ndarray:
    """Uniform non-special ids in [4, vocab-1] drawn with rng_int."""
    r = Rng(seed)
    return np.array([r.int(4, vocab - 1) for _ in range(n)], dtype=np.uint16)


def ref_random_prompt(n: int, vocab: int, seed: int) -> np.ndarray:
    """The same prompt drawn with the reference's own rng_seed/rng_int
    (util.c:11-33) from oracle/_ref, for processes that must run nothing but
    the reference (the benchmark's reference arm)."""
    lib = _load_ref()
    st = C.c_uint64(0)
    lib.rng_seed(C.byref(st), seed)
    return np.array([lib.rng_int(C.byref(st), 4, vocab - 1) for _ in range(n)], dtype=np.uint16)


class _ModelBase:
    dims: Dims

    def tensors(self):
        """The nine weight arrays as numpy views (MODEL_ARRAYS order)."""
        out = []
        for i, shape in enumerate(self.dims.tensor_shapes()):
            n = C.c_size_t()
            p = self._tensor(i, n)
            arr = np.ctypeslib.as_array(p, shape=(n.value,)).reshape(shape)
            out.append(arr)
        return out


class RefModel(_ModelBase):
    """The reference's own model_init_config weights and decode path."""

    def __init__(self, dims: Dims, seed: int):
        self.lib = _load_ref()
        self.dims = dims
        self.h = self.lib.refsh_model_create(dims.vocab, dims.dim, dims.n_layers,
                                             dims.n_heads, dims.ffn_dim, dims.max_seq, seed)
        if not self.h:
            raise ValueError(f"reference rejected dims {dims}")

    def _tensor(self, i, n):
        return self.lib.refsh_tensor(self.h, i, C.byref(n))

    def param_count(self):
        return self.lib.refsh_param_count(self.h)

    def generate(self, prompt, out_cap, cache_max_seq, options, rng_state):
        p, pp = _u16(prompt)
        out = np.zeros(out_cap, dtype=np.uint16)
        st = C.c_uint64(rng_state)
        fp = C.c_int(0)
        n = self.lib.refsh_generate(self.h, pp, len(p), out.ctypes.data_as(_u16p), out_cap,
                                    cache_max_seq, C.byref(options), C.byref(st), C.byref(fp))
        return out[:n].copy(), st.value, fp.value

    def forward_logits(self, tokens):
        t, tp = _u16(tokens)
        out = np.zeros((len(t), self.dims.vocab), dtype=np.float32)
        if not self.lib.refsh_forward_logits(self.h, tp, len(t), out.ctypes.data_as(_f32p)):
            raise ValueError("model_forward rejected input")
        return out

    def check_kv_cache(self, tokens, tol):
        t, tp = _u16(tokens)
        return bool(self.lib.refsh_check_kv_cache(self.h, tp, len(t), tol))

    def checkpoint_save(self, path, optimizer=0, step=3, total_steps=10, rng_state=77,
                        tokenizer_hash=0x1234, moment_fill=0.0):
        """The reference's checkpoint_save (checkpoint.c:154-234) of these
        weights with a fresh optimizer of type `optimizer` (0 AdamW, 1 Lion)."""
        return bool(self.lib.refsh_checkpoint_save(self.h, os.fsencode(path), optimizer, step,
                                                   total_steps, rng_state, tokenizer_hash,
                                                   moment_fill))

    def checkpoint_load(self, path, optimizer=0, tokenizer_hash=0x1234):
        """The reference's checkpoint_load (checkpoint.c:301-426) into this
        model; returns (rng_state, step) or None when it rejects the file."""
        rng = C.c_uint64(0)
        step = C.c_int64(0)
        ok = self.lib.refsh_checkpoint_load(self.h, os.fsencode(path), optimizer, tokenizer_hash,
                                            C.byref(rng), C.byref(step))
        return (rng.value, step.value) if ok else None

    def close(self):
        if self.h:
            self.lib.refsh_model_free(self.h)
            self.h = None

    __del__ = close


class OrcModel(_ModelBase):
    """The restated CPU decoder (limits lifted)."""

    def __init__(self, dims: Dims, seed: int, bf16: bool = False):
        self.lib = _load_orc()
        self.dims = dims
        self.h = self.lib.orc_model_create(dims.vocab, dims.dim, dims.n_layers, dims.n_heads,
                                           dims.ffn_dim, dims.max_seq, seed, int(bf16))
        if not self.h:
            raise ValueError(f"oracle rejected dims {dims}")

    def _tensor(self, i, n):
        return self.lib.orc_model_tensor(self.h, i, C.byref(n))

    def forward_prefixes(self, tokens):
        t, tp = _u16(tokens)
        out = np.zeros((len(t), self.dims.vocab), dtype=np.float32)
        if not self.lib.orc_forward_prefixes(self.h, tp, len(t), out.ctypes.data_as(_f32p)):
            raise ValueError("bad tokens")
        return out

    def generate(self, prompt, out_cap, cache_max_seq, options, rng_state, trace_steps=0):
        p, pp = _u16(prompt)
        out = np.zeros(out_cap, dtype=np.uint16)
        st = C.c_uint64(rng_state)
        fp = C.c_int(0)
        trace = np.zeros((max(trace_steps, 1), self.dims.vocab), dtype=np.float32)
        n = self.lib.orc_generate(self.h, pp, len(p), out.ctypes.data_as(_u16p), out_cap,
                                  cache_max_seq, C.byref(options), C.byref(st),
                                  trace.ctypes.data_as(_f32p) if trace_steps else None,
                                  trace_steps, C.byref(fp))
        res = (out[:n].copy(), st.value, fp.value)
        return res + (trace[:trace_steps],) if trace_steps else res

    def generate_batch(self, prompts, prompt_lens, out_cap, cache_max_seq, options,
                       rng_states, nthreads=0):
        prompts = np.ascontiguousarray(prompts, dtype=np.uint16)
        B, stride = prompts.shape
        lens = np.ascontiguousarray(prompt_lens, dtype=np.int32)
        out = np.zeros((B, out_cap), dtype=np.uint16)
        st = np.ascontiguousarray(rng_states, dtype=np.uint64).copy()
        counts = np.zeros(B, dtype=np.int32)
        ok = self.lib.orc_generate_batch(self.h, B, prompts.ctypes.data_as(_u16p), stride,
                                         lens.ctypes.data_as(_intp), out.ctypes.data_as(_u16p),
                                         out_cap, cache_max_seq, C.byref(options),
                                         st.ctypes.data_as(_u64p),
                                         counts.ctypes.data_as(_intp), nthreads)
        return bool(ok), out, counts, st

    def close(self):
        if self.h:
            self.lib.orc_model_free(self.h)
            self.h = None

    __del__ = close


def sample(logits, options, history, rng_state):
    """Teacher-forced sampler: returns (id, new_rng_state)."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    h, hp = _u16(history)
    st = C.c_uint64(rng_state)
    r = _load_orc().orc_sample(lg.ctypes.data_as(_f32p), len(lg), C.byref(options), hp,
                               len(h), C.byref(st))
    return r, st.value
