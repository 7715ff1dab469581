"""minima_b200 — Minima's decode token loop on B200 (sm_100a).

Python mirror of the reference's generation interface for tests, the
benchmark and interactive use.  Everything here is a thin ctypes layer over
the in-tree native libraries:

* ``libminima_generate.so`` — the drop-in ``generate.h`` (generate.c's entry
  points, same signatures and return values) over the CUDA token loop;
* ``libminima_cuda.so``     — the C ABI ``include/minima_cuda.h``;
* ``libminima_host.so``     — seeded ``model_init_config`` / arena / RNG for
  programs that do not link the rest of Minima.

There is no CPU fallback: if the libraries are missing or the device is not
an sm_100 GPU, calls raise.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_CUDA = os.path.join(PKG, "libminima_cuda.so")
LIB_GEN = os.path.join(PKG, "libminima_generate.so")
LIB_HOST = os.path.join(PKG, "libminima_host.so")
LIB_FWD = os.path.join(PKG, "libminima_forward.so")

# Exported entry points, as declared in include/minima_cuda.h and
# include/minima_generate.h.
CUDA_SYMBOLS = ("mc_init", "mc_model_create", "mc_model_update", "mc_model_destroy",
                "mc_session_create", "mc_session_destroy", "mc_generate", "mc_forward_logits",
                "mc_last_kernel_ms", "mc_last_launch_count", "mc_last_step_times",
                "mc_last_kernel_name", "mc_last_prefill", "mc_session_stream", "mc_last_error",
                "mc_session_cluster_variant",
                "mc_checkpoint_inspect", "mc_model_load_checkpoint", "mc_gemm",
                "mc_model_forward", "mc_next_token_stats", "mc_generate_static",
                "mc_session_create_paged", "mc_model_forward_caches", "mc_matmul")
GENERATE_SYMBOLS = ("kvcache_init", "kvcache_reset", "generation_check_kv_cache",
                    "generation_inspect_next_tokens", "generate", "generate_with_options",
                    "generate_ex", "generate_batch_with_options", "minima_cuda_select_device",
                    "minima_cuda_model_sync", "minima_cuda_release_model",
                    "minima_cuda_release_cache", "minima_cuda_last_error",
                    "minima_cuda_last_kernel_ms")
FORWARD_SYMBOLS = ("activations_init", "rmsnorm", "matmul", "silu", "model_forward")
HOST_SYMBOLS = ("rng_seed", "rng_u64", "rng_f32", "rng_int", "arena_init", "arena_free",
                "arena_alloc", "arena_reset", "model_init_config", "model_config_validate",
                "model_validate", "model_param_count", "minima_host_model_arena_bytes",
                "minima_host_round_bf16")

MC_OK = 0
MC_WEIGHTS_F32 = 0
MC_WEIGHTS_BF16 = 1
MC_DEVICE_POINTERS = 1
TOK_MAX_VOCAB = 32768


# ----------------------------------------------------------------- structs
class ModelConfig(C.Structure):
    """config.h:25-32"""
    _fields_ = [("vocab_size", C.c_int), ("dim", C.c_int), ("n_layers", C.c_int),
                ("n_heads", C.c_int), ("ffn_dim", C.c_int), ("max_seq", C.c_int)]


class ArenaBudget(C.Structure):
    """arena.h:8-15"""
    _fields_ = [("limit", C.c_size_t), ("committed", C.c_size_t),
                ("external_committed", C.c_size_t), ("peak", C.c_size_t),
                ("failed", C.c_size_t), ("lock", C.c_long)]


class Arena(C.Structure):
    """arena.h:17-25"""
    _fields_ = [("base", C.c_void_p), ("size", C.c_size_t), ("used", C.c_size_t),
                ("peak", C.c_size_t), ("committed", C.c_size_t), ("page_size", C.c_size_t),
                ("budget", C.POINTER(ArenaBudget))]


_f32p = C.POINTER(C.c_float)


class Model(C.Structure):
    """model.h:9-41"""
    _fields_ = [("vocab_size", C.c_int), ("dim", C.c_int), ("n_layers", C.c_int),
                ("n_heads", C.c_int), ("n_kv_heads", C.c_int), ("head_dim", C.c_int),
                ("kv_dim", C.c_int), ("qkv_dim", C.c_int), ("ffn_dim", C.c_int),
                ("max_seq", C.c_int),
                ("tok_emb", _f32p), ("attn_qkv", _f32p), ("attn_proj", _f32p),
                ("ffn_up", _f32p), ("ffn_gate", _f32p), ("ffn_down", _f32p),
                ("rms1_scale", _f32p), ("rms2_scale", _f32p), ("rms_final_scale", _f32p),
                ("weight_bytes", C.c_size_t), ("memory_budget", C.POINTER(ArenaBudget))]


class Rng(C.Structure):
    """util.h:10-12"""
    _fields_ = [("state", C.c_uint64)]


class KVCache(C.Structure):
    """generate.h:11-24"""
    _fields_ = [("max_seq", C.c_int), ("n_layers", C.c_int), ("n_heads", C.c_int),
                ("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("dim", C.c_int),
                ("kv_dim", C.c_int), ("k_cache", _f32p), ("v_cache", _f32p), ("pos", C.c_int)]


class Merge(C.Structure):
    """tokenizer.h:20-23"""
    _fields_ = [("left", C.c_uint16), ("right", C.c_uint16)]


class Tokenizer(C.Structure):
    """tokenizer.h:25-41 (generation reads vocab_size, token_str, token_len)"""
    _fields_ = [("vocab_size", C.c_int), ("n_merges", C.c_int),
                ("memory_budget", C.POINTER(ArenaBudget)),
                ("token_str", C.c_char_p * TOK_MAX_VOCAB),
                ("token_len", C.c_int * TOK_MAX_VOCAB),
                ("merges", Merge * (TOK_MAX_VOCAB - 260)),
                ("merge_rank_index", C.c_void_p), ("merge_rank_capacity", C.c_uint32)]


class GenerationOptions(C.Structure):
    """generate.h:50-63 (also the layout of mc_sampling)"""
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float),
                ("repetition_penalty", C.c_float), ("min_p", C.c_float),
                ("frequency_penalty", C.c_float), ("presence_penalty", C.c_float),
                ("top_k", C.c_int), ("max_new_tokens", C.c_int), ("min_new_tokens", C.c_int),
                ("no_repeat_ngram_size", C.c_int),
                ("stop_sequence_ids", C.POINTER(C.c_uint16)), ("stop_sequence_len", C.c_int)]


class ModelDesc(C.Structure):
    """mc_model_desc (include/minima_cuda.h)"""
    _fields_ = [(n, C.c_int) for n in ("vocab_size", "dim", "n_layers", "n_heads", "n_kv_heads",
                                       "head_dim", "kv_dim", "qkv_dim", "ffn_dim", "max_seq")] + \
               [(n, _f32p) for n in ("tok_emb", "attn_qkv", "attn_proj", "ffn_up", "ffn_gate",
                                     "ffn_down", "rms1_scale", "rms2_scale", "rms_final_scale")]


def options(temperature=1.0, top_k=1, top_p=1.0, repetition_penalty=1.0, min_p=0.0,
            frequency_penalty=0.0, presence_penalty=0.0, max_new_tokens=0, min_new_tokens=0,
            no_repeat_ngram_size=0, stop=None) -> GenerationOptions:
    """GenerationOptions with generate_ex's defaults (generate.c:604-625)."""
    o = GenerationOptions(temperature, top_p, repetition_penalty, min_p, frequency_penalty,
                          presence_penalty, top_k, max_new_tokens, min_new_tokens,
                          no_repeat_ngram_size, None, 0)
    if stop:
        arr = (C.c_uint16 * len(stop))(*stop)
        o._keep = arr
        o.stop_sequence_ids = C.cast(arr, C.POINTER(C.c_uint16))
        o.stop_sequence_len = len(stop)
    return o


# ----------------------------------------------------------------- loading
_libs = {}


class MinimaCudaError(RuntimeError):
    pass


def libs():
    """(host, cuda, generate) ctypes handles; raises if a library is missing."""
    if not _libs:
        for path in (LIB_HOST, LIB_CUDA, LIB_GEN):
            if not os.path.exists(path):
                raise MinimaCudaError(f"{os.path.basename(path)} is not built: run "
                                      "python -m minima_b200.build (or __graft_entry__.build())")
        # host support first and global, so the drop-in resolves model_validate
        # and arena_alloc against it as it would against Minima's own files.
        host = C.CDLL(LIB_HOST, mode=C.RTLD_GLOBAL)
        cuda = C.CDLL(LIB_CUDA, mode=C.RTLD_GLOBAL)
        gen = C.CDLL(LIB_GEN)
        _declare(host, cuda, gen)
        _libs.update(host=host, cuda=cuda, gen=gen)
    return _libs["host"], _libs["cuda"], _libs["gen"]


def forward_lib():
    """ctypes handle of libminima_forward.so, the drop-in forward.h (loaded
    after the libraries it depends on)."""
    if "fwd" not in _libs:
        libs()
        if not os.path.exists(LIB_FWD):
            raise MinimaCudaError("libminima_forward.so is not built: run python -m minima_b200.build")
        fwd = C.CDLL(LIB_FWD)
        fwd.activations_init.restype = C.c_bool
        fwd.model_forward.restype = C.POINTER(C.c_float)
        fwd.silu.restype = C.c_float
        fwd.silu.argtypes = [C.c_float]
        _libs["fwd"] = fwd
    return _libs["fwd"]


def _declare(host, cuda, gen):
    u16p, i32p, u64p = C.POINTER(C.c_uint16), C.POINTER(C.c_int), C.POINTER(C.c_uint64)
    vp = C.c_void_p
    host.arena_init.restype = C.c_bool
    host.arena_init.argtypes = [C.POINTER(Arena), C.c_size_t]
    host.arena_free.argtypes = [C.POINTER(Arena)]
    host.model_init_config.restype = C.c_bool
    host.model_init_config.argtypes = [C.POINTER(Model), C.POINTER(Arena), C.c_uint64,
                                       C.POINTER(ModelConfig)]
    host.model_validate.restype = C.c_bool
    host.model_validate.argtypes = [C.POINTER(Model)]
    host.model_param_count.restype = C.c_size_t
    host.model_param_count.argtypes = [C.POINTER(Model)]
    host.minima_host_model_arena_bytes.restype = C.c_size_t
    host.minima_host_model_arena_bytes.argtypes = [C.POINTER(ModelConfig)]
    host.minima_host_round_bf16.argtypes = [C.POINTER(Model)]
    host.rng_seed.argtypes = [C.POINTER(Rng), C.c_uint64]
    host.rng_int.restype = C.c_int
    host.rng_int.argtypes = [C.POINTER(Rng), C.c_int, C.c_int]

    cuda.mc_init.argtypes = [C.c_int]
    cuda.mc_model_create.argtypes = [C.POINTER(ModelDesc), C.c_int, C.POINTER(vp)]
    cuda.mc_model_update.argtypes = [vp, C.POINTER(ModelDesc)]
    cuda.mc_model_destroy.argtypes = [vp]
    cuda.mc_session_create.argtypes = [vp, C.c_int, C.c_int, C.POINTER(vp)]
    cuda.mc_session_create_paged.argtypes = [vp, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(vp)]
    cuda.mc_session_destroy.argtypes = [vp]
    cuda.mc_generate.argtypes = [vp, C.c_int, vp, C.c_int, i32p, vp, C.c_int,
                                 C.POINTER(GenerationOptions), vp, vp, vp, C.c_uint, _f32p, C.c_int]
    cuda.mc_forward_logits.argtypes = [vp, C.c_int, u16p, C.c_int, _f32p]
    cuda.mc_last_kernel_ms.argtypes = [vp, _f32p]
    cuda.mc_last_launch_count.argtypes = [vp, i32p]
    cuda.mc_last_step_times.argtypes = [vp, u64p, C.c_int, i32p]
    cuda.mc_session_stream.argtypes = [vp, C.POINTER(vp)]
    cuda.mc_last_prefill.argtypes = [vp, i32p, _f32p]
    cuda.mc_last_kernel_name.restype = C.c_char_p
    cuda.mc_last_kernel_name.argtypes = [vp]
    cuda.mc_session_cluster_variant.argtypes = [vp, C.POINTER(C.c_int)]
    cuda.mc_last_error.restype = C.c_char_p
    cuda.mc_model_forward.argtypes = [vp, C.c_int, C.c_int, u16p, _f32p, C.c_uint]
    cuda.mc_gemm.argtypes = [C.c_int, vp, vp, _f32p, C.c_int, C.c_int, C.c_int, C.c_uint, _f32p]
    cuda.mc_checkpoint_inspect.argtypes = [C.c_char_p, C.POINTER(CheckpointInfo)]
    cuda.mc_model_load_checkpoint.argtypes = [C.c_char_p, C.c_int, C.c_uint64, C.c_uint,
                                              C.POINTER(vp), C.POINTER(CheckpointInfo)]

    gen.kvcache_init.restype = C.c_bool
    gen.kvcache_init.argtypes = [C.POINTER(KVCache), C.POINTER(Arena), C.POINTER(Model), C.c_int]
    gen.kvcache_reset.argtypes = [C.POINTER(KVCache)]
    gen.generate_with_options.restype = C.c_int
    gen.generate_with_options.argtypes = [C.POINTER(Model), C.POINTER(Tokenizer),
                                          C.POINTER(KVCache), u16p, C.c_int, u16p, C.c_int,
                                          C.POINTER(GenerationOptions), C.POINTER(Rng)]
    gen.generate_ex.restype = C.c_int
    gen.generate_ex.argtypes = [C.POINTER(Model), C.POINTER(Tokenizer), C.POINTER(KVCache), u16p,
                                C.c_int, u16p, C.c_int, C.c_int, C.c_float, C.c_int, C.c_float,
                                C.c_float, C.POINTER(Rng)]
    gen.generate.restype = C.c_int
    gen.generate.argtypes = [C.POINTER(Model), C.POINTER(Tokenizer), C.POINTER(KVCache), u16p,
                             C.c_int, u16p, C.c_int, C.c_int, C.c_float, C.c_int, C.POINTER(Rng)]
    gen.generate_batch_with_options.restype = C.c_int
    gen.generate_batch_with_options.argtypes = [C.POINTER(Model), C.POINTER(Tokenizer),
                                                C.POINTER(KVCache), C.c_int, u16p, C.c_int, i32p,
                                                u16p, C.c_int, C.POINTER(GenerationOptions),
                                                C.POINTER(Rng), i32p]
    gen.generation_inspect_next_tokens.restype = C.c_bool
    gen.generation_inspect_next_tokens.argtypes = [C.POINTER(Model), C.POINTER(Tokenizer),
                                                   C.POINTER(KVCache), u16p, C.c_int, C.c_int]
    gen.minima_cuda_select_device.restype = C.c_int
    gen.minima_cuda_select_device.argtypes = [C.c_int]
    gen.minima_cuda_model_sync.restype = C.c_int
    gen.minima_cuda_model_sync.argtypes = [C.POINTER(Model)]
    gen.minima_cuda_release_model.argtypes = [C.POINTER(Model)]
    gen.minima_cuda_release_cache.argtypes = [C.POINTER(KVCache)]
    gen.minima_cuda_last_error.restype = C.c_char_p
    gen.minima_cuda_last_kernel_ms.restype = C.c_float


def _check(status, what):
    if status != MC_OK:
        msg = libs()[1].mc_last_error().decode(errors="replace")
        raise MinimaCudaError(f"{what}: status {status}: {msg}")


def kv_head_count(n_heads: int) -> int:
    """model_kv_head_count (model.c:34-40)."""
    if n_heads <= 1:
        return 1
    for kv in range(n_heads // 2, 0, -1):
        if n_heads % kv == 0:
            return kv
    return 1


# -------------------------------------------------------------- host model
class HostModel:
    """A Model filled by model_init_config(seed) in its own arena."""

    def __init__(self, vocab_size, dim, n_layers, n_heads, ffn_dim, max_seq, seed, bf16=False):
        host, _, _ = libs()
        self.config = ModelConfig(vocab_size, dim, n_layers, n_heads, ffn_dim, max_seq)
        self.arena = Arena()
        nbytes = host.minima_host_model_arena_bytes(C.byref(self.config))
        if not host.arena_init(C.byref(self.arena), nbytes):
            raise MemoryError("arena_init")
        self.model = Model()
        if not host.model_init_config(C.byref(self.model), C.byref(self.arena), seed,
                                      C.byref(self.config)):
            host.arena_free(C.byref(self.arena))
            raise ValueError(f"model_init_config rejected {self.config_tuple()}")
        if bf16:
            host.minima_host_round_bf16(C.byref(self.model))
        self.bf16 = bf16

    def config_tuple(self):
        c = self.config
        return (c.vocab_size, c.dim, c.n_layers, c.n_heads, c.ffn_dim, c.max_seq)

    def param_count(self):
        return libs()[0].model_param_count(C.byref(self.model))

    def tensors(self):
        """numpy views of the nine arrays (MODEL_ARRAYS order)."""
        m = self.model
        V, D, L, F, Q = m.vocab_size, m.dim, m.n_layers, m.ffn_dim, m.qkv_dim
        shapes = [(V, D), (L, Q, D), (L, D, D), (L, F, D), (L, F, D), (L, D, F), (L, D), (L, D), (D,)]
        ptrs = [m.tok_emb, m.attn_qkv, m.attn_proj, m.ffn_up, m.ffn_gate, m.ffn_down,
                m.rms1_scale, m.rms2_scale, m.rms_final_scale]
        return [np.ctypeslib.as_array(p, shape=(int(np.prod(s)),)).reshape(s)
                for p, s in zip(ptrs, shapes)]

    def desc(self) -> ModelDesc:
        m = self.model
        return ModelDesc(m.vocab_size, m.dim, m.n_layers, m.n_heads, m.n_kv_heads, m.head_dim,
                         m.kv_dim, m.qkv_dim, m.ffn_dim, m.max_seq, m.tok_emb, m.attn_qkv,
                         m.attn_proj, m.ffn_up, m.ffn_gate, m.ffn_down, m.rms1_scale,
                         m.rms2_scale, m.rms_final_scale)

    def close(self):
        if getattr(self, "arena", None) is not None and self.arena.base:
            host, _, gen = libs()
            gen.minima_cuda_release_model(C.byref(self.model))
            host.arena_free(C.byref(self.arena))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def make_tokenizer(vocab_size: int) -> Tokenizer:
    """A Tokenizer with only vocab_size set (all generate.c reads from it)."""
    t = Tokenizer()
    t.vocab_size = vocab_size
    return t


class Caches:
    """`batch` KVCache structs from kvcache_init, backed by one arena."""

    def __init__(self, hm: HostModel, batch: int, max_seq: int):
        host, _, gen = libs()
        m = hm.model
        self.arena = Arena()
        per = m.n_layers * max_seq * m.kv_dim * 4
        if not host.arena_init(C.byref(self.arena), batch * (2 * per + 256) + 4096):
            raise MemoryError("arena_init")
        self.caches = (KVCache * batch)()
        for b in range(batch):
            if not gen.kvcache_init(C.byref(self.caches[b]), C.byref(self.arena), C.byref(m),
                                    max_seq):
                raise ValueError("kvcache_init rejected the configuration")

    def close(self):
        if self.arena.base:
            host, _, gen = libs()
            for c in self.caches:
                gen.minima_cuda_release_cache(C.byref(c))
            host.arena_free(C.byref(self.arena))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def last_error() -> str:
    return libs()[2].minima_cuda_last_error().decode(errors="replace")


def generate_with_options(hm: HostModel, tok: Tokenizer, cache: KVCache, prompt, out_cap,
                          opts: GenerationOptions, rng_state: int):
    """generate_with_options through the drop-in; returns (ids, rng_state, cache.pos)."""
    _, _, gen = libs()
    p = np.ascontiguousarray(prompt, dtype=np.uint16)
    out = np.zeros(max(out_cap, 1), dtype=np.uint16)
    rng = Rng(rng_state)
    n = gen.generate_with_options(C.byref(hm.model), C.byref(tok), C.byref(cache),
                                  p.ctypes.data_as(C.POINTER(C.c_uint16)), len(p),
                                  out.ctypes.data_as(C.POINTER(C.c_uint16)), out_cap,
                                  C.byref(opts), C.byref(rng))
    return out[:n].copy(), rng.state, cache.pos


def generate_batch(hm: HostModel, tok: Tokenizer, caches: Caches, prompts, prompt_lens, out_cap,
                   opts: GenerationOptions, rng_states):
    """generate_batch_with_options; returns (ok, out[B, out_cap], counts, rng_states)."""
    _, _, gen = libs()
    prompts = np.ascontiguousarray(prompts, dtype=np.uint16)
    B, stride = prompts.shape
    lens = np.ascontiguousarray(prompt_lens, dtype=np.int32)
    out = np.zeros((B, out_cap), dtype=np.uint16)
    rngs = (Rng * B)(*[Rng(int(s)) for s in rng_states])
    counts = np.zeros(B, dtype=np.int32)
    ok = gen.generate_batch_with_options(C.byref(hm.model), C.byref(tok), caches.caches, B,
                                         prompts.ctypes.data_as(C.POINTER(C.c_uint16)), stride,
                                         lens.ctypes.data_as(C.POINTER(C.c_int)),
                                         out.ctypes.data_as(C.POINTER(C.c_uint16)), out_cap,
                                         C.byref(opts), rngs,
                                         counts.ctypes.data_as(C.POINTER(C.c_int)))
    return bool(ok), out, counts, np.array([r.state for r in rngs], dtype=np.uint64)


# ------------------------------------------------------------ C ABI layer
MC_CKPT_ANY_TOKENIZER = 0x1
MC_GEMM_TF32, MC_GEMM_BF16 = 0, 1


def gemm(a, b, kind=MC_GEMM_TF32, device=0):
    """mc_gemm: a[M][K] . b[N][K]^T on the tensor cores (host arrays).  For
    MC_GEMM_BF16, a and b are uint16 arrays of bf16 bit patterns.  Returns
    (C fp32 [M][N], kernel milliseconds)."""
    _, cuda, _ = libs()
    _check(cuda.mc_init(device), "mc_init")
    dt = np.float32 if kind == MC_GEMM_TF32 else np.uint16
    a = np.ascontiguousarray(a, dtype=dt)
    b = np.ascontiguousarray(b, dtype=dt)
    (M, K), (N, K2) = a.shape, b.shape
    assert K == K2
    c = np.zeros((M, N), dtype=np.float32)
    ms = C.c_float(0.0)
    _check(cuda.mc_gemm(kind, a.ctypes.data, b.ctypes.data, c.ctypes.data_as(_f32p), M, N, K, 0,
                        C.byref(ms)), "mc_gemm")
    return c, ms.value


class CheckpointInfo(C.Structure):
    """mc_checkpoint_info: a checkpoint's header (checkpoint.c:154-234)."""
    _fields_ = [("version", C.c_uint32), ("vocab_size", C.c_int32), ("dim", C.c_int32),
                ("n_layers", C.c_int32), ("n_heads", C.c_int32), ("ffn_dim", C.c_int32),
                ("max_seq", C.c_int32), ("n_params", C.c_uint64), ("step", C.c_int64),
                ("rng_state", C.c_uint64), ("tokenizer_hash", C.c_uint64), ("lr", C.c_float),
                ("beta1", C.c_float), ("beta2", C.c_float), ("eps", C.c_float),
                ("weight_decay", C.c_float), ("schedule_base_lr", C.c_float),
                ("schedule_total_steps", C.c_int64), ("schedule_warmup_steps", C.c_int64),
                ("schedule_type", C.c_int32), ("optimizer_type", C.c_int32),
                ("header_bytes", C.c_uint64), ("file_bytes", C.c_uint64)]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


def checkpoint_inspect(path):
    """mc_checkpoint_inspect: header and length checks of checkpoint_load, no
    device work.  Returns the header as a dict; raises MinimaCudaError when
    the file would be rejected."""
    _, cuda, _ = libs()
    info = CheckpointInfo()
    _check(cuda.mc_checkpoint_inspect(os.fsencode(path), C.byref(info)), "mc_checkpoint_inspect")
    return info.as_dict()


class DeviceModel:
    """mc_model: weights of a HostModel resident on the current device."""

    def __init__(self, hm: HostModel, dtype=MC_WEIGHTS_F32, device=0):
        _, cuda, _ = libs()
        _check(cuda.mc_init(device), "mc_init")
        self.h = C.c_void_p()
        self._desc = hm.desc()
        self.info = None
        _check(cuda.mc_model_create(C.byref(self._desc), dtype, C.byref(self.h)), "mc_model_create")

    @classmethod
    def from_checkpoint(cls, path, dtype=MC_WEIGHTS_F32, tokenizer_hash=None, device=0):
        """mc_model_load_checkpoint: the model arrays of a reference
        checkpoint streamed to the device.  tokenizer_hash=None accepts any
        fingerprint.  The header is kept in .info."""
        _, cuda, _ = libs()
        _check(cuda.mc_init(device), "mc_init")
        self = cls.__new__(cls)
        self.h = C.c_void_p()
        info = CheckpointInfo()
        flags = MC_CKPT_ANY_TOKENIZER if tokenizer_hash is None else 0
        _check(cuda.mc_model_load_checkpoint(os.fsencode(path), dtype, tokenizer_hash or 0, flags,
                                             C.byref(self.h), C.byref(info)),
               "mc_model_load_checkpoint")
        self.info = info.as_dict()
        # dimensions only: the weights live on the device
        K = kv_head_count(info.n_heads)
        hd = info.dim // info.n_heads
        self._desc = ModelDesc(info.vocab_size, info.dim, info.n_layers, info.n_heads, K, hd,
                               K * hd, info.dim + 2 * K * hd, info.ffn_dim, info.max_seq)
        return self

    def close(self):
        if self.h:
            libs()[1].mc_model_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Session:
    """mc_session: device KV cache and work buffers for up to max_batch sequences."""

    def __init__(self, dm: DeviceModel, max_batch: int, max_seq: int, page_len: int = 0,
                 n_pages: int = 0):
        """page_len > 0: a paged KV cache of n_pages pages of page_len
        positions (mc_session_create_paged); else every sequence owns
        max_seq positions."""
        _, cuda, _ = libs()
        self.dm = dm
        self.h = C.c_void_p()
        if page_len:
            _check(cuda.mc_session_create_paged(dm.h, max_batch, max_seq, page_len, n_pages,
                                                C.byref(self.h)), "mc_session_create_paged")
        else:
            _check(cuda.mc_session_create(dm.h, max_batch, max_seq, C.byref(self.h)),
                   "mc_session_create")

    def generate(self, prompts, prompt_lens, out_cap, opts, rng_states, trace_steps=0):
        """mc_generate with host buffers; returns (out, counts, rng_states, final_pos[, trace])."""
        _, cuda, _ = libs()
        prompts = np.ascontiguousarray(prompts, dtype=np.uint16)
        B, stride = prompts.shape
        lens = np.ascontiguousarray(prompt_lens, dtype=np.int32)
        out = np.zeros((B, out_cap), dtype=np.uint16)
        st = np.ascontiguousarray(rng_states, dtype=np.uint64).copy()
        counts = np.zeros(B, dtype=np.int32)
        fpos = np.zeros(B, dtype=np.int32)
        V = self.dm._desc.vocab_size
        trace = np.zeros((B, trace_steps, V), dtype=np.float32) if trace_steps else None
        _check(cuda.mc_generate(self.h, B, prompts.ctypes.data, stride,
                                lens.ctypes.data_as(C.POINTER(C.c_int)), out.ctypes.data, out_cap,
                                C.byref(opts), st.ctypes.data, counts.ctypes.data, fpos.ctypes.data,
                                0, trace.ctypes.data_as(_f32p) if trace_steps else None,
                                trace_steps), "mc_generate")
        res = (out, counts, st, fpos)
        return res + (trace,) if trace_steps else res

    def generate_device(self, prompts_ptr, prompt_stride, prompt_lens, out_ptr, out_cap, opts,
                        rng_ptr, counts_ptr, fpos_ptr=None):
        """mc_generate on device-resident buffers (MC_DEVICE_POINTERS)."""
        _, cuda, _ = libs()
        lens = np.ascontiguousarray(prompt_lens, dtype=np.int32)
        self._lens = lens
        _check(cuda.mc_generate(self.h, len(lens), prompts_ptr, prompt_stride,
                                lens.ctypes.data_as(C.POINTER(C.c_int)), out_ptr, out_cap,
                                C.byref(opts), rng_ptr, counts_ptr, fpos_ptr, MC_DEVICE_POINTERS,
                                None, 0), "mc_generate")

    def forward_logits(self, tokens):
        """Teacher-forced per-prefix logits, tokens [B, n] -> [B, n, V]."""
        _, cuda, _ = libs()
        t = np.ascontiguousarray(tokens, dtype=np.uint16)
        B, n = t.shape
        V = self.dm._desc.vocab_size
        out = np.zeros((B, n, V), dtype=np.float32)
        _check(cuda.mc_forward_logits(self.h, B, t.ctypes.data_as(C.POINTER(C.c_uint16)), n,
                                      out.ctypes.data_as(_f32p)), "mc_forward_logits")
        return out

    def last_kernel_ms(self):
        ms = C.c_float()
        _check(libs()[1].mc_last_kernel_ms(self.h, C.byref(ms)), "mc_last_kernel_ms")
        return ms.value

    def last_launch_count(self):
        n = C.c_int()
        _check(libs()[1].mc_last_launch_count(self.h, C.byref(n)), "mc_last_launch_count")
        return n.value

    def last_step_times_ns(self, cap=1 << 16):
        """%globaltimer stamps at the start of each token step of the last call."""
        buf = np.zeros(cap, dtype=np.uint64)
        n = C.c_int()
        _check(libs()[1].mc_last_step_times(self.h, buf.ctypes.data_as(C.POINTER(C.c_uint64)),
                                            cap, C.byref(n)), "mc_last_step_times")
        return buf[:n.value]

    def model_forward(self, tokens):
        """mc_model_forward: logits [B][S][V] of every position (batched causal
        forward) for tokens [B][S]."""
        _, cuda, _ = libs()
        t = np.ascontiguousarray(tokens, dtype=np.uint16)
        B, S = t.shape
        V = self.dm._desc.vocab_size
        out = np.zeros((B, S, V), dtype=np.float32)
        _check(cuda.mc_model_forward(self.h, B, S, t.ctypes.data_as(C.POINTER(C.c_uint16)),
                                     out.ctypes.data_as(_f32p), 0), "mc_model_forward")
        return out

    def last_prefill(self):
        """(positions prefilled in one batch, prefill device ms) of the last call."""
        n, ms = C.c_int(), C.c_float()
        _check(libs()[1].mc_last_prefill(self.h, C.byref(n), C.byref(ms)), "mc_last_prefill")
        return n.value, ms.value

    def last_kernel_name(self) -> str:
        return libs()[1].mc_last_kernel_name(self.h).decode()

    def cluster_variant(self) -> int:
        """Layer loop of the cluster-resident plan (-1 none, 0 five phases,
        1 two phases with cluster barriers, 2 two phases, dataflow)."""
        v = C.c_int()
        _check(libs()[1].mc_session_cluster_variant(self.h, C.byref(v)), "mc_session_cluster_variant")
        return v.value

    def stream_handle(self) -> int:
        """cudaStream_t of this session, as an integer handle."""
        h = C.c_void_p()
        _check(libs()[1].mc_session_stream(self.h, C.byref(h)), "mc_session_stream")
        return h.value or 0

    def close(self):
        if self.h:
            libs()[1].mc_session_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
