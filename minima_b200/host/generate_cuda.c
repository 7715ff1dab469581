/*
 * generate_cuda.c — drop-in replacement for the Minima reference's
 * generate.c, running the token loop on a B200 through minima_cuda.h.
 *
 * Same entry points, signatures, validation order and return values as
 * generate.c (cited per function).  Host-side dependencies are the ones
 * generate.c has on the rest of the program: model_validate (model.c:55-89)
 * and arena_alloc / arena_reset (arena.c:127-177).  Inside Minima those
 * come from its own files; a standalone program links libminima_host.so
 * instead.  generation_check_kv_cache compares two device paths, as the
 * reference compares its two CPU paths: the token loop position by position
 * and the batched causal forward (the drop-in model_forward's kernels).
 *
 * Device state (uploaded weights, device KV caches) is kept in small side
 * tables keyed by the caller's Model* / KVCache*, so the reference structs
 * are used exactly as laid out by the caller.
 */
#include "minima_generate.h"
#include "minima_cuda.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>


/* Host program symbols (generate.c's own dependencies). */
bool model_validate(const Model* model);
void* arena_alloc(Arena* a, size_t n);
void arena_reset(Arena* a);

/* ------------------------------------------------------------ side tables */

typedef struct {
    const Model* key;
    mc_model* dev;
    uint64_t sig;
    int dims[6];
} ModelEntry;

typedef struct {
    const KVCache* key;
    mc_session* sess;
    mc_model* dev;
    int cap;
    int bcap;
} CacheEntry;

#define MAX_MODELS 16
#define MAX_CACHES 64
static ModelEntry g_models[MAX_MODELS];
static CacheEntry g_caches[MAX_CACHES];
static int g_device = -1;
static char g_err[512];
static float g_last_ms;

static void set_err(const char* what) {
    snprintf(g_err, sizeof(g_err), "%s: %s", what, mc_last_error());
}

const char* minima_cuda_last_error(void) { return g_err; }
float minima_cuda_last_kernel_ms(void) { return g_last_ms; }

int minima_cuda_select_device(int device) {
    if (mc_init(device) != MC_OK) {
        set_err("mc_init");
        return 0;
    }
    g_device = device;
    return 1;
}

static int ensure_device(void) {
    if (g_device >= 0) return mc_init(g_device) == MC_OK;
    const char* env = getenv("MINIMA_CUDA_DEVICE");
    return minima_cuda_select_device(env ? atoi(env) : 0);
}

/* Cheap change detector over the weights: dims, pointers and a few hundred
   sampled values per tensor.  minima_cuda_model_sync forces an upload. */
static uint64_t mix(uint64_t h, uint64_t v) {
    h ^= v + 0x9E3779B97F4A7C15ULL + (h << 6) + (h >> 2);
    return h;
}

static uint64_t weight_signature(const Model* m) {
    const size_t D = (size_t)m->dim, L = (size_t)m->n_layers, F = (size_t)m->ffn_dim;
    const float* t[9] = {m->tok_emb, m->attn_qkv, m->attn_proj, m->ffn_up, m->ffn_gate,
        m->ffn_down, m->rms1_scale, m->rms2_scale, m->rms_final_scale};
    const size_t n[9] = {(size_t)m->vocab_size * D, L * (size_t)m->qkv_dim * D, L * D * D,
        L * F * D, L * F * D, L * D * F, L * D, L * D, D};
    uint64_t h = 0x243F6A8885A308D3ULL;
    for (int i = 0; i < 9; i++) {
        h = mix(h, (uint64_t)(uintptr_t)t[i]);
        h = mix(h, n[i]);
        const size_t step = n[i] > 512 ? n[i] / 512 : 1;
        for (size_t k = 0; k < n[i]; k += step) {
            uint32_t u;
            memcpy(&u, t[i] + k, 4);
            h = mix(h, u);
        }
        for (size_t k = 0; k < 64 && k < n[i]; k++) {   /* row starts of tok_emb etc. */
            const size_t at = (k * D) < n[i] ? k * D : n[i] - 1;
            uint32_t u;
            memcpy(&u, t[i] + at, 4);
            h = mix(h, u);
        }
    }
    return h;
}

static int weight_dtype(void) {
    const char* env = getenv("MINIMA_CUDA_WEIGHTS");
    return (env && strcmp(env, "bf16") == 0) ? MC_WEIGHTS_BF16 : MC_WEIGHTS_F32;
}

static mc_model_desc describe(const Model* m) {
    mc_model_desc d;
    d.vocab_size = m->vocab_size; d.dim = m->dim; d.n_layers = m->n_layers;
    d.n_heads = m->n_heads; d.n_kv_heads = m->n_kv_heads; d.head_dim = m->head_dim;
    d.kv_dim = m->kv_dim; d.qkv_dim = m->qkv_dim; d.ffn_dim = m->ffn_dim;
    d.max_seq = m->max_seq;
    d.tok_emb = m->tok_emb; d.attn_qkv = m->attn_qkv; d.attn_proj = m->attn_proj;
    d.ffn_up = m->ffn_up; d.ffn_gate = m->ffn_gate; d.ffn_down = m->ffn_down;
    d.rms1_scale = m->rms1_scale; d.rms2_scale = m->rms2_scale;
    d.rms_final_scale = m->rms_final_scale;
    return d;
}

static void drop_forward_sessions_of(mc_model* dev);

static void drop_sessions_of(mc_model* dev) {
    drop_forward_sessions_of(dev);
    for (int i = 0; i < MAX_CACHES; i++)
        if (g_caches[i].key && g_caches[i].dev == dev) {
            mc_session_destroy(g_caches[i].sess);
            memset(&g_caches[i], 0, sizeof(g_caches[i]));
        }
}

static mc_model* device_model(const Model* m, int force) {
    if (!ensure_device()) return NULL;
    const uint64_t sig = weight_signature(m);
    const int dims[6] = {m->vocab_size, m->dim, m->n_layers, m->n_heads, m->ffn_dim, m->max_seq};
    ModelEntry* e = NULL;
    for (int i = 0; i < MAX_MODELS; i++)
        if (g_models[i].key == m) { e = &g_models[i]; break; }
    const mc_model_desc d = describe(m);
    if (e && memcmp(e->dims, dims, sizeof(dims)) == 0) {
        if (!force && e->sig == sig) return e->dev;
        if (mc_model_update(e->dev, &d) != MC_OK) { set_err("mc_model_update"); return NULL; }
        e->sig = sig;
        return e->dev;
    }
    if (e) {
        drop_sessions_of(e->dev);
        mc_model_destroy(e->dev);
        memset(e, 0, sizeof(*e));
    } else {
        for (int i = 0; i < MAX_MODELS && !e; i++)
            if (!g_models[i].key) e = &g_models[i];
        if (!e) {   /* table full: evict slot 0 */
            e = &g_models[0];
            drop_sessions_of(e->dev);
            mc_model_destroy(e->dev);
            memset(e, 0, sizeof(*e));
        }
    }
    mc_model* dev = NULL;
    if (mc_model_create(&d, weight_dtype(), &dev) != MC_OK) { set_err("mc_model_create"); return NULL; }
    e->key = m;
    e->dev = dev;
    e->sig = sig;
    memcpy(e->dims, dims, sizeof(dims));
    return dev;
}

static mc_session* device_session(const KVCache* cache, mc_model* dev, int batch) {
    CacheEntry* e = NULL;
    for (int i = 0; i < MAX_CACHES; i++)
        if (g_caches[i].key == cache) { e = &g_caches[i]; break; }
    if (e && e->dev == dev && e->cap == cache->max_seq && e->bcap >= batch) return e->sess;
    if (e) {
        mc_session_destroy(e->sess);
        memset(e, 0, sizeof(*e));
    } else {
        for (int i = 0; i < MAX_CACHES && !e; i++)
            if (!g_caches[i].key) e = &g_caches[i];
        if (!e) {
            e = &g_caches[0];
            mc_session_destroy(e->sess);
            memset(e, 0, sizeof(*e));
        }
    }
    mc_session* s = NULL;
    if (mc_session_create(dev, batch, cache->max_seq, &s) != MC_OK) {
        set_err("mc_session_create");
        return NULL;
    }
    e->key = cache;
    e->sess = s;
    e->dev = dev;
    e->cap = cache->max_seq;
    e->bcap = batch;
    return s;
}

/* Forward sessions, one per model (the drop-in model_forward's device
   state), grown to the largest batch and sequence length asked for. */
typedef struct {
    const Model* key;
    mc_session* sess;
    mc_model* dev;
    int bcap, cap;
} ForwardEntry;
static ForwardEntry g_forward[MAX_MODELS];

struct mc_session* minima_cuda_forward_session(const Model* model, int batch, int seq) {
    if (!model || batch <= 0 || seq <= 0 || batch > MC_MAX_BATCH || seq > model->max_seq) return NULL;
    mc_model* dev = device_model(model, 0);
    if (!dev) return NULL;
    ForwardEntry* e = NULL;
    for (int i = 0; i < MAX_MODELS && !e; i++)
        if (g_forward[i].key == model) e = &g_forward[i];
    if (e && e->dev == dev && e->bcap >= batch && e->cap >= seq) return e->sess;
    int bcap = batch, cap = seq;
    if (e) {
        if (e->dev == dev) {
            bcap = e->bcap > bcap ? e->bcap : bcap;
            cap = e->cap > cap ? e->cap : cap;
        }
        mc_session_destroy(e->sess);
        memset(e, 0, sizeof(*e));
    } else {
        for (int i = 0; i < MAX_MODELS && !e; i++)
            if (!g_forward[i].key) e = &g_forward[i];
        if (!e) {
            e = &g_forward[0];
            mc_session_destroy(e->sess);
            memset(e, 0, sizeof(*e));
        }
    }
    mc_session* s = NULL;
    if (mc_session_create(dev, bcap, cap, &s) != MC_OK) {
        set_err("mc_session_create");
        return NULL;
    }
    e->key = model;
    e->sess = s;
    e->dev = dev;
    e->bcap = bcap;
    e->cap = cap;
    return s;
}

static void drop_forward_sessions_of(mc_model* dev) {
    for (int i = 0; i < MAX_MODELS; i++)
        if (g_forward[i].key && g_forward[i].dev == dev) {
            mc_session_destroy(g_forward[i].sess);
            memset(&g_forward[i], 0, sizeof(g_forward[i]));
        }
}

int minima_cuda_model_sync(const Model* model) {
    return model && model_validate(model) && device_model(model, 1) != NULL;
}

void minima_cuda_release_model(const Model* model) {
    for (int i = 0; i < MAX_MODELS; i++)
        if (g_models[i].key == model) {
            drop_sessions_of(g_models[i].dev);
            mc_model_destroy(g_models[i].dev);
            memset(&g_models[i], 0, sizeof(g_models[i]));
        }
}

void minima_cuda_release_cache(const KVCache* cache) {
    for (int i = 0; i < MAX_CACHES; i++)
        if (g_caches[i].key == cache) {
            mc_session_destroy(g_caches[i].sess);
            memset(&g_caches[i], 0, sizeof(g_caches[i]));
        }
}

/* ---------------------------------------------------------------- KV cache */

/* Size checks shared by every entry point; generate.c:14-22 with the
   envelope of this implementation. */
static bool model_shape_ok(const Model* model) {
    return model->n_layers > 0 && model->n_layers <= MC_MAX_LAYERS &&
        model->dim > 0 && model->dim <= MC_MAX_DIM &&
        model->ffn_dim > 0 && model->ffn_dim <= MC_MAX_FFN &&
        model->vocab_size > 0 && model->vocab_size <= MC_MAX_VOCAB &&
        model->n_heads > 0 && model->head_dim > 0 &&
        model->n_heads * model->head_dim == model->dim;
}

static bool cache_matches(const KVCache* cache, const Model* model) {
    return cache->n_layers == model->n_layers && cache->dim == model->dim &&
        cache->n_heads == model->n_heads && cache->n_kv_heads == model->n_kv_heads &&
        cache->head_dim == model->head_dim && cache->kv_dim == model->kv_dim &&
        cache->k_cache && cache->v_cache;
}

/* generate.c:13-47 */
bool kvcache_init(KVCache* cache, Arena* arena, const Model* model, int max_seq) {
    if (!cache || !arena || !model || !model_validate(model) || max_seq <= 0 ||
        max_seq > model->max_seq || max_seq > MC_MAX_SEQ || !model_shape_ok(model))
        return false;
    minima_cuda_release_cache(cache);
    memset(cache, 0, sizeof(*cache));
    cache->max_seq = max_seq;
    cache->n_layers = model->n_layers;
    cache->n_heads = model->n_heads;
    cache->n_kv_heads = model->n_kv_heads;
    cache->head_dim = model->head_dim;
    cache->dim = model->dim;
    cache->kv_dim = model->kv_dim;
    const size_t count = (size_t)model->n_layers * (size_t)max_seq * (size_t)model->kv_dim;
    if (count > SIZE_MAX / sizeof(float)) return false;
    const size_t bytes = count * sizeof(float);
    cache->k_cache = arena_alloc(arena, bytes);
    cache->v_cache = arena_alloc(arena, bytes);
    if (!cache->k_cache || !cache->v_cache) {
        memset(cache, 0, sizeof(*cache));
        return false;
    }
    cache->pos = 0;
    return true;
}

/* generate.c:49-51 */
void kvcache_reset(KVCache* cache) {
    if (cache) cache->pos = 0;
}

/* ------------------------------------------------------------- generation */

static bool options_ok(const GenerationOptions* o) {   /* generate.c:528-541 */
    return o->max_new_tokens >= 0 &&
        isfinite(o->temperature) && o->temperature > 0.0f &&
        isfinite(o->top_p) && o->top_p > 0.0f && o->top_p <= 1.0f &&
        isfinite(o->repetition_penalty) && o->repetition_penalty >= 1.0f &&
        isfinite(o->min_p) && o->min_p >= 0.0f && o->min_p <= 1.0f &&
        isfinite(o->frequency_penalty) && o->frequency_penalty >= -2.0f &&
        o->frequency_penalty <= 2.0f &&
        isfinite(o->presence_penalty) && o->presence_penalty >= -2.0f &&
        o->presence_penalty <= 2.0f &&
        o->no_repeat_ngram_size >= 0 && o->no_repeat_ngram_size <= 16 &&
        o->min_new_tokens >= 0 && o->min_new_tokens <= 512 &&
        o->min_new_tokens <= o->max_new_tokens &&
        o->stop_sequence_len >= 0 && o->stop_sequence_len <= 1024 &&
        !(o->stop_sequence_len > 0 && !o->stop_sequence_ids);
}

/*
 * Shared body of generate_with_options (generate.c:522-602) for `batch`
 * sequences.  Host-side checks run per sequence in the reference's order;
 * sequences with n_new <= 0 are answered on the host (generate.c:557-560)
 * and the others go to the device in one token loop.  Returns 1 if every
 * sequence was accepted.
 */
static int run_generate(Model* model, Tokenizer* tok, KVCache* caches, int batch,
    const uint16_t* prompts, int prompt_stride, const int* prompt_lens,
    uint16_t* out_ids, int out_cap, const GenerationOptions* options, Rng* rngs,
    int* out_counts) {
    for (int b = 0; b < batch; b++) out_counts[b] = 0;
    if (!model || !model_validate(model) || !tok || !caches || !prompts || !out_ids ||
        !options || !rngs || out_cap <= 0 || batch <= 0 || !options_ok(options) ||
        !model_shape_ok(model) || tok->vocab_size != model->vocab_size)
        return 0;
    int* active = (int*)malloc(sizeof(int) * (size_t)batch);
    int* lens = (int*)malloc(sizeof(int) * (size_t)batch);
    uint64_t* states = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)batch);
    int* counts = (int*)malloc(sizeof(int) * (size_t)batch);
    int* fpos = (int*)malloc(sizeof(int) * (size_t)batch);
    int n_active = 0, ok = active && lens && states && counts && fpos;
    for (int b = 0; ok && b < batch; b++) {
        const KVCache* cache = &caches[b];
        const int prompt_len = prompt_lens[b];
        const uint16_t* prompt = prompts + (size_t)b * prompt_stride;
        if (!cache_matches(cache, model) || cache->max_seq <= 0 ||
            cache->max_seq > MC_MAX_SEQ || prompt_len <= 0 || prompt_len > prompt_stride ||
            (b > 0 && cache->max_seq != caches[0].max_seq)) { ok = 0; break; }
        if (prompt_len > out_cap || prompt_len > cache->max_seq) { ok = 0; break; }
        int n_new = options->max_new_tokens;
        if (n_new > out_cap - prompt_len) n_new = out_cap - prompt_len;
        if (n_new > cache->max_seq - prompt_len) n_new = cache->max_seq - prompt_len;
        if (n_new <= 0) {
            memcpy(out_ids + (size_t)b * out_cap, prompt, (size_t)prompt_len * sizeof(uint16_t));
            out_counts[b] = prompt_len;
            continue;
        }
        for (int i = 0; i < prompt_len && ok; ++i)
            if (prompt[i] >= model->vocab_size || prompt[i] >= tok->vocab_size) ok = 0;
        for (int i = 0; i < options->stop_sequence_len && ok; ++i)
            if (options->stop_sequence_ids[i] >= model->vocab_size ||
                options->stop_sequence_ids[i] >= tok->vocab_size) ok = 0;
        if (ok) active[n_active++] = b;
    }
    if (ok && n_active > 0) {
        mc_model* dev = device_model(model, 0);
        mc_session* sess = dev ? device_session(&caches[active[0]], dev, n_active) : NULL;
        ok = sess != NULL;
        uint16_t* pbuf = NULL;
        uint16_t* obuf = NULL;
        const int contiguous = n_active == batch;
        if (ok && !contiguous) {
            pbuf = (uint16_t*)malloc((size_t)n_active * prompt_stride * sizeof(uint16_t));
            obuf = (uint16_t*)malloc((size_t)n_active * out_cap * sizeof(uint16_t));
            ok = pbuf && obuf;
        }
        if (ok) {
            for (int i = 0; i < n_active; i++) {
                const int b = active[i];
                lens[i] = prompt_lens[b];
                states[i] = rngs[b].state;
                kvcache_reset(&caches[b]);                     /* generate.c:573 */
                if (!contiguous)
                    memcpy(pbuf + (size_t)i * prompt_stride, prompts + (size_t)b * prompt_stride,
                        (size_t)prompt_lens[b] * sizeof(uint16_t));
            }
            const mc_status st = mc_generate(sess, n_active, contiguous ? prompts : pbuf,
                prompt_stride, lens, contiguous ? out_ids : obuf, out_cap,
                (const mc_sampling*)options, states, counts, fpos, 0u, NULL, 0);
            if (st != MC_OK) {
                set_err("mc_generate");
                ok = 0;
            } else {
                mc_last_kernel_ms(sess, &g_last_ms);
                for (int i = 0; i < n_active; i++) {
                    const int b = active[i];
                    if (!contiguous)
                        memcpy(out_ids + (size_t)b * out_cap, obuf + (size_t)i * out_cap,
                            (size_t)counts[i] * sizeof(uint16_t));
                    out_counts[b] = counts[i];
                    rngs[b].state = states[i];
                    caches[b].pos = fpos[i];
                }
            }
        }
        free(pbuf);
        free(obuf);
    }
    if (!ok)
        for (int b = 0; b < batch; b++) out_counts[b] = 0;
    free(active); free(lens); free(states); free(counts); free(fpos);
    return ok;
}

/* generate.c:522-602 */
int generate_with_options(Model* model, Tokenizer* tok, KVCache* cache,
    const uint16_t* prompt_ids, int prompt_len,
    uint16_t* out_ids, int out_cap,
    const GenerationOptions* options, Rng* rng) {
    if (!cache || !prompt_ids || prompt_len <= 0) return 0;
    int count = 0;
    const int len = prompt_len;
    run_generate(model, tok, cache, 1, prompt_ids, prompt_len, &len, out_ids, out_cap,
        options, rng, &count);
    return count;
}

/* generate.c:604-625 */
int generate_ex(Model* model, Tokenizer* tok, KVCache* cache,
    const uint16_t* prompt_ids, int prompt_len,
    uint16_t* out_ids, int out_cap, int n_new,
    float temperature, int top_k, float top_p,
    float repetition_penalty, Rng* rng) {
    GenerationOptions options;
    memset(&options, 0, sizeof(options));
    options.temperature = temperature;
    options.top_p = top_p;
    options.repetition_penalty = repetition_penalty;
    options.top_k = top_k;
    options.max_new_tokens = n_new;
    return generate_with_options(model, tok, cache, prompt_ids, prompt_len, out_ids, out_cap,
        &options, rng);
}

/* generate.c:627-633 */
int generate(Model* model, Tokenizer* tok, KVCache* cache,
    const uint16_t* prompt_ids, int prompt_len,
    uint16_t* out_ids, int out_cap, int n_new,
    float temperature, int top_k, Rng* rng) {
    return generate_ex(model, tok, cache, prompt_ids, prompt_len, out_ids, out_cap, n_new,
        temperature, top_k, 1.0f, 1.0f, rng);
}

int generate_batch_with_options(Model* model, Tokenizer* tok, KVCache* caches, int batch,
    const uint16_t* prompts, int prompt_stride, const int* prompt_lens,
    uint16_t* out_ids, int out_cap, const GenerationOptions* options, Rng* rngs,
    int* out_counts) {
    if (!out_counts || batch <= 0 || batch > MC_MAX_BATCH || !prompt_lens) return 0;
    return run_generate(model, tok, caches, batch, prompts, prompt_stride, prompt_lens,
        out_ids, out_cap, options, rngs, out_counts);
}

/* --------------------------------------------------------------- checking */

/* Per-prefix device logits for one sequence (forward_one per position). */
static float* device_prefix_logits(Model* model, KVCache* cache, const uint16_t* tokens, int n) {
    mc_model* dev = device_model(model, 0);
    mc_session* sess = dev ? device_session(cache, dev, 1) : NULL;
    if (!sess) return NULL;
    float* out = (float*)malloc((size_t)n * (size_t)model->vocab_size * sizeof(float));
    if (!out) return NULL;
    if (mc_forward_logits(sess, 1, tokens, n, out) != MC_OK) {
        set_err("mc_forward_logits");
        free(out);
        return NULL;
    }
    return out;
}

/* generate.c:202-265: the device token loop (forward_one per position)
   against the device batched causal forward (model_forward's arithmetic),
   with the full-forward logits kept in the caller's temp arena as the
   reference keeps its activations there. */
bool generation_check_kv_cache(Model* model, KVCache* cache, Arena* temp_arena,
    const uint16_t* tokens, int seq, float tolerance) {
    if (!model || !model_validate(model) || !cache || !temp_arena || !tokens || seq <= 0 ||
        seq > model->max_seq || seq > cache->max_seq || seq > MC_MAX_SEQ ||
        !isfinite(tolerance) || tolerance <= 0.0f || !model_shape_ok(model) ||
        !cache_matches(cache, model))
        return false;
    for (int i = 0; i < seq; i++)
        if (tokens[i] >= model->vocab_size) return false;
    arena_reset(temp_arena);
    float* full_logits = (float*)arena_alloc(temp_arena,
        (size_t)seq * (size_t)model->vocab_size * sizeof(float));
    if (!full_logits) return false;
    struct mc_session* fs = minima_cuda_forward_session(model, 1, seq);
    if (!fs) return false;
    if (mc_model_forward(fs, 1, seq, tokens, full_logits, 0u) != MC_OK) {
        set_err("mc_model_forward");
        return false;
    }
    kvcache_reset(cache);
    float* cached = device_prefix_logits(model, cache, tokens, seq);
    if (!cached) return false;
    float max_abs = 0.0f, max_rel = 0.0f;
    const size_t total = (size_t)seq * (size_t)model->vocab_size;
    for (size_t i = 0; i < total; i++) {
        const float diff = fabsf(full_logits[i] - cached[i]);
        const float denom = fmaxf(fabsf(full_logits[i]), 1e-6f);
        const float rel = diff / denom;
        if (diff > max_abs) max_abs = diff;
        if (rel > max_rel) max_rel = rel;
    }
    free(cached);
    cache->pos = seq;
    printf("KV-cache parity check\n");
    printf("  prefix positions: %d\n", seq);
    printf("  max abs error   : %.8e\n", max_abs);
    printf("  max rel error   : %.8e\n", max_rel);
    printf("  tolerance       : %.8e\n", tolerance);
    printf("  result          : %s\n", max_abs <= tolerance ? "PASS" : "FAIL");
    return max_abs <= tolerance;
}

/* The quoted, byte-safe form the reference prints for a token
   (generate.c:267-287): printable ASCII as is, backslash, double quote,
   newline, carriage return and tab as their C escapes, every other byte as
   \xHH with upper-case hex digits; an id outside the tokenizer prints as
   "<invalid>".  Formatted into a local buffer (flushed every 256 output
   bytes) and written to stdout with fwrite. */
static void write_quoted_token(const Tokenizer* tok, int id) {
    if (!tok || id < 0 || id >= tok->vocab_size) {
        fputs("\"<invalid>\"", stdout);
        return;
    }
    static const char kHex[] = "0123456789ABCDEF";
    const unsigned char* bytes = (const unsigned char*)tok->token_str[id];
    char buf[256 + 8];
    size_t n = 0;
    buf[n++] = '"';
    for (int i = 0; i < tok->token_len[id]; i++) {
        const unsigned char c = bytes[i];
        char esc = 0;
        switch (c) {
        case '\\': esc = '\\'; break;
        case '"': esc = '"'; break;
        case '\n': esc = 'n'; break;
        case '\r': esc = 'r'; break;
        case '\t': esc = 't'; break;
        default: break;
        }
        if (esc) {
            buf[n++] = '\\';
            buf[n++] = esc;
        } else if (c >= 0x20 && c < 0x7F) {
            buf[n++] = (char)c;
        } else {
            buf[n++] = '\\';
            buf[n++] = 'x';
            buf[n++] = kHex[c >> 4];
            buf[n++] = kHex[c & 15];
        }
        if (n >= 256) {
            fwrite(buf, 1, n, stdout);
            n = 0;
        }
    }
    buf[n++] = '"';
    fwrite(buf, 1, n, stdout);
}

/* generate.c:289-388.  The prompt runs through the device token loop
   teacher-forced, and the statistics of the last position's logits
   (maximum, softmax denominator and entropy in double precision, top-n by
   logit with ties to the lower id, cumulative masses) are computed on the
   device by mc_next_token_stats; this function validates like the
   reference and prints the same report. */
bool generation_inspect_next_tokens(Model* model, const Tokenizer* tok,
    KVCache* cache, const uint16_t* prompt_ids, int prompt_len, int top_n) {
    if (!model || !model_validate(model) || !tok || !cache || !prompt_ids || prompt_len <= 0 ||
        top_n <= 0 || !model_shape_ok(model) || tok->vocab_size != model->vocab_size ||
        prompt_len > model->max_seq || prompt_len > cache->max_seq ||
        !cache_matches(cache, model))
        return false;
    if (top_n > MC_STATS_MAX_TOP) top_n = MC_STATS_MAX_TOP;
    kvcache_reset(cache);
    /* the reference feeds ids until the first out-of-vocabulary one and
       leaves cache->pos at that index */
    for (int i = 0; i < prompt_len; i++)
        if (prompt_ids[i] >= model->vocab_size) {
            cache->pos = i;
            return false;
        }
    mc_model* dev = device_model(model, 0);
    mc_session* sess = dev ? device_session(cache, dev, 1) : NULL;
    if (!sess) return false;
    mc_token_stats st;
    if (mc_next_token_stats(sess, prompt_ids, prompt_len, top_n, &st) != MC_OK) {
        set_err("mc_next_token_stats");
        return false;
    }
    cache->pos = prompt_len;
    if (st.status != 0) return false;

    printf("  Next-token distribution (top %d, sampleable-vocabulary probabilities):\n",
        st.found);
    printf("    entropy=%.4f bits, top-1=%.2f%%, top-5=%.2f%%, top-10=%.2f%%\n",
        st.entropy_bits, st.top1_mass * 100.0, st.top5_mass * 100.0, st.top10_mass * 100.0);
    for (int rank = 0; rank < st.found; rank++) {
        printf("    %2d. id=%4d  p=%8.4f%%  token=", rank + 1, st.ids[rank],
            st.probability[rank] * 100.0);
        write_quoted_token(tok, st.ids[rank]);
        fputc('\n', stdout);
    }
    return true;
}
