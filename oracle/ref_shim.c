/*
 * ref_shim.c — flat C entry points over the Minima reference's own API, so
 * that Python tests can drive the reference through ctypes.  TEST
 * INFRASTRUCTURE ONLY: compiled against the reference headers and linked
 * with the reference's unmodified objects into oracle/_ref/libminima_ref.so.
 *
 * Every call goes through the reference's public functions:
 * model_init_config (model.h:45), kvcache_init (generate.h:26),
 * generate_with_options (generate.h:65), activations_init/model_forward
 * (forward.h:43-57), generation_check_kv_cache (generate.h:31),
 * optim_init_type (optim.h:62) and checkpoint_save / checkpoint_load
 * (checkpoint.h:10-24).
 */
#include "generate.h"
#include "forward.h"
#include "checkpoint.h"
#include "optim.h"

#include <stdlib.h>
#include <string.h>

typedef struct {
    Arena arena;
    Model model;
} RefModel;

static Tokenizer g_tok;   /* generate() reads only vocab_size (generate.c:550) */

/* The reference arena commits whole pages inside its reservation
   (arena.c:137-141), so reservations are rounded up to whole pages. */
static size_t pages(size_t bytes) { return (bytes + 2 * 65536 - 1) / 65536 * 65536; }

void* refsh_model_create(int vocab, int dim, int layers, int heads, int ffn,
    int max_seq, uint64_t seed) {
    RefModel* h = (RefModel*)calloc(1, sizeof(RefModel));
    if (!h) return NULL;
    const ModelConfig cfg = { vocab, dim, layers, heads, ffn, max_seq };
    if (!model_config_validate(&cfg)) { free(h); return NULL; }
    /* upper bound on the weights (qkv_dim <= 3*dim) plus alignment slack */
    const size_t bytes = ((size_t)vocab * dim + (size_t)layers * 3 * (size_t)dim * dim +
        (size_t)layers * dim * dim + 3 * (size_t)layers * ffn * dim +
        2 * (size_t)layers * dim + dim) * sizeof(float) + 16 * 64;
    if (!arena_init(&h->arena, pages(bytes))) { free(h); return NULL; }
    if (!model_init_config(&h->model, &h->arena, seed, &cfg)) {
        arena_free(&h->arena);
        free(h);
        return NULL;
    }
    return h;
}

void refsh_model_free(void* p) {
    RefModel* h = (RefModel*)p;
    if (!h) return;
    arena_free(&h->arena);
    free(h);
}

float* refsh_tensor(void* p, int which, size_t* count) {
    RefModel* h = (RefModel*)p;
    Model* m = &h->model;
    const size_t D = (size_t)m->dim, L = (size_t)m->n_layers, F = (size_t)m->ffn_dim;
    switch (which) {
    case 0: *count = (size_t)m->vocab_size * D; return m->tok_emb;
    case 1: *count = L * (size_t)m->qkv_dim * D; return m->attn_qkv;
    case 2: *count = L * D * D; return m->attn_proj;
    case 3: *count = L * F * D; return m->ffn_up;
    case 4: *count = L * F * D; return m->ffn_gate;
    case 5: *count = L * D * F; return m->ffn_down;
    case 6: *count = L * D; return m->rms1_scale;
    case 7: *count = L * D; return m->rms2_scale;
    case 8: *count = D; return m->rms_final_scale;
    default: *count = 0; return NULL;
    }
}

size_t refsh_param_count(void* p) {
    return model_param_count(&((RefModel*)p)->model);
}

int refsh_generate(void* p, const uint16_t* prompt, int prompt_len,
    uint16_t* out_ids, int out_cap, int cache_max_seq,
    const GenerationOptions* o, uint64_t* rng_state, int* final_pos) {
    RefModel* h = (RefModel*)p;
    Arena cache_arena;
    const size_t kv_bytes = (size_t)h->model.n_layers * (size_t)cache_max_seq *
        (size_t)h->model.kv_dim * sizeof(float);
    if (!arena_init(&cache_arena, pages(2 * kv_bytes + 256))) return 0;
    KVCache cache;
    int r = 0;
    if (kvcache_init(&cache, &cache_arena, &h->model, cache_max_seq)) {
        g_tok.vocab_size = h->model.vocab_size;
        Rng rng = { *rng_state };
        r = generate_with_options(&h->model, &g_tok, &cache, prompt, prompt_len,
            out_ids, out_cap, o, &rng);
        *rng_state = rng.state;
        if (final_pos) *final_pos = cache.pos;
    }
    arena_free(&cache_arena);
    return r;
}

/* logits_out: [seq, vocab], position i = logits after tokens[0..i]. */
int refsh_forward_logits(void* p, const uint16_t* tokens, int seq, float* logits_out) {
    RefModel* h = (RefModel*)p;
    Model* m = &h->model;
    const size_t n = (size_t)seq, D = (size_t)m->dim, F = (size_t)m->ffn_dim;
    const size_t L = (size_t)m->n_layers, V = (size_t)m->vocab_size;
    const size_t floats = n * D * 2 + L * n * ((size_t)m->qkv_dim + 4 * D + 3 * F) +
        n * V + n * (5 * D + (size_t)m->qkv_dim + 3 * F) + n;
    Arena temp;
    if (!arena_init(&temp, pages(floats * sizeof(float) + 64 * 64))) return 0;
    Activations act;
    int ok = 0;
    if (activations_init(&act, &temp, 1, seq, m)) {
        float* logits = model_forward(m, &act, tokens, 1, seq);
        if (logits) {
            memcpy(logits_out, logits, n * V * sizeof(float));
            ok = 1;
        }
    }
    arena_free(&temp);
    return ok;
}

int refsh_check_kv_cache(void* p, const uint16_t* tokens, int seq, float tol) {
    RefModel* h = (RefModel*)p;
    Model* m = &h->model;
    const size_t n = (size_t)seq, D = (size_t)m->dim, F = (size_t)m->ffn_dim;
    const size_t L = (size_t)m->n_layers, V = (size_t)m->vocab_size;
    const size_t floats = n * D * 2 + L * n * ((size_t)m->qkv_dim + 4 * D + 3 * F) +
        n * V + n * (5 * D + (size_t)m->qkv_dim + 3 * F) + n;
    Arena temp, cache_arena;
    if (!arena_init(&temp, pages(floats * sizeof(float) + 64 * 64))) return 0;
    if (!arena_init(&cache_arena, pages(2 * L * n * (size_t)m->kv_dim * sizeof(float) + 256))) {
        arena_free(&temp);
        return 0;
    }
    KVCache cache;
    int ok = kvcache_init(&cache, &cache_arena, m, seq) &&
        generation_check_kv_cache(m, &cache, &temp, tokens, seq, tol);
    arena_free(&cache_arena);
    arena_free(&temp);
    return ok;
}

/* A freshly initialised optimizer (optim_init_type, optim.h:62) of `type`
   in its own arena, with a valid schedule and every moment set to `fill`. */
static int shim_optim(Arena* a, Optim* opt, const Model* m, int type, int64_t step,
    int64_t total_steps, float fill) {
    const size_t n = model_param_count(m);
    if (!arena_init(a, pages(2 * n * sizeof(float) + 32 * 64))) return 0;
    if (!optim_init_type(opt, m, a, (OptimizerType)type, 1e-3f, 0.9f, 0.95f, 1e-8f, 0.1f)) {
        arena_free(a);
        return 0;
    }
    opt->step = step;
    opt->schedule_base_lr = 1e-3f;
    opt->schedule_total_steps = total_steps;
    opt->schedule_warmup_steps = 0;
    opt->schedule_type = 0;
    float* moments[18] = {
        opt->m_tok_emb, opt->m_attn_qkv, opt->m_attn_proj, opt->m_ffn_up, opt->m_ffn_gate,
        opt->m_ffn_down, opt->m_rms1_scale, opt->m_rms2_scale, opt->m_rms_final_scale,
        opt->v_tok_emb, opt->v_attn_qkv, opt->v_attn_proj, opt->v_ffn_up, opt->v_ffn_gate,
        opt->v_ffn_down, opt->v_rms1_scale, opt->v_rms2_scale, opt->v_rms_final_scale };
    const size_t D = (size_t)m->dim, L = (size_t)m->n_layers, F = (size_t)m->ffn_dim;
    const size_t counts[9] = { (size_t)m->vocab_size * D, L * (size_t)m->qkv_dim * D, L * D * D,
        L * F * D, L * F * D, L * D * F, L * D, L * D, D };
    for (int k = 0; k < 18; k++)
        if (moments[k])
            for (size_t i = 0; i < counts[k % 9]; i++) moments[k][i] = fill;
    return 1;
}

/* checkpoint_save of this model with an optimizer of `type` (0 AdamW,
   1 Lion) at global step `step` of `total_steps`, RNG state and tokenizer
   fingerprint as given. */
int refsh_checkpoint_save(void* p, const char* path, int type, int64_t step, int64_t total_steps,
    uint64_t rng_state, uint64_t tokenizer_hash, float moment_fill) {
    RefModel* h = (RefModel*)p;
    Arena a;
    Optim opt;
    if (!shim_optim(&a, &opt, &h->model, type, step, total_steps, moment_fill)) return 0;
    Rng rng = { rng_state };
    const int ok = checkpoint_save(path, &h->model, &opt, &rng, tokenizer_hash) ? 1 : 0;
    arena_free(&a);
    return ok;
}

/* checkpoint_load into this model and a fresh optimizer of `type`; the
   RNG state and step it restores are returned. */
int refsh_checkpoint_load(void* p, const char* path, int type, uint64_t tokenizer_hash,
    uint64_t* rng_out, int64_t* step_out) {
    RefModel* h = (RefModel*)p;
    Arena a;
    Optim opt;
    if (!shim_optim(&a, &opt, &h->model, type, 0, 1, 0.0f)) return 0;
    Rng rng = { 1 };
    const int ok = checkpoint_load(path, &h->model, &opt, &rng, tokenizer_hash) ? 1 : 0;
    if (ok) {
        *rng_out = rng.state;
        *step_out = opt.step;
    }
    arena_free(&a);
    return ok;
}
