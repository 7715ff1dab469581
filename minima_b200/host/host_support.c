/*
 * host_support.c — the host functions generate.c relies on, for programs
 * that use the drop-in without the rest of Minima (bench.py, the tests).
 * Inside a Minima build the reference's model.c / arena.c / util.c provide
 * these symbols instead and this file is not linked.
 *
 * The seeded initialisation must reproduce the reference's weights bit for
 * bit (they are the parity fixture), so it follows model_init_config
 * (model.c:95-167), randn / fill_normal (model.c:18-30) and the xorshift64*
 * generator (util.c:11-33) step for step.  The size envelope is the one of
 * minima_cuda.h instead of config.h:7-14, so the larger Minima-architecture
 * decoders can be built; the reference's defaults are unchanged.  The arena
 * is a plain 64-byte-aligned bump allocator over one malloc'd block
 * (arena.h's contract without Win32 page commits or budgets).
 */
#include "minima_generate.h"
#include "minima_cuda.h"

#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define MIN_VOCAB 260        /* config.h:7 */
#define MIN_SEQ 32           /* config.h:13 */

/* ------------------------------------------------------------ util.c:11-33 */

void rng_seed(Rng* r, uint64_t seed) { r->state = seed ? seed : 0x123456789abcdef0ULL; }

uint64_t rng_u64(Rng* r) {
    uint64_t x = r->state;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    r->state = x;
    return x * 0x2545F4914F6CDD1DULL;
}

float rng_f32(Rng* r) { return (rng_u64(r) >> 40) * (1.0f / 16777216.0f); }

int rng_int(Rng* r, int lo, int hi) {
    if (lo >= hi) return lo;
    const uint64_t range = (uint64_t)(hi - lo + 1);
    return lo + (int)(rng_u64(r) % range);
}

void die(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vfprintf(stderr, fmt, ap);
    va_end(ap);
    fputc('\n', stderr);
    exit(1);
}

/* ------------------------------------------------------------------ arena */

bool arena_init_with_budget(Arena* a, size_t size, ArenaBudget* budget) {
    if (!a || size == 0) return false;
    memset(a, 0, sizeof(*a));
    a->base = (uint8_t*)aligned_alloc(64, (size + 63) & ~(size_t)63);
    if (!a->base) return false;
    a->size = size;
    a->committed = size;
    a->page_size = 4096;
    a->budget = budget;
    return true;
}

bool arena_init(Arena* a, size_t size) { return arena_init_with_budget(a, size, NULL); }

void arena_free(Arena* a) {
    if (!a || !a->base) return;
    free(a->base);
    memset(a, 0, sizeof(*a));
}

void* arena_alloc(Arena* a, size_t n) {
    if (!a || !a->base || n == 0) return NULL;
    const size_t align = 64;
    if (a->used > SIZE_MAX - (align - 1)) return NULL;
    const size_t offset = (a->used + (align - 1)) & ~(align - 1);
    if (offset > a->size || n > a->size - offset) return NULL;
    a->used = offset + n;
    if (a->used > a->peak) a->peak = a->used;
    return a->base + offset;
}

void* arena_alloc_zero(Arena* a, size_t n) {
    void* p = arena_alloc(a, n);
    if (p) memset(p, 0, n);
    return p;
}

void arena_reset(Arena* a) {
    if (a) a->used = 0;
}

size_t arena_remaining(const Arena* a) {
    if (!a || a->used > a->size) return 0;
    return a->size - a->used;
}

/* ---------------------------------------------------------- model.c:18-167 */

static float randn(Rng* rng) {
    float u1 = rng_f32(rng);
    float u2 = rng_f32(rng);
    if (u1 < 1e-7f) u1 = 1e-7f;
    return sqrtf(-2.0f * logf(u1)) * cosf(2.0f * 3.14159265f * u2);
}

static void fill_normal(float* p, size_t n, float std, Rng* rng) {
    for (size_t i = 0; i < n; i++) p[i] = randn(rng) * std;
}

static int kv_head_count(int n_heads) {
    if (n_heads <= 1) return 1;
    for (int kv = n_heads / 2; kv >= 1; kv--)
        if (n_heads % kv == 0) return kv;
    return 1;
}

bool model_config_validate(const ModelConfig* c) {
    return c && c->vocab_size >= MIN_VOCAB && c->vocab_size <= MC_MAX_VOCAB &&
        c->dim > 0 && c->dim <= MC_MAX_DIM &&
        c->n_layers > 0 && c->n_layers <= MC_MAX_LAYERS &&
        c->n_heads > 0 && c->n_heads <= MC_MAX_HEADS &&
        c->dim % c->n_heads == 0 && c->dim / c->n_heads >= 2 &&
        c->dim / c->n_heads <= MC_MAX_HEAD_DIM &&
        c->ffn_dim > 0 && c->ffn_dim <= MC_MAX_FFN &&
        c->max_seq >= MIN_SEQ && c->max_seq <= MC_MAX_SEQ;
}

static size_t param_total(const Model* m) {
    const size_t D = (size_t)m->dim, L = (size_t)m->n_layers, F = (size_t)m->ffn_dim;
    return (size_t)m->vocab_size * D + L * (size_t)m->qkv_dim * D + L * D * D +
        L * F * D * 2 + L * D * F + L * D * 2 + D;
}

bool model_validate(const Model* m) {
    if (!m) return false;
    const ModelConfig c = {m->vocab_size, m->dim, m->n_layers, m->n_heads, m->ffn_dim, m->max_seq};
    if (!model_config_validate(&c) || m->head_dim != m->dim / m->n_heads || !m->tok_emb ||
        !m->attn_qkv || !m->attn_proj || !m->ffn_up || !m->ffn_gate || !m->ffn_down ||
        !m->rms1_scale || !m->rms2_scale || !m->rms_final_scale)
        return false;
    const int kv = kv_head_count(m->n_heads);
    if (m->n_kv_heads != kv || m->kv_dim != kv * m->head_dim ||
        m->qkv_dim != m->dim + 2 * m->kv_dim)
        return false;
    return m->weight_bytes == param_total(m) * sizeof(float);
}

size_t model_param_count(const Model* m) { return m->weight_bytes / sizeof(float); }

bool model_init_config(Model* m, Arena* arena, uint64_t seed, const ModelConfig* c) {
    if (!m || !arena || !model_config_validate(c)) return false;
    memset(m, 0, sizeof(*m));
    m->memory_budget = arena->budget;
    m->vocab_size = c->vocab_size;
    m->dim = c->dim;
    m->n_layers = c->n_layers;
    m->n_heads = c->n_heads;
    m->head_dim = c->dim / c->n_heads;
    m->n_kv_heads = kv_head_count(c->n_heads);
    m->kv_dim = m->n_kv_heads * m->head_dim;
    m->qkv_dim = m->dim + 2 * m->kv_dim;
    m->ffn_dim = c->ffn_dim;
    m->max_seq = c->max_seq;
    const size_t D = (size_t)m->dim, L = (size_t)m->n_layers, F = (size_t)m->ffn_dim;
    const size_t n_emb = (size_t)m->vocab_size * D, n_qkv = L * (size_t)m->qkv_dim * D;
    const size_t n_proj = L * D * D, n_up = L * F * D, n_down = L * D * F, n_rms = L * D;
    m->tok_emb = (float*)arena_alloc(arena, n_emb * 4);
    m->attn_qkv = (float*)arena_alloc(arena, n_qkv * 4);
    m->attn_proj = (float*)arena_alloc(arena, n_proj * 4);
    m->ffn_up = (float*)arena_alloc(arena, n_up * 4);
    m->ffn_gate = (float*)arena_alloc(arena, n_up * 4);
    m->ffn_down = (float*)arena_alloc(arena, n_down * 4);
    m->rms1_scale = (float*)arena_alloc(arena, n_rms * 4);
    m->rms2_scale = (float*)arena_alloc(arena, n_rms * 4);
    m->rms_final_scale = (float*)arena_alloc(arena, D * 4);
    if (!m->tok_emb || !m->attn_qkv || !m->attn_proj || !m->ffn_up || !m->ffn_gate ||
        !m->ffn_down || !m->rms1_scale || !m->rms2_scale || !m->rms_final_scale)
        die("model weight allocation failed - increase arena size");
    Rng rng;
    rng_seed(&rng, seed);
    fill_normal(m->tok_emb, n_emb, 0.02f, &rng);
    const float std_main = 0.02f;
    const float std_res = 0.02f / sqrtf((float)m->n_layers);
    fill_normal(m->attn_qkv, n_qkv, std_main, &rng);
    fill_normal(m->attn_proj, n_proj, std_res, &rng);
    fill_normal(m->ffn_up, n_up, std_main, &rng);
    fill_normal(m->ffn_gate, n_up, std_main, &rng);
    fill_normal(m->ffn_down, n_down, std_res, &rng);
    for (size_t i = 0; i < n_rms; i++) { m->rms1_scale[i] = 1.0f; m->rms2_scale[i] = 1.0f; }
    for (size_t i = 0; i < D; i++) m->rms_final_scale[i] = 1.0f;
    m->weight_bytes = param_total(m) * sizeof(float);
    return true;
}

bool model_init(Model* m, Arena* arena, uint64_t seed, int vocab_size) {
    ModelConfig c = {30000, 128, 8, 4, 512, 128};   /* config.h:17-22 */
    c.vocab_size = vocab_size;
    return model_init_config(m, arena, seed, &c);
}

/* Bytes an arena needs for model_init_config(c): weights plus alignment. */
size_t minima_host_model_arena_bytes(const ModelConfig* c) {
    if (!c) return 0;
    const size_t D = (size_t)c->dim, L = (size_t)c->n_layers, F = (size_t)c->ffn_dim;
    const size_t hd = c->n_heads > 0 ? D / (size_t)c->n_heads : 0;
    const size_t Q = D + 2 * (size_t)kv_head_count(c->n_heads) * hd;
    const size_t floats = (size_t)c->vocab_size * D + L * Q * D + L * D * D + 3 * L * F * D +
        2 * L * D + D;
    return floats * 4 + 16 * 64;
}

/* Round every matrix of `m` to bfloat16 (round-to-nearest-even) in place,
   the weight format of the bf16 decoder configurations. */
void minima_host_round_bf16(Model* m) {
    const size_t D = (size_t)m->dim, L = (size_t)m->n_layers, F = (size_t)m->ffn_dim;
    float* t[6] = {m->tok_emb, m->attn_qkv, m->attn_proj, m->ffn_up, m->ffn_gate, m->ffn_down};
    const size_t n[6] = {(size_t)m->vocab_size * D, L * (size_t)m->qkv_dim * D, L * D * D,
        L * F * D, L * F * D, L * D * F};
    for (int k = 0; k < 6; k++)
        for (size_t i = 0; i < n[k]; i++) {
            uint32_t u;
            memcpy(&u, &t[k][i], 4);
            if ((u & 0x7F800000u) != 0x7F800000u) {
                u += 0x7FFFu + ((u >> 16) & 1u);
                u &= 0xFFFF0000u;
                memcpy(&t[k][i], &u, 4);
            }
        }
}
