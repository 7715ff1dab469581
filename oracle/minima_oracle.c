/*
 * minima_oracle.c — CPU restatement of Minima's decode path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker; never linked by the product).
 * Every function names the reference lines whose arithmetic it restates; the
 * floating-point operations run in the same order so that, compiled the same
 * way (gcc -O2, no FMA contraction), results are bit-identical to the
 * reference on every configuration the reference accepts.
 */
#include "minima_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <omp.h>

#define ORC_SPECIAL_COUNT 4      /* reserved ids 0..3 (tokenizer.h:14-18) */
#define ORC_MAX_VOCAB 65536
#define ORC_MAX_TOPK 256

struct OrcModel {
    int vocab, dim, n_layers, n_heads, n_kv_heads, head_dim, kv_dim, qkv_dim,
        ffn_dim, max_seq;
    float* block;
    float* t[9];
    size_t n[9];
};

/* ---------------- RNG: util.c:11-27 ---------------- */

uint64_t orc_rng_seed(uint64_t seed) { return seed ? seed : 0x123456789abcdef0ULL; }

uint64_t orc_rng_u64(uint64_t* s) {
    uint64_t x = *s;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *s = x;
    return x * 0x2545F4914F6CDD1DULL;
}

float orc_rng_f32(uint64_t* s) {
    return (orc_rng_u64(s) >> 40) * (1.0f / 16777216.0f);
}

int orc_rng_int(uint64_t* s, int lo, int hi) {
    if (lo >= hi) return lo;
    uint64_t range = (uint64_t)(hi - lo + 1);
    return lo + (int)(orc_rng_u64(s) % range);
}

/* ---------------- init: model.c:18-40, 95-167 ---------------- */

static float orc_randn(uint64_t* s) {
    float u1 = orc_rng_f32(s);
    float u2 = orc_rng_f32(s);
    if (u1 < 1e-7f) u1 = 1e-7f;
    return sqrtf(-2.0f * logf(u1)) * cosf(2.0f * 3.14159265f * u2);
}

static void orc_fill_normal(float* p, size_t n, float std, uint64_t* s) {
    for (size_t i = 0; i < n; i++) p[i] = orc_randn(s) * std;
}

int orc_kv_head_count(int n_heads) {
    if (n_heads <= 1) return 1;
    for (int kv = n_heads / 2; kv >= 1; kv--)
        if (n_heads % kv == 0) return kv;
    return 1;
}

static float orc_bf16_round(float v) {
    uint32_t u;
    memcpy(&u, &v, 4);
    if ((u & 0x7F800000u) == 0x7F800000u) return v;   /* inf / nan unchanged */
    u += 0x7FFFu + ((u >> 16) & 1u);
    u &= 0xFFFF0000u;
    memcpy(&v, &u, 4);
    return v;
}

OrcModel* orc_model_create(int vocab, int dim, int n_layers, int n_heads,
    int ffn_dim, int max_seq, uint64_t seed, int bf16_round) {
    if (vocab < ORC_SPECIAL_COUNT + 1 || vocab > ORC_MAX_VOCAB || dim <= 0 ||
        n_layers <= 0 || n_heads <= 0 || dim % n_heads != 0 ||
        dim / n_heads < 2 || ffn_dim <= 0 || max_seq <= 0)
        return NULL;
    OrcModel* m = (OrcModel*)calloc(1, sizeof(OrcModel));
    if (!m) return NULL;
    m->vocab = vocab; m->dim = dim; m->n_layers = n_layers; m->n_heads = n_heads;
    m->head_dim = dim / n_heads;
    m->n_kv_heads = orc_kv_head_count(n_heads);
    m->kv_dim = m->n_kv_heads * m->head_dim;
    m->qkv_dim = dim + 2 * m->kv_dim;
    m->ffn_dim = ffn_dim; m->max_seq = max_seq;
    const size_t L = (size_t)n_layers, D = (size_t)dim, F = (size_t)ffn_dim;
    m->n[0] = (size_t)vocab * D;
    m->n[1] = L * (size_t)m->qkv_dim * D;
    m->n[2] = L * D * D;
    m->n[3] = L * F * D;
    m->n[4] = L * F * D;
    m->n[5] = L * D * F;
    m->n[6] = L * D;
    m->n[7] = L * D;
    m->n[8] = D;
    size_t total = 0;
    for (int i = 0; i < 9; i++) total += m->n[i];
    m->block = (float*)malloc(total * sizeof(float));
    if (!m->block) { free(m); return NULL; }
    size_t off = 0;
    for (int i = 0; i < 9; i++) { m->t[i] = m->block + off; off += m->n[i]; }

    uint64_t s = orc_rng_seed(seed);
    orc_fill_normal(m->t[0], m->n[0], 0.02f, &s);
    const float std_main = 0.02f;
    const float std_res = 0.02f / sqrtf((float)n_layers);
    orc_fill_normal(m->t[1], m->n[1], std_main, &s);
    orc_fill_normal(m->t[2], m->n[2], std_res, &s);
    orc_fill_normal(m->t[3], m->n[3], std_main, &s);
    orc_fill_normal(m->t[4], m->n[4], std_main, &s);
    orc_fill_normal(m->t[5], m->n[5], std_res, &s);
    for (size_t i = 0; i < m->n[6]; i++) { m->t[6][i] = 1.0f; m->t[7][i] = 1.0f; }
    for (size_t i = 0; i < m->n[8]; i++) m->t[8][i] = 1.0f;
    if (bf16_round)
        for (int k = 0; k < 6; k++)
            for (size_t i = 0; i < m->n[k]; i++) m->t[k][i] = orc_bf16_round(m->t[k][i]);
    return m;
}

void orc_model_free(OrcModel* m) {
    if (!m) return;
    free(m->block);
    free(m);
}

float* orc_model_tensor(OrcModel* m, int which, size_t* count) {
    if (!m || which < 0 || which >= 9) return NULL;
    if (count) *count = m->n[which];
    return m->t[which];
}

void orc_model_dims(const OrcModel* m, int* d) {
    d[0] = m->vocab; d[1] = m->dim; d[2] = m->n_layers; d[3] = m->n_heads;
    d[4] = m->n_kv_heads; d[5] = m->head_dim; d[6] = m->kv_dim;
    d[7] = m->qkv_dim; d[8] = m->ffn_dim; d[9] = m->max_seq;
}

/* ---------------- single-token forward: generate.c:57-194 ---------------- */

typedef struct {
    int max_seq;
    int pos;
    float* k;       /* [L, max_seq, kv_dim] */
    float* v;
    float* x;       /* [dim] */
    float* x_norm;  /* [dim] */
    float* qkv;     /* [qkv_dim] */
    float* attn;    /* [dim] */
    float* proj;    /* [dim] */
    float* up;      /* [ffn] */
    float* gate;    /* [ffn] */
    float* scores;  /* [max_seq] */
    float* logits;  /* [vocab] */
} OrcState;

static int orc_state_init(OrcState* st, const OrcModel* m, int max_seq) {
    memset(st, 0, sizeof(*st));
    st->max_seq = max_seq;
    const size_t kv = (size_t)m->n_layers * (size_t)max_seq * (size_t)m->kv_dim;
    st->k = (float*)malloc(kv * sizeof(float));
    st->v = (float*)malloc(kv * sizeof(float));
    st->x = (float*)malloc((size_t)m->dim * sizeof(float));
    st->x_norm = (float*)malloc((size_t)m->dim * sizeof(float));
    st->qkv = (float*)malloc((size_t)m->qkv_dim * sizeof(float));
    st->attn = (float*)malloc((size_t)m->dim * sizeof(float));
    st->proj = (float*)malloc((size_t)m->dim * sizeof(float));
    st->up = (float*)malloc((size_t)m->ffn_dim * sizeof(float));
    st->gate = (float*)malloc((size_t)m->ffn_dim * sizeof(float));
    st->scores = (float*)malloc((size_t)max_seq * sizeof(float));
    st->logits = (float*)malloc((size_t)m->vocab * sizeof(float));
    return st->k && st->v && st->x && st->x_norm && st->qkv && st->attn &&
        st->proj && st->up && st->gate && st->scores && st->logits;
}

static void orc_state_free(OrcState* st) {
    free(st->k); free(st->v); free(st->x); free(st->x_norm); free(st->qkv);
    free(st->attn); free(st->proj); free(st->up); free(st->gate);
    free(st->scores); free(st->logits);
    memset(st, 0, sizeof(*st));
}

/* rmsnorm_inplace, generate.c:57-63 */
static void orc_rmsnorm_inplace(float* x, const float* scale, int dim, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < dim; i++) ss += x[i] * x[i];
    float inv = 1.0f / sqrtf(ss / dim + eps);
    for (int i = 0; i < dim; i++) x[i] = x[i] * inv * scale[i];
}

/* matvec, generate.c:65-73 */
static void orc_matvec(float* out, const float* x, const float* w, int d_in, int d_out) {
    for (int j = 0; j < d_out; j++) {
        float sum = 0.0f;
        const float* row = w + (size_t)j * d_in;
        for (int k = 0; k < d_in; k++) sum += x[k] * row[k];
        out[j] = sum;
    }
}

/* rotary_apply_qkv for one token, rotary.h:9-40 */
static void orc_rotary(float* qkv, int n_heads, int n_kv_heads, int head_dim, int pos) {
    const int pairs = head_dim / 2;
    for (int pair = 0; pair < pairs; pair++) {
        const float exponent = (2.0f * (float)pair) / (float)head_dim;
        const float angle = (float)pos * powf(10000.0f, -exponent);
        const float c = cosf(angle);
        const float s = sinf(angle);
        for (int h = 0; h < n_heads; h++) {
            float* x = qkv + h * head_dim + pair * 2;
            const float a = x[0], z = x[1];
            x[0] = a * c - z * s;
            x[1] = a * s + z * c;
        }
        for (int h = 0; h < n_kv_heads; h++) {
            float* x = qkv + n_heads * head_dim + h * head_dim + pair * 2;
            const float a = x[0], z = x[1];
            x[0] = a * c - z * s;
            x[1] = a * s + z * c;
        }
    }
}

/* forward_one, generate.c:76-194: leaves logits in st->logits, pos++ */
static void orc_forward_one(const OrcModel* m, OrcState* st, uint16_t token) {
    const int dim = m->dim, n_heads = m->n_heads, head_dim = m->head_dim;
    const int ffn = m->ffn_dim, kv_dim = m->kv_dim, pos = st->pos;
    const float* tok = m->t[0] + (size_t)token * dim;
    float* x = st->x;
    for (int d = 0; d < dim; d++) x[d] = tok[d];

    for (int layer = 0; layer < m->n_layers; layer++) {
        memcpy(st->x_norm, x, (size_t)dim * sizeof(float));
        orc_rmsnorm_inplace(st->x_norm, m->t[6] + (size_t)layer * dim, dim, 1e-5f);
        const float* w_qkv = m->t[1] + (size_t)layer * m->qkv_dim * dim;
        orc_matvec(st->qkv, st->x_norm, w_qkv, dim, m->qkv_dim);
        orc_rotary(st->qkv, n_heads, m->n_kv_heads, head_dim, pos);

        float* kl = st->k + (size_t)layer * st->max_seq * kv_dim;
        float* vl = st->v + (size_t)layer * st->max_seq * kv_dim;
        memcpy(kl + (size_t)pos * kv_dim, st->qkv + dim, (size_t)kv_dim * sizeof(float));
        memcpy(vl + (size_t)pos * kv_dim, st->qkv + dim + kv_dim,
            (size_t)kv_dim * sizeof(float));

        memset(st->attn, 0, (size_t)dim * sizeof(float));
        const float scale = 1.0f / sqrtf((float)head_dim);
        for (int h = 0; h < n_heads; h++) {
            const int kv_head = h / (n_heads / m->n_kv_heads);
            const float* q = st->qkv + h * head_dim;
            float* scores = st->scores;
            float max_score = -1e30f;
            for (int kj = 0; kj <= pos; kj++) {
                const float* k = kl + (size_t)kj * kv_dim + kv_head * head_dim;
                float dot = 0.0f;
                for (int d = 0; d < head_dim; d++) dot += q[d] * k[d];
                scores[kj] = dot * scale;
                if (scores[kj] > max_score) max_score = scores[kj];
            }
            float sum = 0.0f;
            for (int kj = 0; kj <= pos; kj++) {
                scores[kj] = expf(scores[kj] - max_score);
                sum += scores[kj];
            }
            float inv = 1.0f / sum;
            for (int kj = 0; kj <= pos; kj++) scores[kj] *= inv;
            float* out_h = st->attn + h * head_dim;
            for (int kj = 0; kj <= pos; kj++) {
                const float* v = vl + (size_t)kj * kv_dim + kv_head * head_dim;
                float s = scores[kj];
                for (int d = 0; d < head_dim; d++) out_h[d] += s * v[d];
            }
        }

        const float* w_proj = m->t[2] + (size_t)layer * dim * dim;
        orc_matvec(st->proj, st->attn, w_proj, dim, dim);
        for (int d = 0; d < dim; d++) x[d] += st->proj[d];

        memcpy(st->x_norm, x, (size_t)dim * sizeof(float));
        orc_rmsnorm_inplace(st->x_norm, m->t[7] + (size_t)layer * dim, dim, 1e-5f);
        const float* w_up = m->t[3] + (size_t)layer * ffn * dim;
        const float* w_gate = m->t[4] + (size_t)layer * ffn * dim;
        const float* w_down = m->t[5] + (size_t)layer * dim * ffn;
        orc_matvec(st->up, st->x_norm, w_up, dim, ffn);
        orc_matvec(st->gate, st->x_norm, w_gate, dim, ffn);
        for (int i = 0; i < ffn; i++) {
            float s = st->gate[i] / (1.0f + expf(-st->gate[i]));
            st->up[i] = s * st->up[i];
        }
        orc_matvec(st->proj, st->up, w_down, ffn, dim);
        for (int d = 0; d < dim; d++) x[d] += st->proj[d];
    }
    orc_rmsnorm_inplace(x, m->t[8], dim, 1e-5f);
    orc_matvec(st->logits, x, m->t[0], dim, m->vocab);
    st->pos++;
}

int orc_forward_prefixes(const OrcModel* m, const uint16_t* tokens, int n,
    float* logits_out) {
    if (!m || !tokens || n <= 0 || !logits_out) return 0;
    OrcState st;
    if (!orc_state_init(&st, m, n)) { orc_state_free(&st); return 0; }
    for (int i = 0; i < n; i++) {
        if (tokens[i] >= m->vocab) { orc_state_free(&st); return 0; }
        orc_forward_one(m, &st, tokens[i]);
        memcpy(logits_out + (size_t)i * m->vocab, st.logits, (size_t)m->vocab * sizeof(float));
    }
    orc_state_free(&st);
    return 1;
}

/* ---------------- sampler: generate.c:394-516 ---------------- */

static void orc_mark_repeated_ngrams(const uint16_t* history, int history_len,
    int ngram_size, uint8_t* banned, int vocab) {
    if (ngram_size <= 0 || !history || !banned || history_len <= 0) return;
    if (ngram_size == 1) {
        for (int i = 0; i < history_len; ++i)
            if (history[i] < (uint16_t)vocab) banned[history[i]] = 1;
        return;
    }
    const int prefix_len = ngram_size - 1;
    if (history_len < prefix_len) return;
    const int current_start = history_len - prefix_len;
    for (int start = 0; start + prefix_len < history_len; ++start) {
        if (memcmp(history + start, history + current_start,
                (size_t)prefix_len * sizeof(uint16_t)) == 0) {
            const uint16_t next = history[start + prefix_len];
            if (next < (uint16_t)vocab) banned[next] = 1;
        }
    }
}

static int orc_sample_impl(const float* logits, int vocab, float temperature,
    int top_k, float top_p, float repetition_penalty, float min_p,
    float frequency_penalty, float presence_penalty, int no_repeat_ngram_size,
    const uint16_t* history, int history_len, uint64_t* rng,
    uint8_t* seen, uint8_t* banned, uint16_t* counts) {
    int idx[ORC_MAX_TOPK];
    float vals[ORC_MAX_TOPK];
    int n = 0;
    memset(seen, 0, (size_t)vocab);
    memset(banned, 0, (size_t)vocab);
    memset(counts, 0, (size_t)vocab * sizeof(uint16_t));
    if (top_k < 1) top_k = 1;
    if (top_k > vocab) top_k = vocab;
    if (top_k > ORC_MAX_TOPK) top_k = ORC_MAX_TOPK;
    if (no_repeat_ngram_size > 0)
        orc_mark_repeated_ngrams(history, history_len, no_repeat_ngram_size, banned, vocab);
    if (repetition_penalty > 1.0f || frequency_penalty != 0.0f || presence_penalty != 0.0f) {
        for (int j = 0; j < history_len; ++j) {
            const uint16_t id = history[j];
            if (id >= (uint16_t)vocab) continue;
            seen[id] = 1;
            if (counts[id] < UINT16_MAX) ++counts[id];
        }
    }
    for (int id = 0; id < vocab; ++id) {
        float value = logits[id];
        if (seen[id] && repetition_penalty > 1.0f)
            value = value > 0.0f ? value / repetition_penalty : value * repetition_penalty;
        if (counts[id] > 0)
            value -= frequency_penalty * (float)counts[id] + presence_penalty;
        if (banned[id]) value = -INFINITY;
        value /= temperature;
        if (n < top_k) {
            idx[n] = id;
            vals[n] = value;
            ++n;
        } else {
            int min_i = 0;
            for (int j = 1; j < n; ++j)
                if (vals[j] < vals[min_i]) min_i = j;
            if (value > vals[min_i]) {
                idx[min_i] = id;
                vals[min_i] = value;
            }
        }
    }
    for (int i = 0; i < n; ++i) {
        for (int j = i + 1; j < n; ++j) {
            if (vals[j] > vals[i]) {
                float tv = vals[i]; vals[i] = vals[j]; vals[j] = tv;
                int ti = idx[i]; idx[i] = idx[j]; idx[j] = ti;
            }
        }
    }
    if (n == 0) return 0;
    if (!isfinite(vals[0])) {
        if (no_repeat_ngram_size > 0)
            return orc_sample_impl(logits, vocab, temperature, top_k, top_p,
                repetition_penalty, min_p, frequency_penalty, presence_penalty,
                0, history, history_len, rng, seen, banned, counts);
        return idx[0];
    }
    float maxv = vals[0], probs[ORC_MAX_TOPK], sum = 0.0f;
    for (int i = 0; i < n; ++i) {
        probs[i] = expf(vals[i] - maxv);
        sum += probs[i];
    }
    if (!(sum > 0.0f) || !isfinite(sum)) return idx[0];
    if (min_p > 0.0f) {
        const float min_probability = (probs[0] / sum) * min_p;
        int keep = 1;
        for (int i = 1; i < n; ++i) {
            if (probs[i] / sum < min_probability) break;
            ++keep;
        }
        n = keep;
        sum = 0.0f;
        for (int i = 0; i < n; ++i) sum += probs[i];
    }
    if (top_p < 1.0f) {
        float cumulative = 0.0f;
        int keep = 0;
        for (int i = 0; i < n; ++i) {
            cumulative += probs[i] / sum;
            ++keep;
            if (cumulative >= top_p) break;
        }
        n = keep;
    }
    sum = 0.0f;
    for (int i = 0; i < n; ++i) sum += probs[i];
    float draw = orc_rng_f32(rng) * sum;
    for (int i = 0; i < n; ++i) {
        draw -= probs[i];
        if (draw <= 0.0f) return idx[i];
    }
    return idx[n - 1];
}

int orc_sample(const float* logits, int vocab, const OrcOptions* o,
    const uint16_t* history, int history_len, uint64_t* rng_state) {
    if (!logits || vocab <= 0 || vocab > ORC_MAX_VOCAB || !o || !rng_state) return -1;
    uint8_t* seen = (uint8_t*)malloc((size_t)vocab);
    uint8_t* banned = (uint8_t*)malloc((size_t)vocab);
    uint16_t* counts = (uint16_t*)malloc((size_t)vocab * sizeof(uint16_t));
    int r = -1;
    if (seen && banned && counts)
        r = orc_sample_impl(logits, vocab, o->temperature, o->top_k, o->top_p,
            o->repetition_penalty, o->min_p, o->frequency_penalty,
            o->presence_penalty, o->no_repeat_ngram_size, history, history_len,
            rng_state, seen, banned, counts);
    free(seen); free(banned); free(counts);
    return r;
}

/* ---------------- generate loop: generate.c:522-602 ---------------- */

static int orc_options_valid(const OrcOptions* o) {
    return o && o->max_new_tokens >= 0 &&
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

int orc_generate(const OrcModel* m, const uint16_t* prompt, int prompt_len,
    uint16_t* out_ids, int out_cap, int cache_max_seq, const OrcOptions* o,
    uint64_t* rng_state, float* trace_logits, int trace_steps, int* final_pos) {
    if (final_pos) *final_pos = 0;
    if (!m || !prompt || !out_ids || !rng_state || prompt_len <= 0 || out_cap <= 0 ||
        cache_max_seq <= 0 || !orc_options_valid(o))
        return 0;
    if (prompt_len > out_cap || prompt_len > cache_max_seq) return 0;
    int n_new = o->max_new_tokens;
    if (n_new > out_cap - prompt_len) n_new = out_cap - prompt_len;
    if (n_new > cache_max_seq - prompt_len) n_new = cache_max_seq - prompt_len;
    if (n_new <= 0) {
        memcpy(out_ids, prompt, (size_t)prompt_len * sizeof(uint16_t));
        return prompt_len;
    }
    int top_k = o->top_k;
    if (top_k < 1) top_k = 1;
    if (top_k > m->vocab) top_k = m->vocab;
    if (top_k > ORC_MAX_TOPK) top_k = ORC_MAX_TOPK;
    for (int i = 0; i < prompt_len; ++i)
        if (prompt[i] >= m->vocab) return 0;
    for (int i = 0; i < o->stop_sequence_len; ++i)
        if (o->stop_sequence_ids[i] >= m->vocab) return 0;

    OrcState st;
    uint8_t* seen = (uint8_t*)malloc((size_t)m->vocab);
    uint8_t* banned = (uint8_t*)malloc((size_t)m->vocab);
    uint16_t* counts = (uint16_t*)malloc((size_t)m->vocab * sizeof(uint16_t));
    int ok = orc_state_init(&st, m, cache_max_seq) && seen && banned && counts;
    int result = 0;
    if (ok) {
        for (int i = 0; i < prompt_len; ++i) {
            out_ids[i] = prompt[i];
            orc_forward_one(m, &st, prompt[i]);
        }
        result = prompt_len + n_new;
        for (int i = 0; i < n_new; ++i) {
            for (int s = 0; s < ORC_SPECIAL_COUNT && s < m->vocab; ++s)
                st.logits[s] = -INFINITY;
            if (trace_logits && i < trace_steps)
                memcpy(trace_logits + (size_t)i * m->vocab, st.logits,
                    (size_t)m->vocab * sizeof(float));
            const int next = orc_sample_impl(st.logits, m->vocab, o->temperature,
                top_k, o->top_p, o->repetition_penalty, o->min_p,
                o->frequency_penalty, o->presence_penalty, o->no_repeat_ngram_size,
                out_ids, prompt_len + i, rng_state, seen, banned, counts);
            if (next < 0 || next >= m->vocab) { result = 0; break; }
            out_ids[prompt_len + i] = (uint16_t)next;
            const int generated = i + 1;
            if (o->stop_sequence_len > 0 && generated >= o->min_new_tokens &&
                generated >= o->stop_sequence_len) {
                const int stop_start = prompt_len + generated - o->stop_sequence_len;
                if (memcmp(out_ids + stop_start, o->stop_sequence_ids,
                        (size_t)o->stop_sequence_len * sizeof(uint16_t)) == 0) {
                    result = prompt_len + generated - o->stop_sequence_len;
                    break;
                }
            }
            orc_forward_one(m, &st, (uint16_t)next);
        }
        if (final_pos) *final_pos = st.pos;
    }
    orc_state_free(&st);
    free(seen); free(banned); free(counts);
    return result;
}

int orc_generate_batch(const OrcModel* m, int batch, const uint16_t* prompts,
    int prompt_stride, const int* prompt_lens, uint16_t* out_ids, int out_cap,
    int cache_max_seq, const OrcOptions* o, uint64_t* rng_states, int* counts,
    int nthreads) {
    if (!m || batch <= 0 || !prompts || !prompt_lens || !out_ids || !rng_states || !counts)
        return 0;
    int all_ok = 1;
    if (nthreads <= 0) nthreads = omp_get_max_threads();
    #pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads) reduction(&&:all_ok)
    for (int b = 0; b < batch; b++) {
        counts[b] = orc_generate(m, prompts + (size_t)b * prompt_stride, prompt_lens[b],
            out_ids + (size_t)b * out_cap, out_cap, cache_max_seq, o, &rng_states[b],
            NULL, 0, NULL);
        all_ok = all_ok && counts[b] > 0;
    }
    return all_ok;
}
