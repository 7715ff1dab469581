/*
 * forward_cuda.c — drop-in replacement for the Minima reference's forward.c
 * (forward.h:43-57): the batched causal forward runs on a B200 through
 * minima_cuda.h.  Declared in include/minima_forward.h.
 *
 * Host-side dependencies are those forward.c has on the rest of the
 * program: model_validate (model.c:55-89) and arena_alloc (arena.c:127-177),
 * from Minima's own files or from libminima_host.so.  The device state
 * (uploaded weights, one forward session per model) lives in the side
 * tables of libminima_generate.so.
 */
#include "minima_forward.h"
#include "minima_cuda.h"

#include <limits.h>
#include <math.h>
#include <stdio.h>
#include <string.h>

bool model_validate(const Model* model);
void* arena_alloc(Arena* a, size_t n);

/* forward.c:124-170: the forward caches and the backward workspace, from
   the caller's arena, in the reference's order (callers locate buffers by
   their place in the arena, e.g. the attention scratch at the end). */
bool activations_init(Activations* act, Arena* temp_arena, int batch, int seq, const Model* model) {
    if (!act || !temp_arena || batch <= 0 || seq <= 0 || batch > INT_MAX / seq ||
        !model_validate(model) || seq > model->max_seq)
        return false;
    memset(act, 0, sizeof(*act));
    const size_t n = (size_t)batch * (size_t)seq, L = (size_t)model->n_layers;
    const size_t D = (size_t)model->dim, F = (size_t)model->ffn_dim, Q = (size_t)model->qkv_dim;
    const size_t V = (size_t)model->vocab_size, f = sizeof(float);
    struct {
        float** dst;
        size_t floats;
    } plan[] = {
        {&act->x, n * D}, {&act->x_norm, n * D},
        {&act->qkv, L * n * Q}, {&act->attn_out, L * n * D}, {&act->ffn_buf, L * n * F},
        {&act->up_buf, L * n * F}, {&act->gate_buf, L * n * F}, {&act->resid_attn, L * n * D},
        {&act->resid_ffn, L * n * D},
        {&act->logits, n * V},
        {&act->dx, n * D}, {&act->dx_tmp, n * D}, {&act->dx_norm, n * D}, {&act->dattn, n * D},
        {&act->dqkv, n * Q}, {&act->dffn, n * F}, {&act->dup, n * F}, {&act->dgate, n * F},
        {&act->attention_scores, (size_t)seq},
    };
    bool ok = true;
    for (size_t i = 0; i < sizeof(plan) / sizeof(plan[0]); i++) {
        *plan[i].dst = (float*)arena_alloc(temp_arena, plan[i].floats * f);
        ok = ok && *plan[i].dst != NULL;
    }
    return ok;
}

/* forward.c:13-22 */
void rmsnorm(float* out, const float* x, const float* scale, int dim, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < dim; i++) ss += x[i] * x[i];
    const float inv = 1.0f / sqrtf(ss / (float)dim + eps);
    for (int i = 0; i < dim; i++) out[i] = x[i] * inv * scale[i];
}

/* forward.c:58-60 */
float silu(float x) { return x / (1.0f + expf(-x)); }

/* forward.c:24-40 on the device.  The reference has no error path here; a
   device failure is reported on stderr and leaves `out` unwritten. */
void matmul(float* out, const float* x, const float* w, int n, int d_in, int d_out) {
    if (n <= 0 || d_out <= 0) return;
    if (mc_matmul(out, x, w, n, d_in, d_out) != MC_OK)
        fprintf(stderr, "minima_cuda matmul: %s\n", mc_last_error());
}

/* forward.c:176-274 */
float* model_forward(Model* model, Activations* act, const uint16_t* tokens, int batch, int seq) {
    if (!model_validate(model) || !act || !tokens || batch <= 0 || seq <= 0 ||
        batch > INT_MAX / seq || seq > model->max_seq || !act->x || !act->x_norm || !act->qkv ||
        !act->attn_out || !act->up_buf || !act->gate_buf || !act->ffn_buf || !act->resid_attn ||
        !act->resid_ffn || !act->logits || !act->attention_scores)
        return NULL;
    const size_t n = (size_t)batch * (size_t)seq;
    for (size_t i = 0; i < n; i++)
        if (tokens[i] >= model->vocab_size) return NULL;
    struct mc_session* s = minima_cuda_forward_session(model, batch, seq);
    if (!s) return NULL;
    const mc_forward_caches caches = {
        act->x, act->x_norm, act->qkv, act->attn_out, act->ffn_buf, act->up_buf, act->gate_buf,
        act->resid_attn, act->resid_ffn, act->logits,
    };
    if (mc_model_forward_caches(s, batch, seq, tokens, &caches) != MC_OK) {
        fprintf(stderr, "minima_cuda model_forward: %s\n", mc_last_error());
        return NULL;
    }
    return act->logits;
}
