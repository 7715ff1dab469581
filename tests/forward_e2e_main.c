/*
 * forward_e2e_main.c — model_forward followed by Minima's own
 * model_backward (backward.c), with every array written to a file, so that
 * the same program linked over the reference's forward.c
 * (oracle/_ref/forward_e2e_ref) and over the drop-in libminima_forward.so
 * (oracle/_ref/forward_e2e_cuda) can be compared array by array
 * (tests/test_gpu_forward.py).  TEST INFRASTRUCTURE ONLY.
 *
 * usage: forward_e2e OUT vocab dim layers heads ffn max_seq batch seq seed
 * OUT receives, for each array in order, a uint64 count and that many
 * floats: x, x_norm, qkv, attn_out, ffn_buf, up_buf, gate_buf, resid_attn,
 * resid_ffn, logits, then the nine gradient arrays in MODEL_ARRAYS order.
 */
#include "backward.h"
#include "forward.h"
#include "model.h"
#include "util.h"

#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

static void put(FILE* f, const float* p, size_t n) {
    const uint64_t c = n;
    fwrite(&c, sizeof(c), 1, f);
    fwrite(p, sizeof(float), n, f);
}

int main(int argc, char** argv) {
    if (argc != 11) {
        fprintf(stderr, "usage: %s OUT vocab dim layers heads ffn max_seq batch seq seed\n", argv[0]);
        return 2;
    }
    const ModelConfig cfg = {atoi(argv[2]), atoi(argv[3]), atoi(argv[4]), atoi(argv[5]),
                             atoi(argv[6]), atoi(argv[7])};
    const int batch = atoi(argv[8]), seq = atoi(argv[9]);
    const uint64_t seed = strtoull(argv[10], NULL, 10);
    Arena model_arena, grad_arena, temp_arena;
    if (!arena_init(&model_arena, 64u << 20) || !arena_init(&grad_arena, 64u << 20) ||
        !arena_init(&temp_arena, 512u << 20))
        return 3;
    Model model;
    Gradients grads;
    if (!model_init_config(&model, &model_arena, seed, &cfg) ||
        !gradients_init(&grads, &grad_arena, &model))
        return 4;
    const size_t n = (size_t)batch * seq;
    uint16_t* tokens = (uint16_t*)malloc(n * sizeof(uint16_t));
    float* dlogits = (float*)malloc(n * (size_t)cfg.vocab_size * sizeof(float));
    if (!tokens || !dlogits) return 5;
    Rng r;
    rng_seed(&r, seed + 1000);
    for (size_t i = 0; i < n; i++) tokens[i] = (uint16_t)rng_int(&r, 4, cfg.vocab_size - 1);
    for (size_t i = 0; i < n * (size_t)cfg.vocab_size; i++)
        dlogits[i] = (float)((int)(i % 13u) - 6) * 1.0e-3f;

    Activations act;
    if (!activations_init(&act, &temp_arena, batch, seq, &model)) return 6;
    if (!model_forward(&model, &act, tokens, batch, seq)) {
        fprintf(stderr, "model_forward failed\n");
        return 7;
    }
    FILE* f = fopen(argv[1], "wb");
    if (!f) return 8;
    const size_t L = (size_t)model.n_layers, D = (size_t)model.dim, F = (size_t)model.ffn_dim;
    const size_t Q = (size_t)model.qkv_dim, V = (size_t)model.vocab_size;
    put(f, act.x, n * D);
    put(f, act.x_norm, n * D);
    put(f, act.qkv, L * n * Q);
    put(f, act.attn_out, L * n * D);
    put(f, act.ffn_buf, L * n * F);
    put(f, act.up_buf, L * n * F);
    put(f, act.gate_buf, L * n * F);
    put(f, act.resid_attn, L * n * D);
    put(f, act.resid_ffn, L * n * D);
    put(f, act.logits, n * V);
    gradients_zero(&grads, &model);
    model_backward(&model, &grads, &act, dlogits, tokens, batch, seq);
    put(f, grads.tok_emb, V * D);
    put(f, grads.attn_qkv, L * Q * D);
    put(f, grads.attn_proj, L * D * D);
    put(f, grads.ffn_up, L * F * D);
    put(f, grads.ffn_gate, L * F * D);
    put(f, grads.ffn_down, L * D * F);
    put(f, grads.rms1_scale, L * D);
    put(f, grads.rms2_scale, L * D);
    put(f, grads.rms_final_scale, D);
    fclose(f);
    printf("forward_e2e: ok\n");
    return 0;
}
