/*
 * minima_oracle.h — CPU restatement of Minima's decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the checker that the CUDA path is
 * compared against; the product never links or calls it.  It restates, in
 * the same floating-point operation order, the reference's
 *   model_init_config / randn / fill_normal   (model.c:95-167, 18-30)
 *   forward_one / rmsnorm_inplace / matvec    (generate.c:57-194)
 *   rotary_apply_qkv                          (rotary.h:9-40)
 *   sample_top_k_top_p / mark_repeated_ngrams (generate.c:394-516)
 *   generate_with_options                     (generate.c:522-602)
 *   xorshift64* rng_seed/rng_u64/rng_f32      (util.c:11-27)
 * with the reference's size envelope (config.h:7-14, generate.c:14-22) lifted
 * so that the larger Minima-architecture decoders can be checked too.  It is
 * pinned bit-for-bit against the reference itself (oracle/_ref, built from
 * the reference's unmodified sources) on configurations the reference
 * accepts; see tests/test_oracle.py.
 */
#ifndef MINIMA_ORACLE_H
#define MINIMA_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same field order and types as the reference's GenerationOptions
   (generate.h:50-63), so one ctypes structure serves both. */
typedef struct {
    float temperature;
    float top_p;
    float repetition_penalty;
    float min_p;
    float frequency_penalty;
    float presence_penalty;
    int top_k;
    int max_new_tokens;
    int min_new_tokens;
    int no_repeat_ngram_size;
    const uint16_t* stop_sequence_ids;
    int stop_sequence_len;
} OrcOptions;

typedef struct OrcModel OrcModel;

/* Seeded initialisation identical to model_init_config (model.c:95-167).
   bf16_round != 0 rounds every matrix and the embedding to bfloat16
   (round-to-nearest-even) after initialisation; the stored values stay
   fp32 so the arithmetic below is unchanged.  Returns NULL on bad dims. */
OrcModel* orc_model_create(int vocab, int dim, int n_layers, int n_heads,
    int ffn_dim, int max_seq, uint64_t seed, int bf16_round);
void orc_model_free(OrcModel* m);

/* Tensor access in the reference's MODEL_ARRAYS order: 0 tok_emb, 1 attn_qkv,
   2 attn_proj, 3 ffn_up, 4 ffn_gate, 5 ffn_down, 6 rms1, 7 rms2, 8 rms_final. */
float* orc_model_tensor(OrcModel* m, int which, size_t* count);
/* dims[0..9] = vocab, dim, layers, heads, kv_heads, head_dim, kv_dim,
   qkv_dim, ffn_dim, max_seq */
void orc_model_dims(const OrcModel* m, int* dims);
int orc_kv_head_count(int n_heads);

/* Per-prefix logits: logits_out[i*V .. (i+1)*V) are the logits after
   feeding tokens[0..i] one at a time (forward_one semantics). */
int orc_forward_prefixes(const OrcModel* m, const uint16_t* tokens, int n,
    float* logits_out);

/* Sampler, teacher-forced: same logits, history and RNG state in, same id
   out.  logits are used as given (no reserved-id masking here). */
int orc_sample(const float* logits, int vocab, const OrcOptions* o,
    const uint16_t* history, int history_len, uint64_t* rng_state);

/* generate_with_options for one sequence.  out_ids receives prompt +
   generated ids; returns the count (0 on invalid input).  If trace_logits
   is non-NULL, the masked logits the sampler saw at decode step i are
   stored at trace_logits[i*V] for i < trace_steps.  *final_pos receives the
   KV position the reference leaves in cache->pos. */
int orc_generate(const OrcModel* m, const uint16_t* prompt, int prompt_len,
    uint16_t* out_ids, int out_cap, int cache_max_seq, const OrcOptions* o,
    uint64_t* rng_state, float* trace_logits, int trace_steps, int* final_pos);

/* Independent sequences in parallel (OpenMP, nthreads <= 0: all cores).
   prompts[b*prompt_stride ..], prompt_lens[b], out_ids[b*out_cap ..],
   rng_states[b], counts[b].  Returns 1 when every sequence succeeded. */
int orc_generate_batch(const OrcModel* m, int batch, const uint16_t* prompts,
    int prompt_stride, const int* prompt_lens, uint16_t* out_ids, int out_cap,
    int cache_max_seq, const OrcOptions* o, uint64_t* rng_states, int* counts,
    int nthreads);

uint64_t orc_rng_seed(uint64_t seed);
uint64_t orc_rng_u64(uint64_t* state);
float orc_rng_f32(uint64_t* state);
int orc_rng_int(uint64_t* state, int lo, int hi);

#ifdef __cplusplus
}
#endif
#endif
