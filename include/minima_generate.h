/*
 * minima_generate.h — the drop-in generation API, served by the B200 path.
 *
 * libminima_generate.so exports exactly the functions of the reference's
 * generate.h (generate.h:26-76) with identical C signatures, argument
 * meaning and error behaviour (0 / false on any invalid argument, no
 * exceptions, no exit), so a Minima build links it in place of generate.c.
 * Each declaration below names the reference line it replaces.
 *
 * Inside a Minima source tree define MINIMA_REFERENCE_HEADERS so that the
 * reference's own headers provide the types; standalone, the types are
 * restated below field for field (same order, same C types), because the
 * drop-in must accept the caller's structs as they are laid out there.
 *
 * Differences from generate.c, all on the permissive side:
 *  - the size envelope is minima_cuda.h's MC_MAX_* instead of config.h:7-14
 *    and the 512/1024 stack-buffer limits of generate.c:14-22, 542-550;
 *  - the KV cache lives on the device; KVCache.k_cache/v_cache are still
 *    allocated from the caller's arena (generate.c:38-39) so that callers
 *    that test them keep working, but they are not written;
 *  - the forward of the last sampled id, whose logits are never read
 *    (generate.c:599 on the final iteration), is not run; cache->pos is
 *    still left where the reference leaves it.
 */
#ifndef MINIMA_GENERATE_H
#define MINIMA_GENERATE_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef MINIMA_REFERENCE_HEADERS
#include "generate.h"
#include "forward.h"
#else

/* config.h:25-32 */
typedef struct {
    int vocab_size;
    int dim;
    int n_layers;
    int n_heads;
    int ffn_dim;
    int max_seq;
} ModelConfig;

/* arena.h:8-15 */
typedef struct {
    size_t limit;
    size_t committed;
    size_t external_committed;
    size_t peak;
    size_t failed;
    volatile long lock;
} ArenaBudget;

/* arena.h:17-25 */
typedef struct {
    uint8_t* base;
    size_t size;
    size_t used;
    size_t peak;
    size_t committed;
    size_t page_size;
    ArenaBudget* budget;
} Arena;

/* model.h:9-41 */
typedef struct {
    int vocab_size;
    int dim;
    int n_layers;
    int n_heads;
    int n_kv_heads;
    int head_dim;
    int kv_dim;
    int qkv_dim;
    int ffn_dim;
    int max_seq;
    float* tok_emb;
    float* attn_qkv;
    float* attn_proj;
    float* ffn_up;
    float* ffn_gate;
    float* ffn_down;
    float* rms1_scale;
    float* rms2_scale;
    float* rms_final_scale;
    size_t weight_bytes;
    ArenaBudget* memory_budget;
} Model;

/* util.h:10-12 */
typedef struct {
    uint64_t state;
} Rng;

/* tokenizer.h:9-41 (generation reads vocab_size, token_str, token_len) */
#define MINIMA_TOK_MAX_VOCAB 32768
typedef struct {
    uint16_t left;
    uint16_t right;
} Merge;
typedef struct {
    int vocab_size;
    int n_merges;
    ArenaBudget* memory_budget;
    char* token_str[MINIMA_TOK_MAX_VOCAB];
    int token_len[MINIMA_TOK_MAX_VOCAB];
    Merge merges[MINIMA_TOK_MAX_VOCAB - 260];
    void* merge_rank_index;
    uint32_t merge_rank_capacity;
} Tokenizer;

/* generate.h:11-24 */
typedef struct {
    int max_seq;
    int n_layers;
    int n_heads;
    int n_kv_heads;
    int head_dim;
    int dim;
    int kv_dim;
    float* k_cache;
    float* v_cache;
    int pos;
} KVCache;

/* forward.h:10-39 (passed to the host program's model_forward) */
typedef struct {
    float* x;
    float* x_norm;
    float* qkv;
    float* attn_out;
    float* ffn_buf;
    float* up_buf;
    float* gate_buf;
    float* resid_attn;
    float* resid_ffn;
    float* logits;
    float* dx;
    float* dx_tmp;
    float* dx_norm;
    float* dattn;
    float* dqkv;
    float* dffn;
    float* dup;
    float* dgate;
    float* attention_scores;
} Activations;

/* generate.h:50-63 */
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
} GenerationOptions;

#ifdef __cplusplus
extern "C" {
#endif

/* generate.h:26 */
bool kvcache_init(KVCache* cache, Arena* arena, const Model* model, int max_seq);
/* generate.h:27 */
void kvcache_reset(KVCache* cache);
/* generate.h:31-32 (needs the host program's model_forward, forward.h:56) */
bool generation_check_kv_cache(Model* model, KVCache* cache, Arena* temp_arena,
    const uint16_t* tokens, int seq, float tolerance);
/* generate.h:34-35 */
bool generation_inspect_next_tokens(Model* model, const Tokenizer* tok,
    KVCache* cache, const uint16_t* prompt_ids, int prompt_len, int top_n);
/* generate.h:43-48 */
int generate(Model* model, Tokenizer* tok, KVCache* cache,
    const uint16_t* prompt_ids, int prompt_len,
    uint16_t* out_ids, int out_cap,
    int n_new,
    float temperature, int top_k,
    Rng* rng);
/* generate.h:65-68 */
int generate_with_options(Model* model, Tokenizer* tok, KVCache* cache,
    const uint16_t* prompt_ids, int prompt_len,
    uint16_t* out_ids, int out_cap,
    const GenerationOptions* options, Rng* rng);
/* generate.h:70-74 */
int generate_ex(Model* model, Tokenizer* tok, KVCache* cache,
    const uint16_t* prompt_ids, int prompt_len,
    uint16_t* out_ids, int out_cap, int n_new,
    float temperature, int top_k, float top_p,
    float repetition_penalty, Rng* rng);

#ifdef __cplusplus
}
#endif
#endif /* MINIMA_REFERENCE_HEADERS */

#ifdef __cplusplus
extern "C" {
#endif

/*
 * Extensions (no counterpart in the reference, which decodes one sequence
 * per call).  generate_batch_with_options runs `batch` independent
 * generate_with_options calls in one device token loop: caches[b] and
 * rngs[b] belong to sequence b (each cache from kvcache_init with the same
 * max_seq), prompt b is prompts[b*prompt_stride .. + prompt_lens[b]),
 * output b goes to out_ids[b*out_cap ..], and out_counts[b] receives what
 * generate_with_options would have returned for it.  Returns 1 when every
 * sequence was accepted, 0 otherwise (out_counts then all 0).
 */
int generate_batch_with_options(Model* model, Tokenizer* tok, KVCache* caches, int batch,
    const uint16_t* prompts, int prompt_stride, const int* prompt_lens,
    uint16_t* out_ids, int out_cap, const GenerationOptions* options, Rng* rngs,
    int* out_counts);

/* Select the CUDA device the drop-in uses in this process (default: the
   MINIMA_CUDA_DEVICE environment variable, else 0).  Returns 0 on failure. */
int minima_cuda_select_device(int device);

/* Re-upload the weights of `model` to the device before the next call
   (after the caller modified them in place).  Returns 0 on failure. */
int minima_cuda_model_sync(const Model* model);

/* Release the device state held for `model` / `cache`. */
void minima_cuda_release_model(const Model* model);
void minima_cuda_release_cache(const KVCache* cache);

/* Text of the last device-side failure (empty if none). */
const char* minima_cuda_last_error(void);

/* Device kernel time of the last generation call, milliseconds. */
float minima_cuda_last_kernel_ms(void);

/* The device session the drop-in model_forward (minima_forward.h) runs a
   batch x seq forward of `model` on: one per model, grown as needed, with
   the weights re-uploaded when they changed (the same side table as the
   generation entry points).  NULL on failure (minima_cuda_last_error). */
struct mc_session* minima_cuda_forward_session(const Model* model, int batch, int seq);

#ifdef __cplusplus
}
#endif
#endif
