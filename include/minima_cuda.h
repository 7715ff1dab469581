/*
 * minima_cuda.h — C ABI of the B200 (sm_100a) decode path for Minima.
 *
 * Plain C: opaque handles, host pointers and sizes, integer status codes; no
 * CUDA, C++ or PyTorch types cross this boundary.  The drop-in
 * implementation of the reference's generate.h (minima_b200/host/
 * generate_cuda.c) is the intended caller; tests and bench.py call it too.
 *
 * Reference interfaces this boundary stands under:
 *   mc_model_create      <- the weights a Model holds (model.h:9-41, filled by
 *                           model_init_config, model.c:95-167)
 *   mc_session_create    <- kvcache_init (generate.h:26; generate.c:13-47)
 *   mc_generate          <- generate_with_options (generate.h:65-68;
 *                           generate.c:522-602), for a batch of independent
 *                           sequences, each with its own Rng (util.h:10-12)
 *   mc_forward_logits    <- forward_one per prefix (generate.c:76-194), the
 *                           quantity generation_check_kv_cache compares
 *                           (generate.c:202-265)
 *
 * Error convention: every entry point returns MC_OK (0) or a positive
 * status; mc_last_error() gives a one-line description of the last failure
 * on the calling thread.  No entry point aborts the process.
 *
 * Threading: one host thread per device; handles are not thread-safe.
 */
#ifndef MINIMA_CUDA_H
#define MINIMA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int mc_status;
#define MC_OK              0
#define MC_ERR_INVALID     1   /* argument outside the supported envelope   */
#define MC_ERR_CUDA        2   /* a CUDA runtime call failed                */
#define MC_ERR_NOMEM       3   /* device or pinned-host allocation failed   */
#define MC_ERR_TIMEOUT     4   /* a device-side wait ran past its deadline  */
#define MC_ERR_DEVICE      5   /* the kernel reported an inconsistency      */
#define MC_ERR_UNSUPPORTED 6   /* no kernel for this shape / device         */

#define MC_WEIGHTS_F32  0      /* fp32 weights, fp32 arithmetic              */
#define MC_WEIGHTS_BF16 1      /* bf16 weights (RNE from fp32), fp32 math    */

/* mc_generate flags */
#define MC_DEVICE_POINTERS 0x1u /* prompts/out_ids/rng/counts/final_pos are
                                   device pointers (resident in HBM)       */

typedef struct mc_model mc_model;
typedef struct mc_session mc_session;

/* Dimensions plus host pointers to the nine fp32 weight arrays in the
   reference's layout and MODEL_ARRAYS order (checkpoint.c:43-52):
   tok_emb [V,D]; attn_qkv [L,Q,D] (Q heads, then K heads, then V heads);
   attn_proj [L,D,D]; ffn_up, ffn_gate [L,F,D]; ffn_down [L,D,F];
   rms1_scale, rms2_scale [L,D]; rms_final_scale [D]. */
typedef struct {
    int vocab_size, dim, n_layers, n_heads, n_kv_heads, head_dim, kv_dim,
        qkv_dim, ffn_dim, max_seq;
    const float* tok_emb;
    const float* attn_qkv;
    const float* attn_proj;
    const float* ffn_up;
    const float* ffn_gate;
    const float* ffn_down;
    const float* rms1_scale;
    const float* rms2_scale;
    const float* rms_final_scale;
} mc_model_desc;

/* Field-for-field the reference's GenerationOptions (generate.h:50-63), so a
   GenerationOptions* may be passed where an mc_sampling* is expected. */
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
} mc_sampling;

/* Envelope of this implementation (the reference's is config.h:7-14). */
#define MC_MAX_VOCAB     32768
#define MC_MAX_DIM       4096
#define MC_MAX_LAYERS    64
#define MC_MAX_HEADS     64
#define MC_MAX_HEAD_DIM  256
#define MC_MAX_FFN       16384
#define MC_MAX_SEQ       8192
#define MC_MAX_BATCH     1024
#define MC_MAX_TOPK      256     /* generate.c:564 */
#define MC_MAX_STOP      1024    /* generate.c:540 */

/* Select the CUDA device for the calling thread (cudaSetDevice). */
mc_status mc_init(int device);

/* Upload weights (host fp32) to the current device as fp32 or bf16.
   Dimensions are validated against the envelope above and against the
   reference's derived-size rules (model.c:55-89). */
mc_status mc_model_create(const mc_model_desc* desc, int weight_dtype, mc_model** out);
/* Re-upload weights of identical dimensions (after the caller edited them). */
mc_status mc_model_update(mc_model* model, const mc_model_desc* desc);
mc_status mc_model_destroy(mc_model* model);

/* Device KV cache and work buffers for up to max_batch sequences of up to
   max_seq tokens each (max_seq <= the model's max_seq). */
mc_status mc_session_create(mc_model* model, int max_batch, int max_seq,
    mc_session** out);

/*
 * A session whose KV cache is paged: a pool of n_pages pages, each holding
 * page_len consecutive positions of one sequence for every layer and KV
 * head (page_len a power of two >= MC_MIN_PAGE_LEN), and a per-sequence
 * page table.  The reference's KVCache (generate.h:11-24; kvcache_init,
 * generate.c:13-47) reserves max_seq positions per sequence; here each
 * mc_generate call gives every sequence ceil((prompt + new ids - 1) /
 * page_len) pages (mc_forward_logits / mc_model_forward: the positions
 * they feed), so a batch of mixed lengths needs only the pages it fills.
 * A call whose sequences need more pages than the pool holds returns
 * MC_ERR_NOMEM.  mc_session_create is the same with an identity table of
 * max_batch * ceil(max_seq / MC_MIN_PAGE_LEN) pages.
 */
#define MC_MIN_PAGE_LEN 64
mc_status mc_session_create_paged(mc_model* model, int max_batch, int max_seq, int page_len,
    int n_pages, mc_session** out);
mc_status mc_session_destroy(mc_session* session);

/*
 * Run generate_with_options for `batch` independent sequences in one
 * device-resident token loop (no host round trip per token).
 *   prompts      [batch * prompt_stride] u16; sequence b is
 *                prompts[b*prompt_stride .. + prompt_lens[b])
 *   prompt_lens  [batch] host ints, 1 <= len <= out_cap, len <= max_seq
 *   out_ids      [batch * out_cap] u16: prompt followed by generated ids
 *   opts         validated as generate.c:526-551 does
 *   rng_states   [batch] xorshift64* states, advanced exactly as the
 *                reference advances its Rng
 *   out_counts   [batch] ints: what generate_with_options would return
 *   final_pos    [batch] ints (optional): the KV position the reference
 *                leaves in cache->pos
 * With MC_DEVICE_POINTERS, prompts/out_ids/rng_states/out_counts/final_pos
 * are device pointers and no host<->device copy is made; prompt_lens and
 * opts stay on the host either way.
 * trace_logits (optional, host, [batch][trace_steps][vocab]) receives the
 * masked logits the sampler saw at each of the first trace_steps steps.
 */
mc_status mc_generate(mc_session* session, int batch,
    const uint16_t* prompts, int prompt_stride, const int* prompt_lens,
    uint16_t* out_ids, int out_cap, const mc_sampling* opts,
    uint64_t* rng_states, int* out_counts, int* final_pos, unsigned flags,
    float* trace_logits, int trace_steps);

/* Teacher-forced logits: feed tokens[b*n .. b*n+n) one position at a time
   and store the logits after each position into logits_out[(b*n+i)*V]
   (host).  Equals forward_one per prefix (generate.c:76-194). */
mc_status mc_forward_logits(mc_session* session, int batch, const uint16_t* tokens,
    int n, float* logits_out);

/*
 * Next-token distribution after a prompt, computed on the device: the
 * statistics generation_inspect_next_tokens prints (generate.c:291-388).
 * tokens[0..n) are fed one position at a time (forward_one per prefix,
 * generate.c:76-194); over the last position's logits with the reserved
 * ids 0..3 excluded, the device computes the maximum, the softmax
 * denominator and the entropy in bits (double precision) and the top_n
 * (1..MC_STATS_MAX_TOP) ids by logit, ties to the lower id, with their
 * probabilities and the cumulative top-1/5/10 masses.  The session's KV
 * cache is overwritten.  out->status is 0, or 1 when a sampleable logit is
 * not finite, or 2 when the denominator is not positive and finite (the
 * reference's rejections); the call itself returns MC_OK in those cases.
 */
#define MC_STATS_MAX_TOP 20
typedef struct {
    int status;
    int found;                               /* ids filled: min(top_n, vocab - 4) */
    int ids[MC_STATS_MAX_TOP];
    float logits[MC_STATS_MAX_TOP];
    double probability[MC_STATS_MAX_TOP];
    double max_logit, denominator, entropy_bits;
    double top1_mass, top5_mass, top10_mass;  /* 0 where fewer ids were found */
} mc_token_stats;
mc_status mc_next_token_stats(mc_session* session, const uint16_t* tokens, int n, int top_n,
    mc_token_stats* out);

/* Batched causal forward of tokens[b*seq .. b*seq+seq) at every position —
   the logits of model_forward (forward.c:176-274), equal to forward_one per
   prefix (generate.c:76-194) within fp32 rounding: logits_out[(b*seq+t)*V].
   Runs the prefill kernels plus the final norm and tied lm_head (tcgen05
   GEMMs with MINIMA_CUDA_PREFILL=tcgen05 and fp32 weights); the session's KV
   cache is overwritten.  Token ids >= vocab are rejected (MC_ERR_INVALID) as
   forward.c:179-186 rejects them.  With MC_DEVICE_POINTERS, tokens and
   logits_out are device pointers. */
mc_status mc_model_forward(mc_session* session, int batch, int seq, const uint16_t* tokens,
    float* logits_out, unsigned flags);

/*
 * model_forward (forward.c:176-274) with its caches: the batched causal
 * forward of mc_model_forward on the fp32 CUDA-core GEMMs, also storing
 * every per-layer activation that Minima's model_backward reads
 * (backward.c:440-600), into host arrays laid out as the reference's
 * Activations (forward.h:10-26): per-layer arrays [n_layers][batch*seq][w]
 * with row b*seq + t, final arrays [batch*seq][w].  A NULL pointer is not
 * written.  qkv holds Q and K after RoPE and V as projected
 * (forward.c:224-227); x and x_norm are the final residual stream and the
 * final RMSNorm output; logits [batch*seq][vocab].
 */
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
} mc_forward_caches;
mc_status mc_model_forward_caches(mc_session* session, int batch, int seq, const uint16_t* tokens,
    const mc_forward_caches* out);

/* matmul of forward.h:49-50 (forward.c:24-40) on the device of the calling
   thread: out[n][d_out] = x[n][d_in] . w[d_out][d_in]^T, fp32, k ascending
   per output (FMA accumulation).  Host pointers; the operands are copied in
   and the result out on every call. */
mc_status mc_matmul(float* out, const float* x, const float* w, int n, int d_in, int d_out);

/* Kernel time of the last mc_generate / mc_forward_logits on this session,
   measured with CUDA events on the launching stream (milliseconds). */
mc_status mc_last_kernel_ms(mc_session* session, float* ms);

/* Prompt positions the last mc_generate ran as one batched prefill (all
   sequences' positions [0, shortest prompt - 1), no logits computed for
   them) and its device time in milliseconds (included in
   mc_last_kernel_ms).  The token loop starts at that position. */
mc_status mc_last_prefill(mc_session* session, int* positions, float* ms);

/* Number of kernels the last call launched on the device. */
mc_status mc_last_launch_count(mc_session* session, int* launches);

/* Device timestamps (%globaltimer, ns) taken at the start of every token
   step of the last call, plus one at loop exit: ns[0..*n).  The difference
   of consecutive stamps is the per-token latency of that step.  Sequences
   are in prefill while t < prompt length. */
mc_status mc_last_step_times(mc_session* session, unsigned long long* ns, int cap, int* n);

/* Name of the kernel the last call ran: "mc::token_loop_kernel" (grid-barrier
   loop) or "mc::cluster_loop_kernel" (cluster-resident greedy loop). */
const char* mc_last_kernel_name(mc_session* session);

/* Layer loop of this session's cluster-resident plan: -1 none (the
   grid-barrier loop serves every call), 0 five phases per layer, 1 two
   phases closed by cluster barriers, 2 two phases whose partials move by
   bulk copies onto the receivers' mbarriers.  MINIMA_CUDA_LOOP=grid,
   cluster1 or cluster2 (read at mc_session_create) caps the choice. */
mc_status mc_session_cluster_variant(mc_session* session, int* variant);

/* The CUDA stream (cudaStream_t) every call on this session is issued on,
   so that callers can time or order their own work against it. */
mc_status mc_session_stream(mc_session* session, void** stream);

/*
 * mc_generate_static — mc_generate that allocates nothing.  No counterpart
 * in the reference (whose decode runs on the host stack).
 *
 * For callers that cannot call cudaMalloc: real-time hosts that must not
 * take its cost (or the device-wide wait of a later cudaFree) mid-session,
 * hosts that carve their device memory up front from their own pool,
 * plugins that must not grow the device footprint after start-up.  The caller passes device buffers for everything it owns:
 *   w            dims plus DEVICE pointers to the nine fp32 weight arrays
 *                (layout as in mc_model_desc)
 *   prompts, out_ids, rng_states, out_counts   device pointers, as with
 *                MC_DEVICE_POINTERS in mc_generate
 *   prompt_lens, opts   host memory
 *   max_seq      KV-cache capacity per sequence (<= w->max_seq)
 *   stream       cudaStream_t to run on (NULL: the legacy default stream);
 *                the call returns after that stream has finished it
 * The KV cache and all work buffers come from one static __device__ array
 * of MC_STATIC_SCRATCH_BYTES that every GPU loading this library holds
 * until the process exits; a model/batch/max_seq that needs more (the
 * reference's default 5.8M model fits at batch 4 and max_seq 512) is
 * rejected with MC_ERR_INVALID, as are batch > MC_STATIC_MAX_BATCH and
 * max_seq * head_dim/2 > MC_STATIC_MAX_ROPE; a shape whose shared-memory
 * plan exceeds the device's per-block limit returns MC_ERR_UNSUPPORTED.
 * It runs the grid-barrier token loop from position 0 (no batched
 * prefill), so its ids equal mc_generate's within the token loop's fp32
 * numerics (identical wherever no step is a near-tie).  The device-side
 * waits honour MINIMA_CUDA_WAIT_NS / MINIMA_CUDA_TEST_STALL as the other
 * loops do and end in MC_ERR_TIMEOUT.
 *
 * Every call looks up the array's device address and sets the kernel's
 * shared-memory limit (nothing cached goes stale across a device reset);
 * the first call on a device also loads the kernel: make it before any
 * stream capture.  Calls share the array (its contents persist between
 * calls; what must start at zero is cleared by each call), so calls that
 * overlap on the GPU race.  The host-side staging (sequence table, RoPE
 * table) is process-global too: not thread-safe.
 */
#define MC_STATIC_SCRATCH_BYTES (16u << 20)
#define MC_STATIC_MAX_BATCH     64
#define MC_STATIC_MAX_ROPE      (1 << 17)
mc_status mc_generate_static(const mc_model_desc* w, int batch,
    const uint16_t* prompts, int prompt_stride, const int* prompt_lens,
    uint16_t* out_ids, int out_cap, const mc_sampling* opts,
    uint64_t* rng_states, int* out_counts, int max_seq, void* stream);

/*
 * Checkpoints — the reference's on-disk format (checkpoint.c:154-234):
 * "MINIMA04" / "MINIMA05", a 112-byte header (v5: 116, the optimizer type
 * appended), the nine model arrays in MODEL_ARRAYS order (checkpoint.c:43-52),
 * then the optimizer moments (m, and v for AdamW, per array), all fp32
 * little-endian, nothing after them.
 *
 * mc_checkpoint_inspect    <- the header and length checks of checkpoint_load
 *                             (checkpoint.c:301-400); reads no array, touches
 *                             no device.  Fills *info when it returns MC_OK.
 * mc_model_load_checkpoint <- checkpoint_load's model half, straight to the
 *                             device: the file streams through pinned staging
 *                             buffers into the model's device arrays (bf16
 *                             RNE on the device when weights_dtype is
 *                             MC_WEIGHTS_BF16); the moments stream through
 *                             too, because checkpoint_load rejects a file with
 *                             any non-finite float (checkpoint.c:403-405) and
 *                             that check runs on the device.  Transactional:
 *                             on failure *out stays NULL.  The tokenizer
 *                             fingerprint must equal expected_tokenizer_hash
 *                             (checkpoint.c:376) unless flags has
 *                             MC_CKPT_ANY_TOKENIZER.  The optimizer type is
 *                             reported, not matched (a decoder has none).
 * Rejections return MC_ERR_INVALID and name the failed check.
 */
#define MC_CKPT_ANY_TOKENIZER 0x1u
typedef struct {
    uint32_t version;                  /* 4 or 5 */
    int32_t vocab_size, dim, n_layers, n_heads, ffn_dim, max_seq;
    uint64_t n_params;                 /* model floats (checkpoint.c:33-41) */
    int64_t step;
    uint64_t rng_state;                /* as checkpoint_load restores it: 0 -> 0x123456789abcdef0 */
    uint64_t tokenizer_hash;
    float lr, beta1, beta2, eps, weight_decay, schedule_base_lr;
    int64_t schedule_total_steps, schedule_warmup_steps;
    int32_t schedule_type;             /* 0 cosine, 1 constant */
    int32_t optimizer_type;            /* 0 AdamW, 1 Lion (v4: AdamW) */
    uint64_t header_bytes, file_bytes;
} mc_checkpoint_info;
mc_status mc_checkpoint_inspect(const char* path, mc_checkpoint_info* info);
mc_status mc_model_load_checkpoint(const char* path, int weights_dtype,
    uint64_t expected_tokenizer_hash, unsigned flags, mc_model** out,
    mc_checkpoint_info* info);

/*
 * mc_gemm — C[M][N] = A[M][K] . B[N][K]^T on the tensor cores (tcgen05.mma,
 * TMEM accumulator, TMA-fed 128 x 128 tiles): the kernel the prefill uses
 * with MINIMA_CUDA_PREFILL=tcgen05, exposed for tests and measurement.
 * No reference counterpart (the reference's matmul is forward.c:24-40 on the
 * CPU).  MC_GEMM_TF32: A, B fp32 (multiplied as tf32, fp32 accumulate);
 * MC_GEMM_BF16: A, B bf16 bit patterns (uint16).  C is fp32, row-major with
 * leading dimension N.  K * element size must be a multiple of 16 bytes.
 * Host pointers unless flags has MC_DEVICE_POINTERS (then 16-byte aligned
 * device pointers).  *ms (optional) receives the kernel's device time.
 */
#define MC_GEMM_TF32 0
#define MC_GEMM_BF16 1
mc_status mc_gemm(int kind, const void* A, const void* B, float* C, int M, int N, int K,
    unsigned flags, float* ms);

const char* mc_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
