/* End-to-end text generation through Minima's own chat front end
 * (chat.c, compiled unmodified), linked either against the reference
 * generate.c (CPU) or against this repository's drop-in generate
 * (libminima_generate.so, the B200 token loop).  Test infrastructure: the
 * two builds read the same stdin and must print the same transcript.
 *
 *   chat_e2e console   chat_run_console (chat.c:179-366): the CHAT_* line
 *                      protocol the GUI drives, on stdin/stdout, with greedy
 *                      replies (a penalty, n-gram bans and a stop sequence)
 *   chat_e2e sampled   the same with seeded top-k/top-p sampling
 *   chat_e2e bench     chat_run_generation_benchmark (chat.c:457-556):
 *                      greedy and seeded sampled continuations of fixed
 *                      prompts plus their repetition statistics
 *
 * The model is model_init_config(seed 11) of a small config and the
 * tokenizer is trained by tokenizer_train (tokenizer.c) on the corpus
 * below, so no file is read.  CHAT_STATS lines carry wall-clock rates and
 * are the only lines expected to differ between the builds.
 */
#include "arena.h"
#include "chat.h"
#include "config.h"
#include "generate.h"
#include "model.h"
#include "tokenizer.h"
#include "util.h"

#include <stdbool.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static const char kCorpus[] =
    "Human: hello there, how is the weather today?\n"
    "Assistant: the weather is mild and the sky is clear over the hills.\n"
    "Human: what should we cook for dinner tonight?\n"
    "Assistant: a warm soup with bread would suit a quiet evening.\n"
    "Human: tell me something about rivers.\n"
    "Assistant: rivers carry water from the mountains down to the sea.\n"
    "Human: can you count to five?\n"
    "Assistant: one, two, three, four, five.\n"
    "Human: which colour is the grass in spring?\n"
    "Assistant: the grass in spring is bright green after the rain.\n"
    "Human: what do cats like to do?\n"
    "Assistant: cats like to sleep in the sun and chase small things.\n"
    "Human: how far away is the moon?\n"
    "Assistant: the moon is about three hundred and eighty thousand kilometres away.\n"
    "Human: thank you for the help.\n"
    "Assistant: you are welcome, have a pleasant day.\n";

/* The drop-in's error text (absent from the reference build). */
extern const char* minima_cuda_last_error(void) __attribute__((weak));

static void report_drop_in_error(void) {
    if (minima_cuda_last_error && minima_cuda_last_error()[0])
        fprintf(stderr, "drop-in: %s\n", minima_cuda_last_error());
}

int main(int argc, char** argv) {
    atexit(report_drop_in_error);
    const char* mode = argc > 1 ? argv[1] : "console";
    static Tokenizer tok;
    Arena model_arena, tok_arena, cache_arena;
    if (!arena_init(&model_arena, 8u << 20) || !arena_init(&tok_arena, 64u << 20) ||
        !arena_init(&cache_arena, 8u << 20)) {
        fprintf(stderr, "arena_init failed\n");
        return 2;
    }
    const ModelConfig config = {320, 64, 2, 4, 128, 256};
    Model model;
    if (!model_init_config(&model, &model_arena, 11, &config)) {
        fprintf(stderr, "model_init_config failed\n");
        return 2;
    }
    if (!tokenizer_train(&tok, &tok_arena, (const uint8_t*)kCorpus, sizeof(kCorpus) - 1,
                         config.vocab_size)) {
        fprintf(stderr, "tokenizer_train failed\n");
        return 2;
    }
    KVCache cache;
    if (!kvcache_init(&cache, &cache_arena, &model, config.max_seq)) {
        fprintf(stderr, "kvcache_init failed\n");
        return 2;
    }
    if (strcmp(mode, "bench") == 0) return chat_run_generation_benchmark(&model, &tok, &cache) ? 0 : 1;
    const bool sampled = strcmp(mode, "sampled") == 0;
    ChatOptions options;
    memset(&options, 0, sizeof(options));
    options.seed = 7;
    options.sampling_seed = 99;          /* fixed: the reply does not depend on clock() */
    options.temperature = sampled ? 0.8f : 1.0f;
    options.top_p = sampled ? 0.9f : 1.0f;
    options.repetition_penalty = 1.1f;
    options.top_k = sampled ? 40 : 1;
    options.max_new_tokens = 48;
    options.no_repeat_ngram_size = 3;
    options.stop_sequence = "\nHuman:";
    return chat_run_console(&model, &tok, &cache, &options);
}
