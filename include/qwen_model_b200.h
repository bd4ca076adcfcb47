/* qwen_model_b200.h — the reference's C++ decode API (qwen_model.cuh and
 * sampler.h, Ramshankar07/qwen600-ROCm-inference) on top of libqwen_b200.so.
 *
 * A program written against the reference keeps its calls (and, host-only,
 * its tokenizer.h calls: Tokenizer, build_tokenizer, encode, decode):
 *
 *     Transformer t;  build_transformer(&t, "model.safetensors");
 *     Sampler s;      build_sampler(&s, 0.6f, 0.95f, 20, seed);
 *     float* logits = forward(&t, token, pos);      // qwen_model.cuh:772
 *     int next = sample(&s, logits);                // sampler.h:120
 *     free_sampler(&s); free_transformer(&t);
 *
 * Same names and argument meaning as qwen_model.cuh:26-60 (TransformerWeights,
 * RunState, Transformer with its weights / state / h_logits members),
 * :82 (build_transformer), :94 (free_transformer), :772 (forward) and
 * sampler.h:11-24 (ProbIndex, Sampler), :100 (build_sampler), :115
 * (free_sampler), :120 (sample).  Differences, all in the direction of safety:
 *   - errors throw std::runtime_error with qwen_last_error()'s message (the
 *     reference throws on I/O errors, static_loader.h:411-434, and exit()s on
 *     CUDA errors, static_loader.h:22-30);
 *   - build_transformer takes an optional device index (the reference uses
 *     device 0);
 *   - forward() returns the handle's pinned fp32 logits, overwritten by every
 *     call, exactly as the reference's Transformer.h_logits;
 *   - sample() with top_k = 0 (full vocabulary) is served: the reference's
 *     quickselect indexes one past the array in that case (sampler.h:54-79).
 * Everything is inline, so several translation units may include this header
 * (the reference's headers define non-inline functions and allow only one).
 */
#ifndef QWEN_MODEL_B200_H
#define QWEN_MODEL_B200_H

#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>

#include "qwen_b200.h"
#include "static_loader_b200.h"

using TransformerWeights = qwen_loader::QwenWeights;   /* qwen_model.cuh:26 */

/* RunState (qwen_model.cuh:31-49): the engine keeps its activations in
 * exchange buffers of its own layout, so only the members with the same
 * meaning and layout are set; the rest stay nullptr rather than point at
 * differently laid-out memory (the engine's K/V cache is
 * [layer][kv_head][pos][head_dim], the reference's [layer][pos][kv_dim]). */
struct RunState {
    qwen_loader::bf16 *x = nullptr, *xb = nullptr, *xb2 = nullptr, *hb = nullptr, *hb2 = nullptr, *q = nullptr;
    float* att = nullptr;
    qwen_loader::bf16* logits = nullptr;
    qwen_loader::bf16 *key_cache = nullptr, *value_cache = nullptr;
    const float* d_logits_fp32 = nullptr;   /* the last step's fp32 logits on the device [VOCAB] */
};

/* Transformer (qwen_model.cuh:51-60).  `weights` points into the handle's
 * device weight block (the handle owns it); the engine uses no cuBLAS, so
 * cublas_handle stays nullptr. */
struct Transformer {
    TransformerWeights weights;
    RunState state;
    void* cublas_handle = nullptr;
    float* h_logits = nullptr;   /* pinned host logits [VOCAB] owned by the handle */
    qwen_t* handle = nullptr;
};

inline void qwen_model_b200_check(int rc, const char* what) {
    if (rc != QWEN_OK) throw std::runtime_error(std::string(what) + ": " + qwen_last_error());
}

inline void build_transformer(Transformer* t, const char* checkpoint_path, int device = 0) {
    qwen_model_b200_check(qwen_create(checkpoint_path, device, &t->handle), "build_transformer");
    t->h_logits = qwen_host_logits(t->handle);
    qwen_loader::assign_weight_pointers(const_cast<void*>(qwen_device_weights(t->handle)), t->weights);
    t->state = RunState{};
    t->state.d_logits_fp32 = qwen_device_logits(t->handle);
}

inline void free_transformer(Transformer* t) {
    qwen_destroy(t->handle);
    t->handle = nullptr;
    t->h_logits = nullptr;
    t->weights = TransformerWeights{};
    t->state = RunState{};
}

/* Logits of position `pos` for `token`; positions must arrive in order
 * (0..pos cached), pos < SEQ_LEN. */
inline float* forward(Transformer* t, int token, int pos) {
    qwen_model_b200_check(qwen_forward(t->handle, token, pos, t->h_logits), "forward");
    return t->h_logits;
}

typedef struct {
    float prob;
    int index;
} ProbIndex;

typedef struct {
    float temperature;
    float topp;
    int top_k;
    unsigned long long rng_state;
    ProbIndex* probindex;   /* unused: the library's sampler keeps its own scratch */
} Sampler;

inline void build_sampler(Sampler* s, float temperature, float topp, int top_k, unsigned long long rng_seed) {
    s->temperature = temperature;
    s->topp = topp;
    s->top_k = top_k == 0 ? qwen_vocab_size() : top_k;
    s->rng_state = rng_seed;
    s->probindex = nullptr;
}

inline void free_sampler(Sampler* s) { s->probindex = nullptr; }

inline int sample(Sampler* s, float* logits) {
    qwen_sampling_t sp;
    sp.temperature = s->temperature;
    sp.topp = s->topp;
    sp.top_k = s->top_k;
    int tok = -1;
    qwen_model_b200_check(qwen_sample_host(logits, qwen_vocab_size(), &sp, &s->rng_state, &tok), "sample");
    return tok;
}

/* ---- tokenizer.h -------------------------------------------------------- */
/* Tokenizer, build_tokenizer, free_tokenizer, decode, encode with the names and
 * argument meaning of tokenizer.h:14-23, :38, :76, :80, :104.  build_tokenizer
 * reads <dir_path>/tokenizer.bin and the two template files of the mode
 * (template_user[_thinking].txt, template_system[_thinking].txt) as the
 * reference does; encode writes at most strlen(text) ids (one per input byte
 * is the most the reference's scheme produces) and skips bytes without a
 * one-byte entry instead of leaving an unwritten slot.  Host-only: no GPU. */
struct Tokenizer {
    qwen_tokenizer_t* handle = nullptr;
    int vocab_size = 0;
    unsigned int max_token_length = 0;
    unsigned int bos_token_id = 0;
    unsigned int eos_token_id = 0;
    char prompt_template[1024] = {0};
    char system_prompt_template[1024] = {0};
};

inline void qwen_model_b200_read_template(char* buf, size_t size, const std::string& path) {
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) throw std::runtime_error("cannot open template file " + path);
    const size_t n = fread(buf, 1, size - 1, f);
    buf[n] = 0;
    fclose(f);
}

inline void build_tokenizer(Tokenizer* t, const char* dir_path, int enable_thinking) {
    std::string dir(dir_path);
    if (!dir.empty() && dir.back() != '/') dir += '/';
    qwen_model_b200_check(qwen_tokenizer_load((dir + "tokenizer.bin").c_str(), 0, &t->handle), "build_tokenizer");
    int v = 0, m = 0, b = 0, e = 0;
    qwen_model_b200_check(qwen_tokenizer_info(t->handle, &v, &m, &b, &e), "build_tokenizer");
    t->vocab_size = v;
    t->max_token_length = (unsigned)m;
    t->bos_token_id = (unsigned)b;
    t->eos_token_id = (unsigned)e;
    const char* sfx = enable_thinking ? "_thinking.txt" : ".txt";
    qwen_model_b200_read_template(t->prompt_template, sizeof(t->prompt_template), dir + "template_user" + sfx);
    qwen_model_b200_read_template(t->system_prompt_template, sizeof(t->system_prompt_template), dir + "template_system" + sfx);
}

inline void free_tokenizer(Tokenizer* t) {
    qwen_tokenizer_free(t->handle);
    t->handle = nullptr;
}

inline char* decode(Tokenizer* t, int token) {
    const char* piece = nullptr;
    qwen_model_b200_check(qwen_tokenizer_decode(t->handle, token, &piece), "decode");
    return const_cast<char*>(piece);
}

inline void encode(Tokenizer* t, char* text, int* tokens, int* n_tokens) {
    const int cap = (int)strlen(text);
    qwen_model_b200_check(qwen_tokenizer_encode(t->handle, text, tokens, cap, n_tokens, nullptr), "encode");
}

#endif /* QWEN_MODEL_B200_H */
