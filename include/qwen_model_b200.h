/* qwen_model_b200.h — the reference's C++ decode API (qwen_model.cuh and
 * sampler.h, Ramshankar07/qwen600-ROCm-inference) on top of libqwen_b200.so.
 *
 * A program written against the reference keeps its calls:
 *
 *     Transformer t;  build_transformer(&t, "model.safetensors");
 *     Sampler s;      build_sampler(&s, 0.6f, 0.95f, 20, seed);
 *     float* logits = forward(&t, token, pos);      // qwen_model.cuh:772
 *     int next = sample(&s, logits);                // sampler.h:120
 *     free_sampler(&s); free_transformer(&t);
 *
 * Same names and argument meaning as qwen_model.cuh:51-60 (Transformer),
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

#include <stdexcept>
#include <string>

#include "qwen_b200.h"

struct Transformer {
    qwen_t* handle = nullptr;
    float* h_logits = nullptr;   /* pinned host logits [VOCAB] owned by the handle */
};

inline void qwen_model_b200_check(int rc, const char* what) {
    if (rc != QWEN_OK) throw std::runtime_error(std::string(what) + ": " + qwen_last_error());
}

inline void build_transformer(Transformer* t, const char* checkpoint_path, int device = 0) {
    qwen_model_b200_check(qwen_create(checkpoint_path, device, &t->handle), "build_transformer");
    t->h_logits = qwen_host_logits(t->handle);
}

inline void free_transformer(Transformer* t) {
    qwen_destroy(t->handle);
    t->handle = nullptr;
    t->h_logits = nullptr;
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

#endif /* QWEN_MODEL_B200_H */
