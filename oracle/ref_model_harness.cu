// ref_model_harness.cu — TEST INFRASTRUCTURE.  Compiles the reference's own
// CUDA decode path (qwen_model.cuh with static_loader.h and config.h, included
// from the reference tree via -I) for sm_100a and exposes build_transformer /
// forward / free_transformer through C symbols, so a GPU-side script can record
// the reference's logits on the synthetic checkpoint as golden vectors.
// The reference's attention is only valid for pos < 1024 (one thread per
// position, qwen_model.cuh:560-564, 626).
#include <cstring>
#include "qwen_model.cuh"

static Transformer* g_t = nullptr;

extern "C" int ref_build(const char* path) {
    if (g_t) return -1;
    g_t = new Transformer();
    build_transformer(g_t, path);
    return 0;
}

extern "C" int ref_forward(int token, int pos, float* logits_out) {
    if (!g_t || pos < 0 || pos >= 1024) return -1;
    float* l = forward(g_t, token, pos);
    memcpy(logits_out, l, sizeof(float) * VOCAB_SIZE);
    return 0;
}

extern "C" void ref_free(void) {
    if (!g_t) return;
    free_transformer(g_t);
    delete g_t;
    g_t = nullptr;
}
