// config.h — compile-time model constants of the Qwen3-0.6B decode engine.
//
// Drop-in mirror of the reference's config.h (config.h:9-40): the same names
// and values, so code written against the reference compiles unchanged.  The
// values are the Qwen3-0.6B architecture: hidden 1024, 28 layers, 16 query
// heads and 8 KV heads of 128, SwiGLU width 3072, vocabulary 151936, RMSNorm
// epsilon 1e-6, RoPE theta 1e6, and an 8192-position KV cache.
#pragma once

#define COLOR_RESET    "\x1b[0m"
#define COLOR_BOLD_RED "\x1b[1;31m"
#define COLOR_GREEN    "\x1b[32m"
#define COLOR_YELLOW   "\x1b[33m"
#define COLOR_ORANGE   "\x1b[33m"
#define COLOR_CYAN     "\033[36m"

#define MAX_LINE_WIDTH 80

constexpr int SEQ_LEN = 8192;
constexpr int PROMPT_BUFFER_SIZE = 32768;
constexpr int VOCAB_SIZE = 151936;

constexpr int DIM = 1024;
constexpr int HIDDEN_DIM = 3072;
constexpr int N_LAYERS = 28;
constexpr int N_HEADS = 16;
constexpr int N_KV_HEADS = 8;
constexpr int HEAD_DIM = 128;

constexpr float INV_HEAD_DIM = 1.0f / HEAD_DIM;
constexpr float INV_DIM = 1.0f / DIM;

constexpr float ROPE_THETA = 1000000.0f;
constexpr float EPS = 1e-6f;

constexpr int Q_DIM = N_HEADS * HEAD_DIM;      // 2048
constexpr int KV_DIM = N_KV_HEADS * HEAD_DIM;  // 1024
