// Drives the reference-named C++ API (include/qwen_model_b200.h) the way the
// reference's main.cu:141-145 loop does: forward() then sample(), greedy.
// usage: shim_greedy <checkpoint> <n_prompt> <n_gen> <prompt token ids...>
// prints the generated token ids, one line, space separated.
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "qwen_model_b200.h"

int main(int argc, char** argv) {
    if (argc < 4) { std::fprintf(stderr, "usage: %s ckpt n_prompt n_gen ids...\n", argv[0]); return 2; }
    const int n_prompt = std::atoi(argv[2]), n_gen = std::atoi(argv[3]);
    if (argc != 4 + n_prompt || n_prompt < 1) { std::fprintf(stderr, "bad prompt\n"); return 2; }
    std::vector<int> prompt(n_prompt);
    for (int i = 0; i < n_prompt; i++) prompt[i] = std::atoi(argv[4 + i]);
    try {
        Transformer t;
        build_transformer(&t, argv[1]);
        Sampler s;
        build_sampler(&s, 0.0f, 0.9f, 0, 1234ull);   // temperature 0: argmax, as the reference's greedy runs
        int tok = prompt[0], pos = 0;
        for (; pos < n_prompt - 1; pos++) forward(&t, prompt[pos], pos);
        tok = prompt[n_prompt - 1];
        for (int i = 0; i < n_gen; i++, pos++) {
            float* logits = forward(&t, tok, pos);
            tok = sample(&s, logits);
            std::printf(i ? " %d" : "%d", tok);
        }
        std::printf("\n");
        free_sampler(&s);
        free_transformer(&t);
    } catch (const std::exception& e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 1;
    }
    return 0;
}
