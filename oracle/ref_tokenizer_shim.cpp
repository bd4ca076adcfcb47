// ref_tokenizer_shim.cpp — TEST INFRASTRUCTURE.  Exposes the reference's own
// tokenizer (tokenizer.h, included from the reference tree via -I: its
// build_tokenizer and encode) through a C symbol, so the golden-vector script
// can record the reference's token ids for the library's tokenizer tests.
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "tokenizer.h"

// tokenizer.h declares construct_path; the reference defines it in its driver.
void construct_path(char* out_path, size_t out_size, const char* dir, const char* filename) {
    snprintf(out_path, out_size, "%s/%s", dir, filename);
}

// Token ids of `text` under <dir>/tokenizer.bin (dir must also hold the
// template_user.txt / template_system.txt files build_tokenizer reads).
// Writes at most cap ids; returns the count.
extern "C" int ref_tokenizer_encode(const char* dir, const char* text, int* tokens, int cap) {
    static Tokenizer t;
    static std::string loaded;
    if (loaded != dir) {
        if (!loaded.empty()) free_tokenizer(&t);
        build_tokenizer(&t, dir, 0);
        loaded = dir;
    }
    std::vector<int> buf(std::string(text).size() + 8, -1);
    int n = 0;
    encode(&t, const_cast<char*>(text), buf.data(), &n);
    for (int i = 0; i < n && i < cap; i++) tokens[i] = buf[i];
    return n;
}
