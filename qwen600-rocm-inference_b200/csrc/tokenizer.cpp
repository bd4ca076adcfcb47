// tokenizer.cpp — host-side tokenizer of the chat driver: the reference's
// tokenizer.bin format (written by export.py:168-244, read by
// tokenizer.h:38-70) and its encode / decode (tokenizer.h:80-185).
//
// Same results as the reference on every input the reference handles
// defined-ly, with hash lookups instead of its linear vocabulary scans
// (tokenizer.h:87-94 scans all 151,936 entries per lookup, O(n^2 V) per
// prompt) and a per-pair candidate cache, so one merge costs O(n):
//   - vocabulary strings are C strings: an entry is compared up to its first
//     NUL byte, and the first entry with a given string wins (str_lookup);
//   - a '<' starts a special token when a '>' follows within 64 bytes and the
//     whole "<...>" is a vocabulary entry (tokenizer.h:115-137);
//   - otherwise each input byte is the one-byte entry for that byte;
//   - then, while some adjacent pair concatenates to an entry, the pair whose
//     entry has the highest score (first pair on ties; scores must exceed
//     -1e10) is merged (tokenizer.h:150-181).
// Deliberate differences, where the reference is undefined: a byte with no
// one-byte entry is skipped and counted (the reference counts a token slot it
// never writes, tokenizer.h:145-147); the '>' search stops at the end of the
// text (the reference may read past it, tokenizer.h:118-123).
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/qwen_b200.h"
#include "../host/config.h"

int qwen_internal_fail(int code, const std::string& msg);   // engine.cu: sets qwen_last_error()

struct qwen_tokenizer {
    std::vector<std::string> vocab;   // C-string view of every entry (cut at its first NUL)
    std::vector<float> score;
    std::unordered_map<std::string, int> index;   // string -> lowest id
    unsigned max_token_length = 0, bos = 0, eos = 0;
    int lookup(const std::string& s) const {
        auto it = index.find(s);
        return it == index.end() ? -1 : it->second;
    }
};

extern "C" int qwen_tokenizer_load(const char* path, int vocab_size, qwen_tokenizer_t** out) {
    if (!path || !out) return qwen_internal_fail(QWEN_E_ARG, "NULL argument");
    if (vocab_size <= 0) vocab_size = VOCAB_SIZE;
    *out = nullptr;
    FILE* f = fopen(path, "rb");
    if (!f) return qwen_internal_fail(QWEN_E_IO, std::string("cannot open tokenizer file ") + path);
    auto* t = new qwen_tokenizer;
    uint32_t hdr[3];
    if (fread(hdr, sizeof(uint32_t), 3, f) != 3) {
        fclose(f);
        delete t;
        return qwen_internal_fail(QWEN_E_FORMAT, "tokenizer file shorter than its 12-byte header");
    }
    t->max_token_length = hdr[0];
    t->bos = hdr[1];
    t->eos = hdr[2];
    t->vocab.resize(vocab_size);
    t->score.assign(vocab_size, 0.0f);
    std::string buf;
    for (int i = 0; i < vocab_size; i++) {
        float sc;
        if (fread(&sc, sizeof(float), 1, f) != 1) continue;   // past the end: empty entry (tokenizer.h:53-56)
        t->score[i] = sc;
        uint32_t len = 0;
        if (fread(&len, sizeof(uint32_t), 1, f) != 1 || len > (1u << 20)) {
            fclose(f);
            delete t;
            return qwen_internal_fail(QWEN_E_FORMAT, "tokenizer entry " + std::to_string(i) + ": bad length");
        }
        buf.resize(len);
        if (len && fread(&buf[0], 1, len, f) != len) {
            fclose(f);
            delete t;
            return qwen_internal_fail(QWEN_E_FORMAT, "tokenizer entry " + std::to_string(i) + ": truncated");
        }
        t->vocab[i] = std::string(buf.c_str());   // C-string semantics: up to the first NUL
    }
    fclose(f);
    for (int i = vocab_size - 1; i >= 0; i--) t->index[t->vocab[i]] = i;   // lowest id wins
    *out = t;
    return QWEN_OK;
}

extern "C" void qwen_tokenizer_free(qwen_tokenizer_t* t) { delete t; }

extern "C" int qwen_tokenizer_info(const qwen_tokenizer_t* t, int* vocab_size, int* max_token_length, int* bos, int* eos) {
    if (!t) return qwen_internal_fail(QWEN_E_ARG, "NULL tokenizer");
    if (vocab_size) *vocab_size = (int)t->vocab.size();
    if (max_token_length) *max_token_length = (int)t->max_token_length;
    if (bos) *bos = (int)t->bos;
    if (eos) *eos = (int)t->eos;
    return QWEN_OK;
}

extern "C" int qwen_tokenizer_decode(const qwen_tokenizer_t* t, int token, const char** piece) {
    if (!t || !piece) return qwen_internal_fail(QWEN_E_ARG, "NULL argument");
    if (token < 0 || token >= (int)t->vocab.size()) return qwen_internal_fail(QWEN_E_ARG, "token out of range");
    *piece = t->vocab[token].c_str();
    return QWEN_OK;
}

extern "C" int qwen_tokenizer_encode(const qwen_tokenizer_t* t, const char* text, int* tokens, int cap, int* n_tokens,
                                     int* n_unknown) {
    if (!t || !text || !n_tokens || (cap > 0 && !tokens) || cap < 0) return qwen_internal_fail(QWEN_E_ARG, "NULL argument or negative cap");
    std::vector<int> ids;
    int unknown = 0;
    const size_t n = strlen(text);
    for (size_t i = 0; i < n; i++) {
        int id = -1;
        if (text[i] == '<') {
            for (size_t k = 0; k < 64 && i + k < n; k++) {
                if (text[i + k] == '>') {
                    id = t->lookup(std::string(text + i, k + 1));
                    if (id != -1) i += k;
                    break;
                }
            }
        }
        if (id == -1) id = t->lookup(std::string(1, text[i]));
        if (id == -1) { unknown++; continue; }
        ids.push_back(id);
    }
    // cand[i]: the entry for ids[i] ++ ids[i + 1] (or -1)
    auto pair_id = [&](int a, int b) { return t->lookup(t->vocab[a] + t->vocab[b]); };
    std::vector<int> cand(ids.size() > 1 ? ids.size() - 1 : 0);
    for (size_t i = 0; i + 1 < ids.size(); i++) cand[i] = pair_id(ids[i], ids[i + 1]);
    for (;;) {
        float best = -1e10f;
        int at = -1;
        for (size_t i = 0; i < cand.size(); i++)
            if (cand[i] != -1 && t->score[cand[i]] > best) { best = t->score[cand[i]]; at = (int)i; }
        if (at < 0) break;
        ids[at] = cand[at];
        ids.erase(ids.begin() + at + 1);
        cand.erase(cand.begin() + at);
        if (at > 0) cand[at - 1] = pair_id(ids[at - 1], ids[at]);
        if ((size_t)at < cand.size()) cand[at] = pair_id(ids[at], ids[at + 1]);
    }
    *n_tokens = (int)ids.size();
    if (n_unknown) *n_unknown = unknown;
    if ((int)ids.size() > cap) return qwen_internal_fail(QWEN_E_ARG, "token buffer too small: need " + std::to_string(ids.size()));
    std::copy(ids.begin(), ids.end(), tokens);
    return QWEN_OK;
}
