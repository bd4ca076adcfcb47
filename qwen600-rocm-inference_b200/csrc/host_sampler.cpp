// host_sampler.cpp — host-side sampling entry points of the C ABI.
//
// qwen_sample_host: the reference's host sampler (sampler.h:27-175), restated
// for drop-in callers of sample(float* logits): xorshift64* (sampler.h:27-38),
// argmax with the first maximum winning (sampler.h:82-97), Hoare quickselect of
// the top_k candidates (sampler.h:54-79), temperature softmax (sampler.h:143-151),
// qsort-ordered top-p cut (sampler.h:153-165) and the inverse-CDF draw
// (sampler.h:167-174).  Candidate order follows the reference exactly, so the
// same logits and RNG state give the same token.
//
// qwen_sample_candidates: the device sampler's math (candidates in descending
// logit order, ties by ascending id) on a host list, for merging the per-GPU
// top-k lists of a vocabulary-sharded LM head.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <vector>

#include "../../include/qwen_b200.h"

namespace {

struct Cand { float p; int i; };

unsigned int xorshift_u32(unsigned long long* s) {
    *s ^= *s >> 12;
    *s ^= *s << 25;
    *s ^= *s >> 27;
    return (unsigned int)((*s * 0x2545F4914F6CDD1DULL) >> 32);
}
float xorshift_f32(unsigned long long* s) { return (xorshift_u32(s) >> 8) / 16777216.0f; }

void select_top(Cand* a, int n, int k) {   // Hoare's FIND: the k largest end up in [0, k)
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        const float pivot = a[k].p;
        int i = lo, j = hi;
        do {
            while (a[i].p > pivot) i++;
            while (a[j].p < pivot) j--;
            if (i <= j) { std::swap(a[i], a[j]); i++; j--; }
        } while (i <= j);
        if (j < k) lo = i;
        if (i > k) hi = j;
    }
}

int by_prob_desc(const void* x, const void* y) {
    const float a = static_cast<const Cand*>(x)->p, b = static_cast<const Cand*>(y)->p;
    return a > b ? -1 : (a < b ? 1 : 0);
}

// softmax / top-p / draw over candidates already in scan order
int draw(Cand* c, int nc, float temperature, float topp, unsigned long long* rng, bool sort_for_topp) {
    float mx = c[0].p;
    for (int i = 1; i < nc; i++) if (c[i].p > mx) mx = c[i].p;
    float sum = 0.0f;
    for (int i = 0; i < nc; i++) { const float e = expf((c[i].p - mx) / temperature); c[i].p = e; sum += e; }
    for (int i = 0; i < nc; i++) c[i].p /= sum;
    if (topp > 0.0f && topp < 1.0f) {
        if (sort_for_topp) qsort(c, nc, sizeof(Cand), by_prob_desc);
        float cum = 0.0f;
        int last = nc - 1;
        for (int i = 0; i < nc; i++) { cum += c[i].p; if (cum > topp) { last = i; break; } }
        nc = last + 1;
        sum = cum;
    }
    const float coin = xorshift_f32(rng) * sum;
    float cdf = 0.0f;
    for (int i = 0; i < nc; i++) { cdf += c[i].p; if (coin < cdf) return c[i].i; }
    return c[nc - 1].i;
}

}  // namespace

extern "C" int qwen_sample_host(const float* logits, int n, const qwen_sampling_t* sp, unsigned long long* rng, int* token_out) {
    if (!logits || !sp || !rng || !token_out || n <= 0) return QWEN_E_ARG;
    const int top_k = sp->top_k == 0 ? n : sp->top_k;
    if (sp->temperature == 0.0f || top_k == 1) {
        int mi = 0; float mp = logits[0];
        for (int i = 1; i < n; i++) if (logits[i] > mp) { mi = i; mp = logits[i]; }
        *token_out = mi;
        return QWEN_OK;
    }
    if (top_k < 0) return QWEN_E_ARG;
    std::vector<Cand> c(n);
    for (int i = 0; i < n; i++) { c[i].p = logits[i]; c[i].i = i; }
    const int nc = top_k < n ? top_k : n;
    // top_k >= n: every entry is a candidate, in index order (the reference's
    // quick_select would read its pivot past the end for k == n, sampler.h:63).
    if (nc < n) select_top(c.data(), n, nc);
    *token_out = draw(c.data(), nc, sp->temperature, sp->topp, rng, true);
    return QWEN_OK;
}

extern "C" int qwen_sample_candidates(const float* values, const int* ids, int n, const qwen_sampling_t* sp,
                                      unsigned long long* rng, int* token_out) {
    if (!values || !ids || !sp || !rng || !token_out || n <= 0) return QWEN_E_ARG;
    std::vector<Cand> c(n);
    for (int i = 0; i < n; i++) { c[i].p = values[i]; c[i].i = ids[i]; }
    std::sort(c.begin(), c.end(), [](const Cand& a, const Cand& b) { return a.p > b.p || (a.p == b.p && a.i < b.i); });
    const bool greedy = sp->temperature == 0.0f || sp->top_k == 1;
    if (greedy) { *token_out = c[0].i; return QWEN_OK; }
    if (sp->top_k < 1) return QWEN_E_UNSUPPORTED;
    const int nc = std::min(sp->top_k, n);
    *token_out = draw(c.data(), nc, sp->temperature, sp->topp, rng, false);
    return QWEN_OK;
}
