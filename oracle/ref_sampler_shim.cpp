// ref_sampler_shim.cpp — TEST INFRASTRUCTURE.  Exposes the reference's own
// sampler (sampler.h, included from the reference tree via -I) through a C
// symbol so tests can pin the oracle's restated sampler against it.
#include "sampler.h"

extern "C" int ref_sample(const float* logits, float temperature, float topp, int top_k, unsigned long long* rng) {
    Sampler s;
    build_sampler(&s, temperature, topp, top_k, *rng);
    const int t = sample(&s, const_cast<float*>(logits));
    *rng = s.rng_state;
    free_sampler(&s);
    return t;
}

extern "C" unsigned int ref_random_u32(unsigned long long* rng) { return random_u32(rng); }
