// ref_sampler_shim.cpp -- TEST INFRASTRUCTURE ONLY.
// C entry points over the reference's own sampler (gsv.cpp src/gsv_sampler.{h,cpp}), which is
// compiled from the read-only reference tree by oracle/Makefile into oracle/_ref/. Used to pin
// the oracle's sampler restatement and to generate tests/golden/ sampler fixtures.
#include "gsv_sampler.h"

#include <cstdint>

extern "C" {

void ref_logits_to_probs(int top_k, float top_p, float temperature, float rep, float* logits, int V,
                         const int32_t* prev, int n_prev, float* probs) {
    gsv_sampler_cfg c;
    c.top_k = top_k;
    c.top_p = top_p;
    c.temperature = temperature;
    c.repetition_penalty = rep;
    gsv_logits_to_probs(c, logits, V, prev, n_prev, probs);
}

uint64_t ref_rng_init(uint64_t seed) { return gsv_rng(seed).s; }

int ref_sample(const float* probs, int V, uint64_t* state) {
    gsv_rng r;
    r.s = *state;
    const int t = gsv_sample(probs, V, r, nullptr);
    *state = r.s;
    return t;
}

}  // extern "C"
