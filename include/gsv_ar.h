// gsv_ar.h -- the AR semantic-token decoder (GPT-SoVITS Text2SemanticDecoder) behind the B200 library.
//
// Drop-in for gsv.cpp's src/gsv_ar.h:13-67: the same types, members, defaults and signatures, so
// gsv_engine (src/gsv_engine.cpp:217,407,467,479) and the request scheduler
// (tools/svc_core.h:1329) compile and run unchanged. The implementation
// (gsv.cpp_b200/csrc/gsv_ar.cpp) forwards to the C ABI in gsvcu.h.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "gsv_sampler.h"

// One sequence: phone ids (any length; sequences of a batch may differ), BERT features laid out
// [bert_dim][n_phones] row-major (bert[k * T + t]), and the reference prompt's semantic codes.
struct gsv_ar_request {
    std::vector<int32_t> phones;
    std::vector<float> bert;
    std::vector<int32_t> prompt;
};

struct gsv_ar_cfg {
    int n_threads = 0;        // unused by the CUDA build (kept for source compatibility)
    int max_batch = 8;        // unused: the KV pool is sized from the actual batch
    bool verbose = false;
    std::string device;       // "" / "cuda" / "gpu" -> GPU 0; "N" or "x:N" -> GPU N; "cpu" is rejected
    bool disable_coopmat2 = true;   // Vulkan-only option of the reference; ignored
};

struct gsv_ar_result {
    std::vector<std::vector<int32_t>> tokens;   // per sequence: prompt + generated, without the stopping token
    std::vector<int> lens;                      // generated counts, in the order sequences finished
};

class gsv_ar {
public:
    // nullptr on failure (message on stderr); the caller owns the object.
    static gsv_ar* load(const std::string& gguf_path, const gsv_ar_cfg& cfg);
    ~gsv_ar();

    int hidden_dim() const;
    int vocab_size() const;
    int eos() const;
    int bert_dim() const;
    int prompt_len_expected() const;   // prompt length of the last call, 0 before any

    // Blocking generation with the reference stop rules: EOS masked for the first 11 steps,
    // early_stop_num (-1 = off) checked on sequence 0, max_steps, optional teacher forcing with
    // oracle_tokens (same token for every sequence), per-sequence seeds (else seed_base + 0x9E3779B9*b).
    gsv_ar_result generate(const std::vector<gsv_ar_request>& reqs, const gsv_sampler_cfg& sampler, uint64_t seed_base,
                           int early_stop_num = -1, int max_steps = 1500,
                           const std::vector<int32_t>* oracle_tokens = nullptr,
                           const std::vector<uint64_t>* seeds = nullptr);

    // Prefill only: last-position logits, B rows of vocab_size() values.
    void first_logits(const std::vector<gsv_ar_request>& reqs, std::vector<float>& logits_out);

    // Return the KV pool and step buffers to the device allocator.
    void release_cache();

private:
    gsv_ar();
    struct impl;
    impl* p;
};
