// gsv_ar_smoke.cpp -- exercises the drop-in `class gsv_ar` the way gsv.cpp's callers do
// (src/gsv_engine.cpp:467, tests/bench_ar_width.cpp:38-74) and prints the results as JSON lines.
//   gsv_ar_smoke <ar.gguf> <requests.bin> <max_steps> <early_stop> <seed_base>
// requests.bin: int32 B, then per request int32 T, int32 P, T phones, T*1024 float bert, P prompt.
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "gsv_ar.h"

int main(int argc, char** argv) {
    if (argc < 6) {
        std::fprintf(stderr, "usage: %s <ar.gguf> <requests.bin> <max_steps> <early_stop> <seed_base>\n", argv[0]);
        return 2;
    }
    gsv_ar_cfg cfg;
    cfg.device = "cuda";
    gsv_ar* ar = gsv_ar::load(argv[1], cfg);
    if (!ar) return 1;
    FILE* f = std::fopen(argv[2], "rb");
    if (!f) return 1;
    int32_t B = 0;
    if (std::fread(&B, 4, 1, f) != 1) return 1;
    std::vector<gsv_ar_request> reqs(B);
    for (auto& r : reqs) {
        int32_t T = 0, P = 0;
        if (std::fread(&T, 4, 1, f) != 1 || std::fread(&P, 4, 1, f) != 1) return 1;
        r.phones.resize(T);
        r.bert.resize((size_t)T * 1024);
        r.prompt.resize(P);
        if (std::fread(r.phones.data(), 4, T, f) != (size_t)T) return 1;
        if (std::fread(r.bert.data(), 4, r.bert.size(), f) != r.bert.size()) return 1;
        if (std::fread(r.prompt.data(), 4, P, f) != (size_t)P) return 1;
    }
    std::fclose(f);
    gsv_sampler_cfg sc;
    std::vector<float> lg;
    ar->first_logits(reqs, lg);
    std::printf("{\"first_logits\": [");
    for (size_t i = 0; i < 8 && i < lg.size(); i++) std::printf("%s%.9g", i ? ", " : "", lg[i]);
    std::printf("]}\n");
    gsv_ar_result res = ar->generate(reqs, sc, std::strtoull(argv[5], nullptr, 10), std::atoi(argv[4]), std::atoi(argv[3]));
    for (size_t b = 0; b < res.tokens.size(); b++) {
        std::printf("{\"seq\": %zu, \"tokens\": [", b);
        for (size_t i = 0; i < res.tokens[b].size(); i++) std::printf("%s%d", i ? ", " : "", res.tokens[b][i]);
        std::printf("]}\n");
    }
    std::printf("{\"lens\": [");
    for (size_t i = 0; i < res.lens.size(); i++) std::printf("%s%d", i ? ", " : "", res.lens[i]);
    std::printf("], \"hidden\": %d, \"vocab\": %d, \"eos\": %d}\n", ar->hidden_dim(), ar->vocab_size(), ar->eos());
    ar->release_cache();
    delete ar;
    return 0;
}
