// gsv_ar_server_test.cpp -- submits tasks to gsv_ar_server from several threads, the way a service's
// request handlers call svc::ArBatcher::enqueue (tools/svc_core.h:1265-1273), and prints each task's
// semantic tokens as a JSON line (in task order), then {"done": n}.
//   gsv_ar_server_test <ar.gguf> <tasks.bin> <threads> <slots>
// tasks.bin: int32 N, then per task: int32 Pt, Pp, C, max_steps, early_stop, top_k; float top_p,
// temperature, repetition_penalty; uint64 seed; Pt phones, Pt*1024 bert, Pp prompt phones,
// Pp*1024 prompt bert, C prompt codes.
#include <cstdio>
#include <future>
#include <thread>
#include <vector>

#include "gsv_ar_server.h"

template <typename T>
static bool rd(FILE* f, T* p, size_t n) {
    return std::fread(p, sizeof(T), n, f) == n;
}

int main(int argc, char** argv) {
    if (argc < 5) {
        std::fprintf(stderr, "usage: %s <ar.gguf> <tasks.bin> <threads> <slots>\n", argv[0]);
        return 2;
    }
    FILE* f = std::fopen(argv[2], "rb");
    if (!f) return 1;
    int32_t N = 0;
    if (!rd(f, &N, 1) || N < 1) return 1;
    std::vector<gsv_ar_task> tasks((size_t)N);
    for (auto& t : tasks) {
        int32_t h[6];
        float s[3];
        if (!rd(f, h, 6) || !rd(f, s, 3) || !rd(f, &t.seed, 1)) return 1;
        const int Pt = h[0], Pp = h[1], C = h[2];
        t.max_steps = h[3];
        t.early_stop = h[4];
        t.sampler.top_k = h[5];
        t.sampler.top_p = s[0];
        t.sampler.temperature = s[1];
        t.sampler.repetition_penalty = s[2];
        t.phones.resize((size_t)Pt);
        t.bert.resize((size_t)Pt * 1024);
        t.prompt_phones.resize((size_t)Pp);
        t.prompt_bert.resize((size_t)Pp * 1024);
        t.prompt_codes.resize((size_t)C);
        if (!rd(f, t.phones.data(), t.phones.size()) || !rd(f, t.bert.data(), t.bert.size()) ||
            !rd(f, t.prompt_phones.data(), t.prompt_phones.size()) ||
            !rd(f, t.prompt_bert.data(), t.prompt_bert.size()) || !rd(f, t.prompt_codes.data(), t.prompt_codes.size()))
            return 1;
    }
    std::fclose(f);

    gsv_ar_server_cfg cfg;
    cfg.slots = std::atoi(argv[4]);
    cfg.max_ctx = 1024;
    gsv_ar_server* srv = gsv_ar_server::create(argv[1], cfg);
    if (!srv) return 1;
    const int nth = std::max(1, std::atoi(argv[3]));
    std::vector<std::future<std::vector<int32_t>>> futs((size_t)N);
    std::vector<std::thread> th;
    for (int k = 0; k < nth; k++)   // thread k submits tasks k, k + nth, ...
        th.emplace_back([&, k] {
            for (int i = k; i < N; i += nth) futs[(size_t)i] = srv->submit(tasks[(size_t)i]);
        });
    for (auto& x : th) x.join();
    for (int i = 0; i < N; i++) {
        const std::vector<int32_t> toks = futs[(size_t)i].get();
        std::printf("{\"task\": %d, \"tokens\": [", i);
        for (size_t j = 0; j < toks.size(); j++) std::printf(j ? ", %d" : "%d", toks[j]);
        std::printf("]}\n");
    }
    std::printf("{\"done\": %llu}\n", (unsigned long long)srv->tasks_done());
    delete srv;
    return 0;
}
