// gsv_ar_server.h -- continuous-batching AR front end for a service, over the gsvcu C ABI.
//
// It takes the place of gsv.cpp's svc::ArBatcher (tools/svc_core.h:1244-1340) and its call of
// gsv_engine::ar_generate_batch (src/gsv_engine.cpp:418-470): instead of grouping at most
// kMaxBatch = 8 tasks of one ar_key within a 20 ms grace window and running them as one blocking
// batch, every submitted task is admitted into a free slot of one running batch as soon as a slot
// and KV pages are free, and its future is fulfilled the moment it finishes. Tasks of different
// keys (voice, prompt, sampler settings, limits) share the batch.
//
// A task carries the AR inputs of an ArTask (tools/svc_core.h:1231-1242). Its sequence is built as
// ar_generate_batch builds it: phones = prompt_phones ++ phones, BERT features [1024][Pp + Pt] =
// prompt_bert ++ bert column-wise (zeros where a side is empty), reference prompt = prompt_codes; the
// result is the generated semantic tokens (prompt codes excluded). Each task is its own group for
// the early-stop rule, i.e. it decodes as gsv_ar::generate of that one sequence.
//
// Thread safety: submit() may be called from any thread; one worker thread owns the GPU context.
#pragma once
#include <cstdint>
#include <future>
#include <memory>
#include <string>
#include <vector>

#include "gsv_sampler.h"

struct gsv_ar_task {
    std::vector<int32_t> phones;          // target text phones
    std::vector<float> bert;              // [1024][phones.size()] or empty (zeros)
    std::vector<int32_t> prompt_phones;   // reference text phones (non-empty)
    std::vector<int32_t> prompt_codes;    // reference semantic codes
    std::vector<float> prompt_bert;       // [1024][prompt_phones.size()] or empty (zeros)
    int max_steps = 1500;
    int early_stop = 400;                 // -1: off
    gsv_sampler_cfg sampler;
    uint64_t seed = 0;
};

struct gsv_ar_server_cfg {
    int device = 0;
    int slots = 64;            // sequences in flight
    int max_ctx = 2048;        // longest prompt_phones + phones + prompt_codes + max_steps
    bool kv_f32 = false;       // F16 paged KV by default
    int chunk = 16;            // decode steps between admissions / completions
};

class gsv_ar_server {
public:
    // nullptr on failure (message on stderr), like gsv_ar::load.
    static gsv_ar_server* create(const std::string& model_path, const gsv_ar_server_cfg& cfg);
    ~gsv_ar_server();   // shutdown()

    // Semantic tokens of the task; an empty vector if the task is invalid or the server stops first.
    std::future<std::vector<int32_t>> submit(gsv_ar_task task);

    // Stops the worker; tasks not finished yet get empty results.
    void shutdown();

    uint64_t tasks_done() const;
    gsv_ar_server(const gsv_ar_server&) = delete;
    gsv_ar_server& operator=(const gsv_ar_server&) = delete;

private:
    struct impl;
    explicit gsv_ar_server(impl* p);
    impl* p_;
};
