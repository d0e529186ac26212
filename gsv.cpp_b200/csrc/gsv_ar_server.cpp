// gsv_ar_server.cpp -- continuous-batching front end over the gsvcu C ABI (see include/gsv_ar_server.h).
#include "gsv_ar_server.h"

#include <condition_variable>
#include <cstdio>
#include <cstring>
#include <deque>
#include <mutex>
#include <thread>
#include <unordered_map>

#include "gsvcu.h"

namespace {

constexpr int BERT_DIM = 1024;

struct pending {
    gsv_ar_task task;
    std::promise<std::vector<int32_t>> prom;
};

// The sequence ar_generate_batch builds for one item (src/gsv_engine.cpp:440-462).
struct built_request {
    std::vector<int32_t> phones, prompt;
    std::vector<float> bert;
    gsvcu_request view() const {
        return gsvcu_request{phones.data(), (int32_t)phones.size(), bert.data(), prompt.data(),
                             (int32_t)prompt.size()};
    }
};

bool build(const gsv_ar_task& t, built_request& out) {
    const size_t Pp = t.prompt_phones.size(), Pt = t.phones.size(), P = Pp + Pt;
    if (Pp == 0 || Pt == 0) return false;
    if (!t.prompt_bert.empty() && t.prompt_bert.size() != (size_t)BERT_DIM * Pp) return false;
    if (!t.bert.empty() && t.bert.size() != (size_t)BERT_DIM * Pt) return false;
    out.phones.clear();
    out.phones.insert(out.phones.end(), t.prompt_phones.begin(), t.prompt_phones.end());
    out.phones.insert(out.phones.end(), t.phones.begin(), t.phones.end());
    out.bert.assign((size_t)BERT_DIM * P, 0.0f);
    for (int k = 0; k < BERT_DIM; k++) {
        if (!t.prompt_bert.empty())
            std::memcpy(out.bert.data() + (size_t)k * P, t.prompt_bert.data() + (size_t)k * Pp, Pp * sizeof(float));
        if (!t.bert.empty())
            std::memcpy(out.bert.data() + (size_t)k * P + Pp, t.bert.data() + (size_t)k * Pt, Pt * sizeof(float));
    }
    out.prompt = t.prompt_codes;
    return true;
}

}  // namespace

struct gsv_ar_server::impl {
    gsv_ar_server_cfg cfg;
    gsvcu_ctx* ctx = nullptr;
    std::mutex m;
    std::condition_variable cv;
    std::deque<std::unique_ptr<pending>> queue;                            // submitted, not admitted
    std::unordered_map<int32_t, std::unique_ptr<pending>> running;         // by tag
    int32_t next_tag = 0;
    bool stop = false;
    uint64_t done = 0;
    std::thread worker;

    void run();
};

gsv_ar_server::gsv_ar_server(impl* p) : p_(p) {}

gsv_ar_server* gsv_ar_server::create(const std::string& model_path, const gsv_ar_server_cfg& cfg) {
    if (cfg.slots < 1 || cfg.max_ctx < 1 || cfg.chunk < 1) {
        std::fprintf(stderr, "[gsv_ar_server] invalid configuration\n");
        return nullptr;
    }
    gsvcu_ctx* ctx = nullptr;
    int rc = gsvcu_create(cfg.device, &ctx);
    if (rc == GSVCU_OK) rc = gsvcu_load_gguf(ctx, model_path.c_str());
    if (rc == GSVCU_OK) rc = gsvcu_kv_reserve(ctx, cfg.slots, cfg.max_ctx, cfg.kv_f32 ? GSVCU_KV_F32 : GSVCU_KV_F16);
    if (rc != GSVCU_OK) {
        std::fprintf(stderr, "[gsv_ar_server] %s\n", ctx ? gsvcu_last_error(ctx) : "no device context");
        if (ctx) gsvcu_destroy(ctx);
        return nullptr;
    }
    impl* p = new impl();
    p->cfg = cfg;
    p->ctx = ctx;
    p->worker = std::thread([p] { p->run(); });
    return new gsv_ar_server(p);
}

gsv_ar_server::~gsv_ar_server() {
    shutdown();
    if (p_->ctx) gsvcu_destroy(p_->ctx);
    delete p_;
}

std::future<std::vector<int32_t>> gsv_ar_server::submit(gsv_ar_task task) {
    auto item = std::make_unique<pending>();
    item->task = std::move(task);
    auto fut = item->prom.get_future();
    {
        std::lock_guard<std::mutex> lk(p_->m);
        if (p_->stop) {
            item->prom.set_value({});
            return fut;
        }
        p_->queue.push_back(std::move(item));
    }
    p_->cv.notify_all();
    return fut;
}

void gsv_ar_server::shutdown() {
    {
        std::lock_guard<std::mutex> lk(p_->m);
        if (p_->stop && !p_->worker.joinable()) return;
        p_->stop = true;
    }
    p_->cv.notify_all();
    if (p_->worker.joinable()) p_->worker.join();
    std::lock_guard<std::mutex> lk(p_->m);
    for (auto& q : p_->queue) q->prom.set_value({});
    p_->queue.clear();
    for (auto& r : p_->running) r.second->prom.set_value({});
    p_->running.clear();
    if (p_->ctx) gsvcu_serve_reset(p_->ctx);
}

uint64_t gsv_ar_server::tasks_done() const {
    std::lock_guard<std::mutex> lk(p_->m);
    return p_->done;
}

// Worker: admit queued tasks into free slots, run a chunk of decode steps, hand out what finished.
void gsv_ar_server::impl::run() {
    std::vector<gsvcu_finished> fin((size_t)cfg.slots);
    std::vector<int32_t> toks;
    for (;;) {
        std::vector<std::unique_ptr<pending>> admit;
        {
            std::unique_lock<std::mutex> lk(m);
            cv.wait(lk, [&] { return stop || !queue.empty() || !running.empty(); });
            if (stop) return;
            const int free = cfg.slots - (int)running.size();
            for (int i = 0; i < free && !queue.empty(); i++) {
                admit.push_back(std::move(queue.front()));
                queue.pop_front();
            }
        }
        std::vector<std::unique_ptr<pending>> back;   // admission refused for lack of KV pages: retried later
        for (auto& item : admit) {
            built_request br;
            if (!build(item->task, br) || item->task.max_steps < 1) {
                item->prom.set_value({});
                continue;
            }
            const gsv_ar_task& t = item->task;
            const gsvcu_sampler_cfg sc{t.sampler.top_k, t.sampler.top_p, t.sampler.temperature,
                                       t.sampler.repetition_penalty};
            const gsvcu_request req = br.view();
            const int32_t tag = next_tag++;
            const int rc = gsvcu_serve_admit(ctx, &req, 1, &sc, &t.seed, &tag, t.max_steps, t.early_stop);
            if (rc == GSVCU_OK) {
                std::lock_guard<std::mutex> lk(m);
                running.emplace(tag, std::move(item));
            } else if (rc == GSVCU_ERR_OOM && !running.empty()) {
                back.push_back(std::move(item));
            } else {   // cannot run at all (too long for the pool, invalid ids, ...)
                std::fprintf(stderr, "[gsv_ar_server] task refused: %s\n", gsvcu_last_error(ctx));
                item->prom.set_value({});
            }
        }
        if (!back.empty()) {
            std::lock_guard<std::mutex> lk(m);
            for (auto it = back.rbegin(); it != back.rend(); ++it) queue.push_front(std::move(*it));
        }
        bool any;
        {
            std::lock_guard<std::mutex> lk(m);
            any = !running.empty();
        }
        if (!any) continue;
        // token capacity: every running sequence could finish in this chunk with all its tokens
        size_t cap = 0;
        {
            std::lock_guard<std::mutex> lk(m);
            for (auto& r : running) cap += (size_t)r.second->task.max_steps + 1;
        }
        toks.resize(cap);
        const int n = gsvcu_serve_step(ctx, cfg.chunk, fin.data(), (int32_t)fin.size(), toks.data(), (int32_t)cap);
        if (n < 0) {
            std::fprintf(stderr, "[gsv_ar_server] decode failed: %s\n", gsvcu_last_error(ctx));
            std::lock_guard<std::mutex> lk(m);
            for (auto& r : running) r.second->prom.set_value({});
            running.clear();
            gsvcu_serve_reset(ctx);
            continue;
        }
        size_t off = 0;
        std::lock_guard<std::mutex> lk(m);
        for (int i = 0; i < n; i++) {
            auto it = running.find(fin[(size_t)i].tag);
            const size_t nt = (size_t)fin[(size_t)i].n_tokens;
            if (it != running.end()) {
                it->second->prom.set_value(std::vector<int32_t>(toks.begin() + (long)off, toks.begin() + (long)(off + nt)));
                running.erase(it);
                done++;
            }
            off += nt;
        }
    }
}
