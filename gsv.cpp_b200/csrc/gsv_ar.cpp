// gsv_ar.cpp -- `class gsv_ar` (the unchanged API of gsv.cpp's src/gsv_ar.h) implemented on the
// C ABI of the B200 library (gsvcu.h). Replaces reference src/gsv_ar.cpp: no ggml graphs; the KV
// cache, decode loop and sampler live on the GPU.
#include "gsv_ar.h"

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "device_parse.h"
#include "gsvcu.h"

#if defined(__has_include)
#if __has_include("gsv_progress.h")
#include "gsv_progress.h"
#define GSV_AR_HAVE_PROGRESS 1
#endif
#endif

namespace {

using gsvcu::parse_device;

void on_progress(void* user, int32_t steps) {
    int* last = (int*)user;
#ifdef GSV_AR_HAVE_PROGRESS
    for (int i = *last; i < steps; i++) gsvprog::tick();
#endif
    *last = steps;
}

}  // namespace

struct gsv_ar::impl {
    gsvcu_ctx* ctx = nullptr;
    gsvcu_hparams hp{};
    int prompt_len = 0;
    bool verbose = false;
};

gsv_ar::gsv_ar() : p(new impl()) {}

gsv_ar::~gsv_ar() {
    if (p->ctx) gsvcu_destroy(p->ctx);
    delete p;
}

int gsv_ar::hidden_dim() const { return p->hp.hidden_dim; }
int gsv_ar::vocab_size() const { return p->hp.vocab_size; }
int gsv_ar::eos() const { return p->hp.eos; }
int gsv_ar::bert_dim() const { return p->hp.bert_dim; }
int gsv_ar::prompt_len_expected() const { return p->prompt_len; }

gsv_ar* gsv_ar::load(const std::string& gguf_path, const gsv_ar_cfg& cfg) {
    int dev = 0;
    if (!parse_device(cfg.device, &dev)) {
        std::fprintf(stderr, "[gsv_ar] device '%s': this build runs on CUDA GPUs only\n", cfg.device.c_str());
        return nullptr;
    }
    gsv_ar* m = new gsv_ar();
    m->p->verbose = cfg.verbose;
    int rc = gsvcu_create(dev, &m->p->ctx);
    if (rc != GSVCU_OK) {
        std::fprintf(stderr, "[device] GPU %d not usable (code %d; needs an sm_100 device)\n", dev, rc);
        delete m;
        return nullptr;
    }
    rc = gsvcu_load_gguf(m->p->ctx, gguf_path.c_str());
    if (rc != GSVCU_OK) {
        std::fprintf(stderr, "[gsv_ar] failed to load %s: %s\n", gguf_path.c_str(), gsvcu_last_error(m->p->ctx));
        delete m;
        return nullptr;
    }
    gsvcu_get_hparams(m->p->ctx, &m->p->hp);
    if (cfg.verbose)
        std::printf("[gsv_ar] loaded %s on cuda:%d: D=%d head=%d layers=%d vocab=%d EOS=%d alpha=(%.4f, %.4f)\n",
                    gguf_path.c_str(), dev, m->p->hp.hidden_dim, m->p->hp.n_head, m->p->hp.n_layer,
                    m->p->hp.vocab_size, m->p->hp.eos, m->p->hp.text_pe_alpha, m->p->hp.audio_pe_alpha);
    return m;
}

static std::vector<gsvcu_request> to_c(const std::vector<gsv_ar_request>& reqs) {
    std::vector<gsvcu_request> out(reqs.size());
    for (size_t i = 0; i < reqs.size(); i++) {
        out[i].phones = reqs[i].phones.data();
        out[i].n_phones = (int32_t)reqs[i].phones.size();
        out[i].bert = reqs[i].bert.data();
        out[i].prompt = reqs[i].prompt.data();
        out[i].n_prompt = (int32_t)reqs[i].prompt.size();
    }
    return out;
}

static bool check_bert(const std::vector<gsv_ar_request>& reqs, int bert_dim) {
    for (const auto& r : reqs)
        if (r.bert.size() < (size_t)bert_dim * r.phones.size()) {
            std::fprintf(stderr, "[gsv_ar] bert has %zu values, expected %d x %zu\n", r.bert.size(), bert_dim,
                         r.phones.size());
            return false;
        }
    return true;
}

gsv_ar_result gsv_ar::generate(const std::vector<gsv_ar_request>& reqs, const gsv_sampler_cfg& sampler,
                               uint64_t seed_base, int early_stop_num, int max_steps,
                               const std::vector<int32_t>* oracle_tokens, const std::vector<uint64_t>* seeds) {
    gsv_ar_result res;
    const int B = (int)reqs.size();
    if (B == 0) return res;
    if (!check_bert(reqs, p->hp.bert_dim)) return res;
    p->prompt_len = (int)reqs[0].prompt.size();
    std::vector<gsvcu_request> cr = to_c(reqs);
    size_t maxp = 0;
    for (const auto& r : reqs) maxp = std::max(maxp, r.prompt.size());
    const int cap = (int)maxp + max_steps;
    std::vector<int32_t> toks((size_t)B * cap), ntok(B), lens(B);
    const gsvcu_sampler_cfg sc{sampler.top_k, sampler.top_p, sampler.temperature, sampler.repetition_penalty};
    int last = 0;
#ifdef GSV_AR_HAVE_PROGRESS
    gsvprog::begin(2, max_steps);
#endif
    const int rc = gsvcu_generate(p->ctx, cr.data(), B, &sc, seed_base, early_stop_num, max_steps,
                                  oracle_tokens ? oracle_tokens->data() : nullptr,
                                  oracle_tokens ? (int32_t)oracle_tokens->size() : 0, seeds ? seeds->data() : nullptr,
                                  seeds ? (int32_t)seeds->size() : 0, toks.data(), ntok.data(), lens.data(), cap,
                                  on_progress, &last);
    if (rc != GSVCU_OK) {
        std::fprintf(stderr, "[gsv_ar] generate failed: %s\n", gsvcu_last_error(p->ctx));
        return res;
    }
    res.tokens.resize(B);
    for (int b = 0; b < B; b++)
        res.tokens[b].assign(toks.begin() + (size_t)b * cap, toks.begin() + (size_t)b * cap + std::min(ntok[b], cap));
    res.lens.assign(lens.begin(), lens.end());
    return res;
}

void gsv_ar::first_logits(const std::vector<gsv_ar_request>& reqs, std::vector<float>& logits_out) {
    if (reqs.empty()) return;
    if (!check_bert(reqs, p->hp.bert_dim)) return;
    if (p->prompt_len == 0) p->prompt_len = (int)reqs[0].prompt.size();
    std::vector<gsvcu_request> cr = to_c(reqs);
    logits_out.assign((size_t)reqs.size() * p->hp.vocab_size, 0.0f);
    if (gsvcu_first_logits(p->ctx, cr.data(), (int32_t)reqs.size(), logits_out.data()) != GSVCU_OK)
        std::fprintf(stderr, "[gsv_ar] first_logits failed: %s\n", gsvcu_last_error(p->ctx));
}

void gsv_ar::release_cache() {
    if (p && p->ctx) gsvcu_release_cache(p->ctx);
}
