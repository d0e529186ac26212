// gsv_dit.cpp -- `class gsv_dit` (the unchanged API of gsv.cpp's src/gsv_dit.h) implemented on the C ABI of
// the B200 library (gsvcu_dit_* in gsvcu.h). Replaces reference src/gsv_dit.cpp: no ggml graphs; the
// estimator, the static cache and the CFM loop run on the GPU.
#include "gsv_dit.h"

#include <cmath>
#include <cstdio>
#include <string>
#include <vector>

#include "device_parse.h"
#include "gsvcu.h"

struct gsv_dit::impl {
    gsvcu_dit* ctx = nullptr;
    gsvcu_dit_hparams hp{};
    bool verbose = false;
    // cache-dit settings (gsv_dit_cfg::dbcache_*), passed to the library whole on every change
    int db_fn = 0, db_warmup = 8, db_iv = 1, db_max_cached = -1, db_max_cont = -1, db_ds = 4;
    float db_thr = 0.08f, db_max_accum = 0.0f;
    std::vector<float> inv_freq;   // [32]

    bool ok(int rc, const char* what) {
        if (rc == GSVCU_OK) return true;
        std::fprintf(stderr, "[gsv_dit] %s: %s\n", what, gsvcu_dit_last_error(ctx));
        return false;
    }
    void push_dbcache() {
        gsvcu_dit_set_dbcache(ctx, db_fn, db_thr, db_warmup, db_iv, db_max_cached, db_max_cont, db_max_accum, db_ds);
    }
};

gsv_dit::gsv_dit() : p(new impl) {}

gsv_dit::~gsv_dit() {
    if (p->ctx) gsvcu_dit_destroy(p->ctx);
    delete p;
}

gsv_dit* gsv_dit::load(const std::string& gguf_path, const gsv_dit_cfg& cfg) {
    int dev = 0;
    if (!gsvcu::parse_device(cfg.device, &dev)) {
        std::fprintf(stderr, "[gsv_dit] device '%s': this build runs on CUDA GPUs only\n", cfg.device.c_str());
        return nullptr;
    }
    gsv_dit* m = new gsv_dit();
    if (gsvcu_dit_load(dev, gguf_path.c_str(), &m->p->ctx) != GSVCU_OK) {
        delete m;
        return nullptr;
    }
    impl& s = *m->p;
    gsvcu_dit_get_hparams(s.ctx, &s.hp);
    s.verbose = cfg.verbose;
    s.db_fn = cfg.dbcache_fn > 0 ? cfg.dbcache_fn : 0;
    s.db_thr = cfg.dbcache_threshold;
    s.db_warmup = cfg.dbcache_warmup;
    s.db_iv = cfg.dbcache_warmup_interval;
    s.db_max_cached = cfg.dbcache_max_cached;
    s.db_max_cont = cfg.dbcache_max_cont;
    s.db_max_accum = cfg.dbcache_max_accum;
    s.db_ds = cfg.dbcache_downsample >= 1 ? cfg.dbcache_downsample : 1;
    s.push_dbcache();
    s.inv_freq.assign(32, 0.0f);
    gsvcu_dit_get_inv_freq(s.ctx, s.inv_freq.data());
    gsvcu_dit_set_alg(s.ctx, cfg.alg_uncond_reuse);
    if (s.verbose)
        std::printf("[gsv_dit] loaded %s on GPU %d: dim %d, depth %d\n", gguf_path.c_str(), dev, s.hp.dim, s.hp.depth);
    return m;
}

int gsv_dit::mel_dim() const { return p->hp.mel_dim; }
int gsv_dit::dim() const { return p->hp.dim; }
int gsv_dit::depth() const { return p->hp.depth; }
int gsv_dit::cur_T() const { return cur_T_; }
int gsv_dit::cur_prompt_T() const { return cur_prompt_T_; }

bool gsv_dit::prepare(const float* prompt_mel, const float* mu, int T, int x_lens, int P) {
    if (T <= 0) return false;
    if (!p->ok(gsvcu_dit_prepare(p->ctx, prompt_mel, mu, T, x_lens), "prepare")) return false;
    cur_T_ = T;
    cur_prompt_T_ = (P <= 0 || P >= T) ? 0 : P;
    return true;
}

bool gsv_dit::velocity(const float* x_mel, float t, bool negative, float* vel) {
    return p->ok(gsvcu_dit_velocity(p->ctx, x_mel, t, negative ? 1 : 0, vel), "velocity");
}

bool gsv_dit::sample(const float* mu, const float* prompt, int P, int T, int steps, float cfg, uint64_t seed,
                     const float* x0, std::vector<float>& mel_out, int skip_steps) {
    if (T <= 0 || steps <= 0 || P <= 0 || P >= T) return false;
    mel_out.resize((size_t)p->hp.mel_dim * (T - P));
    if (!p->ok(gsvcu_dit_sample_full(p->ctx, mu, prompt, P, T, steps, cfg, seed, x0, skip_steps, mel_out.data()),
               "sample"))
        return false;
    cur_T_ = T;
    cur_prompt_T_ = P;
    return true;
}

bool gsv_dit::synthesize(const float* fea_ref, int R, const float* fea_todo, int N, const float* mel_ref,
                         int mel_ref_T, int steps, float cfg, uint64_t seed, int block_override,
                         const std::vector<const float*>* x0_chunks, std::vector<float>& mel_out, int skip_steps) {
    if (R <= 0 || N <= 0) return false;
    mel_out.resize((size_t)p->hp.mel_dim * N);
    const float* const* xc = x0_chunks ? x0_chunks->data() : nullptr;
    const int nx = x0_chunks ? (int)x0_chunks->size() : 0;
    return p->ok(gsvcu_dit_synthesize(p->ctx, fea_ref, R, fea_todo, N, mel_ref, mel_ref_T, steps, cfg, seed,
                                      block_override, xc, nx, skip_steps, mel_out.data()),
                 "synthesize");
}

void gsv_dit::time_sin(float t, float* out256) { gsvcu_dit_time_sin(t, out256); }

void gsv_dit::db_set_step(int j) { gsvcu_dit_db_set_step(p->ctx, j); }

void gsv_dit::db_get_stats(db_stats& st) const {
    int32_t steps = 0, hits[2] = {0, 0}, misses[2] = {0, 0};
    gsvcu_dit_db_get_stats(p->ctx, &steps, hits, misses, st.last_fd, st.acc);
    st.steps = steps;
    for (int b = 0; b < 2; b++) {
        st.hits[b] = hits[b];
        st.misses[b] = misses[b];
    }
}

void gsv_dit::set_dbcache(int fn, float threshold, int warmup, int downsample) {
    p->db_fn = fn > 0 ? fn : 0;
    p->db_thr = threshold;
    p->db_warmup = warmup;
    p->db_ds = downsample >= 1 ? downsample : 1;
    p->push_dbcache();
}

int gsv_dit::dbcache_fn() const { return p->db_fn; }

void gsv_dit::set_alg(const gsv_dit_alg& a) { gsvcu_dit_set_alg(p->ctx, a.uncond_reuse); }

gsv_dit_alg gsv_dit::alg() const {
    gsv_dit_alg a;
    int32_t ur = 0;
    gsvcu_dit_get_alg(p->ctx, &ur);
    a.uncond_reuse = ur;
    return a;
}

void gsv_dit::debug_tables(std::vector<float>& cos_tab, std::vector<float>& sin_tab) const {
    const int T = cur_T_;
    cos_tab.resize((size_t)32 * T);
    sin_tab.resize((size_t)32 * T);
    for (int n = 0; n < T; n++)
        for (int i = 0; i < 32; i++) {
            const float a = (float)n * p->inv_freq[(size_t)i];
            cos_tab[(size_t)i + 32 * (size_t)n] = std::cos(a);
            sin_tab[(size_t)i + 32 * (size_t)n] = std::sin(a);
        }
}

bool gsv_dit::debug_read(const char*, std::vector<float>& out) {
    out.clear();
    return false;
}
