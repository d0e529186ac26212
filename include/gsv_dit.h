// gsv_dit.h -- the v5 DiT / CFM estimator (F5-style DiT, 22 blocks) behind the B200 library.
//
// Drop-in for gsv.cpp's src/gsv_dit.h: the same types, members, defaults and signatures, so gsv_engine and
// the synthesis scheduler keep calling it unchanged. The implementation (gsv.cpp_b200/csrc/gsv_dit.cpp)
// forwards to the gsvcu_dit_* entry points of gsvcu.h. Layouts are the reference's torch layouts
// (mel [100][T], mu [512][T], index c * T + t).
//
// Difference a caller can see: debug_read has no named intermediate tensors and returns false.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

struct gsv_dit_cfg {
    int  n_threads = 0;       // unused by the CUDA build (kept for source compatibility)
    bool verbose   = false;
    std::string device;       // "" / "gpu" / "vulkan" / "cuda" -> GPU 0; "N" or "x:N" -> GPU N; "cpu" is rejected

    // cache-dit (DBCache): fn > 0 caches the middle blocks' residual across steps behind the gates below
    int   dbcache_fn              = 0;
    float dbcache_threshold       = 0.08f;
    int   dbcache_warmup          = 8;
    int   dbcache_warmup_interval = 1;
    int   dbcache_max_cached      = -1;
    int   dbcache_max_cont        = -1;
    float dbcache_max_accum       = 0.0f;
    int   dbcache_downsample      = 4;

    // 0 = off; 1 = odd guided steps reuse the last computed unconditional velocity; 2 = odd steps
    // extrapolate 2 neg[k-1] - neg[k-2]
    int   alg_uncond_reuse = 0;
};

struct gsv_dit_alg {
    int   uncond_reuse  = 0;
};

class gsv_dit {
public:
    static gsv_dit * load(const std::string & gguf_path, const gsv_dit_cfg & cfg);
    ~gsv_dit();

    int mel_dim() const;      // 100
    int dim()     const;      // 1024
    int depth()   const;      // 22

    // the static cache: prompt_mel [mel_dim][T] (prompt frames then zeros), mu [text_dim][T], x_lens valid
    // frames (<= 0 or > T: T), P prompt frames (<= 0 or >= T: 0)
    bool prepare(const float * prompt_mel, const float * mu, int T, int x_lens, int P);
    int  cur_T() const;
    int  cur_prompt_T() const;

    // one estimator pass: x_mel [mel_dim][T] -> vel [mel_dim][T]; negative: the unconditional branch
    bool velocity(const float * x_mel, float t, bool negative, float * vel);

    // CFM.inference: mu [text_dim][T], prompt [mel_dim][P] -> mel_out [mel_dim][T - P]; x0 [mel_dim][T] or
    // null (then randn * 0.875 from gsv_rng(seed)); the first skip_steps Euler steps leave x unchanged
    bool sample(const float * mu, const float * prompt, int P, int T, int steps, float cfg,
                uint64_t seed, const float * x0, std::vector<float> & mel_out, int skip_steps = 0);

    // synthesize_v5_mel: chunks with a rolling prompt; fea_ref [512][R], fea_todo [512][N],
    // mel_ref [100][mel_ref_T] -> mel_out [100][N]
    bool synthesize(const float * fea_ref, int R, const float * fea_todo, int N,
                    const float * mel_ref, int mel_ref_T, int steps, float cfg, uint64_t seed,
                    int block_override, const std::vector<const float *> * x0_chunks,
                    std::vector<float> & mel_out, int skip_steps = 0);

    static void time_sin(float t, float * out256);

    struct db_stats {
        int   steps;
        int   hits[2];
        int   misses[2];
        float last_fd[2];
        float acc[2];
    };
    void db_set_step(int j);
    void db_get_stats(db_stats & st) const;
    void set_dbcache(int fn, float threshold, int warmup, int downsample);
    int  dbcache_fn() const;
    void set_alg(const gsv_dit_alg & a);
    gsv_dit_alg alg() const;
    // RoPE angle tables of the last prepare: cos / sin [32 * T], index i + 32 * t
    void debug_tables(std::vector<float> & cos_tab, std::vector<float> & sin_tab) const;
    bool debug_read(const char * name, std::vector<float> & out);

private:
    gsv_dit();
    struct impl;
    impl * p;
    int cur_T_ = 0;
    int cur_prompt_T_ = 0;
};
