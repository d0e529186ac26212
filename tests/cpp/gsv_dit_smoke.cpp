// gsv_dit_smoke.cpp -- exercises the drop-in `class gsv_dit` as gsv.cpp's callers do and prints its outputs
// as JSON lines (checksums of the arrays).
//   gsv_dit_smoke <dit.gguf> <in.bin>
//   in.bin: int32 T, P, R, N, MT, then f32 mu [512][T], prompt [100][P], x_mel [100][T], fea_ref [512][R],
//           fea_todo [512][N], mel_ref [100][MT]
#include <cstdio>
#include <vector>

#include "gsv_dit.h"

static double checksum(const std::vector<float>& v) {
    double s = 0.0;
    for (size_t i = 0; i < v.size(); i++) s += (double)v[i] * (double)((i % 7) + 1);
    return s;
}

static bool read(FILE* f, std::vector<float>& v, size_t n) {
    v.resize(n);
    return std::fread(v.data(), 4, n, f) == n;
}

int main(int argc, char** argv) {
    if (argc < 3) {
        std::fprintf(stderr, "usage: %s <dit.gguf> <in.bin>\n", argv[0]);
        return 2;
    }
    FILE* f = std::fopen(argv[2], "rb");
    if (!f) return 2;
    int hdr[5];
    if (std::fread(hdr, 4, 5, f) != 5) return 2;
    const int T = hdr[0], P = hdr[1], R = hdr[2], N = hdr[3], MT = hdr[4];
    std::vector<float> mu, prompt, xmel, fea_ref, fea_todo, mel_ref;
    if (!read(f, mu, (size_t)512 * T) || !read(f, prompt, (size_t)100 * P) || !read(f, xmel, (size_t)100 * T) ||
        !read(f, fea_ref, (size_t)512 * R) || !read(f, fea_todo, (size_t)512 * N) || !read(f, mel_ref, (size_t)100 * MT))
        return 2;
    std::fclose(f);
    gsv_dit_cfg cfg;
    gsv_dit* m = gsv_dit::load(argv[1], cfg);
    if (!m) return 1;
    std::printf("{\"mel_dim\": %d, \"dim\": %d, \"depth\": %d}\n", m->mel_dim(), m->dim(), m->depth());
    // prepare with the prompt in the first P frames, then both velocities
    std::vector<float> px((size_t)100 * T, 0.0f);
    for (int c = 0; c < 100; c++)
        for (int t = 0; t < P; t++) px[(size_t)c * T + t] = prompt[(size_t)c * P + t];
    if (!m->prepare(px.data(), mu.data(), T, T, P)) return 1;
    std::vector<float> vp((size_t)100 * T), vn((size_t)100 * T);
    if (!m->velocity(xmel.data(), 0.3f, false, vp.data()) || !m->velocity(xmel.data(), 0.3f, true, vn.data())) return 1;
    std::printf("{\"cur_T\": %d, \"cur_P\": %d, \"vel\": %.10e, \"vel_neg\": %.10e}\n", m->cur_T(), m->cur_prompt_T(),
                checksum(vp), checksum(vn));
    std::vector<float> mel;
    if (!m->sample(mu.data(), prompt.data(), P, T, 3, 1.3f, 5, nullptr, mel, 1)) return 1;
    gsv_dit_alg a;
    a.uncond_reuse = 1;
    m->set_alg(a);
    std::vector<float> mel_r;
    if (!m->sample(mu.data(), prompt.data(), P, T, 3, 1.3f, 5, nullptr, mel_r)) return 1;
    std::printf("{\"sample\": %.10e, \"n\": %zu, \"sample_reuse\": %.10e, \"alg\": %d}\n", checksum(mel), mel.size(),
                checksum(mel_r), m->alg().uncond_reuse);
    a.uncond_reuse = 0;
    m->set_alg(a);
    std::vector<float> syn;
    if (!m->synthesize(fea_ref.data(), R, fea_todo.data(), N, mel_ref.data(), MT, 2, 1.3f, 9, 40, nullptr, syn)) return 1;
    std::vector<float> ts(256), ct, st;
    gsv_dit::time_sin(0.25f, ts.data());
    m->debug_tables(ct, st);
    m->set_dbcache(8, 0.02f, 8, 4);
    gsv_dit::db_stats dbs;
    m->db_get_stats(dbs);
    std::vector<float> dummy;
    std::printf("{\"synth\": %.10e, \"n\": %zu, \"time_sin\": %.10e, \"tables\": %zu, \"dbcache_fn\": %d, \"hits\": %d, "
                "\"debug_read\": %d}\n",
                checksum(syn), syn.size(), checksum(ts), ct.size(), m->dbcache_fn(), dbs.hits[0],
                (int)m->debug_read("dbg_b0_out", dummy));
    delete m;
    return 0;
}
