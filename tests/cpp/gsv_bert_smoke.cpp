// gsv_bert_smoke.cpp -- exercises the drop-in `class gsv_bert` as gsv.cpp's callers do and prints its
// outputs as JSON lines (checksums of the feature arrays).
//   gsv_bert_smoke <bert.gguf> <ids.bin>      ids.bin: int32 B, Tmax, lens[B], ids[B][Tmax]
#include <cstdio>
#include <vector>

#include "gsv_bert.h"

static double checksum(const std::vector<float>& v) {
    double s = 0.0;
    for (size_t i = 0; i < v.size(); i++) s += (double)v[i] * (double)((i % 7) + 1);
    return s;
}

int main(int argc, char** argv) {
    if (argc < 3) {
        std::fprintf(stderr, "usage: %s <bert.gguf> <ids.bin>\n", argv[0]);
        return 2;
    }
    FILE* f = std::fopen(argv[2], "rb");
    if (!f) return 2;
    int B = 0, Tmax = 0;
    if (std::fread(&B, 4, 1, f) != 1 || std::fread(&Tmax, 4, 1, f) != 1) return 2;
    std::vector<int> lens((size_t)B);
    std::vector<int32_t> ids((size_t)B * Tmax);
    if (std::fread(lens.data(), 4, (size_t)B, f) != (size_t)B || std::fread(ids.data(), 4, ids.size(), f) != ids.size())
        return 2;
    std::fclose(f);
    gsv_bert_cfg cfg;
    cfg.feat_cache = 2;
    gsv_bert* m = gsv_bert::load(argv[1], cfg);
    if (!m) return 1;
    std::printf("{\"hidden\": %d, \"layers_used\": %d, \"max_pos\": %d}\n", m->hidden(), m->layers_used(), m->max_pos());
    std::vector<std::vector<float>> feats;
    if (!m->encode_feat_batch(B, ids.data(), lens.data(), Tmax, feats)) return 1;
    for (int b = 0; b < B; b++) {
        std::vector<float> one, cached;
        m->encode_feat(ids.data() + (size_t)b * Tmax, lens[(size_t)b], one);
        m->encode_feat_cached(ids.data() + (size_t)b * Tmax, lens[(size_t)b], cached);
        std::printf("{\"seq\": %d, \"n\": %zu, \"batch\": %.10e, \"single\": %.10e, \"cached\": %.10e}\n", b,
                    feats[(size_t)b].size(), checksum(feats[(size_t)b]), checksum(one), checksum(cached));
    }
    std::vector<float> again;
    m->encode_feat_cached(ids.data(), lens[0], again);   // a hit (cache of 2 holds the last two sequences
    int hits = 0, misses = 0;                             // unless B <= 2)
    m->feat_cache_stats(hits, misses);
    std::vector<float> full;
    std::vector<std::vector<float>> per_layer;
    m->encode_layers(ids.data(), lens[0], full, per_layer);
    std::printf("{\"hits\": %d, \"misses\": %d, \"layers\": %zu, \"full\": %.10e}\n", hits, misses, per_layer.size(),
                checksum(full));
    delete m;
    return 0;
}
