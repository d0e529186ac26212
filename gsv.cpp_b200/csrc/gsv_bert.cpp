// gsv_bert.cpp -- `class gsv_bert` (the unchanged API of gsv.cpp's src/gsv_bert.h) implemented on the C
// ABI of the B200 library (gsvcu_bert_* in gsvcu.h). Replaces reference src/gsv_bert.cpp: no ggml graphs;
// the layers run on the GPU. The feature cache is the reference's host-side LRU (src/gsv_bert.cpp:241-266).
#include "gsv_bert.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "device_parse.h"
#include "gsvcu.h"

namespace {

using gsvcu::parse_device;

uint64_t hash_ids(const int32_t* ids, int T) {   // FNV-1a over the ids and T
    uint64_t h = 1469598103934665603ull;
    for (int i = 0; i < T; i++) {
        h ^= (uint32_t)ids[i];
        h *= 1099511628211ull;
    }
    h ^= (uint64_t)(uint32_t)T;
    h *= 1099511628211ull;
    return h;
}

}  // namespace

struct gsv_bert::impl {
    gsvcu_bert* ctx = nullptr;
    gsvcu_bert_hparams hp{};
    struct entry {
        uint64_t h = 0, use = 0;
        std::vector<int32_t> ids;
        std::vector<float> feat;
    };
    std::vector<entry> cache;
    int cache_n = 0, hits = 0, misses = 0;
    uint64_t clock = 0;
};

gsv_bert::gsv_bert() : p(new impl()) {}

gsv_bert::~gsv_bert() {
    if (p->ctx) gsvcu_bert_destroy(p->ctx);
    delete p;
}

int gsv_bert::hidden() const { return p->hp.hidden; }
int gsv_bert::layers_used() const { return p->hp.layers_used; }
int gsv_bert::max_pos() const { return p->hp.max_pos; }

gsv_bert* gsv_bert::load(const std::string& gguf_path, const gsv_bert_cfg& cfg) {
    int dev = 0;
    if (!parse_device(cfg.device, &dev)) {
        std::fprintf(stderr, "[gsv_bert] device '%s': this build runs on CUDA GPUs only\n", cfg.device.c_str());
        return nullptr;
    }
    gsv_bert* m = new gsv_bert();
    if (gsvcu_bert_load(dev, gguf_path.c_str(), &m->p->ctx) != GSVCU_OK) {
        std::fprintf(stderr, "[gsv_bert] failed to load %s on cuda:%d\n", gguf_path.c_str(), dev);
        delete m;
        return nullptr;
    }
    gsvcu_bert_get_hparams(m->p->ctx, &m->p->hp);
    m->p->cache_n = cfg.feat_cache > 0 ? cfg.feat_cache : 0;
    if (cfg.verbose)
        std::printf("[gsv_bert] loaded %s on cuda:%d: hidden=%d heads=%d inter=%d layers_used=%d\n",
                    gguf_path.c_str(), dev, m->p->hp.hidden, m->p->hp.n_head, m->p->hp.inter, m->p->hp.layers_used);
    return m;
}

void gsv_bert::encode(const int32_t* ids, int T, std::vector<float>& features) {
    features.assign((size_t)p->hp.hidden * (T > 0 ? T : 0), 0.0f);
    if (gsvcu_bert_encode(p->ctx, ids, T, -1, features.data()) != GSVCU_OK) {
        std::fprintf(stderr, "[gsv_bert] encode failed: %s\n", gsvcu_bert_last_error(p->ctx));
        features.clear();
    }
}

void gsv_bert::encode_feat(const int32_t* ids, int T, std::vector<float>& feat) {
    if (T - 2 <= 0) {
        feat.clear();
        return;
    }
    feat.assign((size_t)p->hp.hidden * (T - 2), 0.0f);
    if (gsvcu_bert_encode_feat_batch(p->ctx, 1, ids, &T, T, feat.data(), 0) != GSVCU_OK) {
        std::fprintf(stderr, "[gsv_bert] encode_feat failed: %s\n", gsvcu_bert_last_error(p->ctx));
        feat.clear();
    }
}

void gsv_bert::encode_feat_cached(const int32_t* ids, int T, std::vector<float>& feat) {
    impl& s = *p;
    if (s.cache_n <= 0) {
        encode_feat(ids, T, feat);
        return;
    }
    const uint64_t h = hash_ids(ids, T);
    for (impl::entry& e : s.cache)
        if (e.h == h && (int)e.ids.size() == T && std::memcmp(e.ids.data(), ids, (size_t)T * 4) == 0) {
            feat = e.feat;
            e.use = ++s.clock;
            s.hits++;
            return;
        }
    s.misses++;
    encode_feat(ids, T, feat);
    if ((int)s.cache.size() >= s.cache_n) {   // least recently used out
        size_t victim = 0;
        for (size_t i = 1; i < s.cache.size(); i++)
            if (s.cache[i].use < s.cache[victim].use) victim = i;
        s.cache.erase(s.cache.begin() + (long)victim);
    }
    impl::entry e;
    e.h = h;
    e.use = ++s.clock;
    e.ids.assign(ids, ids + T);
    e.feat = feat;
    s.cache.push_back(std::move(e));
}

void gsv_bert::feat_cache_stats(int& hits, int& misses) const {
    hits = p->hits;
    misses = p->misses;
}

bool gsv_bert::encode_feat_batch(int B, const int32_t* ids_flat, const int* lens, int Tmax,
                                 std::vector<std::vector<float>>& feats) {
    feats.assign((size_t)(B > 0 ? B : 0), {});
    if (B <= 0 || !ids_flat || !lens) return false;
    size_t total = 0;
    std::vector<int32_t> l32((size_t)B);
    for (int b = 0; b < B; b++) {
        l32[(size_t)b] = lens[b];
        if (lens[b] > 2) total += (size_t)p->hp.hidden * (lens[b] - 2);
    }
    std::vector<float> flat(total > 0 ? total : 1);
    if (gsvcu_bert_encode_feat_batch(p->ctx, B, ids_flat, l32.data(), Tmax, flat.data(), 0) != GSVCU_OK) {
        std::fprintf(stderr, "[gsv_bert] encode_feat_batch: %s\n", gsvcu_bert_last_error(p->ctx));
        return false;
    }
    size_t at = 0;
    for (int b = 0; b < B; b++) {
        if (lens[b] <= 2) continue;
        const size_t n = (size_t)p->hp.hidden * (lens[b] - 2);
        feats[(size_t)b].assign(flat.begin() + (long)at, flat.begin() + (long)(at + n));
        at += n;
    }
    return true;
}

void gsv_bert::encode_layers(const int32_t* ids, int T, std::vector<float>& features,
                             std::vector<std::vector<float>>& per_layer) {
    features.clear();
    per_layer.assign((size_t)p->hp.layers_used + 1, {});
    for (int k = 0; k <= p->hp.layers_used; k++) {
        std::vector<float> out((size_t)p->hp.hidden * (T > 0 ? T : 0));
        if (gsvcu_bert_encode(p->ctx, ids, T, k, out.data()) != GSVCU_OK) {
            std::fprintf(stderr, "[gsv_bert] encode_layers failed: %s\n", gsvcu_bert_last_error(p->ctx));
            return;
        }
        if (k == p->hp.layers_used) features = out;
        per_layer[(size_t)k] = std::move(out);
    }
}
