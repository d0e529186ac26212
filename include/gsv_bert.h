// gsv_bert.h -- the BERT feature producer (chinese-roberta-wwm-ext-large up to hidden_states[-3]) behind
// the B200 library.
//
// Drop-in for gsv.cpp's src/gsv_bert.h: the same types, members, defaults and signatures, so gsv_engine
// keeps calling it unchanged. The implementation (gsv.cpp_b200/csrc/gsv_bert.cpp) forwards to the
// gsvcu_bert_* entry points of gsvcu.h.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

struct gsv_bert_cfg {
    int n_threads = 0;        // unused by the CUDA build (kept for source compatibility)
    bool verbose = false;
    std::string device;       // "" / "cuda" / "gpu" / "vulkan" -> GPU 0; "N" or "x:N" -> GPU N; "cpu" is rejected
    int feat_cache = 0;       // entries of the encode_feat_cached LRU (0 = off)
};

class gsv_bert {
public:
    static gsv_bert* load(const std::string& gguf_path, const gsv_bert_cfg& cfg);
    ~gsv_bert();

    int hidden() const;
    int layers_used() const;
    int max_pos() const;

    // ids with [CLS] / [SEP], no padding, T <= max_pos; features [hidden][T] row-major (hidden_states[-3])
    void encode(const int32_t* ids, int T, std::vector<float>& features);
    // pipeline features without [CLS] / [SEP]: [hidden][T - 2]
    void encode_feat(const int32_t* ids, int T, std::vector<float>& feat);
    // encode_feat behind an LRU cache keyed on the ids (cfg.feat_cache entries; 0: plain encode_feat)
    void encode_feat_cached(const int32_t* ids, int T, std::vector<float>& feat);
    void feat_cache_stats(int& hits, int& misses) const;
    // B sequences of lens[b] ids each, in slots of Tmax ids in ids_flat; feats[b] = [hidden][lens[b] - 2]
    bool encode_feat_batch(int B, const int32_t* ids_flat, const int* lens, int Tmax,
                           std::vector<std::vector<float>>& feats);
    // per_layer[0] = embeddings + LayerNorm, per_layer[k] = output of layer k - 1; layers_used + 1 entries
    void encode_layers(const int32_t* ids, int T, std::vector<float>& features,
                       std::vector<std::vector<float>>& per_layer);

private:
    gsv_bert();
    struct impl;
    impl* p;
};
