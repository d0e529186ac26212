// engine.cu -- the gsvcu context: model upload, paged KV manager, prefill, the CUDA-graph decode
// step, generate (gsv_ar::generate semantics) and the continuous-batching entry points.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/gsvcu.h"
#include "gguf_reader.h"
#include "kernels.h"

using namespace gsvcu;

namespace {

struct LayerW {
    int mt[4] = {8, 8, 8, 8};   // qkv, out, ffn1, ffn2: 8 Q8_0 kernels (Q8_0 / Q4_0 / Q5_0 / IQ4_NL), 0 F32,
                                //   1 F16, 30 BF16 (k_gemm_fx), 3 Q4_1 / Q5_1 (k_gemm_qm), 12 K-quants (k_gemm_qk)
    uint16_t* wm[4] = {nullptr, nullptr, nullptr, nullptr};  // Q4_1 / Q5_1: fp16 m planes (d in wd); K-quants: dmin
    uint8_t* wmins[4] = {nullptr, nullptr, nullptr, nullptr};  // Q4_K / Q5_K: sub-block mins
    uint4* wq[4] = {nullptr, nullptr, nullptr, nullptr};     // Q8_0: fragment planes
    uint16_t* wd[4] = {nullptr, nullptr, nullptr, nullptr};  //       matching fp16 scale planes
    __half* w16[4] = {nullptr, nullptr, nullptr, nullptr};   //       the integers as fp16 [N][K] (tcgen05 prefill)
    const void* wf[4] = {nullptr, nullptr, nullptr, nullptr};  // F32 / F16: the GGUF rows [N][K] as stored
    float *b_qkv = nullptr, *b_out = nullptr, *n1w = nullptr, *n1b = nullptr;
    float *b_f1 = nullptr, *b_f2 = nullptr, *n2w = nullptr, *n2b = nullptr;
};

constexpr int PE_MAX = 8192;          // positional table rows (reference: 4096, src/gsv_ar.cpp:44)
constexpr int PREFILL_ROWS = 16384;   // rows of one prefill pass
constexpr int STEP_CHUNK = 16;        // decode steps between host status reads in generate
constexpr int GRAPH_CHUNK = 16;       // decode steps captured in one graph (no launch gap between them)
constexpr int TC_MIN_ROWS = 128;      // prefill rows from which the Q8_0 GEMMs run on tcgen05

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

// xorshift64 (without the output multiplier) as a 64x64 GF(2) matrix: column b = image of bit b.
struct Gf2 {
    uint64_t c[64];
};
uint64_t xs_step_h(uint64_t s) {
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    return s;
}
uint64_t gf2_apply(const Gf2& m, uint64_t v) {
    uint64_t r = 0;
    for (int b = 0; b < 64; b++)
        if ((v >> b) & 1ull) r ^= m.c[b];
    return r;
}
Gf2 gf2_mul(const Gf2& a, const Gf2& b) {   // a after b
    Gf2 r;
    for (int i = 0; i < 64; i++) r.c[i] = gf2_apply(a, b.c[i]);
    return r;
}
Gf2 gf2_identity() {
    Gf2 r;
    for (int i = 0; i < 64; i++) r.c[i] = 1ull << i;
    return r;
}
Gf2 gf2_pow(Gf2 base, uint64_t e) {
    Gf2 r = gf2_identity();
    while (e) {
        if (e & 1) r = gf2_mul(base, r);
        base = gf2_mul(base, base);
        e >>= 1;
    }
    return r;
}
// Jump matrices T^(j * dpl), j = 0..31, for the sampler's lane-parallel draws.
std::vector<uint64_t> jump_matrices(int dpl) {
    Gf2 T;
    for (int b = 0; b < 64; b++) T.c[b] = xs_step_h(1ull << b);
    const Gf2 step = gf2_pow(T, (uint64_t)dpl);
    std::vector<uint64_t> jm(32 * 64);
    Gf2 cur = gf2_identity();
    for (int j = 0; j < 32; j++) {
        std::memcpy(jm.data() + (size_t)j * 64, cur.c, 64 * 8);
        cur = gf2_mul(step, cur);
    }
    return jm;
}

// ------------------------------------------------------------------ model validation
// Checks the GGUF against what gsv_ar::load binds (src/gsv_ar.cpp:571-662): KV hyper-parameters,
// every tensor name, shape and type (attention/FFN Q8_0, the rest F32, src/gsv_ar.cpp:632-637).
struct ModelView {
    gsvcu_hparams hp{};
    const GgufTensor *te = nullptr, *ae = nullptr, *bp = nullptr, *bb = nullptr, *ta = nullptr, *aa = nullptr,
                     *pr = nullptr;
    std::vector<const GgufTensor*> mats, vecs;   // [layer][4], [layer][8]
};

const char* kMatNames[4] = {"qkv_w", "out_w", "ffn1_w", "ffn2_w"};

// ggml types run by the Q8_0 kernels: Q8_0 itself, and Q4_0 / Q5_0 / IQ4_NL repacked into Q8_0 blocks
bool q8_class(uint32_t type) { return type == 8 || type == 2 || type == 6 || type == 20; }

// IQ4_NL's 16 values of a 4-bit code (ggml kvalues_iq4nl; part of the GGUF format)
constexpr int8_t kIq4nl[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

// Q4_0 / Q5_0 / IQ4_NL blocks (ggml block_q4_0 / block_q5_0 / block_iq4_nl: fp16 d; Q5_0 then the 32
// fifth bits as a little-endian uint32; then 16 bytes whose low nibbles are values 0..15 and high
// nibbles values 16..31) as Q8_0 blocks holding the same signed values (nibble - 8, five-bit value - 16,
// kIq4nl[nibble]) and the same d. ggml's dot of these types against Q8_0 activations is an integer
// block dot scaled by d_w * d_x, so on these blocks it is the Q8_0 block dot.
// Q4_1 / Q5_1 blocks (ggml block_q4_1 / block_q5_1: fp16 d, m; Q5_1 then the fifth bits as a
// little-endian uint32; then 16 bytes of nibbles, values 0..15 low, 16..31 high) as k_gemm_qm's planes:
// the unsigned values as bytes [N][K], d and m as fp16 [N][K/32] each.
void unpack_q_1(const GgufTensor* t, std::vector<uint8_t>& q, std::vector<uint16_t>& d, std::vector<uint16_t>& mn) {
    const size_t bs = t->type == 7 ? 24 : 20, nb = t->nbytes / bs;
    q.resize(nb * 32);
    d.resize(nb);
    mn.resize(nb);
    for (size_t b = 0; b < nb; b++) {
        const uint8_t* src = t->data + b * bs;
        std::memcpy(&d[b], src, 2);
        std::memcpy(&mn[b], src + 2, 2);
        const uint8_t* qs = src + (t->type == 7 ? 8 : 4);
        uint32_t qh = 0;
        if (t->type == 7) std::memcpy(&qh, src + 4, 4);
        for (int j = 0; j < 16; j++) {
            q[b * 32 + j] = (uint8_t)((qs[j] & 15) | (((qh >> j) & 1u) << 4));
            q[b * 32 + j + 16] = (uint8_t)((qs[j] >> 4) | (((qh >> (j + 16)) & 1u) << 4));
        }
    }
}

// K-quant blocks as k_gemm_qk's planes: per 256-value super-block the values times their sub-block
// scale as int16, lane-major (value e at (e % 8) * 32 + e / 8), d and dmin fp16, the 8 sub-block mins.
// block_q4_K {fp16 d, dmin; u8 scales[12]; u8 qs[128]} / block_q5_K {d, dmin, scales[12], u8 qh[32],
// qs[128]}: 8 sub-blocks of 32 with 6-bit scale and min (scale j < 4: scales[j] & 63, min scales[j+4] &
// 63; j >= 4: scale (scales[j+4] & 15) | (scales[j-4] >> 6) << 4, min (scales[j+4] >> 4) | (scales[j] >> 6)
// << 4); value 64g + 32h + l = nibble h of qs[32g + l] (+ 16 * bit 2g + h of qh[l] for Q5_K).
// block_q6_K {u8 ql[128]; u8 qh[64]; i8 scales[16]; fp16 d}: value 128h + 32k + l = (nibble k / 2 of
// ql[64h + 32(k & 1) + l] | bits 2k, 2k+1 of qh[32h + l] << 4) - 32, scale scales[value / 16].
void unpack_kquant(const GgufTensor* t, std::vector<int16_t>& w, std::vector<uint16_t>& d, std::vector<uint16_t>& dmin,
                   std::vector<uint8_t>& mins) {
    const size_t bs = t->type == 12 ? 144 : t->type == 13 ? 176 : 210, nsb = t->nbytes / bs;
    w.assign(nsb * 256, 0);
    d.assign(nsb, 0);
    dmin.assign(nsb, 0);
    mins.assign(nsb * 8, 0);
    for (size_t b = 0; b < nsb; b++) {
        const uint8_t* src = t->data + b * bs;
        int16_t* dst = w.data() + b * 256;
        int val[256], scl[256];
        if (t->type == 14) {
            std::memcpy(&d[b], src + 208, 2);
            for (int hh = 0; hh < 2; hh++)
                for (int k = 0; k < 4; k++)
                    for (int l = 0; l < 32; l++) {
                        const int e = 128 * hh + 32 * k + l;
                        const uint8_t lo = src[64 * hh + 32 * (k & 1) + l];
                        const int nib = k < 2 ? (lo & 15) : (lo >> 4);
                        val[e] = (nib | (((src[128 + 32 * hh + l] >> (2 * k)) & 3) << 4)) - 32;
                        scl[e] = (int8_t)src[192 + e / 16];
                    }
        } else {
            std::memcpy(&d[b], src, 2);
            std::memcpy(&dmin[b], src + 2, 2);
            const uint8_t* s = src + 4;
            int sc[8];
            for (int j = 0; j < 8; j++) {
                sc[j] = j < 4 ? (s[j] & 63) : ((s[j + 4] & 15) | ((s[j - 4] >> 6) << 4));
                mins[b * 8 + j] = (uint8_t)(j < 4 ? (s[j + 4] & 63) : ((s[j + 4] >> 4) | ((s[j] >> 6) << 4)));
            }
            const uint8_t* qh = src + 16;
            const uint8_t* qs = src + (t->type == 12 ? 16 : 48);
            for (int g = 0; g < 4; g++)
                for (int h = 0; h < 2; h++)
                    for (int l = 0; l < 32; l++) {
                        const int e = 64 * g + 32 * h + l;
                        int q = h ? (qs[32 * g + l] >> 4) : (qs[32 * g + l] & 15);
                        if (t->type == 13) q += ((qh[l] >> (2 * g + h)) & 1) * 16;
                        val[e] = q;
                        scl[e] = sc[e / 32];
                    }
        }
        for (int e = 0; e < 256; e++) dst[(e % 8) * 32 + e / 8] = (int16_t)(val[e] * scl[e]);
    }
}

// fp16 bit pattern of a small integer (|v| <= 128: exact)
uint16_t i8_as_f16_bits(int8_t v) {
    if (v == 0) return 0;
    const uint32_t a = (uint32_t)(v < 0 ? -(int)v : (int)v);
    int e = 31 - __builtin_clz(a);                        // a = 1.m * 2^e, e <= 7
    const uint32_t mant = (a << (10 - e)) & 0x3ffu;
    return (uint16_t)((v < 0 ? 0x8000u : 0u) | ((uint32_t)(e + 15) << 10) | mant);
}

std::vector<uint8_t> to_q8_0_blocks(const GgufTensor* t) {
    const size_t bs = t->type == 6 ? 22 : 18, nb = t->nbytes / bs;
    std::vector<uint8_t> out(nb * 34);
    for (size_t b = 0; b < nb; b++) {
        const uint8_t* src = t->data + b * bs;
        uint8_t* dst = out.data() + b * 34;
        dst[0] = src[0];
        dst[1] = src[1];
        int8_t* q = (int8_t*)(dst + 2);
        if (t->type == 2) {
            for (int j = 0; j < 16; j++) {
                q[j] = (int8_t)((src[2 + j] & 15) - 8);
                q[j + 16] = (int8_t)((src[2 + j] >> 4) - 8);
            }
        } else if (t->type == 20) {
            for (int j = 0; j < 16; j++) {
                q[j] = kIq4nl[src[2 + j] & 15];
                q[j + 16] = kIq4nl[src[2 + j] >> 4];
            }
        } else {
            uint32_t qh;
            std::memcpy(&qh, src + 2, 4);
            for (int j = 0; j < 16; j++) {
                q[j] = (int8_t)(((src[6 + j] & 15) | (((qh >> j) & 1u) << 4)) - 16);
                q[j + 16] = (int8_t)(((src[6 + j] >> 4) | (((qh >> (j + 16)) & 1u) << 4)) - 16);
            }
        }
    }
    return out;
}
const char* kVecNames[8] = {"qkv_b", "out_b", "norm1_w", "norm1_b", "ffn1_b", "ffn2_b", "norm2_w", "norm2_b"};

int validate_model(const GgufFile& f, ModelView& mv, std::string& err) {
    uint32_t v = 0;
    auto kv = [&](const char* k, int def) { return f.get_u32(k, v) ? (int)v : def; };
    gsvcu_hparams& hp = mv.hp;
    hp.hidden_dim = kv("ar.hidden_dim", 512);
    hp.n_head = kv("ar.head", 16);
    hp.n_layer = kv("ar.n_layer", 24);
    hp.vocab_size = kv("ar.vocab_size", 1025);
    hp.phoneme_vocab_size = kv("ar.phoneme_vocab_size", 732);
    hp.eos = kv("ar.eos", 1024);
    hp.bert_dim = 1024;
    hp.head_dim = hp.n_head > 0 ? hp.hidden_dim / hp.n_head : 0;
    hp.ffn_dim = 4 * hp.hidden_dim;
    if (hp.hidden_dim != D || hp.n_head != NH) {
        err = "unsupported AR dims: hidden " + std::to_string(hp.hidden_dim) + ", heads " + std::to_string(hp.n_head) +
              " (this build: 512 x 16)";
        return GSVCU_ERR_FORMAT;
    }
    if (hp.n_layer < 1 || hp.n_layer > 64 || hp.vocab_size < 2 || hp.vocab_size > 1280 || hp.eos < 0 ||
        hp.eos >= hp.vocab_size || hp.phoneme_vocab_size < 1) {
        err = "AR hyper-parameters out of range";
        return GSVCU_ERR_FORMAT;
    }
    const int NL = hp.n_layer, V = hp.vocab_size, PV = hp.phoneme_vocab_size, BD = hp.bert_dim;
    // accepted ggml types: 0 = F32, 1 = F16, 2 = Q4_0, 3 = Q4_1, 6 = Q5_0, 7 = Q5_1, 8 = Q8_0, 12 = Q4_K,
    // 13 = Q5_K, 14 = Q6_K, 20 = IQ4_NL, 30 = BF16
    auto need = [&](const std::string& name, std::vector<uint32_t> types, std::vector<int64_t> dims,
                    const GgufTensor** out) -> int {
        const GgufTensor* t = f.tensor(name);
        if (!t) { err = "missing tensor " + name; return GSVCU_ERR_FORMAT; }
        if (std::find(types.begin(), types.end(), t->type) == types.end()) {
            std::string want;
            for (uint32_t ty : types) want += (want.empty() ? "" : " or ") + std::to_string(ty);
            err = "tensor " + name + " has ggml type " + std::to_string(t->type) + ", expected " + want +
                  " (0 F32, 1 F16, 2 Q4_0, 3 Q4_1, 6 Q5_0, 7 Q5_1, 8 Q8_0, 12 Q4_K, 13 Q5_K, 14 Q6_K, 20 IQ4_NL, 30 BF16)";
            return GSVCU_ERR_FORMAT;
        }
        int64_t ne = 1, ne_want = 1;
        for (int64_t d : t->dims) ne *= d;
        for (int64_t d : dims) ne_want *= d;
        if (ne != ne_want || t->dims[0] != dims[0] || !t->data) {
            err = "tensor " + name + " has unexpected shape";
            return GSVCU_ERR_FORMAT;
        }
        *out = t;
        return GSVCU_OK;
    };
    int r;
    // embeddings: F32, or F16 / BF16 (exporter --spec emb=f16 / bf16) widened to F32 on load; predict and
    // layer matrices: F32, F16, BF16, Q8_0, Q4_0, Q4_1, Q5_0, Q5_1, IQ4_NL, Q4_K, Q5_K or Q6_K (--spec
    // predict=.., attn=.., ffn=..)
    if ((r = need("ar.text_emb", {0, 1, 30}, {D, PV}, &mv.te)) ||
        (r = need("ar.audio_emb", {0, 1, 30}, {D, V}, &mv.ae)) ||
        (r = need("ar.bert_proj", {0}, {BD, D}, &mv.bp)) || (r = need("ar.bert_proj_b", {0}, {D}, &mv.bb)) ||
        (r = need("ar.text_pe_alpha", {0}, {1}, &mv.ta)) || (r = need("ar.audio_pe_alpha", {0}, {1}, &mv.aa)) ||
        (r = need("ar.predict", {0, 8, 1, 2, 3, 6, 7, 12, 13, 14, 20, 30}, {D, V}, &mv.pr)))
        return r;
    std::memcpy(&hp.text_pe_alpha, mv.ta->data, 4);
    std::memcpy(&hp.audio_pe_alpha, mv.aa->data, 4);
    const int NK[4][2] = {{3 * D, D}, {D, D}, {FF, D}, {D, FF}};
    const int VL[8] = {3 * D, D, D, D, FF, D, D, D};
    mv.mats.assign((size_t)NL * 4, nullptr);
    mv.vecs.assign((size_t)NL * 8, nullptr);
    for (int li = 0; li < NL; li++) {
        const std::string pfx = "transformer.block" + std::to_string(li) + ".";
        for (int m = 0; m < 4; m++)
            if ((r = need(pfx + kMatNames[m], {8, 0, 1, 2, 3, 6, 7, 12, 13, 14, 20, 30}, {NK[m][1], NK[m][0]},
                          &mv.mats[(size_t)li * 4 + m])))
                return r;
        // FFN1's epilogue produces what FFN2 reads: Q8_0 blocks for a Q8_0-class ffn2_w, floats otherwise
        // (F32 / F16 / BF16, and Q4_1 / Q5_1 / K-quants, whose kernels quantize their float rows to Q8_1 /
        // Q8_K themselves)
        if (q8_class(mv.mats[(size_t)li * 4 + 2]->type) != q8_class(mv.mats[(size_t)li * 4 + 3]->type)) {
            err = pfx + "ffn1_w / ffn2_w: both Q8_0 / Q4_0 / Q5_0 / IQ4_NL or both F32 / F16 / BF16 / Q4_1 / Q5_1 / "
                        "K-quants (the exporter's ffn group) expected";
            return GSVCU_ERR_FORMAT;
        }
        for (int k = 0; k < 8; k++)
            if ((r = need(pfx + kVecNames[k], {0}, {VL[k]}, &mv.vecs[(size_t)li * 8 + k]))) return r;
    }
    return GSVCU_OK;
}

}  // namespace

struct gsvcu_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    std::string err;

    int fail(int code, const std::string& msg) {
        err = msg;
        return code;
    }

    // ------------------------------------------------------------ model
    std::vector<void*> wallocs;
    bool loaded = false;
    gsvcu_hparams hp{};
    std::vector<LayerW> L;
    float *predict = nullptr, *bert_aug = nullptr, *text_emb = nullptr, *audio_emb = nullptr, *pe = nullptr;
    // Q8_0 predict: packed like the layer matrices, rows padded with zero blocks to V_pad (multiple of 32)
    bool predict_q8 = false;
    int V_pad = 0;
    uint4* predict_wq = nullptr;
    uint16_t* predict_wd = nullptr;
    const void* predict_fx = nullptr;   // F16 / BF16 predict [V][D], or Q4_1 / Q5_1 values (gemm_fx.cu)
    int predict_fx_type = FX_F16;
    uint16_t *predict_qd = nullptr, *predict_qm = nullptr;   // Q4_1 / Q5_1 predict: d, m (K-quants: d, dmin)
    uint8_t* predict_mins = nullptr;                          // Q4_K / Q5_K predict: sub-block mins
    // layer matrices: all Q8_0 (the fused decode step needs that), any F32 / F16 FFN (needs hf)
    bool all_q8 = true, ffn_float = false, any_qx = false;
    float* hf = nullptr;                 // F32 / F16 FFN: relu(W1 n1 + b1) rows [Mmax][FF]
    // K-quant / Q4_1 / Q5_1 matrices: rows quantized to Q8_K or Q8_1 [Mmax][FF], their d [Mmax][FF/32],
    // sums of 16 or s [Mmax][FF/16]
    int8_t* qx_q = nullptr;
    float* qx_d = nullptr;
    void* qx_s = nullptr;
    int launch_logits(const float* xr, int M, int8_t* xq_s, uint16_t* xd_s, float* out, cudaStream_t s);
    // the four GEMMs of layer li over rows [r0, r0 + M) (Q8_0 or F32 / F16 per matrix); kv: K/V store of QKV
    struct LayerIO {
        const float *x, *attn, *n1;        // F32 inputs (x also the out-proj residual)
        const int8_t *xq, *aq, *n1q;       // Q8_0 inputs and their scales
        const uint16_t *xd, *ad, *n1d;
        float *qkv, *pre;
    };
    void layer_gemm(int li, int m, const LayerIO& io, int M, const KvWrite& kv, cudaStream_t s);
    uint64_t* jump = nullptr;
    int dpl = 0;

    // ------------------------------------------------------------ cache / slots
    std::vector<void*> callocs;
    bool reserved = false;
    int max_slots = 0, max_ctx = 0, kv_f32 = 0, max_pages = 0, n_pages = 0;
    void* pool = nullptr;
    int32_t* block_table = nullptr;
    std::vector<int32_t> h_bt;
    std::vector<int> free_pages;
    SlotState* st = nullptr;
    std::vector<SlotState> h_st;
    std::vector<char> slot_used;
    std::vector<std::vector<int>> slot_pages;
    std::vector<int> slot_tag;
    uint16_t* counts = nullptr;
    int32_t* hist = nullptr;
    int32_t* out_tokens = nullptr;
    int tok_cap = 0;
    int32_t* forced = nullptr;
    int forced_cap = 0;
    float* logits = nullptr;
    int Mmax = 0;
    float *x = nullptr, *qkv = nullptr, *pre = nullptr, *n1 = nullptr, *attn_f32 = nullptr;
    int8_t *xq = nullptr, *aq = nullptr, *n1q = nullptr, *hq = nullptr;
    uint16_t *xd = nullptr, *ad = nullptr, *n1d = nullptr, *hd = nullptr;
    float* part = nullptr;
    int max_chunks = 0;
    int4* work = nullptr;          // the decode step's (slot, page) list and its group offsets
    int32_t* work_base = nullptr;
    // prefill staging
    int32_t *p_ids = nullptr, *p_pepos = nullptr, *p_istext = nullptr, *p_tslot = nullptr, *p_tpos = nullptr,
            *p_rowT = nullptr, *p_sstart = nullptr, *p_slen = nullptr, *p_tlen = nullptr, *p_last = nullptr,
            *p_slots = nullptr;
    int64_t* p_rowoff = nullptr;
    PrefillTile* p_tiles = nullptr;
    float *p_feat = nullptr, *p_xl = nullptr, *p_lg = nullptr;
    size_t feat_cap = 0;

    // ------------------------------------------------------------ decode graph
    cudaGraphExec_t graph = nullptr;         // one decode step
    cudaGraphExec_t graph_chunk = nullptr;   // GRAPH_CHUNK decode steps in one graph
    void drop_graphs() {
        if (graph) cudaGraphExecDestroy(graph);
        if (graph_chunk) cudaGraphExecDestroy(graph_chunk);
        graph = graph_chunk = nullptr;
    }
    int capture_steps(int n, cudaGraphExec_t* out);
    gsvcu_sampler_cfg cfg{15, 1.0f, 1.0f, 1.35f};
    int64_t tokens_done = 0;   // generated tokens of finished sequences (serving)
    int64_t launches = 0;      // kernels launched by this context (graph replays count their kernels)
    int graph_kernels = 0;     // kernels in one captured decode step
    // step profiler: events between kernel classes of an instrumented step
    cudaEvent_t prof_ev[2] = {nullptr, nullptr};
    float* prof_ms = nullptr;  // accumulators [GSVCU_PROF_CLASSES] while profiling, else null

    // op-entry scratch
    float* op_part = nullptr;
    size_t op_part_n = 0;
    void* op_a16 = nullptr;   // scratch of gsvcu_op_q8_gemm_tc (bytes)
    size_t op_a16_n = 0;
    // set when a bounded wait in a kernel gave up: [0] decode attention in the decode steps (read and
    // cleared with the slot state), [1] gsvcu_op_decode_attention (read and cleared by gsvcu_sync),
    // [2] the tcgen05 prefill GEMM (read and cleared at the end of each prefill pass)
    int32_t* att_err = nullptr;
    // test-only fault injection (gsvcu_set_wait_fault): extra bytes each K/V page wait expects, poll limit
    uint32_t fault_extra_tx = 0, fault_poll_limit = 0;
    // prefill GEMMs of Q8_0 matrices on the tcgen05 tensor cores (gemm_tc.cu) from TC_MIN_ROWS rows on
    // (gsvcu_set_prefill_gemm; the default: measured on B200 1.4x faster than the mma.sync tiles at 4096
    // rows); a16: the scratch of its activation side
    bool tc_prefill = true;
    void* a16 = nullptr;
    size_t a16_n = 0;
    // decode steps run the fused layer tail (dense.cu) when the device can hold its cluster
    bool dense_ok = false, fused = true;
    bool two_groups = false;   // fused step: split the slots into two groups on forked streams (mode 2)
    // serving lookahead: gsvcu_serve_step leaves the next chunk of steps running when it returns
    bool lookahead = false, inflight = false;
    // two slot groups run their layer chains on these streams, so one group's layer tail overlaps the
    // other group's attention (fork/join events inside the captured step)
    cudaStream_t gstream[2] = {nullptr, nullptr};
    cudaEvent_t gevent[3] = {nullptr, nullptr, nullptr};

    ~gsvcu_ctx();
    int load(const char* path);
    void free_cache();
    int reserve(int slots, int ctx, int kvd);
    int ensure(int need_slots, int need_ctx, int kvd);
    int set_cfg(const gsvcu_sampler_cfg& c);
    int admit(const gsvcu_request* reqs, int n, const uint64_t* seeds, const int32_t* tags, int max_steps,
              int early_stop, bool one_group, const int32_t* forced_tok, int n_forced, bool forced_per_seq,
              std::vector<int>& slots_out, float* dump);
    int prefill_pass(const int* slots, const gsvcu_request* reqs, int n, float* dump, int dump_b0, int dump_B);
    int launch_step(cudaStream_t s, float* dump = nullptr, int dump_row = 0, const int* dump_slots = nullptr,
                    int dump_B = 0);
    int run_steps(int n);
    int read_status();
    void release_slot(int slot);
    int alloc_dev(void** p, size_t bytes, std::vector<void*>& owner) {
        cudaError_t e = cudaMalloc(p, bytes);
        if (e != cudaSuccess) {
            cudaGetLastError();
            *p = nullptr;
            return fail(GSVCU_ERR_OOM, "cudaMalloc(" + std::to_string(bytes) + ") failed: " + cudaGetErrorString(e));
        }
        owner.push_back(*p);
        return GSVCU_OK;
    }
};

#define CK(call)                                                                                        \
    do {                                                                                                \
        cudaError_t e_ = (call);                                                                        \
        if (e_ != cudaSuccess) return fail(GSVCU_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)
#define CKC(ctx, call)                                                                                  \
    do {                                                                                                \
        cudaError_t e_ = (call);                                                                        \
        if (e_ != cudaSuccess)                                                                          \
            return (ctx)->fail(GSVCU_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_));     \
    } while (0)
#define TRY(expr)                      \
    do {                               \
        int r_ = (expr);               \
        if (r_ != GSVCU_OK) return r_; \
    } while (0)

gsvcu_ctx::~gsvcu_ctx() {
    DeviceGuard g(device);
    free_cache();
    for (void* p : wallocs) cudaFree(p);
    if (op_part) cudaFree(op_part);
    if (op_a16) cudaFree(op_a16);
    if (att_err) cudaFree(att_err);
    for (cudaStream_t gs : gstream)
        if (gs) cudaStreamDestroy(gs);
    for (cudaEvent_t ge : gevent)
        if (ge) cudaEventDestroy(ge);
    for (cudaEvent_t e : prof_ev)
        if (e) cudaEventDestroy(e);
    if (stream) cudaStreamDestroy(stream);
}

// ------------------------------------------------------------------ model load (src/gsv_ar.cpp:490-705)
int gsvcu_ctx::load(const char* path) {
    GgufFile f;
    std::string e;
    if (!f.open(path, e)) return fail(GSVCU_ERR_IO, e);
    ModelView mv;
    const int vr = validate_model(f, mv, e);
    if (vr != GSVCU_OK) return fail(vr, e);
    hp = mv.hp;
    const int NL = hp.n_layer, V = hp.vocab_size, BD = hp.bert_dim;
    auto upload = [&](const void* src, size_t bytes, void** dst) -> int {
        TRY(alloc_dev(dst, bytes, wallocs));
        CK(cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice));
        return GSVCU_OK;
    };
    auto upload_emb = [&](const GgufTensor* t, float** dst) -> int {   // F16 / BF16 tables widened exactly
        if (t->type == 0) return upload(t->data, t->nbytes, (void**)dst);
        const size_t n = t->nbytes / 2;
        std::vector<float> f32(n);
        const __half* h = (const __half*)t->data;
        const uint16_t* b = (const uint16_t*)t->data;
        for (size_t i = 0; i < n; i++) {
            if (t->type == 1) {
                f32[i] = __half2float(h[i]);
            } else {   // BF16: the upper half of the F32 bits
                const uint32_t bits = (uint32_t)b[i] << 16;
                std::memcpy(&f32[i], &bits, 4);
            }
        }
        return upload(f32.data(), n * 4, (void**)dst);
    };
    TRY(upload_emb(mv.te, &text_emb));
    TRY(upload_emb(mv.ae, &audio_emb));
    if (mv.pr->type == 1 || mv.pr->type == 30) {   // F16 / BF16 predict, evaluated by gemm_fx
        predict_q8 = false;
        predict_fx_type = mv.pr->type == 1 ? FX_F16 : FX_BF16;
        TRY(upload(mv.pr->data, mv.pr->nbytes, (void**)&predict_fx));
    } else if (mv.pr->type == 12 || mv.pr->type == 13 || mv.pr->type == 14) {   // K-quant predict (k_gemm_qk)
        predict_q8 = false;
        predict_fx_type = FX_QK;
        std::vector<int16_t> kw;
        std::vector<uint16_t> kd, kdm;
        std::vector<uint8_t> kmn;
        unpack_kquant(mv.pr, kw, kd, kdm, kmn);
        TRY(upload(kw.data(), kw.size() * 2, (void**)&predict_fx));
        TRY(upload(kd.data(), kd.size() * 2, (void**)&predict_qd));
        if (mv.pr->type != 14) {
            TRY(upload(kdm.data(), kdm.size() * 2, (void**)&predict_qm));
            TRY(upload(kmn.data(), kmn.size(), (void**)&predict_mins));
        }
    } else if (mv.pr->type == 3 || mv.pr->type == 7) {   // Q4_1 / Q5_1 predict (k_gemm_qm)
        predict_q8 = false;
        predict_fx_type = FX_QM;
        std::vector<uint8_t> q;
        std::vector<uint16_t> qd, qm;
        unpack_q_1(mv.pr, q, qd, qm);
        TRY(upload(q.data(), q.size(), (void**)&predict_fx));
        TRY(upload(qd.data(), qd.size() * 2, (void**)&predict_qd));
        TRY(upload(qm.data(), qm.size() * 2, (void**)&predict_qm));
    } else if (q8_class(mv.pr->type)) {   // Q8_0 predict (Q4_0 / Q5_0 / IQ4_NL as Q8_0 blocks)
        predict_q8 = true;
        V_pad = (V + 31) / 32 * 32;
        std::vector<uint8_t> raw((size_t)V_pad * (D / QK) * 34, 0);   // zero blocks: scale 0, quants 0
        if (mv.pr->type == 8) std::memcpy(raw.data(), mv.pr->data, (size_t)V * (D / QK) * 34);
        else {
            const std::vector<uint8_t> b = to_q8_0_blocks(mv.pr);
            std::memcpy(raw.data(), b.data(), b.size());
        }
        std::vector<uint8_t> pq((size_t)V_pad * D);
        std::vector<uint16_t> pd((size_t)V_pad * D / QK);
        pack_q8_0_host(raw.data(), V_pad, D, pq.data(), pd.data());
        TRY(upload(pq.data(), pq.size(), (void**)&predict_wq));
        TRY(upload(pd.data(), pd.size() * 2, (void**)&predict_wd));
    } else {
        predict_q8 = false;
        TRY(upload(mv.pr->data, mv.pr->nbytes, (void**)&predict));
    }
    {   // [W | b] augmented BERT projection (src/gsv_ar.cpp:648-656)
        std::vector<float> aug((size_t)D * (BD + 1));
        const float* w = (const float*)mv.bp->data;
        const float* b = (const float*)mv.bb->data;
        for (int d = 0; d < D; d++) {
            std::memcpy(aug.data() + (size_t)d * (BD + 1), w + (size_t)d * BD, (size_t)BD * 4);
            aug[(size_t)d * (BD + 1) + BD] = b[d];
        }
        TRY(upload(aug.data(), aug.size() * 4, (void**)&bert_aug));
    }
    L.assign(NL, LayerW());
    std::vector<uint8_t> wq_tmp;
    std::vector<uint16_t> wd_tmp;
    const int NK[4][2] = {{3 * D, D}, {D, D}, {FF, D}, {D, FF}};
    all_q8 = true;
    ffn_float = false;
    any_qx = (predict_fx_type == FX_QK || predict_fx_type == FX_QM) && predict_fx;
    for (int li = 0; li < NL; li++) {
        for (int m = 0; m < 4; m++) {
            const GgufTensor* t = mv.mats[(size_t)li * 4 + m];
            const int N = NK[m][0], K = NK[m][1];
            L[li].mt[m] = q8_class(t->type) ? 8 : t->type == 7 ? 3 : (t->type == 13 || t->type == 14) ? 12 : (int)t->type;
            if (t->type == 12 || t->type == 13 || t->type == 14) {   // K-quants: k_gemm_qk planes
                all_q8 = false;
                any_qx = true;
                ffn_float |= m >= 2;
                std::vector<int16_t> kw;
                std::vector<uint16_t> kd, kdm;
                std::vector<uint8_t> kmn;
                unpack_kquant(t, kw, kd, kdm, kmn);
                void* dst = nullptr;
                TRY(upload(kw.data(), kw.size() * 2, &dst));
                L[li].wf[m] = dst;
                TRY(upload(kd.data(), kd.size() * 2, (void**)&L[li].wd[m]));
                if (t->type != 14) {
                    TRY(upload(kdm.data(), kdm.size() * 2, (void**)&L[li].wm[m]));
                    TRY(upload(kmn.data(), kmn.size(), (void**)&L[li].wmins[m]));
                }
                continue;
            }
            if (t->type == 3 || t->type == 7) {   // Q4_1 / Q5_1: value bytes + d, m planes (k_gemm_qm)
                all_q8 = false;
                any_qx = true;
                ffn_float |= m >= 2;
                std::vector<uint8_t> q;
                std::vector<uint16_t> qd, qm;
                unpack_q_1(t, q, qd, qm);
                void* dst = nullptr;
                TRY(upload(q.data(), q.size(), &dst));
                L[li].wf[m] = dst;
                TRY(upload(qd.data(), qd.size() * 2, (void**)&L[li].wd[m]));
                TRY(upload(qm.data(), qm.size() * 2, (void**)&L[li].wm[m]));
                continue;
            }
            if (!q8_class(t->type)) {   // F32 / F16 / BF16: kept as stored, row-major [N][K]
                all_q8 = false;
                ffn_float |= m >= 2;
                void* dst = nullptr;
                TRY(upload(t->data, t->nbytes, &dst));
                L[li].wf[m] = dst;
                continue;
            }
            wq_tmp.resize((size_t)N * K);
            wd_tmp.resize((size_t)N * K / QK);
            std::vector<uint16_t> w16_tmp;
            if (t->type == 8) pack_q8_0_host(t->data, N, K, wq_tmp.data(), wd_tmp.data());
            else pack_q8_0_host(to_q8_0_blocks(t).data(), N, K, wq_tmp.data(), wd_tmp.data());
            TRY(upload(wq_tmp.data(), wq_tmp.size(), (void**)&L[li].wq[m]));
            TRY(upload(wd_tmp.data(), wd_tmp.size() * 2, (void**)&L[li].wd[m]));
            {   // the same integers as fp16, row-major [N][K]: the tensor-core prefill GEMM's operand
                const std::vector<uint8_t> conv = t->type == 8 ? std::vector<uint8_t>() : to_q8_0_blocks(t);
                const uint8_t* blocks = t->type == 8 ? (const uint8_t*)t->data : conv.data();
                w16_tmp.resize((size_t)N * K);
                for (size_t r = 0; r < (size_t)N; r++)
                    for (int kb = 0; kb < K / QK; kb++) {
                        const int8_t* qv = (const int8_t*)(blocks + (r * (K / QK) + kb) * 34 + 2);
                        for (int j = 0; j < QK; j++) w16_tmp[r * K + kb * QK + j] = i8_as_f16_bits(qv[j]);
                    }
                TRY(upload(w16_tmp.data(), w16_tmp.size() * 2, (void**)&L[li].w16[m]));
            }
        }
        float** dst[8] = {&L[li].b_qkv, &L[li].b_out, &L[li].n1w, &L[li].n1b,
                          &L[li].b_f1, &L[li].b_f2, &L[li].n2w, &L[li].n2b};
        for (int k = 0; k < 8; k++) {
            const GgufTensor* t = mv.vecs[(size_t)li * 8 + k];
            TRY(upload(t->data, t->nbytes, (void**)dst[k]));
        }
    }
    {   // mk_pe (src/gsv_ar.cpp:173-181), same float expressions, extended to PE_MAX rows
        std::vector<float> tab((size_t)PE_MAX * D);
        for (int pos = 0; pos < PE_MAX; pos++)
            for (int i = 0; i < D; i += 2) {
                const float div = std::exp((float)i * -(std::log(10000.0f) / (float)D));
                tab[(size_t)pos * D + i] = std::sin((float)pos * div);
                tab[(size_t)pos * D + i + 1] = std::cos((float)pos * div);
            }
        TRY(upload(tab.data(), tab.size() * 4, (void**)&pe));
    }
    dpl = (V + 31) / 32;
    {
        std::vector<uint64_t> jm = jump_matrices(dpl);
        TRY(upload(jm.data(), jm.size() * 8, (void**)&jump));
    }
    loaded = true;
    return GSVCU_OK;
}

// ------------------------------------------------------------------ KV pool and buffers
void gsvcu_ctx::free_cache() {
    if (stream) cudaStreamSynchronize(stream);
    drop_graphs();
    for (void* p : callocs) cudaFree(p);
    callocs.clear();
    p_feat = nullptr;
    a16 = nullptr;
    reserved = false;
    max_slots = max_ctx = n_pages = max_pages = 0;
    h_bt.clear();
    free_pages.clear();
    h_st.clear();
    slot_used.clear();
    slot_pages.clear();
    slot_tag.clear();
    feat_cap = 0;
}

int gsvcu_ctx::reserve(int slots, int ctx, int kvd) {
    if (!loaded) return fail(GSVCU_ERR_STATE, "no model loaded");
    if (slots < 1 || slots > 4096 || ctx < 1 || ctx > PE_MAX || (kvd != GSVCU_KV_F16 && kvd != GSVCU_KV_F32))
        return fail(GSVCU_ERR_ARG, "kv_reserve: slots in [1, 4096], ctx in [1, 8192], kv dtype F16/F32");
    for (char u : slot_used)
        if (u) return fail(GSVCU_ERR_STATE, "kv_reserve while sequences are in flight");
    free_cache();
    const int NL = hp.n_layer, V = hp.vocab_size;
    max_slots = (slots + 7) / 8 * 8;
    max_ctx = ctx;
    kv_f32 = kvd;
    max_pages = (ctx + PAGE - 1) / PAGE;
    n_pages = max_slots * max_pages;
    max_chunks = decode_chunks(ctx);
    tok_cap = ctx;
    forced_cap = ctx;
    Mmax = std::max(PREFILL_ROWS, max_slots);
    const size_t page_bytes = (size_t)NL * 2 * NH * PAGE * HD * (kvd == GSVCU_KV_F32 ? 4 : 2);
    const size_t M = (size_t)Mmax;
    struct A { void** p; size_t bytes; };
    const A list[] = {
        {&pool, page_bytes * n_pages},
        {(void**)&block_table, (size_t)max_slots * max_pages * 4},
        {(void**)&st, sizeof(SlotState) * max_slots},
        {(void**)&counts, (size_t)max_slots * V * 2},
        {(void**)&hist, (size_t)max_slots * HIST * 4},
        {(void**)&out_tokens, (size_t)max_slots * tok_cap * 4},
        {(void**)&forced, (size_t)max_slots * forced_cap * 4},
        {(void**)&logits, (size_t)max_slots * V * 4},
        {(void**)&x, M * D * 4}, {(void**)&qkv, M * 3 * D * 4}, {(void**)&pre, M * D * 4},
        {(void**)&n1, M * D * 4}, {(void**)&attn_f32, M * D * 4},
        {(void**)&xq, M * D}, {(void**)&aq, M * D}, {(void**)&n1q, M * D}, {(void**)&hq, M * FF},
        {(void**)&xd, M * D / QK * 2}, {(void**)&ad, M * D / QK * 2}, {(void**)&n1d, M * D / QK * 2},
        {(void**)&hd, M * FF / QK * 2},
        {(void**)&part, (size_t)max_slots * NH * max_chunks * PART_STRIDE * 4},
        {(void**)&work, (size_t)max_slots * max_chunks * sizeof(int4)}, {(void**)&work_base, 4 * 4},
        {(void**)&p_ids, M * 4}, {(void**)&p_pepos, M * 4}, {(void**)&p_istext, M * 4},
        {(void**)&p_tslot, M * 4}, {(void**)&p_tpos, M * 4}, {(void**)&p_rowT, M * 4}, {(void**)&p_rowoff, M * 8},
        {(void**)&p_sstart, (size_t)max_slots * 4}, {(void**)&p_slen, (size_t)max_slots * 4},
        {(void**)&p_tlen, (size_t)max_slots * 4}, {(void**)&p_last, (size_t)max_slots * 4},
        {(void**)&p_slots, (size_t)max_slots * 4},
        {(void**)&p_tiles, (M / PREF_QTILE + max_slots) * sizeof(PrefillTile)},
        {(void**)&p_xl, (size_t)max_slots * D * 4}, {(void**)&p_lg, (size_t)max_slots * V * 4},
        {(void**)&hf, ffn_float ? M * FF * 4 : 0},
        {(void**)&qx_q, any_qx ? M * FF : 0}, {(void**)&qx_d, any_qx ? M * (FF / 32) * 4 : 0},
        {&qx_s, any_qx ? M * (FF / 16) * 4 : 0},
        {(void**)&a16, a16_n = tc_scratch_bytes((int)M, FF, FF)},
    };
    for (const A& a : list) {
        if (!a.bytes) {
            *a.p = nullptr;
            continue;
        }
        const int r = alloc_dev(a.p, a.bytes, callocs);
        if (r != GSVCU_OK) {
            free_cache();
            return r;
        }
    }
    CK(cudaMemsetAsync(st, 0, sizeof(SlotState) * max_slots, stream));
    CK(cudaMemsetAsync(xq, 0, M * D, stream));
    CK(cudaMemsetAsync(xd, 0, M * D / QK * 2, stream));
    CK(cudaMemsetAsync(x, 0, M * D * 4, stream));
    CK(cudaMemsetAsync(block_table, 0, (size_t)max_slots * max_pages * 4, stream));
    h_bt.assign((size_t)max_slots * max_pages, 0);
    free_pages.resize(n_pages);
    for (int i = 0; i < n_pages; i++) free_pages[i] = n_pages - 1 - i;
    h_st.assign(max_slots, SlotState{});
    slot_used.assign(max_slots, 0);
    slot_pages.assign(max_slots, {});
    slot_tag.assign(max_slots, 0);
    CK(cudaStreamSynchronize(stream));
    reserved = true;
    return GSVCU_OK;
}

int gsvcu_ctx::ensure(int need_slots, int need_ctx, int kvd) {
    if (reserved && max_slots >= need_slots && max_ctx >= need_ctx && kv_f32 == kvd) return GSVCU_OK;
    for (char u : slot_used)
        if (u) return fail(GSVCU_ERR_OOM, "KV pool too small for this batch while other sequences are in flight");
    const int slots = std::max(need_slots, reserved ? max_slots : 0);
    const int ctx = std::max(need_ctx, reserved ? max_ctx : 0);
    return reserve(slots, ctx, kvd);
}

// Sampler settings of the next admissions; every slot keeps those it was admitted with, so sequences
// with different settings share the running batch.
int gsvcu_ctx::set_cfg(const gsvcu_sampler_cfg& c) {
    cfg = c;
    return GSVCU_OK;
}

void gsvcu_ctx::release_slot(int slot) {
    for (int pg : slot_pages[slot]) free_pages.push_back(pg);
    slot_pages[slot].clear();
    slot_used[slot] = 0;
}

// ------------------------------------------------------------------ prefill
// Packs the sequences' rows back to back (no padding; the reference's left-pad keys are always
// masked, src/gsv_ar.cpp:219, so they contribute nothing) and runs the layers over all rows.
// logits of M rows xr [M][D] f32 into out [M][V] (src/gsv_ar.cpp:266, ggml mul_mat with `predict`): the F32
// path of k_gemm_f32d, or for a Q8_0 predict the rows quantized to Q8_0 (into xq_s, xd_s) and the Q8_0
// GEMM, as for the layer matrices. Returns the kernels launched.
int gsvcu_ctx::launch_logits(const float* xr, int M, int8_t* xq_s, uint16_t* xd_s, float* out, cudaStream_t s) {
    const int V = hp.vocab_size;
    if (predict_fx) {
        GemmFxParams g;
        g.x = xr; g.ldx = D; g.M = M; g.w = predict_fx; g.wtype = predict_fx_type; g.N = V; g.K = D; g.y = out;
        g.ldy = V; g.wd = predict_qd; g.wm = predict_qm; g.wmins = predict_mins;
        g.qx_q = qx_q; g.qx_d = qx_d; g.qx_s = qx_s;
        launch_gemm_fx(g, FXE_BIAS, s);
        return 1;
    }
    if (!predict_q8) {
        launch_gemm_f32d(xr, D, nullptr, M, predict, V, D, nullptr, 0, out, V, s);
        return 1;
    }
    launch_quantize_q8(xr, M, D, xq_s, xd_s, s);
    GemmQ8Params g;
    g.xq = xq_s; g.xd = xd_s; g.M = M; g.wq = predict_wq; g.wd = predict_wd; g.N = V_pad; g.K = D;
    g.y = out; g.ldy = V; g.n_store = V;
    launch_gemm_q8(g, EPI_BIAS, s);
    return 2;
}

int gsvcu_ctx::prefill_pass(const int* slots, const gsvcu_request* reqs, int n, float* dump, int dump_b0,
                            int dump_B) {
    const int NL = hp.n_layer, V = hp.vocab_size, BD = hp.bert_dim;
    int M = 0;
    for (int i = 0; i < n; i++) M += reqs[i].n_phones + reqs[i].n_prompt;
    std::vector<int32_t> ids(M), pepos(M), istext(M), tslot(M), tpos(M), rowT(M), sstart(n), slen(n), tlen(n), last(n),
        sl(n);
    std::vector<int64_t> rowoff(M, 0);
    std::vector<PrefillTile> tiles;
    size_t feat_n = 0;
    for (int i = 0; i < n; i++) feat_n += (size_t)BD * reqs[i].n_phones;
    std::vector<size_t> feat_off(n);
    int m = 0;
    size_t fo = 0;
    for (int i = 0; i < n; i++) {
        const gsvcu_request& r = reqs[i];
        const int T = r.n_phones, P = r.n_prompt;
        sstart[i] = m;
        slen[i] = T + P;
        tlen[i] = T;
        last[i] = m + T + P - 1;
        sl[i] = slots[i];
        feat_off[i] = fo;
        for (int t = 0; t < T; t++, m++) {
            ids[m] = r.phones[t];
            pepos[m] = t;
            istext[m] = 1;
            tslot[m] = slots[i];
            tpos[m] = t;
            rowT[m] = T;
            rowoff[m] = (int64_t)fo + t;
        }
        for (int t = 0; t < P; t++, m++) {
            ids[m] = r.prompt[t];
            pepos[m] = t;
            istext[m] = 0;
            tslot[m] = slots[i];
            tpos[m] = T + t;
            rowT[m] = -1;
        }
        for (int q0 = 0; q0 < T + P; q0 += PREF_QTILE) tiles.push_back({i, q0});
        fo += (size_t)BD * T;
    }
    cudaStream_t s = stream;
    if (feat_n > feat_cap) {
        if (p_feat) {
            cudaStreamSynchronize(s);
            cudaFree(p_feat);
            callocs.erase(std::find(callocs.begin(), callocs.end(), (void*)p_feat));
            p_feat = nullptr;
            feat_cap = 0;
        }
        TRY(alloc_dev((void**)&p_feat, feat_n * 4, callocs));
        feat_cap = feat_n;
    }
    auto h2d = [&](void* dst, const void* src, size_t bytes) {
        return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s);
    };
    CK(h2d(p_ids, ids.data(), (size_t)M * 4));
    CK(h2d(p_pepos, pepos.data(), (size_t)M * 4));
    CK(h2d(p_istext, istext.data(), (size_t)M * 4));
    CK(h2d(p_tslot, tslot.data(), (size_t)M * 4));
    CK(h2d(p_tpos, tpos.data(), (size_t)M * 4));
    CK(h2d(p_rowT, rowT.data(), (size_t)M * 4));
    CK(h2d(p_rowoff, rowoff.data(), (size_t)M * 8));
    CK(h2d(p_sstart, sstart.data(), (size_t)n * 4));
    CK(h2d(p_slen, slen.data(), (size_t)n * 4));
    CK(h2d(p_tlen, tlen.data(), (size_t)n * 4));
    CK(h2d(p_last, last.data(), (size_t)n * 4));
    CK(h2d(p_slots, sl.data(), (size_t)n * 4));
    CK(h2d(p_tiles, tiles.data(), tiles.size() * sizeof(PrefillTile)));
    // BERT features: host or device memory (unified addressing picks the copy direction)
    for (int i = 0; i < n; i++)
        if (reqs[i].n_phones)
            CK(cudaMemcpyAsync(p_feat + feat_off[i], reqs[i].bert, (size_t)BD * reqs[i].n_phones * 4, cudaMemcpyDefault,
                               s));

    PrefEmbedParams ep;
    ep.ids = p_ids; ep.pe_pos = p_pepos; ep.is_text = p_istext; ep.text_emb = text_emb; ep.audio_emb = audio_emb;
    ep.pe = pe; ep.text_alpha = hp.text_pe_alpha; ep.audio_alpha = hp.audio_pe_alpha; ep.M = M; ep.x = x;
    launch_prefill_embed(ep, s);
    // cur = x + bert_aug . [bert; 1] on text rows (src/gsv_ar.cpp:241); prompt rows gather zeros
    F32Gather gth;
    gth.feat = p_feat; gth.row_off = p_rowoff; gth.row_T = p_rowT; gth.bert_dim = BD;
    launch_gemm_f32d(nullptr, 0, &gth, M, bert_aug, D, BD + 1, x, D, x, D, s);
    launch_quantize_q8(x, M, D, xq, xd, s);

    const float scale = 1.0f / std::sqrt((float)HD);
    auto dump_rows = [&](int li, int item, const float* src) -> int {
        for (int i = 0; i < n; i++) {
            float* dst = dump + ((((size_t)0 * dump_B + dump_b0 + i) * NL + li) * 4 + item) * D;
            CK(cudaMemcpyAsync(dst, src + (size_t)last[i] * D, D * 4, cudaMemcpyDeviceToHost, s));
        }
        return GSVCU_OK;
    };
    const LayerIO io{x, attn_f32, n1, xq, aq, n1q, xd, ad, n1d, qkv, pre};
    for (int li = 0; li < NL; li++) {
        const LayerW& w = L[li];
        KvWrite kv;
        kv.pool = pool; kv.kv_f32 = kv_f32; kv.n_layer = NL; kv.layer = li; kv.block_table = block_table;
        kv.max_pages = max_pages; kv.tok_slot = p_tslot; kv.tok_pos = p_tpos;
        layer_gemm(li, 0, io, M, kv, s);
        PrefAttnParams a;
        a.qkv = qkv; a.seq_start = p_sstart; a.seq_len = p_slen; a.text_len = p_tlen; a.tiles = p_tiles;
        a.n_tiles = (int)tiles.size(); a.scale = scale; a.out_q = aq; a.out_d = ad;
        a.out_f32 = dump || w.mt[1] != 8 ? attn_f32 : nullptr;
        launch_prefill_attention(a, s);
        layer_gemm(li, 1, io, M, KvWrite(), s);
        launch_layernorm_q8(pre, M, w.n1w, w.n1b, n1, n1q, n1d, s);
        layer_gemm(li, 2, io, M, KvWrite(), s);
        layer_gemm(li, 3, io, M, KvWrite(), s);
        if (dump) {
            TRY(dump_rows(li, 0, attn_f32));
            TRY(dump_rows(li, 1, n1));
            TRY(dump_rows(li, 2, pre));
        }
        launch_layernorm_q8(pre, M, w.n2w, w.n2b, x, xq, xd, s);
        if (dump) TRY(dump_rows(li, 3, x));
    }
    // logits of each sequence's last position (src/gsv_ar.cpp:266-269) into its slot's row
    launch_copy_rows(p_xl, nullptr, x, p_last, n, D, s);
    const int nlg = launch_logits(p_xl, n, xq, xd, p_lg, s);   // the pass's Q8_0 rows are consumed
    launch_copy_rows(logits, p_slots, p_lg, nullptr, n, V, s);
    launches += 3 + (int64_t)NL * 7 + 2 + nlg;
    CK(cudaGetLastError());
    // host staging vectors die at return: finish the pass before they go
    int32_t gerr = 0;
    CK(cudaMemcpyAsync(&gerr, att_err + 2, sizeof(gerr), cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    if (gerr) {
        CK(cudaMemsetAsync(att_err + 2, 0, sizeof(int32_t), s));
        CK(cudaStreamSynchronize(s));
        return fail(GSVCU_ERR_CUDA, "prefill GEMM: staged tiles never arrived (bounded wait gave up)");
    }
    return GSVCU_OK;
}

// Layer li's GEMM m (0 QKV, 1 out, 2 FFN1, 3 FFN2) over M rows: QKV = x W^T + b (+ K/V store),
// pre = (x + attn W^T) + b, FFN1 -> relu(n1 W^T + b) (Q8_0 blocks hq/hd or floats hf, as FFN2 reads),
// pre = (n1 + h W^T) + b.
void gsvcu_ctx::layer_gemm(int li, int m, const LayerIO& io, int M, const KvWrite& kv, cudaStream_t s) {
    const LayerW& w = L[li];
    const float* bias[4] = {w.b_qkv, w.b_out, w.b_f1, w.b_f2};
    const int N[4] = {3 * D, D, FF, D}, K[4] = {D, D, D, FF};
    if (w.mt[m] == 8) {
        GemmQ8Params g;
        g.M = M; g.wq = w.wq[m]; g.wd = w.wd[m]; g.N = N[m]; g.K = K[m]; g.bias = bias[m];
        if (tc_prefill && a16 && w.w16[m] && M >= TC_MIN_ROWS) {   // tcgen05 path (k_tc_prep + k_gemm_q8_tc)
            g.w16 = w.w16[m]; g.tc_scratch = a16; g.tc_scratch_n = a16_n; g.err = att_err + 2;
            launches++;
        }
        if (m == 0) { g.xq = io.xq; g.xd = io.xd; g.y = io.qkv; g.kv = kv; launch_gemm_q8(g, EPI_BIAS, s); }
        if (m == 1) { g.xq = io.aq; g.xd = io.ad; g.resid = io.x; g.y = io.pre; launch_gemm_q8(g, EPI_RESID, s); }
        if (m == 2) { g.xq = io.n1q; g.xd = io.n1d; g.yq = hq; g.yd = hd; launch_gemm_q8(g, EPI_RELU_Q8, s); }
        if (m == 3) { g.xq = hq; g.xd = hd; g.resid = io.n1; g.y = io.pre; launch_gemm_q8(g, EPI_RESID, s); }
        return;
    }
    GemmFxParams g;
    g.M = M; g.w = w.wf[m];
    g.wtype = w.mt[m] == 1 ? FX_F16 : w.mt[m] == 30 ? FX_BF16 : w.mt[m] == 3 ? FX_QM : w.mt[m] == 12 ? FX_QK : FX_F32;
    g.wd = w.wd[m]; g.wm = w.wm[m]; g.wmins = w.wmins[m]; g.N = N[m]; g.K = K[m]; g.bias = bias[m];
    g.ldx = K[m];
    g.qx_q = qx_q; g.qx_d = qx_d; g.qx_s = qx_s;
    if (m == 0) { g.x = io.x; g.y = io.qkv; g.kv = kv; launch_gemm_fx(g, FXE_BIAS, s); }
    if (m == 1) { g.x = io.attn; g.resid = io.x; g.y = io.pre; launch_gemm_fx(g, FXE_RESID, s); }
    if (m == 2) { g.x = io.n1; g.y = hf; launch_gemm_fx(g, FXE_RELU, s); }
    if (m == 3) { g.x = hf; g.resid = io.n1; g.y = io.pre; launch_gemm_fx(g, FXE_RESID, s); }
}

// Admit n sequences into free slots: pages, slot state, repetition window, prefill.
int gsvcu_ctx::admit(const gsvcu_request* reqs, int n, const uint64_t* seeds, const int32_t* tags, int max_steps,
                     int early_stop, bool one_group, const int32_t* forced_tok, int n_forced, bool forced_per_seq,
                     std::vector<int>& slots_out, float* dump) {
    const int V = hp.vocab_size;
    slots_out.clear();
    if (n <= 0) return GSVCU_OK;
    if (max_steps < 1) return fail(GSVCU_ERR_ARG, "max_steps must be >= 1");
    int total_rows = 0;
    for (int i = 0; i < n; i++) {
        const gsvcu_request& r = reqs[i];
        if (r.n_phones <= 0 || !r.phones || !r.bert) return fail(GSVCU_ERR_ARG, "request without phones/bert");
        if (r.n_prompt < 0 || (r.n_prompt > 0 && !r.prompt)) return fail(GSVCU_ERR_ARG, "bad prompt");
        for (int t = 0; t < r.n_phones; t++)
            if (r.phones[t] < 0 || r.phones[t] >= hp.phoneme_vocab_size)
                return fail(GSVCU_ERR_ARG, "phone id out of range");
        for (int t = 0; t < r.n_prompt; t++)
            if (r.prompt[t] < 0 || r.prompt[t] >= V) return fail(GSVCU_ERR_ARG, "prompt code out of range");
        const int S = r.n_phones + r.n_prompt;
        if (S + max_steps > max_ctx) return fail(GSVCU_ERR_ARG, "sequence longer than the reserved context");
        if (r.n_prompt + max_steps > PE_MAX || r.n_phones > PE_MAX) return fail(GSVCU_ERR_ARG, "position beyond PE table");
        if (S > Mmax) return fail(GSVCU_ERR_ARG, "prefix longer than a prefill pass");
        total_rows += S;
    }
    if (dump && total_rows > Mmax) return fail(GSVCU_ERR_ARG, "debug dumps need a single prefill pass");
    if (forced_tok)
        for (int i = 0; i < (forced_per_seq ? n * n_forced : n_forced); i++)
            if (forced_tok[i] < 0 || forced_tok[i] >= V) return fail(GSVCU_ERR_ARG, "forced token out of range");
    int need_pages = 0;
    for (int i = 0; i < n; i++) need_pages += (reqs[i].n_phones + reqs[i].n_prompt + max_steps + PAGE - 1) / PAGE;
    int free_slots = 0;
    for (char u : slot_used) free_slots += !u;
    if (free_slots < n) return fail(GSVCU_ERR_OOM, "no free sequence slot");
    if ((int)free_pages.size() < need_pages) return fail(GSVCU_ERR_OOM, "KV page pool exhausted");
    int next = 0;
    for (int i = 0; i < n; i++) {
        while (slot_used[next]) next++;
        slots_out.push_back(next);
        slot_used[next] = 1;
        next++;
    }
    cudaStream_t s = stream;
    const int first = slots_out[0];
    std::vector<uint16_t> cnt(V);
    for (int i = 0; i < n; i++) {
        const int slot = slots_out[i];
        const gsvcu_request& r = reqs[i];
        const int S = r.n_phones + r.n_prompt;
        const int np = (S + max_steps + PAGE - 1) / PAGE;
        slot_pages[slot].clear();
        for (int k = 0; k < np; k++) {
            slot_pages[slot].push_back(free_pages.back());
            h_bt[(size_t)slot * max_pages + k] = free_pages.back();
            free_pages.pop_back();
        }
        slot_tag[slot] = tags ? tags[i] : i;
        CK(cudaMemcpyAsync(block_table + (size_t)slot * max_pages, h_bt.data() + (size_t)slot * max_pages,
                           (size_t)np * 4, cudaMemcpyHostToDevice, s));
        // repetition window: the last <= 4096 prompt tokens (src/gsv_ar.cpp:769-771)
        std::fill(cnt.begin(), cnt.end(), 0);
        const int nh = std::min(r.n_prompt, HIST);
        for (int t = r.n_prompt - nh; t < r.n_prompt; t++) cnt[r.prompt[t]]++;
        CK(cudaMemcpyAsync(counts + (size_t)slot * V, cnt.data(), (size_t)V * 2, cudaMemcpyHostToDevice, s));
        if (nh) CK(cudaMemcpyAsync(hist + (size_t)slot * HIST, r.prompt + (r.n_prompt - nh), (size_t)nh * 4,
                                   cudaMemcpyHostToDevice, s));
        SlotState& ss = h_st[slot];
        ss = SlotState{};
        ss.active = 1;
        ss.kvlen = S;
        ss.kvpos = 0;
        ss.prompt_len = r.n_prompt;
        ss.n_samp = 0;
        ss.max_steps = max_steps;
        ss.early_stop = early_stop;
        ss.group_first = one_group ? first : slot;
        ss.finish_kind = -1;
        ss.finish_idx = -1;
        ss.hist_len = nh;
        ss.hist_head = 0;
        ss.decode_now = 0;
        ss.top_k = cfg.top_k;
        ss.top_p = cfg.top_p;
        ss.temperature = cfg.temperature;
        ss.rep = cfg.repetition_penalty;
        const uint64_t seed = seeds ? seeds[i] : (uint64_t)i;
        ss.rng = seed ? seed : 1;   // gsv_rng(seed) (src/gsv_sampler.h:35)
        ss.n_forced = 0;
        if (forced_tok && n_forced > 0) {
            const int nf = std::min(n_forced, forced_cap);
            ss.n_forced = nf;
            CK(cudaMemcpyAsync(forced + (size_t)slot * forced_cap,
                               forced_tok + (forced_per_seq ? (size_t)i * n_forced : 0), (size_t)nf * 4,
                               cudaMemcpyHostToDevice, s));
        }
        CK(cudaMemcpyAsync(st + slot, &ss, sizeof(SlotState), cudaMemcpyHostToDevice, s));
    }
    // prefill in passes of at most Mmax rows
    int i = 0;
    while (i < n) {
        int rows = 0, j = i;
        while (j < n && rows + reqs[j].n_phones + reqs[j].n_prompt <= Mmax) {
            rows += reqs[j].n_phones + reqs[j].n_prompt;
            j++;
        }
        TRY(prefill_pass(slots_out.data() + i, reqs + i, j - i, dump, i, n));
        i = j;
    }
    return GSVCU_OK;
}

// ------------------------------------------------------------------ decode step
// One step for every slot: sample from the current logits, apply the stop rules, embed the new
// token, run the layers (K/V appended in the QKV epilogue, split-KV attention over the pages),
// project to logits. All per-step values live on the device, so the sequence is graph-captured.
// With `dump` (host), every layer's rows of the slots in dump_slots are copied out (no capture).
int gsvcu_ctx::launch_step(cudaStream_t s, float* dump, int dump_row, const int* dump_slots, int dump_B) {
    const int NL = hp.n_layer, V = hp.vocab_size, M = max_slots;
    int nk = 0;
    // class timing (profiler only): mark(c) closes the interval since the previous mark into class c
    auto mark = [&](int c) -> int {
        if (!prof_ms) return GSVCU_OK;
        CK(cudaEventRecord(prof_ev[1], s));
        CK(cudaEventSynchronize(prof_ev[1]));
        float ms = 0.f;
        CK(cudaEventElapsedTime(&ms, prof_ev[0], prof_ev[1]));
        prof_ms[c] += ms;
        CK(cudaEventRecord(prof_ev[0], s));
        return GSVCU_OK;
    };
    if (prof_ms) CK(cudaEventRecord(prof_ev[0], s));
    SamplerParams sp;
    sp.logits = logits; sp.V = V; sp.eos = hp.eos; sp.nslots = M;
    sp.st = st; sp.counts = counts; sp.hist = hist; sp.out_tokens = out_tokens; sp.tok_cap = tok_cap;
    sp.forced = forced; sp.forced_cap = forced_cap; sp.jump = jump; sp.draws_per_lane = dpl;
    launch_sampler(sp, s);
    nk++;
    TRY(mark(0));
    StepPrepParams pp;
    pp.st = st; pp.nslots = M; pp.eos = hp.eos; pp.out_tokens = out_tokens; pp.tok_cap = tok_cap;
    pp.audio_emb = audio_emb; pp.pe = pe; pp.audio_alpha = hp.audio_pe_alpha;
    pp.x = x; pp.xq = xq; pp.xd = xd;
    launch_step_prep(pp, s);
    nk++;
    TRY(mark(1));
    const float scale = 1.0f / std::sqrt((float)HD);
    if (fused && dense_ok && all_q8 && !dump) {
        // fused layers for slots [s0, s0 + rows): QKV of layer 0, then per layer the page attention and
        // the cluster layer tail (merge, out, LN1, FFN1, FFN2, LN2, next layer's QKV), then the logits
        auto chain = [&](cudaStream_t cs, int s0, int rows) -> int {
            {
                const LayerW& w = L[0];
                GemmQ8Params g;
                g.xq = xq + (size_t)s0 * D; g.xd = xd + (size_t)s0 * (D / QK); g.M = rows; g.wq = w.wq[0];
                g.wd = w.wd[0]; g.N = 3 * D; g.K = D; g.bias = w.b_qkv; g.y = qkv + (size_t)s0 * 3 * D;
                g.kv.pool = pool; g.kv.kv_f32 = kv_f32; g.kv.n_layer = NL; g.kv.layer = 0;
                g.kv.block_table = block_table + (size_t)s0 * max_pages; g.kv.max_pages = max_pages;
                g.kv.st = st + s0;
                launch_gemm_q8(g, EPI_BIAS, cs);
                nk++;
                TRY(mark(GSVCU_PROF_QKV_GEMM));
            }
            for (int li = 0; li < NL; li++) {
                const LayerW& w = L[li];
                DecAttnParams a;
                a.q = qkv; a.q_stride = 3 * D; a.pool = pool; a.kv_f32 = kv_f32; a.n_layer = NL; a.layer = li;
                a.block_table = block_table; a.max_pages = max_pages; a.st = st; a.slot0 = s0; a.B = rows;
                a.max_chunks = max_chunks; a.scale = scale; a.out_q = aq; a.out_d = ad; a.part = part;
                a.part_ml = part_ml_of(part, (size_t)max_slots * NH * max_chunks);
                a.partials_only = 1; a.err = att_err;
                a.fault_extra_tx = fault_extra_tx; a.poll_limit = fault_poll_limit;
                a.work = work; a.work_base = work_base; a.group = s0 ? 1 : 0;
                nk += launch_decode_attention(a, cs);
                TRY(mark(GSVCU_PROF_DECODE_ATTN));
                DenseParams d;
                d.slot0 = s0; d.M = rows; d.st = st; d.part = part; d.max_chunks = max_chunks;
                d.part_ml = part_ml_of(part, (size_t)max_slots * NH * max_chunks);
                d.w_out = w.wq[1]; d.d_out = w.wd[1]; d.b_out = w.b_out; d.n1w = w.n1w; d.n1b = w.n1b;
                d.w_f1 = w.wq[2]; d.d_f1 = w.wd[2]; d.b_f1 = w.b_f1; d.w_f2 = w.wq[3]; d.d_f2 = w.wd[3];
                d.b_f2 = w.b_f2; d.n2w = w.n2w; d.n2b = w.n2b; d.x = x; d.err = att_err;
                if (li + 1 < NL) {
                    const LayerW& wn = L[li + 1];
                    d.w_qkv = wn.wq[0]; d.d_qkv = wn.wd[0]; d.b_qkv = wn.b_qkv; d.q = qkv; d.q_stride = 3 * D;
                    d.kv.pool = pool; d.kv.kv_f32 = kv_f32; d.kv.n_layer = NL; d.kv.layer = li + 1;
                    d.kv.block_table = block_table; d.kv.max_pages = max_pages; d.kv.st = st;
                }
                launch_dense_layer(d, cs);
                nk++;
                TRY(mark(GSVCU_PROF_DENSE));
            }
            nk += launch_logits(x + (size_t)s0 * D, rows, xq + (size_t)s0 * D, xd + (size_t)s0 * (D / QK),
                                logits + (size_t)s0 * V, cs);
            TRY(mark(GSVCU_PROF_PREDICT));
            return GSVCU_OK;
        };
        const bool two = two_groups && !prof_ms && M >= 32 && M % 32 == 0;
        launch_page_list(st, M, two ? M / 2 : M, block_table, max_pages, work, work_base, s);
        nk++;
        if (!two) {
            TRY(chain(s, 0, M));
        } else {
            // two slot groups on their own streams; the step's tail joins them back into s
            const int half = M / 2;
            CK(cudaEventRecord(gevent[2], s));
            for (int gi = 0; gi < 2; gi++) {
                CK(cudaStreamWaitEvent(gstream[gi], gevent[2], 0));
                TRY(chain(gstream[gi], gi * half, half));
                CK(cudaEventRecord(gevent[gi], gstream[gi]));
            }
            CK(cudaStreamWaitEvent(s, gevent[0], 0));
            CK(cudaStreamWaitEvent(s, gevent[1], 0));
        }
        graph_kernels = nk;
        return GSVCU_OK;
    }
    const LayerIO io{x, attn_f32, n1, xq, aq, n1q, xd, ad, n1d, qkv, pre};
    for (int li = 0; li < NL; li++) {
        const LayerW& w = L[li];
        KvWrite kv;
        kv.pool = pool; kv.kv_f32 = kv_f32; kv.n_layer = NL; kv.layer = li; kv.block_table = block_table;
        kv.max_pages = max_pages; kv.st = st;
        layer_gemm(li, 0, io, M, kv, s);
        TRY(mark(2));
        DecAttnParams a;
        a.q = qkv; a.q_stride = 3 * D; a.pool = pool; a.kv_f32 = kv_f32; a.n_layer = NL; a.layer = li;
        a.block_table = block_table; a.max_pages = max_pages; a.st = st; a.B = M; a.max_chunks = max_chunks;
        a.scale = scale; a.out_q = aq; a.out_d = ad; a.out_f32 = dump || w.mt[1] != 8 ? attn_f32 : nullptr;
        a.part = part; a.part_ml = part_ml_of(part, (size_t)max_slots * NH * max_chunks); a.err = att_err;
        a.fault_extra_tx = fault_extra_tx; a.poll_limit = fault_poll_limit;
        nk += launch_decode_attention(a, s);
        TRY(mark(3));
        layer_gemm(li, 1, io, M, KvWrite(), s);
        TRY(mark(4));
        launch_layernorm_q8(pre, M, w.n1w, w.n1b, n1, n1q, n1d, s);
        TRY(mark(5));
        layer_gemm(li, 2, io, M, KvWrite(), s);
        TRY(mark(6));
        layer_gemm(li, 3, io, M, KvWrite(), s);
        TRY(mark(7));
        nk += 6;
        if (dump) {
            const float* items[3] = {attn_f32, n1, pre};
            for (int it = 0; it < 3; it++)
                for (int b = 0; b < dump_B; b++)
                    CK(cudaMemcpyAsync(dump + ((((size_t)dump_row * dump_B + b) * NL + li) * 4 + it) * D,
                                       items[it] + (size_t)dump_slots[b] * D, D * 4, cudaMemcpyDeviceToHost, s));
        }
        launch_layernorm_q8(pre, M, w.n2w, w.n2b, x, xq, xd, s);
        TRY(mark(5));
        if (dump)
            for (int b = 0; b < dump_B; b++)
                CK(cudaMemcpyAsync(dump + ((((size_t)dump_row * dump_B + b) * NL + li) * 4 + 3) * D,
                                   x + (size_t)dump_slots[b] * D, D * 4, cudaMemcpyDeviceToHost, s));
    }
    nk += launch_logits(x, M, xq, xd, logits, s);
    TRY(mark(8));
    graph_kernels = nk;
    return GSVCU_OK;
}

// Capture n consecutive decode steps into one executable graph. Every per-slot value lives in device
// memory, so one capture serves every later launch; inside the graph the programmatic edges also join
// the last kernel of a step to the first of the next.
int gsvcu_ctx::capture_steps(int n, cudaGraphExec_t* out) {
    cudaGraph_t gr;
    CK(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
    int lr = GSVCU_OK;
    for (int k = 0; k < n && lr == GSVCU_OK; k++) lr = launch_step(stream);
    cudaError_t e = cudaStreamEndCapture(stream, &gr);
    if (lr != GSVCU_OK) return lr;
    if (e != cudaSuccess) return fail(GSVCU_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
    e = cudaGraphInstantiate(out, gr, 0);
    cudaGraphDestroy(gr);
    if (e != cudaSuccess) {
        *out = nullptr;
        return fail(GSVCU_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
    }
    return GSVCU_OK;
}

int gsvcu_ctx::run_steps(int nsteps) {
    int left = nsteps;
    if (left >= GRAPH_CHUNK) {
        if (!graph_chunk) TRY(capture_steps(GRAPH_CHUNK, &graph_chunk));
        for (; left >= GRAPH_CHUNK; left -= GRAPH_CHUNK) CK(cudaGraphLaunch(graph_chunk, stream));
    }
    if (left > 0) {
        if (!graph) TRY(capture_steps(1, &graph));
        for (int i = 0; i < left; i++) CK(cudaGraphLaunch(graph, stream));
    }
    launches += (int64_t)nsteps * graph_kernels;
    return GSVCU_OK;
}

int gsvcu_ctx::read_status() {
    int32_t aerr = 0;
    CK(cudaMemcpyAsync(h_st.data(), st, sizeof(SlotState) * max_slots, cudaMemcpyDeviceToHost, stream));
    CK(cudaMemcpyAsync(&aerr, att_err, sizeof(aerr), cudaMemcpyDeviceToHost, stream));
    CK(cudaStreamSynchronize(stream));
    if (aerr) {   // reported once: the word is cleared so the context stays usable
        CK(cudaMemsetAsync(att_err, 0, sizeof(int32_t), stream));
        CK(cudaStreamSynchronize(stream));
        return fail(GSVCU_ERR_CUDA, "decode attention: staged K/V never arrived (bounded wait gave up)");
    }
    return GSVCU_OK;
}

// ------------------------------------------------------------------ C ABI
static int max_prefix(const gsvcu_request* reqs, int B) {
    int m = 0;
    for (int i = 0; i < B; i++) m = std::max(m, reqs[i].n_phones + reqs[i].n_prompt);
    return m;
}

// Generate for one group of sequences (gsv_ar::generate loop, src/gsv_ar.cpp:761-810).
static int generate_group(gsvcu_ctx* ctx, const gsvcu_request* reqs, int B, const uint64_t* seeds, int early_stop,
                          int max_steps, const int32_t* forced, int n_forced, bool forced_per_seq,
                          gsvcu_progress_fn progress, void* user, std::vector<int>& slots) {
    TRY(ctx->admit(reqs, B, seeds, nullptr, max_steps, early_stop, true, forced, n_forced, forced_per_seq, slots,
                   nullptr));
    int done_steps = 0, reported = 0;
    while (done_steps < max_steps) {
        const int n = std::min(STEP_CHUNK, max_steps - done_steps);
        TRY(ctx->run_steps(n));
        done_steps += n;
        TRY(ctx->read_status());
        bool all = true;
        int iters = 0;
        for (int sl : slots) {
            const SlotState& s = ctx->h_st[sl];
            if (s.active) all = false;
            iters = std::max(iters, s.finish_kind >= 0 ? s.finish_idx + 1 : s.n_samp);
        }
        if (progress && iters > reported) {
            progress(user, iters);
            reported = iters;
        }
        if (all) break;
    }
    return GSVCU_OK;
}

extern "C" {

int gsvcu_create(int device, gsvcu_ctx** out) {
    if (!out) return GSVCU_ERR_ARG;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        cudaGetLastError();
        return GSVCU_ERR_DEVICE;
    }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10) return GSVCU_ERR_DEVICE;
    DeviceGuard g(device);
    bool dense_usable = false;
    if (gemm_q8_init_device() != cudaSuccess || gemm_tc_init_device() != cudaSuccess ||
        gemm_fx_init_device() != cudaSuccess || attention_init_device() != cudaSuccess ||
        logits_init_device() != cudaSuccess || dense_init_device(&dense_usable) != cudaSuccess) {
        cudaGetLastError();
        return GSVCU_ERR_CUDA;
    }
    gsvcu_ctx* c = new gsvcu_ctx();
    c->device = device;
    c->dense_ok = dense_usable;
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc((void**)&c->att_err, 3 * sizeof(int32_t)) != cudaSuccess ||
        cudaMemset(c->att_err, 0, 3 * sizeof(int32_t)) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->gstream[0], cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->gstream[1], cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->gevent[0], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->gevent[1], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->gevent[2], cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        delete c;
        return GSVCU_ERR_CUDA;
    }
    *out = c;
    return GSVCU_OK;
}

void gsvcu_destroy(gsvcu_ctx* ctx) { delete ctx; }

const char* gsvcu_last_error(const gsvcu_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

int gsvcu_load_gguf(gsvcu_ctx* ctx, const char* path) {
    if (!ctx || !path) return GSVCU_ERR_ARG;
    if (ctx->loaded) return ctx->fail(GSVCU_ERR_STATE, "model already loaded");
    DeviceGuard g(ctx->device);
    const int r = ctx->load(path);
    if (r != GSVCU_OK) {
        for (void* p : ctx->wallocs) cudaFree(p);
        ctx->wallocs.clear();
        ctx->loaded = false;
    }
    return r;
}

int gsvcu_get_hparams(const gsvcu_ctx* ctx, gsvcu_hparams* out) {
    if (!ctx || !out) return GSVCU_ERR_ARG;
    if (!ctx->loaded) return GSVCU_ERR_STATE;
    *out = ctx->hp;
    return GSVCU_OK;
}

int gsvcu_kv_reserve(gsvcu_ctx* ctx, int32_t max_slots, int32_t max_ctx, int32_t kv_dtype) {
    if (!ctx) return GSVCU_ERR_ARG;
    DeviceGuard g(ctx->device);
    if (ctx->inflight) return ctx->fail(GSVCU_ERR_STATE, "kv_reserve while a serving chunk is running");
    return ctx->reserve(max_slots, max_ctx, kv_dtype);
}

int gsvcu_release_cache(gsvcu_ctx* ctx) {
    if (!ctx) return GSVCU_ERR_ARG;
    DeviceGuard g(ctx->device);
    if (ctx->inflight) {
        CKC(ctx, cudaStreamSynchronize(ctx->stream));
        ctx->inflight = false;
    }
    ctx->free_cache();
    return GSVCU_OK;
}

int gsvcu_inspect_gguf(const char* path, gsvcu_hparams* out, char* err, int32_t err_cap) {
    if (!path) return GSVCU_ERR_ARG;
    GgufFile f;
    std::string e;
    int rc = GSVCU_OK;
    ModelView mv;
    if (!f.open(path, e)) rc = GSVCU_ERR_IO;
    else rc = validate_model(f, mv, e);
    if (rc == GSVCU_OK && out) *out = mv.hp;
    if (err && err_cap > 0) {
        std::strncpy(err, e.c_str(), (size_t)err_cap - 1);
        err[err_cap - 1] = 0;
    }
    return rc;
}

int gsvcu_first_logits(gsvcu_ctx* ctx, const gsvcu_request* reqs, int32_t B, float* logits_out) {
    if (!ctx || !reqs || B <= 0 || !logits_out) return GSVCU_ERR_ARG;
    if (!ctx->loaded) return ctx->fail(GSVCU_ERR_STATE, "no model loaded");
    DeviceGuard g(ctx->device);
    TRY(ctx->ensure(B, max_prefix(reqs, B) + 8, ctx->reserved ? ctx->kv_f32 : GSVCU_KV_F16));
    std::vector<int> slots;
    const int rc0 = ctx->admit(reqs, B, nullptr, nullptr, 1, -1, true, nullptr, 0, false, slots, nullptr);
    int rc = rc0;
    const int V = ctx->hp.vocab_size;
    for (int b = 0; b < B && rc == GSVCU_OK; b++) {
        cudaError_t e = cudaMemcpyAsync(logits_out + (size_t)b * V, ctx->logits + (size_t)slots[b] * V, (size_t)V * 4,
                                        cudaMemcpyDeviceToHost, ctx->stream);
        if (e != cudaSuccess) rc = ctx->fail(GSVCU_ERR_CUDA, cudaGetErrorString(e));
    }
    if (rc == GSVCU_OK && cudaStreamSynchronize(ctx->stream) != cudaSuccess) rc = ctx->fail(GSVCU_ERR_CUDA, "sync");
    for (int sl : slots) ctx->release_slot(sl);
    return rc;
}

int gsvcu_generate(gsvcu_ctx* ctx, const gsvcu_request* reqs, int32_t B, const gsvcu_sampler_cfg* sampler,
                   uint64_t seed_base, int32_t early_stop_num, int32_t max_steps, const int32_t* oracle_tokens,
                   int32_t n_oracle, const uint64_t* seeds, int32_t n_seeds, int32_t* tokens_out, int32_t* n_tokens_out,
                   int32_t* lens_out, int32_t cap, gsvcu_progress_fn progress, void* user) {
    if (!ctx || !reqs || B <= 0 || !tokens_out || !n_tokens_out || !lens_out || cap < 0 || max_steps < 1)
        return GSVCU_ERR_ARG;
    if (!ctx->loaded) return ctx->fail(GSVCU_ERR_STATE, "no model loaded");
    DeviceGuard g(ctx->device);
    gsvcu_sampler_cfg sc = sampler ? *sampler : gsvcu_sampler_cfg{15, 1.0f, 1.0f, 1.35f};
    TRY(ctx->ensure(B, max_prefix(reqs, B) + max_steps + 8, ctx->reserved ? ctx->kv_f32 : GSVCU_KV_F16));
    TRY(ctx->set_cfg(sc));
    std::vector<uint64_t> sd(B);
    for (int b = 0; b < B; b++)   // src/gsv_ar.cpp:752-758
        sd[b] = (seeds && b < n_seeds) ? seeds[b] : seed_base + 0x9E3779B9ull * (uint64_t)b;
    std::vector<int> slots;
    int rc = generate_group(ctx, reqs, B, sd.data(), early_stop_num, max_steps, oracle_tokens,
                            oracle_tokens ? n_oracle : 0, false, progress, user, slots);
    if (rc == GSVCU_OK) {
        // results: prompt + generated, lens in finish order (EOS and early stop in step order,
        // then the sequences that ran to max_steps), src/gsv_ar.cpp:780-815
        struct Fin { int idx, kind, b; };
        std::vector<Fin> order;
        std::vector<int32_t> gen((size_t)max_steps);
        for (int b = 0; b < B && rc == GSVCU_OK; b++) {
            const SlotState& s = ctx->h_st[slots[b]];
            const int ns = s.n_samp;
            if (ns > 0) {
                cudaError_t e = cudaMemcpyAsync(gen.data(), ctx->out_tokens + (size_t)slots[b] * ctx->tok_cap,
                                                (size_t)ns * 4, cudaMemcpyDeviceToHost, ctx->stream);
                if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
                if (e != cudaSuccess) { rc = ctx->fail(GSVCU_ERR_CUDA, cudaGetErrorString(e)); break; }
            }
            const int kind = s.finish_kind < 0 ? 2 : s.finish_kind;
            const int keep = kind == 2 ? ns : ns - 1;
            const int P = reqs[b].n_prompt;
            const int total = P + keep;
            n_tokens_out[b] = total;
            int32_t* row = tokens_out + (size_t)b * cap;
            for (int t = 0; t < total && t < cap; t++) row[t] = t < P ? reqs[b].prompt[t] : gen[t - P];
            order.push_back({kind == 2 ? max_steps : s.finish_idx, kind, b});
        }
        if (rc == GSVCU_OK) {
            std::stable_sort(order.begin(), order.end(), [](const Fin& a, const Fin& b) {
                if ((a.kind == 2) != (b.kind == 2)) return b.kind == 2;
                if (a.kind == 2) return a.b < b.b;
                if (a.idx != b.idx) return a.idx < b.idx;
                if (a.kind != b.kind) return a.kind < b.kind;
                return a.b < b.b;
            });
            for (int i = 0; i < B; i++) lens_out[i] = order[i].idx;
        }
    }
    for (int sl : slots) ctx->release_slot(sl);
    return rc;
}

int gsvcu_debug_trace(gsvcu_ctx* ctx, const gsvcu_request* reqs, int32_t B, const int32_t* forced, int32_t n_steps,
                      float* logits_out, float* dump) {
    if (!ctx || !reqs || B <= 0 || n_steps < 0 || !logits_out || (n_steps > 0 && !forced)) return GSVCU_ERR_ARG;
    if (!ctx->loaded) return ctx->fail(GSVCU_ERR_STATE, "no model loaded");
    DeviceGuard g(ctx->device);
    for (int i = 0; i < B * n_steps; i++)
        if (forced[i] == ctx->hp.eos) return ctx->fail(GSVCU_ERR_ARG, "trace tokens must not be EOS");
    TRY(ctx->ensure(B, max_prefix(reqs, B) + n_steps + 8, ctx->reserved ? ctx->kv_f32 : GSVCU_KV_F16));
    std::vector<uint64_t> sd(B, 1);
    std::vector<int> slots;
    TRY(ctx->admit(reqs, B, sd.data(), nullptr, n_steps + 1, -1, true, forced, n_steps, true, slots, dump));
    const int V = ctx->hp.vocab_size;
    auto fetch_logits = [&](int row) -> int {   // ordered after the step on the context's stream
        for (int b = 0; b < B; b++)
            CKC(ctx, cudaMemcpyAsync(logits_out + ((size_t)row * B + b) * V, ctx->logits + (size_t)slots[b] * V,
                                     (size_t)V * 4, cudaMemcpyDeviceToHost, ctx->stream));
        CKC(ctx, cudaStreamSynchronize(ctx->stream));
        return GSVCU_OK;
    };
    int rc = fetch_logits(0);
    for (int s = 0; s < n_steps && rc == GSVCU_OK; s++) {
        if (dump) rc = ctx->launch_step(ctx->stream, dump, s + 1, slots.data(), B);   // instrumented, no graph
        else rc = ctx->run_steps(1);
        if (rc != GSVCU_OK) break;
        if (cudaGetLastError() != cudaSuccess) { rc = ctx->fail(GSVCU_ERR_CUDA, "kernel launch failed"); break; }
        rc = fetch_logits(s + 1);
    }
    if (rc == GSVCU_OK && cudaStreamSynchronize(ctx->stream) != cudaSuccess) rc = ctx->fail(GSVCU_ERR_CUDA, "sync");
    for (int sl : slots) ctx->release_slot(sl);
    return rc;
}

int gsvcu_serve_admit(gsvcu_ctx* ctx, const gsvcu_request* reqs, int32_t n, const gsvcu_sampler_cfg* sampler,
                      const uint64_t* seeds, const int32_t* tags, int32_t max_steps, int32_t early_stop_num) {
    if (!ctx || (!reqs && n > 0) || n < 0) return GSVCU_ERR_ARG;
    if (!ctx->loaded) return ctx->fail(GSVCU_ERR_STATE, "no model loaded");
    if (!ctx->reserved) return ctx->fail(GSVCU_ERR_STATE, "call gsvcu_kv_reserve before serving");
    DeviceGuard g(ctx->device);
    gsvcu_sampler_cfg sc = sampler ? *sampler : gsvcu_sampler_cfg{15, 1.0f, 1.0f, 1.35f};
    TRY(ctx->set_cfg(sc));
    std::vector<int> slots;
    return ctx->admit(reqs, n, seeds, tags, max_steps, early_stop_num, false, nullptr, 0, false, slots, nullptr);
}

int gsvcu_serve_step(gsvcu_ctx* ctx, int32_t n_steps, gsvcu_finished* done, int32_t max_done, int32_t* tokens,
                     int32_t tok_cap) {
    if (!ctx || n_steps < 0 || max_done < 0 || (max_done > 0 && !done)) return GSVCU_ERR_ARG;
    if (!ctx->reserved) return ctx->fail(GSVCU_ERR_STATE, "no KV pool reserved");
    DeviceGuard g(ctx->device);
    bool any = false;
    for (char u : ctx->slot_used) any |= u != 0;
    if (!any && !ctx->inflight) return 0;
    if (ctx->lookahead && !ctx->inflight) {
        // nothing running yet: start the first chunk and report nothing
        if (n_steps > 0) {
            TRY(ctx->run_steps(n_steps));
            ctx->inflight = true;
        }
        return 0;
    }
    if (!ctx->lookahead && n_steps > 0) TRY(ctx->run_steps(n_steps));
    TRY(ctx->read_status());   // with lookahead: the chunk started by the previous call
    ctx->inflight = false;
    int nd = 0, used = 0;
    for (int sl = 0; sl < ctx->max_slots; sl++) {
        if (!ctx->slot_used[sl]) continue;
        const SlotState& s = ctx->h_st[sl];
        if (s.active || s.finish_kind < 0) continue;
        if (nd >= max_done) break;
        const int keep = s.finish_kind == 2 ? s.n_samp : s.n_samp - 1;
        gsvcu_finished& f = done[nd++];
        f.slot = sl;
        f.tag = ctx->slot_tag[sl];
        f.finish_kind = s.finish_kind;
        f.n_generated = s.finish_kind == 2 ? s.max_steps : s.finish_idx;
        f.n_tokens = 0;
        if (tokens && keep > 0 && used + keep <= tok_cap) {   // copied below, one synchronisation for all
            CKC(ctx, cudaMemcpyAsync(tokens + used, ctx->out_tokens + (size_t)sl * ctx->tok_cap, (size_t)keep * 4,
                                     cudaMemcpyDeviceToHost, ctx->stream));
            f.n_tokens = keep;
            used += keep;
        }
        ctx->tokens_done += keep;
    }
    if (used) CKC(ctx, cudaStreamSynchronize(ctx->stream));
    for (int i = 0; i < nd; i++) ctx->release_slot(done[i].slot);
    if (ctx->lookahead && n_steps > 0) {
        bool active = false;
        for (int sl = 0; sl < ctx->max_slots; sl++) active |= ctx->slot_used[sl] && ctx->h_st[sl].active;
        if (active) {   // the next chunk runs while the caller handles these results and admits
            TRY(ctx->run_steps(n_steps));
            ctx->inflight = true;
        }
    }
    return nd;
}

int gsvcu_set_serve_lookahead(gsvcu_ctx* ctx, int32_t on) {
    if (!ctx) return GSVCU_ERR_ARG;
    DeviceGuard g(ctx->device);
    if (ctx->inflight) {   // finish the running chunk under the old rule; its results are reported next call
        CKC(ctx, cudaStreamSynchronize(ctx->stream));
    }
    ctx->lookahead = on != 0;
    if (!ctx->lookahead) ctx->inflight = false;
    return GSVCU_OK;
}

int gsvcu_serve_active(const gsvcu_ctx* ctx) {
    if (!ctx) return GSVCU_ERR_ARG;
    int n = 0;
    for (char u : ctx->slot_used) n += u != 0;
    return n;
}

int64_t gsvcu_serve_tokens_total(const gsvcu_ctx* ctx) {
    if (!ctx) return GSVCU_ERR_ARG;
    int64_t t = ctx->tokens_done;
    for (int sl = 0; sl < (int)ctx->slot_used.size(); sl++)
        if (ctx->slot_used[sl]) t += ctx->h_st[sl].n_samp;
    return t;
}

// ------------------------------------------------------------------ kernel-level entry points
int gsvcu_op_quantize_q8_0(gsvcu_ctx* ctx, const float* x_dev, int32_t rows, int32_t K, int8_t* q_dev, uint16_t* d_dev) {
    if (!ctx || !x_dev || !q_dev || !d_dev || rows < 0 || K <= 0 || K % QK) return GSVCU_ERR_ARG;
    DeviceGuard g(ctx->device);
    launch_quantize_q8(x_dev, rows, K, q_dev, d_dev, ctx->stream);
    CKC(ctx, cudaGetLastError());
    return GSVCU_OK;
}

int gsvcu_op_pack_q8_0(gsvcu_ctx* ctx, const uint8_t* raw_host, int32_t N, int32_t K, void* wq_dev, void* wd_dev) {
    if (!ctx || !raw_host || !wq_dev || !wd_dev || N <= 0 || K <= 0 || N % 32 || K % QK) return GSVCU_ERR_ARG;
    DeviceGuard g(ctx->device);
    std::vector<uint8_t> wq((size_t)N * K);
    std::vector<uint16_t> wd((size_t)N * K / QK);
    pack_q8_0_host(raw_host, N, K, wq.data(), wd.data());
    CKC(ctx, cudaMemcpy(wq_dev, wq.data(), wq.size(), cudaMemcpyHostToDevice));
    CKC(ctx, cudaMemcpy(wd_dev, wd.data(), wd.size() * 2, cudaMemcpyHostToDevice));
    return GSVCU_OK;
}

int gsvcu_op_q8_gemm(gsvcu_ctx* ctx, const int8_t* xq_dev, const uint16_t* xd_dev, int32_t M, const void* wq_dev,
                     const void* wd_dev, int32_t N, int32_t K, const float* bias_dev, const float* resid_dev, int32_t epi,
                     float* y_dev, int8_t* yq_dev, uint16_t* yd_dev) {
    if (!ctx || !xq_dev || !xd_dev || !wq_dev || !wd_dev || M <= 0 || N <= 0 || N % 32 || (K != 512 && K != 2048))
        return GSVCU_ERR_ARG;
    if (epi < 0 || epi > 2 || (epi < 2 && !y_dev) || (epi == 1 && !resid_dev) || (epi == 2 && (!yq_dev || !yd_dev)))
        return GSVCU_ERR_ARG;
    DeviceGuard g(ctx->device);
    GemmQ8Params p;
    p.xq = xq_dev; p.xd = xd_dev; p.M = M; p.wq = (const uint4*)wq_dev; p.wd = (const uint16_t*)wd_dev; p.N = N; p.K = K;
    p.bias = bias_dev; p.resid = resid_dev; p.y = y_dev; p.yq = yq_dev; p.yd = yd_dev;
    launch_gemm_q8(p, epi, ctx->stream);
    CKC(ctx, cudaGetLastError());
    return GSVCU_OK;
}

int gsvcu_op_pack_q8_0_f16(gsvcu_ctx* ctx, const uint8_t* raw_host, int32_t N, int32_t K, void* w16_dev) {
    if (!ctx || !raw_host || !w16_dev || N <= 0 || K <= 0 || K % QK) return GSVCU_ERR_ARG;
    DeviceGuard g(ctx->device);
    std::vector<uint16_t> h((size_t)N * K);
    for (size_t r = 0; r < (size_t)N; r++)
        for (int kb = 0; kb < K / QK; kb++)
            for (int j = 0; j < QK; j++)
                h[r * K + kb * QK + j] = i8_as_f16_bits((int8_t)raw_host[(r * (K / QK) + kb) * 34 + 2 + j]);
    CKC(ctx, cudaMemcpy(w16_dev, h.data(), h.size() * 2, cudaMemcpyHostToDevice));
    return GSVCU_OK;
}

int gsvcu_op_q8_gemm_tc(gsvcu_ctx* ctx, const int8_t* xq_dev, const uint16_t* xd_dev, int32_t M, const void* w16_dev,
                        const void* wd_dev, int32_t N, int32_t K, const float* bias_dev, const float* resid_dev,
                        int32_t epi, float* y_dev, int8_t* yq_dev, uint16_t* yd_dev) {
    if (!ctx || !xq_dev || !xd_dev || !w16_dev || !wd_dev || M <= 0 || N <= 0 || N % 128 || K % 64 || K > 2048 ||
        ((uintptr_t)xq_dev & 15) || ((uintptr_t)w16_dev & 15))
        return GSVCU_ERR_ARG;
    if (epi < 0 || epi > 2 || (epi < 2 && !y_dev) || (epi == 1 && !resid_dev) || (epi == 2 && (!yq_dev || !yd_dev)))
        return GSVCU_ERR_ARG;
    DeviceGuard g(ctx->device);
    const size_t need = tc_scratch_bytes(M, N, K);
    if (need > ctx->op_a16_n) {
        if (ctx->op_a16) {
            cudaStreamSynchronize(ctx->stream);
            cudaFree(ctx->op_a16);
        }
        ctx->op_a16 = nullptr;
        ctx->op_a16_n = 0;
        CKC(ctx, cudaMalloc(&ctx->op_a16, need));
        ctx->op_a16_n = need;
    }
    GemmQ8Params p;
    p.xq = xq_dev; p.xd = xd_dev; p.M = M; p.wd = (const uint16_t*)wd_dev; p.N = N; p.K = K;
    p.bias = bias_dev; p.resid = resid_dev; p.y = y_dev; p.yq = yq_dev; p.yd = yd_dev;
    p.w16 = (const __half*)w16_dev; p.tc_scratch = ctx->op_a16; p.tc_scratch_n = ctx->op_a16_n;
    p.err = ctx->att_err + 1;
    if (!gemm_tc_usable(p)) return ctx->fail(GSVCU_ERR_ARG, "tensor-core GEMM not usable for this shape / driver");
    if (!launch_gemm_q8_tc(p, epi, ctx->stream)) return ctx->fail(GSVCU_ERR_CUDA, "tensor map encoding failed");
    CKC(ctx, cudaGetLastError());
    return GSVCU_OK;
}

int gsvcu_op_layernorm_q8(gsvcu_ctx* ctx, const float* v_dev, int32_t rows, const float* w_dev, const float* b_dev,
                          float* y_dev, int8_t* yq_dev, uint16_t* yd_dev) {
    if (!ctx || !v_dev || !w_dev || !b_dev || !y_dev || !yq_dev || !yd_dev || rows < 0) return GSVCU_ERR_ARG;
    DeviceGuard g(ctx->device);
    launch_layernorm_q8(v_dev, rows, w_dev, b_dev, y_dev, yq_dev, yd_dev, ctx->stream);
    CKC(ctx, cudaGetLastError());
    return GSVCU_OK;
}

int gsvcu_op_f32_gemm(gsvcu_ctx* ctx, const float* x_dev, int32_t M, const float* w_dev, int32_t N, int32_t K,
                      const float* add_dev, float* y_dev) {
    if (!ctx || !x_dev || !w_dev || !y_dev || M < 0 || N <= 0 || K <= 0) return GSVCU_ERR_ARG;
    DeviceGuard g(ctx->device);
    launch_gemm_f32d(x_dev, K, nullptr, M, w_dev, N, K, add_dev, N, y_dev, N, ctx->stream);
    CKC(ctx, cudaGetLastError());
    return GSVCU_OK;
}

int gsvcu_op_fx_gemm(gsvcu_ctx* ctx, const float* x_dev, int32_t M, const void* w_dev, int32_t wtype, int32_t N,
                     int32_t K, const float* bias_dev, float* y_dev) {
    if (!ctx || !x_dev || !w_dev || !y_dev || M < 0 || N <= 0 || K <= 0 || K % 256 || wtype < 0 || wtype > 2 ||
        ((uintptr_t)x_dev & 15) || ((uintptr_t)w_dev & 15))
        return GSVCU_ERR_ARG;
    DeviceGuard g(ctx->device);
    GemmFxParams p;
    p.x = x_dev; p.ldx = K; p.M = M; p.w = w_dev; p.wtype = wtype; p.N = N; p.K = K;
    p.bias = bias_dev; p.y = y_dev;
    launch_gemm_fx(p, FXE_BIAS, ctx->stream);
    CKC(ctx, cudaGetLastError());
    return GSVCU_OK;
}

int gsvcu_op_decode_attention(gsvcu_ctx* ctx, const float* q_dev, int32_t q_stride, const void* pool_dev,
                              int32_t kv_dtype, int32_t n_layer, int32_t layer, const int32_t* block_table_dev,
                              int32_t max_pages, const int32_t* kvpos_dev, const int32_t* active_dev, int32_t B,
                              int8_t* out_q_dev, uint16_t* out_d_dev, float* out_f32_dev) {
    if (!ctx || !q_dev || !pool_dev || !block_table_dev || !kvpos_dev || !active_dev || !out_q_dev || !out_d_dev ||
        B <= 0 || max_pages <= 0 || n_layer <= 0 || layer < 0 || layer >= n_layer || q_stride < D ||
        (kv_dtype != GSVCU_KV_F16 && kv_dtype != GSVCU_KV_F32) || !decode_attention_aligned(q_dev, q_stride, pool_dev,
                                                                                            out_q_dev, out_f32_dev))
        return GSVCU_ERR_ARG;
    DeviceGuard g(ctx->device);
    const int max_chunks = decode_chunks(max_pages * PAGE);
    const size_t need_part = (size_t)B * NH * max_chunks * PART_STRIDE;
    if (need_part > ctx->op_part_n) {
        if (ctx->op_part) {
            cudaStreamSynchronize(ctx->stream);
            cudaFree(ctx->op_part);
        }
        ctx->op_part = nullptr;
        ctx->op_part_n = 0;
        CKC(ctx, cudaMalloc((void**)&ctx->op_part, need_part * 4));
        ctx->op_part_n = need_part;
    }
    DecAttnParams a;
    a.q = q_dev; a.q_stride = q_stride; a.pool = pool_dev; a.kv_f32 = kv_dtype; a.n_layer = n_layer; a.layer = layer;
    a.block_table = block_table_dev; a.max_pages = max_pages; a.kvpos = kvpos_dev; a.active = active_dev; a.B = B;
    a.max_chunks = max_chunks; a.scale = 1.0f / std::sqrt((float)HD); a.out_q = out_q_dev; a.out_d = out_d_dev;
    a.out_f32 = out_f32_dev; a.part = ctx->op_part; a.err = ctx->att_err + 1;
    a.fault_extra_tx = ctx->fault_extra_tx; a.poll_limit = ctx->fault_poll_limit;
    a.part_ml = part_ml_of(ctx->op_part, (size_t)B * NH * max_chunks);
    launch_decode_attention(a, ctx->stream);
    CKC(ctx, cudaGetLastError());
    return GSVCU_OK;
}

int gsvcu_op_prefill_attention(gsvcu_ctx* ctx, const float* qkv_dev, int32_t n_seq, const int32_t* seq_start,
                               const int32_t* seq_len, const int32_t* text_len, int8_t* out_q_dev, uint16_t* out_d_dev,
                               float* out_f32_dev) {
    if (!ctx || !qkv_dev || n_seq <= 0 || !seq_start || !seq_len || !text_len || !out_q_dev || !out_d_dev)
        return GSVCU_ERR_ARG;
    DeviceGuard g(ctx->device);
    std::vector<PrefillTile> tiles;
    for (int i = 0; i < n_seq; i++) {
        if (seq_len[i] <= 0 || text_len[i] < 0 || text_len[i] > seq_len[i]) return GSVCU_ERR_ARG;
        for (int q0 = 0; q0 < seq_len[i]; q0 += PREF_QTILE) tiles.push_back({i, q0});
    }
    std::vector<int32_t> tab((size_t)3 * n_seq);
    std::memcpy(tab.data(), seq_start, (size_t)n_seq * 4);
    std::memcpy(tab.data() + n_seq, seq_len, (size_t)n_seq * 4);
    std::memcpy(tab.data() + 2 * n_seq, text_len, (size_t)n_seq * 4);
    const size_t tab_bytes = ((size_t)n_seq * 12 + 15) / 16 * 16;
    uint8_t* blk = nullptr;
    CKC(ctx, cudaMalloc((void**)&blk, tab_bytes + tiles.size() * sizeof(PrefillTile)));
    cudaMemcpyAsync(blk, tab.data(), (size_t)n_seq * 12, cudaMemcpyHostToDevice, ctx->stream);
    cudaMemcpyAsync(blk + tab_bytes, tiles.data(), tiles.size() * sizeof(PrefillTile), cudaMemcpyHostToDevice,
                    ctx->stream);
    PrefAttnParams a;
    a.qkv = qkv_dev;
    a.seq_start = (const int32_t*)blk;
    a.seq_len = a.seq_start + n_seq;
    a.text_len = a.seq_len + n_seq;
    a.tiles = (const PrefillTile*)(blk + tab_bytes);
    a.n_tiles = (int)tiles.size();
    a.scale = 1.0f / std::sqrt((float)HD);
    a.out_q = out_q_dev; a.out_d = out_d_dev; a.out_f32 = out_f32_dev;
    launch_prefill_attention(a, ctx->stream);
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    cudaFree(blk);
    if (e != cudaSuccess) return ctx->fail(GSVCU_ERR_CUDA, cudaGetErrorString(e));
    return GSVCU_OK;
}

int gsvcu_op_sample(gsvcu_ctx* ctx, const float* logits_dev, int32_t B, int32_t V, int32_t eos,
                    const gsvcu_sampler_cfg* cfg, const int32_t* prev_host, const int32_t* n_prev_host,
                    int32_t prev_stride, const int32_t* step_host, uint64_t* rng_host, int32_t* tokens_host) {
    if (!ctx || !logits_dev || B <= 0 || V < 2 || V > 1280 || eos < 0 || eos >= V || !cfg || !step_host || !rng_host ||
        !tokens_host || (prev_host && (!n_prev_host || prev_stride <= 0)))
        return GSVCU_ERR_ARG;
    DeviceGuard g(ctx->device);
    int cap = 1;
    for (int b = 0; b < B; b++) {
        if (step_host[b] < 0) return GSVCU_ERR_ARG;
        cap = std::max(cap, step_host[b] + 1);
    }
    const int dpl = (V + 31) / 32;
    std::vector<uint64_t> jm = jump_matrices(dpl);
    std::vector<SlotState> hs(B);
    std::vector<uint16_t> cnt((size_t)B * V, 0);
    std::vector<int32_t> ring((size_t)B * HIST, 0);
    for (int b = 0; b < B; b++) {
        SlotState& ss = hs[b];
        ss = SlotState{};
        ss.active = 1;
        ss.n_samp = step_host[b];
        ss.max_steps = cap + 1;
        ss.early_stop = -1;
        ss.group_first = b;
        ss.finish_kind = -1;
        ss.rng = rng_host[b];
        ss.top_k = cfg->top_k;
        ss.top_p = cfg->top_p;
        ss.temperature = cfg->temperature;
        ss.rep = cfg->repetition_penalty;
        const int np = prev_host ? n_prev_host[b] : 0;
        if (np < 0 || np > prev_stride * (prev_host != nullptr)) return GSVCU_ERR_ARG;
        const int nh = std::min(np, HIST);
        for (int i = 0; i < nh; i++) {
            const int t = prev_host[(size_t)b * prev_stride + (np - nh) + i];
            ring[(size_t)b * HIST + i] = t;
            if (t >= 0 && t < V) cnt[(size_t)b * V + t]++;
        }
        ss.hist_len = nh;
    }
    // one device block: states | counts | ring | tokens | jump
    const size_t o_st = 0, o_cnt = o_st + sizeof(SlotState) * B, o_ring = (o_cnt + (size_t)B * V * 2 + 15) / 16 * 16,
                 o_tok = o_ring + (size_t)B * HIST * 4, o_jump = (o_tok + (size_t)B * cap * 4 + 15) / 16 * 16,
                 total = o_jump + jm.size() * 8;
    uint8_t* blk = nullptr;
    CKC(ctx, cudaMalloc((void**)&blk, total));
    cudaStream_t s = ctx->stream;
    cudaMemcpyAsync(blk + o_st, hs.data(), sizeof(SlotState) * B, cudaMemcpyHostToDevice, s);
    cudaMemcpyAsync(blk + o_cnt, cnt.data(), cnt.size() * 2, cudaMemcpyHostToDevice, s);
    cudaMemcpyAsync(blk + o_ring, ring.data(), ring.size() * 4, cudaMemcpyHostToDevice, s);
    cudaMemcpyAsync(blk + o_jump, jm.data(), jm.size() * 8, cudaMemcpyHostToDevice, s);
    SamplerParams sp;
    sp.logits = logits_dev; sp.V = V; sp.eos = eos; sp.nslots = B;
    sp.st = (SlotState*)(blk + o_st); sp.counts = (uint16_t*)(blk + o_cnt); sp.hist = (int32_t*)(blk + o_ring);
    sp.out_tokens = (int32_t*)(blk + o_tok); sp.tok_cap = cap; sp.jump = (const uint64_t*)(blk + o_jump);
    sp.draws_per_lane = dpl;
    launch_sampler(sp, s);
    cudaMemcpyAsync(hs.data(), blk + o_st, sizeof(SlotState) * B, cudaMemcpyDeviceToHost, s);
    std::vector<int32_t> toks((size_t)B * cap);
    cudaMemcpyAsync(toks.data(), blk + o_tok, toks.size() * 4, cudaMemcpyDeviceToHost, s);
    cudaError_t e = cudaStreamSynchronize(s);
    cudaFree(blk);
    if (e != cudaSuccess) return ctx->fail(GSVCU_ERR_CUDA, cudaGetErrorString(e));
    for (int b = 0; b < B; b++) {
        tokens_host[b] = toks[(size_t)b * cap + step_host[b]];
        rng_host[b] = hs[b].rng;
    }
    return GSVCU_OK;
}

void* gsvcu_stream(const gsvcu_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

int64_t gsvcu_kernel_launches(const gsvcu_ctx* ctx) { return ctx ? ctx->launches : (int64_t)GSVCU_ERR_ARG; }

int gsvcu_serve_reset(gsvcu_ctx* ctx) {
    if (!ctx) return GSVCU_ERR_ARG;
    if (!ctx->reserved) return GSVCU_OK;
    DeviceGuard g(ctx->device);
    CKC(ctx, cudaStreamSynchronize(ctx->stream));
    ctx->inflight = false;
    for (int sl = 0; sl < ctx->max_slots; sl++)
        if (ctx->slot_used[sl]) ctx->release_slot(sl);
    CKC(ctx, cudaMemsetAsync(ctx->st, 0, sizeof(SlotState) * ctx->max_slots, ctx->stream));
    for (auto& s : ctx->h_st) s = SlotState{};
    CKC(ctx, cudaStreamSynchronize(ctx->stream));
    return GSVCU_OK;
}

int gsvcu_step_profile(gsvcu_ctx* ctx, int32_t n_steps, float* ms_by_class, int64_t* attn_bytes) {
    if (!ctx || n_steps <= 0 || !ms_by_class) return GSVCU_ERR_ARG;
    if (!ctx->reserved) return ctx->fail(GSVCU_ERR_STATE, "no KV pool reserved");
    DeviceGuard g(ctx->device);
    for (int c = 0; c < GSVCU_PROF_CLASSES; c++) ms_by_class[c] = 0.f;
    int64_t bytes = 0;
    if (!ctx->prof_ev[0]) {
        CKC(ctx, cudaEventCreate(&ctx->prof_ev[0]));
        CKC(ctx, cudaEventCreate(&ctx->prof_ev[1]));
    }
    const size_t elem = ctx->kv_f32 ? 4 : 2;
    for (int i = 0; i < n_steps; i++) {
        TRY(ctx->read_status());
        // keys each decoding slot will read in this step: kvlen + 1 (the token appended by the step)
        for (int sl = 0; sl < ctx->max_slots; sl++) {
            const SlotState& s = ctx->h_st[sl];
            // (a slot that samples EOS this step is counted too; it skips attention, a negligible over-count)
            const bool will_decode = ctx->slot_used[sl] && s.active && s.n_samp + 1 < s.max_steps;
            // per layer: K and V rows of every key, q in (f32), Q8_0 output (512 B + 16 fp16 scales)
            if (will_decode)
                bytes += ((int64_t)(s.kvlen + 1) * 2 * D * elem + (int64_t)D * 4 + D + (D / QK) * 2) * ctx->hp.n_layer;
        }
        ctx->prof_ms = ms_by_class;
        const int rc = ctx->launch_step(ctx->stream);
        ctx->prof_ms = nullptr;
        if (rc != GSVCU_OK) return rc;
        ctx->launches += ctx->graph_kernels;
    }
    CKC(ctx, cudaStreamSynchronize(ctx->stream));
    if (attn_bytes) *attn_bytes = bytes;
    return GSVCU_OK;
}

int gsvcu_set_fused_decode(gsvcu_ctx* ctx, int32_t mode) {
    if (!ctx || mode < 0 || mode > 2) return GSVCU_ERR_ARG;
    DeviceGuard g(ctx->device);
    const bool fused = mode != 0, two = mode == 2;
    if ((ctx->fused != fused || ctx->two_groups != two) && (ctx->graph || ctx->graph_chunk)) {
        cudaStreamSynchronize(ctx->stream);   // the captured steps are the other variant
        ctx->drop_graphs();
    }
    ctx->fused = fused;
    ctx->two_groups = two;
    return GSVCU_OK;
}

int gsvcu_fused_decode(const gsvcu_ctx* ctx) {
    if (!ctx || !ctx->fused || !ctx->dense_ok || !ctx->all_q8) return 0;   // float layer matrices: unfused step
    return ctx->two_groups ? 2 : 1;
}

int gsvcu_sync(gsvcu_ctx* ctx) {
    if (!ctx) return GSVCU_ERR_ARG;
    DeviceGuard g(ctx->device);
    int32_t oerr = 0;
    CKC(ctx, cudaMemcpyAsync(&oerr, ctx->att_err + 1, sizeof(oerr), cudaMemcpyDeviceToHost, ctx->stream));
    CKC(ctx, cudaStreamSynchronize(ctx->stream));
    if (oerr) {
        CKC(ctx, cudaMemsetAsync(ctx->att_err + 1, 0, sizeof(int32_t), ctx->stream));
        CKC(ctx, cudaStreamSynchronize(ctx->stream));
        return ctx->fail(GSVCU_ERR_CUDA, "gsvcu_op_decode_attention: staged K/V never arrived (bounded wait gave up)");
    }
    return GSVCU_OK;
}

int gsvcu_set_prefill_gemm(gsvcu_ctx* ctx, int32_t mode) {
    if (!ctx || mode < 0 || mode > 1) return GSVCU_ERR_ARG;
    ctx->tc_prefill = mode == 1;
    return GSVCU_OK;
}

int gsvcu_set_wait_fault(gsvcu_ctx* ctx, int32_t on) {
    if (!ctx || on < 0 || on > 1) return GSVCU_ERR_ARG;
    DeviceGuard g(ctx->device);
    CKC(ctx, cudaStreamSynchronize(ctx->stream));
    ctx->drop_graphs();   // captured steps hold the launch parameters
    ctx->fault_extra_tx = on ? 16u : 0u;
    ctx->fault_poll_limit = on ? 4096u : 0u;
    return GSVCU_OK;
}

}  // extern "C"
