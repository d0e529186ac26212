// gsv_ar_oracle.cpp -- TEST INFRASTRUCTURE ONLY (the parity checker, never the product).
//
// A CPU restatement of the reference AR path of gsv.cpp (GPT-SoVITS Text2SemanticDecoder):
// prefill with the text-bidirectional / semantic-causal prefix mask, KV-cached decode, the
// sampler and the generate loop, with the arithmetic of the ggml CPU ops the reference calls.
// Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference leg may
// load this library. The CUDA library never links it, calls it or falls back to it.
//
// Reference citations are paths inside the gsv.cpp project. "P:<n>" is a line of
// patches/0001-ggml-audio-patch-port-on-llamacpp.patch.
//
// ggml itself (llama.cpp f0c41e0168dfd4b5ef72b21d1a311b24cc7a894a) is not shipped with the
// reference. The op semantics restated here are ggml's portable C paths:
//   * Q8_0 mul_mat: src1 rows quantized with quantize_row_q8_0_ref semantics (d = amax/127,
//     id = 1/d, roundf, d stored as fp16) -- pinned bit-exactly against gguf-py's Q8_0
//     quantizer, which documents bit-exactness with ggml-quants.c; then per 32-block integer dot,
//     accumulated in float block by block as sumf = fma((float)sumi, d_w*d_x, sumf).
//   * F32 mul_mat of ar.predict and of the BERT projection: products exact in double, accumulated
//     in double, rounded once (ggml_vec_dot_f32; its scalar path rounds each product to float, its
//     FMA-vectorised path accumulates in float: both within roundings of this).
//   * F32 / F16 / BF16 layer matrices and an F16 / BF16 ar.predict: ggml's FMA-vectorised dot
//     (-mavx2 -mfma; ggml_vec_dot_f32 / ggml_vec_dot_f16 with 4 accumulators x 8 float lanes): src1
//     rounded to F16 / BF16 for an F16 / BF16 matrix (ggml's vec_dot_type; BF16 takes the F16 order),
//     32 float FMA chains (chain c takes k = c, c+32, ...),
//     folded as accumulators 0+2, 1+3, then 0+1, then the two 128-bit halves, then two horizontal
//     adds -- i.e. chains c and c^16, ^8, ^4, ^1, ^2 added pairwise in that order (vec_dot_canon).
//   * flash_attn_ext (F32 K/V), prefill rows: scores s = (float)(double sum of the exact products
//     q_e*k_e) * scale (the products are exact as in the FMA-vectorised ggml_vec_dot_f32 of the
//     -mavx2 -mfma build), masked keys skipped; softmax(s) V evaluated in double (double exp, double
//     sums) and rounded once (an order-independent evaluation of ggml's float online softmax, see
//     attn_row).
//   * flash_attn_ext, decode rows: float arithmetic in a fixed page-split order with an own float exp
//     (decode_attention_canonical), the evaluation order of the library's decode kernel.
//   * layernorm_affine (P:1535-1585): v = (x + r) + bias, mean / E[v^2] in double,
//     var = E[v^2] - mean^2, inv = 1/sqrtf(var + eps), y = ((v - mean)*inv)*w + b.
//   * Q4_1 / Q5_1 mul_mat: src1 quantized to Q8_1 (the Q8_0 values and scale plus s = fp16(sum * d)),
//     per block sumf = sumf + fma(d_w*d_x, sumi, m_w*s_x) (ggml's portable vec_dot_q4_1_q8_1 as GCC
//     contracts it).
//   * add_act ReLU (P:1587-1620): y = max(a + b, 0).
// Where the reference's C++ is compiled with -mavx2 -mfma (CMakeLists.txt:88-92) GCC contracts
// a*b+c into an FMA; the restatement writes those FMAs out with fmaf() and is itself compiled
// with -ffp-contract=off so nothing else is fused.

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <numeric>
#include <string>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif
#include <immintrin.h>

namespace {

// ------------------------------------------------------------------ fp16
// IEEE binary32 -> binary16 with round-to-nearest-even (what GGML_FP32_TO_FP16 does via F16C).
inline uint16_t f32_to_f16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t mant = x & 0x7fffffu;
    const int32_t exp = (int32_t)((x >> 23) & 0xffu);
    if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | (mant ? (0x200u | (mant >> 13)) : 0u));
    const int32_t e = exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        const int shift = 14 - e;
        uint32_t h = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1u);
        const uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)h;
}

inline float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x3ffu;
    uint32_t x;
    if (exp == 0) {
        if (mant == 0) {
            x = sign;
        } else {
            int e = -1;
            do { mant <<= 1; e++; } while (!(mant & 0x400u));
            mant &= 0x3ffu;
            x = sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
        }
    } else if (exp == 31) {
        x = sign | 0x7f800000u | (mant << 13);
    } else {
        x = sign | ((exp - 15 + 127) << 23) | (mant << 13);
    }
    float f;
    std::memcpy(&f, &x, 4);
    return f;
}

inline float round_f16(float f) { return f16_to_f32(f32_to_f16(f)); }

// ------------------------------------------------------------------ Q8_0
constexpr int QK = 32;
constexpr int QKK = 256;   // K-quant super-block
constexpr int Q8_BYTES = 34;   // fp16 d + 32 x int8

// quantize_row_q8_0_ref semantics (ggml-quants.c; pinned via gguf-py's Q8_0 quantizer).
void quantize_q8_0(const float* x, int64_t n, uint8_t* blocks) {
    const int64_t nb = n / QK;
    for (int64_t i = 0; i < nb; i++) {
        float amax = 0.0f;
        for (int j = 0; j < QK; j++) amax = std::max(amax, std::fabs(x[i * QK + j]));
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint8_t* b = blocks + i * Q8_BYTES;
        const uint16_t dh = f32_to_f16(d);
        std::memcpy(b, &dh, 2);
        for (int j = 0; j < QK; j++) {
            const float v = x[i * QK + j] * id;
            b[2 + j] = (uint8_t)(int8_t)std::roundf(v);
        }
    }
}

// quantize_row_q8_1_ref (the src1 conversion of ggml's Q4_1 / Q5_1 mul_mat): the Q8_0 values and
// scale, plus s = fp16(sum of the 32 values * d) with the unrounded d. Returns the values [n], the
// fp16-rounded d and s of each block as floats.
void quantize_q8_1(const float* x, int64_t n, int8_t* q, float* d_out, float* s_out) {
    for (int64_t i = 0; i < n / QK; i++) {
        float amax = 0.0f;
        for (int j = 0; j < QK; j++) amax = std::max(amax, std::fabs(x[i * QK + j]));
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        int sum = 0;
        for (int j = 0; j < QK; j++) {
            const int v = (int)std::roundf(x[i * QK + j] * id);
            q[i * QK + j] = (int8_t)v;
            sum += v;
        }
        d_out[i] = f16_to_f32(f32_to_f16(d));
        s_out[i] = f16_to_f32(f32_to_f16((float)sum * d));
    }
}

// quantize_row_q8_K_ref (the src1 conversion of ggml's K-quant mul_mat), per 256 values: max = the
// value of largest magnitude (first one wins), iscale = -127/max, q = min(127, nearest_int(iscale*x))
// (round half to even), d = 1/iscale (0, q = 0 for an all-zero block), bsums = sums of 16 values.
void quantize_q8_k(const float* x, int64_t n, int8_t* q, float* d_out, int32_t* bsums) {
    for (int64_t i = 0; i < n / QKK; i++) {
        const float* xb = x + i * QKK;
        float amax = 0.0f, mx = 0.0f;
        for (int j = 0; j < QKK; j++)
            if (std::fabs(xb[j]) > amax) {
                amax = std::fabs(xb[j]);
                mx = xb[j];
            }
        if (amax == 0.0f) {
            d_out[i] = 0.0f;
            for (int j = 0; j < QKK; j++) q[i * QKK + j] = 0;
        } else {
            const float iscale = -127.0f / mx;
            for (int j = 0; j < QKK; j++) q[i * QKK + j] = (int8_t)std::min(127, (int)std::nearbyint(iscale * xb[j]));
            d_out[i] = 1.0f / iscale;
        }
        for (int g = 0; g < QKK / 16; g++) {
            int s = 0;
            for (int j = 0; j < 16; j++) s += q[i * QKK + g * 16 + j];
            bsums[i * (QKK / 16) + g] = s;
        }
    }
}

// fp16 -> f32 of every bit pattern, tabulated once from f16_to_f32 (same values, no per-call work).
const float* f16_table() {
    static const std::vector<float> t = [] {
        std::vector<float> v(65536);
        for (uint32_t h = 0; h < 65536; h++) v[h] = f16_to_f32((uint16_t)h);
        return v;
    }();
    return t.data();
}

inline float q8_d(const uint8_t* blk) {
    uint16_t h;
    std::memcpy(&h, blk, 2);
    return f16_table()[h];
}

// ggml_vec_dot_q8_0_q8_0 semantics: exact integer block dot, float accumulation in block order.
// Scalar statement; vec_dot_q8_0 below is the same arithmetic with the integer dot in AVX2.
inline float vec_dot_q8_0_scalar(int64_t K, const uint8_t* w, const uint8_t* x) {
    const int64_t nb = K / QK;
    float sumf = 0.0f;
    for (int64_t ib = 0; ib < nb; ib++) {
        const int8_t* a = (const int8_t*)(w + ib * Q8_BYTES + 2);
        const int8_t* b = (const int8_t*)(x + ib * Q8_BYTES + 2);
        int32_t sumi = 0;
        for (int j = 0; j < QK; j++) sumi += (int32_t)a[j] * (int32_t)b[j];
        const float d = q8_d(w + ib * Q8_BYTES) * q8_d(x + ib * Q8_BYTES);
        sumf = std::fmaf((float)sumi, d, sumf);
    }
    return sumf;
}

// Exact int32 sum of the 32 products of one block pair. |a| (unsigned) times sign(a)*b is a*b for
// every int8 a and every b in [-127, 127] (Q8_0 quantizers never write -128 for the activations);
// pairs of such products fit int16 (<= 2 * 128 * 127), so the sums are exact.
inline __m256i block_dot_i32x8(const uint8_t* wq, const uint8_t* xq) {
    const __m256i a = _mm256_loadu_si256((const __m256i*)wq);
    const __m256i b = _mm256_loadu_si256((const __m256i*)xq);
    const __m256i p16 = _mm256_maddubs_epi16(_mm256_sign_epi8(a, a), _mm256_sign_epi8(b, a));
    return _mm256_madd_epi16(p16, _mm256_set1_epi16(1));
}
inline int32_t hsum_i32x8(__m256i v) {
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4e));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xb1));
    return _mm_cvtsi128_si32(s);
}

inline float vec_dot_q8_0(int64_t K, const uint8_t* w, const uint8_t* x) {
    const int64_t nb = K / QK;
    float sumf = 0.0f;
    for (int64_t ib = 0; ib < nb; ib++) {
        const int32_t sumi = hsum_i32x8(block_dot_i32x8(w + ib * Q8_BYTES + 2, x + ib * Q8_BYTES + 2));
        const float d = q8_d(w + ib * Q8_BYTES) * q8_d(x + ib * Q8_BYTES);
        sumf = std::fmaf((float)sumi, d, sumf);
    }
    return sumf;
}


// ggml_vec_dot_f32 (the F32 matrices: BERT projection, logits) with products exact in double,
// accumulated in double, rounded once. ggml's scalar path rounds each product to float first and its
// FMA-vectorised path accumulates in float lanes; both differ from this by roundings only.
inline float vec_dot_f32(int64_t n, const float* x, const float* y) {
    double s = 0.0;
    for (int64_t i = 0; i < n; i++) s = std::fma((double)x[i], (double)y[i], s);
    return (float)s;
}

int g_threads = 0;
inline int nthreads() {
#ifdef _OPENMP
    return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
    return 1;
#endif
}

enum { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13,
       T_Q6_K = 14, T_IQ4_NL = 20, T_BF16 = 30 };

// IEEE binary32 -> bfloat16 -> binary32, round-to-nearest-even (ggml's GGML_FP32_TO_BF16 for non-NaN)
inline float round_bf16(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return f;
    u = ((u + 0x7fffu + ((u >> 16) & 1u)) >> 16) << 16;
    std::memcpy(&f, &u, 4);
    return f;
}
inline float bf16_bits_to_float(uint16_t b) {
    const uint32_t u = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// A weight matrix [N][K] (torch [out,in] == ggml ne0=in): F32, F16 or BF16 (widened to f), Q8_0 raw
// GGUF blocks (q), or Q4_1 / Q5_1 as their unsigned values (qv, 0..31) and per-block d, m (dm).
// canon: evaluated by vec_dot_canon, with src1 rounded first to F16 (xround 1) or BF16 (xround 2).
struct Mat {
    int type = T_F32;
    int64_t N = 0, K = 0;
    bool canon = false;
    int xround = 0;
    std::vector<float> f;
    std::vector<uint8_t> q;
    std::vector<int8_t> qv;
    std::vector<float> dm;   // [N][K/32][2]: d, m; K-quants: [N][K/256][2]: d, dmin
    std::vector<int16_t> ksc;   // K-quants: sub-block scale of every value [N][K]
    std::vector<uint8_t> kmin;  // Q4_K / Q5_K: the 8 sub-block mins of each super-block [N][K/256][8]
};

// ggml's AVX2 F32/F16 dot in float (K a multiple of 32): chain c accumulates w[k]*x[k] for
// k = c, c+32, ... with FMA; the 32 chain sums are folded pairwise, c with c^16, then ^8, ^4, ^1, ^2
// (the accumulator / lane reduction of the 4 x 8-lane vector sums).
inline float vec_dot_canon(int64_t K, const float* w, const float* x) {
    float s[32] = {};
    for (int64_t k0 = 0; k0 < K; k0 += 32)
        for (int c = 0; c < 32; c++) s[c] = std::fmaf(w[k0 + c], x[k0 + c], s[c]);
    for (int off : {16, 8, 4, 1, 2})
        for (int c = 0; c < 32; c++)
            if (!(c & off)) s[c] = s[c] + s[c | off];
    return s[0];
}

// Y[M][N] = mul_mat(W, X) for X [M][K]   (src/gsv_ar.cpp:244,260,262,263; ggml mul_mat)
void mul_mat(const Mat& W, const float* X, int64_t M, float* Y) {
    const int64_t N = W.N, K = W.K;
    if (W.canon) {   // F32 / F16 layer matrices, F16 predict
        std::vector<float> xr(X, X + M * K);
        if (W.xround == 1)
            for (float& v : xr) v = round_f16(v);
        if (W.xround == 2)
            for (float& v : xr) v = round_bf16(v);
        #pragma omp parallel for num_threads(nthreads()) schedule(static)
        for (int64_t n = 0; n < N; n++) {
            const float* w = W.f.data() + n * K;
            for (int64_t m = 0; m < M; m++) Y[m * N + n] = vec_dot_canon(K, w, xr.data() + m * K);
        }
        return;
    }
    if (W.type == T_Q4_K || W.type == T_Q5_K || W.type == T_Q6_K) {
        // ggml_vec_dot_q{4,5,6}_K_q8_K (portable C): per super-block eight integer lane sums,
        // aux32[l] = sum over the values e = l (mod 8) of scale(e) * a_e * q_e; the lanes accumulate
        // sums[l] += (d_w*d_x) * aux32[l] (contracted to fma) over super-blocks; Q4_K / Q5_K also
        // sumf -= (dmin_w*d_x) * sum_g bsums[g]*min[g/2] (contracted); at the end sumf += sums[l], l = 0..7.
        const int64_t nsb = K / QKK;
        std::vector<int8_t> xq((size_t)(M * K));
        std::vector<float> xd((size_t)(M * nsb));
        std::vector<int32_t> xb((size_t)(M * nsb * 16));
        for (int64_t m = 0; m < M; m++)
            quantize_q8_k(X + m * K, K, xq.data() + m * K, xd.data() + m * nsb, xb.data() + m * nsb * 16);
        const bool has_min = W.type != T_Q6_K;
        #pragma omp parallel for num_threads(nthreads()) schedule(static)
        for (int64_t n = 0; n < N; n++)
            for (int64_t m = 0; m < M; m++) {
                float sums[8] = {}, sumf = 0.0f;
                for (int64_t sb = 0; sb < nsb; sb++) {
                    int32_t aux32[8] = {};
                    for (int e = 0; e < QKK; e++) {
                        const size_t wi = (size_t)(n * K + sb * QKK + e);
                        aux32[e % 8] += (int32_t)W.ksc[wi] * ((int32_t)W.qv[wi] * (int32_t)xq[(size_t)(m * K + sb * QKK + e)]);
                    }
                    const float d = W.dm[(size_t)((n * nsb + sb) * 2)] * xd[(size_t)(m * nsb + sb)];
                    for (int l = 0; l < 8; l++) sums[l] = std::fmaf(d, (float)aux32[l], sums[l]);
                    if (has_min) {
                        int32_t sumi = 0;
                        for (int g = 0; g < 16; g++)
                            sumi += xb[(size_t)((m * nsb + sb) * 16 + g)] * (int32_t)W.kmin[(size_t)((n * nsb + sb) * 8 + g / 2)];
                        const float dmin = W.dm[(size_t)((n * nsb + sb) * 2 + 1)] * xd[(size_t)(m * nsb + sb)];
                        sumf = std::fmaf(-dmin, (float)sumi, sumf);
                    }
                }
                for (int l = 0; l < 8; l++) sumf = sumf + sums[l];
                Y[m * N + n] = sumf;
            }
        return;
    }
    if (W.type == T_Q4_1 || W.type == T_Q5_1) {
        // ggml_vec_dot_q4_1_q8_1 / q5_1_q8_1 (portable C): per block the exact integer dot sumi of the
        // unsigned values with the Q8_1 values, then sumf += (d_w*d_x)*sumi + m_w*s_x, which GCC
        // contracts (-mfma) to sumf + fma(d_w*d_x, sumi, m_w*s_x); blocks in order.
        const int64_t nb = K / QK;
        std::vector<int8_t> xq((size_t)(M * K));
        std::vector<float> xd((size_t)(M * nb)), xs((size_t)(M * nb));
        for (int64_t m = 0; m < M; m++) quantize_q8_1(X + m * K, K, xq.data() + m * K, xd.data() + m * nb, xs.data() + m * nb);
        #pragma omp parallel for num_threads(nthreads()) schedule(static)
        for (int64_t n = 0; n < N; n++)
            for (int64_t m = 0; m < M; m++) {
                float acc = 0.0f;
                for (int64_t b = 0; b < nb; b++) {
                    int32_t sumi = 0;
                    for (int j = 0; j < QK; j++)
                        sumi += (int32_t)W.qv[(size_t)(n * K + b * QK + j)] * (int32_t)xq[(size_t)(m * K + b * QK + j)];
                    const float dd = W.dm[(size_t)((n * nb + b) * 2)] * xd[(size_t)(m * nb + b)];
                    const float ms = W.dm[(size_t)((n * nb + b) * 2 + 1)] * xs[(size_t)(m * nb + b)];
                    acc = acc + std::fmaf(dd, (float)sumi, ms);
                }
                Y[m * N + n] = acc;
            }
        return;
    }
    if (W.type == T_Q8_0) {
        std::vector<uint8_t> xq((size_t)M * (K / QK) * Q8_BYTES);
        #pragma omp parallel for num_threads(nthreads()) schedule(static)
        for (int64_t m = 0; m < M; m++) quantize_q8_0(X + m * K, K, xq.data() + m * (K / QK) * Q8_BYTES);
        const int64_t rowb = (K / QK) * Q8_BYTES, nb = K / QK, N8 = N / 8 * 8;
        // groups of 8 weight rows: the 8 rows' float chains run in the lanes of one vector (block
        // order per lane, as vec_dot_q8_0); the int32 block sums of the 8 rows are reduced together
        std::vector<float> dsc((size_t)(N8 * nb));   // [N/8][nb][8] weight scales
        for (int64_t n = 0; n < N8; n++)
            for (int64_t b = 0; b < nb; b++) dsc[(size_t)(((n >> 3) * nb + b) * 8 + (n & 7))] = q8_d(W.q.data() + n * rowb + b * Q8_BYTES);
        #pragma omp parallel for num_threads(nthreads()) schedule(static)
        for (int64_t g = 0; g < N8 / 8; g++) {
            const uint8_t* w0 = W.q.data() + g * 8 * rowb;
            const float* ds = dsc.data() + (size_t)(g * nb * 8);
            for (int64_t m = 0; m < M; m++) {
                const uint8_t* x = xq.data() + m * rowb;
                __m256 acc = _mm256_setzero_ps();
                for (int64_t b = 0; b < nb; b++) {
                    const size_t o = (size_t)b * Q8_BYTES;
                    __m256i p[8];
                    for (int r = 0; r < 8; r++) p[r] = block_dot_i32x8(w0 + r * rowb + o + 2, x + o + 2);
                    const __m256i h01 = _mm256_hadd_epi32(p[0], p[1]), h23 = _mm256_hadd_epi32(p[2], p[3]);
                    const __m256i h45 = _mm256_hadd_epi32(p[4], p[5]), h67 = _mm256_hadd_epi32(p[6], p[7]);
                    const __m256i a = _mm256_hadd_epi32(h01, h23), c = _mm256_hadd_epi32(h45, h67);
                    const __m256i sumi = _mm256_add_epi32(_mm256_permute2x128_si256(a, c, 0x20),
                                                          _mm256_permute2x128_si256(a, c, 0x31));
                    const __m256 d = _mm256_mul_ps(_mm256_loadu_ps(ds + b * 8), _mm256_set1_ps(q8_d(x + o)));
                    acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(sumi), d, acc);
                }
                float out[8];
                _mm256_storeu_ps(out, acc);
                for (int r = 0; r < 8; r++) Y[m * N + g * 8 + r] = out[r];
            }
        }
        for (int64_t n = N8; n < N; n++) {
            const uint8_t* w = W.q.data() + n * rowb;
            for (int64_t m = 0; m < M; m++) Y[m * N + n] = vec_dot_q8_0(K, w, xq.data() + m * rowb);
        }
    } else {
        #pragma omp parallel for num_threads(nthreads()) schedule(static)
        for (int64_t n = 0; n < N; n++) {
            const float* w = W.f.data() + n * K;
            for (int64_t m = 0; m < M; m++) Y[m * N + n] = vec_dot_f32(K, w, X + m * K);
        }
    }
}

// layernorm_affine (P:1535-1585) as called by ln_affine (src/gsv_ar.cpp:157-165).
void ln_affine(const float* x, const float* r, const float* bias, const float* w, const float* b,
               int64_t rows, int64_t n, float eps, float* y) {
    for (int64_t row = 0; row < rows; row++) {
        const float* xr = x + row * n;
        const float* rr = r ? r + row * n : nullptr;
        double sum = 0.0, sum2 = 0.0;
        for (int64_t i = 0; i < n; i++) {
            const float v = (xr[i] + (rr ? rr[i] : 0.0f)) + (bias ? bias[i] : 0.0f);
            sum += v;
            sum2 += (double)v * (double)v;
        }
        const float mean = (float)(sum / (double)n);
        const float var = std::fmaf(-mean, mean, (float)(sum2 / (double)n));
        const float inv = 1.0f / std::sqrt(var + eps);
        float* yr = y + row * n;
        for (int64_t i = 0; i < n; i++) {
            const float v = (xr[i] + (rr ? rr[i] : 0.0f)) + (bias ? bias[i] : 0.0f);
            yr[i] = std::fmaf((v - mean) * inv, w[i], b[i]);
        }
    }
}

// add_act (P:1587-1620): act(a[i] + b[i % n]); act 1 = ReLU, 0 = identity.
// act: 0 identity, 1 ReLU, 2 GELU (erf form: 0.5*v*(1 + erff(v/sqrt(2))), P:1615, with erf in double)
void add_act(const float* a, const float* b, int64_t rows, int64_t n, int act, float* y) {
    for (int64_t r = 0; r < rows; r++)
        for (int64_t i = 0; i < n; i++) {
            const float v = a[r * n + i] + b[i];
            // erf evaluated in double and rounded to float: the value glibc's erff approximates to within
            // an ulp (the CUDA path evaluates the same expression)
            if (act == 2) y[r * n + i] = 0.5f * v * (1.0f + (float)std::erf((double)(v * 0.70710678118654752440f)));
            else y[r * n + i] = act == 1 ? (v > 0.0f ? v : 0.0f) : v;
        }
}

// flash_attn_ext for one query row of one head (F32 K/V), masked keys skipped
// (the -inf/0 mask of src/gsv_ar.cpp:215-223, 450; keep(k) decides visibility).
// Scores: s = (float)(sum of the exact products q_e*k_e, accumulated in double) * scale. A float
// product of two floats is exact in double, so the sum carries ~1e-16 relative error and its rounding
// to float does not depend on the summation order. The softmax-weighted sum
// softmax(s) V is then evaluated in double (weights exp(s - max) with the double exp, sums in double)
// and rounded to float once. ggml's float online softmax is one float evaluation of the same
// expression; this order-independent evaluation is what any other reduction order (split-KV chunks,
// per-warp token groups) reproduces bit for bit after the final rounding.
template <class Keep>
void attn_row(const float* q, const float* K, const float* Vv, int64_t kstride, int64_t nk, int hd, float scale,
              Keep keep, float* out) {
    std::vector<float> sc((size_t)nk);
    float M = -INFINITY;
    for (int64_t ic = 0; ic < nk; ic++) {
        if (!keep(ic)) continue;
        const float* k = K + ic * kstride;
        double dot = 0.0;
        for (int d = 0; d < hd; d++) dot += (double)q[d] * (double)k[d];
        sc[ic] = (float)dot * scale;
        M = std::max(M, sc[ic]);
    }
    double l = 0.0, acc[256];
    for (int d = 0; d < hd; d++) acc[d] = 0.0;
    for (int64_t ic = 0; ic < nk; ic++) {
        if (!keep(ic)) continue;
        const double p = std::exp((double)sc[ic] - (double)M);
        l += p;
        const float* v = Vv + ic * kstride;
        for (int d = 0; d < hd; d++) acc[d] += p * (double)v[d];
    }
    for (int d = 0; d < hd; d++) out[d] = l > 0.0 ? (float)(acc[d] / l) : 0.0f;
}

// exp(x) for x <= 0 in float: Cody-Waite reduction x = n*ln2 + r (ln2 split into a 15-bit head and a
// float tail, so n*head is exact), degree-7 Taylor polynomial of exp(r) by Horner with fma, times 2^n.
// x < -87 (or -inf) gives 0. Max error ~1.2 ulp.
inline float exp_c(float x) {
    if (!(x >= -87.0f)) return 0.0f;
    const float n = rintf(x * 0x1.715476p+0f);
    float r = std::fma(-n, 0x1.62e4p-1f, x);
    r = std::fma(-n, 0x1.7f7d1cp-20f, r);
    float p = 0x1.a01a02p-13f;
    p = std::fma(p, r, 0x1.6c16c2p-10f);
    p = std::fma(p, r, 0x1.111112p-7f);
    p = std::fma(p, r, 0x1.555556p-5f);
    p = std::fma(p, r, 0x1.555556p-3f);
    p = std::fma(p, r, 0.5f);
    p = std::fma(p, r, 1.0f);
    p = std::fma(p, r, 1.0f);
    uint32_t bits = (uint32_t)((int)n + 127) << 23;
    float sc;
    std::memcpy(&sc, &bits, 4);
    return p * sc;
}

// Decode attention of one query row of one head (HD = 32) over nk cached keys, in the library's
// fixed evaluation order (flash_attn_ext of src/gsv_ar.cpp:450-456 for a decode row, with ggml's
// float online softmax replaced by a page-split evaluation whose every operation is pinned):
// keys are split into 64-key pages; in a page, key t belongs to group g = t % 8, dims are split into
// 4 slices of 8.
//   score: D_s = fma chain over slice s from 0; dot = (D0 + D1) + (D2 + D3); s_t = dot * scale
//   page:  m = max s_t; p_t = exp_c(s_t - m); per group: L_g = sum of p_t, O_g[d] = fma chain of
//          p_t * v_t[d], both in ascending t; l = ((L0+L1)+(L2+L3))+((L4+L5)+(L6+L7)), o[d] likewise
//   merge: M = max over pages of m; per page in order: w = exp_c(m - M), L = fma(w, l, L),
//          O[d] = fma(w, o[d], O[d]); out[d] = O[d] / L.
void decode_attention_canonical(const float* q, const float* K, const float* Vv, int64_t kstride, int64_t nk,
                                float scale, float* out) {
    constexpr int HD = 32, PG = 64;
    float L = 0.0f, O[HD] = {}, M = -INFINITY;
    const int64_t npg = (nk + PG - 1) / PG;
    std::vector<float> pm((size_t)npg), pl((size_t)npg), po((size_t)npg * HD);
    for (int64_t c = 0; c < npg; c++) {
        const int64_t n = std::min<int64_t>(PG, nk - c * PG);
        float sc[PG], m = -INFINITY;
        for (int64_t t = 0; t < n; t++) {
            const float* k = K + (c * PG + t) * kstride;
            float Ds[4];
            for (int sl = 0; sl < 4; sl++) {
                float d = 0.0f;
                for (int e = 0; e < 8; e++) d = std::fma(q[sl * 8 + e], k[sl * 8 + e], d);
                Ds[sl] = d;
            }
            sc[t] = ((Ds[0] + Ds[1]) + (Ds[2] + Ds[3])) * scale;
            m = std::max(m, sc[t]);
        }
        float Lg[8] = {}, Og[8][HD] = {};
        for (int64_t t = 0; t < n; t++) {
            const float pt = exp_c(sc[t] - m);
            const float* v = Vv + (c * PG + t) * kstride;
            const int g = (int)(t % 8);
            Lg[g] = Lg[g] + pt;
            for (int d = 0; d < HD; d++) Og[g][d] = std::fma(pt, v[d], Og[g][d]);
        }
        auto tree = [](const float* x) { return ((x[0] + x[1]) + (x[2] + x[3])) + ((x[4] + x[5]) + (x[6] + x[7])); };
        pm[c] = m;
        pl[c] = tree(Lg);
        for (int d = 0; d < HD; d++) {
            float col[8];
            for (int g = 0; g < 8; g++) col[g] = Og[g][d];
            po[(size_t)c * HD + d] = tree(col);
        }
        M = std::max(M, m);
    }
    for (int64_t c = 0; c < npg; c++) {
        const float w = exp_c(pm[c] - M);
        L = std::fma(w, pl[c], L);
        for (int d = 0; d < HD; d++) O[d] = std::fma(w, po[(size_t)c * HD + d], O[d]);
    }
    for (int d = 0; d < HD; d++) out[d] = O[d] / L;
}

// exp_c on 8 lanes: the same operations as the scalar exp_c, lane by lane.
inline __m256 exp_c8(__m256 x) {
    const __m256 valid = _mm256_cmp_ps(x, _mm256_set1_ps(-87.0f), _CMP_GE_OQ);
    const __m256 n = _mm256_round_ps(_mm256_mul_ps(x, _mm256_set1_ps(0x1.715476p+0f)),
                                     _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
    const __m256 nn = _mm256_sub_ps(_mm256_setzero_ps(), n);
    __m256 r = _mm256_fmadd_ps(nn, _mm256_set1_ps(0x1.62e4p-1f), x);
    r = _mm256_fmadd_ps(nn, _mm256_set1_ps(0x1.7f7d1cp-20f), r);
    __m256 p = _mm256_set1_ps(0x1.a01a02p-13f);
    p = _mm256_fmadd_ps(p, r, _mm256_set1_ps(0x1.6c16c2p-10f));
    p = _mm256_fmadd_ps(p, r, _mm256_set1_ps(0x1.111112p-7f));
    p = _mm256_fmadd_ps(p, r, _mm256_set1_ps(0x1.555556p-5f));
    p = _mm256_fmadd_ps(p, r, _mm256_set1_ps(0x1.555556p-3f));
    p = _mm256_fmadd_ps(p, r, _mm256_set1_ps(0.5f));
    p = _mm256_fmadd_ps(p, r, _mm256_set1_ps(1.0f));
    p = _mm256_fmadd_ps(p, r, _mm256_set1_ps(1.0f));
    const __m256i bits = _mm256_slli_epi32(_mm256_add_epi32(_mm256_cvtps_epi32(n), _mm256_set1_epi32(127)), 23);
    return _mm256_and_ps(_mm256_mul_ps(p, _mm256_castsi256_ps(bits)), valid);
}

// K cache layout of the oracle's sequences: per (layer, head), blocks of 8 keys, dims major inside a
// block ([key / 8][32 dims][key % 8]), so the 8 keys of a block sit in one vector per dimension.
inline size_t kt_index(int64_t li, int h, int64_t t, int d, int NH, int64_t capb) {
    return ((((size_t)li * NH + h) * capb + (size_t)(t >> 3)) * 32 + d) * 8 + (size_t)(t & 7);
}

// decode_attention_canonical over the blocked K layout (Kt: one head's blocks, V rows at vstride),
// evaluated 8 keys per vector: every key's score, weight and sums go through the same operations in
// the same order as the scalar statement, so the results are identical.
void decode_attention_kt(const float* q, const float* Kt, const float* Vv, int64_t vstride, int64_t nk, float scale,
                         float* out) {
    constexpr int HD = 32, PG = 64;
    const int64_t npg = (nk + PG - 1) / PG;
    thread_local std::vector<float> pm, pl, po;
    pm.resize((size_t)npg);
    pl.resize((size_t)npg);
    po.resize((size_t)npg * HD);
    __m256 qb[HD];
    for (int d = 0; d < HD; d++) qb[d] = _mm256_set1_ps(q[d]);
    const __m256 vscale = _mm256_set1_ps(scale), ninf = _mm256_set1_ps(-INFINITY);
    const __m256i lane = _mm256_setr_epi32(0, 1, 2, 3, 4, 5, 6, 7);
    float M = -INFINITY;
    alignas(32) float og[8][HD];
    for (int64_t c = 0; c < npg; c++) {
        const int n = (int)std::min<int64_t>(PG, nk - c * PG);
        const int nblk = (n + 7) >> 3;
        __m256 sc[8];
        __m256 vm = ninf;
        for (int u = 0; u < nblk; u++) {
            const float* kb = Kt + (size_t)(c * 8 + u) * HD * 8;
            __m256 D0 = _mm256_setzero_ps(), D1 = D0, D2 = D0, D3 = D0;
            for (int e = 0; e < 8; e++) {
                D0 = _mm256_fmadd_ps(qb[e], _mm256_loadu_ps(kb + (0 + e) * 8), D0);
                D1 = _mm256_fmadd_ps(qb[8 + e], _mm256_loadu_ps(kb + (8 + e) * 8), D1);
                D2 = _mm256_fmadd_ps(qb[16 + e], _mm256_loadu_ps(kb + (16 + e) * 8), D2);
                D3 = _mm256_fmadd_ps(qb[24 + e], _mm256_loadu_ps(kb + (24 + e) * 8), D3);
            }
            __m256 sv = _mm256_mul_ps(_mm256_add_ps(_mm256_add_ps(D0, D1), _mm256_add_ps(D2, D3)), vscale);
            const __m256 live = _mm256_castsi256_ps(_mm256_cmpgt_epi32(_mm256_set1_epi32(n - u * 8), lane));
            sv = _mm256_blendv_ps(ninf, sv, live);
            sc[u] = sv;
            vm = _mm256_max_ps(vm, sv);
        }
        float mv[8];
        _mm256_storeu_ps(mv, vm);
        float m = -INFINITY;
        for (int j = 0; j < 8; j++) m = std::max(m, mv[j]);
        const __m256 vmm = _mm256_set1_ps(m);
        alignas(32) float pbuf[PG];
        __m256 Lg = _mm256_setzero_ps();
        for (int u = 0; u < nblk; u++) {
            const __m256 p = exp_c8(_mm256_sub_ps(sc[u], vmm));
            _mm256_store_ps(pbuf + u * 8, p);
            Lg = _mm256_add_ps(Lg, p);   // masked lanes add +0
        }
        for (int g = 0; g < 8; g++) {   // group g: keys g, g + 8, ... in ascending order
            __m256 O0 = _mm256_setzero_ps(), O1 = O0, O2 = O0, O3 = O0;
            for (int t = g; t < n; t += 8) {
                const __m256 pt = _mm256_set1_ps(pbuf[t]);
                const float* v = Vv + (c * PG + t) * vstride;
                O0 = _mm256_fmadd_ps(pt, _mm256_loadu_ps(v + 0), O0);
                O1 = _mm256_fmadd_ps(pt, _mm256_loadu_ps(v + 8), O1);
                O2 = _mm256_fmadd_ps(pt, _mm256_loadu_ps(v + 16), O2);
                O3 = _mm256_fmadd_ps(pt, _mm256_loadu_ps(v + 24), O3);
            }
            _mm256_store_ps(og[g] + 0, O0);
            _mm256_store_ps(og[g] + 8, O1);
            _mm256_store_ps(og[g] + 16, O2);
            _mm256_store_ps(og[g] + 24, O3);
        }
        for (int j = 0; j < 4; j++) {   // ((0+1)+(2+3))+((4+5)+(6+7)) over the groups
            auto ld = [&](int gg) { return _mm256_load_ps(og[gg] + 8 * j); };
            const __m256 o = _mm256_add_ps(_mm256_add_ps(_mm256_add_ps(ld(0), ld(1)), _mm256_add_ps(ld(2), ld(3))),
                                           _mm256_add_ps(_mm256_add_ps(ld(4), ld(5)), _mm256_add_ps(ld(6), ld(7))));
            _mm256_storeu_ps(po.data() + (size_t)c * HD + 8 * j, o);
        }
        float lg[8];
        _mm256_storeu_ps(lg, Lg);
        pm[c] = m;
        pl[c] = ((lg[0] + lg[1]) + (lg[2] + lg[3])) + ((lg[4] + lg[5]) + (lg[6] + lg[7]));
        M = std::max(M, m);
    }
    float L = 0.0f;
    __m256 O[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps()};
    for (int64_t c = 0; c < npg; c++) {
        const float w = exp_c(pm[c] - M);
        L = std::fma(w, pl[c], L);
        const __m256 vw = _mm256_set1_ps(w);
        for (int j = 0; j < 4; j++) O[j] = _mm256_fmadd_ps(vw, _mm256_loadu_ps(po.data() + (size_t)c * HD + 8 * j), O[j]);
    }
    const __m256 vl = _mm256_set1_ps(L);
    for (int j = 0; j < 4; j++) _mm256_storeu_ps(out + 8 * j, _mm256_div_ps(O[j], vl));
}

// ------------------------------------------------------------------ sampler (src/gsv_sampler.cpp)
struct SamplerCfg {
    int top_k = 15;
    float top_p = 1.0f, temperature = 1.0f, rep = 1.35f;
};

// gsv_logits_to_probs (src/gsv_sampler.cpp:8-68). Consumes `logits` in place.
void logits_to_probs(const SamplerCfg& c, float* logits, int V, const int32_t* prev, int n_prev, float* probs) {
    // 1) repetition penalty, applied once per occurrence (compounds on repeats), :14-20
    if (prev && n_prev > 0 && c.rep != 1.0f) {
        for (int i = 0; i < n_prev; i++) {
            const int t = prev[i];
            if (t < 0 || t >= V) continue;
            const float s = logits[t];
            logits[t] = s < 0.0f ? s * c.rep : s / c.rep;
        }
    }
    // 2) nucleus: stable descending order, softmax in that order, cumulative sum, rank 0 kept, :23-42
    if (c.top_p < 1.0f) {
        std::vector<int> idx(V);
        std::iota(idx.begin(), idx.end(), 0);
        std::stable_sort(idx.begin(), idx.end(), [&](int a, int b) { return logits[a] > logits[b]; });
        const float mx = logits[idx[0]];
        float sum = 0.0f;
        for (int k = 0; k < V; k++) sum += std::exp(logits[idx[k]] - mx);
        const float inv_sum = 1.0f / sum;
        float cum = 0.0f;
        for (int k = 0; k < V; k++) {
            cum = std::fmaf(std::exp(logits[idx[k]] - mx), inv_sum, cum);
            if (k > 0 && cum > c.top_p) logits[idx[k]] = -INFINITY;
        }
    }
    // 3) temperature, :45-46
    const float t = std::max(c.temperature, 1e-5f);
    for (int i = 0; i < V; i++) logits[i] /= t;
    // 4) top-k: pivot = k-th largest value, strictly smaller -> -inf (ties kept), :49-56
    if (c.top_k > 0 && c.top_k < V) {
        std::vector<float> tmp(logits, logits + V);
        std::sort(tmp.begin(), tmp.end(), std::greater<float>());
        const float pivot = tmp[c.top_k - 1];
        for (int i = 0; i < V; i++)
            if (logits[i] < pivot) logits[i] = -INFINITY;
    }
    // 5) softmax, float accumulation in index order, :58-67
    float mx = -INFINITY;
    for (int i = 0; i < V; i++) mx = std::max(mx, logits[i]);
    float sum = 0.0f;
    for (int i = 0; i < V; i++) {
        probs[i] = logits[i] == -INFINITY ? 0.0f : std::exp(logits[i] - mx);
        sum += probs[i];
    }
    const float inv = 1.0f / sum;
    for (int i = 0; i < V; i++) probs[i] *= inv;
}

// gsv_rng (src/gsv_sampler.h:33-42): xorshift64*, U = (next >> 40) / 2^24, q = -logf(1 - U).
struct Rng {
    uint64_t s;
    explicit Rng(uint64_t seed) : s(seed ? seed : 1) {}
    uint64_t next() {
        s ^= s >> 12;
        s ^= s << 25;
        s ^= s >> 27;
        return s * 0x2545F4914F6CDD1Dull;
    }
    float uniform01() { return (float)((double)(next() >> 40) * (1.0 / 16777216.0)); }
    float exponential() { return -std::log(1.0f - uniform01()); }
};

// gsv_sample + gsv_argmax_probs_over_q (src/gsv_sampler.cpp:70-89).
int sample(const float* probs, int V, Rng& rng) {
    std::vector<float> q(V);
    for (int i = 0; i < V; i++) q[i] = rng.exponential();
    int best = 0;
    float bv = -INFINITY;
    for (int i = 0; i < V; i++) {
        const float v = probs[i] > 0.0f ? probs[i] / q[i] : 0.0f;
        if (v > bv) { bv = v; best = i; }
    }
    return best;
}

}  // namespace

// ================================================================== model
struct orc_layer {
    Mat qkv_w, out_w, f1w, f2w;
    std::vector<float> qkv_b, out_b, n1w, n1b, f1b, f2b, n2w, n2b;
};

struct orc_model {
    int D = 512, NH = 16, HD = 32, NL = 24, V = 1025, PV = 732, EOS = 1024, BERT = 1024;
    std::vector<orc_layer> L;
    std::vector<float> text_emb, audio_emb, bert_proj, bert_proj_b;
    Mat predict;
    Mat bert_aug;     // [D][BERT+1] = [W | b]   (src/gsv_ar.cpp:648-656)
    float text_alpha = 1.0f, audio_alpha = 1.0f;
    std::vector<float> pe;   // [pe_max][D]  (src/gsv_ar.cpp:173-181)
    int pe_max = 0;
    std::string err;
};

namespace {

// canon_f32: an F32 matrix is a layer matrix (vec_dot_canon) rather than the predict / BERT
// projection (vec_dot_f32). F16 / BF16 matrices are always evaluated by vec_dot_canon.
bool set_mat(Mat& m, int type, const void* data, int64_t nbytes, int64_t N, int64_t K, std::string& err, const char* name,
             bool canon_f32 = false) {
    m.type = type;
    m.N = N;
    m.K = K;
    m.canon = false;
    m.xround = 0;
    if (type == T_F32) {
        if (nbytes != N * K * 4) { err = std::string("bad size for ") + name; return false; }
        m.f.assign((const float*)data, (const float*)data + N * K);
        m.canon = canon_f32 && K % 32 == 0;
    } else if (type == T_F16 || type == T_BF16) {
        if (K % 32 || nbytes != N * K * 2) { err = std::string("bad size for ") + name; return false; }
        m.f.resize((size_t)(N * K));
        const uint16_t* h = (const uint16_t*)data;
        for (int64_t i = 0; i < N * K; i++) m.f[(size_t)i] = type == T_F16 ? f16_to_f32(h[i]) : bf16_bits_to_float(h[i]);
        m.canon = true;
        m.xround = type == T_F16 ? 1 : 2;
    } else if (type == T_Q8_0) {
        if (K % QK || nbytes != N * (K / QK) * Q8_BYTES) { err = std::string("bad size for ") + name; return false; }
        m.q.assign((const uint8_t*)data, (const uint8_t*)data + nbytes);
    } else if (type == T_Q4_K || type == T_Q5_K || type == T_Q6_K) {
        // ggml block_q4_K {fp16 d, dmin; u8 scales[12]; u8 qs[128]}, block_q5_K {fp16 d, dmin;
        // u8 scales[12]; u8 qh[32]; u8 qs[128]}, block_q6_K {u8 ql[128]; u8 qh[64]; i8 scales[16]; fp16 d}.
        // Q4_K / Q5_K: 8 sub-blocks of 32 with 6-bit scale and min (get_scale_min_k4); value e of the
        // 64-value group g: nibble (low for e < 32) of qs[32g + e % 32], + 16 * bit (2g + e/32) of
        // qh[e % 32] for Q5_K; weight = d*scale*q - dmin*min. Q6_K: 16 sub-blocks of 16 with int8 scale;
        // value e = 128h + 32k + l: low / high nibble (k = 0, 1 / 2, 3) of ql[64h + l + 32 (k odd)] | bits
        // 2k..2k+1 of qh[32h + l] << 4, minus 32; weight = d*scale*q.
        const int64_t bs = type == T_Q4_K ? 144 : type == T_Q5_K ? 176 : 210, nsb = N * (K / QKK);
        if (K % QKK || nbytes != nsb * bs) { err = std::string("bad size for ") + name; return false; }
        m.qv.assign((size_t)(N * K), 0);
        m.ksc.assign((size_t)(N * K), 0);
        m.dm.assign((size_t)(nsb * 2), 0.0f);
        m.kmin.assign((size_t)(nsb * 8), 0);
        for (int64_t b = 0; b < nsb; b++) {
            const uint8_t* src = (const uint8_t*)data + b * bs;
            int8_t* qv = m.qv.data() + b * QKK;
            int16_t* sc = m.ksc.data() + b * QKK;
            if (type == T_Q6_K) {
                uint16_t h;
                std::memcpy(&h, src + 208, 2);
                m.dm[(size_t)(b * 2)] = f16_to_f32(h);
                const uint8_t* ql = src;
                const uint8_t* qh = src + 128;
                const int8_t* s8 = (const int8_t*)(src + 192);
                for (int e = 0; e < QKK; e++) {
                    const int hh = e / 128, k = (e % 128) / 32, l = e % 32;
                    const uint8_t lo = ql[64 * hh + l + (k & 1) * 32];
                    const int nib = k < 2 ? (lo & 15) : (lo >> 4);
                    qv[e] = (int8_t)((nib | (((qh[32 * hh + l] >> (2 * k)) & 3) << 4)) - 32);
                    sc[e] = s8[e / 16];
                }
            } else {
                uint16_t h[2];
                std::memcpy(h, src, 4);
                m.dm[(size_t)(b * 2)] = f16_to_f32(h[0]);
                m.dm[(size_t)(b * 2 + 1)] = f16_to_f32(h[1]);
                const uint8_t* s = src + 4;
                int scl[8], mnv[8];
                for (int j = 0; j < 8; j++) {
                    if (j < 4) {
                        scl[j] = s[j] & 63;
                        mnv[j] = s[j + 4] & 63;
                    } else {
                        scl[j] = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
                        mnv[j] = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
                    }
                    m.kmin[(size_t)(b * 8 + j)] = (uint8_t)mnv[j];
                }
                const uint8_t* qh = src + 16;
                const uint8_t* qs = src + (type == T_Q4_K ? 16 : 48);
                for (int e = 0; e < QKK; e++) {
                    const int g = e / 64, hi = (e % 64) / 32, l = e % 32;
                    int q = hi ? (qs[32 * g + l] >> 4) : (qs[32 * g + l] & 15);
                    if (type == T_Q5_K) q += ((qh[l] >> (2 * g + hi)) & 1) * 16;
                    qv[e] = (int8_t)q;
                    sc[e] = (int16_t)scl[e / 32];
                }
            }
        }
    } else if (type == T_Q4_1 || type == T_Q5_1) {
        // ggml block_q4_1 {fp16 d, m; u8 qs[16]} / block_q5_1 {fp16 d, m; u8 qh[4]; u8 qs[16]}: value i is
        // d * q_i + m, q_i the low (i < 16) or high (i >= 16) nibble of qs[i % 16] (+ bit i of qh as bit 4)
        const int64_t bs = type == T_Q4_1 ? 20 : 24, nb = N * (K / QK);
        if (K % QK || nbytes != nb * bs) { err = std::string("bad size for ") + name; return false; }
        m.qv.assign((size_t)(N * K), 0);
        m.dm.assign((size_t)(nb * 2), 0.0f);
        for (int64_t b = 0; b < nb; b++) {
            const uint8_t* src = (const uint8_t*)data + b * bs;
            uint16_t h[2];
            std::memcpy(h, src, 4);
            m.dm[(size_t)(b * 2)] = f16_to_f32(h[0]);
            m.dm[(size_t)(b * 2 + 1)] = f16_to_f32(h[1]);
            const uint8_t* qs = src + (type == T_Q4_1 ? 4 : 8);
            uint32_t qh = 0;
            if (type == T_Q5_1) std::memcpy(&qh, src + 4, 4);
            for (int i = 0; i < QK; i++) {
                int q = i < 16 ? (qs[i] & 0x0f) : (qs[i - 16] >> 4);
                if (type == T_Q5_1) q += (int)((qh >> i) & 1u) * 16;
                m.qv[(size_t)(b * QK + i)] = (int8_t)q;
            }
        }
    } else if (type == T_Q4_0 || type == T_Q5_0 || type == T_IQ4_NL) {
        // ggml block_q4_0 / block_iq4_nl {fp16 d; u8 qs[16]} / block_q5_0 {fp16 d; u8 qh[4]; u8 qs[16]}:
        // value i (0..31) is d * (q_i - 8) / d * kvalues_iq4nl[q_i] / d * (q_i - 16), q_i = low (i < 16) or
        // high (i >= 16) nibble of qs[i % 16], plus bit i of qh as bit 4 for Q5_0. ggml's dot of these
        // types against Q8_0 activations is the integer dot of those signed values with the activation
        // block, scaled by d_w * d_x: the Q8_0 dot of a block holding them.
        static const int kv_iq4nl[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
        const int64_t bs = type == T_Q5_0 ? 22 : 18, nb = N * (K / QK);
        if (K % QK || nbytes != nb * bs) { err = std::string("bad size for ") + name; return false; }
        m.type = T_Q8_0;
        m.q.assign((size_t)(nb * Q8_BYTES), 0);
        for (int64_t b = 0; b < nb; b++) {
            const uint8_t* src = (const uint8_t*)data + b * bs;
            uint8_t* dst = m.q.data() + b * Q8_BYTES;
            std::memcpy(dst, src, 2);
            const uint8_t* qs = src + (type == T_Q5_0 ? 6 : 2);
            uint32_t qh = 0;
            if (type == T_Q5_0) std::memcpy(&qh, src + 2, 4);
            for (int i = 0; i < QK; i++) {
                int q = i < 16 ? (qs[i] & 0x0f) : (qs[i - 16] >> 4);
                if (type == T_Q5_0) q += (int)((qh >> i) & 1u) * 16;
                const int v = type == T_IQ4_NL ? kv_iq4nl[q] : q - (type == T_Q4_0 ? 8 : 16);
                dst[2 + i] = (uint8_t)(int8_t)v;
            }
        }
    } else {
        err = std::string("unsupported type for ") + name;
        return false;
    }
    return true;
}

bool set_vec(std::vector<float>& v, int type, const void* data, int64_t nbytes, int64_t n, std::string& err, const char* name) {
    if (type != T_F32 || nbytes != n * 4) { err = std::string("expected F32[") + std::to_string(n) + "] for " + name; return false; }
    v.assign((const float*)data, (const float*)data + n);
    return true;
}

// IEEE binary16 -> binary32, exact (normal, subnormal, zero, inf, NaN).
float half_bits_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    uint32_t bits;
    if (e == 0x1fu) bits = sign | 0x7f800000u | (m << 13);
    else if (e != 0) bits = sign | ((e + 112u) << 23) | (m << 13);
    else if (m == 0) bits = sign;
    else {   // subnormal: normalise
        int shift = 0;
        uint32_t mm = m;
        while (!(mm & 0x400u)) { mm <<= 1; shift++; }
        bits = sign | ((uint32_t)(113 - shift) << 23) | ((mm & 0x3ffu) << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// Embedding table: F32, or F16 widened to F32 on load (ggml get_rows of an F16 table yields the same
// values). The reference loader accepts F32 only (src/gsv_ar.cpp:633-637); F16 is what the exporter
// writes for --spec emb=f16.
bool set_emb(std::vector<float>& v, int type, const void* data, int64_t nbytes, int64_t n, std::string& err, const char* name) {
    if ((type == T_F16 || type == T_BF16) && nbytes == n * 2) {
        v.resize((size_t)n);
        const uint16_t* h = (const uint16_t*)data;
        for (int64_t i = 0; i < n; i++) v[(size_t)i] = type == T_F16 ? half_bits_to_float(h[i]) : bf16_bits_to_float(h[i]);
        return true;
    }
    return set_vec(v, type, data, nbytes, n, err, name);
}

// mk_pe (src/gsv_ar.cpp:173-181)
void make_pe(orc_model& m, int pe_max) {
    m.pe_max = pe_max;
    m.pe.assign((size_t)pe_max * m.D, 0.0f);
    for (int pos = 0; pos < pe_max; pos++)
        for (int i = 0; i < m.D; i += 2) {
            const float div = std::exp((float)i * -(std::log(10000.0f) / (float)m.D));
            m.pe[(size_t)pos * m.D + i] = std::sin((float)pos * div);
            m.pe[(size_t)pos * m.D + i + 1] = std::cos((float)pos * div);
        }
}

// One sequence's request (gsv_ar_request, src/gsv_ar.h:13-17).
struct Req {
    const int32_t* phones;
    int T;
    const float* bert;   // [BERT][T]
    const int32_t* prompt;
    int P;
};

// Per-sequence KV cache (F32, or values rounded through fp16 when emulating an F16 cache): V as
// [layer][pos][D] with head h at dims h*HD..; K in the blocked layout of kt_index (capb blocks of 8
// positions per layer and head).
struct SeqCache {
    int len = 0, cap = 0;
    int64_t capb = 0;
    std::vector<float> k, v;
};

// Prefill of one sequence (build_inputs src/gsv_ar.cpp:186-225 without left padding; run_first
// :228-293). Left padding keys are always masked in the reference, so a sequence computed alone
// produces the same values. Returns last-row logits; K/V land in the cache.
// dump (optional): per layer, last position: [attn out, n1, (n1 + W2 h) + b2, layer out].
void prefill_one(const orc_model& m, const Req& r, bool kv_f16, SeqCache& cache, float* logits, float* dump) {
    const int D = m.D, S = r.T + r.P, HD = m.HD, NH = m.NH;
    std::vector<float> x((size_t)S * D), cur((size_t)S * D);
    for (int t = 0; t < r.T; t++) {
        const float* tok = m.text_emb.data() + (size_t)r.phones[t] * D;
        for (int d = 0; d < D; d++) x[(size_t)t * D + d] = std::fmaf(m.text_alpha, m.pe[(size_t)t * D + d], tok[d]);
    }
    for (int t = 0; t < r.P; t++) {
        const float* e = m.audio_emb.data() + (size_t)r.prompt[t] * D;
        for (int d = 0; d < D; d++)
            x[(size_t)(r.T + t) * D + d] = std::fmaf(m.audio_alpha, m.pe[(size_t)t * D + d], e[d]);
    }
    // cur = x + bert_aug . feat  (src/gsv_ar.cpp:241); feat = [bert; 1] on text rows, zeros on prompt rows
    {
        std::vector<float> feat((size_t)r.T * (m.BERT + 1));
        for (int t = 0; t < r.T; t++) {
            for (int k = 0; k < m.BERT; k++) feat[(size_t)t * (m.BERT + 1) + k] = r.bert[(size_t)k * r.T + t];
            feat[(size_t)t * (m.BERT + 1) + m.BERT] = 1.0f;
        }
        std::vector<float> proj((size_t)r.T * D);
        mul_mat(m.bert_aug, feat.data(), r.T, proj.data());
        for (int t = 0; t < S; t++)
            for (int d = 0; d < D; d++)
                cur[(size_t)t * D + d] = x[(size_t)t * D + d] + (t < r.T ? proj[(size_t)t * D + d] : 0.0f);
    }
    cache.len = 0;
    const float scale = 1.0f / std::sqrt((float)HD);
    const int FF = (int)m.L[0].f1w.N;
    std::vector<float> qkv((size_t)S * 3 * D), att((size_t)S * D), o((size_t)S * D), n1((size_t)S * D),
        h((size_t)S * FF), h2((size_t)S * D);
    for (int li = 0; li < m.NL; li++) {
        const orc_layer& w = m.L[li];
        mul_mat(w.qkv_w, cur.data(), S, qkv.data());
        for (int t = 0; t < S; t++)
            for (int j = 0; j < 3 * D; j++) qkv[(size_t)t * 3 * D + j] += w.qkv_b[j];
        // K/V into the cache (src/gsv_ar.cpp:271-275)
        for (int t = 0; t < S; t++)
            for (int d = 0; d < D; d++) {
                const float kk = qkv[(size_t)t * 3 * D + D + d], vv = qkv[(size_t)t * 3 * D + 2 * D + d];
                cache.k[kt_index(li, d / HD, t, d % HD, NH, cache.capb)] = kv_f16 ? round_f16(kk) : kk;
                cache.v[((size_t)li * cache.cap + t) * D + d] = kv_f16 ? round_f16(vv) : vv;
            }
        // prefix-masked attention on the F32 K/V of this pass (src/gsv_ar.cpp:257, mask :215-223)
        const int T = r.T;
        #pragma omp parallel for collapse(2) num_threads(nthreads()) schedule(static)
        for (int hh = 0; hh < NH; hh++)
            for (int qi = 0; qi < S; qi++) {
                const float* q = qkv.data() + (size_t)qi * 3 * D + hh * HD;
                const float* K = qkv.data() + D + hh * HD;
                const float* Vv = qkv.data() + 2 * D + hh * HD;
                auto keep = [&](int64_t k) { return qi < T ? (k < T) : (k <= qi); };
                attn_row(q, K, Vv, 3 * D, S, HD, scale, keep, att.data() + (size_t)qi * D + hh * HD);
            }
        mul_mat(w.out_w, att.data(), S, o.data());
        ln_affine(cur.data(), o.data(), w.out_b.data(), w.n1w.data(), w.n1b.data(), S, D, 1e-5f, n1.data());
        mul_mat(w.f1w, n1.data(), S, h.data());
        add_act(h.data(), w.f1b.data(), S, FF, 1, h.data());
        mul_mat(w.f2w, h.data(), S, h2.data());
        ln_affine(n1.data(), h2.data(), w.f2b.data(), w.n2w.data(), w.n2b.data(), S, D, 1e-5f, cur.data());
        if (dump) {
            float* dd = dump + (size_t)li * 4 * D;
            const size_t lr = (size_t)(S - 1) * D;
            std::memcpy(dd + 0 * D, att.data() + lr, D * 4);
            std::memcpy(dd + 1 * D, n1.data() + lr, D * 4);
            for (int d = 0; d < D; d++) dd[2 * D + d] = (n1[lr + d] + h2[lr + d]) + w.f2b[d];
            std::memcpy(dd + 3 * D, cur.data() + lr, D * 4);
        }
    }
    cache.len = S;
    mul_mat(m.predict, cur.data() + (size_t)(S - 1) * D, 1, logits);
}

// One decode step for a set of sequences (run_decode / run_decode_cached, src/gsv_ar.cpp:296-358,
// 380-467): x [B][D] -> logits [B][V]. The new K/V are written at index len before attention
// reads [0, len] (write-before-read, :398-405).
void decode_step(const orc_model& m, std::vector<SeqCache*>& caches, const float* x_in, bool kv_f16, float* logits,
                 float* dump) {
    const int B = (int)caches.size(), D = m.D, HD = m.HD, NH = m.NH;
    const int FF = (int)m.L[0].f1w.N;
    std::vector<float> cur(x_in, x_in + (size_t)B * D), qkv((size_t)B * 3 * D), att((size_t)B * D),
        o((size_t)B * D), n1((size_t)B * D), h((size_t)B * FF), h2((size_t)B * D);
    const float scale = 1.0f / std::sqrt((float)HD);
    for (int li = 0; li < m.NL; li++) {
        const orc_layer& w = m.L[li];
        mul_mat(w.qkv_w, cur.data(), B, qkv.data());
        for (int b = 0; b < B; b++)
            for (int j = 0; j < 3 * D; j++) qkv[(size_t)b * 3 * D + j] += w.qkv_b[j];
        for (int b = 0; b < B; b++) {
            SeqCache& c = *caches[b];
            for (int d = 0; d < D; d++) {
                const float kk = qkv[(size_t)b * 3 * D + D + d], vv = qkv[(size_t)b * 3 * D + 2 * D + d];
                c.k[kt_index(li, d / HD, c.len, d % HD, NH, c.capb)] = kv_f16 ? round_f16(kk) : kk;
                c.v[((size_t)li * c.cap + c.len) * D + d] = kv_f16 ? round_f16(vv) : vv;
            }
        }
        #pragma omp parallel for collapse(2) num_threads(nthreads()) schedule(static)
        for (int b = 0; b < B; b++)
            for (int hh = 0; hh < NH; hh++) {
                SeqCache& c = *caches[b];
                const float* q = qkv.data() + (size_t)b * 3 * D + hh * HD;
                const float* Kt = c.k.data() + kt_index(li, hh, 0, 0, NH, c.capb);
                const float* Vv = c.v.data() + (size_t)li * c.cap * D + hh * HD;
                decode_attention_kt(q, Kt, Vv, D, c.len + 1, scale, att.data() + (size_t)b * D + hh * HD);
            }
        mul_mat(w.out_w, att.data(), B, o.data());
        ln_affine(cur.data(), o.data(), w.out_b.data(), w.n1w.data(), w.n1b.data(), B, D, 1e-5f, n1.data());
        mul_mat(w.f1w, n1.data(), B, h.data());
        add_act(h.data(), w.f1b.data(), B, FF, 1, h.data());
        mul_mat(w.f2w, h.data(), B, h2.data());
        ln_affine(n1.data(), h2.data(), w.f2b.data(), w.n2w.data(), w.n2b.data(), B, D, 1e-5f, cur.data());
        if (dump) {
            for (int b = 0; b < B; b++) {
                float* dd = dump + ((size_t)b * m.NL + li) * 4 * D;
                std::memcpy(dd + 0 * D, att.data() + (size_t)b * D, D * 4);
                std::memcpy(dd + 1 * D, n1.data() + (size_t)b * D, D * 4);
                for (int d = 0; d < D; d++) dd[2 * D + d] = (n1[(size_t)b * D + d] + h2[(size_t)b * D + d]) + w.f2b[d];
                std::memcpy(dd + 3 * D, cur.data() + (size_t)b * D, D * 4);
            }
        }
    }
    for (auto* c : caches) c->len += 1;
    mul_mat(m.predict, cur.data(), B, logits);
}

std::vector<Req> make_reqs(const orc_model& m, int B, const int32_t* phones, const int32_t* n_phones, const float* bert,
                           const int32_t* prompts, const int32_t* n_prompt) {
    std::vector<Req> reqs(B);
    size_t po = 0, bo = 0, qo = 0;
    for (int b = 0; b < B; b++) {
        reqs[b].phones = phones + po;
        reqs[b].T = n_phones[b];
        reqs[b].bert = bert + bo;
        reqs[b].prompt = prompts + qo;
        reqs[b].P = n_prompt[b];
        po += n_phones[b];
        bo += (size_t)m.BERT * n_phones[b];
        qo += n_prompt[b];
    }
    return reqs;
}

bool check_reqs(orc_model* m, const std::vector<Req>& reqs) {
    for (const Req& r : reqs) {
        if (r.T <= 0) { m->err = "empty phones"; return false; }
        for (int t = 0; t < r.T; t++)
            if (r.phones[t] < 0 || r.phones[t] >= m->PV) { m->err = "phone id out of range"; return false; }
        for (int t = 0; t < r.P; t++)
            if (r.prompt[t] < 0 || r.prompt[t] >= m->V) { m->err = "prompt code out of range"; return false; }
    }
    return true;
}

void init_cache(const orc_model& m, SeqCache& c, int cap) {
    c.cap = cap;
    c.capb = (cap + 63) / 64 * 8;   // whole 64-key pages
    c.len = 0;
    c.k.assign((size_t)m.NL * m.NH * c.capb * 8 * m.HD, 0.0f);
    c.v.assign((size_t)m.NL * cap * m.D, 0.0f);
}

}  // namespace

extern "C" {

void orc_set_threads(int n) { g_threads = n; }
int orc_get_threads(void) { return nthreads(); }

// ---------------------------------------------------------------- primitive ops
void orc_fp32_to_fp16(const float* x, uint16_t* y, int64_t n) { for (int64_t i = 0; i < n; i++) y[i] = f32_to_f16(x[i]); }
void orc_fp16_to_fp32(const uint16_t* x, float* y, int64_t n) { for (int64_t i = 0; i < n; i++) y[i] = f16_to_f32(x[i]); }
void orc_quantize_q8_0(const float* x, int64_t n, uint8_t* blocks) { quantize_q8_0(x, n, blocks); }

// Y[M][N] = W[N][K] . X[M][K]^T with W raw Q8_0 / Q4_0 / Q5_0 / IQ4_NL / Q4_1 / Q5_1 blocks (type 8 / 2 /
// 6 / 20 / 3 / 7), F32 (type 0), F16 (type 1) or BF16 (type 30);
// layer != 0: W is a layer matrix (an F32 W is then evaluated like an F16 one, by vec_dot_canon).
int orc_mul_mat(int type, const void* W, int64_t N, int64_t K, const float* X, int64_t M, float* Y, int layer) {
    Mat w;
    std::string err;
    const int64_t nbytes = type == T_Q8_0   ? N * (K / QK) * Q8_BYTES
                           : type == T_Q4_K ? N * (K / QKK) * 144
                           : type == T_Q5_K ? N * (K / QKK) * 176
                           : type == T_Q6_K ? N * (K / QKK) * 210
                           : type == T_Q4_1 ? N * (K / QK) * 20
                           : type == T_Q5_1 ? N * (K / QK) * 24
                           : type == T_Q4_0 || type == T_IQ4_NL ? N * (K / QK) * 18
                           : type == T_Q5_0 ? N * (K / QK) * 22
                                            : N * K * (type == T_F16 || type == T_BF16 ? 2 : 4);
    if (!set_mat(w, type, W, nbytes, N, K, err, "W", layer != 0)) return -1;
    mul_mat(w, X, M, Y);
    return 0;
}

void orc_ln_affine(const float* x, const float* r, const float* bias, const float* w, const float* b, int64_t rows,
                   int64_t n, float eps, float* y) {
    ln_affine(x, r, bias, w, b, rows, n, eps, y);
}

void orc_add_act(const float* a, const float* b, int64_t rows, int64_t n, int act, float* y) { add_act(a, b, rows, n, act, y); }

// Decode attention over a contiguous per-sequence cache: q [B][NH][HD], k/v [B][Lmax][NH][HD],
// lens [B] keys visible per sequence; out [B][NH][HD].
void orc_decode_attention(const float* q, const float* k, const float* v, const int32_t* lens, int B, int Lmax, int NH,
                          int HD, float scale, float* out) {
    if (HD != 32) {
        std::fprintf(stderr, "orc_decode_attention: head dim must be 32\n");
        std::abort();
    }
    #pragma omp parallel for collapse(2) num_threads(nthreads()) schedule(dynamic)
    for (int b = 0; b < B; b++)
        for (int h = 0; h < NH; h++) {
            const size_t base = (size_t)b * Lmax * NH * HD + (size_t)h * HD;
            decode_attention_canonical(q + ((size_t)b * NH + h) * HD, k + base, v + base, (int64_t)NH * HD, lens[b],
                                       scale, out + ((size_t)b * NH + h) * HD);
        }
}

// Prefix-masked prefill attention over packed sequences: qkv [Mtot][3*NH*HD] rows (q|k|v),
// seq b occupies rows [off_b, off_b + S_b) with its first T_b rows text. out [Mtot][NH*HD].
void orc_prefill_attention(const float* qkv, const int32_t* seq_len, const int32_t* text_len, int B, int NH, int HD,
                           float scale, float* out) {
    const int D = NH * HD;
    std::vector<int64_t> off(B + 1, 0);
    for (int b = 0; b < B; b++) off[b + 1] = off[b] + seq_len[b];
    for (int b = 0; b < B; b++) {
        const int S = seq_len[b], T = text_len[b];
        const float* base = qkv + off[b] * 3 * D;
        #pragma omp parallel for collapse(2) num_threads(nthreads()) schedule(static)
        for (int h = 0; h < NH; h++)
            for (int qi = 0; qi < S; qi++) {
                auto keep = [&](int64_t kk) { return qi < T ? (kk < T) : (kk <= qi); };
                attn_row(base + (size_t)qi * 3 * D + h * HD, base + D + h * HD, base + 2 * D + h * HD, 3 * D, S, HD,
                         scale, keep, out + (off[b] + qi) * D + h * HD);
            }
    }
}

void orc_logits_to_probs(int top_k, float top_p, float temperature, float rep, float* logits, int V,
                         const int32_t* prev, int n_prev, float* probs) {
    SamplerCfg c;
    c.top_k = top_k;
    c.top_p = top_p;
    c.temperature = temperature;
    c.rep = rep;
    logits_to_probs(c, logits, V, prev, n_prev, probs);
}

uint64_t orc_rng_init(uint64_t seed) { return seed ? seed : 1; }

int orc_sample(const float* probs, int V, uint64_t* state) {
    Rng r(1);
    r.s = *state;
    const int t = sample(probs, V, r);
    *state = r.s;
    return t;
}

// ---------------------------------------------------------------- model
orc_model* orc_model_new(int D, int NH, int NL, int V, int PV, int EOS, int BERT) {
    orc_model* m = new orc_model();
    m->D = D; m->NH = NH; m->HD = D / NH; m->NL = NL; m->V = V; m->PV = PV; m->EOS = EOS; m->BERT = BERT;
    m->L.resize(NL);
    return m;
}

void orc_model_free(orc_model* m) { delete m; }
const char* orc_model_error(orc_model* m) { return m ? m->err.c_str() : "null model"; }

// Tensor names follow tools/export_gguf/convert_ar.py:106-130. type: 0 F32, 8 Q8_0.
int orc_model_set(orc_model* m, const char* name, int type, const void* data, int64_t nbytes) {
    const int D = m->D, FF = 4 * D;
    std::string n(name);
    if (n == "ar.text_emb") return set_emb(m->text_emb, type, data, nbytes, (int64_t)m->PV * D, m->err, name) ? 0 : -1;
    if (n == "ar.audio_emb") return set_emb(m->audio_emb, type, data, nbytes, (int64_t)m->V * D, m->err, name) ? 0 : -1;
    if (n == "ar.bert_proj") return set_vec(m->bert_proj, type, data, nbytes, (int64_t)D * m->BERT, m->err, name) ? 0 : -1;
    if (n == "ar.bert_proj_b") return set_vec(m->bert_proj_b, type, data, nbytes, D, m->err, name) ? 0 : -1;
    if (n == "ar.text_pe_alpha" || n == "ar.audio_pe_alpha") {
        if (type != T_F32 || nbytes != 4) { m->err = "alpha must be F32[1]"; return -1; }
        (n == "ar.text_pe_alpha" ? m->text_alpha : m->audio_alpha) = *(const float*)data;
        return 0;
    }
    if (n == "ar.predict") return set_mat(m->predict, type, data, nbytes, m->V, D, m->err, name) ? 0 : -1;
    int li = -1;
    char field[64] = {0};
    if (std::sscanf(name, "transformer.block%d.%63s", &li, field) == 2 && li >= 0 && li < m->NL) {
        orc_layer& L = m->L[li];
        std::string f(field);
        if (f == "qkv_w") return set_mat(L.qkv_w, type, data, nbytes, 3 * D, D, m->err, name, true) ? 0 : -1;
        if (f == "out_w") return set_mat(L.out_w, type, data, nbytes, D, D, m->err, name, true) ? 0 : -1;
        if (f == "ffn1_w") return set_mat(L.f1w, type, data, nbytes, FF, D, m->err, name, true) ? 0 : -1;
        if (f == "ffn2_w") return set_mat(L.f2w, type, data, nbytes, D, FF, m->err, name, true) ? 0 : -1;
        if (f == "qkv_b") return set_vec(L.qkv_b, type, data, nbytes, 3 * D, m->err, name) ? 0 : -1;
        if (f == "out_b") return set_vec(L.out_b, type, data, nbytes, D, m->err, name) ? 0 : -1;
        if (f == "ffn1_b") return set_vec(L.f1b, type, data, nbytes, FF, m->err, name) ? 0 : -1;
        if (f == "ffn2_b") return set_vec(L.f2b, type, data, nbytes, D, m->err, name) ? 0 : -1;
        if (f == "norm1_w") return set_vec(L.n1w, type, data, nbytes, D, m->err, name) ? 0 : -1;
        if (f == "norm1_b") return set_vec(L.n1b, type, data, nbytes, D, m->err, name) ? 0 : -1;
        if (f == "norm2_w") return set_vec(L.n2w, type, data, nbytes, D, m->err, name) ? 0 : -1;
        if (f == "norm2_b") return set_vec(L.n2b, type, data, nbytes, D, m->err, name) ? 0 : -1;
    }
    return 1;   // unknown tensor: ignored, like the reference loader (src/gsv_ar.cpp:556-559)
}

// After all tensors: bert_aug [W | b] (src/gsv_ar.cpp:648-656), PE table.
int orc_model_finalize(orc_model* m, int pe_max) {
    const int D = m->D, BD = m->BERT;
    if (m->bert_proj.size() != (size_t)D * BD || m->bert_proj_b.size() != (size_t)D || m->text_emb.empty() ||
        m->audio_emb.empty() || m->predict.N == 0) {
        m->err = "missing tensors";
        return -1;
    }
    for (int li = 0; li < m->NL; li++)
        if (m->L[li].qkv_w.N == 0 || m->L[li].out_w.N == 0 || m->L[li].f1w.N == 0 || m->L[li].f2w.N == 0 ||
            m->L[li].n2b.empty()) {
            m->err = "missing layer tensors";
            return -1;
        }
    m->bert_aug.type = T_F32;
    m->bert_aug.N = D;
    m->bert_aug.K = BD + 1;
    m->bert_aug.f.assign((size_t)D * (BD + 1), 0.0f);
    for (int d = 0; d < D; d++) {
        std::memcpy(m->bert_aug.f.data() + (size_t)d * (BD + 1), m->bert_proj.data() + (size_t)d * BD, BD * 4);
        m->bert_aug.f[(size_t)d * (BD + 1) + BD] = m->bert_proj_b[d];
    }
    make_pe(*m, pe_max > 0 ? pe_max : 4096);
    return 0;
}

// PE table access for tests.
const float* orc_model_pe(orc_model* m) { return m->pe.data(); }

// first_logits (src/gsv_ar.cpp:707-717) for B requests; dump (optional) gets, per sequence, the
// last position's [attn out, n1, (n1 + W2 h) + b2, layer out] for each layer: [B][NL][4][D].
int orc_first_logits(orc_model* m, int B, const int32_t* phones, const int32_t* n_phones, const float* bert,
                     const int32_t* prompts, const int32_t* n_prompt, int kv_f16, float* logits, float* dump) {
    std::vector<Req> reqs = make_reqs(*m, B, phones, n_phones, bert, prompts, n_prompt);
    if (!check_reqs(m, reqs)) return -1;
    for (int b = 0; b < B; b++) {
        SeqCache c;
        init_cache(*m, c, reqs[b].T + reqs[b].P + 1);
        prefill_one(*m, reqs[b], kv_f16 != 0, c, logits + (size_t)b * m->V,
                    dump ? dump + (size_t)b * m->NL * 4 * m->D : nullptr);
    }
    return 0;
}

// Teacher-forced decode trace: prefill, then feed `forced` tokens [B][n_steps] (audio_emb + PE at
// pos = P_b + step, src/gsv_ar.cpp:798-806) and record the raw logits of every step:
// logits_out [n_steps + 1][B][V] (row 0 = prefill). dump (optional) [n_steps][B][NL][4][D].
int orc_decode_trace(orc_model* m, int B, const int32_t* phones, const int32_t* n_phones, const float* bert,
                     const int32_t* prompts, const int32_t* n_prompt, int kv_f16, const int32_t* forced, int n_steps,
                     float* logits_out, float* dump) {
    std::vector<Req> reqs = make_reqs(*m, B, phones, n_phones, bert, prompts, n_prompt);
    if (!check_reqs(m, reqs)) return -1;
    const int D = m->D, V = m->V;
    std::vector<SeqCache> caches(B);
    for (int b = 0; b < B; b++) {
        init_cache(*m, caches[b], reqs[b].T + reqs[b].P + n_steps + 1);
        prefill_one(*m, reqs[b], kv_f16 != 0, caches[b], logits_out + (size_t)b * V, nullptr);
    }
    std::vector<SeqCache*> ptrs(B);
    for (int b = 0; b < B; b++) ptrs[b] = &caches[b];
    std::vector<float> x((size_t)B * D);
    for (int s = 0; s < n_steps; s++) {
        for (int b = 0; b < B; b++) {
            const int tok = forced[(size_t)b * n_steps + s];
            if (tok < 0 || tok >= V) { m->err = "forced token out of range"; return -1; }
            const int pos = reqs[b].P + s;
            for (int d = 0; d < D; d++)
                x[(size_t)b * D + d] = std::fmaf(m->audio_alpha, m->pe[(size_t)pos * D + d], m->audio_emb[(size_t)tok * D + d]);
        }
        decode_step(*m, ptrs, x.data(), kv_f16 != 0, logits_out + (size_t)(s + 1) * B * V,
                    dump ? dump + (size_t)s * B * m->NL * 4 * D : nullptr);
    }
    return 0;
}

// gsv_ar::generate (src/gsv_ar.cpp:719-824) for B requests.
//   tokens_out [B][cap]: prompt + generated tokens (without the stopping token), n_tokens_out [B]
//   lens_out [B]: generated counts in the order sequences finished (res.lens semantics)
// Sequences are computed independently (equal to the reference's left-padded batch, whose pad keys
// are always masked); PE of generated token idx is prompt_len_b + idx with prompt_len_b the
// sequence's own prompt length (the reference requires equal prompt lengths, :730-733).
// Wall time of the last orc_generate call on this thread, split into the prefills and the decode
// steps (a timing aid for the CPU baseline: the two parts differ by orders of magnitude per token).
static thread_local double g_gen_prefill_s = 0.0, g_gen_decode_s = 0.0;
static thread_local int g_gen_decode_steps = 0;
void orc_last_generate_seconds(double* prefill_s, double* decode_s, int* decode_steps) {
    *prefill_s = g_gen_prefill_s;
    *decode_s = g_gen_decode_s;
    *decode_steps = g_gen_decode_steps;
}

int orc_generate(orc_model* m, int B, const int32_t* phones, const int32_t* n_phones, const float* bert,
                 const int32_t* prompts, const int32_t* n_prompt, int top_k, float top_p, float temperature, float rep,
                 uint64_t seed_base, int early_stop_num, int max_steps, const int32_t* oracle_tokens, int n_oracle,
                 const uint64_t* seeds, int n_seeds, int kv_f16, int32_t* tokens_out, int32_t* n_tokens_out,
                 int32_t* lens_out, int cap, float* first_logits_out) {
    std::vector<Req> reqs = make_reqs(*m, B, phones, n_phones, bert, prompts, n_prompt);
    if (!check_reqs(m, reqs)) return -1;
    const int D = m->D, V = m->V;
    SamplerCfg sc;
    sc.top_k = top_k; sc.top_p = top_p; sc.temperature = temperature; sc.rep = rep;
    std::vector<SeqCache> caches(B);
    std::vector<float> lg((size_t)B * V);
    using clk = std::chrono::steady_clock;
    const auto t_start = clk::now();
    for (int b = 0; b < B; b++) {
        init_cache(*m, caches[b], reqs[b].T + reqs[b].P + max_steps + 8);
        prefill_one(*m, reqs[b], kv_f16 != 0, caches[b], lg.data() + (size_t)b * V, nullptr);
    }
    g_gen_prefill_s = std::chrono::duration<double>(clk::now() - t_start).count();
    g_gen_decode_s = 0.0;
    g_gen_decode_steps = 0;
    if (first_logits_out) std::memcpy(first_logits_out, lg.data(), lg.size() * 4);
    std::vector<std::vector<int32_t>> y(B);
    for (int b = 0; b < B; b++) y[b].assign(reqs[b].prompt, reqs[b].prompt + reqs[b].P);
    std::vector<int> idx_list(B, -1);
    std::vector<std::vector<int32_t>> res(B);
    std::vector<int32_t> lens;
    std::vector<Rng> rng;
    for (int b = 0; b < B; b++)
        rng.emplace_back(seeds && b < n_seeds ? seeds[b] : seed_base + 0x9E3779B9ull * (uint64_t)b);
    const int prompt_len0 = reqs[0].P;
    std::vector<float> row(V), probs(V), x;
    std::vector<int32_t> prev;
    for (int idx = 0; idx < max_steps; idx++) {
        for (int b = 0; b < B; b++) {
            if (idx_list[b] >= 0) continue;
            std::memcpy(row.data(), lg.data() + (size_t)b * V, V * 4);
            if (idx < 11) row[m->EOS] = -INFINITY;
            const int np = (int)std::min<size_t>(y[b].size(), 4096);
            prev.assign(y[b].end() - np, y[b].end());
            logits_to_probs(sc, row.data(), V, prev.data(), np, probs.data());
            int tok = sample(probs.data(), V, rng[b]);
            if (oracle_tokens && idx < n_oracle) tok = oracle_tokens[idx];
            y[b].push_back(tok);
            if (tok == m->EOS) {
                idx_list[b] = idx;
                res[b].assign(y[b].begin(), y[b].end() - 1);
                lens.push_back(idx);
            }
        }
        if (early_stop_num != -1 && ((int)y[0].size() - prompt_len0) > early_stop_num) {
            for (int b = 0; b < B; b++)
                if (idx_list[b] < 0) {
                    idx_list[b] = idx;
                    res[b].assign(y[b].begin(), y[b].end() - 1);
                    lens.push_back(idx);
                }
        }
        bool any = false;
        for (int b = 0; b < B; b++) any |= idx_list[b] < 0;
        if (!any) break;
        // Only unfinished sequences need the next step: finished ones are never read again.
        std::vector<SeqCache*> ptrs;
        std::vector<int> which;
        for (int b = 0; b < B; b++)
            if (idx_list[b] < 0) {
                ptrs.push_back(&caches[b]);
                which.push_back(b);
            }
        x.assign(which.size() * D, 0.0f);
        for (size_t j = 0; j < which.size(); j++) {
            const int b = which[j];
            const int pos = reqs[b].P + idx;
            const int tok = y[b].back();
            for (int d = 0; d < D; d++)
                x[j * D + d] = std::fmaf(m->audio_alpha, m->pe[(size_t)pos * D + d], m->audio_emb[(size_t)tok * D + d]);
        }
        std::vector<float> lg2(which.size() * V);
        const auto t_step = clk::now();
        decode_step(*m, ptrs, x.data(), kv_f16 != 0, lg2.data(), nullptr);
        g_gen_decode_s += std::chrono::duration<double>(clk::now() - t_step).count();
        g_gen_decode_steps++;
        for (size_t j = 0; j < which.size(); j++)
            std::memcpy(lg.data() + (size_t)which[j] * V, lg2.data() + j * V, V * 4);
    }
    for (int b = 0; b < B; b++)
        if (idx_list[b] < 0) {
            res[b] = y[b];
            lens.push_back(max_steps);
        }
    for (int b = 0; b < B; b++) {
        const int n = (int)std::min<size_t>(res[b].size(), (size_t)cap);
        std::memcpy(tokens_out + (size_t)b * cap, res[b].data(), (size_t)n * 4);
        n_tokens_out[b] = (int32_t)res[b].size();
        lens_out[b] = lens[b];
    }
    return 0;
}

// ------------------------------------------------------------------ continuous batching
// CPU restatement of the serving entry (gsv_engine::ar_generate_batch behind svc::ArBatcher,
// tools/svc_core.h:1244-1340, generalised to refill as the library's gsvcu_serve_* do): a fixed set
// of slots; admitted sequences prefill at once; one iteration samples one token for every slot in
// flight, applies the stop rules of src/gsv_ar.cpp:764-815 per sequence (EOS, early stop on the
// sequence's own count, max_steps), then runs one batched decode step over the slots still in
// flight. Each sequence therefore produces exactly the tokens of orc_generate on that sequence
// alone. Also the timed CPU arm of the serving benchmark.
struct orc_server {
    orc_model* m = nullptr;
    bool kv_f16 = false;
    int max_ctx = 0;
    struct Slot {
        bool used = false, active = false;
        SeqCache cache;
        std::vector<int32_t> y;
        std::vector<float> logits;
        int P = 0, idx = 0, max_steps = 0, early_stop = -1, tag = 0, kind = -1, n_gen = 0;
        uint64_t rng = 1;
        SamplerCfg sc;
    };
    std::vector<Slot> s;
    int64_t tokens_done = 0;
    double prefill_s = 0.0, decode_s = 0.0;
    int64_t decode_rows = 0;
};

orc_server* orc_serve_new(orc_model* m, int slots, int max_ctx, int kv_f16) {
    if (!m || slots <= 0 || max_ctx <= 0) return nullptr;
    orc_server* v = new orc_server();
    v->m = m;
    v->kv_f16 = kv_f16 != 0;
    v->max_ctx = max_ctx;
    v->s.resize(slots);
    for (auto& sl : v->s) {
        init_cache(*m, sl.cache, max_ctx);
        sl.logits.assign(m->V, 0.0f);
    }
    return v;
}

void orc_serve_free(orc_server* v) { delete v; }

// Admit n sequences (packed as for orc_generate) into free slots, lowest index first; returns 0, or
// -1 with the model's error (no free slot, context too long, bad ids).
int orc_serve_admit(orc_server* v, int n, const int32_t* phones, const int32_t* n_phones, const float* bert,
                    const int32_t* prompts, const int32_t* n_prompt, const uint64_t* seeds, const int32_t* tags,
                    int max_steps, int early_stop, int top_k, float top_p, float temperature, float rep) {
    orc_model* m = v->m;
    std::vector<Req> reqs = make_reqs(*m, n, phones, n_phones, bert, prompts, n_prompt);
    if (!check_reqs(m, reqs)) return -1;
    int free_slots = 0;
    for (auto& sl : v->s) free_slots += !sl.used;
    if (free_slots < n) { m->err = "no free sequence slot"; return -1; }
    for (const Req& r : reqs)
        if (max_steps < 1 || r.T + r.P + max_steps + 1 > v->max_ctx) { m->err = "sequence longer than the context"; return -1; }
    using clk = std::chrono::steady_clock;
    const auto t0 = clk::now();
    int next = 0;
    for (int i = 0; i < n; i++) {
        while (v->s[next].used) next++;
        orc_server::Slot& sl = v->s[next++];
        const Req& r = reqs[i];
        sl.used = sl.active = true;
        sl.P = r.P;
        sl.idx = 0;
        sl.max_steps = max_steps;
        sl.early_stop = early_stop;
        sl.tag = tags ? tags[i] : i;
        sl.kind = -1;
        sl.n_gen = 0;
        const uint64_t seed = seeds ? seeds[i] : (uint64_t)i;
        sl.rng = seed ? seed : 1;   // gsv_rng(seed) (src/gsv_sampler.h:35)
        sl.sc.top_k = top_k; sl.sc.top_p = top_p; sl.sc.temperature = temperature; sl.sc.rep = rep;
        sl.y.assign(r.prompt, r.prompt + r.P);
        prefill_one(*m, r, v->kv_f16, sl.cache, sl.logits.data(), nullptr);
    }
    v->prefill_s += std::chrono::duration<double>(clk::now() - t0).count();
    return 0;
}

// Run n_steps iterations, then report the finished sequences: done [max_done][5] = {slot, tag,
// finish_kind (0 EOS, 1 early stop, 2 max_steps), generated count (gsv_ar_result::lens value), tokens
// copied}, their generated tokens (prompt excluded, stopping token excluded) concatenated into tokens
// (capacity tok_cap, may be NULL). Finished slots are freed. Returns the number of records.
int orc_serve_step(orc_server* v, int n_steps, int32_t* done, int max_done, int32_t* tokens, int tok_cap) {
    orc_model* m = v->m;
    const int D = m->D, V = m->V;
    std::vector<float> row(V), probs(V), x, lg2;
    std::vector<int32_t> prev;
    std::vector<SeqCache*> ptrs;
    std::vector<int> which;
    using clk = std::chrono::steady_clock;
    for (int it = 0; it < n_steps; it++) {
        for (auto& sl : v->s) {
            if (!sl.active) continue;
            Rng rng(sl.rng);
            std::memcpy(row.data(), sl.logits.data(), (size_t)V * 4);
            if (sl.idx < 11) row[m->EOS] = -INFINITY;
            const int np = (int)std::min<size_t>(sl.y.size(), 4096);
            prev.assign(sl.y.end() - np, sl.y.end());
            logits_to_probs(sl.sc, row.data(), V, prev.data(), np, probs.data());
            const int tok = sample(probs.data(), V, rng);
            sl.rng = rng.s;
            sl.y.push_back(tok);
            const int n_samp = (int)sl.y.size() - sl.P;
            if (tok == m->EOS) sl.kind = 0;
            else if (sl.early_stop != -1 && n_samp > sl.early_stop) sl.kind = 1;
            else if (n_samp >= sl.max_steps) sl.kind = 2;
            if (sl.kind >= 0) {
                sl.active = false;
                sl.n_gen = sl.kind == 2 ? sl.max_steps : sl.idx;
            }
        }
        ptrs.clear();
        which.clear();
        for (int i = 0; i < (int)v->s.size(); i++)
            if (v->s[i].active) {
                ptrs.push_back(&v->s[i].cache);
                which.push_back(i);
            }
        if (which.empty()) break;
        x.assign(which.size() * D, 0.0f);
        for (size_t j = 0; j < which.size(); j++) {
            const orc_server::Slot& sl = v->s[which[j]];
            const int pos = sl.P + sl.idx;
            const int tok = sl.y.back();
            for (int d = 0; d < D; d++)
                x[j * D + d] = std::fmaf(m->audio_alpha, m->pe[(size_t)pos * D + d], m->audio_emb[(size_t)tok * D + d]);
        }
        lg2.resize(which.size() * V);
        const auto t0 = clk::now();
        decode_step(*m, ptrs, x.data(), v->kv_f16, lg2.data(), nullptr);
        v->decode_s += std::chrono::duration<double>(clk::now() - t0).count();
        v->decode_rows += (int64_t)which.size();
        for (size_t j = 0; j < which.size(); j++) {
            orc_server::Slot& sl = v->s[which[j]];
            std::memcpy(sl.logits.data(), lg2.data() + j * V, (size_t)V * 4);
            sl.idx++;
        }
    }
    int nd = 0, used = 0;
    for (int i = 0; i < (int)v->s.size() && nd < max_done; i++) {
        orc_server::Slot& sl = v->s[i];
        if (!sl.used || sl.active) continue;
        const int keep = (int)sl.y.size() - sl.P - (sl.kind == 2 ? 0 : 1);
        int32_t* rec = done + (size_t)nd * 5;
        rec[0] = i;
        rec[1] = sl.tag;
        rec[2] = sl.kind;
        rec[3] = sl.n_gen;
        rec[4] = 0;
        if (tokens && keep > 0 && used + keep <= tok_cap) {
            std::memcpy(tokens + used, sl.y.data() + sl.P, (size_t)keep * 4);
            rec[4] = keep;
            used += keep;
        }
        v->tokens_done += keep;
        sl.used = false;
        nd++;
    }
    return nd;
}

// Generated tokens so far: finished sequences plus those sampled by the sequences in flight.
int64_t orc_serve_tokens_total(const orc_server* v) {
    int64_t t = v->tokens_done;
    for (const auto& sl : v->s)
        if (sl.used) t += (int64_t)sl.y.size() - sl.P;
    return t;
}

// Drop every sequence in flight (nothing reported).
void orc_serve_reset(orc_server* v) {
    for (auto& sl : v->s) sl.used = sl.active = false;
}

int orc_serve_active(const orc_server* v) {
    int n = 0;
    for (const auto& sl : v->s) n += sl.used;
    return n;
}

// Seconds spent in prefills and in batched decode steps, and decoded rows, since orc_serve_new.
void orc_serve_seconds(const orc_server* v, double* prefill_s, double* decode_s, int64_t* decode_rows) {
    *prefill_s = v->prefill_s;
    *decode_s = v->decode_s;
    *decode_rows = v->decode_rows;
}


// ================================================================== BERT feature producer
// chinese-roberta-wwm-ext-large as src/gsv_bert.cpp runs it (gsv_bert::impl::run_g, :102-183) for one
// sequence: x = (word_emb[id] + pos_emb[t]) + type_emb[0], LayerNorm; per layer (post-LN, HF BertLayer):
// qkv = W_qkv x + b, per head flash_attn_ext over all keys (scale 1/sqrt(HD), no mask), cur = LN(cur +
// W_out attn + b_out), h = GELU_erf(W1 cur + b1), cur = LN(cur + W2 h + b2). Only the first
// bert.layers_used layers run (hidden_states[-3]); the output is [D][T]. The matrices take the layer
// mul_mat semantics above (F32 / F16 in the FMA-vectorised order, quantized types by their dots); the
// attention is attn_row; LayerNorm is ln_affine with eps = bert.ln_eps.
struct orc_bert_layer {
    Mat qkv_w, out_w, f1w, f2w;
    std::vector<float> qkv_b, out_b, ln1_w, ln1_b, f1b, f2b, ln2_w, ln2_b;
};

struct orc_bert {
    int D = 1024, NH = 16, HD = 64, FF = 4096, NL = 22, VOCAB = 21128, MAXPOS = 512;
    float EPS = 1e-12f;
    std::vector<float> word, pos, type, eln_w, eln_b;
    std::vector<orc_bert_layer> L;
    std::string err;
};

orc_bert* orc_bert_new(int D, int NH, int FF, int NL, int vocab, int maxpos, float eps) {
    orc_bert* m = new orc_bert();
    m->D = D; m->NH = NH; m->HD = NH > 0 ? D / NH : 0; m->FF = FF; m->NL = NL; m->VOCAB = vocab; m->MAXPOS = maxpos;
    m->EPS = eps;
    m->L.resize((size_t)std::max(NL, 0));
    return m;
}
void orc_bert_free(orc_bert* m) { delete m; }
const char* orc_bert_error(const orc_bert* m) { return m ? m->err.c_str() : "null model"; }

// Tensor names of tools/export_gguf/convert_bert.py:62-88 (bert.word_emb, bert.l<i>.qkv_w, ...); tensors
// of layers >= layers_used are ignored (0), unknown names are an error (-1).
int orc_bert_set(orc_bert* m, const char* name, int type, const void* data, int64_t nbytes) {
    const std::string n(name);
    const int D = m->D, FF = m->FF;
    if (n == "bert.word_emb") return set_emb(m->word, type, data, nbytes, (int64_t)m->VOCAB * D, m->err, name) ? 0 : -1;
    if (n == "bert.pos_emb") return set_emb(m->pos, type, data, nbytes, (int64_t)m->MAXPOS * D, m->err, name) ? 0 : -1;
    if (n == "bert.type_emb") {
        if (nbytes < (int64_t)D * (type == T_F32 ? 4 : 2)) { m->err = "bad size for bert.type_emb"; return -1; }
        return set_emb(m->type, type, data, nbytes, nbytes / (type == T_F32 ? 4 : 2), m->err, name) ? 0 : -1;
    }
    if (n == "bert.emb_ln_w") return set_vec(m->eln_w, type, data, nbytes, D, m->err, name) ? 0 : -1;
    if (n == "bert.emb_ln_b") return set_vec(m->eln_b, type, data, nbytes, D, m->err, name) ? 0 : -1;
    int li = -1, off = 0;
    if (std::sscanf(name, "bert.l%d.%n", &li, &off) == 1 && off > 0) {
        if (li < 0) { m->err = std::string("bad layer in ") + name; return -1; }
        if (li >= m->NL) return 0;
        orc_bert_layer& L = m->L[(size_t)li];
        const std::string f = n.substr((size_t)off);
        if (f == "qkv_w") return set_mat(L.qkv_w, type, data, nbytes, 3 * D, D, m->err, name, true) ? 0 : -1;
        if (f == "attn_out_w") return set_mat(L.out_w, type, data, nbytes, D, D, m->err, name, true) ? 0 : -1;
        if (f == "ff1_w") return set_mat(L.f1w, type, data, nbytes, FF, D, m->err, name, true) ? 0 : -1;
        if (f == "ff2_w") return set_mat(L.f2w, type, data, nbytes, D, FF, m->err, name, true) ? 0 : -1;
        if (f == "qkv_b") return set_vec(L.qkv_b, type, data, nbytes, 3 * D, m->err, name) ? 0 : -1;
        if (f == "attn_out_b") return set_vec(L.out_b, type, data, nbytes, D, m->err, name) ? 0 : -1;
        if (f == "attn_ln_w") return set_vec(L.ln1_w, type, data, nbytes, D, m->err, name) ? 0 : -1;
        if (f == "attn_ln_b") return set_vec(L.ln1_b, type, data, nbytes, D, m->err, name) ? 0 : -1;
        if (f == "ff1_b") return set_vec(L.f1b, type, data, nbytes, FF, m->err, name) ? 0 : -1;
        if (f == "ff2_b") return set_vec(L.f2b, type, data, nbytes, D, m->err, name) ? 0 : -1;
        if (f == "out_ln_w") return set_vec(L.ln2_w, type, data, nbytes, D, m->err, name) ? 0 : -1;
        if (f == "out_ln_b") return set_vec(L.ln2_b, type, data, nbytes, D, m->err, name) ? 0 : -1;
    }
    m->err = std::string("unknown tensor ") + name;
    return -1;
}

int orc_bert_finalize(orc_bert* m) {
    if (m->D <= 0 || m->NH <= 0 || m->D % m->NH || m->HD > 256 || m->word.empty() || m->pos.empty() ||
        m->type.size() < (size_t)m->D || m->eln_w.empty() || m->eln_b.empty()) {
        m->err = "incomplete BERT model (embeddings / dims)";
        return -1;
    }
    for (const orc_bert_layer& L : m->L)
        if (L.qkv_w.N == 0 || L.out_w.N == 0 || L.f1w.N == 0 || L.f2w.N == 0 || L.qkv_b.empty() || L.ln2_b.empty()) {
            m->err = "incomplete BERT layer";
            return -1;
        }
    return 0;
}

// ids [T] (with [CLS] / [SEP], T <= max_pos) -> out [D][T] after the first n_layers layers (n_layers < 0 or
// > layers_used: all of them; 0: the embedding LayerNorm output), as gsv_bert::encode / encode_layers.
int orc_bert_run(orc_bert* m, const int32_t* ids, int T, int n_layers, float* out) {
    const int D = m->D, HD = m->HD, NH = m->NH, FF = m->FF;
    if (T < 1 || T > m->MAXPOS) { m->err = "bad sequence length"; return -1; }
    for (int t = 0; t < T; t++)
        if (ids[t] < 0 || ids[t] >= m->VOCAB) { m->err = "token id out of range"; return -1; }
    if (n_layers < 0 || n_layers > m->NL) n_layers = m->NL;
    std::vector<float> x((size_t)T * D), cur((size_t)T * D);
    for (int t = 0; t < T; t++)
        for (int d = 0; d < D; d++)
            x[(size_t)t * D + d] = (m->word[(size_t)ids[t] * D + d] + m->pos[(size_t)t * D + d]) + m->type[(size_t)d];
    ln_affine(x.data(), nullptr, nullptr, m->eln_w.data(), m->eln_b.data(), T, D, m->EPS, cur.data());
    const float scale = 1.0f / std::sqrt((float)HD);
    std::vector<float> qkv((size_t)T * 3 * D), att((size_t)T * D), ao((size_t)T * D), h((size_t)T * FF), fo((size_t)T * D);
    for (int li = 0; li < n_layers; li++) {
        const orc_bert_layer& L = m->L[(size_t)li];
        mul_mat(L.qkv_w, cur.data(), T, qkv.data());
        for (int t = 0; t < T; t++)
            for (int j = 0; j < 3 * D; j++) qkv[(size_t)t * 3 * D + j] += L.qkv_b[(size_t)j];
        #pragma omp parallel for num_threads(nthreads()) schedule(static) collapse(2)
        for (int t = 0; t < T; t++)
            for (int hh = 0; hh < NH; hh++)
                attn_row(qkv.data() + (size_t)t * 3 * D + hh * HD, qkv.data() + D + hh * HD, qkv.data() + 2 * D + hh * HD,
                         3 * D, T, HD, scale, [](int64_t) { return true; }, att.data() + (size_t)t * D + hh * HD);
        mul_mat(L.out_w, att.data(), T, ao.data());
        ln_affine(cur.data(), ao.data(), L.out_b.data(), L.ln1_w.data(), L.ln1_b.data(), T, D, m->EPS, x.data());
        mul_mat(L.f1w, x.data(), T, h.data());
        add_act(h.data(), L.f1b.data(), T, FF, 2, h.data());
        mul_mat(L.f2w, h.data(), T, fo.data());
        ln_affine(x.data(), fo.data(), L.f2b.data(), L.ln2_w.data(), L.ln2_b.data(), T, D, m->EPS, cur.data());
    }
    for (int d = 0; d < D; d++)
        for (int t = 0; t < T; t++) out[(size_t)d * T + t] = cur[(size_t)t * D + d];
    return 0;
}

}  // extern "C"
