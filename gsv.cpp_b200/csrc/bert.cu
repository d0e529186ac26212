// bert.cu -- gsv.cpp's BERT feature producer (src/gsv_bert.{h,cpp}: chinese-roberta-wwm-ext-large, the
// layers up to hidden_states[-3]) on B200. It produces the `bert` input of the AR path.
//
// Per token row: x = (word[id] + pos[t]) + type[0], LayerNorm (eps bert.ln_eps); then per layer (post-LN,
// HF BertLayer, src/gsv_bert.cpp:118-150): qkv = W_qkv x + b; per head (head dim 64) softmax(q k^T / 8) v
// over every key of the row's own sequence; x = LN((x + W_o a) + b_o); h = GELU_erf(W_1 x + b_1);
// x = LN((x + W_2 h) + b_2). Features are [D][T] per sequence; encode_feat drops [CLS] / [SEP].
//
// Arithmetic, operation for operation that of the CPU restatement (oracle):
//   * F32 / F16 / BF16 matrices: k_gemm_fx, ggml's FMA-vectorised dot order (32 chains folded pairwise);
//     Q8_0 matrices: activations quantized to Q8_0, the exact integer block dots and the block-ordered
//     float chain (k_gemm_q8).
//   * LayerNorm: sums in double, mean and var in float, y = fma((v - mean) * inv, w, b).
//   * attention: scores from products exact in double, softmax and weighted sum in double, one rounding.
//   * GELU: y = (0.5 * v) * (1 + erf(v * 0.70710678)) with erf evaluated in double and rounded to float.
// Several sequences run as one pass over their concatenated rows; attention stays within each row's
// sequence (the block-diagonal mask of gsv_bert::encode_feat_batch, src/gsv_bert.cpp:271-301), so each
// sequence's features equal those of its own pass.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/gsvcu.h"
#include "gguf_reader.h"
#include "kernels.h"

namespace gsvcu {
namespace {

constexpr int BHD = 64;            // head dim the attention kernel is built for
constexpr int B_MAXD = 1024;       // widest hidden size of the row kernels (D % 128 == 0)
constexpr int B_QT = 64;           // queries per attention CTA (two threads each)

// ------------------------------------------------------------------ row kernels
// LayerNorm of one row of D values held as float4 per lane (D / 128 of them): sums in double.
__device__ __forceinline__ void ln_row(float4 (&v)[B_MAXD / 128], int nv, int D, const float* w, const float* b,
                                       float eps, float* y, int lane) {
    double s = 0.0, s2 = 0.0;
#pragma unroll
    for (int i = 0; i < B_MAXD / 128; i++)
        if (i < nv) {
            const float e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
            for (int k = 0; k < 4; k++) {
                s += (double)e[k];
                s2 += (double)e[k] * (double)e[k];
            }
        }
    s = warp_sum_d(s);
    s2 = warp_sum_d(s2);
    const float mean = (float)(s / (double)D);
    const float var = fmaf(-mean, mean, (float)(s2 / (double)D));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
    for (int i = 0; i < B_MAXD / 128; i++)
        if (i < nv) {
            const int c = (i * 32 + lane) * 4;
            const float4 ww = *(const float4*)(w + c), bb = *(const float4*)(b + c);
            float4 o;
            o.x = fmaf(__fmul_rn(__fsub_rn(v[i].x, mean), inv), ww.x, bb.x);
            o.y = fmaf(__fmul_rn(__fsub_rn(v[i].y, mean), inv), ww.y, bb.y);
            o.z = fmaf(__fmul_rn(__fsub_rn(v[i].z, mean), inv), ww.z, bb.z);
            o.w = fmaf(__fmul_rn(__fsub_rn(v[i].w, mean), inv), ww.w, bb.w);
            *(float4*)(y + c) = o;
        }
}

// Embeddings + LayerNorm, one warp per row: x = (word[id] + pos[t]) + type[0].
__global__ void __launch_bounds__(128) k_bert_embed(const int32_t* __restrict__ ids, const int32_t* __restrict__ tpos,
                                                    int rows, int D, const float* __restrict__ word,
                                                    const float* __restrict__ pos, const float* __restrict__ type,
                                                    const float* __restrict__ w, const float* __restrict__ b, float eps,
                                                    float* __restrict__ y) {
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    griddep_wait();
    griddep_launch();
    if (row >= rows) return;
    const int nv = D / 128;
    const float* wr = word + (size_t)ids[row] * D;
    const float* pr = pos + (size_t)tpos[row] * D;
    float4 v[B_MAXD / 128];
#pragma unroll
    for (int i = 0; i < B_MAXD / 128; i++)
        if (i < nv) {
            const int c = (i * 32 + lane) * 4;
            const float4 a = *(const float4*)(wr + c), p = *(const float4*)(pr + c), t = *(const float4*)(type + c);
            v[i] = make_float4(__fadd_rn(__fadd_rn(a.x, p.x), t.x), __fadd_rn(__fadd_rn(a.y, p.y), t.y),
                               __fadd_rn(__fadd_rn(a.z, p.z), t.z), __fadd_rn(__fadd_rn(a.w, p.w), t.w));
        }
    ln_row(v, nv, D, w, b, eps, y + (size_t)row * D, lane);
}

// LayerNorm of rows already summed as (x + r) + bias (the GEMM's residual epilogue).
__global__ void __launch_bounds__(128) k_bert_ln(const float* __restrict__ vin, int rows, int D,
                                                 const float* __restrict__ w, const float* __restrict__ b, float eps,
                                                 float* __restrict__ y) {
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    griddep_wait();
    griddep_launch();
    if (row >= rows) return;
    const int nv = D / 128;
    float4 v[B_MAXD / 128];
#pragma unroll
    for (int i = 0; i < B_MAXD / 128; i++)
        if (i < nv) v[i] = *(const float4*)(vin + (size_t)row * D + (i * 32 + lane) * 4);
    ln_row(v, nv, D, w, b, eps, y + (size_t)row * D, lane);
}

// GELU (erf form, the patch's add_act act 2, P:1615) in place: (0.5 v) (1 + erf(v / sqrt 2)), erf in double.
__global__ void __launch_bounds__(256) k_bert_gelu(float* __restrict__ h, size_t n) {
    griddep_wait();
    griddep_launch();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float v = h[i];
        const float e = (float)erf((double)__fmul_rn(v, 0.70710678118654752440f));
        h[i] = __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, e));
    }
}

// Attention over each row's own sequence, head dim 64: two threads per query (dims 0-31 / 32-63), key and
// value tiles of 64 rows widened to double in shared memory. Scores: the two halves' double dots added
// (products exact in double), rounded to float, times the scale; online softmax and weighted sum in
// double, rounded once.
struct BertTile { int32_t start, len, q0, pad; };
__global__ void __launch_bounds__(2 * B_QT) k_bert_attn(const float* __restrict__ qkv, int D,
                                                       const BertTile* __restrict__ tiles, float scale,
                                                       float* __restrict__ out) {
    extern __shared__ __align__(16) double bsm[];
    double* Ks = bsm;                       // [64 keys][64]
    double* Vs = bsm + B_QT * BHD;          // [64 keys][64]
    const int h = blockIdx.x, tid = threadIdx.x, half = tid & 1, qloc = tid >> 1;
    griddep_wait();
    griddep_launch();
    const BertTile tl = tiles[blockIdx.y];
    const int qi = tl.q0 + qloc;
    const bool valid = qi < tl.len;
    const size_t ld = (size_t)3 * D;
    double qd[32], od[32];
#pragma unroll
    for (int d = 0; d < 32; d++) {
        qd[d] = valid ? (double)qkv[(size_t)(tl.start + qi) * ld + h * BHD + half * 32 + d] : 0.0;
        od[d] = 0.0;
    }
    float m = -INFINITY;
    double l = 0.0;
    for (int kt = 0; kt < tl.len; kt += B_QT) {
        __syncthreads();
        for (int i = tid; i < B_QT * (BHD / 4); i += 2 * B_QT) {   // 64 rows x 16 float4, K and V
            const int key = kt + i / (BHD / 4), c = (i % (BHD / 4)) * 4;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (key < tl.len) {
                const float* kr = qkv + (size_t)(tl.start + key) * ld + D + h * BHD + c;
                kv = *(const float4*)kr;
                vv = *(const float4*)(kr + D);
            }
            double* kd = Ks + (size_t)(i / (BHD / 4)) * BHD + c;
            double* vd = Vs + (size_t)(i / (BHD / 4)) * BHD + c;
            kd[0] = kv.x; kd[1] = kv.y; kd[2] = kv.z; kd[3] = kv.w;
            vd[0] = vv.x; vd[1] = vv.y; vd[2] = vv.z; vd[3] = vv.w;
        }
        __syncthreads();
        const int nk = min(B_QT, tl.len - kt);
        for (int j = 0; j < nk; j++) {
            const double* kr = Ks + (size_t)j * BHD + half * 32;
            double dot = 0.0;
#pragma unroll
            for (int d = 0; d < 32; d++) dot = fma(qd[d], kr[d], dot);
            dot = dot + __shfl_xor_sync(0xffffffffu, dot, 1);
            if (!valid) continue;
            const float s = __fmul_rn((float)dot, scale);
            if (s > m) {
                const double r = m == -INFINITY ? 0.0 : exp((double)m - (double)s);
                l *= r;
#pragma unroll
                for (int d = 0; d < 32; d++) od[d] *= r;
                m = s;
            }
            const double pj = exp((double)s - (double)m);
            l += pj;
            const double* vr = Vs + (size_t)j * BHD + half * 32;
#pragma unroll
            for (int d = 0; d < 32; d++) od[d] = fma(pj, vr[d], od[d]);
        }
    }
    if (!valid) return;
    float* o = out + (size_t)(tl.start + qi) * D + h * BHD + half * 32;
#pragma unroll
    for (int d = 0; d < 32; d += 4)
        *(float4*)(o + d) = make_float4((float)(od[d] / l), (float)(od[d + 1] / l), (float)(od[d + 2] / l),
                                        (float)(od[d + 3] / l));
}

// Rows [start, start + len) of each sequence -> [D][len - 2 * skip] at out + off (feature-major), the
// first and last `skip` rows dropped.
struct BertOut { int32_t start, len, skip, pad; int64_t off; };
__global__ void __launch_bounds__(256) k_bert_out(const float* __restrict__ x, int D, const BertOut* __restrict__ seqs,
                                                  int nseq, float* __restrict__ out) {
    griddep_wait();
    griddep_launch();
    const BertOut so = seqs[blockIdx.y];
    const int T2 = so.len - 2 * so.skip;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < D * T2; i += gridDim.x * blockDim.x) {
        const int d = i / T2, t = i - d * T2;
        out[so.off + i] = x[(size_t)(so.start + so.skip + t) * D + d];
    }
}

struct BertLayer {
    int mt[4] = {0, 0, 0, 0};            // 0 F32, 1 F16, 30 BF16, 8 Q8_0: qkv, out, ffn1, ffn2
    const void* wf[4] = {};              // float types: rows [N][K] as stored
    uint4* wq[4] = {};                   // Q8_0: fragment planes
    uint16_t* wd[4] = {};
    float *qkv_b = nullptr, *out_b = nullptr, *ln1_w = nullptr, *ln1_b = nullptr;
    float *f1b = nullptr, *f2b = nullptr, *ln2_w = nullptr, *ln2_b = nullptr;
};

}  // namespace
}  // namespace gsvcu

using namespace gsvcu;

struct gsvcu_bert {
    int device = 0;
    cudaStream_t stream = nullptr;
    std::string err;
    gsvcu_bert_hparams hp{};
    int n_layer_file = 0;
    float *word = nullptr, *pos = nullptr, *type = nullptr, *eln_w = nullptr, *eln_b = nullptr;
    std::vector<BertLayer> L;
    std::vector<void*> wallocs;
    // per-call buffers, grown on demand: rows of the pass
    int cap_rows = 0;
    std::vector<void*> ballocs;
    int32_t *ids = nullptr, *tpos = nullptr;
    float *x = nullptr, *cur = nullptr, *qkv = nullptr, *att = nullptr, *tmp = nullptr, *h = nullptr;
    int8_t* aq = nullptr;
    uint16_t* ad = nullptr;
    BertTile* tiles = nullptr;
    int cap_tiles = 0;
    BertOut* outs = nullptr;
    int cap_outs = 0;
    float* dout = nullptr;
    size_t cap_dout = 0;

    int fail(int code, const std::string& m) {
        err = m;
        return code;
    }
    ~gsvcu_bert() {
        int prev = -1;
        cudaGetDevice(&prev);
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        for (void* p : wallocs) cudaFree(p);
        for (void* p : ballocs) cudaFree(p);
        cudaFree(tiles);
        cudaFree(outs);
        cudaFree(dout);
        if (stream) cudaStreamDestroy(stream);
        if (prev >= 0) cudaSetDevice(prev);
    }
    int upload(const void* src, size_t bytes, void** dst) {
        if (cudaMalloc(dst, bytes) != cudaSuccess) {
            cudaGetLastError();
            return fail(GSVCU_ERR_OOM, "cudaMalloc of BERT weights failed");
        }
        wallocs.push_back(*dst);
        if (cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice) != cudaSuccess)
            return fail(GSVCU_ERR_CUDA, "BERT weight upload failed");
        return GSVCU_OK;
    }
    int reserve_rows(int rows);
    int run(const int32_t* ids_host, const int32_t* tpos_host, int rows, const std::vector<BertTile>& tl, int n_layers);
};

namespace {

// F32 / F16 / BF16 widened on the host to f32 (embeddings, vectors)
bool to_f32(const GgufTensor* t, int64_t n, std::vector<float>& out) {
    out.resize((size_t)n);
    if (t->type == 0 && t->nbytes >= (uint64_t)n * 4) {
        std::memcpy(out.data(), t->data, (size_t)n * 4);
        return true;
    }
    if ((t->type == 1 || t->type == 30) && t->nbytes >= (uint64_t)n * 2) {
        const uint16_t* hsrc = (const uint16_t*)t->data;
        for (int64_t i = 0; i < n; i++) {
            uint32_t bits;
            if (t->type == 30) {
                bits = (uint32_t)hsrc[i] << 16;
            } else {   // fp16 -> f32, exact
                const uint32_t hv = hsrc[i], sgn = (hv & 0x8000u) << 16, ex = (hv >> 10) & 0x1f;
                uint32_t mant = hv & 0x3ffu;
                if (ex == 0) {
                    if (mant == 0) bits = sgn;
                    else {
                        int e = -1;
                        do { mant <<= 1; e++; } while (!(mant & 0x400u));
                        bits = sgn | ((uint32_t)(127 - 15 - e) << 23) | ((mant & 0x3ffu) << 13);
                    }
                } else if (ex == 31) bits = sgn | 0x7f800000u | (mant << 13);
                else bits = sgn | ((ex - 15 + 127) << 23) | (mant << 13);
            }
            std::memcpy(&out[(size_t)i], &bits, 4);
        }
        return true;
    }
    return false;
}

}  // namespace

int gsvcu_bert::reserve_rows(int rows) {
    if (rows <= cap_rows) return GSVCU_OK;
    cudaStreamSynchronize(stream);
    for (void* p : ballocs) cudaFree(p);
    ballocs.clear();
    cap_rows = 0;
    const int D = hp.hidden, FF = hp.inter;
    const size_t R = (size_t)rows;
    struct A { void** p; size_t bytes; };
    const A list[] = {{(void**)&ids, R * 4}, {(void**)&tpos, R * 4}, {(void**)&x, R * D * 4},
                      {(void**)&cur, R * D * 4}, {(void**)&qkv, R * 3 * D * 4}, {(void**)&att, R * D * 4},
                      {(void**)&tmp, R * D * 4}, {(void**)&h, R * FF * 4}, {(void**)&aq, R * FF},
                      {(void**)&ad, R * FF / 16}};
    for (const A& a : list) {
        if (cudaMalloc(a.p, a.bytes) != cudaSuccess) {
            cudaGetLastError();
            for (void* p : ballocs) cudaFree(p);
            ballocs.clear();
            return fail(GSVCU_ERR_OOM, "cudaMalloc of BERT activations failed");
        }
        ballocs.push_back(*a.p);
    }
    cap_rows = rows;
    return GSVCU_OK;
}

// One GEMM of layer li, matrix m: y = x W^T + b (epi FXE_BIAS) or (resid + x W^T) + b (FXE_RESID).
static void bert_gemm(gsvcu_bert* c, const BertLayer& w, int m, const float* xin, int M, int N, int K, const float* bias,
                      const float* resid, int epi, float* y) {
    if (w.mt[m] == 8) {
        launch_quantize_q8(xin, M, K, c->aq, c->ad, c->stream);
        GemmQ8Params g;
        g.xq = c->aq; g.xd = c->ad; g.M = M; g.wq = w.wq[m]; g.wd = w.wd[m]; g.N = N; g.K = K; g.bias = bias;
        g.resid = resid; g.y = y;
        launch_gemm_q8(g, epi == FXE_RESID ? EPI_RESID : EPI_BIAS, c->stream);
        return;
    }
    GemmFxParams g;
    g.x = xin; g.ldx = K; g.M = M; g.w = w.wf[m]; g.wtype = w.mt[m] == 1 ? FX_F16 : w.mt[m] == 30 ? FX_BF16 : FX_F32;
    g.N = N; g.K = K; g.bias = bias; g.resid = resid; g.y = y;
    launch_gemm_fx(g, epi, c->stream);
}

int gsvcu_bert::run(const int32_t* ids_host, const int32_t* tpos_host, int rows, const std::vector<BertTile>& tl,
                    int n_layers) {
    const int D = hp.hidden, FF = hp.inter;
    if (int rc = reserve_rows(rows)) return rc;
    if ((int)tl.size() > cap_tiles) {
        cudaStreamSynchronize(stream);
        cudaFree(tiles);
        tiles = nullptr;
        cap_tiles = 0;
        if (cudaMalloc((void**)&tiles, tl.size() * sizeof(BertTile)) != cudaSuccess) {
            cudaGetLastError();
            return fail(GSVCU_ERR_OOM, "cudaMalloc of attention tiles failed");
        }
        cap_tiles = (int)tl.size();
    }
    cudaStream_t s = stream;
    if (cudaMemcpyAsync(ids, ids_host, (size_t)rows * 4, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(tpos, tpos_host, (size_t)rows * 4, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(tiles, tl.data(), tl.size() * sizeof(BertTile), cudaMemcpyHostToDevice, s) != cudaSuccess)
        return fail(GSVCU_ERR_CUDA, "BERT input upload failed");
    launch_pdl(k_bert_embed, dim3((rows + 3) / 4), dim3(128), 0, s, (const int32_t*)ids, (const int32_t*)tpos, rows, D,
               (const float*)word, (const float*)pos, (const float*)type, (const float*)eln_w, (const float*)eln_b,
               hp.ln_eps, cur);
    const float scale = 1.0f / std::sqrt((float)BHD);
    const size_t asmem = (size_t)2 * B_QT * BHD * sizeof(double);
    for (int li = 0; li < n_layers; li++) {
        const BertLayer& w = L[(size_t)li];
        bert_gemm(this, w, 0, cur, rows, 3 * D, D, w.qkv_b, nullptr, FXE_BIAS, qkv);
        launch_pdl(k_bert_attn, dim3(hp.n_head, (unsigned)tl.size()), dim3(2 * B_QT), asmem, s, (const float*)qkv, D,
                   (const BertTile*)tiles, scale, att);
        bert_gemm(this, w, 1, att, rows, D, D, w.out_b, cur, FXE_RESID, tmp);     // (x + W_o a) + b_o
        launch_pdl(k_bert_ln, dim3((rows + 3) / 4), dim3(128), 0, s, (const float*)tmp, rows, D, (const float*)w.ln1_w,
                   (const float*)w.ln1_b, hp.ln_eps, x);
        bert_gemm(this, w, 2, x, rows, FF, D, w.f1b, nullptr, FXE_BIAS, h);        // W_1 x + b_1
        const size_t nh = (size_t)rows * FF;
        launch_pdl(k_bert_gelu, dim3((unsigned)std::min<size_t>((nh + 255) / 256, 148 * 16)), dim3(256), 0, s, h, nh);
        bert_gemm(this, w, 3, h, rows, D, FF, w.f2b, x, FXE_RESID, tmp);           // (x + W_2 h) + b_2
        launch_pdl(k_bert_ln, dim3((rows + 3) / 4), dim3(128), 0, s, (const float*)tmp, rows, D, (const float*)w.ln2_w,
                   (const float*)w.ln2_b, hp.ln_eps, cur);
    }
    if (cudaGetLastError() != cudaSuccess) return fail(GSVCU_ERR_CUDA, "BERT kernel launch failed");
    return GSVCU_OK;
}

extern "C" {

int gsvcu_bert_load(int device, const char* path, gsvcu_bert** out) {
    if (!out || !path) return GSVCU_ERR_ARG;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        cudaGetLastError();
        return GSVCU_ERR_DEVICE;
    }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10) return GSVCU_ERR_DEVICE;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    gsvcu_bert* c = new gsvcu_bert();
    c->device = device;
    auto done = [&](int rc) {
        if (prev >= 0) cudaSetDevice(prev);
        if (rc == GSVCU_OK) *out = c;
        else {
            std::fprintf(stderr, "gsvcu_bert_load: %s\n", c->err.c_str());
            delete c;
        }
        return rc;
    };
    if (gemm_q8_init_device() != cudaSuccess || gemm_fx_init_device() != cudaSuccess ||
        cudaFuncSetAttribute(k_bert_attn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             2 * B_QT * BHD * (int)sizeof(double)) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
        cudaGetLastError();
        return done(c->fail(GSVCU_ERR_CUDA, "device set-up failed"));
    }
    GgufFile f;
    std::string e;
    if (!f.open(path, e)) return done(c->fail(GSVCU_ERR_IO, e));
    uint32_t v = 0;
    auto u32 = [&](const char* k, int def) { return f.get_u32(k, v) ? (int)v : def; };
    gsvcu_bert_hparams& hp = c->hp;
    hp.hidden = u32("bert.hidden", 1024);
    hp.n_head = u32("bert.head", 16);
    hp.inter = u32("bert.inter", 4096);
    c->n_layer_file = u32("bert.n_layer", 24);
    hp.layers_used = u32("bert.layers_used", c->n_layer_file - 2);
    hp.vocab = u32("bert.vocab", 21128);
    hp.max_pos = u32("bert.max_pos", 512);
    float eps = 1e-12f;
    f.get_f32("bert.ln_eps", eps);
    hp.ln_eps = eps;
    const int D = hp.hidden, FF = hp.inter;
    if (D <= 0 || D % 128 || D > B_MAXD || hp.n_head <= 0 || D / hp.n_head != BHD || D % hp.n_head || FF <= 0 ||
        FF % 64 || hp.layers_used < 0 || hp.layers_used > c->n_layer_file || hp.vocab <= 0 || hp.max_pos <= 0)
        return done(c->fail(GSVCU_ERR_FORMAT, "unsupported BERT dims (hidden a multiple of 128 up to 1024, head dim "
                                              "64, inter a multiple of 64)"));
    auto vec = [&](const std::string& name, int64_t nvals, float** dst) -> int {
        const GgufTensor* t = f.tensor(name);
        std::vector<float> hst;
        if (!t || !to_f32(t, nvals, hst)) return c->fail(GSVCU_ERR_FORMAT, "missing or bad tensor " + name);
        return c->upload(hst.data(), hst.size() * 4, (void**)dst);
    };
    int rc;
    if ((rc = vec("bert.word_emb", (int64_t)hp.vocab * D, &c->word)) || (rc = vec("bert.pos_emb", (int64_t)hp.max_pos * D, &c->pos)) ||
        (rc = vec("bert.type_emb", D, &c->type)) || (rc = vec("bert.emb_ln_w", D, &c->eln_w)) ||
        (rc = vec("bert.emb_ln_b", D, &c->eln_b)))
        return done(rc);
    c->L.resize((size_t)hp.layers_used);
    const char* mats[4] = {"qkv_w", "attn_out_w", "ff1_w", "ff2_w"};
    const int N[4] = {3 * D, D, FF, D}, K[4] = {D, D, D, FF};
    std::vector<uint8_t> wq_tmp;
    std::vector<uint16_t> wd_tmp;
    for (int li = 0; li < hp.layers_used; li++) {
        BertLayer& w = c->L[(size_t)li];
        const std::string p = "bert.l" + std::to_string(li) + ".";
        for (int m = 0; m < 4; m++) {
            const GgufTensor* t = f.tensor(p + mats[m]);
            if (!t) return done(c->fail(GSVCU_ERR_FORMAT, "missing tensor " + p + mats[m]));
            const int64_t nv = (int64_t)N[m] * K[m];
            if (t->type == 0 || t->type == 1 || t->type == 30) {
                if (t->nbytes != (uint64_t)nv * (t->type == 0 ? 4 : 2))
                    return done(c->fail(GSVCU_ERR_FORMAT, "bad size of " + p + mats[m]));
                void* dst = nullptr;
                if ((rc = c->upload(t->data, t->nbytes, &dst))) return done(rc);
                w.mt[m] = (int)t->type;
                w.wf[m] = dst;
            } else if (t->type == 8) {
                if (t->nbytes != (uint64_t)nv / 32 * 34 || N[m] % 64 || K[m] % 256)
                    return done(c->fail(GSVCU_ERR_FORMAT, "bad Q8_0 matrix " + p + mats[m]));
                wq_tmp.resize((size_t)nv);
                wd_tmp.resize((size_t)nv / QK);
                pack_q8_0_host(t->data, N[m], K[m], wq_tmp.data(), wd_tmp.data());
                if ((rc = c->upload(wq_tmp.data(), wq_tmp.size(), (void**)&w.wq[m])) ||
                    (rc = c->upload(wd_tmp.data(), wd_tmp.size() * 2, (void**)&w.wd[m])))
                    return done(rc);
                w.mt[m] = 8;
            } else {
                return done(c->fail(GSVCU_ERR_FORMAT, "BERT matrix type not supported on B200 (F32, F16, BF16 or "
                                                      "Q8_0): " + p + mats[m]));
            }
        }
        const char* vn[8] = {"qkv_b", "attn_out_b", "attn_ln_w", "attn_ln_b", "ff1_b", "ff2_b", "out_ln_w", "out_ln_b"};
        const int vl[8] = {3 * D, D, D, D, FF, D, D, D};
        float** vd[8] = {&w.qkv_b, &w.out_b, &w.ln1_w, &w.ln1_b, &w.f1b, &w.f2b, &w.ln2_w, &w.ln2_b};
        for (int k = 0; k < 8; k++)
            if ((rc = vec(p + vn[k], vl[k], vd[k]))) return done(rc);
    }
    return done(GSVCU_OK);
}

void gsvcu_bert_destroy(gsvcu_bert* c) { delete c; }

const char* gsvcu_bert_last_error(const gsvcu_bert* c) { return c ? c->err.c_str() : "null BERT context"; }

int gsvcu_bert_get_hparams(const gsvcu_bert* c, gsvcu_bert_hparams* out) {
    if (!c || !out) return GSVCU_ERR_ARG;
    *out = c->hp;
    return GSVCU_OK;
}

// B sequences (ids in slots of Tmax, lens[b] valid) through the first n_layers layers as one pass; out gets,
// per sequence, [D][lens[b] - 2 skip] (skip 1: [CLS] / [SEP] dropped), concatenated.
static int bert_pass(gsvcu_bert* c, int B, const int32_t* ids_flat, const int32_t* lens, int Tmax, int n_layers,
                     int skip, float* out, int out_on_device) {
    const gsvcu_bert_hparams& hp = c->hp;
    const int D = hp.hidden;
    std::vector<int32_t> ids, tpos;
    std::vector<BertTile> tl;
    std::vector<BertOut> so;
    int64_t off = 0;
    for (int b = 0; b < B; b++) {
        const int len = lens[b];
        const int start = (int)ids.size();
        for (int i = 0; i < len; i++) {
            const int id = ids_flat[(size_t)b * Tmax + i];
            if (id < 0 || id >= hp.vocab) return c->fail(GSVCU_ERR_ARG, "token id out of range");
            ids.push_back(id);
            tpos.push_back(i);
        }
        for (int q0 = 0; q0 < len; q0 += B_QT) tl.push_back(BertTile{start, len, q0, 0});
        const int T2 = len - 2 * skip;
        if (T2 > 0) {
            so.push_back(BertOut{start, len, skip, 0, off});
            off += (int64_t)D * T2;
        }
    }
    const int rows = (int)ids.size();
    if (n_layers < 0 || n_layers > hp.layers_used) n_layers = hp.layers_used;
    int rc = c->run(ids.data(), tpos.data(), rows, tl, n_layers);
    if (rc) return rc;
    if (so.empty()) return cudaStreamSynchronize(c->stream) == cudaSuccess ? GSVCU_OK : c->fail(GSVCU_ERR_CUDA, "sync");
    if ((int)so.size() > c->cap_outs) {
        cudaStreamSynchronize(c->stream);
        cudaFree(c->outs);
        c->outs = nullptr;
        c->cap_outs = 0;
        if (cudaMalloc((void**)&c->outs, so.size() * sizeof(BertOut)) != cudaSuccess) {
            cudaGetLastError();
            return c->fail(GSVCU_ERR_OOM, "cudaMalloc failed");
        }
        c->cap_outs = (int)so.size();
    }
    float* dst = out;
    if (!out_on_device) {
        if ((size_t)off > c->cap_dout) {
            cudaStreamSynchronize(c->stream);
            cudaFree(c->dout);
            c->dout = nullptr;
            c->cap_dout = 0;
            if (cudaMalloc((void**)&c->dout, (size_t)off * 4) != cudaSuccess) {
                cudaGetLastError();
                return c->fail(GSVCU_ERR_OOM, "cudaMalloc failed");
            }
            c->cap_dout = (size_t)off;
        }
        dst = c->dout;
    }
    cudaStream_t s = c->stream;
    if (cudaMemcpyAsync(c->outs, so.data(), so.size() * sizeof(BertOut), cudaMemcpyHostToDevice, s) != cudaSuccess)
        return c->fail(GSVCU_ERR_CUDA, "upload failed");
    launch_pdl(k_bert_out, dim3(64, (unsigned)so.size()), dim3(256), 0, s, (const float*)c->cur, D,
               (const BertOut*)c->outs, (int)so.size(), dst);
    if (!out_on_device &&
        cudaMemcpyAsync(out, c->dout, (size_t)off * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess)
        return c->fail(GSVCU_ERR_CUDA, "download failed");
    if (cudaStreamSynchronize(s) != cudaSuccess) return c->fail(GSVCU_ERR_CUDA, "BERT pass failed");
    return GSVCU_OK;
}

int gsvcu_bert_encode(gsvcu_bert* c, const int32_t* ids, int32_t T, int32_t n_layers, float* out) {
    if (!c || !ids || !out) return GSVCU_ERR_ARG;
    if (T < 1 || T > c->hp.max_pos) return c->fail(GSVCU_ERR_ARG, "bad sequence length");
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(c->device);
    const int rc = bert_pass(c, 1, ids, &T, T, n_layers, 0, out, 0);
    if (prev >= 0) cudaSetDevice(prev);
    return rc;
}

int gsvcu_bert_encode_feat_batch(gsvcu_bert* c, int32_t B, const int32_t* ids_flat, const int32_t* lens, int32_t Tmax,
                                 float* out, int32_t out_on_device) {
    if (!c || !ids_flat || !lens || !out) return GSVCU_ERR_ARG;
    if (B <= 0 || Tmax < 3 || Tmax > c->hp.max_pos) return c->fail(GSVCU_ERR_ARG, "encode_feat_batch: bad args");
    for (int b = 0; b < B; b++)
        if (lens[b] < 1 || lens[b] > Tmax) return c->fail(GSVCU_ERR_ARG, "encode_feat_batch: bad length");
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(c->device);
    const int rc = bert_pass(c, B, ids_flat, lens, Tmax, -1, 1, out, out_on_device);
    if (prev >= 0) cudaSetDevice(prev);
    return rc;
}

}  // extern "C"
