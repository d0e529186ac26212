// misc.cu -- LayerNorm + Q8_0, activation quantization, F32 GEMM with double accumulation,
// embeddings, row gathers and the per-step stop rules.
#include "kernels.h"

namespace gsvcu {

// ------------------------------------------------------------------ LayerNorm (+ Q8_0)
// layernorm_affine (P:1535-1585) on a row already summed as v = (x + r) + bias: mean and E[v^2]
// in double, var = E[v^2] - mean^2 (FMA), inv = 1/sqrtf(var + 1e-5), y = ((v - mean)*inv)*w + b
// (FMA). One warp per 512-wide row, 16 consecutive values per lane; the Q8_0 block of 32 values
// spans a lane pair.
__global__ void __launch_bounds__(128) k_layernorm_q8(const float* __restrict__ v, int rows, const float* __restrict__ w,
                                                      const float* __restrict__ b, float* __restrict__ y,
                                                      int8_t* __restrict__ yq, uint16_t* __restrict__ yd) {
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    griddep_wait();
    griddep_launch();
    if (row >= rows) return;
    float x[16];
    const float4* src = (const float4*)(v + (size_t)row * D + lane * 16);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float4 t = src[i];
        x[4 * i] = t.x; x[4 * i + 1] = t.y; x[4 * i + 2] = t.z; x[4 * i + 3] = t.w;
    }
    double s = 0.0, s2 = 0.0;
#pragma unroll
    for (int i = 0; i < 16; i++) {
        s += (double)x[i];
        s2 += (double)x[i] * (double)x[i];
    }
    s = warp_sum_d(s);
    s2 = warp_sum_d(s2);
    const float mean = (float)(s / (double)D);
    const float var = fmaf(-mean, mean, (float)(s2 / (double)D));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; i++) {
        const int c = lane * 16 + i;
        x[i] = fmaf(__fmul_rn(__fsub_rn(x[i], mean), inv), w[c], b[c]);
        amax = fmaxf(amax, fabsf(x[i]));
    }
    float4* dst = (float4*)(y + (size_t)row * D + lane * 16);
#pragma unroll
    for (int i = 0; i < 4; i++) dst[i] = make_float4(x[4 * i], x[4 * i + 1], x[4 * i + 2], x[4 * i + 3]);
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    float dsc, id;
    q8_scale(amax, dsc, id);
    uint32_t pk[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        uint32_t u = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) u |= (uint32_t)(uint8_t)q8_val(x[4 * i + j], id) << (8 * j);
        pk[i] = u;
    }
    *(uint4*)(yq + (size_t)row * D + lane * 16) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    if ((lane & 1) == 0) yd[(size_t)row * (D / QK) + lane / 2] = f2h(dsc);
}

void launch_layernorm_q8(const float* v, int rows, const float* w, const float* b, float* y, int8_t* yq, uint16_t* yd,
                         cudaStream_t s) {
    if (rows <= 0) return;
    launch_pdl(k_layernorm_q8, dim3((rows + 3) / 4), dim3(128), 0, s, v, rows, w, b, y, yq, yd);
}

// ------------------------------------------------------------------ quantize
// quantize_row_q8_0 on rows of K floats: one thread per 32-value block.
__global__ void k_quantize_q8(const float* __restrict__ x, int nblocks, int8_t* __restrict__ q, uint16_t* __restrict__ d) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    griddep_wait();
    griddep_launch();
    if (i >= nblocks) return;
    float v[32], amax = 0.0f;
    const float4* src = (const float4*)(x + (size_t)i * 32);
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float4 t = src[j];
        v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
    }
#pragma unroll
    for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(v[j]));
    float dsc, id;
    q8_scale(amax, dsc, id);
    uint32_t pk[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        uint32_t u = 0;
#pragma unroll
        for (int k = 0; k < 4; k++) u |= (uint32_t)(uint8_t)q8_val(v[4 * j + k], id) << (8 * k);
        pk[j] = u;
    }
    uint4* dst = (uint4*)(q + (size_t)i * 32);
    dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
    d[i] = f2h(dsc);
}

void launch_quantize_q8(const float* x, int rows, int K, int8_t* q, uint16_t* d, cudaStream_t s) {
    const int nb = rows * (K / QK);
    if (nb <= 0) return;
    launch_pdl(k_quantize_q8, dim3((nb + 127) / 128), dim3(128), 0, s, x, nb, q, d);
}

// ------------------------------------------------------------------ F32 GEMM, double accumulation
// ggml F32 mul_mat (src/gsv_ar.cpp:241 BERT projection with the [W|b] augmented weight, :266 logits):
// products exact in double (fma of the widened operands), accumulated in double and rounded once.
// The double sum is exact or within a few double ulps of the serial sum, so its rounding to float
// matches the serial order except in vanishingly rare ties. Tile: 32 outputs x 32 rows, K in steps
// of 32.
__global__ void __launch_bounds__(256) k_gemm_f32d(const float* __restrict__ x, int ldx, F32Gather gth, int use_gather,
                                                   int M, const float* __restrict__ w, int N, int K,
                                                   const float* __restrict__ add, int ldadd, float* __restrict__ y,
                                                   int ldy) {
    __shared__ float Ws[32][33];
    __shared__ float Xs[32][33];
    const int tid = threadIdx.x, tn = tid & 31, tm = tid >> 5;
    const int n0 = blockIdx.x * 32, m0 = blockIdx.y * 32;
    griddep_wait();
    griddep_launch();
    double acc[4][2];
#pragma unroll
    for (int i = 0; i < 4; i++) acc[i][0] = acc[i][1] = 0.0;
    for (int k0 = 0; k0 < K; k0 += 32) {
        for (int i = tid; i < 1024; i += 256) {
            const int r = i >> 5, c = i & 31;
            const int n = n0 + r, k = k0 + c;
            Ws[r][c] = (n < N && k < K) ? w[(size_t)n * K + k] : 0.0f;
        }
        if (use_gather) {
            for (int i = tid; i < 1024; i += 256) {
                const int c = i >> 5, r = i & 31;
                const int m = m0 + r, k = k0 + c;
                float val = 0.0f;
                if (m < M && k < K && gth.row_T[m] >= 0) {
                    if (k < gth.bert_dim) val = gth.feat[gth.row_off[m] + (int64_t)k * gth.row_T[m]];
                    else if (k == gth.bert_dim) val = 1.0f;
                }
                Xs[r][c] = val;
            }
        } else {
            for (int i = tid; i < 1024; i += 256) {
                const int r = i >> 5, c = i & 31;
                const int m = m0 + r, k = k0 + c;
                Xs[r][c] = (m < M && k < K) ? x[(size_t)m * ldx + k] : 0.0f;
            }
        }
        __syncthreads();
#pragma unroll 4
        for (int kk = 0; kk < 32; kk++) {
            const float wv = Ws[tn][kk];
#pragma unroll
            for (int i = 0; i < 4; i++) acc[i][kk & 1] = fma((double)wv, (double)Xs[tm * 4 + i][kk], acc[i][kk & 1]);
        }
        __syncthreads();
    }
    const int n = n0 + tn;
    if (n >= N) return;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int m = m0 + tm * 4 + i;
        if (m >= M) continue;
        float r = (float)(acc[i][0] + acc[i][1]);
        if (add) r = __fadd_rn(add[(size_t)m * ldadd + n], r);
        y[(size_t)m * ldy + n] = r;
    }
}

// Rows x of width K = 512 (M <= 256) times F32 weights w [N][512] (the logits, src/gsv_ar.cpp:266),
// the arithmetic of k_gemm_f32d: products exact in double, accumulated in double, rounded once. A CTA
// owns 8 output columns x 32 rows; its weights (constant) are widened into shared memory before the
// wait for the rows. The 8 warps split K into 64-wide ranges with lane = row, 8 independent double
// chains per lane (one per column, each x value reused 8 times); the 8 range sums are added in range
// order.
constexpr int LG_COLS = 8, LG_ROWS = 32, LG_XSTR = D + 1;   // odd row stride: lane = row reads conflict-free
constexpr size_t LG_SMEM = (size_t)D * LG_COLS * 8 + (size_t)LG_ROWS * LG_XSTR * 4;
__global__ void __launch_bounds__(256) k_logits512(const float* __restrict__ x, int ldx, int M,
                                                   const float* __restrict__ w, int N, const float* __restrict__ add,
                                                   int ldadd, float* __restrict__ y, int ldy) {
    extern __shared__ __align__(16) uint8_t lg_sm[];
    double* sw = (double*)lg_sm;                                    // [D][LG_COLS], later [8][32][LG_COLS] sums
    float* sx = (float*)(lg_sm + (size_t)D * LG_COLS * 8);          // [LG_ROWS][LG_XSTR]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * LG_COLS, m0 = blockIdx.y * LG_ROWS;
    for (int i = tid; i < D * LG_COLS; i += 256) {
        const int c = i / D, k = i - c * D, n = n0 + c;
        sw[k * LG_COLS + c] = n < N ? (double)w[(size_t)n * D + k] : 0.0;
    }
    griddep_wait();
    griddep_launch();
    for (int i = tid; i < LG_ROWS * D; i += 256) {
        const int r = i / D, k = i - r * D, m = m0 + r;
        sx[r * LG_XSTR + k] = m < M ? x[(size_t)m * ldx + k] : 0.0f;
    }
    __syncthreads();
    double acc[LG_COLS];
#pragma unroll
    for (int j = 0; j < LG_COLS; j++) acc[j] = 0.0;
    const float* xr = sx + lane * LG_XSTR;
#pragma unroll 4
    for (int k = warp * 64; k < warp * 64 + 64; k++) {
        const double xv = (double)xr[k];
        const double2* wp = (const double2*)(sw + k * LG_COLS);
#pragma unroll
        for (int j = 0; j < LG_COLS / 2; j++) {
            const double2 ww = wp[j];
            acc[2 * j] = fma(xv, ww.x, acc[2 * j]);
            acc[2 * j + 1] = fma(xv, ww.y, acc[2 * j + 1]);
        }
    }
    __syncthreads();   // every warp is done with the weights: their space takes the range sums
    double* sred = sw;
#pragma unroll
    for (int j = 0; j < LG_COLS; j++) sred[(warp * LG_ROWS + lane) * LG_COLS + j] = acc[j];
    __syncthreads();
    const int r = tid / LG_COLS, c = tid % LG_COLS, m = m0 + r, n = n0 + c;
    double sum = 0.0;
#pragma unroll
    for (int q = 0; q < 8; q++) sum += sred[(q * LG_ROWS + r) * LG_COLS + c];
    if (m < M && n < N) {
        float v = (float)sum;
        if (add) v = __fadd_rn(add[(size_t)m * ldadd + n], v);
        y[(size_t)m * ldy + n] = v;
    }
}

// The same product on the FP64 tensor cores (mma.sync m8n8k4 .f64): a CTA owns 64 rows x 8 columns,
// warp w the 8 rows 64 blockIdx.y + 8 w. K is permuted between the k-steps (the double sums do not depend
// on their order at float precision): lane (r, c) supplies k = 128 c + ks of its row (A) and of column r
// (B) at k-step ks, so each lane streams two contiguous 512-byte runs with 16-byte loads. Two accumulator
// pairs (even / odd k-steps) are added at the end; the sum is rounded to float once.
__device__ __forceinline__ void lg_dmma(double& d0, double& d1, double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
                 : "+d"(d0), "+d"(d1)
                 : "d"(a), "d"(b));
}

__global__ void __launch_bounds__(256) k_logits_mma(const float* __restrict__ x, int ldx, int M,
                                                   const float* __restrict__ w, int N, const float* __restrict__ add,
                                                   int ldadd, float* __restrict__ y, int ldy) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, r = lane >> 2, c = lane & 3;
    const int n0 = blockIdx.x * 8, m0 = blockIdx.y * 64 + warp * 8;
    // the weights (constant) stream from before the wait for the rows
    const float4* wr = (const float4*)(w + (size_t)min(n0 + r, N - 1) * D + 128 * c);
    float4 wv[8];
#pragma unroll
    for (int j = 0; j < 8; j++) wv[j] = __ldg(wr + j);
    griddep_wait();
    griddep_launch();
    if (m0 >= M) return;
    const float4* xr = (const float4*)(x + (size_t)min(m0 + r, M - 1) * ldx + 128 * c);
    double a0 = 0.0, a1 = 0.0, b0 = 0.0, b1 = 0.0;
#pragma unroll
    for (int ch = 0; ch < 4; ch++) {   // 4 chunks of 32 k-steps (8 float4 of x and of w per lane)
        float4 xv[8];
#pragma unroll
        for (int j = 0; j < 8; j++) xv[j] = __ldg(xr + ch * 8 + j);
        float4 wn[8];
        if (ch < 3) {
#pragma unroll
            for (int j = 0; j < 8; j++) wn[j] = __ldg(wr + (ch + 1) * 8 + j);
        }
#pragma unroll
        for (int j = 0; j < 8; j++) {
            lg_dmma(a0, a1, (double)xv[j].x, (double)wv[j].x);
            lg_dmma(b0, b1, (double)xv[j].y, (double)wv[j].y);
            lg_dmma(a0, a1, (double)xv[j].z, (double)wv[j].z);
            lg_dmma(b0, b1, (double)xv[j].w, (double)wv[j].w);
        }
        if (ch < 3) {
#pragma unroll
            for (int j = 0; j < 8; j++) wv[j] = wn[j];
        }
    }
    // D[row r][column 2c + e]
#pragma unroll
    for (int e = 0; e < 2; e++) {
        const int m = m0 + r, n = n0 + 2 * c + e;
        if (m < M && n < N) {
            float v = (float)(e ? a1 + b1 : a0 + b0);
            if (add) v = __fadd_rn(add[(size_t)m * ldadd + n], v);
            y[(size_t)m * ldy + n] = v;
        }
    }
}

cudaError_t logits_init_device() {
    return cudaFuncSetAttribute(k_logits512, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)LG_SMEM);
}

void launch_gemm_f32d(const float* x, int ldx, const F32Gather* gather, int M, const float* w, int N, int K,
                      const float* add, int ldadd, float* y, int ldy, cudaStream_t s) {
    if (M <= 0) return;
    if (!gather && K == D && M <= 256 && (ldx & 3) == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)w & 15) == 0) {
        launch_pdl(k_logits_mma, dim3((N + 7) / 8, (M + 63) / 64), dim3(256), 0, s, x, ldx, M, w, N, add, ldadd, y,
                   ldy);
        return;
    }
    dim3 grid((N + 31) / 32, (M + 31) / 32);
    F32Gather g;
    if (gather) g = *gather;
    launch_pdl(k_gemm_f32d, grid, dim3(256), 0, s, x, ldx, g, gather ? 1 : 0, M, w, N, K, add, ldadd, y, ldy);
}

// ------------------------------------------------------------------ embeddings
// build_inputs (src/gsv_ar.cpp:201-214): text row = text_emb[ph] + alpha_t * pe[t],
// prompt row = audio_emb[code] + alpha_a * pe[t] (FMA, as the reference compiles with -mfma).
__global__ void k_prefill_embed(const PrefEmbedParams p) {
    const int m = blockIdx.x, d = threadIdx.x;
    griddep_wait();
    griddep_launch();
    if (m >= p.M) return;
    const int id = p.ids[m], pos = p.pe_pos[m];
    const bool text = p.is_text[m] != 0;
    const float e = text ? p.text_emb[(size_t)id * D + d] : p.audio_emb[(size_t)id * D + d];
    const float a = text ? p.text_alpha : p.audio_alpha;
    p.x[(size_t)m * D + d] = fmaf(a, p.pe[(size_t)pos * D + d], e);
}

void launch_prefill_embed(const PrefEmbedParams& p, cudaStream_t s) {
    if (p.M <= 0) return;
    launch_pdl(k_prefill_embed, dim3(p.M), dim3(D), 0, s, p);
}

// ------------------------------------------------------------------ step control
// Stop rules of the generate loop (src/gsv_ar.cpp:780-796) after this step's sampling, in the
// reference's order: EOS, then early stop keyed on the group's first sequence, then max_steps.
// Sequences still running get the next input, x = audio_emb[tok] + alpha_a * pe[prompt_len + idx]
// (:798-806), its Q8_0 planes, and their KV write position. One warp per slot.
__global__ void __launch_bounds__(128) k_step_prep(const StepPrepParams p) {
    const int slot = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    griddep_wait();
    griddep_launch();
    if (slot >= p.nslots) return;
    SlotState* st = p.st + slot;
    if (!st->active) {
        if (lane == 0) st->decode_now = 0;
        return;
    }
    const int idx = st->n_samp - 1;
    const int tok = p.out_tokens[(size_t)slot * p.tok_cap + idx];
    int kind = -1;
    if (tok == p.eos) kind = 0;
    else if (st->early_stop != -1 && p.st[st->group_first].n_samp > st->early_stop) kind = 1;
    else if (st->n_samp >= st->max_steps) kind = 2;
    __syncwarp();
    if (kind >= 0) {
        if (lane == 0) {
            st->finish_kind = kind;
            st->finish_idx = idx;
            st->active = 0;
            st->decode_now = 0;
        }
        return;
    }
    const int kvlen = st->kvlen;
    __syncwarp();
    if (lane == 0) {
        st->decode_now = 1;
        st->kvpos = kvlen;
        st->kvlen = kvlen + 1;
    }
    const int pos = st->prompt_len + idx;
    float x[16], amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; i++) {
        const int c = lane * 16 + i;
        x[i] = fmaf(p.audio_alpha, p.pe[(size_t)pos * D + c], p.audio_emb[(size_t)tok * D + c]);
        amax = fmaxf(amax, fabsf(x[i]));
    }
    float4* dst = (float4*)(p.x + (size_t)slot * D + lane * 16);
#pragma unroll
    for (int i = 0; i < 4; i++) dst[i] = make_float4(x[4 * i], x[4 * i + 1], x[4 * i + 2], x[4 * i + 3]);
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    float dsc, id;
    q8_scale(amax, dsc, id);
    uint32_t pk[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        uint32_t u = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) u |= (uint32_t)(uint8_t)q8_val(x[4 * i + j], id) << (8 * j);
        pk[i] = u;
    }
    *(uint4*)(p.xq + (size_t)slot * D + lane * 16) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    if ((lane & 1) == 0) p.xd[(size_t)slot * (D / QK) + lane / 2] = f2h(dsc);
}

void launch_step_prep(const StepPrepParams& p, cudaStream_t s) {
    launch_pdl(k_step_prep, dim3((p.nslots + 3) / 4), dim3(128), 0, s, p);
}

// ------------------------------------------------------------------ row gather / scatter
__global__ void k_copy_rows(float* __restrict__ dst, const int32_t* __restrict__ didx, const float* __restrict__ src,
                            const int32_t* __restrict__ sidx, int width) {
    const int r = blockIdx.x;
    griddep_wait();
    griddep_launch();
    const size_t so = (size_t)(sidx ? sidx[r] : r) * width, dof = (size_t)(didx ? didx[r] : r) * width;
    for (int c = threadIdx.x; c < width; c += blockDim.x) dst[dof + c] = src[so + c];
}

void launch_copy_rows(float* dst, const int32_t* didx, const float* src, const int32_t* sidx, int nrows, int width,
                      cudaStream_t s) {
    if (nrows <= 0) return;
    launch_pdl(k_copy_rows, dim3(nrows), dim3(256), 0, s, dst, didx, src, sidx, width);
}

}  // namespace gsvcu
