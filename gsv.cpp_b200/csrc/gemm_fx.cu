// gemm_fx.cu -- GEMMs that read float activations: F32 / F16 / BF16 weight matrices (the layer
// matrices of the exporter's default (F32) and --f16 files, tools/export_gguf/export.py:48-54, or of
// --spec ...=bf16, and an F16 / BF16 ar.predict: k_gemm_fx) and Q4_1 / Q5_1 matrices (k_gemm_qm, which
// quantizes its activation rows to Q8_1 itself).
//
// Arithmetic: ggml's F32 / F16 mul_mat (src/gsv_ar.cpp:244,260,262,263,266) in the order of its
// FMA-vectorised dot (ggml_vec_dot_f32 / ggml_vec_dot_f16 built with -mavx2 -mfma: four 8-lane
// float accumulators over steps of 32 values). For an F16 / BF16 matrix the activations are first
// rounded to F16 / BF16 (round-to-nearest-even), as ggml converts src1 to the matrix's vec_dot_type;
// F16 and BF16 products are then exact in float. BF16 takes the same order (ggml's AVX2 BF16 dot may
// pair the last two lane sums the other way round; this build defines it as the F16 order). Chain c
// (c = 0..31) accumulates w[k] * x[k] for k = c, c + 32, ... with one FMA per term; the 32 chain sums
// are then added pairwise: chain c with c^16 (accumulators 0+2, 1+3), ^8 (0+1), ^4 (the two 128-bit
// halves), ^1 and ^2 (the two horizontal adds). K is a multiple of 32.
//
// Mapping: lane c of a warp runs chain c. A warp owns 8 rows x 8 columns (64 chains per lane: each x
// value feeds 8 FMAs, each weight 8); the pairwise fold is a transposing butterfly that halves the
// values a lane holds at each level (32 + 16 + 8 + 4 + 2 shuffles for 64 outputs), after which each
// lane holds two finished outputs. A CTA of 4 warps covers 16 rows x 16 columns and streams its x rows
// and weight rows through a cp.async pipeline of 256-value (F16 / BF16) or 128-value (F32) slices (a
// lane reads k = 32t + c of a slice from shared memory, conflict-free); the weight slices of the first
// stages are requested before the wait for the predecessor kernel. K is a multiple of 256 here.
#include <cuda_bf16.h>

#include <type_traits>

#include "kernels.h"

namespace gsvcu {
namespace {

constexpr int FX_RW = 8, FX_CW = 8;              // warp tile: rows x columns
constexpr int FX_WM = 2, FX_WN = 2;              // warps per CTA along rows / columns
constexpr int FX_TM = FX_RW * FX_WM, FX_TN = FX_CW * FX_WN;
constexpr int FX_NV = FX_RW * FX_CW;             // outputs per warp
// Pipeline: stages of FX_KC<WT> k values (8 or 4 chain steps), FX_ST<WT> of them in flight, 48 KB of
// shared memory: at decode sizes a GEMM is a few long stages, so it pays few load round trips.
template <int WT> constexpr int FX_KC = WT == FX_F32 ? 128 : 256;
template <int WT> constexpr int FX_ST = WT == FX_F32 ? 3 : 2;
constexpr int FX_KMULT = 256;                    // K must be a multiple of this (every type's stage)

template <int WT>
using fx_wt = typename std::conditional<WT == FX_F16, __half,
                                        typename std::conditional<WT == FX_BF16, __nv_bfloat16, float>::type>::type;

template <int WT>
struct FxSmem {
    float x[FX_ST<WT>][FX_TM][FX_KC<WT>];
    fx_wt<WT> w[FX_ST<WT>][FX_TN][FX_KC<WT>];
};

__device__ __forceinline__ void fx_cp16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}

__device__ __forceinline__ float widen(float v) { return v; }
__device__ __forceinline__ float widen(__half v) { return __half2float(v); }
__device__ __forceinline__ float widen(__nv_bfloat16 v) { return __bfloat162float(v); }

// the activation as ggml converts src1 for a matrix of type WT (vec_dot_type): F16 / BF16, RNE
template <int WT>
__device__ __forceinline__ float round_x(float v) {
    if (WT == FX_F16) return __half2float(__float2half_rn(v));
    if (WT == FX_BF16) return __bfloat162float(__float2bfloat16_rn(v));
    return v;
}

// One level of the pairwise fold over the first N values of every lane: lanes l and l^OFF hold the
// same outputs' sums of chain groups l and l^OFF; lane l keeps the lower half of the outputs when bit
// OFF of l is clear, the upper half otherwise, and receives its partner's sums for them.
template <int OFF, int N>
__device__ __forceinline__ void fold(float (&v)[FX_NV], int lane) {
    const bool up = (lane & OFF) != 0;
#pragma unroll
    for (int i = 0; i < N / 2; i++) {
        const float send = up ? v[i] : v[i + N / 2];
        const float keep = up ? v[i + N / 2] : v[i];
        v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, OFF));
    }
}

// K/V column f (in [D, 3D)) of row n into its KV page: the layout and conversion of the Q8_0 GEMM's
// epilogue (prefill rows by tok_slot / tok_pos, decode rows by the slot state).
__device__ __forceinline__ void kv_store(const KvWrite& kv, int n, int f, float y) {
    int slot, pos;
    if (kv.tok_pos) {
        slot = kv.tok_slot[n];
        pos = kv.tok_pos[n];
    } else {
        if (!kv.st[n].decode_now) return;
        slot = n;
        pos = kv.st[n].kvpos;
    }
    const int kvsel = (f - D) >> 9, fh = (f - D) & (D - 1);
    const int h = fh >> 5, dd = fh & 31;
    const int page = kv.block_table[(size_t)slot * kv.max_pages + pos / PAGE];
    const size_t e = ((((size_t)page * kv.n_layer + kv.layer) * 2 + kvsel) * NH + h) * (PAGE * HD) +
                     (size_t)(pos % PAGE) * HD + dd;
    if (kv.kv_f32) ((float*)kv.pool)[e] = y;
    else ((__half*)kv.pool)[e] = __float2half_rn(y);
}

// One output's epilogue: bias (+ K/V page store), residual or bias + ReLU.
template <int EPI>
__device__ __forceinline__ void fx_store(const GemmFxParams& p, int m, int n, float a) {
    if (m >= p.M || n >= p.N) return;
    const float bias = p.bias ? p.bias[n] : 0.0f;
    if (EPI == FXE_BIAS) {
        const float y = __fadd_rn(a, bias);
        if (n < (p.n_store ? p.n_store : p.N)) p.y[(size_t)m * (p.ldy ? p.ldy : p.N) + n] = y;
        if (p.kv.pool && n >= D) kv_store(p.kv, m, n, y);
    } else if (EPI == FXE_RESID) {
        const float r = p.resid[(size_t)m * p.N + n];
        p.y[(size_t)m * p.N + n] = __fadd_rn(__fadd_rn(r, a), bias);
    } else {   // FXE_RELU
        const float h = __fadd_rn(a, bias);
        p.y[(size_t)m * p.N + n] = h > 0.0f ? h : 0.0f;
    }
}

template <int WT, int EPI>
__global__ void __launch_bounds__(128) k_gemm_fx(const GemmFxParams p) {
    __shared__ __align__(16) FxSmem<WT> sm;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mt = blockIdx.y * FX_TM, nt = blockIdx.x * FX_TN;   // the CTA's first row / column
    const int wr = (warp / FX_WN) * FX_RW, wc = (warp % FX_WN) * FX_CW;
    const int m0 = mt + wr, n0 = nt + wc;
    constexpr int KC = FX_KC<WT>, ST = FX_ST<WT>;
    const int nch = p.K / KC;
    // one stage = the CTA's 16 x rows and 16 weight rows over 64 k values, in 16-byte copies; rows /
    // columns past the edge copy the last valid one (their sums are never stored)
    constexpr int XCH = KC * 4 / 16, WCH = KC * (int)sizeof(fx_wt<WT>) / 16;   // 16-byte chunks per row
    auto load_w = [&](int st, int c) {
        for (int q = tid; q < FX_TN * WCH; q += 128) {
            const int j = q / WCH, part = q % WCH;
            const fx_wt<WT>* src = (const fx_wt<WT>*)p.w + (size_t)min(nt + j, p.N - 1) * p.K + c * KC +
                                   part * (16 / (int)sizeof(fx_wt<WT>));
            fx_cp16(&sm.w[st][j][part * (16 / (int)sizeof(fx_wt<WT>))], src);
        }
    };
    auto load_x = [&](int st, int c) {
        for (int q = tid; q < FX_TM * XCH; q += 128) {
            const int r = q / XCH, part = q % XCH;
            fx_cp16(&sm.x[st][r][part * 4], p.x + (size_t)min(mt + r, p.M - 1) * p.ldx + c * KC + part * 4);
        }
    };
    float acc[FX_NV];
#pragma unroll
    for (int i = 0; i < FX_NV; i++) acc[i] = 0.0f;
    for (int s = 0; s < ST - 1; s++)   // weights do not depend on the predecessor kernel
        if (s < nch) load_w(s, s);
    griddep_wait();
    griddep_launch();
    for (int s = 0; s < ST - 1; s++) {   // group s: stage s's x (group 0 also the weights above)
        if (s < nch) load_x(s, s);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (int c = 0; c < nch; c++) {
        asm volatile("cp.async.wait_group %0;" ::"n"(ST - 2) : "memory");   // stage c has landed
        __syncthreads();   // ... for every thread, and stage c - 1 is free again
        const int cn = c + ST - 1;
        if (cn < nch) {
            load_w(cn % ST, cn);
            load_x(cn % ST, cn);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        const int st = c % ST;
#pragma unroll
        for (int t = 0; t < KC / 32; t++) {   // chain step k = c*KC + 32t + lane
            float xv[FX_RW], wv[FX_CW];
#pragma unroll
            for (int r = 0; r < FX_RW; r++) {
                xv[r] = round_x<WT>(sm.x[st][wr + r][32 * t + lane]);
            }
#pragma unroll
            for (int j = 0; j < FX_CW; j++) wv[j] = widen(sm.w[st][wc + j][32 * t + lane]);
#pragma unroll
            for (int r = 0; r < FX_RW; r++)
#pragma unroll
                for (int j = 0; j < FX_CW; j++) acc[r * FX_CW + j] = fmaf(wv[j], xv[r], acc[r * FX_CW + j]);
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    fold<16, 64>(acc, lane);
    fold<8, 32>(acc, lane);
    fold<4, 16>(acc, lane);
    fold<1, 8>(acc, lane);
    fold<2, 4>(acc, lane);
    // acc[e], e = 0, 1: output index 32 b4 + 16 b3 + 8 b2 + 4 b0 + 2 b1 + e (b = the lane's bits),
    // i.e. row 4 b4 + 2 b3 + b2 and column 4 b0 + 2 b1 + e of the warp tile
    const int m = m0 + ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
    const int nb = n0 + (lane & 1) * 4 + ((lane >> 1) & 1) * 2;
#pragma unroll
    for (int e = 0; e < 2; e++) fx_store<EPI>(p, m, nb + e, acc[e]);
}

// Q4_1 / Q5_1 matrices: ggml's Q4_1 / Q5_1 x Q8_1 mul_mat in the order of its portable C dot, in two
// kernels. k_quant_q8_1 quantizes every activation row once to Q8_1 (quantize_row_q8_1_ref: the Q8_0
// values and fp16 scale, plus s = fp16(sum of the values * d) with the unrounded d), a thread per block.
// k_gemm_qm: a CTA owns 32 rows x 8 columns; the columns' weights (before the wait for the predecessor)
// and the rows' Q8_1 values are staged in shared memory by cp.async. Warp w runs column w for the 32
// rows, lane = row, block by block: sumi = the exact integer dot of the weight's unsigned 4- / 5-bit
// values (bytes since load) with the activation block, acc = acc + fma(d_w*d_x, sumi, m_w*s_x). K is a
// multiple of 32, at most QM_KMAX.
constexpr int QM_R = 32, QM_C = 8, QM_KMAX = 2048;
// shared memory: the columns' weights, the rows' Q8_1 values (padded rows), the rows' d and s
// block-major, the columns' (d, m) block-major
constexpr size_t qm_smem_bytes(int K) {
    return (size_t)QM_C * K + (size_t)QM_R * (K + 16) + (size_t)(K / 32) * QM_R * 8 + (size_t)(K / 32) * QM_C * 8;
}
constexpr size_t QM_SMEM = qm_smem_bytes(QM_KMAX);

__global__ void __launch_bounds__(256) k_quant_q8_1(const float* __restrict__ x, int ldx, int M, int K,
                                                    int8_t* __restrict__ xq, float* __restrict__ xd,
                                                    float* __restrict__ xs) {
    griddep_wait();
    griddep_launch();
    const int nb = K / 32;
    const int i = blockIdx.x * 256 + threadIdx.x;
    if (i >= M * nb) return;
    const int r = i / nb, b = i - r * nb;
    const float* src = x + (size_t)r * ldx + b * 32;
    float v[32], amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
        *(float4*)&v[j] = *(const float4*)(src + j);
#pragma unroll
        for (int k = 0; k < 4; k++) amax = fmaxf(amax, fabsf(v[j + k]));
    }
    float d, id;
    q8_scale(amax, d, id);
    int sum = 0;
    int8_t* dst = xq + (size_t)r * K + b * 32;
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
        const int8_t q0 = q8_val(v[j], id), q1 = q8_val(v[j + 1], id), q2 = q8_val(v[j + 2], id),
                     q3 = q8_val(v[j + 3], id);
        *(uint32_t*)(dst + j) = (uint32_t)(uint8_t)q0 | ((uint32_t)(uint8_t)q1 << 8) | ((uint32_t)(uint8_t)q2 << 16) |
                                ((uint32_t)(uint8_t)q3 << 24);
        sum += q0 + q1 + q2 + q3;
    }
    xd[(size_t)r * nb + b] = h2f(f2h(d));
    xs[(size_t)r * nb + b] = h2f(f2h(__fmul_rn((float)sum, d)));
}

template <int EPI>
__global__ void __launch_bounds__(256) k_gemm_qm(const GemmFxParams p) {
    extern __shared__ __align__(16) uint8_t qm_smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nb = p.K / 32, ldx = p.K + 16;
    uint8_t* ws = qm_smem;                                     // [8 columns][K]
    int8_t* xs = (int8_t*)(qm_smem + (size_t)QM_C * p.K);      // [32 rows][K + 16]
    float* sd = (float*)(xs + (size_t)QM_R * ldx);              // [block][32 rows] d of the rows
    float* ss = sd + nb * QM_R;                                 // [block][32 rows] s of the rows
    float2* swm = (float2*)(ss + nb * QM_R);                    // [block][8 columns] (d, m) of the weights
    const int mt = blockIdx.y * QM_R, nt = blockIdx.x * QM_C;
    // the weights and their scales do not depend on the predecessor: staged before its wait
    for (int q = tid; q < QM_C * p.K / 16; q += 256) {
        const int c = q / (p.K / 16), part = q - c * (p.K / 16);
        fx_cp16(ws + (size_t)c * p.K + part * 16, (const uint8_t*)p.w + (size_t)min(nt + c, p.N - 1) * p.K + part * 16);
    }
    for (int i = tid; i < nb * QM_C; i += 256) {
        const int b = i / QM_C, col = min(nt + i % QM_C, p.N - 1);
        swm[i] = make_float2(h2f(p.wd[(size_t)col * nb + b]), h2f(p.wm[(size_t)col * nb + b]));
    }
    griddep_wait();
    griddep_launch();
    for (int q = tid; q < QM_R * p.K / 16; q += 256) {
        const int r = q / (p.K / 16), part = q - r * (p.K / 16);
        fx_cp16(xs + (size_t)r * ldx + part * 16, p.qx_q + (size_t)min(mt + r, p.M - 1) * p.K + part * 16);
    }
    for (int i = tid; i < nb * QM_R; i += 256) {
        const int b = i / QM_R, row = min(mt + i % QM_R, p.M - 1);
        sd[i] = p.qx_d[(size_t)row * nb + b];
        ss[i] = ((const float*)p.qx_s)[(size_t)row * nb + b];
    }
    asm volatile("cp.async.commit_group;\n cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    const int col = nt + warp, row = mt + lane;
    if (col >= p.N || row >= p.M) return;
    const int4* wl = (const int4*)(ws + (size_t)warp * p.K);
    const int4* xl = (const int4*)(xs + (size_t)lane * ldx);
    float acc = 0.0f;
    for (int b = 0; b < nb; b++) {
        const int4 w0 = wl[2 * b], w1 = wl[2 * b + 1], x0 = xl[2 * b], x1 = xl[2 * b + 1];
        int sumi = __dp4a(w0.x, x0.x, 0);
        sumi = __dp4a(w0.y, x0.y, sumi);
        sumi = __dp4a(w0.z, x0.z, sumi);
        sumi = __dp4a(w0.w, x0.w, sumi);
        sumi = __dp4a(w1.x, x1.x, sumi);
        sumi = __dp4a(w1.y, x1.y, sumi);
        sumi = __dp4a(w1.z, x1.z, sumi);
        sumi = __dp4a(w1.w, x1.w, sumi);
        const float2 wm2 = swm[b * QM_C + warp];
        const float dd = __fmul_rn(wm2.x, sd[b * QM_R + lane]);
        const float ms = __fmul_rn(wm2.y, ss[b * QM_R + lane]);
        acc = __fadd_rn(acc, fmaf(dd, (float)sumi, ms));
    }
    fx_store<EPI>(p, row, col, acc);
}

// K-quant matrices (Q4_K / Q5_K / Q6_K): ggml's K-quant x Q8_K mul_mat in the order of its portable C
// dot, in two kernels.
// k_quant_q8k quantizes every activation row once to Q8_K (quantize_row_q8_K_ref, per 256 values: max =
// the value of largest magnitude, first one winning; iscale = -127/max; q = min(127,
// round-half-even(iscale*x)); d = 1/iscale; sums of 16), a warp per (row, super-block): lane l holds
// values 8l..8l+7, the max is a shuffle reduction of (|v|, first index), and the super-block is stored
// lane-major like the weights (value e at (e % 8) * 32 + e / 8).
// k_gemm_qk: a CTA owns 32 rows x 8 columns; the columns' weights (before the wait for the predecessor)
// and the rows' Q8_K values are staged in shared memory by cp.async. Its warps then take (column,
// super-block) tasks: lane = row, the column's weights one broadcast load for the warp, the eight exact
// lane sums of a super-block (value e to lane e % 8) of the pre-scaled int16 weights times the int8
// activations (16 dp2a per lane) into shared memory. Then thread (row, column) runs the float chain in super-block order: sums[l] =
// fma(d_w*d_x, lane_l, sums[l]); Q4_K / Q5_K also sumf = fma(-dmin_w*d_x, sum_g bsums[g]*min[g/2],
// sumf); at the end sumf + sums[0] + ... + sums[7]. K is a multiple of 256, at most QK_KMAX.
constexpr int QK_R = 32, QK_C = 8, QK_KMAX = 2048;
// shared memory: the columns' weights, the rows' Q8_K values (padded rows), the int32 lane sums
constexpr size_t qk_smem_bytes(int K) {
    return (size_t)QK_C * K * 2 + (size_t)QK_R * (K + 16) + (size_t)QK_C * (K / 256) * 8 * QK_R * 4 +
           (size_t)(K / 256) * QK_R * 4              // the rows' d, super-block-major
           + (size_t)(K / 256) * QK_C * (8 + 8)      // the columns' (d, dmin) and 8 sub-block mins
           + (size_t)(K / 16) * QK_R * 4;            // the rows' sums of 16, group-major
}
constexpr size_t QK_SMEM = qk_smem_bytes(QK_KMAX);

__global__ void __launch_bounds__(256) k_quant_q8k(const float* __restrict__ x, int ldx, int M, int K,
                                                   int8_t* __restrict__ xq, float* __restrict__ xd,
                                                   int32_t* __restrict__ xbs) {
    griddep_wait();
    griddep_launch();
    const int lane = threadIdx.x & 31, nsb = K / 256;
    const int task = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (task >= M * nsb) return;
    const int r = task / nsb, sb = task - r * nsb;
    const float* src = x + (size_t)r * ldx + sb * 256 + lane * 8;
    float v[8];
    *(float4*)&v[0] = *(const float4*)src;
    *(float4*)&v[4] = *(const float4*)(src + 4);
    float amax = 0.0f, mx = 0.0f;
    int idx = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < 8; i++)
        if (fabsf(v[i]) > amax) {
            amax = fabsf(v[i]);
            mx = v[i];
            idx = lane * 8 + i;
        }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {   // larger magnitude wins, the first index on a tie
        const float oa = __shfl_xor_sync(0xffffffffu, amax, off), om = __shfl_xor_sync(0xffffffffu, mx, off);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
        if (oa > amax || (oa == amax && oi < idx)) {
            amax = oa;
            mx = om;
            idx = oi;
        }
    }
    const float iscale = amax != 0.0f ? __fdiv_rn(-127.0f, mx) : 0.0f;
    int8_t* dst = xq + (size_t)r * K + sb * 256;
    int s = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {   // value e = 8 lane + i at (e % 8) * 32 + e / 8 = i * 32 + lane
        const int q = amax != 0.0f ? min(127, __float2int_rn(__fmul_rn(iscale, v[i]))) : 0;
        dst[i * 32 + lane] = (int8_t)q;
        s += q;
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);   // sum of 16: lanes 2g, 2g + 1
    if ((lane & 1) == 0) xbs[(size_t)r * (K / 16) + sb * 16 + (lane >> 1)] = s;
    if (lane == 0) xd[(size_t)r * nsb + sb] = amax != 0.0f ? __fdiv_rn(1.0f, iscale) : 0.0f;
}

template <int EPI>
__global__ void __launch_bounds__(256) k_gemm_qk(const GemmFxParams p) {
    extern __shared__ __align__(16) uint8_t qk_smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nsb = p.K / 256, ldx = p.K + 16;
    int16_t* ws = (int16_t*)qk_smem;                                  // [8 columns][K]
    int8_t* xs = (int8_t*)(qk_smem + (size_t)QK_C * p.K * 2);         // [32 rows][K + 16]
    int32_t* ls = (int32_t*)(xs + (size_t)QK_R * ldx);                // [column][super-block][lane 8][row 32]
    float* sxd = (float*)(ls + (size_t)QK_C * nsb * 8 * QK_R);        // [super-block][row 32]
    float2* swd = (float2*)(sxd + nsb * QK_R);                         // [super-block][column 8] (d, dmin)
    uint2* smn = (uint2*)(swd + nsb * QK_C);                           // [super-block][column 8] mins
    int32_t* sbs = (int32_t*)(smn + nsb * QK_C);                       // [group of 16][row 32]
    const int mt = blockIdx.y * QK_R, nt = blockIdx.x * QK_C;
    // the columns' weights and scales do not depend on the predecessor kernel: staged before its wait
    for (int q = tid; q < QK_C * p.K / 8; q += 256) {
        const int c = q / (p.K / 8), part = q - c * (p.K / 8);
        fx_cp16(ws + (size_t)c * p.K + part * 8, (const int16_t*)p.w + (size_t)min(nt + c, p.N - 1) * p.K + part * 8);
    }
    for (int i = tid; i < nsb * QK_C; i += 256) {
        const int sb = i / QK_C, col = min(nt + i % QK_C, p.N - 1);
        const size_t e = (size_t)col * nsb + sb;
        swd[i] = make_float2(h2f(p.wd[e]), p.wmins ? h2f(p.wm[e]) : 0.0f);
        smn[i] = p.wmins ? *(const uint2*)(p.wmins + e * 8) : make_uint2(0u, 0u);
    }
    griddep_wait();
    griddep_launch();
    for (int q = tid; q < QK_R * p.K / 16; q += 256) {
        const int r = q / (p.K / 16), part = q - r * (p.K / 16);
        fx_cp16(xs + (size_t)r * ldx + part * 16, p.qx_q + (size_t)min(mt + r, p.M - 1) * p.K + part * 16);
    }
    for (int i = tid; i < nsb * QK_R; i += 256) {
        const int sb = i / QK_R, row = min(mt + i % QK_R, p.M - 1);
        sxd[i] = p.qx_d[(size_t)row * nsb + sb];
    }
    if (p.wmins)
        for (int i = tid; i < (p.K / 16) * QK_R; i += 256) {
            const int gg = i / QK_R, row = min(mt + i % QK_R, p.M - 1);
            sbs[i] = ((const int32_t*)p.qx_s)[(size_t)row * (p.K / 16) + gg];
        }
    asm volatile("cp.async.commit_group;\n cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    // (column, super-block) tasks: lane = row, the eight exact lane sums of the super-block; the 16 dp2a
    // of a lane sum run as two chains (integer sums: exact in any order)
    for (int task = warp; task < QK_C * nsb; task += 8) {
        const int c = task / nsb, sb = task - c * nsb;
        const int4* wl = (const int4*)(ws + (size_t)c * p.K) + sb * 32;
        const int4* xl = (const int4*)(xs + (size_t)lane * ldx + sb * 256);
        int32_t* dst = ls + ((size_t)(c * nsb + sb) * 8) * QK_R + lane;
#pragma unroll
        for (int l = 0; l < 8; l++) {   // lane l of the super-block: 32 activations, 32 weights
            const int4 x0 = xl[2 * l], x1 = xl[2 * l + 1];
            const int xw[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            int a0 = 0, a1 = 0;
#pragma unroll
            for (int k = 0; k < 4; k += 2) {
                const int4 w = wl[l * 4 + k], v = wl[l * 4 + k + 1];
                a0 = __dp2a_lo(w.x, xw[2 * k], a0);
                a0 = __dp2a_hi(w.y, xw[2 * k], a0);
                a0 = __dp2a_lo(w.z, xw[2 * k + 1], a0);
                a0 = __dp2a_hi(w.w, xw[2 * k + 1], a0);
                a1 = __dp2a_lo(v.x, xw[2 * k + 2], a1);
                a1 = __dp2a_hi(v.y, xw[2 * k + 2], a1);
                a1 = __dp2a_lo(v.z, xw[2 * k + 3], a1);
                a1 = __dp2a_hi(v.w, xw[2 * k + 3], a1);
            }
            dst[l * QK_R] = a0 + a1;
        }
    }
    __syncthreads();
    // thread (row = lane, column = warp): the float chain over the super-blocks
    const int col = nt + warp, row = mt + lane;
    if (col >= p.N || row >= p.M) return;
    float sums[8], sumf = 0.0f;
#pragma unroll
    for (int l = 0; l < 8; l++) sums[l] = 0.0f;
    for (int sb = 0; sb < nsb; sb++) {
        const float xds = sxd[sb * QK_R + lane];
        const float2 wdm = swd[sb * QK_C + warp];
        const float dd = __fmul_rn(wdm.x, xds);
        const int32_t* lsb = ls + ((size_t)(warp * nsb + sb) * 8) * QK_R + lane;
#pragma unroll
        for (int l = 0; l < 8; l++) sums[l] = fmaf(dd, (float)lsb[l * QK_R], sums[l]);
        if (p.wmins) {
            const uint2 m8 = smn[sb * QK_C + warp];
            const uint32_t mw[2] = {m8.x, m8.y};
            int sumi = 0;
#pragma unroll
            for (int g = 0; g < 16; g++)
                sumi += sbs[(sb * 16 + g) * QK_R + lane] * (int)((mw[g >> 3] >> (8 * ((g >> 1) & 3))) & 0xff);
            const float dmin = __fmul_rn(wdm.y, xds);
            sumf = fmaf(-dmin, (float)sumi, sumf);
        }
    }
#pragma unroll
    for (int l = 0; l < 8; l++) sumf = __fadd_rn(sumf, sums[l]);
    fx_store<EPI>(p, row, col, sumf);
}

template <int WT>
void launch_wt(const GemmFxParams& p, int epi, cudaStream_t s) {
    const dim3 grid((p.N + FX_TN - 1) / FX_TN, (p.M + FX_TM - 1) / FX_TM), block(128);
    switch (epi) {
        case FXE_BIAS: launch_pdl(k_gemm_fx<WT, FXE_BIAS>, grid, block, 0, s, p); break;
        case FXE_RESID: launch_pdl(k_gemm_fx<WT, FXE_RESID>, grid, block, 0, s, p); break;
        default: launch_pdl(k_gemm_fx<WT, FXE_RELU>, grid, block, 0, s, p); break;
    }
}

}  // namespace

cudaError_t gemm_fx_init_device() {
    cudaError_t e;
#define GSVCU_QK_SMEM(EPI_)                                                                                     \
    if ((e = cudaFuncSetAttribute(k_gemm_qk<EPI_>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)QK_SMEM)))    \
        return e;
    GSVCU_QK_SMEM(FXE_BIAS) GSVCU_QK_SMEM(FXE_RESID) GSVCU_QK_SMEM(FXE_RELU)
#undef GSVCU_QK_SMEM
#define GSVCU_QM_SMEM(EPI_)                                                                                     \
    if ((e = cudaFuncSetAttribute(k_gemm_qm<EPI_>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)QM_SMEM)))    \
        return e;
    GSVCU_QM_SMEM(FXE_BIAS) GSVCU_QM_SMEM(FXE_RESID) GSVCU_QM_SMEM(FXE_RELU)
#undef GSVCU_QM_SMEM
    return cudaSuccess;
}

void launch_gemm_fx(const GemmFxParams& p, int epi, cudaStream_t s) {
    if (p.M <= 0 || p.N <= 0) return;
    if (p.wtype == FX_QK) {
        if (p.K % 256 || p.K > QK_KMAX || !p.qx_q || !p.qx_d || !p.qx_s) return;
        const int tasks = p.M * (p.K / 256);
        launch_pdl(k_quant_q8k, dim3((tasks + 7) / 8), dim3(256), 0, s, p.x, p.ldx, p.M, p.K, p.qx_q, p.qx_d,
                   (int32_t*)p.qx_s);
        const dim3 grid((p.N + QK_C - 1) / QK_C, (p.M + QK_R - 1) / QK_R), block(256);
        const size_t smem = qk_smem_bytes(p.K);
        switch (epi) {
            case FXE_BIAS: launch_pdl(k_gemm_qk<FXE_BIAS>, grid, block, smem, s, p); break;
            case FXE_RESID: launch_pdl(k_gemm_qk<FXE_RESID>, grid, block, smem, s, p); break;
            default: launch_pdl(k_gemm_qk<FXE_RELU>, grid, block, smem, s, p); break;
        }
        return;
    }
    if (p.wtype == FX_QM) {
        if (p.K % 32 || p.K > QM_KMAX || !p.qx_q || !p.qx_d || !p.qx_s) return;
        const int blocks = p.M * (p.K / 32);
        launch_pdl(k_quant_q8_1, dim3((blocks + 255) / 256), dim3(256), 0, s, p.x, p.ldx, p.M, p.K, p.qx_q, p.qx_d,
                   (float*)p.qx_s);
        const dim3 grid((p.N + QM_C - 1) / QM_C, (p.M + QM_R - 1) / QM_R), block(256);
        const size_t smem = qm_smem_bytes(p.K);
        switch (epi) {
            case FXE_BIAS: launch_pdl(k_gemm_qm<FXE_BIAS>, grid, block, smem, s, p); break;
            case FXE_RESID: launch_pdl(k_gemm_qm<FXE_RESID>, grid, block, smem, s, p); break;
            default: launch_pdl(k_gemm_qm<FXE_RELU>, grid, block, smem, s, p); break;
        }
        return;
    }
    if (p.K % FX_KMULT) return;
    if (p.wtype == FX_F16) launch_wt<FX_F16>(p, epi, s);
    else if (p.wtype == FX_BF16) launch_wt<FX_BF16>(p, epi, s);
    else launch_wt<FX_F32>(p, epi, s);
}

}  // namespace gsvcu
