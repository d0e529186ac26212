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
// and weight rows through a 4-stage cp.async pipeline of 64-value slices (a lane reads k = 32t + c of
// a slice from shared memory, conflict-free); the weight slices of the first stages are requested
// before the wait for the predecessor kernel. K is a multiple of 64 here.
#include <cuda_bf16.h>

#include <type_traits>

#include "kernels.h"

namespace gsvcu {
namespace {

constexpr int FX_RW = 8, FX_CW = 8;              // warp tile: rows x columns
constexpr int FX_WM = 2, FX_WN = 2;              // warps per CTA along rows / columns
constexpr int FX_TM = FX_RW * FX_WM, FX_TN = FX_CW * FX_WN;
constexpr int FX_NV = FX_RW * FX_CW;             // outputs per warp
constexpr int FX_KC = 64;                        // k values per pipeline stage (two chain steps)
constexpr int FX_ST = 4;                         // pipeline stages

template <int WT>
using fx_wt = typename std::conditional<WT == FX_F16, __half,
                                        typename std::conditional<WT == FX_BF16, __nv_bfloat16, float>::type>::type;

template <int WT>
struct FxSmem {
    float x[FX_ST][FX_TM][FX_KC];
    fx_wt<WT> w[FX_ST][FX_TN][FX_KC];
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
    const int nch = p.K / FX_KC;
    // one stage = the CTA's 16 x rows and 16 weight rows over 64 k values, in 16-byte copies; rows /
    // columns past the edge copy the last valid one (their sums are never stored)
    constexpr int XCH = FX_KC * 4 / 16, WCH = FX_KC * (int)sizeof(fx_wt<WT>) / 16;   // 16-byte chunks per row
    auto load_w = [&](int st, int c) {
        for (int q = tid; q < FX_TN * WCH; q += 128) {
            const int j = q / WCH, part = q % WCH;
            const fx_wt<WT>* src = (const fx_wt<WT>*)p.w + (size_t)min(nt + j, p.N - 1) * p.K + c * FX_KC +
                                   part * (16 / (int)sizeof(fx_wt<WT>));
            fx_cp16(&sm.w[st][j][part * (16 / (int)sizeof(fx_wt<WT>))], src);
        }
    };
    auto load_x = [&](int st, int c) {
        for (int q = tid; q < FX_TM * XCH; q += 128) {
            const int r = q / XCH, part = q % XCH;
            fx_cp16(&sm.x[st][r][part * 4], p.x + (size_t)min(mt + r, p.M - 1) * p.ldx + c * FX_KC + part * 4);
        }
    };
    float acc[FX_NV];
#pragma unroll
    for (int i = 0; i < FX_NV; i++) acc[i] = 0.0f;
    for (int s = 0; s < FX_ST - 1; s++)   // weights do not depend on the predecessor kernel
        if (s < nch) load_w(s, s);
    griddep_wait();
    griddep_launch();
    for (int s = 0; s < FX_ST - 1; s++) {   // group s: stage s's x (group 0 also the weights above)
        if (s < nch) load_x(s, s);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (int c = 0; c < nch; c++) {
        asm volatile("cp.async.wait_group %0;" ::"n"(FX_ST - 2) : "memory");   // stage c has landed
        __syncthreads();   // ... for every thread, and stage c - 1 is free again
        const int cn = c + FX_ST - 1;
        if (cn < nch) {
            load_w(cn % FX_ST, cn);
            load_x(cn % FX_ST, cn);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        const int st = c % FX_ST;
#pragma unroll
        for (int t = 0; t < FX_KC / 32; t++) {   // chain step k = c*64 + 32t + lane
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

// Q4_1 / Q5_1 matrices: ggml's Q4_1 / Q5_1 x Q8_1 mul_mat in the order of its portable C dot. The CTA
// first quantizes its 16 activation rows to Q8_1 in shared memory (quantize_row_q8_1_ref: the Q8_0
// values and fp16 scale, plus s = fp16(sum of the values * d) with the unrounded d); thread (r, c) then
// runs output (row r, column c) block by block: sumi = the exact integer dot of the weight's unsigned
// 4- / 5-bit values (bytes since load) with the activation block, acc = acc + fma(d_w*d_x, sumi,
// m_w*s_x). K is a multiple of 32, at most QM_KMAX.
constexpr int QM_T = 16, QM_KMAX = 2048;

template <int EPI>
__global__ void __launch_bounds__(256) k_gemm_qm(const GemmFxParams p) {
    __shared__ __align__(16) int8_t xq[QM_T][QM_KMAX];
    __shared__ float xd[QM_T][QM_KMAX / 32], xs[QM_T][QM_KMAX / 32];
    const int tid = threadIdx.x, nb = p.K / 32;
    const int mt = blockIdx.y * QM_T, nt = blockIdx.x * QM_T;
    griddep_wait();
    griddep_launch();
    for (int i = tid; i < QM_T * nb; i += 256) {
        const int r = i / nb, b = i - r * nb;
        const float* src = p.x + (size_t)min(mt + r, p.M - 1) * p.ldx + b * 32;
        float v[32], amax = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; j++) {
            v[j] = src[j];
            amax = fmaxf(amax, fabsf(v[j]));
        }
        float d, id;
        q8_scale(amax, d, id);
        int sum = 0;
#pragma unroll
        for (int j = 0; j < 32; j++) {
            const int8_t q = q8_val(v[j], id);
            xq[r][b * 32 + j] = q;
            sum += q;
        }
        xd[r][b] = h2f(f2h(d));
        xs[r][b] = h2f(f2h(__fmul_rn((float)sum, d)));
    }
    __syncthreads();
    const int r = tid / QM_T, c = tid % QM_T;
    const int nc = min(nt + c, p.N - 1);
    const int4* wrow = (const int4*)((const int8_t*)p.w + (size_t)nc * p.K);
    const uint16_t* wdr = p.wd + (size_t)nc * nb;
    const uint16_t* wmr = p.wm + (size_t)nc * nb;
    float acc = 0.0f;
    for (int b = 0; b < nb; b++) {
        const int4 w0 = __ldg(wrow + 2 * b), w1 = __ldg(wrow + 2 * b + 1);
        const int4* xr = (const int4*)&xq[r][b * 32];
        const int4 x0 = xr[0], x1 = xr[1];
        int sumi = __dp4a(w0.x, x0.x, 0);
        sumi = __dp4a(w0.y, x0.y, sumi);
        sumi = __dp4a(w0.z, x0.z, sumi);
        sumi = __dp4a(w0.w, x0.w, sumi);
        sumi = __dp4a(w1.x, x1.x, sumi);
        sumi = __dp4a(w1.y, x1.y, sumi);
        sumi = __dp4a(w1.z, x1.z, sumi);
        sumi = __dp4a(w1.w, x1.w, sumi);
        const float dd = __fmul_rn(h2f(wdr[b]), xd[r][b]);
        const float ms = __fmul_rn(h2f(wmr[b]), xs[r][b]);
        acc = __fadd_rn(acc, fmaf(dd, (float)sumi, ms));
    }
    fx_store<EPI>(p, mt + r, nt + c, acc);
}

// K-quant matrices (Q4_K / Q5_K / Q6_K): ggml's K-quant x Q8_K mul_mat in the order of its portable C
// dot. The CTA quantizes its 16 activation rows to Q8_K in shared memory (quantize_row_q8_K_ref, per 256
// values: max = the value of largest magnitude, first one winning; iscale = -127/max; q = min(127,
// round-half-even(iscale*x)); d = 1/iscale; sums of 16), storing each super-block lane-major like the
// weights (value e at (e % 8) * 32 + e / 8). Thread (r, c) runs output (row r, column c): per
// super-block eight exact lane sums (value e to lane e % 8) of the pre-scaled int16 weights times the
// int8 activations (16 dp2a per lane), sums[l] = fma(d_w*d_x, lane, sums[l]); Q4_K / Q5_K also sumf =
// fma(-dmin_w*d_x, sum_g bsums[g]*min[g/2], sumf); at the end sumf + sums[0] + ... + sums[7]. K is a
// multiple of 256, at most QK_KMAX.
constexpr int QK_T = 16, QK_KMAX = 2048;

template <int EPI>
__global__ void __launch_bounds__(256) k_gemm_qk(const GemmFxParams p) {
    __shared__ __align__(16) int8_t xq[QK_T][QK_KMAX];
    __shared__ float xd[QK_T][QK_KMAX / 256];
    __shared__ int32_t xbs[QK_T][QK_KMAX / 16];
    const int tid = threadIdx.x, nsb = p.K / 256;
    const int mt = blockIdx.y * QK_T, nt = blockIdx.x * QK_T;
    griddep_wait();
    griddep_launch();
    for (int i = tid; i < QK_T * nsb; i += 256) {
        const int r = i / nsb, sb = i - r * nsb;
        const float* src = p.x + (size_t)min(mt + r, p.M - 1) * p.ldx + sb * 256;
        float amax = 0.0f, mx = 0.0f;
        for (int j = 0; j < 256; j++) {
            const float v = src[j];
            if (fabsf(v) > amax) {
                amax = fabsf(v);
                mx = v;
            }
        }
        const float iscale = amax != 0.0f ? __fdiv_rn(-127.0f, mx) : 0.0f;
        int8_t* dst = &xq[r][sb * 256];
        for (int g = 0; g < 16; g++) {
            int s = 0;
            for (int j = 0; j < 16; j++) {
                const int e = g * 16 + j;
                const int v = amax != 0.0f ? min(127, __float2int_rn(__fmul_rn(iscale, src[e]))) : 0;
                dst[(e & 7) * 32 + (e >> 3)] = (int8_t)v;
                s += v;
            }
            xbs[r][sb * 16 + g] = s;
        }
        xd[r][sb] = amax != 0.0f ? __fdiv_rn(1.0f, iscale) : 0.0f;
    }
    __syncthreads();
    const int r = tid / QK_T, c = tid % QK_T;
    const int nc = min(nt + c, p.N - 1);
    const int4* wrow = (const int4*)((const int16_t*)p.w + (size_t)nc * p.K);
    float sums[8], sumf = 0.0f;
#pragma unroll
    for (int l = 0; l < 8; l++) sums[l] = 0.0f;
    for (int sb = 0; sb < nsb; sb++) {
        const int4* xr = (const int4*)&xq[r][sb * 256];
        const float xds = xd[r][sb];
        const float dd = __fmul_rn(h2f(p.wd[(size_t)nc * nsb + sb]), xds);
#pragma unroll
        for (int l = 0; l < 8; l++) {   // lane l: 32 pre-scaled weights (4 x int4) and 32 activations (2 x int4)
            const int4 x0 = xr[l * 2], x1 = xr[l * 2 + 1];
            const int xw[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            int acc = 0;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int4 w = __ldg(wrow + (size_t)sb * 32 + l * 4 + k);
                acc = __dp2a_lo(w.x, xw[2 * k], acc);
                acc = __dp2a_hi(w.y, xw[2 * k], acc);
                acc = __dp2a_lo(w.z, xw[2 * k + 1], acc);
                acc = __dp2a_hi(w.w, xw[2 * k + 1], acc);
            }
            sums[l] = fmaf(dd, (float)acc, sums[l]);
        }
        if (p.wmins) {
            const uint8_t* mn = p.wmins + ((size_t)nc * nsb + sb) * 8;
            int sumi = 0;
#pragma unroll
            for (int g = 0; g < 16; g++) sumi += xbs[r][sb * 16 + g] * (int)mn[g >> 1];
            const float dmin = __fmul_rn(h2f(p.wm[(size_t)nc * nsb + sb]), xds);
            sumf = fmaf(-dmin, (float)sumi, sumf);
        }
    }
#pragma unroll
    for (int l = 0; l < 8; l++) sumf = __fadd_rn(sumf, sums[l]);
    fx_store<EPI>(p, mt + r, nt + c, sumf);
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

void launch_gemm_fx(const GemmFxParams& p, int epi, cudaStream_t s) {
    if (p.M <= 0 || p.N <= 0) return;
    if (p.wtype == FX_QK) {
        if (p.K % 256 || p.K > QK_KMAX) return;
        const dim3 grid((p.N + QK_T - 1) / QK_T, (p.M + QK_T - 1) / QK_T), block(256);
        switch (epi) {
            case FXE_BIAS: launch_pdl(k_gemm_qk<FXE_BIAS>, grid, block, 0, s, p); break;
            case FXE_RESID: launch_pdl(k_gemm_qk<FXE_RESID>, grid, block, 0, s, p); break;
            default: launch_pdl(k_gemm_qk<FXE_RELU>, grid, block, 0, s, p); break;
        }
        return;
    }
    if (p.wtype == FX_QM) {
        if (p.K % 32 || p.K > QM_KMAX) return;
        const dim3 grid((p.N + QM_T - 1) / QM_T, (p.M + QM_T - 1) / QM_T), block(256);
        switch (epi) {
            case FXE_BIAS: launch_pdl(k_gemm_qm<FXE_BIAS>, grid, block, 0, s, p); break;
            case FXE_RESID: launch_pdl(k_gemm_qm<FXE_RESID>, grid, block, 0, s, p); break;
            default: launch_pdl(k_gemm_qm<FXE_RELU>, grid, block, 0, s, p); break;
        }
        return;
    }
    if (p.K % FX_KC) return;
    if (p.wtype == FX_F16) launch_wt<FX_F16>(p, epi, s);
    else if (p.wtype == FX_BF16) launch_wt<FX_BF16>(p, epi, s);
    else launch_wt<FX_F32>(p, epi, s);
}

}  // namespace gsvcu
