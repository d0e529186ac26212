// dit.cu -- the v5 DiT / CFM velocity estimator (reference src/gsv_dit.cpp, class gsv_dit) on B200.
//
// One estimator pass (gsv_dit::velocity, src/gsv_dit.cpp:1325; graph build_step :592-620):
//   x   = proj_mel(x_mel) + condition                      (build_trunk :533-549, static cache :508-516)
//   x  += mask * Mish(conv2(Mish(conv1(mask * x))))        (grouped conv1d k=31, 16 groups, :195-217)
//   22 x DiTBlock: AdaLN-Zero(t) -> QKV (RoPE on head 0) -> attention -> to_out * mask, gated residual
//                  -> AdaLN -> FFN (GELU tanh) -> gated residual                         (:286-433)
//   vel = proj_out(LN(x) * (1 + scale) + shift)            (build_head :563-576)
// and the CFM Euler loop with classifier-free guidance (gsv_dit::sample, :1410-1478). The positive and
// the negative (unconditional) branch share x_mel and t and differ only in the condition rows, so a
// guided step runs both as one batch of 2T rows. Also here: the static cache of prepare (text path with
// 4 ConvNeXtV2 blocks and the context projection, :486-531), synthesize's chunking (:1480-1581), the
// unconditional-velocity reuse of gsv_dit_alg, and cache-dit (DBCache, :1124-1323).
//
// Kernels (sm_100a):
//   k_dit_gemm    every linear layer and both convolutions: a tcgen05.mma kind::f16 GEMM, f16 operands
//                 staged by TMA (128-byte swizzle, no multicast), f32 accumulator in TMEM (128 frames x BN
//                 features per CTA), fused epilogues (bias, GELU / Mish, RoPE of head 0, gated and
//                 masked residual add into the f32 hidden state, condition add). The convolutions are
//                 implicit GEMMs: K runs over the 31 taps x 64 input channels of a group, and the tap's
//                 activation tile is a TMA load at frame offset tap - 15 of a 3D [branch][frame][channel]
//                 map, whose out-of-range frames read as zero (the conv's zero padding, per branch).
//   k_dit_attn_tc 16 heads x 64 dims, non-causal, key padding mask, on tcgen05: S = Q K^T and O += P V^T
//                 in TMEM, the softmax in registers (two threads per query row), P through shared memory;
//                 one pass, O rescaled in TMEM only when a row's maximum grows by more than 2^8. The QKV
//                 epilogue writes v transposed ([branch][head][dim][frame]) for the K-major P V^T operand.
//   k_dit_lnmod   LayerNorm (eps 1e-6, no affine) * (1 + scale) + shift -> f16 GEMM operand.
//   k_dit_gemv    the time MLP and every block's AdaLN projection (one launch for all blocks per step).
//   k_dit_dwconv_ln, k_dit_gelu_colnorm, k_dit_grn: the ConvNeXtV2 pieces around two GEMMs (prepare).
//   k_dit_fd_partial / _final: cache-dit's criterion (relative L1 change of the front residual).
//   small kernels for the mel packing, the masked conv input and the Euler / guidance update.
// Numerics: f16 GEMM operands (what ggml's mul_mat does with F16 weights: the activations are
// converted to F16 first), f32 accumulation, f32 elsewhere; parity with the CPU restatement is within
// a relative L2 tolerance, not bitwise.
#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "gguf_reader.h"
#include "gsvcu.h"
#include "kernels.h"
#include "tc_common.cuh"

namespace gsvcu {
namespace dit {

using namespace tc;

constexpr int DM = 1024;          // dim
constexpr int NHD = 16;           // heads
constexpr int HDD = 64;           // head dim
constexpr int MEL = 100;          // mel channels
constexpr int MELP = 128;         // mel channels padded (GEMM K)
constexpr int FFD = 2048;         // FFN width
constexpr int ADA = 6 * DM;       // AdaLN-Zero modulation per block
constexpr int KCP = 31;           // conv_pos kernel
constexpr int GCP = 16;           // conv_pos groups
constexpr int ICG = 64;           // channels per group
constexpr int KCONV = KCP * ICG;  // conv GEMM K per group (tap-major)
constexpr int TSIN = 256;         // sinusoidal time features
constexpr float LN_EPS = 1e-6f;
constexpr float ATTN_SCALE = 0.125f;   // 1/sqrt(64)

// ------------------------------------------------------------------ tcgen05 GEMM
constexpr int GM = 128;           // frames per tile (UMMA M, TMEM lanes)
constexpr int GK = 64;            // K per stage (one 128-byte swizzle row of f16)
// stages: 3 (about 97 KB of shared memory at BN = 128: two CTAs per SM) when the grid has more tiles than
// SMs, else 6 (one CTA per SM keeps 192 KB of operands in flight)
constexpr int G_THREADS = 192;    // warp 0 TMA, warp 1 TMEM + MMA, warps 2-5 epilogue

enum { DE_F16 = 0, DE_QKV = 1, DE_RESID = 2, DE_F32 = 3 };
enum { ACT_NONE = 0, ACT_GELU_TANH = 1, ACT_MISH = 2 };

struct DitGemmArgs {
    int R;                  // rows (frames of every branch)
    int T;                  // frames per branch (row r is frame r % T of branch r / T)
    int N, K;
    const float* bias;      // [N] or null
    __half* out16;          // DE_F16 / DE_QKV: [R][ld]
    float* out32;           // DE_RESID (in place) / DE_F32: [R][ld]
    int ld;
    const float* add;       // DE_F32: [R][ld] addend or null
    const float* gate;      // DE_RESID: [N] per-feature gate or null (1)
    int x_lens;             // DE_RESID with mask: frames >= x_lens add nothing
    int use_mask;
    const float* rcos;      // DE_QKV: [T][32] RoPE tables of head 0
    const float* rsin;
    __half* vt16;           // DE_QKV: v transposed, [branch][head][64 dims][tp frames], or null
    int tp;
    int* err;
};

// Shared memory: the operand stages (1024-byte aligned), barriers, TMEM address and abort flag, the tile's
// bias and gate (f32), and for PRE epilogues the tile's rows of the residual / addend (f32, rows padded by
// 16 bytes so that 32 lanes reading 32 rows hit distinct banks).
template <int BN, int GS, bool PRE>
struct GemmSmem {
    static constexpr int STAGE_A = GM * GK * 2;
    static constexpr int STAGE_B = BN * GK * 2;
    static constexpr int XSTR = BN * 4 + 16;
    static constexpr size_t OFF_B = (size_t)GS * STAGE_A;
    static constexpr size_t OFF_BAR = OFF_B + (size_t)GS * STAGE_B;
    static constexpr size_t OFF_PAR = OFF_BAR + (2 * GS + 1) * 8 + 8;
    static constexpr size_t OFF_X = OFF_PAR + 2 * BN * 4;
    static constexpr size_t SMEM = OFF_X + (PRE ? (size_t)GM * XSTR : 0) + 1024;   // + slack for the alignment
};

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *(const uint32_t*)&h;
}

static_assert(GemmSmem<128, 6, false>::SMEM <= 232448 && 2 * GemmSmem<128, 3, false>::SMEM <= 233472 &&
                  GemmSmem<128, 4, true>::SMEM <= 232448 && 2 * GemmSmem<64, 3, true>::SMEM <= 233472,
              "shared memory per SM");

template <int ACT>
__device__ __forceinline__ float act_f(float v) {
    if (ACT == ACT_GELU_TANH) {   // torch GELU(approximate="tanh")
        const float u = 0.7978845608028654f * (v + 0.044715f * v * v * v);
        return 0.5f * v * (1.0f + tanhf(u));
    }
    if (ACT == ACT_MISH) {        // x * tanh(softplus(x)), softplus with torch's threshold 20
        const float sp = v > 20.0f ? v : log1pf(expf(v));
        return v * tanhf(sp);
    }
    return v;
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
    const int n = pred ? 16 : 0;   // zero-fill when the row is out of range
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}

// D[frames][features] = A[frames][K] . B[features][K]^T, K-major f16 operands. CONV: A is the 3D map
// [branch][frame][1024] and stage s is tap s of group blockIdx.x (channels 64 g .. 64 g + 63).
template <int EPI, int ACT, int BN, bool CONV, int GS>
__global__ void __launch_bounds__(G_THREADS) k_dit_gemm(const __grid_constant__ CUtensorMap ma,
                                                        const __grid_constant__ CUtensorMap mb, const DitGemmArgs p) {
    constexpr bool PRE = EPI == DE_RESID || EPI == DE_F32;
    using L = GemmSmem<BN, GS, PRE>;
    constexpr uint32_t IDESC = idesc_f16(GM, BN);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = smem_raw + ((1024u - (su32(smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t bar0 = su32(sm + L::OFF_BAR);
    auto full = [&](int s) { return bar0 + 8u * s; };
    auto empty = [&](int s) { return bar0 + 8u * (GS + s); };
    const uint32_t tfull = bar0 + 8u * (2 * GS);
    uint32_t* tmem_slot = (uint32_t*)(sm + L::OFF_BAR + (2 * GS + 1) * 8);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

    const int n0 = blockIdx.x * BN;
    int row0, branch = 0, f0 = 0;
    if (CONV) {
        const int tpb = (p.T + GM - 1) / GM;
        branch = blockIdx.y / tpb;
        f0 = (blockIdx.y % tpb) * GM;
        row0 = branch * p.T + f0;
    } else {
        row0 = blockIdx.y * GM;
    }
    const int nstage = CONV ? KCP : p.K / GK;

    if (tid == 0) {
        for (int s = 0; s < GS; s++) { bar_init(full(s), 1); bar_init(empty(s), 1); }
        bar_init(tfull, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&ma) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&mb) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                     "r"(BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    griddep_wait();
    griddep_launch();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {   // TMA producer
            int ks = 0;
            for (; ks < nstage; ks++) {
                const int s = ks % GS;
                if (!bar_wait_short(empty(s), ((uint32_t)(ks / GS) & 1u) ^ 1u, abort_flag)) break;
                bar_expect_tx(full(s), L::STAGE_A + L::STAGE_B);
                const uint32_t da = su32(sm + (size_t)s * L::STAGE_A), db = su32(sm + L::OFF_B + (size_t)s * L::STAGE_B);
                if (CONV) {
                    tma_load_3d(da, &ma, n0, f0 + ks - KCP / 2, branch, full(s));
                    tma_load_2d(db, &mb, ks * GK, n0, full(s));
                } else {
                    tma_load_2d(da, &ma, ks * GK, row0, full(s));
                    tma_load_2d(db, &mb, ks * GK, n0, full(s));
                }
            }
            if (ks < nstage) {
                if (p.err) atomicExch(p.err, 1);
                *abort_flag = 1;
            }
            // the copies issued have landed before the CTA may exit (bounded)
            for (int k = ks - 1; k >= 0 && k >= ks - GS; k--)
                for (uint32_t it = 0; it < TC_POLL_LIMIT; it++)
                    if (bar_try(full(k % GS), (uint32_t)(k / GS) & 1u)) break;
        }
    } else if (warp == 1) {
        if (lane == 0) {   // MMA issuer
            int ks = 0;
            for (; ks < nstage; ks++) {
                const int s = ks % GS;
                if (!bar_wait_short(full(s), (uint32_t)(ks / GS) & 1u, abort_flag)) break;
                tc_fence_after();
                const uint32_t a = su32(sm + (size_t)s * L::STAGE_A), b = su32(sm + L::OFF_B + (size_t)s * L::STAGE_B);
#pragma unroll
                for (int kk = 0; kk < GK / 16; kk++)
                    umma_f16(tmem, umma_desc(a + 32u * kk), umma_desc(b + 32u * kk), IDESC, (uint32_t)(ks | kk));
                umma_commit(empty(s));
            }
            if (ks < nstage) {
                if (p.err) atomicExch(p.err, 1);
                *abort_flag = 1;
            }
            umma_commit(tfull);   // every MMA issued above has completed when tfull completes
            for (uint32_t it = 0; it < TC_POLL_LIMIT; it++)
                if (bar_try(tfull, 0)) break;
        }
    } else {
        // epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 = frames of this tile. While the MMAs run,
        // the tile's bias and gate go to shared memory and the tile's rows of the residual (or addend) are
        // copied in by coalesced cp.async, so no dependent global load is left for after the accumulator.
        const int q = warp & 3;
        const int fr = 32 * q + lane;   // frame (row) within the tile
        const int row = row0 + fr;
        const bool valid = CONV ? f0 + fr < p.T : row < p.R;
        const int et = tid - 64;        // 0..127 over the epilogue warps
        float* sbias = (float*)(sm + L::OFF_PAR);
        float* sgate = sbias + BN;
        for (int i = et; i < BN; i += 128) {
            sbias[i] = p.bias ? p.bias[n0 + i] : 0.0f;
            sgate[i] = (EPI == DE_RESID && p.gate) ? p.gate[n0 + i] : 1.0f;
        }
        const float* xsrc = EPI == DE_RESID ? p.out32 : p.add;
        uint8_t* sx = sm + L::OFF_X;
        if (PRE && xsrc) {
            constexpr int CPR = BN / 4;   // 16-byte chunks per row
#pragma unroll 4
            for (int i = et; i < GM * CPR; i += 128) {
                const int r = i / CPR, ch = i - r * CPR;
                const bool in = CONV ? f0 + r < p.T : row0 + r < p.R;
                const float* g = xsrc + (size_t)(in ? row0 + r : 0) * p.ld + n0 + 4 * ch;
                cp_async16(su32(sx + (size_t)r * L::XSTR + 16 * ch), g, in);
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");   // the four epilogue warps: staging complete
        const bool ok = bar_wait_warp(tfull, 0, abort_flag) && !*abort_flag;
        tc_fence_after();
        if (ok) {
            const int t = row % p.T;
            const float mask = (EPI == DE_RESID && p.use_mask && t >= p.x_lens) ? 0.0f : 1.0f;
            const uint32_t tb = tmem + ((uint32_t)(32 * q) << 16);
            const float* xrow = (const float*)(sx + (size_t)fr * L::XSTR);
#pragma unroll 1
            for (int c = 0; c < BN; c += 16) {
                float v[16];
                __syncwarp();   // converged for the .sync.aligned TMEM load
                tmem_ld16(tb + (uint32_t)c, v);
                tmem_wait_ld();
                tmem_bind(v);
                const int f = n0 + c;
#pragma unroll
                for (int i = 0; i < 16; i++) v[i] += sbias[c + i];
                if (valid) {
                    if (EPI == DE_QKV && (n0 == 0 || n0 == DM) && c < HDD) {
                        // RoPE on head 0 of q and k: pairs (2i, 2i + 1) share angle t * inv_freq[i]
#pragma unroll
                        for (int i = 0; i < 16; i += 2) {
                            const int pi = (c + i) >> 1;
                            const float cs = __ldg(p.rcos + (size_t)t * 32 + pi), sn = __ldg(p.rsin + (size_t)t * 32 + pi);
                            const float x0 = v[i], x1 = v[i + 1];
                            v[i] = x0 * cs - x1 * sn;
                            v[i + 1] = x0 * sn + x1 * cs;
                        }
                    }
                    if (EPI == DE_QKV && p.vt16 && n0 >= 2 * DM) {
                        // v also as [branch][head][dim][frame]: 32 lanes = 32 consecutive frames of one dim
                        const int bq = row / p.T, hd0 = f - 2 * DM;
                        __half* vt = p.vt16 + ((size_t)bq * DM + hd0) * p.tp + t;
#pragma unroll
                        for (int i = 0; i < 16; i++) vt[(size_t)i * p.tp] = __float2half_rn(v[i]);
                    }
                    if (EPI == DE_F16 || EPI == DE_QKV) {
                        // (v columns go only to vt16 when it is given)
                        if (EPI == DE_F16 || !(p.vt16 && n0 >= 2 * DM)) {
                            uint32_t w[8];
#pragma unroll
                            for (int i = 0; i < 8; i++) w[i] = pack_h2(act_f<ACT>(v[2 * i]), act_f<ACT>(v[2 * i + 1]));
                            uint4* dst = (uint4*)(p.out16 + (size_t)row * p.ld + f);
                            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
                            dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
                        }
                    } else if (EPI == DE_RESID) {
                        float4* dst = (float4*)(p.out32 + (size_t)row * p.ld + f);
#pragma unroll
                        for (int i = 0; i < 16; i += 4) {
                            float4 x = *(const float4*)(xrow + c + i);
                            x.x += act_f<ACT>(v[i]) * mask * sgate[c + i];
                            x.y += act_f<ACT>(v[i + 1]) * mask * sgate[c + i + 1];
                            x.z += act_f<ACT>(v[i + 2]) * mask * sgate[c + i + 2];
                            x.w += act_f<ACT>(v[i + 3]) * mask * sgate[c + i + 3];
                            dst[i / 4] = x;
                        }
                    } else {   // DE_F32: + the addend row (none: + 0)
                        float4* dst = (float4*)(p.out32 + (size_t)row * p.ld + f);
#pragma unroll
                        for (int i = 0; i < 16; i += 4) {
                            const float4 a4 = xsrc ? *(const float4*)(xrow + c + i) : make_float4(0.f, 0.f, 0.f, 0.f);
                            dst[i / 4] = make_float4(v[i] + a4.x, v[i + 1] + a4.y, v[i + 2] + a4.z, v[i + 3] + a4.w);
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN) : "memory");
    }
}

// ------------------------------------------------------------------ attention on tcgen05
// One CTA per (128 queries, head, branch), one pass over the key tiles of 64 (keys < x_lens): S = Q K^T into
// TMEM, P = exp2(S * scale * log2 e - m) as f16 into shared memory (the 128-byte-swizzled K-major layout the
// MMA reads), row sums, O += P V^T in TMEM. The reference value m of a row is raised only when a tile's
// maximum exceeds it by more than FA_TAU (so P <= 2^FA_TAU, well inside f16): then the row's O in TMEM and
// its running sum are scaled by exp2(m_old - m_new), after the previous P V^T has completed. Rows raise
// their m on the first tile and rarely after it.
// Warps: 0 TMA (Q once, then K + V^T tiles into a 3-stage ring), 1 TMEM + MMA, 2-9 softmax: two threads per
// query row (TMEM lane), each on 32 of a tile's 64 keys, exchanging their tile maxima through shared memory.
// S and P are double-buffered, so the MMAs of tile j + 1 overlap the softmax of tile j.
constexpr int FQ = 128, FK = 64, FKS = 3;
struct AttnMaps {
    CUtensorMap q;    // qkv16 [R][3072], box 64 x 128
    CUtensorMap k;    // qkv16 [R][3072], box 64 x 64
    CUtensorMap vt;   // vt16 [B * 16 * 64][T (pitch tp)], box 64 x 64
};
struct FaSmem {
    static constexpr size_t OFF_Q = 0;                          // 16 KB
    static constexpr size_t OFF_K = OFF_Q + FQ * HDD * 2;       // FKS x 8 KB
    static constexpr size_t OFF_V = OFF_K + FKS * FK * HDD * 2; // FKS x 8 KB
    static constexpr size_t OFF_P = OFF_V + FKS * HDD * FK * 2; // 2 x 16 KB
    static constexpr size_t OFF_X = OFF_P + 2 * FQ * FK * 2;   // [2 tiles][2 halves][128 rows] f32 exchanges
    static constexpr size_t OFF_BAR = OFF_X + 4 * FQ * 4;
    // qfull, kvfull[FKS], kvempty[FKS], sfull[2], sfree[2], pfull[2], pfree[2], ofull
    static constexpr int NBAR = 1 + 2 * FKS + 8 + 1;
    static constexpr size_t SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
};
constexpr int FA_THREADS = 320;   // warp 0 TMA, warp 1 MMA, warps 2-9 softmax (two per TMEM lane quarter)
constexpr uint32_t FA_TMEM_COLS = 256;   // S0, S1, O (64 columns each)
constexpr float FA_TAU = 8.0f;             // log2 headroom of P above the row's reference value

__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__global__ void __launch_bounds__(FA_THREADS) k_dit_attn_tc(const __grid_constant__ AttnMaps m, __half* __restrict__ out,
                                                           int T, int x_lens, int* err) {
    using L = FaSmem;
    constexpr uint32_t IDS = idesc_f16(FQ, FK);    // S: 128 x 64 keys
    constexpr uint32_t IDO = idesc_f16(FQ, HDD);   // O: 128 x 64 dims
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = smem_raw + ((1024u - (su32(smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int q0 = blockIdx.x * FQ, h = blockIdx.y, b = blockIdx.z;
    const uint32_t bar0 = su32(sm + L::OFF_BAR);
    const uint32_t qfull = bar0;
    auto kvfull = [&](int s) { return bar0 + 8u * (1 + s); };
    auto kvempty = [&](int s) { return bar0 + 8u * (1 + FKS + s); };
    const uint32_t bx = bar0 + 8u * (1 + 2 * FKS);
    auto sfull = [&](int i) { return bx + 8u * i; };
    auto sfree = [&](int i) { return bx + 16u + 8u * i; };
    auto pfull = [&](int i) { return bx + 32u + 8u * i; };
    auto pfree = [&](int i) { return bx + 48u + 8u * i; };
    const uint32_t ofull = bx + 64u;
    uint32_t* tmem_slot = (uint32_t*)(sm + L::OFF_BAR + L::NBAR * 8);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
    const int nt = (x_lens + FK - 1) / FK;

    if (tid == 0) {
        bar_init(qfull, 1);
        for (int s = 0; s < FKS; s++) { bar_init(kvfull(s), 1); bar_init(kvempty(s), 1); }
        for (int i = 0; i < 2; i++) {
            bar_init(sfull(i), 1);
            bar_init(sfree(i), 256);
            bar_init(pfull(i), 256);
            bar_init(pfree(i), 1);
        }
        bar_init(ofull, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                     "r"(FA_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    griddep_wait();
    griddep_launch();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;   // S0 at columns 0..63, S1 at 64..127, O at 128..191

    if (warp == 0) {
        if (lane == 0) {   // TMA producer
            bar_expect_tx(qfull, FQ * HDD * 2);
            tma_load_2d(su32(sm + L::OFF_Q), &m.q, h * HDD, b * T + q0, qfull);
            int g = 0;
            bool ok = true;
            for (int j = 0; j < nt; j++, g++) {
                const int s = g % FKS;
                if (!bar_wait_short(kvempty(s), ((uint32_t)(g / FKS) & 1u) ^ 1u, abort_flag)) { ok = false; break; }
                bar_expect_tx(kvfull(s), 2u * FK * HDD * 2);
                tma_load_2d(su32(sm + L::OFF_K + (size_t)s * FK * HDD * 2), &m.k, DM + h * HDD, b * T + j * FK, kvfull(s));
                tma_load_2d(su32(sm + L::OFF_V + (size_t)s * HDD * FK * 2), &m.vt, j * FK, (b * NHD + h) * HDD, kvfull(s));
            }
            if (!ok) {
                if (err) atomicExch(err, 1);
                *abort_flag = 1;
            }
            for (int k = g - 1; k >= 0 && k >= g - FKS; k--)
                for (uint32_t it = 0; it < TC_POLL_LIMIT; it++)
                    if (bar_try(kvfull(k % FKS), (uint32_t)(k / FKS) & 1u)) break;
            for (uint32_t it = 0; it < TC_POLL_LIMIT; it++)
                if (bar_try(qfull, 0)) break;
        }
    } else if (warp == 1) {
        if (lane == 0) {   // MMA issuer
            bool ok = bar_wait_short(qfull, 0, abort_flag);
            const uint32_t qa = su32(sm + L::OFF_Q);
            int g = 0, u = 0, v = 0;   // ring stages, S tiles, P tiles consumed
            int prev_s = -1;            // ring stage of the tile whose P V^T is still to be issued
            // P V^T of the previous tile once its P is written: O += P V^T
            auto pv = [&](int j) -> bool {
                const int pb = v & 1;
                if (!bar_wait_short(pfull(pb), ((uint32_t)v >> 1) & 1u, abort_flag)) return false;
                tc_fence_after();
                const uint32_t pa = su32(sm + L::OFF_P + (size_t)pb * FQ * FK * 2);
                const uint32_t va = su32(sm + L::OFF_V + (size_t)prev_s * HDD * FK * 2);
#pragma unroll
                for (int kk = 0; kk < FK / 16; kk++)
                    umma_f16(tmem + 2 * FK, umma_desc(pa + 32u * kk), umma_desc(va + 32u * kk), IDO, (uint32_t)(j | kk));
                umma_commit(kvempty(prev_s));
                umma_commit(pfree(pb));
                v++;
                return true;
            };
            for (int j = 0; j < nt && ok; j++, g++, u++) {
                const int s = g % FKS, sb = u & 1;
                if (!bar_wait_short(kvfull(s), (uint32_t)(g / FKS) & 1u, abort_flag) ||
                    !bar_wait_short(sfree(sb), (((uint32_t)u >> 1) & 1u) ^ 1u, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint32_t ka = su32(sm + L::OFF_K + (size_t)s * FK * HDD * 2);
#pragma unroll
                for (int kk = 0; kk < HDD / 16; kk++)
                    umma_f16(tmem + (uint32_t)(sb * FK), umma_desc(qa + 32u * kk), umma_desc(ka + 32u * kk), IDS,
                             (uint32_t)kk);
                umma_commit(sfull(sb));
                if (j > 0 && !pv(j - 1)) { ok = false; break; }
                prev_s = s;
            }
            if (ok && !pv(nt - 1)) ok = false;
            if (!ok) {
                if (err) atomicExch(err, 1);
                *abort_flag = 1;
            }
            umma_commit(ofull);   // every MMA issued above has completed when ofull completes
            for (uint32_t it = 0; it < TC_POLL_LIMIT; it++)
                if (bar_try(ofull, 0)) break;
        }
    } else {
        // softmax: thread = (query row fr = TMEM lane, half hf): keys 32 hf .. 32 hf + 31 of each tile
        const int q = warp & 3, fr = 32 * q + lane, hf = (warp - 2) >> 2;
        const uint32_t tl = tmem + ((uint32_t)(32 * q) << 16);
        float* xch = (float*)(sm + L::OFF_X);   // [tile parity][half][row]
        const float c = ATTN_SCALE * 1.4426950408889634f;
        float mref = -INFINITY, l = 0.0f;       // the row's reference value (scaled log2 units) and sum
        int v = 0;
        bool ok = true;
        // (every softmax thread runs the same named-barrier sequence, also after a failed wait)
        for (int j = 0; j < nt; j++) {
            const int sb = j & 1;
            float sv[2][16];
            float lm = -INFINITY;
            const int kv = x_lens - j * FK - 32 * hf;   // valid keys of this thread's 32 (may be <= 0)
            if (ok) {
                if (!bar_wait_short_warp(sfull(sb), ((uint32_t)j >> 1) & 1u, abort_flag)) ok = false;
            }
            if (ok) {
                tc_fence_after();
#pragma unroll
                for (int k = 0; k < 2; k++) tmem_ld16(tl + (uint32_t)(sb * FK + 32 * hf + 16 * k), sv[k]);
                tmem_wait_ld();
#pragma unroll
                for (int k = 0; k < 2; k++) tmem_bind(sv[k]);
                tc_fence_before();
                bar_arrive(sfree(sb));
                // max of the raw scores, scaled once (c > 0 and rounding is monotone: the same value)
                float mx = -INFINITY;
                if (kv >= 32) {
#pragma unroll
                    for (int i = 0; i < 32; i++) mx = fmaxf(mx, sv[i >> 4][i & 15]);
                } else {
#pragma unroll
                    for (int i = 0; i < 32; i++)
                        if (i < kv) mx = fmaxf(mx, sv[i >> 4][i & 15]);
                }
                lm = mx * c;
            }
            float* xt = xch + (size_t)(j & 1) * 2 * FQ;
            xt[hf * FQ + fr] = lm;
            asm volatile("bar.sync 1, 256;" ::: "memory");
            const float mt = fmaxf(xt[fr], xt[FQ + fr]);   // the tile's row maximum (scaled)
            if (!ok) continue;
            if (mt > mref + FA_TAU) {   // raise the reference value; rescale what O and l hold so far
                if (j > 0) {
                    const float alpha = ex2f(mref - mt);
                    // O may be rescaled only after the previous tile's P V^T has completed
                    if (!bar_wait_short_warp(pfree((v - 1) & 1), ((uint32_t)(v - 1) >> 1) & 1u, abort_flag)) {
                        ok = false;
                        continue;
                    }
                    tc_fence_after();
                    float o2[2][16];
#pragma unroll
                    for (int k = 0; k < 2; k++) tmem_ld16(tl + (uint32_t)(2 * FK + 32 * hf + 16 * k), o2[k]);
                    tmem_wait_ld();
#pragma unroll
                    for (int k = 0; k < 2; k++) {
                        tmem_bind(o2[k]);
#pragma unroll
                        for (int i = 0; i < 16; i++) o2[k][i] *= alpha;
                        tmem_st16(tl + (uint32_t)(2 * FK + 32 * hf + 16 * k), o2[k]);
                    }
                    tmem_wait_st();
                    l *= alpha;
                }
                mref = mt;
            }
            uint32_t pw[16];
            if (kv >= 32) {   // a full tile: no per-key predicate
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    const float p0 = ex2f(__fmaf_rn(sv[i >> 4][i & 15], c, -mref));
                    const float p1 = ex2f(__fmaf_rn(sv[i >> 4][(i + 1) & 15], c, -mref));
                    l += p0 + p1;
                    pw[i / 2] = pack_h2(p0, p1);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    const float p0 = i < kv ? ex2f(__fmaf_rn(sv[i >> 4][i & 15], c, -mref)) : 0.0f;
                    const float p1 = i + 1 < kv ? ex2f(__fmaf_rn(sv[i >> 4][(i + 1) & 15], c, -mref)) : 0.0f;
                    l += p0 + p1;
                    pw[i / 2] = pack_h2(p0, p1);
                }
            }
            const int pb = v & 1;
            if (!bar_wait_short_warp(pfree(pb), (((uint32_t)v >> 1) & 1u) ^ 1u, abort_flag)) {
                ok = false;
                continue;
            }
            uint8_t* prow = sm + L::OFF_P + (size_t)pb * FQ * FK * 2 + (size_t)fr * 128;
#pragma unroll
            for (int k = 0; k < 4; k++) {   // 128-byte swizzle: chunk ch of row r at ch ^ (r % 8)
                const int ch = 4 * hf + k;
                *(uint4*)(prow + 16 * (ch ^ (fr & 7))) = make_uint4(pw[4 * k], pw[4 * k + 1], pw[4 * k + 2], pw[4 * k + 3]);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc_fence_before();   // the O rescale's TMEM stores before the MMA that accumulates onto them
            bar_arrive(pfull(pb));
            v++;
        }
        // row sums of both halves
        {
            float* xt = xch + (size_t)(nt & 1) * 2 * FQ;
            xt[hf * FQ + fr] = l;
            asm volatile("bar.sync 1, 256;" ::: "memory");
            l = xt[fr] + xt[FQ + fr];
        }
        ok = bar_wait_short_warp(ofull, 0, abort_flag) && ok && !*abort_flag;
        tc_fence_after();
        if (ok) {
            float o2[2][16];
#pragma unroll
            for (int k = 0; k < 2; k++) tmem_ld16(tl + (uint32_t)(2 * FK + 32 * hf + 16 * k), o2[k]);
            tmem_wait_ld();
#pragma unroll
            for (int k = 0; k < 2; k++) tmem_bind(o2[k]);
            if (q0 + fr < T) {
                const float il = 1.0f / l;
                uint4* dst = (uint4*)(out + ((size_t)b * T + q0 + fr) * DM + h * HDD + 32 * hf);
#pragma unroll
                for (int ch = 0; ch < 4; ch++) {
                    const float* o = o2[ch >> 1] + 8 * (ch & 1);
                    dst[ch] = make_uint4(pack_h2(o[0] * il, o[1] * il), pack_h2(o[2] * il, o[3] * il),
                                         pack_h2(o[4] * il, o[5] * il), pack_h2(o[6] * il, o[7] * il));
                }
            }
        } else if (err && lane == 0) {
            atomicExch(err, 1);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(FA_TMEM_COLS) : "memory");
    }
}

// ------------------------------------------------------------------ row kernels
// LayerNorm (no affine, eps 1e-6) * (1 + scale) + shift of each 1024-wide row -> f16. Warp per row.
__global__ void __launch_bounds__(256) k_dit_lnmod(const float* __restrict__ x, int R, const float* __restrict__ shift,
                                                   const float* __restrict__ scale, __half* __restrict__ out) {
    griddep_wait();
    griddep_launch();
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= R) return;
    const float4* xr = (const float4*)(x + (size_t)row * DM);
    float4 v[8];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        v[i] = xr[lane + 32 * i];
        s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    const float mean = s * (1.0f / DM);
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
        q += (a * a + b * b) + (c * c + d * d);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) q += __shfl_xor_sync(0xffffffffu, q, off);
    const float rstd = 1.0f / sqrtf(q * (1.0f / DM) + LN_EPS);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int c = 4 * (lane + 32 * i);
        const float4 sc = __ldg((const float4*)(scale + c)), sh = __ldg((const float4*)(shift + c));
        const float y0 = (v[i].x - mean) * rstd * (1.0f + sc.x) + sh.x;
        const float y1 = (v[i].y - mean) * rstd * (1.0f + sc.y) + sh.y;
        const float y2 = (v[i].z - mean) * rstd * (1.0f + sc.z) + sh.z;
        const float y3 = (v[i].w - mean) * rstd * (1.0f + sc.w) + sh.w;
        *(uint2*)(out + (size_t)row * DM + c) = make_uint2(pack_h2(y0, y1), pack_h2(y2, y3));
    }
}

// f16(x * mask) of every row (the conv input).
__global__ void __launch_bounds__(256) k_dit_mask16(const float* __restrict__ x, int R, int T, int x_lens,
                                                    __half* __restrict__ out) {
    griddep_wait();
    griddep_launch();
    const size_t n4 = (size_t)R * DM / 4;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const int row = (int)(i / (DM / 4));
        const float m = (row % T) < x_lens ? 1.0f : 0.0f;
        const float4 v = ((const float4*)x)[i];
        ((uint2*)out)[i] = make_uint2(pack_h2(v.x * m, v.y * m), pack_h2(v.z * m, v.w * m));
    }
}

// x_mel [100][T] f32 (torch layout) -> rows b T + t of [R][128] f16, channels 100..127 zero.
__global__ void __launch_bounds__(256) k_dit_pack_mel(const float* __restrict__ xm, int T, int B, __half* __restrict__ out) {
    griddep_wait();
    griddep_launch();
    const int n = B * T * MELP;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int c = i / (B * T), r = i - c * (B * T), t = r % T;
        out[(size_t)r * MELP + c] = __float2half_rn(c < MEL ? xm[(size_t)c * T + t] : 0.0f);
    }
}

// Euler step with guidance (gsv_dit::sample, src/gsv_dit.cpp:1449-1469): v = vel + (vel - ng) * cfg with the
// unconditional velocity ng = neg (rows [T][128]) or, given neg2, the extrapolation 2 neg - neg2 (uncond_reuse
// 2); x += dt * v; then the prompt frames are zeroed. update = 0: only the zeroing (before the first step).
__global__ void __launch_bounds__(256) k_dit_euler(const float* __restrict__ vel, int T, int update,
                                                   const float* __restrict__ neg, const float* __restrict__ neg2,
                                                   float cfg, float dt, int P, float* __restrict__ xm) {
    griddep_wait();
    griddep_launch();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < MEL * T; i += gridDim.x * blockDim.x) {
        const int c = i / T, t = i - c * T;
        float x = xm[i];
        if (update) {
            float v = vel[(size_t)t * MELP + c];
            if (neg) {
                float ng = neg[(size_t)t * MELP + c];
                if (neg2) ng = 2.0f * ng - neg2[(size_t)t * MELP + c];
                v = v + (v - ng) * cfg;
            }
            x = x + dt * v;
        }
        xm[i] = t < P ? 0.0f : x;
    }
}

// [T][128] f32 rows -> vel [100][T] (torch layout).
__global__ void __launch_bounds__(256) k_dit_vel_out(const float* __restrict__ vel, int T, float* __restrict__ out) {
    griddep_wait();
    griddep_launch();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < MEL * T; i += gridDim.x * blockDim.x) {
        const int c = i / T, t = i - c * T;
        out[i] = vel[(size_t)t * MELP + c];
    }
}

// y[n] = W[n] . f16(f(in)) + b[n] (f = SiLU when SILU_IN), then SiLU when SILU_OUT. W f16 [N][K], K <= 1024
// and a multiple of 8. Warp per output, 16-byte weight loads.
template <bool SILU_IN, bool SILU_OUT>
__global__ void __launch_bounds__(256) k_dit_gemv(const __half* __restrict__ W, const float* __restrict__ bias,
                                                  const float* __restrict__ in, int N, int K, float* __restrict__ y) {
    __shared__ float sx[DM];
    griddep_wait();
    griddep_launch();
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        const float v = in[k];
        // ggml's mul_mat with an F16 weight converts the activations to F16 first
        sx[k] = __half2float(__float2half_rn(SILU_IN ? v / (1.0f + expf(-v)) : v));
    }
    __syncthreads();
    const int n = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (n >= N) return;
    const uint4* wr = (const uint4*)(W + (size_t)n * K);
    float acc = 0.0f;
    for (int c = lane; c < K / 8; c += 32) {
        const uint4 w = __ldg(wr + c);
        const __half2* h = (const __half2*)&w;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const float2 f = __half22float2(h[e]);
            acc += f.x * sx[8 * c + 2 * e] + f.y * sx[8 * c + 2 * e + 1];
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) {
        const float v = acc + (bias ? bias[n] : 0.0f);
        y[n] = SILU_OUT ? v / (1.0f + expf(-v)) : v;
    }
}

// ------------------------------------------------------------------ static cache (prepare)
constexpr int TXD = 512;          // text dim
constexpr int TXI = 1024;         // ConvNeXtV2 intermediate
constexpr int CTXK = 640;         // [prompt_x (100) | text (512)] padded to a multiple of 64
constexpr int MAXPOS = 4096;      // freqs_cis rows

// tx[t][c] = mu[c][t] + freqs_cis[t][c] (mu in torch layout [512][T]).
__global__ void __launch_bounds__(256) k_dit_text_in(const float* __restrict__ mu, const float* __restrict__ cis, int T,
                                                     float* __restrict__ tx) {
    griddep_wait();
    griddep_launch();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < TXD * T; i += gridDim.x * blockDim.x) {
        const int t = i / TXD, c = i - t * TXD;
        tx[i] = mu[(size_t)c * T + t] + cis[(size_t)t * TXD + c];
    }
}

// Depthwise conv (k = 7, zero padding 3, taps summed in order) + bias, then LayerNorm (eps 1e-6) with
// weight and bias -> f16 [T][512]. Warp per frame, lane = channels lane + 32 j.
__global__ void __launch_bounds__(256) k_dit_dwconv_ln(const float* __restrict__ x, int T, const float* __restrict__ w7,
                                                       const float* __restrict__ b, const float* __restrict__ nw,
                                                       const float* __restrict__ nb, __half* __restrict__ out) {
    griddep_wait();
    griddep_launch();
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= T) return;
    float y[16];
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < 16; j++) {
        const int c = lane + 32 * j;
        float acc = 0.0f;
#pragma unroll
        for (int kw = 0; kw < 7; kw++) {
            const int tt = t + kw - 3;
            const float xv = (tt >= 0 && tt < T) ? x[(size_t)tt * TXD + c] : 0.0f;
            acc = kw ? acc + xv * w7[kw * TXD + c] : xv * w7[c];
        }
        y[j] = acc + b[c];
        s += y[j];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    const float mean = s * (1.0f / TXD);
    float q = 0.0f;
#pragma unroll
    for (int j = 0; j < 16; j++) q += (y[j] - mean) * (y[j] - mean);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) q += __shfl_xor_sync(0xffffffffu, q, off);
    const float rstd = 1.0f / sqrtf(q * (1.0f / TXD) + LN_EPS);
#pragma unroll
    for (int j = 0; j < 16; j++) {
        const int c = lane + 32 * j;
        out[(size_t)t * TXD + c] = __float2half_rn((y[j] - mean) * rstd * nw[c] + nb[c]);
    }
}

// GELU (erf) in place on h [T][1024] and each channel's L2 norm over the frames, gx[c] = sqrt(sum_t h^2).
// CTA = 32 channels x 8 frame groups; partial sums added in a fixed order.
__global__ void __launch_bounds__(256) k_dit_gelu_colnorm(float* __restrict__ h, int T, float* __restrict__ gx) {
    __shared__ float part[8][32];
    griddep_wait();
    griddep_launch();
    const int c = blockIdx.x * 32 + (threadIdx.x & 31), g = threadIdx.x >> 5;
    float s = 0.0f;
    for (int t = g; t < T; t += 8) {
        float* p = h + (size_t)t * TXI + c;
        const float v = *p;
        const float y = 0.5f * v * (1.0f + erff(v * 0.7071067811865476f));
        *p = y;
        s += y * y;
    }
    part[g][threadIdx.x & 31] = s;
    __syncthreads();
    if (g == 0) {
        float a = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; i++) a += part[i][threadIdx.x];
        gx[c] = sqrtf(a);
    }
}

// GRN: out = f16(gamma * (h * Nx) + beta + h), Nx = gx / (mean(gx) + 1e-6). Every CTA sums the 1024 norms
// in the same order.
__global__ void __launch_bounds__(256) k_dit_grn(const float* __restrict__ h, int T, const float* __restrict__ gx,
                                                 const float* __restrict__ gamma, const float* __restrict__ beta,
                                                 __half* __restrict__ out) {
    __shared__ float snx[TXI];
    __shared__ float wsum[8];
    griddep_wait();
    griddep_launch();
    float a = 0.0f;
    for (int c = threadIdx.x; c < TXI; c += 256) a += gx[c];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
    if ((threadIdx.x & 31) == 0) wsum[threadIdx.x >> 5] = a;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) tot += wsum[i];
    const float inv = 1.0f / (tot * (1.0f / TXI) + 1e-6f);
    for (int c = threadIdx.x; c < TXI; c += 256) snx[c] = gx[c] * inv;
    __syncthreads();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < TXI * T; i += gridDim.x * blockDim.x) {
        const int c = i & (TXI - 1);
        const float v = h[i];
        out[i] = __float2half_rn(gamma[c] * (v * snx[c]) + beta[c] + v);
    }
}

// Rows [0, T): [prompt_x^T | text]; rows [T, 2T): [0 | text]; f16 [2T][640], columns 612.. zero.
__global__ void __launch_bounds__(256) k_dit_pack_ctx(const float* __restrict__ px, const float* __restrict__ tx, int T,
                                                      __half* __restrict__ out) {
    griddep_wait();
    griddep_launch();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < 2 * T * CTXK; i += gridDim.x * blockDim.x) {
        const int r = i / CTXK, k = i - r * CTXK, t = r % T;
        float v = 0.0f;
        if (k < MEL) v = r < T ? px[(size_t)k * T + t] : 0.0f;
        else if (k < MEL + TXD) v = tx[(size_t)t * TXD + (k - MEL)];
        out[i] = __float2half_rn(v);
    }
}

// ------------------------------------------------------------------ cache-dit (DBCache)
constexpr int FD_BLOCKS = 296;   // partial sums of the residual-difference criterion

// The front residual of branch b as the reference's criterion reads it (src/gsv_dit.cpp:1157-1163):
// r = x_front - x_trunk, then with ds > 1 the view ne {1024, T / ds} with a row stride of ds floats over r's
// flat [T][1024] storage, i.e. r_cur[t'][i] = r_flat[t' ds + i]. Writes r_cur and per-block partial sums of
// |r_cur - r_prev| and |r_prev| (double).
__global__ void __launch_bounds__(256) k_dit_fd_partial(const float* __restrict__ xf, const float* __restrict__ xt,
                                                        const float* __restrict__ r_prev, int n, int ds,
                                                        float* __restrict__ r_cur, double* __restrict__ part) {
    __shared__ double sa[8], sb[8];
    griddep_wait();
    griddep_launch();
    double a = 0.0, bsum = 0.0;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const size_t src = ds > 1 ? (size_t)(i / DM) * ds + (i % DM) : (size_t)i;
        const float r = xf[src] - xt[src];
        r_cur[i] = r;
        const float rp = r_prev[i];
        a += fabsf(r - rp);
        bsum += fabsf(rp);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        a += __shfl_xor_sync(0xffffffffu, a, off);
        bsum += __shfl_xor_sync(0xffffffffu, bsum, off);
    }
    if ((threadIdx.x & 31) == 0) { sa[threadIdx.x >> 5] = a; sb[threadIdx.x >> 5] = bsum; }
    __syncthreads();
    if (threadIdx.x == 0) {
        double x = 0.0, y = 0.0;
        for (int w = 0; w < 8; w++) { x += sa[w]; y += sb[w]; }
        part[2 * blockIdx.x] = x;
        part[2 * blockIdx.x + 1] = y;
    }
}

// fd = sum |r_cur - r_prev| / (sum |r_prev| + 1e-6), the partial sums added in block order.
__global__ void __launch_bounds__(32) k_dit_fd_final(const double* __restrict__ part, int nblk, float* __restrict__ fd) {
    griddep_wait();
    griddep_launch();
    if (threadIdx.x == 0) {
        double x = 0.0, y = 0.0;
        for (int i = 0; i < nblk; i++) { x += part[2 * i]; y += part[2 * i + 1]; }
        *fd = (float)x / ((float)y + 1e-6f);
    }
}

// dst = a + s * b over n floats (s = +1 or -1).
__global__ void __launch_bounds__(256) k_dit_axpy(const float* __restrict__ a, const float* __restrict__ b, float sgn,
                                                  size_t n, float* __restrict__ dst) {
    griddep_wait();
    griddep_launch();
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = a[i] + sgn * b[i];
}

// ------------------------------------------------------------------ host side
bool map_2d(CUtensorMap* m, const __half* base, uint64_t rows, uint64_t K, uint32_t box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {K, rows};
    const cuuint64_t strides[1] = {K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)GK, box_rows};
    const cuuint32_t estr[2] = {1u, 1u};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void*)base, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
// [B][T][1024] f16, box 64 channels x 128 frames x 1 branch; frames outside [0, T) read as zero.
bool map_conv(CUtensorMap* m, const __half* base, int T, int B) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)DM, (cuuint64_t)T, (cuuint64_t)B};
    const cuuint64_t strides[2] = {(cuuint64_t)DM * 2, (cuuint64_t)T * DM * 2};
    const cuuint32_t box[3] = {(cuuint32_t)GK, (cuuint32_t)GM, 1u};
    const cuuint32_t estr[3] = {1u, 1u, 1u};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, (void*)base, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int EPI, int ACT, int BN, bool CONV, int GS>
cudaError_t set_gemm_smem() {
    return cudaFuncSetAttribute(k_dit_gemm<EPI, ACT, BN, CONV, GS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)GemmSmem<BN, GS, EPI == DE_RESID || EPI == DE_F32>::SMEM);
}
template <int EPI, int ACT, int BN, bool CONV, int GS>
void launch_gemm(dim3 grid, const CUtensorMap& ma, const CUtensorMap& mb, const DitGemmArgs& a, cudaStream_t s) {
    launch_pdl(k_dit_gemm<EPI, ACT, BN, CONV, GS>, grid, dim3(G_THREADS),
               GemmSmem<BN, GS, EPI == DE_RESID || EPI == DE_F32>::SMEM, s, ma, mb, a);
}

std::atomic<int> g_sms{148};   // SMs of the device (set by init_device; contexts may load from several threads)

// The variants the estimator launches: the residual / addend epilogues stage their rows (4 stages, one
// CTA per SM); the others run 3 stages, two CTAs per SM, or 6 when the grid has at most one tile per SM.
cudaError_t init_device() {
    cudaError_t e;
    int dev = 0;
    int sms = 0;
    if ((e = cudaGetDevice(&dev)) || (e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev))) return e;
    g_sms.store(sms, std::memory_order_relaxed);
    if ((e = set_gemm_smem<DE_F32, ACT_NONE, 128, false, 4>())) return e;
    if ((e = set_gemm_smem<DE_RESID, ACT_NONE, 128, false, 4>())) return e;
    if ((e = set_gemm_smem<DE_QKV, ACT_NONE, 128, false, 3>())) return e;
    if ((e = set_gemm_smem<DE_QKV, ACT_NONE, 128, false, 6>())) return e;
    if ((e = set_gemm_smem<DE_F16, ACT_GELU_TANH, 128, false, 3>())) return e;
    if ((e = set_gemm_smem<DE_F16, ACT_GELU_TANH, 128, false, 6>())) return e;
    if ((e = set_gemm_smem<DE_F16, ACT_MISH, 64, true, 3>())) return e;
    if ((e = set_gemm_smem<DE_RESID, ACT_MISH, 64, true, 3>())) return e;
    if ((e = cudaFuncSetAttribute(k_dit_attn_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)FaSmem::SMEM))) return e;
    return cudaSuccess;
}

// Plain GEMM over R rows: A [R][K] f16, W [N][K] f16. epi / act: DE_F32 and DE_RESID without activation,
// DE_QKV, DE_F16 with GELU (tanh).
bool gemm(int epi, const __half* A, const __half* W, const DitGemmArgs& a, cudaStream_t s) {
    CUtensorMap ma, mb;
    const int sms = g_sms.load(std::memory_order_relaxed);
    const int rt = (a.R + GM - 1) / GM;
    if (!map_2d(&ma, A, (uint64_t)a.R, (uint64_t)a.K, GM) || !map_2d(&mb, W, (uint64_t)a.N, (uint64_t)a.K, 128))
        return false;
    const dim3 grid(a.N / 128, rt);
    const bool wide = (int)(grid.x * grid.y) > sms;
    switch (epi) {
        case DE_F32: launch_gemm<DE_F32, ACT_NONE, 128, false, 4>(grid, ma, mb, a, s); break;
        case DE_RESID: launch_gemm<DE_RESID, ACT_NONE, 128, false, 4>(grid, ma, mb, a, s); break;
        case DE_QKV:
            if (wide) launch_gemm<DE_QKV, ACT_NONE, 128, false, 3>(grid, ma, mb, a, s);
            else launch_gemm<DE_QKV, ACT_NONE, 128, false, 6>(grid, ma, mb, a, s);
            break;
        default:
            if (wide) launch_gemm<DE_F16, ACT_GELU_TANH, 128, false, 3>(grid, ma, mb, a, s);
            else launch_gemm<DE_F16, ACT_GELU_TANH, 128, false, 6>(grid, ma, mb, a, s);
            break;
    }
    return true;
}

// Attention of B branches of T frames over the keys < x_lens: q, k from qkv16 [B T][3072], v from vt16
// [B][16][64][tp]; output [B T][1024] f16.
bool attention_tc(const __half* qkv16, const __half* vt16, int tp, int T, int B, int x_lens, __half* out, int* err,
                  cudaStream_t s) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    AttnMaps m;
    if (!map_2d(&m.q, qkv16, (uint64_t)B * T, 3 * DM, FQ) || !map_2d(&m.k, qkv16, (uint64_t)B * T, 3 * DM, FK))
        return false;
    {
        const cuuint64_t dims[2] = {(cuuint64_t)T, (cuuint64_t)B * NHD * HDD};
        const cuuint64_t strides[1] = {(cuuint64_t)tp * 2};
        const cuuint32_t box[2] = {(cuuint32_t)FK, (cuuint32_t)HDD};
        const cuuint32_t estr[2] = {1u, 1u};
        if (enc(&m.vt, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void*)vt16, dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    launch_pdl(k_dit_attn_tc, dim3((unsigned)((T + FQ - 1) / FQ), NHD, (unsigned)B), dim3(FA_THREADS), FaSmem::SMEM, s, m,
               out, T, x_lens, err);
    return true;
}

// Grouped conv (16 groups of 64 channels, 31 taps, zero padding 15) over B branches of T frames, bias +
// Mish: X [B][T][1024] f16, Wc [1024][31 * 64] f16 (tap-major K); DE_F16 or DE_RESID.
bool conv(int epi, const __half* X, const __half* Wc, int B, const DitGemmArgs& a, cudaStream_t s) {
    CUtensorMap ma, mb;
    if (!map_conv(&ma, X, a.T, B) || !map_2d(&mb, Wc, (uint64_t)DM, (uint64_t)KCONV, 64)) return false;
    const dim3 grid(GCP, B * ((a.T + GM - 1) / GM));
    if (epi == DE_F16) launch_gemm<DE_F16, ACT_MISH, 64, true, 3>(grid, ma, mb, a, s);
    else launch_gemm<DE_RESID, ACT_MISH, 64, true, 3>(grid, ma, mb, a, s);
    return true;
}

struct Block {
    __half *wqkv = nullptr, *wo = nullptr, *w1 = nullptr, *w2 = nullptr;
    float *bqkv = nullptr, *bo = nullptr, *b1 = nullptr, *b2 = nullptr;
};

}  // namespace dit
}  // namespace gsvcu

using namespace gsvcu;
using namespace gsvcu::dit;

struct gsvcu_dit {
    int device = 0;
    cudaStream_t stream = nullptr;
    std::string err;
    gsvcu_dit_hparams hp{};
    std::vector<float> inv_freq;   // [32] (the checkpoint's stored values)
    std::vector<void*> wallocs;
    // weights
    __half *w_mel = nullptr, *w_c0 = nullptr, *w_c2 = nullptr, *w_t0 = nullptr, *w_t2 = nullptr, *w_ada = nullptr,
           *w_out = nullptr;
    float *b_c0 = nullptr, *b_c2 = nullptr, *b_t0 = nullptr, *b_t2 = nullptr, *b_ada = nullptr, *b_out = nullptr;
    std::vector<Block> L;
    // static cache (prepare): text path and the context projection, when the file has them
    bool has_text = false;
    float* cis = nullptr;                       // [4096][512]
    struct TextBlock {
        float *w7 = nullptr, *b = nullptr, *nw = nullptr, *nb = nullptr, *b1 = nullptr, *gamma = nullptr,
              *beta = nullptr, *b2 = nullptr;
        __half *w1 = nullptr, *w2 = nullptr;    // [1024][512], [512][1024]
    } TB[4];
    __half* w_ctx = nullptr;                    // [1024][640] (612 used)
    float* b_ctx = nullptr;
    // per-shape state (set_condition / prepare)
    int T = 0, x_lens = 0, cap_rows = 0, cap_T = 0;
    std::vector<void*> ballocs;
    float *cond = nullptr;        // [2][T][1024]: condition, negative condition
    float *rcos = nullptr, *rsin = nullptr;   // [T][32]
    float *xmel = nullptr;        // [100][T]
    float *x = nullptr;           // [R][1024]
    __half *a16 = nullptr;        // [R][1024] GEMM / conv operand
    __half *c16 = nullptr;        // [R][1024] conv 1 output
    __half *qkv16 = nullptr;      // [R][3072]
    __half *vt16 = nullptr;       // [2][16][64][tp]: v transposed for the attention's P V^T
    int tp = 0;                   // T rounded up to 8 (16-byte rows)
    __half *h16 = nullptr;        // [R][2048]
    __half *mel16 = nullptr;      // [R][128]
    float *vel = nullptr;         // [R][128]
    float *tsin = nullptr;        // [steps][256]
    int cap_steps = 0;
    float *temb = nullptr, *th = nullptr, *ada = nullptr;   // [1024], [1024], [depth * 6144 + 2048]
    float *vout = nullptr;        // [100][T]
    float *neg1 = nullptr, *neg2 = nullptr;   // [T][128]: the last two computed unconditional velocities
    int uncond_reuse = 0;         // gsv_dit_alg::uncond_reuse (0, 1 or 2)
    // cache-dit (DBCache, src/gsv_dit.cpp:1124-1323): settings, per-branch gates and device state
    struct DbCfg {
        int fn = 0, warmup = 8, warmup_interval = 1, max_cached = -1, max_cont = -1, ds = 4;
        float thr = 0.08f, max_accum = 0.0f;
    } dbc;
    struct DbBranch {
        int cached_steps = 0, cont = 0, hits = 0, misses = 0;
        bool valid = false;
        float acc = 0.0f, last_fd = 0.0f;
    } dbb[2];
    int db_step = 0;
    float *xtrunk = nullptr, *xfront = nullptr, *rcur = nullptr;   // [T][1024]
    float *rprev[2] = {nullptr, nullptr}, *mrprev[2] = {nullptr, nullptr};   // [T][1024] per branch
    double* fdpart = nullptr;     // [FD_BLOCKS][2]
    float* fd_dev = nullptr;      // [1]
    float *mu_d = nullptr, *px_d = nullptr;   // prepare inputs [512][T], [100][T]
    float *txf = nullptr;         // [T][512] text path (f32)
    __half *tx16 = nullptr;       // [T][512] ConvNeXt operand
    float *hb = nullptr;          // [T][1024] ConvNeXt hidden (f32)
    float *gx = nullptr;          // [1024] GRN norms
    __half *ctx16 = nullptr;      // [2T][640] context projection operand
    int* errw = nullptr;

    int fail(int code, const std::string& m) {
        err = m;
        return code;
    }
    ~gsvcu_dit() {
        int prev = -1;
        cudaGetDevice(&prev);
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        for (void* p : wallocs) cudaFree(p);
        for (void* p : ballocs) cudaFree(p);
        cudaFree(tsin);
        cudaFree(errw);
        if (stream) cudaStreamDestroy(stream);
        if (prev >= 0) cudaSetDevice(prev);
    }
    template <typename TT>
    int upload(const std::vector<TT>& h, TT** dst) {
        if (cudaMalloc((void**)dst, h.size() * sizeof(TT)) != cudaSuccess) {
            cudaGetLastError();
            return fail(GSVCU_ERR_OOM, "cudaMalloc of DiT weights failed");
        }
        wallocs.push_back(*dst);
        if (cudaMemcpy(*dst, h.data(), h.size() * sizeof(TT), cudaMemcpyHostToDevice) != cudaSuccess)
            return fail(GSVCU_ERR_CUDA, "DiT weight upload failed");
        return GSVCU_OK;
    }
    int reserve(int T_, int rows);
    int prepare_dev(const float* prompt_x, const float* mu);
    int forward(int B, int negative, const float* tsin_dev, int l0, int l1, bool trunk, bool head,
                float* save_trunk = nullptr);
    int velocity_cached(int bi, const float* tsin_dev);
    void db_reset_state() {
        for (DbBranch& d : dbb) d = DbBranch();
        db_step = 0;
    }
};

namespace {

uint16_t h16_of(float f) { return __half_as_ushort(__float2half_rn(f)); }

// F32 / F16 tensor widened to f32 on the host.
bool tensor_f32(const GgufTensor* t, size_t n, std::vector<float>& out) {
    if (!t) return false;
    out.resize(n);
    if (t->type == 0 && t->nbytes >= n * 4) {
        std::memcpy(out.data(), t->data, n * 4);
        return true;
    }
    if (t->type == 1 && t->nbytes >= n * 2) {
        const __half* h = (const __half*)t->data;
        for (size_t i = 0; i < n; i++) out[i] = __half2float(h[i]);
        return true;
    }
    return false;
}

}  // namespace

// Buffers for T_ frames and `rows` rows: reused while they are large enough (every buffer is indexed with
// the current T), reallocated otherwise. A change of T zeroes cache-dit's previous front residuals, as the
// reference's rebuilt cache does (src/gsv_dit.cpp:1124-1149).
int gsvcu_dit::reserve(int T_, int rows) {
    if (T_ <= cap_T && rows <= cap_rows) {
        if (T_ != T) {
            T = T_;
            tp = (T_ + 7) & ~7;
            for (int b = 0; b < 2; b++)
                if (cudaMemsetAsync(rprev[b], 0, (size_t)T_ * DM * 4, stream) != cudaSuccess)
                    return fail(GSVCU_ERR_CUDA, "cache reset failed");
        }
        return GSVCU_OK;
    }
    cudaStreamSynchronize(stream);
    for (void* p : ballocs) cudaFree(p);
    ballocs.clear();
    cap_rows = 0;
    cap_T = 0;
    T = 0;
    const size_t R = (size_t)rows, TT = (size_t)T_;
    const size_t nada = (size_t)hp.depth * ADA + 2 * DM;
    struct A { void** p; size_t bytes; };
    const A list[] = {{(void**)&cond, 2 * TT * DM * 4}, {(void**)&rcos, TT * 32 * 4}, {(void**)&rsin, TT * 32 * 4},
                      {(void**)&xmel, MEL * TT * 4}, {(void**)&x, R * DM * 4}, {(void**)&a16, R * DM * 2},
                      {(void**)&c16, R * DM * 2}, {(void**)&qkv16, R * 3 * DM * 2}, {(void**)&h16, R * FFD * 2},
                      {(void**)&vt16, 2 * (size_t)DM * ((TT + 7) & ~(size_t)7) * 2},
                      {(void**)&mel16, R * MELP * 2}, {(void**)&vel, R * MELP * 4}, {(void**)&temb, DM * 4},
                      {(void**)&th, DM * 4}, {(void**)&ada, nada * 4}, {(void**)&vout, MEL * TT * 4},
                      {(void**)&mu_d, TXD * TT * 4}, {(void**)&px_d, MEL * TT * 4}, {(void**)&txf, TT * TXD * 4},
                      {(void**)&tx16, TT * TXD * 2}, {(void**)&hb, TT * TXI * 4}, {(void**)&gx, TXI * 4},
                      {(void**)&ctx16, 2 * TT * CTXK * 2}, {(void**)&neg1, TT * MELP * 4},
                      {(void**)&neg2, TT * MELP * 4}, {(void**)&xtrunk, TT * DM * 4}, {(void**)&xfront, TT * DM * 4},
                      {(void**)&rcur, TT * DM * 4}, {(void**)&rprev[0], TT * DM * 4}, {(void**)&rprev[1], TT * DM * 4},
                      {(void**)&mrprev[0], TT * DM * 4}, {(void**)&mrprev[1], TT * DM * 4},
                      {(void**)&fdpart, FD_BLOCKS * 16}, {(void**)&fd_dev, 16}};
    for (const A& a : list) {
        if (cudaMalloc(a.p, a.bytes) != cudaSuccess) {
            cudaGetLastError();
            return fail(GSVCU_ERR_OOM, "cudaMalloc of DiT activations failed");
        }
        ballocs.push_back(*a.p);
    }
    // rows past R of the padded operands stay zero (the GEMMs' A tiles read them)
    cudaMemsetAsync(mel16, 0, R * MELP * 2, stream);
    // cache-dit's previous front residuals start at zero with new buffers (src/gsv_dit.cpp:1147-1149)
    cudaMemsetAsync(rprev[0], 0, TT * DM * 4, stream);
    cudaMemsetAsync(rprev[1], 0, TT * DM * 4, stream);
    cap_rows = rows;
    cap_T = T_;
    T = T_;
    tp = (T_ + 7) & ~7;
    return GSVCU_OK;
}

// The static cache of gsv_dit::prepare (src/gsv_dit.cpp:486-531): text path (mu^T + freqs_cis, 4 ConvNeXtV2
// blocks), then condition / negative condition = proj_ctx([prompt_x | text] / [0 | text]) + bias into `cond`.
// prompt_x [100][T] and mu [512][T] are host arrays; T and the RoPE tables are set by the caller.
int gsvcu_dit::prepare_dev(const float* prompt_x, const float* mu) {
    cudaStream_t s = stream;
    if (cudaMemcpyAsync(mu_d, mu, (size_t)TXD * T * 4, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(px_d, prompt_x, (size_t)MEL * T * 4, cudaMemcpyHostToDevice, s) != cudaSuccess)
        return fail(GSVCU_ERR_CUDA, "prepare input upload failed");
    const unsigned gb = (unsigned)std::min(2048, (TXD * T + 255) / 256);
    launch_pdl(k_dit_text_in, dim3(gb), dim3(256), 0, s, (const float*)mu_d, (const float*)cis, T, txf);
    DitGemmArgs a{};
    a.R = T; a.T = T; a.x_lens = T; a.err = errw;
    for (int bi = 0; bi < 4; bi++) {
        const TextBlock& w = TB[bi];
        launch_pdl(k_dit_dwconv_ln, dim3((unsigned)((T + 7) / 8)), dim3(256), 0, s, (const float*)txf, T,
                   (const float*)w.w7, (const float*)w.b, (const float*)w.nw, (const float*)w.nb, tx16);
        DitGemmArgs g = a;
        g.N = TXI; g.K = TXD; g.bias = w.b1; g.out32 = hb; g.ld = TXI;
        if (!gemm(DE_F32, tx16, w.w1, g, s)) return fail(GSVCU_ERR_CUDA, "tensor map encoding failed");
        launch_pdl(k_dit_gelu_colnorm, dim3(TXI / 32), dim3(256), 0, s, hb, T, gx);
        launch_pdl(k_dit_grn, dim3((unsigned)std::min(1024, (TXI * T + 255) / 256)), dim3(256), 0, s, (const float*)hb,
                   T, (const float*)gx, (const float*)w.gamma, (const float*)w.beta, h16);
        g = a;
        g.N = TXD; g.K = TXI; g.bias = w.b2; g.out32 = txf; g.ld = TXD;
        if (!gemm(DE_RESID, h16, w.w2, g, s)) return fail(GSVCU_ERR_CUDA, "tensor map encoding failed");
    }
    launch_pdl(k_dit_pack_ctx, dim3((unsigned)std::min(2048, (2 * T * CTXK + 255) / 256)), dim3(256), 0, s,
               (const float*)px_d, (const float*)txf, T, ctx16);
    DitGemmArgs g = a;
    g.R = 2 * T; g.N = DM; g.K = CTXK; g.bias = b_ctx; g.out32 = cond; g.ld = DM;
    if (!gemm(DE_F32, ctx16, w_ctx, g, s)) return fail(GSVCU_ERR_CUDA, "tensor map encoding failed");
    if (cudaPeekAtLastError() != cudaSuccess) return fail(GSVCU_ERR_CUDA, cudaGetErrorString(cudaGetLastError()));
    return GSVCU_OK;
}

// One cache-dit step of branch bi (src/gsv_dit.cpp:1250-1323): the front (trunk + the first fn blocks), the
// criterion fd of its residual against the last computed one, the host-side gates (warmup, threshold,
// max_cached, max_cont, max_accum); on a hit the middle blocks are replaced by the residual they added at
// the last miss, on a miss they run and their residual and the front residual are kept. The velocity goes to
// rows [0, T) of vel.
int gsvcu_dit::velocity_cached(int bi, const float* tsin_dev) {
    cudaStream_t s = stream;
    const int depth = hp.depth, fn = dbc.fn;
    DbBranch& d = dbb[bi];
    int rc;
    if ((rc = forward(1, bi, tsin_dev, 0, fn, true, false, xtrunk))) return rc;
    const int ds = (dbc.ds >= 1 && T % dbc.ds == 0) ? dbc.ds : 1;
    const int n = (T / ds) * DM;
    launch_pdl(k_dit_fd_partial, dim3(FD_BLOCKS), dim3(256), 0, s, (const float*)x, (const float*)xtrunk,
               (const float*)rprev[bi], n, ds, rcur, fdpart);
    launch_pdl(k_dit_fd_final, dim3(1), dim3(32), 0, s, (const double*)fdpart, FD_BLOCKS, fd_dev);
    float fd = 0.0f;
    if (cudaMemcpyAsync(&fd, fd_dev, 4, cudaMemcpyDeviceToHost, s) != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess)
        return fail(GSVCU_ERR_CUDA, std::string("criterion read failed: ") + cudaGetErrorString(cudaGetLastError()));
    d.last_fd = fd;
    bool hit = false;
    const int iv = dbc.warmup_interval < 1 ? 1 : dbc.warmup_interval;
    const bool warm = db_step < dbc.warmup && (db_step % iv) == 0;
    if (d.valid && dbc.thr > 0.0f && !warm) {
        bool ok = fd < dbc.thr;
        if (ok && dbc.max_cached >= 0 && d.cached_steps >= dbc.max_cached) ok = false;
        if (ok && dbc.max_cont >= 0 && d.cont >= dbc.max_cont) {
            ok = false;
            d.cont = 0;
        }
        if (ok && dbc.max_accum > 0.0f && d.acc >= dbc.max_accum) ok = false;
        hit = ok;
    }
    if (fd > 0.0f) d.acc += fd;
    const size_t nx = (size_t)T * DM;
    const unsigned gx = (unsigned)std::min<size_t>(4096, (nx + 255) / 256);
    if (hit) {   // x_mid = x_front + the middle residual of the last miss
        launch_pdl(k_dit_axpy, dim3(gx), dim3(256), 0, s, (const float*)x, (const float*)mrprev[bi], 1.0f, nx, x);
        if ((rc = forward(1, bi, tsin_dev, depth, depth, false, true))) return rc;
        d.hits++;
        d.cached_steps++;
        d.cont++;
    } else {
        if (cudaMemcpyAsync(xfront, x, nx * 4, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
            return fail(GSVCU_ERR_CUDA, "front copy failed");
        if ((rc = forward(1, bi, tsin_dev, fn, depth, false, true))) return rc;
        launch_pdl(k_dit_axpy, dim3(gx), dim3(256), 0, s, (const float*)x, (const float*)xfront, -1.0f, nx, mrprev[bi]);
        if (cudaMemcpyAsync(rprev[bi], rcur, (size_t)n * 4, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
            return fail(GSVCU_ERR_CUDA, "residual copy failed");
        d.misses++;
        d.valid = true;
        d.cont = 0;
    }
    return GSVCU_OK;
}

// One estimator pass over B branches (B = 2: rows [0, T) use the condition, [T, 2T) the negative one;
// B = 1: the condition selected by `negative`) from xmel and the time features at tsin_dev: with `trunk`
// the time embedding, AdaLN modulations and the trunk (a copy of its output into save_trunk when given),
// then DiT blocks [l0, l1) on x, and with `head` the output projection into vel ([R][128]).
int gsvcu_dit::forward(int B, int negative, const float* tsin_dev, int l0, int l1, bool trunk, bool head,
                       float* save_trunk) {
    const int R = B * T;
    cudaStream_t s = stream;
    const int depth = hp.depth;
    auto gemv_blocks = [](int n) { return dim3((unsigned)((n + 7) / 8)); };
    DitGemmArgs a{};
    a.R = R; a.T = T; a.x_lens = x_lens; a.err = errw;
    if (trunk) {
    // time embedding, then every block's AdaLN modulation and norm_out's in one launch
    launch_pdl(k_dit_gemv<false, true>, gemv_blocks(DM), dim3(256), 0, s, (const __half*)w_t0, (const float*)b_t0,
               tsin_dev, DM, TSIN, th);
    launch_pdl(k_dit_gemv<false, false>, gemv_blocks(DM), dim3(256), 0, s, (const __half*)w_t2, (const float*)b_t2,
               (const float*)th, DM, DM, temb);
    const int nada = depth * ADA + 2 * DM;
    launch_pdl(k_dit_gemv<true, false>, gemv_blocks(nada), dim3(256), 0, s, (const __half*)w_ada, (const float*)b_ada,
               (const float*)temb, nada, DM, ada);
    // trunk
    launch_pdl(k_dit_pack_mel, dim3(std::min(1024, (R * MELP + 255) / 256)), dim3(256), 0, s, (const float*)xmel, T, B,
               mel16);
    {
        DitGemmArgs g = a;
        g.N = DM; g.K = MELP; g.out32 = x; g.ld = DM;
        g.add = cond + (B == 1 && negative ? (size_t)T * DM : 0);
        if (!gemm(DE_F32, mel16, w_mel, g, s)) return fail(GSVCU_ERR_CUDA, "tensor map encoding failed");
    }
    launch_pdl(k_dit_mask16, dim3(std::min(2048, (R * DM / 4 + 255) / 256)), dim3(256), 0, s, (const float*)x, R, T,
               x_lens, a16);
    {
        DitGemmArgs g = a;
        g.N = DM; g.K = KCONV; g.bias = b_c0; g.out16 = c16; g.ld = DM;
        if (!conv(DE_F16, a16, w_c0, B, g, s)) return fail(GSVCU_ERR_CUDA, "tensor map encoding failed");
        g.bias = b_c2; g.out16 = nullptr; g.out32 = x; g.use_mask = 1;
        if (!conv(DE_RESID, c16, w_c2, B, g, s)) return fail(GSVCU_ERR_CUDA, "tensor map encoding failed");
    }
    if (save_trunk && cudaMemcpyAsync(save_trunk, x, (size_t)R * DM * 4, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
        return fail(GSVCU_ERR_CUDA, "trunk copy failed");
    }   // trunk
    const dim3 rows8((unsigned)((R + 7) / 8));
    for (int li = l0; li < l1; li++) {
        const Block& w = L[(size_t)li];
        const float* m = ada + (size_t)li * ADA;   // shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp
        launch_pdl(k_dit_lnmod, rows8, dim3(256), 0, s, (const float*)x, R, m, m + DM, a16);
        DitGemmArgs g = a;
        g.N = 3 * DM; g.K = DM; g.bias = w.bqkv; g.out16 = qkv16; g.ld = 3 * DM; g.rcos = rcos; g.rsin = rsin;
        g.vt16 = vt16; g.tp = tp;
        if (!gemm(DE_QKV, a16, w.wqkv, g, s)) return fail(GSVCU_ERR_CUDA, "tensor map encoding failed");
        if (!attention_tc(qkv16, vt16, tp, T, B, x_lens, a16, errw, s)) return fail(GSVCU_ERR_CUDA, "tensor map encoding failed");
        g = a;
        g.N = DM; g.K = DM; g.bias = w.bo; g.out32 = x; g.ld = DM; g.gate = m + 2 * DM; g.use_mask = 1;
        if (!gemm(DE_RESID, a16, w.wo, g, s)) return fail(GSVCU_ERR_CUDA, "tensor map encoding failed");
        launch_pdl(k_dit_lnmod, rows8, dim3(256), 0, s, (const float*)x, R, m + 3 * DM, m + 4 * DM, a16);
        g = a;
        g.N = FFD; g.K = DM; g.bias = w.b1; g.out16 = h16; g.ld = FFD;
        if (!gemm(DE_F16, a16, w.w1, g, s)) return fail(GSVCU_ERR_CUDA, "tensor map encoding failed");
        g = a;
        g.N = DM; g.K = FFD; g.bias = w.b2; g.out32 = x; g.ld = DM; g.gate = m + 5 * DM;
        if (!gemm(DE_RESID, h16, w.w2, g, s)) return fail(GSVCU_ERR_CUDA, "tensor map encoding failed");
    }
    if (head) {
        const float* m = ada + (size_t)depth * ADA;   // norm_out: scale, shift
        launch_pdl(k_dit_lnmod, rows8, dim3(256), 0, s, (const float*)x, R, m + DM, m, a16);
        DitGemmArgs g = a;
        g.N = MELP; g.K = DM; g.bias = b_out; g.out32 = vel; g.ld = MELP;
        if (!gemm(DE_F32, a16, w_out, g, s)) return fail(GSVCU_ERR_CUDA, "tensor map encoding failed");
    }
    if (cudaPeekAtLastError() != cudaSuccess) return fail(GSVCU_ERR_CUDA, cudaGetErrorString(cudaGetLastError()));
    return GSVCU_OK;
}

namespace {

// SinusPositionEmbedding(256) of the time t as the reference evaluates it (src/gsv_dit.cpp:755-769).
void time_sin(float t, float* out) {
    const float e = (float)(std::log(10000.0) / 127.0);
    for (int i = 0; i < 128; i++) {
        const float a = 1000.0f * t * std::exp(-e * (float)i);
        out[i] = std::sin(a);
        out[128 + i] = std::cos(a);
    }
}

int check_err(gsvcu_dit* c) {
    int e = 0;
    if (cudaStreamSynchronize(c->stream) != cudaSuccess) return c->fail(GSVCU_ERR_CUDA, cudaGetErrorString(cudaGetLastError()));
    if (cudaMemcpy(&e, c->errw, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return c->fail(GSVCU_ERR_CUDA, "error word read failed");
    if (e) {
        cudaMemset(c->errw, 0, 4);
        return c->fail(GSVCU_ERR_CUDA, "a DiT GEMM wait timed out");
    }
    return GSVCU_OK;
}

int upload_tsin(gsvcu_dit* c, const std::vector<float>& h) {
    const int steps = (int)(h.size() / TSIN);
    if (steps > c->cap_steps) {
        cudaStreamSynchronize(c->stream);
        cudaFree(c->tsin);
        c->tsin = nullptr;
        c->cap_steps = 0;
        if (cudaMalloc((void**)&c->tsin, h.size() * 4) != cudaSuccess) {
            cudaGetLastError();
            return c->fail(GSVCU_ERR_OOM, "cudaMalloc of time features failed");
        }
        c->cap_steps = steps;
    }
    if (cudaMemcpyAsync(c->tsin, h.data(), h.size() * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
        return c->fail(GSVCU_ERR_CUDA, "time feature upload failed");
    return GSVCU_OK;
}

struct DevGuard {
    int prev = -1;
    explicit DevGuard(int dev) {
        cudaGetDevice(&prev);
        cudaSetDevice(dev);
    }
    ~DevGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

}  // namespace

extern "C" {

int gsvcu_dit_load(int device, const char* path, gsvcu_dit** out) {
    if (!out || !path) return GSVCU_ERR_ARG;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        cudaGetLastError();
        return GSVCU_ERR_DEVICE;
    }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10) return GSVCU_ERR_DEVICE;
    DevGuard dg(device);
    gsvcu_dit* c = new gsvcu_dit();
    c->device = device;
    auto done = [&](int rc) {
        if (rc == GSVCU_OK) *out = c;
        else {
            std::fprintf(stderr, "gsvcu_dit_load: %s\n", c->err.c_str());
            delete c;
        }
        return rc;
    };
    if (init_device() != cudaSuccess || encode_fn() == nullptr ||
        cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc((void**)&c->errw, 4) != cudaSuccess || cudaMemset(c->errw, 0, 4) != cudaSuccess) {
        cudaGetLastError();
        return done(c->fail(GSVCU_ERR_CUDA, "device set-up failed"));
    }
    GgufFile f;
    std::string e;
    if (!f.open(path, e)) return done(c->fail(GSVCU_ERR_IO, e));
    uint32_t v = 0;
    auto u32 = [&](const char* k, int def) { return f.get_u32(k, v) ? (int)v : def; };
    gsvcu_dit_hparams& hp = c->hp;
    hp.dim = u32("dit.dim", DM);
    hp.depth = u32("dit.depth", 22);
    hp.heads = u32("dit.heads", NHD);
    hp.dim_head = u32("dit.dim_head", HDD);
    hp.ff_mult = u32("dit.ff_mult", 2);
    hp.mel_dim = u32("dit.mel_dim", MEL);
    hp.text_dim = u32("dit.text_dim", 512);
    if (hp.dim != DM || hp.heads != NHD || hp.dim_head != HDD || hp.ff_mult != 2 || hp.mel_dim != MEL ||
        u32("dit.conv_pos_groups", GCP) != GCP || u32("dit.conv_pos_kernel", KCP) != KCP ||
        u32("dit.rope_dims", HDD) != HDD || hp.depth <= 0 || hp.depth > 64)
        return done(c->fail(GSVCU_ERR_FORMAT, "unsupported DiT dims (1024 / 16 heads x 64 / FFN 2048 / mel 100, "
                                              "conv_pos 16 groups x 31 taps, RoPE on 64 dims)"));
    // f16 rows [N][Kp] from a [N][K] tensor (K <= Kp, zero padded); rows past N of Np zero
    auto mat = [&](const std::string& name, int N, int K, int Np, int Kp, std::vector<uint16_t>& dst, size_t row0) -> int {
        const GgufTensor* t = f.tensor(name);
        std::vector<float> hst;
        if (!t || !tensor_f32(t, (size_t)N * K, hst)) return c->fail(GSVCU_ERR_FORMAT, "missing or bad tensor " + name);
        (void)Np;
        for (int r = 0; r < N; r++)
            for (int k = 0; k < K; k++) dst[(row0 + r) * (size_t)Kp + k] = h16_of(hst[(size_t)r * K + k]);
        return GSVCU_OK;
    };
    auto vecf = [&](const std::string& name, int n, std::vector<float>& dst, size_t off) -> int {
        std::vector<float> hst;
        if (!tensor_f32(f.tensor(name), (size_t)n, hst)) return c->fail(GSVCU_ERR_FORMAT, "missing or bad tensor " + name);
        std::memcpy(dst.data() + off, hst.data(), (size_t)n * 4);
        return GSVCU_OK;
    };
    int rc;
    std::vector<uint16_t> hw;
    std::vector<float> hb;
    // input projection of the mel channels (no bias: the condition rows carry it), K padded to 128
    hw.assign((size_t)DM * MELP, 0);
    if ((rc = mat("dit.input_embed.proj.weight_mel", DM, MEL, DM, MELP, hw, 0)) ||
        (rc = c->upload(hw, (uint16_t**)&c->w_mel)))
        return done(rc);
    // conv_pos: [G][OCg][ICg * 31] with inner index ic * 31 + tap -> [1024][tap * 64 + ic]
    for (int li = 0; li < 2; li++) {
        const std::string base = std::string("dit.input_embed.conv_pos_embed.conv1d.") + (li ? "2" : "0");
        const GgufTensor* t = f.tensor(base + ".weight");
        std::vector<float> hst;
        if (!t || !tensor_f32(t, (size_t)DM * KCONV, hst)) return done(c->fail(GSVCU_ERR_FORMAT, "missing or bad " + base));
        hw.assign((size_t)DM * KCONV, 0);
        for (int o = 0; o < DM; o++)
            for (int ic = 0; ic < ICG; ic++)
                for (int k = 0; k < KCP; k++)
                    hw[(size_t)o * KCONV + (size_t)k * ICG + ic] = h16_of(hst[(size_t)o * KCONV + (size_t)ic * KCP + k]);
        hb.assign(DM, 0.0f);
        if ((rc = c->upload(hw, (uint16_t**)(li ? &c->w_c2 : &c->w_c0))) || (rc = vecf(base + ".bias", DM, hb, 0)) ||
            (rc = c->upload(hb, li ? &c->b_c2 : &c->b_c0)))
            return done(rc);
    }
    // time MLP 256 -> 1024 -> 1024
    hw.assign((size_t)DM * TSIN, 0);
    hb.assign(DM, 0.0f);
    if ((rc = mat("dit.time_embed.time_mlp.0.weight", DM, TSIN, DM, TSIN, hw, 0)) || (rc = c->upload(hw, (uint16_t**)&c->w_t0)) ||
        (rc = vecf("dit.time_embed.time_mlp.0.bias", DM, hb, 0)) || (rc = c->upload(hb, &c->b_t0)))
        return done(rc);
    hw.assign((size_t)DM * DM, 0);
    if ((rc = mat("dit.time_embed.time_mlp.2.weight", DM, DM, DM, DM, hw, 0)) || (rc = c->upload(hw, (uint16_t**)&c->w_t2)) ||
        (rc = vecf("dit.time_embed.time_mlp.2.bias", DM, hb, 0)) || (rc = c->upload(hb, &c->b_t2)))
        return done(rc);
    // AdaLN projections of every block, then norm_out's, as one matrix
    const size_t nada = (size_t)hp.depth * ADA + 2 * DM;
    hw.assign(nada * DM, 0);
    hb.assign(nada, 0.0f);
    for (int li = 0; li < hp.depth; li++) {
        const std::string b = "dit.transformer_blocks." + std::to_string(li) + ".attn_norm.linear.";
        if ((rc = mat(b + "weight", ADA, DM, ADA, DM, hw, (size_t)li * ADA)) || (rc = vecf(b + "bias", ADA, hb, (size_t)li * ADA)))
            return done(rc);
    }
    if ((rc = mat("dit.norm_out.linear.weight", 2 * DM, DM, 2 * DM, DM, hw, (size_t)hp.depth * ADA)) ||
        (rc = vecf("dit.norm_out.linear.bias", 2 * DM, hb, (size_t)hp.depth * ADA)) ||
        (rc = c->upload(hw, (uint16_t**)&c->w_ada)) || (rc = c->upload(hb, &c->b_ada)))
        return done(rc);
    // output projection, 100 rows padded to 128
    hw.assign((size_t)MELP * DM, 0);
    hb.assign(MELP, 0.0f);
    if ((rc = mat("dit.proj_out.weight", MEL, DM, MELP, DM, hw, 0)) || (rc = vecf("dit.proj_out.bias", MEL, hb, 0)) ||
        (rc = c->upload(hw, (uint16_t**)&c->w_out)) || (rc = c->upload(hb, &c->b_out)))
        return done(rc);
    // blocks
    c->L.resize((size_t)hp.depth);
    for (int li = 0; li < hp.depth; li++) {
        Block& w = c->L[(size_t)li];
        const std::string b = "dit.transformer_blocks." + std::to_string(li) + ".";
        hw.assign((size_t)3 * DM * DM, 0);
        hb.assign((size_t)3 * DM, 0.0f);
        const char* qkv[3] = {"attn.to_q.", "attn.to_k.", "attn.to_v."};
        for (int j = 0; j < 3; j++)
            if ((rc = mat(b + qkv[j] + "weight", DM, DM, DM, DM, hw, (size_t)j * DM)) ||
                (rc = vecf(b + qkv[j] + "bias", DM, hb, (size_t)j * DM)))
                return done(rc);
        if ((rc = c->upload(hw, (uint16_t**)&w.wqkv)) || (rc = c->upload(hb, &w.bqkv))) return done(rc);
        hw.assign((size_t)DM * DM, 0);
        hb.assign(DM, 0.0f);
        if ((rc = mat(b + "attn.to_out.0.weight", DM, DM, DM, DM, hw, 0)) || (rc = vecf(b + "attn.to_out.0.bias", DM, hb, 0)) ||
            (rc = c->upload(hw, (uint16_t**)&w.wo)) || (rc = c->upload(hb, &w.bo)))
            return done(rc);
        hw.assign((size_t)FFD * DM, 0);
        hb.assign(FFD, 0.0f);
        if ((rc = mat(b + "ff.ff.0.0.weight", FFD, DM, FFD, DM, hw, 0)) || (rc = vecf(b + "ff.ff.0.0.bias", FFD, hb, 0)) ||
            (rc = c->upload(hw, (uint16_t**)&w.w1)) || (rc = c->upload(hb, &w.b1)))
            return done(rc);
        hw.assign((size_t)DM * FFD, 0);
        hb.assign(DM, 0.0f);
        if ((rc = mat(b + "ff.ff.2.weight", DM, FFD, DM, FFD, hw, 0)) || (rc = vecf(b + "ff.ff.2.bias", DM, hb, 0)) ||
            (rc = c->upload(hw, (uint16_t**)&w.w2)) || (rc = c->upload(hb, &w.b2)))
            return done(rc);
    }
    c->inv_freq.assign(32, 0.0f);
    if ((rc = vecf("dit.rotary_embed.inv_freq", 32, c->inv_freq, 0))) return done(rc);
    // the static cache's text path and context projection (prepare); optional
    if (f.tensor("dit.text_embed.freqs_cis")) {
        std::vector<float> cis;
        if ((rc = [&]() -> int {
                 cis.assign((size_t)MAXPOS * TXD, 0.0f);
                 return vecf("dit.text_embed.freqs_cis", MAXPOS * TXD, cis, 0);
             }()) ||
            (rc = c->upload(cis, &c->cis)))
            return done(rc);
        for (int bi = 0; bi < 4; bi++) {
            gsvcu_dit::TextBlock& w = c->TB[bi];
            const std::string b = "dit.text_embed.text_blocks." + std::to_string(bi) + ".";
            struct V { const char* n; int len; float** dst; };
            const V vs[] = {{"dwconv.weight", 7 * TXD, &w.w7}, {"dwconv.bias", TXD, &w.b}, {"norm.weight", TXD, &w.nw},
                            {"norm.bias", TXD, &w.nb}, {"pwconv1.bias", TXI, &w.b1}, {"grn.gamma", TXI, &w.gamma},
                            {"grn.beta", TXI, &w.beta}, {"pwconv2.bias", TXD, &w.b2}};
            for (const V& vv : vs) {
                hb.assign((size_t)vv.len, 0.0f);
                if ((rc = vecf(b + vv.n, vv.len, hb, 0)) || (rc = c->upload(hb, vv.dst))) return done(rc);
            }
            hw.assign((size_t)TXI * TXD, 0);
            if ((rc = mat(b + "pwconv1.weight", TXI, TXD, TXI, TXD, hw, 0)) || (rc = c->upload(hw, (uint16_t**)&w.w1)))
                return done(rc);
            hw.assign((size_t)TXD * TXI, 0);
            if ((rc = mat(b + "pwconv2.weight", TXD, TXI, TXD, TXI, hw, 0)) || (rc = c->upload(hw, (uint16_t**)&w.w2)))
                return done(rc);
        }
        hw.assign((size_t)DM * CTXK, 0);
        hb.assign(DM, 0.0f);
        if ((rc = mat("dit.input_embed.proj.weight_ctx", DM, MEL + TXD, DM, CTXK, hw, 0)) ||
            (rc = c->upload(hw, (uint16_t**)&c->w_ctx)) || (rc = vecf("dit.input_embed.proj.bias", DM, hb, 0)) ||
            (rc = c->upload(hb, &c->b_ctx)))
            return done(rc);
        c->has_text = true;
    }
    return done(GSVCU_OK);
}

void gsvcu_dit_destroy(gsvcu_dit* c) { delete c; }

const char* gsvcu_dit_last_error(const gsvcu_dit* c) { return c ? c->err.c_str() : "null DiT context"; }

int gsvcu_dit_get_hparams(const gsvcu_dit* c, gsvcu_dit_hparams* out) {
    if (!c || !out) return GSVCU_ERR_ARG;
    *out = c->hp;
    return GSVCU_OK;
}

}  // extern "C"

namespace {

// Buffers for T frames, x_lens, and the RoPE tables of head 0: angle = n * inv_freq[i] in float
// (src/gsv_dit.cpp:787-793).
int set_shape(gsvcu_dit* c, int T, int x_lens) {
    if (x_lens <= 0 || x_lens > T) x_lens = T;
    int rc;
    const int old_T = c->T;
    if ((rc = c->reserve(T, 2 * T))) return rc;
    if (x_lens != c->x_lens && old_T == T) {   // the reference rebuilds its cache state on a new x_lens too
        for (int b = 0; b < 2; b++)
            if (cudaMemsetAsync(c->rprev[b], 0, (size_t)T * DM * 4, c->stream) != cudaSuccess)
                return c->fail(GSVCU_ERR_CUDA, "cache reset failed");
    }
    c->x_lens = x_lens;
    std::vector<float> cs((size_t)T * 32), sn((size_t)T * 32);
    for (int n = 0; n < T; n++)
        for (int i = 0; i < 32; i++) {
            const float a = (float)n * c->inv_freq[(size_t)i];
            cs[(size_t)n * 32 + i] = std::cos(a);
            sn[(size_t)n * 32 + i] = std::sin(a);
        }
    if (cudaMemcpyAsync(c->rcos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
        cudaMemcpyAsync(c->rsin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
        cudaStreamSynchronize(c->stream) != cudaSuccess)
        return c->fail(GSVCU_ERR_CUDA, "RoPE table upload failed");
    return GSVCU_OK;
}

// randn01 * 0.875 of gsv_dit::sample (src/gsv_dit.cpp:1403-1408, 1436-1438): gsv_rng's xorshift64* draws
// (src/gsv_sampler.h:33-40), two per value, Box-Muller in float.
void seeded_noise(uint64_t seed, float* x, size_t n) {
    uint64_t st = seed ? seed : 1;
    auto uniform01 = [&]() {
        st ^= st >> 12;
        st ^= st << 25;
        st ^= st >> 27;
        return (float)(((st * 0x2545F4914F6CDD1Dull) >> 40) * (1.0 / 16777216.0));
    };
    for (size_t i = 0; i < n; i++) {
        float u1 = uniform01();
        const float u2 = uniform01();
        if (u1 < 1e-30f) u1 = 1e-30f;
        x[i] = sqrtf(-2.0f * logf(u1)) * cosf(6.283185307179586f * u2) * 0.875f;
    }
}

}  // namespace

extern "C" {

int gsvcu_dit_set_condition(gsvcu_dit* c, const float* cond, const float* neg, int32_t T, int32_t x_lens) {
    if (!c || !cond || !neg || T <= 0 || T > 65536) return GSVCU_ERR_ARG;
    DevGuard dg(c->device);
    int rc;
    if ((rc = set_shape(c, T, x_lens))) return rc;
    const size_t cb = (size_t)T * DM * 4;
    if (cudaMemcpyAsync(c->cond, cond, cb, cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
        cudaMemcpyAsync(c->cond + (size_t)T * DM, neg, cb, cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
        cudaStreamSynchronize(c->stream) != cudaSuccess)
        return c->fail(GSVCU_ERR_CUDA, "condition upload failed");
    return GSVCU_OK;
}

int gsvcu_dit_prepare(gsvcu_dit* c, const float* prompt_mel, const float* mu, int32_t T, int32_t x_lens) {
    if (!c || !prompt_mel || !mu || T <= 0) return GSVCU_ERR_ARG;
    if (!c->has_text) return c->fail(GSVCU_ERR_FORMAT, "the model file has no text_embed / proj.weight_ctx tensors");
    if (T > MAXPOS) return c->fail(GSVCU_ERR_ARG, "T beyond the 4096 text positions");
    DevGuard dg(c->device);
    int rc;
    if ((rc = set_shape(c, T, x_lens)) || (rc = c->prepare_dev(prompt_mel, mu))) return rc;
    return check_err(c);
}

int gsvcu_dit_op_condition(gsvcu_dit* c, float* out) {
    if (!c || !out) return GSVCU_ERR_ARG;
    if (c->T <= 0) return c->fail(GSVCU_ERR_ARG, "op before set_condition() / prepare()");
    DevGuard dg(c->device);
    if (cudaMemcpyAsync(out, c->cond, (size_t)2 * c->T * DM * 4, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess)
        return c->fail(GSVCU_ERR_CUDA, std::string("output read failed: ") + cudaGetErrorString(cudaGetLastError()));
    return check_err(c);
}

int gsvcu_dit_sample_full(gsvcu_dit* c, const float* mu, const float* prompt, int32_t P, int32_t T, int32_t steps,
                          float cfg, uint64_t seed, const float* x0, int32_t skip_steps, float* mel_out) {
    if (!c || !mu || !prompt || !mel_out || T <= 0 || steps <= 0) return GSVCU_ERR_ARG;
    if (P <= 0 || P >= T) return c->fail(GSVCU_ERR_ARG, "bad prompt length");
    std::vector<float> px((size_t)MEL * T, 0.0f);
    for (int ch = 0; ch < MEL; ch++) std::memcpy(px.data() + (size_t)ch * T, prompt + (size_t)ch * P, (size_t)P * 4);
    int rc;
    if ((rc = gsvcu_dit_prepare(c, px.data(), mu, T, T))) return rc;
    std::vector<float> noise;
    if (!x0) {
        noise.resize((size_t)MEL * T);
        seeded_noise(seed, noise.data(), noise.size());
        x0 = noise.data();
    }
    return gsvcu_dit_sample(c, x0, P, steps, cfg, skip_steps, mel_out);
}

int gsvcu_dit_velocity(gsvcu_dit* c, const float* x_mel, float t, int32_t negative, float* vel) {
    if (!c || !x_mel || !vel) return GSVCU_ERR_ARG;
    if (c->T <= 0) return c->fail(GSVCU_ERR_ARG, "velocity() before set_condition()");
    DevGuard dg(c->device);
    std::vector<float> ts(TSIN);
    time_sin(t, ts.data());
    int rc;
    if ((rc = upload_tsin(c, ts))) return rc;
    if (cudaMemcpyAsync(c->xmel, x_mel, (size_t)MEL * c->T * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
        return c->fail(GSVCU_ERR_CUDA, "input upload failed");
    if (c->dbc.fn > 0 && c->dbc.fn < c->hp.depth) {   // cache-dit path (src/gsv_dit.cpp:1325-1333)
        if ((rc = c->velocity_cached(negative ? 1 : 0, c->tsin))) return rc;
    } else if ((rc = c->forward(1, negative, c->tsin, 0, c->hp.depth, true, true))) {
        return rc;
    }
    launch_pdl(k_dit_vel_out, dim3((unsigned)std::min(1024, (MEL * c->T + 255) / 256)), dim3(256), 0, c->stream,
               (const float*)c->vel, c->T, c->vout);
    if (cudaMemcpyAsync(vel, c->vout, (size_t)MEL * c->T * 4, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess)
        return c->fail(GSVCU_ERR_CUDA, std::string("output read failed: ") + cudaGetErrorString(cudaGetLastError()));
    return check_err(c);
}

int gsvcu_dit_sample(gsvcu_dit* c, const float* x0, int32_t P, int32_t steps, float cfg, int32_t skip_steps,
                     float* mel_out) {
    if (!c || !x0 || !mel_out || steps <= 0) return GSVCU_ERR_ARG;
    if (c->T <= 0) return c->fail(GSVCU_ERR_ARG, "sample() before set_condition()");
    const int T = c->T;
    if (P <= 0 || P >= T) return c->fail(GSVCU_ERR_ARG, "bad prompt length");
    DevGuard dg(c->device);
    std::vector<float> ts((size_t)steps * TSIN);
    const float dt = 1.0f / (float)steps;
    for (int j = 0; j < steps; j++) time_sin((float)j * dt, ts.data() + (size_t)j * TSIN);
    int rc;
    if ((rc = upload_tsin(c, ts))) return rc;
    if (cudaMemcpyAsync(c->xmel, x0, (size_t)MEL * T * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
        return c->fail(GSVCU_ERR_CUDA, "input upload failed");
    const bool guided = cfg > 1e-5f;
    const dim3 eg((unsigned)std::min(1024, (MEL * T + 255) / 256));
    const float* none = nullptr;
    // x[:, :P] = 0 before the first step (src/gsv_dit.cpp:1440-1441)
    launch_pdl(k_dit_euler, eg, dim3(256), 0, c->stream, (const float*)c->vel, T, 0, none, none, 0.0f, 0.0f, P, c->xmel);
    // uncond_reuse (src/gsv_dit.cpp:1449-1468): odd steps take the last computed unconditional velocity (1) or
    // extrapolate the last two (2) instead of running the negative branch. With cache-dit each branch runs
    // alone through its gates (the unconditional velocity goes to rows [T, 2T) of vel).
    float *p1 = c->neg1, *p2 = c->neg2;
    int neg_count = 0;
    const int ur = c->uncond_reuse;
    const bool cached = c->dbc.fn > 0 && c->dbc.fn < c->hp.depth;
    if (cached) c->db_reset_state();   // a new inference (src/gsv_dit.cpp:1427)
    float* vneg = c->vel + (size_t)T * MELP;
    for (int j = 0; j < steps; j++) {
        c->db_step = j;
        if (j < skip_steps) continue;   // the first skip_steps steps leave x as it is (src/gsv_dit.cpp:1444-1448)
        const float* tj = c->tsin + (size_t)j * TSIN;
        const bool odd = (j & 1) != 0;
        const bool reuse = guided && odd && ((ur == 1 && neg_count >= 1) || (ur == 2 && neg_count >= 2));
        if (guided && !reuse) {   // both velocities
            if (cached) {
                if ((rc = c->velocity_cached(1, tj))) return rc;
                if (cudaMemcpyAsync(vneg, c->vel, (size_t)T * MELP * 4, cudaMemcpyDeviceToDevice, c->stream) != cudaSuccess)
                    return c->fail(GSVCU_ERR_CUDA, "velocity copy failed");
                if ((rc = c->velocity_cached(0, tj))) return rc;
            } else if ((rc = c->forward(2, 0, tj, 0, c->hp.depth, true, true))) {
                return rc;
            }
            if (ur) {   // keep the last two computed unconditional velocities
                std::swap(p1, p2);
                if (cudaMemcpyAsync(p1, vneg, (size_t)T * MELP * 4, cudaMemcpyDeviceToDevice, c->stream) != cudaSuccess)
                    return c->fail(GSVCU_ERR_CUDA, "velocity copy failed");
            }
            neg_count++;
            launch_pdl(k_dit_euler, eg, dim3(256), 0, c->stream, (const float*)c->vel, T, 1, (const float*)vneg, none, cfg,
                       dt, P, c->xmel);
        } else {   // the conditional velocity only (unguided, or the unconditional one reused)
            if (cached) {
                if ((rc = c->velocity_cached(0, tj))) return rc;
            } else if ((rc = c->forward(1, 0, tj, 0, c->hp.depth, true, true))) {
                return rc;
            }
            launch_pdl(k_dit_euler, eg, dim3(256), 0, c->stream, (const float*)c->vel, T, 1,
                       reuse ? (const float*)p1 : none, (reuse && ur == 2) ? (const float*)p2 : none, cfg, dt, P,
                       c->xmel);
        }
    }
    for (int ch = 0; ch < MEL; ch++)
        if (cudaMemcpyAsync(mel_out + (size_t)ch * (T - P), c->xmel + (size_t)ch * T + P, (size_t)(T - P) * 4,
                            cudaMemcpyDeviceToHost, c->stream) != cudaSuccess)
            return c->fail(GSVCU_ERR_CUDA, std::string("output read failed: ") + cudaGetErrorString(cudaGetLastError()));
    return check_err(c);
}

int gsvcu_dit_synthesize(gsvcu_dit* c, const float* fea_ref, int32_t R, const float* fea_todo, int32_t N,
                         const float* mel_ref, int32_t mel_ref_T, int32_t steps, float cfg, uint64_t seed,
                         int32_t block_override, const float* const* x0_chunks, int32_t n_x0, int32_t skip_steps,
                         float* mel_out) {
    if (!c || !fea_ref || !fea_todo || !mel_ref || !mel_out || steps <= 0) return GSVCU_ERR_ARG;
    if (R <= 0 || N <= 0 || mel_ref_T <= 0) return c->fail(GSVCU_ERR_ARG, "synthesize(): bad R, N or mel_ref_T");
    // synthesize_v5_mel's framing (src/gsv_dit.cpp:1480-1581): the reference frames are the last 500 of the
    // common length of mel_ref and fea_ref; chunks of at most 640 frames (block_override > 0: that many),
    // with reference + chunk <= 1000 frames; every chunk after the first takes as prompt the reference
    // frames with their last 32 replaced by the previous chunk's last generated frames (and features).
    constexpr int REF = 500, TAIL = 32, TOTAL = 1000, MAXCHUNK = 640;
    const int ref_common = std::min(mel_ref_T, R);
    const int ref_off = ref_common > REF ? ref_common - REF : 0;
    const int rf = ref_common - ref_off;
    const int chunk = std::min(TOTAL - rf, block_override > 0 ? block_override : MAXCHUNK);
    if (chunk <= 0) return c->fail(GSVCU_ERR_ARG, "synthesize(): reference too long");
    auto cols = [&](const float* src, int C, int ld, int off, int n, float* dst, int dld) {
        for (int ch = 0; ch < C; ch++) std::memcpy(dst + (size_t)ch * dld, src + (size_t)ch * ld + off, (size_t)n * 4);
    };
    std::vector<float> mel_ref_s((size_t)MEL * rf), fea_ref_s((size_t)TXD * rf);
    cols(mel_ref, MEL, mel_ref_T, ref_off, rf, mel_ref_s.data(), rf);
    cols(fea_ref, TXD, R, ref_off, rf, fea_ref_s.data(), rf);
    std::vector<float> roll_mel = mel_ref_s, roll_fea = fea_ref_s, prompt = mel_ref_s, feat = fea_ref_s;
    int roll_n = rf;
    uint64_t cseed = seed;
    int ci = 0;
    for (int start = 0; start < N; start += chunk, ci++) {
        const int tlen = std::min(chunk, N - start);
        if (start > 0) {
            const int tail = std::min({TAIL, rf, roll_n});
            const int prefix = rf - tail;
            for (int ch = 0; ch < MEL; ch++) {
                std::memcpy(prompt.data() + (size_t)ch * rf, mel_ref_s.data() + (size_t)ch * rf, (size_t)prefix * 4);
                std::memcpy(prompt.data() + (size_t)ch * rf + prefix, roll_mel.data() + (size_t)ch * roll_n + (roll_n - tail),
                            (size_t)tail * 4);
            }
            for (int ch = 0; ch < TXD; ch++) {
                std::memcpy(feat.data() + (size_t)ch * rf, fea_ref_s.data() + (size_t)ch * rf, (size_t)prefix * 4);
                std::memcpy(feat.data() + (size_t)ch * rf + prefix, roll_fea.data() + (size_t)ch * roll_n + (roll_n - tail),
                            (size_t)tail * 4);
            }
        }
        const int T = rf + tlen;   // mu = [features of the prompt | the chunk's target features]
        std::vector<float> mu((size_t)TXD * T), gen((size_t)MEL * tlen);
        cols(feat.data(), TXD, rf, 0, rf, mu.data(), T);
        cols(fea_todo, TXD, N, start, tlen, mu.data() + rf, T);
        const float* x0 = (x0_chunks && ci < n_x0) ? x0_chunks[ci] : nullptr;
        int rc;
        if ((rc = gsvcu_dit_sample_full(c, mu.data(), prompt.data(), rf, T, steps, cfg, cseed, x0, ci == 0 ? skip_steps : 0,
                                        gen.data())))
            return rc;
        cseed = cseed * 6364136223846793005ull + 1442695040888963407ull;
        cols(gen.data(), MEL, tlen, 0, tlen, mel_out + start, N);
        const int keep = std::min(rf, tlen);   // roll: the chunk's last frames and their features
        roll_n = keep;
        roll_mel.resize((size_t)MEL * keep);
        roll_fea.resize((size_t)TXD * keep);
        cols(gen.data(), MEL, tlen, tlen - keep, keep, roll_mel.data(), keep);
        cols(fea_todo, TXD, N, start + tlen - keep, keep, roll_fea.data(), keep);
    }
    return GSVCU_OK;
}

void gsvcu_dit_time_sin(float t, float* out256) {
    if (out256) time_sin(t, out256);
}

int gsvcu_dit_get_inv_freq(const gsvcu_dit* c, float* out32) {
    if (!c || !out32) return GSVCU_ERR_ARG;
    std::memcpy(out32, c->inv_freq.data(), 32 * 4);
    return GSVCU_OK;
}

int gsvcu_dit_set_dbcache(gsvcu_dit* c, int32_t fn, float threshold, int32_t warmup, int32_t warmup_interval,
                          int32_t max_cached, int32_t max_cont, float max_accum, int32_t downsample) {
    if (!c) return GSVCU_ERR_ARG;
    const int nfn = fn > 0 ? fn : 0, nds = downsample >= 1 ? downsample : 1;
    const bool structural = nfn != c->dbc.fn || nds != c->dbc.ds;
    c->dbc.fn = nfn;
    c->dbc.thr = threshold;
    c->dbc.warmup = warmup;
    c->dbc.warmup_interval = warmup_interval;
    c->dbc.max_cached = max_cached;
    c->dbc.max_cont = max_cont;
    c->dbc.max_accum = max_accum;
    c->dbc.ds = nds;
    if (structural) {   // new cache state: gates reset, previous residuals zero (src/gsv_dit.cpp:1097-1149)
        c->db_reset_state();
        if (c->T > 0) {
            DevGuard dg(c->device);
            for (int b = 0; b < 2; b++)
                if (cudaMemsetAsync(c->rprev[b], 0, (size_t)c->T * DM * 4, c->stream) != cudaSuccess)
                    return c->fail(GSVCU_ERR_CUDA, "cache reset failed");
            if (cudaStreamSynchronize(c->stream) != cudaSuccess) return c->fail(GSVCU_ERR_CUDA, "cache reset failed");
        }
    }
    return GSVCU_OK;
}

int gsvcu_dit_db_set_step(gsvcu_dit* c, int32_t step) {
    if (!c) return GSVCU_ERR_ARG;
    c->db_step = step;
    return GSVCU_OK;
}

int gsvcu_dit_db_get_stats(const gsvcu_dit* c, int32_t* steps, int32_t* hits2, int32_t* misses2, float* last_fd2,
                           float* acc2) {
    if (!c || !steps || !hits2 || !misses2 || !last_fd2 || !acc2) return GSVCU_ERR_ARG;
    *steps = c->db_step;
    for (int b = 0; b < 2; b++) {
        hits2[b] = c->dbb[b].hits;
        misses2[b] = c->dbb[b].misses;
        last_fd2[b] = c->dbb[b].last_fd;
        acc2[b] = c->dbb[b].acc;
    }
    return GSVCU_OK;
}

int gsvcu_dit_set_alg(gsvcu_dit* c, int32_t uncond_reuse) {
    if (!c) return GSVCU_ERR_ARG;
    c->uncond_reuse = (uncond_reuse < 0 || uncond_reuse > 2) ? 0 : uncond_reuse;
    return GSVCU_OK;
}

int gsvcu_dit_get_alg(const gsvcu_dit* c, int32_t* uncond_reuse) {
    if (!c || !uncond_reuse) return GSVCU_ERR_ARG;
    *uncond_reuse = c->uncond_reuse;
    return GSVCU_OK;
}

int gsvcu_dit_op_hidden(gsvcu_dit* c, const float* x_mel, float t, int32_t n_blocks, float* hidden) {
    if (!c || !x_mel || !hidden || n_blocks < 0) return GSVCU_ERR_ARG;
    if (c->T <= 0) return c->fail(GSVCU_ERR_ARG, "op before set_condition()");
    if (n_blocks > c->hp.depth) n_blocks = c->hp.depth;
    DevGuard dg(c->device);
    std::vector<float> ts(TSIN);
    time_sin(t, ts.data());
    int rc;
    if ((rc = upload_tsin(c, ts))) return rc;
    if (cudaMemcpyAsync(c->xmel, x_mel, (size_t)MEL * c->T * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
        return c->fail(GSVCU_ERR_CUDA, "input upload failed");
    if ((rc = c->forward(2, 0, c->tsin, 0, n_blocks, true, false))) return rc;
    if (cudaMemcpyAsync(hidden, c->x, (size_t)2 * c->T * DM * 4, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess)
        return c->fail(GSVCU_ERR_CUDA, std::string("output read failed: ") + cudaGetErrorString(cudaGetLastError()));
    return check_err(c);
}

int gsvcu_dit_stream(gsvcu_dit* c, void** out) {
    if (!c || !out) return GSVCU_ERR_ARG;
    *out = (void*)c->stream;
    return GSVCU_OK;
}

}  // extern "C"
