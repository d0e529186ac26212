// gemm_tc.cu -- prefill Q8_0 GEMM on the 5th-generation tensor cores: TMA tile loads, tcgen05.mma with
// the accumulator in tensor memory (TMEM), a warp-specialised persistent pipeline.
//
// Semantics: exactly those of k_gemm_q8 / k_gemm_q8_tile (ggml's Q8_0 mul_mat, reference
// src/gsv_ar.cpp:244,260,262,263): per output (feature f, token n) the integer dot of every 32-value
// block is exact, and the float result is accumulated block by block, in block order:
//     acc = fma((float)isum_b, d_w[f][b] * d_x[n][b], acc).
// The tensor cores compute isum_b: weights and activations enter as fp16 numbers holding the Q8_0
// integers (exact), and one block's 32 products (each |q_w q_x| <= 128 * 127) sum to at most 2^19 in
// magnitude, so the fp32 accumulation of tcgen05.mma kind::f16 is exact in any order. One TMEM buffer
// holds one block's 128 x 128 integer sums; the epilogue warps run the float chain on CUDA cores.
//
// Persistent: one CTA per SM walks the output tiles (128 features x 128 tokens) i = blockIdx.x,
// blockIdx.x + gridDim.x, ...; every role keeps its own ring counters across tiles, so the TMA producer
// and the MMA issuer run ahead into the next tile while the epilogue warps finish and store this one.
// 18 warps:
//   warp 0      TMA producer: per tile the tile's scales (d_w of its features and d_x of its tokens, f32,
//               block-major, from the transposed planes k_tc_prep writes) into one of two scale buffers,
//               then the 64-value K slices of W and X (SWIZZLE_128B) into a ring of stages
//   warp 1      TMEM allocator (512 columns = 2 accumulator buffers of two blocks) and the MMA issuer:
//               per stage (two Q8_0 blocks) four tcgen05.mma (K = 16 each), each block into its own 128
//               columns of buffer (stage count) % 2, one commit to that buffer's barrier
//   warps 2..17 epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 (its 32 features), columns
//               32 ((w - 2) / 4) .. +31 (32 tokens) of each block; per stage one wait, then in chunks of
//               16 tokens (each chunk's tcgen05.ld in flight while the previous chunk's chain steps run)
//               acc[t] = fma(sum, d_w * d_x[t], acc[t]): the products
//               two tokens per packed f32x2 multiply (each lane rounded as the scalar operation), the
//               chain steps as scalar FMAs; after the tile's last block the fused epilogue
//               (bias, residual, ReLU + Q8_0 quantization, K/V page store) stores straight from
//               registers: for one token the warp's 32 features are 128 contiguous bytes.
// Every mbarrier wait is bounded; a wait that gives up sets the error word and the CTA's abort flag, the
// other roles stop at their next wait, in-flight copies and MMAs are waited for (bounded) and the TMEM is
// freed before exit. No cluster launch and no multicast: each CTA loads its own tiles from this GPU's
// memory.
#include <cuda.h>

#include <atomic>
#include <cstdio>

#include "kernels.h"
#include "tc_common.cuh"

namespace gsvcu {
namespace {

using namespace tc;

constexpr int TC_BM = 128;          // features per tile
constexpr int TC_BN = 128;          // tokens per tile
constexpr int TC_BK = 64;           // K values per stage (two Q8_0 blocks; one 128-byte swizzle row)
constexpr int TC_TBUF = 2;          // TMEM accumulator buffers, one stage (two Q8_0 blocks) each
constexpr int TC_EPI_WARPS = 16;    // 4 per TMEM lane quarter, 32 token columns each
constexpr int TC_STORE_WARP = 2 + TC_EPI_WARPS;   // issues the bulk stores of staged output tiles
constexpr int TC_THREADS = 32 * (3 + TC_EPI_WARPS);
constexpr int TC_MAX_KB = 64;       // K <= 2048
constexpr int STAGE_W = TC_BM * TC_BK * 2;
constexpr int STAGE_X = TC_BN * TC_BK * 2;

// Shared memory of the variant for K <= 32 * KBMAX: the operand stages (1024-byte aligned for the
// 128-byte swizzle), two scale buffers of [d_w block-major | d_x block-major] f32, for K <= 512 an f32
// output tile [128 tokens][128 features] staged for the bulk store, the barriers, the TMEM address and
// the abort flag.
template <int KBMAX>
struct TcLayout {
    static constexpr int STAGES = KBMAX <= 16 ? 4 : 3;
    static constexpr bool YSTAGE = KBMAX <= 16;
    static constexpr size_t SCALES = (size_t)KBMAX * 128 * 4;   // one of d_w / d_x of one tile
    static constexpr size_t OFF_W = 0;
    static constexpr size_t OFF_X = OFF_W + (size_t)STAGES * STAGE_W;
    static constexpr size_t OFF_S = OFF_X + (size_t)STAGES * STAGE_X;
    static constexpr size_t OFF_Y = OFF_S + 4 * SCALES;
    static constexpr size_t OFF_BAR = OFF_Y + (YSTAGE ? (size_t)TC_BN * TC_BM * 4 : 0);
    // full, empty, tfull, tempty, sfull, sempty, done, ystaged, yfree
    static constexpr int NBAR = 2 * STAGES + 2 * TC_TBUF + 4 + 1 + 2;
    static constexpr size_t OFF_MISC = OFF_BAR + NBAR * 8;
    static constexpr size_t SMEM = OFF_MISC + 16 + 1024;            // + slack to align the base to 1024
};
static_assert(TcLayout<64>::SMEM <= 232448, "shared memory of the K <= 2048 variant");
static_assert(TcLayout<16>::SMEM <= 232448, "shared memory of the K <= 512 variant");

constexpr uint32_t TC_IDESC = idesc_f16(TC_BM, TC_BN);

// Shared-memory loads by shared-window address.
__device__ __forceinline__ float lds_f32(uint32_t a) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
    return v;
}
// four f32 as two packed pairs
__device__ __forceinline__ void lds_f32x4(uint32_t a, uint64_t& lo, uint64_t& hi) {
    asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(lo), "=l"(hi) : "r"(a));
}


struct TcMaps {
    CUtensorMap w;    // f16 [N][K] weight values, box 64 x 128, 128-byte swizzle
    CUtensorMap x;    // f16 [M][K] activation values, same box
    CUtensorMap dw;   // f32 [KB][N] weight scales (transposed), box 128 x KB
    CUtensorMap dx;   // f32 [KB][ld] activation scales (transposed), box 128 x KB
    CUtensorMap y;    // f32 [M][N] output, box 128 x 128 (bulk store of a staged tile; K <= 512, not RELU_Q8)
};

// One block's chain step for 16 of the warp's tokens (acc[t0 + i], i < 16): sums r[i], d_w of this
// thread's feature, d_x of the 16 tokens at shared-window address xa.
__device__ __forceinline__ void chain16(float (&acc)[32], const int t0, const float (&r)[16], float dw, uint32_t xa) {
    const uint64_t dw2 = f2pack(dw, dw);
#pragma unroll
    for (int c = 0; c < 4; c++) {   // acc = fma(sum, d_w * d_x, acc): the products two tokens per
        uint64_t x01, x23;          // instruction, the chain steps one each
        lds_f32x4(xa + 16u * c, x01, x23);
        const uint64_t p01 = fmul2(dw2, x01), p23 = fmul2(dw2, x23);
        acc[t0 + 4 * c] = __fmaf_rn(r[4 * c], f2lo(p01), acc[t0 + 4 * c]);
        acc[t0 + 4 * c + 1] = __fmaf_rn(r[4 * c + 1], f2hi(p01), acc[t0 + 4 * c + 1]);
        acc[t0 + 4 * c + 2] = __fmaf_rn(r[4 * c + 2], f2lo(p23), acc[t0 + 4 * c + 2]);
        acc[t0 + 4 * c + 3] = __fmaf_rn(r[4 * c + 3], f2hi(p23), acc[t0 + 4 * c + 3]);
    }
}

template <int EPI, int KBMAX>
__global__ void __launch_bounds__(TC_THREADS, 1) k_gemm_q8_tc(const __grid_constant__ TcMaps maps, const GemmQ8Params p) {
    using L = TcLayout<KBMAX>;
    constexpr int S = L::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = smem_raw + ((1024u - (su32(smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = p.K, KB = K / QK, nstage = K / TC_BK;
    const int ntf = p.N / TC_BM, ntiles = ntf * ((p.M + TC_BN - 1) / TC_BN);
    uint64_t* bars = (uint64_t*)(sm + L::OFF_BAR);
    const uint32_t bar0 = su32(bars);
    auto full = [&](int s) { return bar0 + 8u * s; };
    auto empty = [&](int s) { return bar0 + 8u * (S + s); };
    auto tfull = [&](int j) { return bar0 + 8u * (2 * S + j); };
    auto tempty = [&](int j) { return bar0 + 8u * (2 * S + TC_TBUF + j); };
    auto sfull = [&](int b) { return bar0 + 8u * (2 * S + 2 * TC_TBUF + b); };
    auto sempty = [&](int b) { return bar0 + 8u * (2 * S + 2 * TC_TBUF + 2 + b); };
    const uint32_t done_bar = bar0 + 8u * (2 * S + 2 * TC_TBUF + 4);
    const uint32_t ystaged = bar0 + 8u * (2 * S + 2 * TC_TBUF + 5), yfree = bar0 + 8u * (2 * S + 2 * TC_TBUF + 6);
    constexpr bool YTMA = L::YSTAGE && EPI != EPI_RELU_Q8;   // output through the staged bulk store
    float* ys = (float*)(sm + L::OFF_Y);                      // [128 tokens][128 features]
    auto scale_dw = [&](int b) { return (float*)(sm + L::OFF_S + (size_t)(2 * b) * L::SCALES); };
    auto scale_dx = [&](int b) { return (float*)(sm + L::OFF_S + (size_t)(2 * b + 1) * L::SCALES); };
    uint32_t* tmem_slot = (uint32_t*)(sm + L::OFF_MISC);
    volatile int* abort_flag = (volatile int*)(sm + L::OFF_MISC + 4);

    if (tid == 0) {
        for (int s = 0; s < S; s++) { bar_init(full(s), 1); bar_init(empty(s), 1); }
        // the epilogue releases buffers with one arrival per thread (no divergent lane-0 branch)
        for (int j = 0; j < TC_TBUF; j++) { bar_init(tfull(j), 1); bar_init(tempty(j), 32 * TC_EPI_WARPS); }
        for (int b = 0; b < 2; b++) { bar_init(sfull(b), 1); bar_init(sempty(b), 32 * TC_EPI_WARPS); }
        bar_init(done_bar, 1);
        bar_init(ystaged, 32 * TC_EPI_WARPS);
        bar_init(yfree, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&maps.w) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&maps.x) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&maps.dw) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&maps.dx) : "memory");
    }
    if (warp == 1) {   // TMEM: 512 columns, address written to shared memory
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                     "r"(512)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // every operand (the fp16 planes and the transposed scales) is written by the preceding k_tc_prep
    griddep_wait();
    griddep_launch();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            int g = 0, lt = 0;   // stage loads and scale loads issued
            bool ok = true;
            for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
                const int f0 = (tile % ntf) * TC_BM, t0 = (tile / ntf) * TC_BN;
                const int b = lt & 1;
                if (!bar_wait(sempty(b), ((uint32_t)(lt >> 1) & 1u) ^ 1u, abort_flag)) { ok = false; break; }
                bar_expect_tx(sfull(b), (uint32_t)(2 * KB * 128 * 4));
                tma_load_2d(su32(scale_dw(b)), &maps.dw, f0, 0, sfull(b));
                tma_load_2d(su32(scale_dx(b)), &maps.dx, t0, 0, sfull(b));
                lt++;
                for (int ks = 0; ks < nstage; ks++, g++) {
                    const int s = g % S;
                    if (!bar_wait(empty(s), ((uint32_t)(g / S) & 1u) ^ 1u, abort_flag)) { ok = false; break; }
                    bar_expect_tx(full(s), STAGE_W + STAGE_X);
                    tma_load_2d(su32(sm + L::OFF_W + (size_t)s * STAGE_W), &maps.w, ks * TC_BK, f0, full(s));
                    tma_load_2d(su32(sm + L::OFF_X + (size_t)s * STAGE_X), &maps.x, ks * TC_BK, t0, full(s));
                }
            }
            if (!ok) {
                if (p.err) atomicExch(p.err, 1);
                *abort_flag = 1;
            }
            // every copy this thread issued has landed before the CTA may exit (bounded): the last S
            // stages and the last two scale loads
            for (int k = g - 1; k >= 0 && k >= g - S; k--)
                for (uint32_t it = 0; it < TC_POLL_LIMIT; it++)
                    if (bar_try(full(k % S), (uint32_t)(k / S) & 1u)) break;
            for (int k = lt - 1; k >= 0 && k >= lt - 2; k--)
                for (uint32_t it = 0; it < TC_POLL_LIMIT; it++)
                    if (bar_try(sfull(k & 1), (uint32_t)(k >> 1) & 1u)) break;
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            int g = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
                for (int ks = 0; ks < nstage; ks++, g++) {
                    const int s = g % S, j = g % TC_TBUF;
                    if (!bar_wait(full(s), (uint32_t)(g / S) & 1u, abort_flag)) { ok = false; break; }
                    if (!bar_wait(tempty(j), ((uint32_t)(g / TC_TBUF) & 1u) ^ 1u, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t wa = su32(sm + L::OFF_W + (size_t)s * STAGE_W);
                    const uint32_t xa = su32(sm + L::OFF_X + (size_t)s * STAGE_X);
#pragma unroll
                    for (int half = 0; half < 2; half++) {   // block 2 ks + half into columns 128 half
                        const uint32_t d = tmem + (uint32_t)(j * 2 * TC_BN + half * TC_BN);
#pragma unroll
                        for (int kk = 0; kk < 2; kk++) {
                            const uint32_t off = (uint32_t)(half * 64 + kk * 32);   // bytes along K in the row
                            umma_f16(d, umma_desc(wa + off), umma_desc(xa + off), TC_IDESC, (uint32_t)kk);
                        }
                    }
                    umma_commit(tfull(j));
                    umma_commit(empty(s));
                }
            }
            if (!ok) {
                if (p.err) atomicExch(p.err, 1);
                *abort_flag = 1;
            }
            // all MMAs issued above have completed before the TMEM is released (bounded)
            umma_commit(done_bar);
            for (uint32_t it = 0; it < TC_POLL_LIMIT; it++)
                if (bar_try(done_bar, 0)) break;
        }
    } else if (warp == TC_STORE_WARP) {
        // ---------------------------------------------------------------- output bulk stores
        if (YTMA && lane == 0) {
            int lt = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, lt++) {
                const int f0 = (tile % ntf) * TC_BM, t0 = (tile / ntf) * TC_BN;
                if (!bar_wait(ystaged, (uint32_t)lt & 1u, abort_flag)) { ok = false; break; }
                tma_store_2d(&maps.y, su32(ys), f0, t0);   // rows past M are not written
                asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");   // the staging tile was read
                bar_arrive(yfree);
            }
            if (!ok) {
                if (p.err) atomicExch(p.err, 1);
                *abort_flag = 1;
            }
            asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");   // every store complete before exit
        }
    } else {
        // ---------------------------------------------------------------- epilogue warps
        const int q = warp & 3;                   // TMEM lane quarter this warp may access
        const int col0 = ((warp - 2) >> 2) * 32;  // its 32 token columns
        const int fl = q * 32 + lane;             // feature (TMEM lane) of this thread
        const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)col0;
        int g = 0, lt = 0;   // stages and tiles consumed
        bool ok = true;
        for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, lt++) {
            const int f0 = (tile % ntf) * TC_BM, t0 = (tile / ntf) * TC_BN;
            const int b = lt & 1;
            if (!bar_wait_warp(sfull(b), (uint32_t)(lt >> 1) & 1u, abort_flag)) { ok = false; break; }
            // scales of block kb: d_w of this feature at dw_a + 512 kb, d_x of this warp's tokens at
            // dx_a + 512 kb (shared-window addresses)
            const uint32_t dw_a = su32(scale_dw(b)) + 4u * fl, dx_a = su32(scale_dx(b)) + 4u * col0;
            const int f = f0 + fl;
            const float bias = p.bias ? p.bias[f] : 0.0f;   // requested now, used after the chain
            float acc[32];   // the chain of each of the warp's 32 tokens
#pragma unroll
            for (int i = 0; i < 32; i++) acc[i] = 0.0f;
            for (int kb = 0; kb < KB; kb += 2, g++) {
                const int j = g % TC_TBUF;
                if (!bar_wait_warp(tfull(j), (uint32_t)(g / TC_TBUF) & 1u, abort_flag)) { ok = false; break; }
                tc_fence_after();
                // four chunks of 16 tokens (block kb: tokens 0-15, 16-31; block kb + 1: the same), each
                // chunk's TMEM load issued before the previous chunk's chain steps run
                const uint32_t ta = tbase + (uint32_t)(j * 2 * TC_BN);
                const float dw0 = lds_f32(dw_a + 512u * kb), dw1 = lds_f32(dw_a + 512u * (kb + 1));
                float ra[16], rb[16];
                tmem_ld16(ta, ra);
                tmem_wait_ld();
                tmem_bind(ra);
                tmem_ld16(ta + 16, rb);
                chain16(acc, 0, ra, dw0, dx_a + 512u * kb);
                tmem_wait_ld();
                tmem_bind(rb);
                tmem_ld16(ta + TC_BN, ra);
                chain16(acc, 16, rb, dw0, dx_a + 512u * kb + 64u);
                tmem_wait_ld();
                tmem_bind(ra);
                tmem_ld16(ta + TC_BN + 16, rb);
                chain16(acc, 0, ra, dw1, dx_a + 512u * (kb + 1));
                tmem_wait_ld();
                tmem_bind(rb);
                chain16(acc, 16, rb, dw1, dx_a + 512u * (kb + 1) + 64u);
                tc_fence_before();
                bar_arrive(tempty(j));   // both blocks' sums are consumed: the buffer is free
            }
            if (!ok) break;
            bar_arrive(sempty(b));   // this tile's scales are no longer read
            // ------------------------------------------------------------ fused epilogue, from registers
            const int nb = t0 + col0;   // first token of this warp
            if (YTMA) {   // the staging tile is free once the previous tile's bulk store has read it
                if (!bar_wait_warp(yfree, ((uint32_t)lt & 1u) ^ 1u, abort_flag)) { ok = false; break; }
            }
            if (EPI == EPI_BIAS) {
                // K/V columns of a QKV GEMM (a feature tile lies wholly in Q, K or V): lane l finds the
                // page row of token nb + l, the store loop takes it by shuffle
                const bool kv = p.kv.pool && f0 >= D;
                size_t tok_off = 0, feat_off = 0;
                if (kv) {
                    const int kvsel = (f - D) >> 9, fh = (f - D) & (D - 1);
                    feat_off = ((size_t)kvsel * NH + (fh >> 5)) * (PAGE * HD) + (fh & 31);
                    const int n = nb + lane;
                    if (n < p.M) {
                        const int slot = p.kv.tok_slot[n], pos = p.kv.tok_pos[n];
                        const int page = p.kv.block_table[(size_t)slot * p.kv.max_pages + pos / PAGE];
                        tok_off = ((size_t)page * p.kv.n_layer + p.kv.layer) * 2 * NH * (PAGE * HD) +
                                  (size_t)(pos % PAGE) * HD;
                    }
                }
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    const int n = nb + i;
                    const float a = acc[i];
                    const float y = __fadd_rn(a, bias);
                    size_t e = 0;
                    if (kv) e = (size_t)__shfl_sync(0xffffffffu, (unsigned long long)tok_off, i) + feat_off;
                    if (YTMA) ys[(col0 + i) * TC_BM + fl] = y;
                    if (n < p.M) {
                        if (!YTMA) p.y[(size_t)n * p.N + f] = y;
                        if (kv) {
                            if (p.kv.kv_f32) ((float*)p.kv.pool)[e] = y;
                            else ((__half*)p.kv.pool)[e] = __float2half_rn(y);
                        }
                    }
                }
            } else if (EPI == EPI_RESID) {
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    const int n = nb + i;
                    const float a = acc[i];
                    if (n < p.M) {
                        const float r = p.resid[(size_t)n * p.N + f];
                        const float y = __fadd_rn(__fadd_rn(r, a), bias);
                        if (YTMA) ys[(col0 + i) * TC_BM + fl] = y;
                        else p.y[(size_t)n * p.N + f] = y;
                    }
                }
            } else {   // relu(acc + bias); the warp's 32 features are one Q8_0 block of each token
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    const int n = nb + i;
                    const float a = acc[i];
                    float h = __fadd_rn(a, bias);
                    h = h > 0.0f ? h : 0.0f;
                    float amax = h;
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
                    float dsc, id;
                    q8_scale(amax, dsc, id);
                    if (n < p.M) {
                        p.yq[(size_t)n * p.N + f] = q8_val(h, id);
                        if (lane == 0) p.yd[(size_t)n * (p.N / QK) + f / QK] = f2h(dsc);
                    }
                }
            }
            if (YTMA) {   // the staged tile, visible to the bulk copy, goes to the store warp
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                bar_arrive(ystaged);
            }
        }
        if (!ok) {
            if (p.err) atomicExch(p.err, 1);
            *abort_flag = 1;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
    }
}

// The activation side of k_gemm_q8_tc, one launch: X's Q8_0 integers as fp16 [M][K]; the activation
// scales transposed to f32 [KB][ld] and the weight scales to f32 [KB][N] (block-major, so one TMA box
// brings a tile's 128 scales of every block).
__global__ void __launch_bounds__(256) k_tc_prep(const int8_t* __restrict__ q, __half* __restrict__ x16, size_t n16,
                                                 const uint16_t* __restrict__ xd, int M, int KB, float* __restrict__ dxT,
                                                 int ld, const uint16_t* __restrict__ wd, int N,
                                                 float* __restrict__ dwT) {
    griddep_wait();
    griddep_launch();
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n16; i += stride) {
        const int4 v = ((const int4*)q)[i];
        const int w[4] = {v.x, v.y, v.z, v.w};
        uint4 o[2];
        uint32_t* ow = (uint32_t*)o;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int a = (int)(int8_t)(w[k >> 1] >> (16 * (k & 1)));
            const int b = (int)(int8_t)(w[k >> 1] >> (16 * (k & 1) + 8));
            ow[k] = (uint32_t)__half_as_ushort(__int2half_rn(a)) | ((uint32_t)__half_as_ushort(__int2half_rn(b)) << 16);
        }
        ((uint4*)x16)[2 * i] = o[0];
        ((uint4*)x16)[2 * i + 1] = o[1];
    }
    const size_t nx = (size_t)KB * M, nw = (size_t)KB * N;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < nx + nw; i += stride) {
        if (i < nx) {
            const int kb = (int)(i / M), m = (int)(i - (size_t)kb * M);
            dxT[(size_t)kb * ld + m] = h2f(xd[(size_t)m * KB + kb]);
        } else {
            const size_t k = i - nx;
            const int kb = (int)(k / N), n = (int)(k - (size_t)kb * N);
            dwT[k] = h2f(wd[(size_t)n * KB + kb]);
        }
    }
}

// ---------------------------------------------------------------- host side
// f16 [rows][K] row-major, tile 64 (K) x 128 rows, 128-byte swizzle; rows past `rows` read as zero.
bool make_map_f16(CUtensorMap* m, const __half* base, int rows, int K) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)TC_BK, 128u};
    const cuuint32_t estr[2] = {1u, 1u};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void*)base, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
// f32 [KB][ld] block-major scales, `cols` valid per row, tile 128 columns x KB rows, no swizzle; columns
// past `cols` read as zero.
bool make_map_scales(CUtensorMap* m, const float* base, int cols, int ld, int KB) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)KB};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
    const cuuint32_t box[2] = {128u, (cuuint32_t)KB};
    const cuuint32_t estr[2] = {1u, 1u};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// f32 [rows][N] output, tile 128 columns x 128 rows, no swizzle (bulk stores clip rows past `rows`).
bool make_map_out(CUtensorMap* m, const float* base, int rows, int N) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)N * 4};
    const cuuint32_t box[2] = {128u, 128u};
    const cuuint32_t estr[2] = {1u, 1u};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

constexpr size_t align128(size_t b) { return (b + 127) & ~(size_t)127; }
int scale_ld(int M) { return (M + 31) & ~31; }

// The scratch carve-up: x16 [M][K] fp16, dxT [KB][scale_ld(M)] f32, dwT [KB][N] f32.
struct TcScratch {
    __half* x16;
    float* dxT;
    float* dwT;
};
TcScratch carve(const GemmQ8Params& p) {
    const int KB = p.K / QK;
    uint8_t* b = (uint8_t*)p.tc_scratch;
    TcScratch s;
    s.x16 = (__half*)b;
    s.dxT = (float*)(b + align128((size_t)p.M * p.K * 2));
    s.dwT = (float*)((uint8_t*)s.dxT + align128((size_t)KB * scale_ld(p.M) * 4));
    return s;
}

std::atomic<int> g_num_sms{0};   // SMs of the device (148 on B200): the persistent grid size

}  // namespace

size_t tc_scratch_bytes(int M, int N, int K) {
    const int KB = K / QK;
    return align128((size_t)M * K * 2) + align128((size_t)KB * scale_ld(M) * 4) + align128((size_t)KB * N * 4);
}

bool gemm_tc_usable(const GemmQ8Params& p) {
    return p.w16 && p.tc_scratch && p.N % TC_BM == 0 && p.K % TC_BK == 0 && p.K / QK <= TC_MAX_KB &&
           p.tc_scratch_n >= tc_scratch_bytes(p.M, p.N, p.K) && p.n_store == 0 && p.ldy == 0 &&
           (p.kv.pool == nullptr || p.kv.tok_pos != nullptr) && ((uintptr_t)p.tc_scratch & 127) == 0 &&
           ((uintptr_t)p.y & 15) == 0 &&
           ((uintptr_t)p.xq & 15) == 0 && ((uintptr_t)p.w16 & 15) == 0 && encode_fn() != nullptr;
}

cudaError_t gemm_tc_init_device() {
    cudaError_t e;
    int dev = 0;
    if ((e = cudaGetDevice(&dev))) return e;
    int sms = 0;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev))) return e;
    g_num_sms.store(sms, std::memory_order_relaxed);
#define GSVCU_TC_SMEM(EPI_, KBM_)                                                                                \
    if ((e = cudaFuncSetAttribute(k_gemm_q8_tc<EPI_, KBM_>, cudaFuncAttributeMaxDynamicSharedMemorySize,          \
                                  (int)TcLayout<KBM_>::SMEM)))                                                   \
        return e;
    GSVCU_TC_SMEM(EPI_BIAS, 16) GSVCU_TC_SMEM(EPI_RESID, 16) GSVCU_TC_SMEM(EPI_RELU_Q8, 16)
    GSVCU_TC_SMEM(EPI_BIAS, 64) GSVCU_TC_SMEM(EPI_RESID, 64) GSVCU_TC_SMEM(EPI_RELU_Q8, 64)
#undef GSVCU_TC_SMEM
    return cudaSuccess;
}

bool launch_gemm_q8_tc(const GemmQ8Params& p, int epi, cudaStream_t s) {
    const int KB = p.K / QK, ld = scale_ld(p.M);
    const TcScratch sc = carve(p);
    TcMaps maps;
    if (!make_map_f16(&maps.w, p.w16, p.N, p.K) || !make_map_f16(&maps.x, sc.x16, p.M, p.K) ||
        !make_map_scales(&maps.dw, sc.dwT, p.N, p.N, KB) || !make_map_scales(&maps.dx, sc.dxT, p.M, ld, KB))
        return false;
    // the output map is used by the staged variants only (K <= 512 and EPI_BIAS / EPI_RESID)
    if (KB <= 16 && epi != EPI_RELU_Q8 && !make_map_out(&maps.y, p.y, p.M, p.N)) return false;
    {   // the activation side: fp16 integers and both transposed scale planes
        const size_t n16 = (size_t)p.M * p.K / 16, work = n16 + (size_t)KB * ((size_t)p.M + p.N);
        const int blocks = (int)std::min<size_t>((work + 255) / 256, (size_t)std::max(g_num_sms.load(), 1) * 8);
        launch_pdl(k_tc_prep, dim3(std::max(blocks, 1)), dim3(256), 0, s, p.xq, sc.x16, n16, p.xd, p.M, KB, sc.dxT,
                   ld, p.wd, p.N, sc.dwT);
    }
    const int ntiles = (p.N / TC_BM) * ((p.M + TC_BN - 1) / TC_BN);
    const dim3 grid(std::max(1, std::min(ntiles, std::max(g_num_sms.load(), 1))));
#define GSVCU_TC_LAUNCH(KBM_)                                                                                          \
    switch (epi) {                                                                                                 \
        case EPI_BIAS: launch_pdl(k_gemm_q8_tc<EPI_BIAS, KBM_>, grid, dim3(TC_THREADS), TcLayout<KBM_>::SMEM, s, maps, p); break; \
        case EPI_RESID: launch_pdl(k_gemm_q8_tc<EPI_RESID, KBM_>, grid, dim3(TC_THREADS), TcLayout<KBM_>::SMEM, s, maps, p); break; \
        default: launch_pdl(k_gemm_q8_tc<EPI_RELU_Q8, KBM_>, grid, dim3(TC_THREADS), TcLayout<KBM_>::SMEM, s, maps, p); break; \
    }
    if (KB <= 16) { GSVCU_TC_LAUNCH(16) } else { GSVCU_TC_LAUNCH(64) }
#undef GSVCU_TC_LAUNCH
    return true;
}

}  // namespace gsvcu
