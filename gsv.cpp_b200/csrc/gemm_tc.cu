// gemm_tc.cu -- prefill Q8_0 GEMM on the 5th-generation tensor cores: TMA tile loads, tcgen05.mma with
// the accumulator in tensor memory (TMEM), a warp-specialised pipeline.
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
// CTA tile: 128 features (UMMA M, TMEM lanes) x 128 tokens (UMMA N, TMEM columns). 10 warps:
//   warp 0      TMA producer: 64-value K slices of W (features) and X (tokens), SWIZZLE_128B, 4 stages
//   warp 1      TMEM allocator (512 columns = 4 accumulator buffers) and the MMA issuer: per Q8_0 block
//               two tcgen05.mma (K = 16 each) into buffer kb % 4, committed to that buffer's barrier
//   warps 2..9  epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 (its 32 features), columns
//               64 ((w - 2) / 4) .. +63 (64 tokens); per block two tcgen05.ld of its 64 sums, then
//               acc[t] = fma(sum, d_w * d_x[t], acc[t]) in registers, two tokens per packed f32x2
//               instruction (each lane rounded as the scalar operation); finally the fused epilogue
//               (bias, residual, ReLU + Q8_0 quantization, K/V page store) with coalesced stores.
// Every mbarrier wait is bounded; a wait that gives up sets the error word, the others stop at their
// next wait, in-flight copies and MMAs are waited for (bounded) and the TMEM is freed before exit.
// No cluster launch and no multicast: each CTA loads its own tiles from this GPU's memory.
#include <cuda.h>

#include <cstdio>
#include <mutex>

#include "kernels.h"

namespace gsvcu {
namespace {

constexpr int TC_BM = 128;          // features per tile
constexpr int TC_BN = 128;          // tokens per tile
constexpr int TC_BK = 64;           // K values per stage (two Q8_0 blocks; one 128-byte swizzle row)
constexpr int TC_STAGES = 4;
constexpr int TC_TBUF = 4;          // TMEM accumulator buffers, one Q8_0 block each
constexpr int TC_EPI_WARPS = 8;     // 2 per TMEM lane quarter, 64 token columns each
constexpr int TC_THREADS = 32 * (2 + TC_EPI_WARPS);
constexpr int TC_MAX_KB = 64;       // K <= 2048
constexpr int STAGE_W = TC_BM * TC_BK * 2;
constexpr int STAGE_X = TC_BN * TC_BK * 2;
constexpr uint32_t TC_POLL_LIMIT = 1u << 22;
// shared memory: stages (1024-byte aligned for the 128-byte swizzle), then the scales as f32
// [block][128] (d_w of the tile's features, d_x of its tokens), then the barriers and the TMEM address.
constexpr size_t OFF_W = 0;
constexpr size_t OFF_X = OFF_W + (size_t)TC_STAGES * STAGE_W;
constexpr size_t OFF_DW = OFF_X + (size_t)TC_STAGES * STAGE_X;
constexpr size_t OFF_DX = OFF_DW + (size_t)TC_MAX_KB * TC_BM * 4;
constexpr size_t OFF_BAR = OFF_DX + (size_t)TC_MAX_KB * TC_BN * 4;
constexpr int NBAR = 2 * TC_STAGES + 2 * TC_TBUF + 1;   // full, empty, tfull, tempty, done
constexpr size_t OFF_MISC = OFF_BAR + NBAR * 8;
constexpr size_t TC_SMEM = OFF_MISC + 16 + 1024;        // + slack to align the base to 1024
constexpr int YS_LD = TC_BM + 1;                         // epilogue staging: [128 tokens][129] floats
static_assert((size_t)TC_BN * YS_LD * 4 <= OFF_DW, "epilogue staging fits in the operand stages");

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void bar_init(uint32_t b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(b), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_expect_tx(uint32_t b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(b), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint32_t b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(b) : "memory");
}
__device__ __forceinline__ bool bar_try(uint32_t b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(b), "r"(parity)
        : "memory");
    return ok != 0;
}
// Non-blocking test of the phase of `parity`.
__device__ __forceinline__ bool bar_test(uint32_t b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(b), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the phase of `parity`: the non-blocking test first (the phase is often complete
// already), then polls that may suspend the thread until it completes; false when the poll limit ran
// out or another role aborted.
__device__ __forceinline__ bool bar_wait(uint32_t b, uint32_t parity, volatile int* abort_flag) {
    if (bar_test(b, parity)) return true;
    for (uint32_t it = 0; it < TC_POLL_LIMIT; it++) {
        if (bar_try(b, parity)) return true;
        if (*abort_flag) return false;
    }
    return false;
}

// The same for a whole warp, with a warp-uniform result (the epilogue warps go on to .sync.aligned
// TMEM loads): a completed phase stays complete until the next one, which needs this warp's own
// arrival first, so after lane 0 saw it every lane may use the buffer.
// Lane 0 polls (one barrier access per poll for the warp) and broadcasts the outcome.
__device__ __forceinline__ bool bar_wait_warp(uint32_t b, uint32_t parity, volatile int* abort_flag) {
    int ok = 0;
    if ((threadIdx.x & 31) == 0) ok = bar_wait(b, parity, abort_flag);
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// 2D TMA tile load (no multicast) completing on an mbarrier; c0 = K offset (elements), c1 = row.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(dst), "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(bar)
        : "memory");
}

// UMMA shared-memory descriptor of a K-major operand tile in the canonical SWIZZLE_128B layout (rows of
// 128 bytes, 8-row atoms of 1024 bytes): start address >> 4, leading offset 1 (unused for swizzled
// K-major), stride offset 1024 >> 4, descriptor version 1, layout type 2 (128-byte swizzle).
__device__ __forceinline__ uint64_t umma_desc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::f16: D f32 (bits 4-5 = 1), A and B f16 (0), both K-major, N >> 3 at bit
// 17, M >> 4 at bit 24.
constexpr uint32_t TC_IDESC = (1u << 4) | ((uint32_t)(TC_BN >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(TC_IDESC), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive TMEM columns of this warp's 32 lanes: lane l gets row (lane base + l), columns c..c+31.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
        "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }


struct TcMaps {
    CUtensorMap w;   // f16 [N][K] weight values
    CUtensorMap x;   // f16 [M][K] activation values
};

template <int EPI>
__global__ void __launch_bounds__(TC_THREADS, 1) k_gemm_q8_tc(const __grid_constant__ TcMaps maps, const GemmQ8Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int f0 = blockIdx.x * TC_BM, t0 = blockIdx.y * TC_BN;
    const int K = p.K, KB = K / QK, nstage = K / TC_BK;
    float* dws = (float*)(sm + OFF_DW);   // [KB][128 features]
    float* dxs = (float*)(sm + OFF_DX);   // [KB][128 tokens]
    uint64_t* bars = (uint64_t*)(sm + OFF_BAR);
    const uint32_t bar0 = su32(bars);
    auto full = [&](int s) { return bar0 + 8u * s; };
    auto empty = [&](int s) { return bar0 + 8u * (TC_STAGES + s); };
    auto tfull = [&](int j) { return bar0 + 8u * (2 * TC_STAGES + j); };
    auto tempty = [&](int j) { return bar0 + 8u * (2 * TC_STAGES + TC_TBUF + j); };
    const uint32_t done_bar = bar0 + 8u * (2 * TC_STAGES + 2 * TC_TBUF);
    uint32_t* tmem_slot = (uint32_t*)(sm + OFF_MISC);
    volatile int* abort_flag = (volatile int*)(sm + OFF_MISC + 4);

    if (tid == 0) {
        for (int s = 0; s < TC_STAGES; s++) { bar_init(full(s), 1); bar_init(empty(s), 1); }
        for (int j = 0; j < TC_TBUF; j++) { bar_init(tfull(j), 1); bar_init(tempty(j), TC_EPI_WARPS); }
        bar_init(done_bar, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&maps.w) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&maps.x) : "memory");
    }
    if (warp == 1) {   // TMEM: 512 columns, address written to shared memory
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                     "r"(512)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // The tile's scales are 128 consecutive rows of KB fp16 each: one 16-byte load per 8 values, all
    // issued before any is used, written to shared memory as f32 [block][row]. Weight scales are
    // constant, so they are staged before the wait for the previous kernel.
    auto stage_scales = [&](const uint16_t* src, int rows_valid, float* dst) {
        const int nvec = KB * 128 / 8;   // <= 1024
        constexpr int ROUNDS = (TC_MAX_KB * 128 / 8 + TC_THREADS - 1) / TC_THREADS;
        uint4 v[ROUNDS];
#pragma unroll
        for (int r = 0; r < ROUNDS; r++) {
            const int i = tid + r * TC_THREADS;
            v[r] = make_uint4(0u, 0u, 0u, 0u);
            if (i < nvec && (i * 8) / KB < rows_valid) v[r] = *(const uint4*)(src + (size_t)i * 8);
        }
#pragma unroll
        for (int r = 0; r < ROUNDS; r++) {
            const int i = tid + r * TC_THREADS;
            if (i >= nvec) continue;
            const uint32_t w[4] = {v[r].x, v[r].y, v[r].z, v[r].w};
#pragma unroll
            for (int e = 0; e < 8; e++) {
                const int idx = i * 8 + e, row = idx / KB, b = idx - row * KB;
                dst[b * 128 + row] = h2f((uint16_t)(w[e >> 1] >> (16 * (e & 1))));
            }
        }
    };
    stage_scales(p.wd + (size_t)f0 * KB, 128, dws);
    griddep_wait();
    griddep_launch();
    stage_scales(p.xd + (size_t)t0 * KB, p.M - t0, dxs);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            int issued = 0;
            for (int ks = 0; ks < nstage; ks++) {
                const int s = ks % TC_STAGES;
                const uint32_t ph = (uint32_t)(ks / TC_STAGES) & 1u;
                if (!bar_wait(empty(s), ph ^ 1u, abort_flag)) {
                    if (p.err) atomicExch(p.err, 1);
                    *abort_flag = 1;
                    break;
                }
                bar_expect_tx(full(s), STAGE_W + STAGE_X);
                tma_load_2d(su32(sm + OFF_W + (size_t)s * STAGE_W), &maps.w, ks * TC_BK, f0, full(s));
                tma_load_2d(su32(sm + OFF_X + (size_t)s * STAGE_X), &maps.x, ks * TC_BK, t0, full(s));
                issued++;
            }
            // every copy this thread issued has landed before the CTA may exit (bounded)
            for (int ks = issued - 1; ks >= 0 && ks >= issued - TC_STAGES; ks--)
                for (uint32_t it = 0; it < TC_POLL_LIMIT; it++)
                    if (bar_try(full(ks % TC_STAGES), (uint32_t)(ks / TC_STAGES) & 1u)) break;
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            int kb = 0;
            bool ok = true;
            for (int ks = 0; ks < nstage && ok; ks++) {
                const int s = ks % TC_STAGES;
                if (!bar_wait(full(s), (uint32_t)(ks / TC_STAGES) & 1u, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint32_t wa = su32(sm + OFF_W + (size_t)s * STAGE_W), xa = su32(sm + OFF_X + (size_t)s * STAGE_X);
                for (int half = 0; half < 2; half++, kb++) {
                    const int j = kb % TC_TBUF;
                    if (!bar_wait(tempty(j), ((uint32_t)(kb / TC_TBUF) & 1u) ^ 1u, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t d = tmem + (uint32_t)(j * TC_BN);
#pragma unroll
                    for (int kk = 0; kk < 2; kk++) {
                        const uint32_t off = (uint32_t)(half * 64 + kk * 32);   // bytes along K inside the row
                        umma_f16(d, umma_desc(wa + off), umma_desc(xa + off), (uint32_t)kk);
                    }
                    umma_commit(tfull(j));
                }
                umma_commit(empty(s));
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
    } else {
        // ---------------------------------------------------------------- epilogue warps
        const int q = warp & 3;                   // TMEM lane quarter this warp may access
        const int col0 = ((warp - 2) >> 2) * 64;  // its 64 token columns
        const int fl = q * 32 + lane;             // feature (TMEM lane) of this thread
        const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)col0;
        uint64_t acc2[32];                        // tokens (2i, 2i + 1) as a packed pair
#pragma unroll
        for (int i = 0; i < 32; i++) acc2[i] = 0ull;
        bool ok = true;
        uint32_t r[64];
        for (int kb = 0; kb < KB; kb++) {
            const int j = kb % TC_TBUF;
            if (!bar_wait_warp(tfull(j), (uint32_t)(kb / TC_TBUF) & 1u, abort_flag)) {
                ok = false;
                break;
            }
            tc_fence_after();
            tmem_ld32(tbase + (uint32_t)(j * TC_BN), *(uint32_t(*)[32])&r[0]);
            tmem_ld32(tbase + (uint32_t)(j * TC_BN + 32), *(uint32_t(*)[32])&r[32]);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive(tempty(j));   // the sums are in registers: the buffer is free
            const float dw = dws[kb * TC_BM + fl];
            const uint64_t dw2 = f2pack(dw, dw);
            const float4* dx4 = (const float4*)(dxs + kb * TC_BN + col0);
#pragma unroll
            for (int c = 0; c < 16; c++) {   // acc = fma(sum, d_w * d_x, acc), two tokens per instruction
                const float4 d = dx4[c];
                const uint64_t p0 = fmul2(dw2, f2pack(d.x, d.y)), p1 = fmul2(dw2, f2pack(d.z, d.w));
                acc2[2 * c] = ffma2(f2pack(__uint_as_float(r[4 * c]), __uint_as_float(r[4 * c + 1])), p0, acc2[2 * c]);
                acc2[2 * c + 1] =
                    ffma2(f2pack(__uint_as_float(r[4 * c + 2]), __uint_as_float(r[4 * c + 3])), p1, acc2[2 * c + 1]);
            }
        }
        if (!ok) {
            if (p.err) atomicExch(p.err, 1);
            *abort_flag = 1;
        } else {
            // The accumulators go through shared memory (the operand stages are idle now: every copy
            // landed and every MMA that read them completed), so the epilogue below is a short loop
            // instead of 64 unrolled copies, which would stream from the instruction cache once each.
            float* ys = (float*)(sm + OFF_W) + (size_t)col0 * YS_LD;   // this warp's 64 token rows
#pragma unroll
            for (int i = 0; i < 32; i++) {
                ys[(2 * i) * YS_LD + fl] = __uint_as_float((uint32_t)acc2[i]);
                ys[(2 * i + 1) * YS_LD + fl] = __uint_as_float((uint32_t)(acc2[i] >> 32));
            }
            __syncwarp();
            const int f = f0 + fl;
            const float bias = p.bias ? p.bias[f] : 0.0f;
            const int tend = min(64, p.M - (t0 + col0));
#pragma unroll 2
            for (int t = 0; t < tend; t++) {
                const int n = t0 + col0 + t;
                const float a = ys[t * YS_LD + fl];
                if (EPI == EPI_BIAS) {
                    const float y = __fadd_rn(a, bias);
                    p.y[(size_t)n * p.N + f] = y;
                    if (p.kv.pool && f >= D) {   // K/V columns of a QKV GEMM: into the row's KV page
                        const int slot = p.kv.tok_slot[n], pos = p.kv.tok_pos[n];
                        const int kvsel = (f - D) >> 9, fh = (f - D) & (D - 1);
                        const int h = fh >> 5, dd = fh & 31;
                        const int page = p.kv.block_table[(size_t)slot * p.kv.max_pages + pos / PAGE];
                        const size_t e = ((((size_t)page * p.kv.n_layer + p.kv.layer) * 2 + kvsel) * NH + h) *
                                             (PAGE * HD) + (size_t)(pos % PAGE) * HD + dd;
                        if (p.kv.kv_f32) ((float*)p.kv.pool)[e] = y;
                        else ((__half*)p.kv.pool)[e] = __float2half_rn(y);
                    }
                } else if (EPI == EPI_RESID) {
                    const float r = p.resid[(size_t)n * p.N + f];
                    p.y[(size_t)n * p.N + f] = __fadd_rn(__fadd_rn(r, a), bias);
                } else {   // relu(acc + bias); the warp's 32 features are one Q8_0 block of row n
                    float h = __fadd_rn(a, bias);
                    h = h > 0.0f ? h : 0.0f;
                    float amax = fabsf(h);
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
                    float dsc, id;
                    q8_scale(amax, dsc, id);
                    p.yq[(size_t)n * p.N + f] = q8_val(h, id);
                    if (lane == 0) p.yd[(size_t)n * (p.N / QK) + f / QK] = f2h(dsc);
                }
            }
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

// Q8_0 integer planes -> the same integers as fp16 (the tensor-core operand of k_gemm_q8_tc).
__global__ void __launch_bounds__(256) k_q8_to_f16(const int8_t* __restrict__ q, __half* __restrict__ out, size_t n16) {
    griddep_wait();
    griddep_launch();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n16; i += (size_t)gridDim.x * blockDim.x) {
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
        ((uint4*)out)[2 * i] = o[0];
        ((uint4*)out)[2 * i + 1] = o[1];
    }
}

// ---------------------------------------------------------------- host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
std::once_flag g_encode_once;

EncodeTiledFn encode_fn() {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = (EncodeTiledFn)fn;
        else
            cudaGetLastError();
    });
    return g_encode;
}

// f16 [rows][K] row-major, tile 64 (K) x 128 rows, 128-byte swizzle; rows past `rows` read as zero.
bool make_map(CUtensorMap* m, const __half* base, int rows, int K) {
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

}  // namespace

bool gemm_tc_usable(const GemmQ8Params& p) {
    return p.x16 && p.w16 && p.N % TC_BM == 0 && p.K % TC_BK == 0 && p.K / QK <= TC_MAX_KB && p.n_store == 0 &&
           p.ldy == 0 && (p.kv.pool == nullptr || p.kv.tok_pos != nullptr) && ((uintptr_t)p.x16 & 15) == 0 &&
           ((uintptr_t)p.w16 & 15) == 0 && encode_fn() != nullptr;
}

cudaError_t gemm_tc_init_device() {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(k_gemm_q8_tc<EPI_BIAS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM)))
        return e;
    if ((e = cudaFuncSetAttribute(k_gemm_q8_tc<EPI_RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM)))
        return e;
    return cudaFuncSetAttribute(k_gemm_q8_tc<EPI_RELU_Q8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM);
}

bool launch_gemm_q8_tc(const GemmQ8Params& p, int epi, cudaStream_t s) {
    TcMaps maps;
    if (!make_map(&maps.w, p.w16, p.N, p.K) || !make_map(&maps.x, p.x16, p.M, p.K)) return false;
    dim3 grid(p.N / TC_BM, (p.M + TC_BN - 1) / TC_BN);
    switch (epi) {
        case EPI_BIAS: launch_pdl(k_gemm_q8_tc<EPI_BIAS>, grid, dim3(TC_THREADS), TC_SMEM, s, maps, p); break;
        case EPI_RESID: launch_pdl(k_gemm_q8_tc<EPI_RESID>, grid, dim3(TC_THREADS), TC_SMEM, s, maps, p); break;
        default: launch_pdl(k_gemm_q8_tc<EPI_RELU_Q8>, grid, dim3(TC_THREADS), TC_SMEM, s, maps, p); break;
    }
    return true;
}

void launch_q8_to_f16(const int8_t* q, __half* out, size_t n, cudaStream_t s) {
    const size_t n16 = n / 16;
    const int blocks = (int)std::min<size_t>((n16 + 255) / 256, 148 * 8);
    launch_pdl(k_q8_to_f16, dim3(std::max(blocks, 1)), dim3(256), 0, s, q, out, n16);
}

}  // namespace gsvcu
