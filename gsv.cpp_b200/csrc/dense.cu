// dense.cu -- the decode step's per-layer tail fused on a 16-CTA thread-block cluster.
//
// After the decode-attention kernel has left one partial result per (slot, head, KV page), one
// cluster of 16 CTAs carries 16 slots through the rest of the layer and the next layer's QKV
// projection (the reference's per-layer graph, src/gsv_ar.cpp:402-467):
//   0  merge of the attention pages, head j = cluster rank j        -> Q8_0 block j of each row
//   1  out-projection, output columns [32j, 32j+32), + residual x + bias, LayerNorm row statistics
//   2  LayerNorm 1 on the CTA's 32 columns                           -> Q8_0 block j of n1
//   3  FFN1, columns [128j, 128j+128), bias + ReLU                   -> Q8_0 blocks 4j..4j+3 of h
//   4  FFN2, columns [32j, 32j+32), + residual n1 + bias, LayerNorm row statistics
//   5  LayerNorm 2                                                   -> x (global) and its Q8_0 block j
//   6  next layer's QKV: q, k, v columns of head j                   -> q (global), K/V page rows
// Every CTA keeps full copies of the Q8_0 rows a GEMM reads, block-major; each CTA computes one
// 32-column block of all 16 rows, stages it, and copies it into all 16 CTAs' shared memory
// (distributed shared memory) with one bulk copy per CTA, counted on the receivers' mbarriers.
// LayerNorm's double row sums go to every CTA as 16-byte remote stores counted the same way.
//
// Arithmetic is that of the unfused kernels (gemm_q8.cu, misc.cu, attention.cu), operation for
// operation: each Q8_0 output is one warp's sequential float chain over the K blocks in order,
// acc = fma((float)isum_b, d_w * d_x, acc), from exact int32 block sums (mma.m16n8k32 s8 with a zero
// accumulator); LayerNorm sums are double; the page merge follows the same page order.
//
// Weights: each CTA's slices of the out, FFN1 and FFN2 matrices (~150 KB per layer) are copied into
// shared memory by TMA bulk copies issued first thing, before griddep_wait (a 230 KB CTA becomes
// resident only once its SM has no attention CTA left, so the copies overlap the prologue and the page
// merge); the next layer's QKV slices follow once FFN1 has consumed the out and FFN1 slices.
#include <cooperative_groups.h>

#include "kernels.h"

namespace cg = cooperative_groups;

namespace gsvcu {

namespace {

constexpr int DR = 16;       // slots (rows) per cluster: two n = 8 tiles of mma.m16n8k32
constexpr int DC = 16;       // CTAs per cluster
constexpr int DT = 512;      // threads per CTA: one warp per row in the row-wise phases
constexpr int NW = DT / 32;  // warps
constexpr int KB1 = D / QK;  // K blocks of a 512-wide input (16)
constexpr int KB2 = FF / QK; // K blocks of a 2048-wide input (64)
// One exchanged Q8_0 block of all DR rows: quants [DR][32], then f32 scales [DR]. Within a row,
// column c sits at byte qpos(c), which places the 8 quants lane (g, t) of mma.m16n8k32 reads as its
// B fragment (columns 4t..4t+3 and 16+4t..16+4t+3) side by side.
constexpr int BLK = DR * 32 + DR * 4;

// shared-memory layout (bytes); activation rows are block-major: [KB][BLK]
constexpr int SM_W_OUT = 0;                        // out rows [32j, 32j+32): 2 row groups x 16 K blocks
constexpr int SM_D_OUT = SM_W_OUT + 2 * KB1 * 512; // [32][16] fp16
constexpr int SM_W_F1 = SM_D_OUT + 32 * KB1 * 2;   // ffn1 rows [128j, +128): 8 row groups
constexpr int SM_D_F1 = SM_W_F1 + 8 * KB1 * 512;   // [128][16]
constexpr int SM_W_F2 = SM_D_F1 + 128 * KB1 * 2;   // ffn2 rows [32j, +32): 2 row groups x 64 K blocks
constexpr int SM_D_F2 = SM_W_F2 + 2 * KB2 * 512;   // [32][64]
constexpr int SM_W_QKV = 0;                        // next layer's q|k|v rows of head j (reuses out + ffn1)
constexpr int SM_D_QKV = SM_W_QKV + 6 * KB1 * 512; // [96][16]
constexpr int ROWS1_BYTES = KB1 * BLK;
constexpr int HROWS_BYTES = KB2 * BLK;
constexpr int SM_AROWS = SM_D_F2 + 32 * KB2 * 2;   // attention output rows (Q8_0), all 16 blocks
constexpr int SM_N1ROWS = SM_AROWS + ROWS1_BYTES;  // n1 rows (Q8_0); later the x rows of the next QKV
constexpr int SM_XROWS = SM_N1ROWS;
constexpr int SM_HROWS = SM_N1ROWS + ROWS1_BYTES;  // h rows (Q8_0), 2048 wide
constexpr int SM_LNP1 = SM_HROWS + HROWS_BYTES;    // [16 src][DR rows] {sum, sum of squares} doubles
constexpr int SM_LNP2 = SM_LNP1 + DC * DR * 16;
constexpr int SM_XOWN = SM_LNP2 + DC * DR * 16;    // [DR][32] f32: this CTA's columns of x (phases 0-1)
constexpr int SM_N1OWN = SM_XOWN;                  // [DR][32] f32: this CTA's columns of n1 (phases 2-4)
constexpr int SM_PRE = SM_N1OWN + DR * 32 * 4;     // [DR][32] f32: pre-LayerNorm sums
constexpr int SM_STG = SM_PRE + DR * 32 * 4;       // staged blocks, one region per exchange (never reused)
constexpr int STG_ATT = 0, STG_N1 = BLK, STG_X = 2 * BLK, STG_H = 3 * BLK, STG_BYTES = 7 * BLK;
constexpr int SM_PAR = SM_STG + STG_BYTES;         // this CTA's bias / LayerNorm parameters (f32)
constexpr int P_BOUT = 0, P_BF1 = 32, P_BF2 = 160, P_N1W = 192, P_N1B = 224, P_N2W = 256, P_N2B = 288, P_BQKV = 320,
              P_COUNT = 416;
constexpr int SM_ROWMETA = SM_PAR + P_COUNT * 4;   // per row: pages to merge (0: not decoding), KV page, KV pos
constexpr int SM_BARS = SM_ROWMETA + DR * 3 * 4;   // 4 weight barriers + 6 exchange barriers
constexpr int SMEM_DENSE = SM_BARS + 11 * 8;
// alias: FFN1's f32 outputs in the attention rows
static_assert(NW == DR, "one warp per row");
static_assert(DR * 128 * 4 <= ROWS1_BYTES, "ffn1 staging");
static_assert(SM_D_QKV + 96 * KB1 * 2 <= SM_W_F2, "qkv weights reuse out + ffn1");
static_assert(SMEM_DENSE <= 232448, "shared memory");
static_assert(SM_PAR % 16 == 0 && SM_XOWN % 16 == 0 && SM_ROWMETA % 4 == 0, "alignment of TMA destinations");
static_assert(SM_AROWS % 16 == 0 && SM_N1ROWS % 16 == 0 && SM_HROWS % 16 == 0 && SM_D_F1 % 16 == 0 &&
                  SM_D_F2 % 16 == 0 && SM_D_QKV % 16 == 0 && SM_LNP1 % 16 == 0 && SM_LNP2 % 16 == 0 &&
                  SM_STG % 16 == 0 && BLK % 16 == 0 && SM_BARS % 8 == 0,
              "alignment");
// bytes each CTA receives per exchange (every CTA sends to all 16, itself included)
constexpr uint32_t EX_BLOCK = DC * BLK;            // one block of all rows per sender
constexpr uint32_t EX_STATS = DC * DR * 16;        // one {sum, sum of squares} per (sender, row)
enum { BW_OUT = 0, BW_F1, BW_F2, BW_QKV, BX_ATT, BX_LN1, BX_N1, BX_H, BX_LN2, BX_X, BW_PAR };

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void d_mbar_init(uint32_t bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void d_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// Bulk global -> shared copy; weights and parameters are reused every step: kept in L2 (evict-last).
__device__ __forceinline__ void d_bulk(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(pol)
        : "memory");
}
// Bounded wait on phase 0 of an mbarrier by a whole warp; false if the limit was reached.
__device__ __forceinline__ bool d_wait(uint32_t bar) {
    uint32_t it = 0, ok = 0;
    for (;;) {
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(bar)
            : "memory");
        if (ok || ++it == (1u << 22)) break;
    }
    return __all_sync(0xffffffffu, ok != 0);
}
// Address of a local shared-memory location in the shared window of cluster CTA `rank`.
__device__ __forceinline__ uint32_t d_mapa(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}
// Remote stores into a peer's shared memory that count their bytes on the peer's mbarrier.
__device__ __forceinline__ void d_st_async16(uint32_t addr, uint4 v, uint32_t bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(addr),
                 "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ void mma_s8(int (&c)[4], const uint4& a, uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};\n"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

// fp16 scale j (0..7) of 8 consecutive ones loaded as a uint4
__device__ __forceinline__ float h2f_pick(const uint4& s, int j) {
    const uint32_t w = (j >> 1) == 0 ? s.x : (j >> 1) == 1 ? s.y : (j >> 1) == 2 ? s.z : s.w;
    return h2f((uint16_t)((j & 1) ? (w >> 16) : (w & 0xffffu)));
}

// One warp: row group lr (16 features) of a weight slice in shared memory against row tile rt (rows
// 8rt..8rt+7) of the block-major rows X, K blocks [kb0, kb0 + NK) in order, continuing acc. Thread
// (g, t) holds features 16lr+g, 16lr+g+8 x rows 8rt+2t, 8rt+2t+1 in acc[0..3].
template <int KB, int NK>
__device__ __forceinline__ void rg_chain(const uint8_t* W, const uint16_t* DW, int lr, const uint8_t* X, int rt,
                                         int kb0, float (&acc)[4]) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int fa = lr * 16 + g, fb = fa + 8;
    const uint4* wp = (const uint4*)W + (size_t)lr * KB * 32 + lane;
    const uint8_t* xq = X + (rt * 8 + g) * 32 + t * 8;        // B fragment of block kb at xq + kb * BLK
    const uint8_t* xd = X + DR * 32 + (rt * 8 + 2 * t) * 4;   // scales of rows 8rt+2t, +1 at xd + kb * BLK
    constexpr int KC = 8;   // K blocks whose MMAs are issued back to back before their chain steps
    static_assert(NK % KC == 0, "K blocks in batches of 8");
#pragma unroll 1
    for (int k0 = kb0; k0 < kb0 + NK; k0 += KC) {
        int c[KC][4];
#pragma unroll
        for (int j = 0; j < KC; j++) {
            const int kb = k0 + j;
            const uint2 bq = *(const uint2*)(xq + kb * BLK);
            mma_s8(c[j], wp[kb * 32], bq.x, bq.y);
        }
        const uint4 sa = *(const uint4*)(DW + fa * KB + k0), sb = *(const uint4*)(DW + fb * KB + k0);
#pragma unroll
        for (int j = 0; j < KC; j++) {
            const float dwa = h2f_pick(sa, j), dwb = h2f_pick(sb, j);
            const float2 dx = *(const float2*)(xd + (k0 + j) * BLK);
            acc[0] = fmaf((float)c[j][0], __fmul_rn(dwa, dx.x), acc[0]);
            acc[1] = fmaf((float)c[j][1], __fmul_rn(dwa, dx.y), acc[1]);
            acc[2] = fmaf((float)c[j][2], __fmul_rn(dwb, dx.x), acc[2]);
            acc[3] = fmaf((float)c[j][3], __fmul_rn(dwb, dx.y), acc[3]);
        }
    }
}
template <int KB>
__device__ __forceinline__ void rg_gemm(const uint8_t* W, const uint16_t* DW, int lr, const uint8_t* X, int rt,
                                        float (&acc)[4]) {
    acc[0] = acc[1] = acc[2] = acc[3] = 0.0f;
    rg_chain<KB, KB>(W, DW, lr, X, rt, 0, acc);
}

// Byte of column c within a row's 32 quants of an exchanged block.
__device__ __forceinline__ int qpos(int c) { return ((c & 15) >> 2) * 8 + ((c >> 4) << 2) + (c & 3); }

// Quantize the 32 values v (lane l holds column l) as row r of the staged block `blk`; the scale is
// stored rounded through fp16 (what a reader of the fp16 scale sees).
__device__ __forceinline__ void stage_row_block(float v, uint8_t* blk, int r) {
    const int lane = threadIdx.x & 31;
    float amax = fabsf(v);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    float dsc, id;
    q8_scale(amax, dsc, id);
    blk[r * 32 + qpos(lane)] = (uint8_t)q8_val(v, id);
    if (lane == 0) *(float*)(blk + DR * 32 + r * 4) = h2f(f2h(dsc));
}

__device__ __forceinline__ void d_bulk_s2c(uint32_t dst_cluster, uint32_t src, uint32_t bytes, uint32_t bar_cluster) {
    asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     dst_cluster),
                 "r"(src), "r"(bytes), "r"(bar_cluster)
                 : "memory");
}

// Every thread of the CTA, after staging: copy the staged bytes into bytes [off, off + bytes) of the
// rows region `rows` of every CTA of the cluster, counted on their `bar`; one bulk copy per CTA.
__device__ __forceinline__ void send_staged(const uint8_t* stg, uint32_t rows, uint32_t off, uint32_t bytes,
                                            uint32_t bar) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // staged bytes -> async proxy
    __syncthreads();
    if (threadIdx.x < DC) d_bulk_s2c(d_mapa(rows + off, threadIdx.x), su32(stg), bytes, d_mapa(bar, threadIdx.x));
}

// LayerNorm row statistics of row r (lane = column, 32 values) in double, sent as slot [rank][r] of
// every CTA's table.
__device__ __forceinline__ void send_row_stats(float v, int r, int rank, uint32_t table, uint32_t bar) {
    const int lane = threadIdx.x & 31;
    double s = (double)v, s2 = (double)v * (double)v;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        s += __shfl_xor_sync(0xffffffffu, s, off);
        s2 += __shfl_xor_sync(0xffffffffu, s2, off);
    }
    if (lane < DC) {
        const uint4 w = make_uint4(__double2loint(s), __double2hiint(s), __double2loint(s2), __double2hiint(s2));
        d_st_async16(d_mapa(table, lane) + (rank * DR + r) * 16, w, d_mapa(bar, lane));
    }
}

// LayerNorm (misc.cu k_layernorm_q8 arithmetic) of one column of row r from the table; w, b: the column's
// weight and bias.
__device__ __forceinline__ float ln_apply(const double* lnp, int r, float v, float w, float b) {
    double s = 0.0, s2 = 0.0;
#pragma unroll
    for (int src = 0; src < DC; src++) {
        s += lnp[(src * DR + r) * 2];
        s2 += lnp[(src * DR + r) * 2 + 1];
    }
    const float mean = (float)(s * (1.0 / D));   // D = 512: exact, equals s / D
    const float var = fmaf(-mean, mean, (float)(s2 * (1.0 / D)));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
    return fmaf(__fmul_rn(__fsub_rn(v, mean), inv), w, b);
}

}  // namespace

template <bool HAS_QKV>
__global__ void __launch_bounds__(DT, 1) k_dense_layer(const DenseParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    cg::cluster_group cl = cg::this_cluster();
    const int rank = (int)cl.block_rank();
    const int r0 = p.slot0 + (blockIdx.x / DC) * DR;   // first slot of this cluster
    const int rend = p.slot0 + p.M;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t bars = su32(sm + SM_BARS);
    auto bar = [&](int i) { return bars + 8 * i; };
    bool ok = true;
    // slot state of row tid (written two or more kernels ago): both fields in one round trip, issued
    // first so the latency overlaps the set-up below
    int st_now = 0, st_pos = 0;
    if (tid < DR && r0 + tid < rend) {
        st_now = p.st[r0 + tid].decode_now;
        st_pos = p.st[r0 + tid].kvpos;
    }

    if (tid == 0) {
        for (int i = 0; i < 11; i++) d_mbar_init(bar(i));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        // exchanges: the bytes the 16 CTAs will send here
        d_expect_tx(bar(BX_ATT), EX_BLOCK);
        d_expect_tx(bar(BX_LN1), EX_STATS);
        d_expect_tx(bar(BX_N1), EX_BLOCK);
        d_expect_tx(bar(BX_H), 4 * EX_BLOCK);
        d_expect_tx(bar(BX_LN2), EX_STATS);
        if (HAS_QKV) d_expect_tx(bar(BX_X), EX_BLOCK);
    }
    __syncthreads();   // the barriers are initialised for every warp of the CTA
    // announce this CTA's armed barriers now (fence.mbarrier_init above publishes the initialisation);
    // wait for the peers' only before the first send
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    if (warp == 0) {   // weights of this CTA's slices (constant), before the wait for the attention kernel
        if (lane == 0) {
            d_expect_tx(bar(BW_OUT), 2 * KB1 * 512 + 32 * KB1 * 2);
            d_expect_tx(bar(BW_F1), 8 * KB1 * 512 + 128 * KB1 * 2);
            d_expect_tx(bar(BW_F2), 2 * KB2 * 512 + 32 * KB2 * 2);
        }
        __syncwarp();
        if (lane == 0) d_bulk(su32(sm + SM_W_OUT), p.w_out + (size_t)(2 * rank) * KB1 * 32, 2 * KB1 * 512, bar(BW_OUT));
        if (lane == 1) d_bulk(su32(sm + SM_D_OUT), p.d_out + (size_t)(32 * rank) * KB1, 32 * KB1 * 2, bar(BW_OUT));
        if (lane == 2) d_bulk(su32(sm + SM_W_F1), p.w_f1 + (size_t)(8 * rank) * KB1 * 32, 8 * KB1 * 512, bar(BW_F1));
        if (lane == 3) d_bulk(su32(sm + SM_D_F1), p.d_f1 + (size_t)(128 * rank) * KB1, 128 * KB1 * 2, bar(BW_F1));
        if (lane == 4) d_bulk(su32(sm + SM_W_F2), p.w_f2 + (size_t)(2 * rank) * KB2 * 32, 2 * KB2 * 512, bar(BW_F2));
        if (lane == 5) d_bulk(su32(sm + SM_D_F2), p.d_f2 + (size_t)(32 * rank) * KB2, 32 * KB2 * 2, bar(BW_F2));
    }
    // x and this CTA's parameters were written two or more kernels ago (or by the host): copied in by
    // TMA while the attention finishes
    float* par = (float*)(sm + SM_PAR);
    int* meta = (int*)(sm + SM_ROWMETA);
    float* xown = (float*)(sm + SM_XOWN);
    if (warp == 1) {   // one copy per lane (the barrier's bytes are armed by lane 0 first)
        const int nrows = max(0, min(DR, rend - r0));
        const uint32_t bp = bar(BW_PAR);
        if (lane == 0) d_expect_tx(bp, (HAS_QKV ? P_COUNT : P_BQKV) * 4 + nrows * 128);
        __syncwarp();
        if (lane < 6) {
            const float* src = lane == 0 ? p.b_out : lane == 1 ? p.b_f2 : lane == 2 ? p.n1w
                             : lane == 3 ? p.n1b : lane == 4 ? p.n2w : p.n2b;
            const int dst = lane == 0 ? P_BOUT : lane == 1 ? P_BF2 : lane == 2 ? P_N1W
                          : lane == 3 ? P_N1B : lane == 4 ? P_N2W : P_N2B;
            d_bulk(su32(par + dst), src + 32 * rank, 128, bp);
        } else if (lane == 6) {
            d_bulk(su32(par + P_BF1), p.b_f1 + 128 * rank, 512, bp);
        } else if (lane < 10) {
            const int part = lane - 7;
            if (HAS_QKV) d_bulk(su32(par + P_BQKV + part * 32), p.b_qkv + part * D + 32 * rank, 128, bp);
        } else if (lane - 10 < nrows) {
            const int r = lane - 10;
            d_bulk(su32(xown + r * 32), p.x + (size_t)(r0 + r) * D + 32 * rank, 128, bp);
        }
    }
    if (tid < DR) {
        meta[tid * 3] = st_now ? st_pos / PAGE + 1 : 0;
        meta[tid * 3 + 2] = st_now ? st_pos : 0;
    }
    griddep_wait();
    griddep_launch();
    __syncthreads();

    uint8_t* stg = sm + SM_STG;
    float* n1own = (float*)(sm + SM_N1OWN);
    float* pre = (float*)(sm + SM_PRE);
    const int r = warp;   // the row of this warp in the row-wise phases

    // ---- phase 0: merge the pages of head `rank` for row r; lane l holds dim l. One round of loads
    // brings m, l and o[l] of up to 32 pages (rows longer than 2048 keys take one more round per 32
    // pages); the pages are then merged in order from registers.
    {
        const int nch = meta[r * 3];
        const size_t item0 = ((size_t)(r0 + r) * NH + rank) * p.max_chunks;
        const float* po = p.part + item0 * HD;
        const float2* pml = (const float2*)p.part_ml + item0;
        float o[32];
        float2 ml;
        auto load_round = [&](int c0) {
            const int cnt = min(32, nch - c0);
            ml = lane < cnt ? __ldcg(pml + c0 + lane) : make_float2(-INFINITY, 0.0f);
#pragma unroll
            for (int j = 0; j < 32; j++) o[j] = j < cnt ? __ldcg(po + (size_t)(c0 + j) * HD + lane) : 0.0f;
        };
        load_round(0);
        float M = ml.x;
        for (int c = 32 + lane; c < nch; c += 32) M = fmaxf(M, __ldcg((const float*)(pml + c)));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
        float L = 0.0f, O = 0.0f;
        for (int c0 = 0; c0 < nch; c0 += 32) {
            if (c0 > 0) load_round(c0);
            const int cnt = min(32, nch - c0);
            const float w = lane < cnt ? exp_canon(ml.x - M) : 0.0f;
#pragma unroll
            for (int j = 0; j < 32; j++) {
                if (j < cnt) {
                    const float wj = __shfl_sync(0xffffffffu, w, j), lj = __shfl_sync(0xffffffffu, ml.y, j);
                    L = fmaf(wj, lj, L);
                    O = fmaf(wj, o[j], O);
                }
            }
        }
        if (nch) {
            stage_row_block(__fdiv_rn(O, L), stg + STG_ATT, r);
        } else {   // not decoding: zero quants, scale 0
            stg[STG_ATT + r * 32 + lane] = 0;
            if (lane == 0) *(float*)(stg + STG_ATT + DR * 32 + r * 4) = 0.0f;
        }
    }
    ok &= d_wait(bar(BW_PAR));   // parameters and x columns
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");   // every peer's barriers are armed
    send_staged(stg + STG_ATT, su32(sm + SM_AROWS), rank * BLK, BLK, bar(BX_ATT));

    // ---- phase 1: out-projection + residual + bias (columns 32*rank + 0..31); an idle warp looks up
    // the KV page of this step's key for phase 6
    if (HAS_QKV && warp == NW - 1 && lane < DR) {
        const int rr = lane;
        meta[rr * 3 + 1] = meta[rr * 3] ? p.kv.block_table[(size_t)(r0 + rr) * p.kv.max_pages + meta[rr * 3 + 2] / PAGE] : 0;
    }
    if (warp < 4) {
        ok &= d_wait(bar(BX_ATT));
        ok &= d_wait(bar(BW_OUT));
        float acc[4];
        const int lr = warp & 1, rt = warp >> 1;
        rg_gemm<KB1>(sm + SM_W_OUT, (const uint16_t*)(sm + SM_D_OUT), lr, sm + SM_AROWS, rt, acc);
        const int g = lane >> 2, t = lane & 3;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int f = lr * 16 + g + (i >= 2 ? 8 : 0), rr = rt * 8 + 2 * t + (i & 1);
            pre[rr * 32 + f] = __fadd_rn(__fadd_rn(xown[rr * 32 + f], acc[i]), par[P_BOUT + f]);
        }
    }
    __syncthreads();
    send_row_stats(pre[r * 32 + lane], r, rank, su32(sm + SM_LNP1), bar(BX_LN1));

    // ---- phase 2: LayerNorm 1 of the CTA's columns -> n1 (kept) and its Q8_0 block (sent)
    ok &= d_wait(bar(BX_LN1));
    {
        const float n1 = ln_apply((const double*)(sm + SM_LNP1), r, pre[r * 32 + lane], par[P_N1W + lane],
                                  par[P_N1B + lane]);
        n1own[r * 32 + lane] = n1;
        stage_row_block(n1, stg + STG_N1, r);
    }
    send_staged(stg + STG_N1, su32(sm + SM_N1ROWS), rank * BLK, BLK, bar(BX_N1));

    // ---- phase 3: FFN1 (columns 128*rank + 0..127), bias + ReLU: warp = (row group, row tile)
    float* hown = (float*)(sm + SM_AROWS);   // [DR][128] f32 (the attention rows are consumed)
    ok &= d_wait(bar(BX_N1));
    ok &= d_wait(bar(BW_F1));
    {
        const int lr = warp & 7, rt = warp >> 3;
        float acc[4];
        rg_gemm<KB1>(sm + SM_W_F1, (const uint16_t*)(sm + SM_D_F1), lr, sm + SM_N1ROWS, rt, acc);
        const int g = lane >> 2, t = lane & 3;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int f = lr * 16 + g + (i >= 2 ? 8 : 0), rr = rt * 8 + 2 * t + (i & 1);
            const float h = __fadd_rn(acc[i], par[P_BF1 + f]);
            hown[rr * 128 + f] = h > 0.0f ? h : 0.0f;
        }
    }
    __syncthreads();
    if (HAS_QKV && tid == 0) {   // out + ffn1 slices are consumed: the next layer's q|k|v rows go there
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        d_expect_tx(bar(BW_QKV), 6 * KB1 * 512 + 96 * KB1 * 2);
        for (int part = 0; part < 3; part++) {
            d_bulk(su32(sm + SM_W_QKV + part * 2 * KB1 * 512),
                   p.w_qkv + (size_t)(part * (D / 16) + 2 * rank) * KB1 * 32, 2 * KB1 * 512, bar(BW_QKV));
            d_bulk(su32(sm + SM_D_QKV + part * 32 * KB1 * 2), p.d_qkv + (size_t)(part * D + 32 * rank) * KB1,
                   32 * KB1 * 2, bar(BW_QKV));
        }
    }
    {   // the row's 4 Q8_0 blocks at once: lane (b, c) quantizes columns 4c..4c+3 of block b = lane / 8
        const int b = lane >> 3, c = lane & 7;
        const float4 v = *(const float4*)(hown + r * 128 + b * 32 + c * 4);
        float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
        for (int off = 4; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
        float dsc, id;
        q8_scale(amax, dsc, id);
        const uint32_t qw = (uint32_t)(uint8_t)q8_val(v.x, id) | (uint32_t)(uint8_t)q8_val(v.y, id) << 8 |
                            (uint32_t)(uint8_t)q8_val(v.z, id) << 16 | (uint32_t)(uint8_t)q8_val(v.w, id) << 24;
        uint8_t* blk = stg + STG_H + b * BLK;
        *(uint32_t*)(blk + r * 32 + qpos(4 * c)) = qw;   // columns 4c..4c+3 are adjacent under qpos
        if (c == 0) *(float*)(blk + DR * 32 + r * 4) = h2f(f2h(dsc));
    }
    send_staged(stg + STG_H, su32(sm + SM_HROWS), 4 * rank * BLK, 4 * BLK, bar(BX_H));

    // ---- phase 4: FFN2 + residual n1 + bias (columns 32*rank + 0..31): warp = (row group, row tile), each
    // the whole 64-block chain (splitting K over warps with hand-offs of the running sums measured slower)
    {
        ok &= d_wait(bar(BX_H));
        ok &= d_wait(bar(BW_F2));
        if (warp < 4) {
            const int lr = warp & 1, rt = warp >> 1;
            float acc[4];
            rg_gemm<KB2>(sm + SM_W_F2, (const uint16_t*)(sm + SM_D_F2), lr, sm + SM_HROWS, rt, acc);
            const int g = lane >> 2, t = lane & 3;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int f = lr * 16 + g + (i >= 2 ? 8 : 0), rr = rt * 8 + 2 * t + (i & 1);
                pre[rr * 32 + f] = __fadd_rn(__fadd_rn(n1own[rr * 32 + f], acc[i]), par[P_BF2 + f]);
            }
        }
    }
    __syncthreads();
    send_row_stats(pre[r * 32 + lane], r, rank, su32(sm + SM_LNP2), bar(BX_LN2));

    // ---- phase 5: LayerNorm 2 -> x (global, next layer's residual) and its Q8_0 block
    ok &= d_wait(bar(BX_LN2));
    {
        const float xv = ln_apply((const double*)(sm + SM_LNP2), r, pre[r * 32 + lane], par[P_N2W + lane],
                                  par[P_N2B + lane]);
        if (r0 + r < rend) p.x[(size_t)(r0 + r) * D + 32 * rank + lane] = xv;
        if (HAS_QKV) stage_row_block(xv, stg + STG_X, r);
    }
    if (HAS_QKV) send_staged(stg + STG_X, su32(sm + SM_XROWS), rank * BLK, BLK, bar(BX_X));

    // ---- phase 6: next layer's q, k, v of head `rank` (+ bias); K/V into the pages. warp = (row group, tile)
    if (HAS_QKV && warp < 12) {
        ok &= d_wait(bar(BX_X));
        ok &= d_wait(bar(BW_QKV));
        const int lr = warp % 6, rt = warp / 6, part = lr >> 1, g = lane >> 2, t = lane & 3;
        float acc[4];
        rg_gemm<KB1>(sm + SM_W_QKV, (const uint16_t*)(sm + SM_D_QKV), lr, sm + SM_XROWS, rt, acc);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int f = (lr & 1) * 16 + g + (i >= 2 ? 8 : 0), rr = rt * 8 + 2 * t + (i & 1), slot = r0 + rr;
            if (slot >= rend) continue;
            const float y = __fadd_rn(acc[i], par[P_BQKV + part * 32 + f]);
            if (part == 0) {
                p.q[(size_t)slot * p.q_stride + 32 * rank + f] = y;
            } else if (meta[rr * 3]) {
                const int page = meta[rr * 3 + 1], pos = meta[rr * 3 + 2];
                const size_t e = ((((size_t)page * p.kv.n_layer + p.kv.layer) * 2 + (part - 1)) * NH + rank) *
                                     (PAGE * HD) +
                                 (size_t)(pos % PAGE) * HD + f;
                if (p.kv.kv_f32) ((float*)p.kv.pool)[e] = y;
                else ((__half*)p.kv.pool)[e] = __float2half_rn(y);
            }
        }
    }
    if (!__all_sync(0xffffffffu, ok)) {
        // a copy or an exchange never completed: flag it and wait (bounded) for what may still arrive
        if (lane == 0 && p.err) atomicExch(p.err, 1);
        for (int i = 0; i < 11; i++)
            if (HAS_QKV || (i != BW_QKV && i != BX_X)) (void)d_wait(bar(i));
    }
    // no CTA leaves while a peer may still be sending to it
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\nbarrier.cluster.wait.aligned;" ::: "memory");
}

static int g_dense_priority = 0;   // the device's highest stream priority

cudaError_t dense_init_device(bool* usable) {
    *usable = false;
    cudaError_t e;
    int least = 0, greatest = 0;
    if ((e = cudaDeviceGetStreamPriorityRange(&least, &greatest))) return e;
    g_dense_priority = greatest;
    void (*ks[2])(const DenseParams) = {k_dense_layer<true>, k_dense_layer<false>};
    for (auto k : ks) {
        if ((e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_DENSE))) return e;
        if ((e = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1))) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(DC);
    cfg.blockDim = dim3(DT);
    cfg.dynamicSmemBytes = SMEM_DENSE;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = DC;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, k_dense_layer<true>, &cfg);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return cudaSuccess;   // not usable: the unfused kernels run instead
    }
    *usable = n >= 1;
    return cudaSuccess;
}

void launch_dense_layer(const DenseParams& p, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((p.M + DR - 1) / DR * DC));
    cfg.blockDim = dim3(DT);
    cfg.dynamicSmemBytes = SMEM_DENSE;
    cfg.stream = s;
    cudaLaunchAttribute at[3];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = DC;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    // latency-bound clusters go first when attention CTAs of the other slot group free SMs
    at[2].id = cudaLaunchAttributePriority;
    at[2].val.priority = g_dense_priority;
    cfg.attrs = at;
    cfg.numAttrs = 3;
    if (p.w_qkv) cudaLaunchKernelEx(&cfg, k_dense_layer<true>, p);
    else cudaLaunchKernelEx(&cfg, k_dense_layer<false>, p);
}

}  // namespace gsvcu
