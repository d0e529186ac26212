// gemm_q8.cu -- Q8_0 x Q8_0 GEMM on the tensor cores (mma.m16n8k32 s8 -> s32) with fused epilogues.
//
// Semantics (ggml Q8_0 mul_mat, as used at reference src/gsv_ar.cpp:244,260,262,263): per output
// (n, m) the integer dot of every 32-element block is exact (int32 MMA with a zero accumulator is
// one Q8_0 block), and the float result is accumulated block by block, in block order:
//     acc = fma((float)isum_b, d_w[n][b] * d_x[m][b], acc).
// So the output is bit-identical to the oracle's restatement.
//
// Tiling. A CTA owns 32 output features x 8T tokens. Its activation rows and scales are staged in
// shared memory; KS warps split every chunk of 4*KS K-blocks (each warp 4 blocks), write the exact
// int32 block sums into shared memory, and after a barrier every thread runs the sequential float
// chain for its outputs. Weights stream from HBM once per token tile with 128-bit non-allocating
// loads in fragment order, prefetched one chunk ahead.
#include <cstring>

#include "kernels.h"

namespace gsvcu {

__device__ __forceinline__ void mma_s8(int (&c)[4], const uint4& a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};\n"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

constexpr int SSTR = 33;   // row stride (words) of the int32 block-sum tile

__host__ __device__ constexpr size_t gemm_smem_bytes(int T, int KS, int K) {
    return (size_t)(8 * T) * (K + 16)                  // Xs
           + (size_t)(8 * T) * (K / 32) * 2            // Xds
           + (size_t)(K / 32) * 32 * 2                 // Wds
           + 16                                        // alignment slack
           + (size_t)(4 * KS) * (8 * T) * SSTR * 4;    // S
}

template <int T, int KS, int EPI>
__global__ void __launch_bounds__(32 * KS) k_gemm_q8(const GemmQ8Params p) {
    constexpr int TOK = 8 * T;
    constexpr int NT = 32 * KS;                 // threads
    constexpr int KC = 4 * KS;                  // K-blocks per chunk
    constexpr int NOUT = (TOK * 32 + NT - 1) / NT;
    extern __shared__ __align__(16) uint8_t smem[];
    const int K = p.K, KB = K / QK;
    const int XSTR = K + 16;
    int8_t* Xs = (int8_t*)smem;
    uint16_t* Xds = (uint16_t*)(smem + (size_t)TOK * XSTR);    // [TOK][KB]
    uint16_t* Wds = Xds + TOK * KB;                             // [KB][32]
    int32_t* S = (int32_t*)(((uintptr_t)(Wds + KB * 32) + 15) & ~(uintptr_t)15);   // [KC][TOK][SSTR]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const int f0 = blockIdx.x * 32, tok0 = blockIdx.y * TOK;

    // weight fragments of this warp for chunk c: kb = c*KC + warp*4 + i
    const uint4* w0 = p.wq + (size_t)(2 * blockIdx.x + 0) * KB * 32 + lane;
    const uint4* w1 = p.wq + (size_t)(2 * blockIdx.x + 1) * KB * 32 + lane;
    uint4 fa[4], fb[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int kb = warp * 4 + i;
        fa[i] = ldg_stream(w0 + (size_t)kb * 32);
        fb[i] = ldg_stream(w1 + (size_t)kb * 32);
    }

    for (int i = tid; i < 32 * KB; i += NT) {
        const int kb = i >> 5, f = i & 31;
        Wds[i] = p.wd[(size_t)(f0 + f) * KB + kb];
    }
    // weights above are constant; the activations below come from the previous kernel
    griddep_wait();
    griddep_launch();
    // stage activations and their scales
    const int vpr = K / 16;
    for (int i = tid; i < TOK * vpr; i += NT) {
        const int r = i / vpr, c = i - r * vpr;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (tok0 + r < p.M) v = *(const uint4*)(p.xq + (size_t)(tok0 + r) * K + c * 16);
        *(uint4*)(Xs + (size_t)r * XSTR + c * 16) = v;
    }
    for (int i = tid; i < TOK * KB; i += NT) {
        const int r = i / KB;
        Xds[i] = tok0 + r < p.M ? p.xd[(size_t)(tok0 + r) * KB + (i - r * KB)] : (uint16_t)0;
    }
    __syncthreads();

    float acc[NOUT];
#pragma unroll
    for (int q = 0; q < NOUT; q++) acc[q] = 0.0f;

    const int nchunks = KB / KC;
    for (int c = 0; c < nchunks; c++) {
        uint4 ca[4], cb[4];
#pragma unroll
        for (int i = 0; i < 4; i++) { ca[i] = fa[i]; cb[i] = fb[i]; }
        if (c + 1 < nchunks) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int kb = (c + 1) * KC + warp * 4 + i;
                fa[i] = ldg_stream(w0 + (size_t)kb * 32);
                fb[i] = ldg_stream(w1 + (size_t)kb * 32);
            }
        }
        // phase 1: exact int32 block sums -> S[kbl][n][f]
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int kbl = warp * 4 + i, kb = c * KC + kbl;
            int32_t* s = S + (size_t)kbl * TOK * SSTR;
#pragma unroll
            for (int j = 0; j < T; j++) {
                const int8_t* xr = Xs + (size_t)(j * 8 + g) * XSTR + kb * 32 + t4 * 4;
                const uint32_t b0 = *(const uint32_t*)xr, b1 = *(const uint32_t*)(xr + 16);
                int c0[4], c1[4];
                mma_s8(c0, ca[i], b0, b1);
                mma_s8(c1, cb[i], b0, b1);
                const int n0 = j * 8 + 2 * t4;
                s[n0 * SSTR + g] = c0[0];
                s[(n0 + 1) * SSTR + g] = c0[1];
                s[n0 * SSTR + g + 8] = c0[2];
                s[(n0 + 1) * SSTR + g + 8] = c0[3];
                s[n0 * SSTR + g + 16] = c1[0];
                s[(n0 + 1) * SSTR + g + 16] = c1[1];
                s[n0 * SSTR + g + 24] = c1[2];
                s[(n0 + 1) * SSTR + g + 24] = c1[3];
            }
        }
        __syncthreads();
        // phase 2: sequential float chain over the chunk's blocks, block order
#pragma unroll
        for (int q = 0; q < NOUT; q++) {
            const int o = tid + q * NT;
            if (o < TOK * 32) {
                const int n = o >> 5, f = o & 31;
                float a = acc[q];
#pragma unroll 4
                for (int kbl = 0; kbl < KC; kbl++) {
                    const int kb = c * KC + kbl;
                    const float dw = h2f(Wds[kb * 32 + f]);
                    const float dx = h2f(Xds[n * KB + kb]);
                    const int32_t si = S[((size_t)kbl * TOK + n) * SSTR + f];
                    a = fmaf((float)si, __fmul_rn(dw, dx), a);
                }
                acc[q] = a;
            }
        }
        __syncthreads();
    }

    // epilogue: thread q-th output (n = o/32, f = o%32); a warp holds 32 consecutive features of one row
#pragma unroll
    for (int q = 0; q < NOUT; q++) {
        const int o = tid + q * NT;
        if (o >= TOK * 32) continue;   // warp-uniform (TOK*32 is a multiple of 32)
        const int nl = o >> 5, f = f0 + (o & 31), n = tok0 + nl;
        const bool valid = n < p.M;
        const float bias = p.bias ? p.bias[f] : 0.0f;
        if (EPI == EPI_BIAS) {
            const float y = __fadd_rn(acc[q], bias);
            if (valid && f < (p.n_store ? p.n_store : p.N)) p.y[(size_t)n * (p.ldy ? p.ldy : p.N) + f] = y;
            if (valid && p.kv.pool && f >= D) {
                int slot, pos;
                bool ok = true;
                if (p.kv.tok_pos) {
                    slot = p.kv.tok_slot[n];
                    pos = p.kv.tok_pos[n];
                } else {
                    slot = n;
                    ok = p.kv.st[n].decode_now != 0;
                    pos = p.kv.st[n].kvpos;
                }
                if (ok) {
                    const int kvsel = (f - D) >> 9, fh = (f - D) & (D - 1);
                    const int h = fh >> 5, dd = fh & 31;
                    const int page = p.kv.block_table[(size_t)slot * p.kv.max_pages + pos / PAGE];
                    const size_t e = ((((size_t)page * p.kv.n_layer + p.kv.layer) * 2 + kvsel) * NH + h) * (PAGE * HD) +
                                     (size_t)(pos % PAGE) * HD + dd;
                    if (p.kv.kv_f32) ((float*)p.kv.pool)[e] = y;
                    else ((__half*)p.kv.pool)[e] = __float2half_rn(y);
                }
            }
        } else if (EPI == EPI_RESID) {
            if (valid) {
                const float r = p.resid[(size_t)n * p.N + f];
                p.y[(size_t)n * p.N + f] = __fadd_rn(__fadd_rn(r, acc[q]), bias);
            }
        } else {   // EPI_RELU_Q8: relu(acc + bias), one Q8_0 block per row across the warp
            float h = __fadd_rn(acc[q], bias);
            h = h > 0.0f ? h : 0.0f;
            float amax = fabsf(h);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
            float dsc, id;
            q8_scale(amax, dsc, id);
            if (valid) {
                p.yq[(size_t)n * p.N + f] = q8_val(h, id);
                if ((o & 31) == 0) p.yd[(size_t)n * (p.N / QK) + f / QK] = f2h(dsc);
            }
        }
    }
}

// ------------------------------------------------------------------ large-M tiles (prefill)
// CTA tile: 64 output features x 64 tokens, 8 warps; warp w owns row group w&3 (16 features) and
// tokens 32*(w>>2) .. +31 (four n = 8 tiles). K advances in chunks of 8 blocks, double-buffered with
// cp.async; every Q8_0 block is one mma.m16n8k32 with a zero accumulator and each output's float chain
// acc = fma((float)isum_b, d_w*d_x, acc) runs in registers in block order (the same chain as above).
// The epilogue goes through shared memory, one token row per warp-iteration, for coalesced stores.
namespace {
constexpr int TF = 64, TT = 64, TKC = 8;        // features, tokens, K blocks per chunk
constexpr int TB_STRIDE = TKC * 32 + 16;        // padded int8 row stride of a token's chunk
constexpr int TS_A = 4 * TKC * 512;             // weight fragments of one chunk
constexpr int TS_B = TT * TB_STRIDE;            // activation rows of one chunk
constexpr int TS_DW = TF * TKC * 2, TS_DX = TT * TKC * 2;
constexpr int TSTAGE = TS_A + TS_B + TS_DW + TS_DX;
constexpr int TSMEM = 2 * TSTAGE;
static_assert(TT * (TF + 1) * 4 <= TSMEM, "epilogue staging fits in the chunk buffers");

__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src), "r"(src_bytes)
                 : "memory");
}
}  // namespace

template <int EPI>
__global__ void __launch_bounds__(256) k_gemm_q8_tile(const GemmQ8Params p) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int K = p.K, KB = K / QK;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int f0 = blockIdx.x * TF, t0 = blockIdx.y * TT;
    const int rg = warp & 3, th = warp >> 2;

    // chunk c -> stage st
    auto load_chunk = [&](int c, int st) {
        uint8_t* base = smem + (size_t)st * TSTAGE;
        const int k0 = c * TKC;
        for (int i = tid; i < 4 * TKC * 32; i += 256) {   // 4 row groups x TKC blocks x 32 lanes of 16 B
            const int r = i / (TKC * 32), rest = i - r * (TKC * 32);
            cp_async16(base + (size_t)i * 16, p.wq + ((size_t)(f0 / 16 + r) * KB + k0) * 32 + rest, 16);
        }
        for (int i = tid; i < TT * TKC * 2; i += 256) {   // TT rows x (TKC*32 B = TKC*2 x 16 B)
            const int n = i / (TKC * 2), j = i - n * (TKC * 2);
            const bool ok = t0 + n < p.M;
            const int8_t* src = p.xq + (size_t)(ok ? t0 + n : 0) * K + k0 * 32 + j * 16;
            cp_async16(base + TS_A + n * TB_STRIDE + j * 16, src, ok ? 16 : 0);
        }
        if (tid < TF) cp_async16(base + TS_A + TS_B + tid * 16, p.wd + (size_t)(f0 + tid) * KB + k0, 16);
        else if (tid < TF + TT) {
            const int n = tid - TF;
            const bool ok = t0 + n < p.M;
            cp_async16(base + TS_A + TS_B + TS_DW + n * 16, p.xd + (size_t)(ok ? t0 + n : 0) * KB + k0, ok ? 16 : 0);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    griddep_wait();
    griddep_launch();
    float acc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; nt++) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.0f;
    const int nchunks = KB / TKC;
    load_chunk(0, 0);
    for (int c = 0; c < nchunks; c++) {
        if (c + 1 < nchunks) {
            load_chunk(c + 1, (c + 1) & 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const uint8_t* base = smem + (size_t)(c & 1) * TSTAGE;
        const uint4* A = (const uint4*)base + (size_t)rg * TKC * 32 + lane;
        const int8_t* B = (const int8_t*)(base + TS_A) + (th * 32 + g) * TB_STRIDE + t * 4;
        const uint16_t* DW = (const uint16_t*)(base + TS_A + TS_B);
        const uint16_t* DX = (const uint16_t*)(base + TS_A + TS_B + TS_DW);
        const int fa = rg * 16 + g, fb = fa + 8;
#pragma unroll 2
        for (int kb = 0; kb < TKC; kb++) {
            const uint4 a = A[kb * 32];
            int cc[4][4];
#pragma unroll
            for (int nt = 0; nt < 4; nt++) {
                const int8_t* br = B + nt * 8 * TB_STRIDE + kb * 32;
                mma_s8(cc[nt], a, *(const uint32_t*)br, *(const uint32_t*)(br + 16));
            }
            const float dwa = h2f(DW[fa * TKC + kb]), dwb = h2f(DW[fb * TKC + kb]);
#pragma unroll
            for (int nt = 0; nt < 4; nt++) {
                const int ra = th * 32 + nt * 8 + 2 * t;
                const float dxa = h2f(DX[ra * TKC + kb]), dxb = h2f(DX[(ra + 1) * TKC + kb]);
                acc[nt][0] = fmaf((float)cc[nt][0], __fmul_rn(dwa, dxa), acc[nt][0]);
                acc[nt][1] = fmaf((float)cc[nt][1], __fmul_rn(dwa, dxb), acc[nt][1]);
                acc[nt][2] = fmaf((float)cc[nt][2], __fmul_rn(dwb, dxa), acc[nt][2]);
                acc[nt][3] = fmaf((float)cc[nt][3], __fmul_rn(dwb, dxb), acc[nt][3]);
            }
        }
        __syncthreads();   // this stage is refilled by the next iteration's prefetch
    }

    // epilogue: ys[token][feature] (stride TF + 1) then one token row per warp iteration
    float* ys = (float*)smem;
#pragma unroll
    for (int nt = 0; nt < 4; nt++) {
        const int ra = th * 32 + nt * 8 + 2 * t, fa = rg * 16 + g;
        ys[ra * (TF + 1) + fa] = acc[nt][0];
        ys[(ra + 1) * (TF + 1) + fa] = acc[nt][1];
        ys[ra * (TF + 1) + fa + 8] = acc[nt][2];
        ys[(ra + 1) * (TF + 1) + fa + 8] = acc[nt][3];
    }
    __syncthreads();
    for (int nl = warp; nl < TT; nl += 8) {
        const int n = t0 + nl;
        if (n >= p.M) break;   // warp-uniform
#pragma unroll
        for (int half = 0; half < 2; half++) {
            const int fl = half * 32 + lane, f = f0 + fl;
            const float a = ys[nl * (TF + 1) + fl];
            const float bias = p.bias ? p.bias[f] : 0.0f;
            if (EPI == EPI_BIAS) {
                const float y = __fadd_rn(a, bias);
                if (f < (p.n_store ? p.n_store : p.N)) p.y[(size_t)n * (p.ldy ? p.ldy : p.N) + f] = y;
                bool ok = p.kv.pool && f >= D;
                int slot = 0, pos = 0;
                if (ok) {
                    if (p.kv.tok_pos) {   // prefill: row n is token tok_pos[n] of slot tok_slot[n]
                        slot = p.kv.tok_slot[n];
                        pos = p.kv.tok_pos[n];
                    } else {              // decode: row n is slot n, at its step position
                        slot = n;
                        ok = p.kv.st[n].decode_now != 0;
                        pos = p.kv.st[n].kvpos;
                    }
                }
                if (ok) {
                    const int kvsel = (f - D) >> 9, fh = (f - D) & (D - 1);
                    const int h = fh >> 5, dd = fh & 31;
                    const int page = p.kv.block_table[(size_t)slot * p.kv.max_pages + pos / PAGE];
                    const size_t e = ((((size_t)page * p.kv.n_layer + p.kv.layer) * 2 + kvsel) * NH + h) * (PAGE * HD) +
                                     (size_t)(pos % PAGE) * HD + dd;
                    if (p.kv.kv_f32) ((float*)p.kv.pool)[e] = y;
                    else ((__half*)p.kv.pool)[e] = __float2half_rn(y);
                }
            } else if (EPI == EPI_RESID) {
                const float r = p.resid[(size_t)n * p.N + f];
                p.y[(size_t)n * p.N + f] = __fadd_rn(__fadd_rn(r, a), bias);
            } else {   // relu(acc + bias), one Q8_0 block per 32 features across the warp
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

template <int T, int KS>
static void launch_t(const GemmQ8Params& p, int epi, cudaStream_t s) {
    const size_t smem = gemm_smem_bytes(T, KS, p.K);
    dim3 grid(p.N / 32, (p.M + 8 * T - 1) / (8 * T));
    dim3 block(32 * KS);
    switch (epi) {
        case EPI_BIAS: launch_pdl(k_gemm_q8<T, KS, EPI_BIAS>, grid, block, smem, s, p); break;
        case EPI_RESID: launch_pdl(k_gemm_q8<T, KS, EPI_RESID>, grid, block, smem, s, p); break;
        default: launch_pdl(k_gemm_q8<T, KS, EPI_RELU_Q8>, grid, block, smem, s, p); break;
    }
}

template <int T, int KS>
static cudaError_t init_t(int K) {
    const int smem = (int)gemm_smem_bytes(T, KS, K);
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(k_gemm_q8<T, KS, EPI_BIAS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem))) return e;
    if ((e = cudaFuncSetAttribute(k_gemm_q8<T, KS, EPI_RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem))) return e;
    return cudaFuncSetAttribute(k_gemm_q8<T, KS, EPI_RELU_Q8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
}

cudaError_t gemm_q8_init_device() {
    cudaError_t e;
    if ((e = init_t<1, 4>(512))) return e;
    if ((e = init_t<1, 8>(4096))) return e;   // K up to 4096 (the BERT FFN's second matrix)
    if ((e = init_t<4, 4>(2048))) return e;
    if ((e = cudaFuncSetAttribute(k_gemm_q8_tile<EPI_BIAS>, cudaFuncAttributeMaxDynamicSharedMemorySize, TSMEM))) return e;
    if ((e = cudaFuncSetAttribute(k_gemm_q8_tile<EPI_RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize, TSMEM))) return e;
    return cudaFuncSetAttribute(k_gemm_q8_tile<EPI_RELU_Q8>, cudaFuncAttributeMaxDynamicSharedMemorySize, TSMEM);
}

void launch_gemm_q8(const GemmQ8Params& p, int epi, cudaStream_t s) {
    // K = 512 -> KS 4 (one chunk of 16 blocks); K = 2048 -> KS 8 at small M (two chunks of 32)
    const int KB = p.K / QK;
    if (p.M > 64 && gemm_tc_usable(p) && launch_gemm_q8_tc(p, epi, s)) return;   // tcgen05 path (prefill)
    if (p.M <= 64 && KB % 16 == 0) {   // the small-M kernels take K in chunks of 16 (KS 4) or 32 (KS 8) blocks
        if (KB % 32 == 0) launch_t<1, 8>(p, epi, s);
        else launch_t<1, 4>(p, epi, s);
    } else if (p.N % TF == 0 && KB % TKC == 0) {
        dim3 grid(p.N / TF, (p.M + TT - 1) / TT);
        switch (epi) {
            case EPI_BIAS: launch_pdl(k_gemm_q8_tile<EPI_BIAS>, grid, dim3(256), TSMEM, s, p); break;
            case EPI_RESID: launch_pdl(k_gemm_q8_tile<EPI_RESID>, grid, dim3(256), TSMEM, s, p); break;
            default: launch_pdl(k_gemm_q8_tile<EPI_RELU_Q8>, grid, dim3(256), TSMEM, s, p); break;
        }
    } else {
        launch_t<4, 4>(p, epi, s);
    }
}

void pack_q8_0_host(const uint8_t* raw, int N, int K, uint8_t* wq_out, uint16_t* wd_out) {
    const int KB = K / QK;
    for (int n = 0; n < N; n++)
        for (int kb = 0; kb < KB; kb++) {
            uint16_t d;
            std::memcpy(&d, raw + ((size_t)n * KB + kb) * 34, 2);
            wd_out[(size_t)n * KB + kb] = d;
        }
    // fragment order of the mma.m16n8k32 A operand: lane l = 4g + t holds
    //   a0: row g,   cols 4t..4t+3     a1: row g+8, cols 4t..4t+3
    //   a2: row g,   cols 16+4t..      a3: row g+8, cols 16+4t..
    for (int rg = 0; rg < N / 16; rg++)
        for (int kb = 0; kb < KB; kb++) {
            uint8_t* dst = wq_out + (((size_t)rg * KB + kb) * 32) * 16;
            for (int lane = 0; lane < 32; lane++) {
                const int g = lane >> 2, t = lane & 3;
                for (int reg = 0; reg < 4; reg++) {
                    const int row = rg * 16 + g + ((reg & 1) ? 8 : 0);
                    const int col = t * 4 + ((reg & 2) ? 16 : 0);
                    const uint8_t* src = raw + ((size_t)row * KB + kb) * 34 + 2 + col;
                    std::memcpy(dst + lane * 16 + reg * 4, src, 4);
                }
            }
        }
}

}  // namespace gsvcu
