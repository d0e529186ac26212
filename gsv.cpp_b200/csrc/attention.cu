// attention.cu -- decode (split-KV flash decoding over paged KV) and prefix-masked prefill attention.
//
// Both evaluate ggml flash_attn_ext as the reference uses it (src/gsv_ar.cpp:257,331,404):
// score = (float)(sum_d (double)(q_d * k_d)) * (1/sqrt(32)), masked keys skipped, softmax(score) V
// with the weights and sums in double, one final rounding to float; then Q8_0-quantized (one head
// = one 32-value block) for the out-projection GEMM.
#include <cfloat>

#include "kernels.h"

namespace gsvcu {

// ------------------------------------------------------------------ decode
// Work item = (slot, head, chunk of ATT_CHUNK keys), one warp each, 4 heads per CTA.
// K/V rows of one head are 32 contiguous elements inside a 64-token page, so a warp reads
// TPI tokens x 64 B (F16) per 128-bit load instruction; U loads of K and U of V are in flight per
// lane, a block of TPI*U (32 for F16) tokens per iteration.
//
// Arithmetic: scores s = (float)(double sum of float products) * scale, as ggml's vec_dot_f32; the
// softmax-weighted sum is carried in double: per block of tokens the warp-uniform running max m is
// raised to the block max (rescaling l and o by exp(m_old - m_new)), lane j computes the weight
// p_j = exp(s_j - m) of token j once, and each lane accumulates o += p * v for its dims. The result
// (float)(o / l) is exact to ~1e-16 before the final rounding, so it does not depend on the
// reduction order (token groups, split-KV chunks) and equals the oracle's evaluation bit for bit.
// Chunks of one (slot, head) are merged by the last warp to finish (atomic ticket, no waiting).
template <typename KT>
__global__ void __launch_bounds__(128) k_decode_attn(const DecAttnParams p) {
    constexpr int EPL = 16 / sizeof(KT);     // elements per lane per load
    constexpr int LPT = HD / EPL;            // lanes per token
    constexpr int TPI = 32 / LPT;            // tokens per warp-load
    constexpr int U = 4;                     // loads in flight per lane (per K and per V)
    constexpr int BLK = TPI * U;             // tokens per block (<= 32)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int slot = blockIdx.z, chunk = blockIdx.y, h = blockIdx.x * 4 + warp;
    int kvpos;
    bool act;
    if (p.st) {
        act = p.st[slot].decode_now != 0;
        kvpos = p.st[slot].kvpos;
    } else {
        act = p.active[slot] != 0;
        kvpos = p.kvpos[slot];
    }
    if (!act) return;
    const int nkeys = kvpos + 1, k0 = chunk * ATT_CHUNK;
    if (k0 >= nkeys) return;
    const int k1 = min(k0 + ATT_CHUNK, nkeys);
    const int nch = (nkeys + ATT_CHUNK - 1) / ATT_CHUNK;
    const int sub = lane % LPT, tk = lane / LPT;

    float q[EPL];
    {
        const float* qp = p.q + (size_t)slot * p.q_stride + h * HD + sub * EPL;
#pragma unroll
        for (int e = 0; e < EPL; e++) q[e] = qp[e];
    }
    const size_t page_elems = (size_t)p.n_layer * 2 * NH * PAGE * HD;
    const size_t koff = ((size_t)p.layer * 2 + 0) * NH * PAGE * HD + (size_t)h * PAGE * HD + sub * EPL;
    const size_t voff = koff + (size_t)NH * PAGE * HD;
    const KT* pool = (const KT*)p.pool;
    const int32_t* bt = p.block_table + (size_t)slot * p.max_pages;

    float m = -INFINITY;      // warp-uniform running max
    double l = 0.0, o[EPL];   // l: this lane's tokens; o: this lane's dims over its tokens
#pragma unroll
    for (int e = 0; e < EPL; e++) o[e] = 0.0;

    for (int base = k0; base < k1; base += BLK) {
        const size_t pbase = (size_t)bt[base / PAGE] * page_elems;
        uint4 kr[U], vr[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int kk = base + u * TPI + tk;
            kr[u] = make_uint4(0u, 0u, 0u, 0u);
            vr[u] = kr[u];
            if (kk < k1) {
                const size_t r = pbase + (size_t)(kk % PAGE) * HD;
                kr[u] = ldg_stream(pool + r + koff);
                vr[u] = ldg_stream(pool + r + voff);
            }
        }
        float sc[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            float kf[EPL];
            if (sizeof(KT) == 2) {
                const __half2* k2 = (const __half2*)&kr[u];
#pragma unroll
                for (int e = 0; e < EPL / 2; e++) {
                    const float2 a = __half22float2(k2[e]);
                    kf[2 * e] = a.x; kf[2 * e + 1] = a.y;
                }
            } else {
                const float* k4 = (const float*)&kr[u];
#pragma unroll
                for (int e = 0; e < EPL; e++) kf[e] = k4[e];
            }
            double dot = 0.0;
#pragma unroll
            for (int e = 0; e < EPL; e++) dot += (double)__fmul_rn(q[e], kf[e]);
#pragma unroll
            for (int off = 1; off < LPT; off <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
            const int kk = base + u * TPI + tk;
            sc[u] = kk < k1 ? __fmul_rn((float)dot, p.scale) : -INFINITY;
        }
        // lane j (< BLK) takes the score of block token j = u*TPI + t, held by lane t*LPT
        float mys = -INFINITY;
#pragma unroll
        for (int u = 0; u < U; u++) {
            const float t = __shfl_sync(0xffffffffu, sc[u], (lane % TPI) * LPT);
            if (lane < BLK && lane / TPI == u) mys = t;
        }
        float bm = mys;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, off));
        if (bm > m) {   // warp-uniform
            const double r = m == -INFINITY ? 0.0 : exp((double)m - (double)bm);
            l *= r;
#pragma unroll
            for (int e = 0; e < EPL; e++) o[e] *= r;
            m = bm;
        }
        const double pj = mys == -INFINITY ? 0.0 : exp((double)mys - (double)m);
        l += pj;
#pragma unroll
        for (int u = 0; u < U; u++) {
            const double pu = __shfl_sync(0xffffffffu, pj, u * TPI + tk);
            if (sizeof(KT) == 2) {
                const __half2* v2 = (const __half2*)&vr[u];
#pragma unroll
                for (int e = 0; e < EPL / 2; e++) {
                    const float2 b = __half22float2(v2[e]);
                    o[2 * e] = fma(pu, (double)b.x, o[2 * e]);
                    o[2 * e + 1] = fma(pu, (double)b.y, o[2 * e + 1]);
                }
            } else {
                const float* v4 = (const float*)&vr[u];
#pragma unroll
                for (int e = 0; e < EPL; e++) o[e] = fma(pu, (double)v4[e], o[e]);
            }
        }
    }
    // sum the token groups (same m everywhere): o over lanes with the same dims, l over the warp
#pragma unroll
    for (int off = LPT; off < 32; off <<= 1) {
#pragma unroll
        for (int e = 0; e < EPL; e++) o[e] += __shfl_xor_sync(0xffffffffu, o[e], off);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);

    if (nch > 1) {
        double* part = p.part + (((size_t)slot * NH + h) * p.max_chunks) * (2 + HD);
        if (tk == 0) {
#pragma unroll
            for (int e = 0; e < EPL; e++) part[(size_t)chunk * (2 + HD) + 2 + sub * EPL + e] = o[e];
            if (sub == 0) {
                part[(size_t)chunk * (2 + HD) + 0] = (double)m;
                part[(size_t)chunk * (2 + HD) + 1] = l;
            }
        }
        __threadfence();
        __syncwarp();
        int ticket = 0;
        if (lane == 0) ticket = atomicAdd(p.counter + (size_t)slot * NH + h, 1);
        ticket = __shfl_sync(0xffffffffu, ticket, 0);
        if (ticket != nch - 1) return;
        __threadfence();
        double M = -INFINITY;
        for (int c = 0; c < nch; c++) M = fmax(M, __ldcg(part + (size_t)c * (2 + HD)));
        l = 0.0;
#pragma unroll
        for (int e = 0; e < EPL; e++) o[e] = 0.0;
        for (int c = 0; c < nch; c++) {
            const double mc = __ldcg(part + (size_t)c * (2 + HD));
            const double w = mc == -INFINITY ? 0.0 : exp(mc - M);
            l = fma(__ldcg(part + (size_t)c * (2 + HD) + 1), w, l);
#pragma unroll
            for (int e = 0; e < EPL; e++) o[e] = fma(__ldcg(part + (size_t)c * (2 + HD) + 2 + sub * EPL + e), w, o[e]);
        }
        if (lane == 0) p.counter[(size_t)slot * NH + h] = 0;   // ready for the next launch
    }

    // finalize and quantize the head's 32 values (one Q8_0 block)
    float out[EPL], amax = 0.0f;
#pragma unroll
    for (int e = 0; e < EPL; e++) {
        out[e] = l > 0.0 ? (float)(o[e] / l) : 0.0f;
        amax = fmaxf(amax, fabsf(out[e]));
    }
#pragma unroll
    for (int off = 1; off < LPT; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    float dsc, id;
    q8_scale(amax, dsc, id);
    if (tk == 0) {
        int8_t* qo = p.out_q + (size_t)slot * D + h * HD + sub * EPL;
#pragma unroll
        for (int e = 0; e < EPL; e++) qo[e] = q8_val(out[e], id);
        if (sub == 0) p.out_d[(size_t)slot * (D / QK) + h] = f2h(dsc);
        if (p.out_f32) {
#pragma unroll
            for (int e = 0; e < EPL; e++) p.out_f32[(size_t)slot * D + h * HD + sub * EPL + e] = out[e];
        }
    }
}

void launch_decode_attention(const DecAttnParams& p, cudaStream_t s) {
    dim3 grid(NH / 4, p.max_chunks, p.B);
    if (p.kv_f32) k_decode_attn<float><<<grid, 128, 0, s>>>(p);
    else k_decode_attn<__half><<<grid, 128, 0, s>>>(p);
}

// ------------------------------------------------------------------ prefill
// One thread per query row of one head; keys visited in order, softmax-weighted sum carried in
// double and rounded once (see the decode kernel). Key/value tiles of 64 rows are staged in shared memory
// and read as broadcasts. Mask (src/gsv_ar.cpp:215-223) in-tile: text query (qi < T) sees text keys
// [0, T); semantic query sees keys [0, qi].
__global__ void __launch_bounds__(PREF_QTILE) k_prefill_attn(const PrefAttnParams p) {
    __shared__ float Ks[PREF_QTILE][HD];
    __shared__ float Vs[PREF_QTILE][HD];
    const int h = blockIdx.x;
    const PrefillTile tile = p.tiles[blockIdx.y];
    const int sq = tile.seq, q0 = tile.q0;
    const int start = p.seq_start[sq], S = p.seq_len[sq], T = p.text_len[sq];
    const int qi = q0 + threadIdx.x;
    const bool valid = qi < S;
    float q[HD], o[HD];
#pragma unroll
    for (int d = 0; d < HD; d++) q[d] = valid ? p.qkv[(size_t)(start + qi) * 3 * D + h * HD + d] : 0.0f;
    float m = -INFINITY;
    double l = 0.0, od[HD];
#pragma unroll
    for (int d = 0; d < HD; d++) od[d] = 0.0;
    const int kend = (q0 + PREF_QTILE <= T) ? T : max(T, min(S, q0 + PREF_QTILE));
    for (int kt = 0; kt < kend; kt += PREF_QTILE) {
        __syncthreads();
        {
            const int key = kt + threadIdx.x;
            const float* kr = p.qkv + (size_t)(start + key) * 3 * D + D + h * HD;
#pragma unroll
            for (int d4 = 0; d4 < HD / 4; d4++) {
                float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
                if (key < S) {
                    kv = *(const float4*)(kr + d4 * 4);
                    vv = *(const float4*)(kr + D + d4 * 4);
                }
                *(float4*)&Ks[threadIdx.x][d4 * 4] = kv;
                *(float4*)&Vs[threadIdx.x][d4 * 4] = vv;
            }
        }
        __syncthreads();
        const int nk = min(PREF_QTILE, kend - kt);
        for (int j = 0; j < nk; j++) {
            const int key = kt + j;
            const bool vis = valid && (qi < T ? key < T : key <= qi);
            if (!vis) continue;
            double dot = 0.0;
#pragma unroll
            for (int d = 0; d < HD; d++) dot += (double)__fmul_rn(q[d], Ks[j][d]);
            const float s = __fmul_rn((float)dot, p.scale);
            if (s > m) {
                const double r = m == -INFINITY ? 0.0 : exp((double)m - (double)s);
                l *= r;
#pragma unroll
                for (int d = 0; d < HD; d++) od[d] *= r;
                m = s;
            }
            const double pj = exp((double)s - (double)m);
            l += pj;
#pragma unroll
            for (int d = 0; d < HD; d++) od[d] = fma(pj, (double)Vs[j][d], od[d]);
        }
    }
    if (!valid) return;
    float amax = 0.0f;
#pragma unroll
    for (int d = 0; d < HD; d++) {
        o[d] = l > 0.0 ? (float)(od[d] / l) : 0.0f;
        amax = fmaxf(amax, fabsf(o[d]));
    }
    float dsc, id;
    q8_scale(amax, dsc, id);
    const size_t row = (size_t)(start + qi);
    int8_t* qo = p.out_q + row * D + h * HD;
#pragma unroll
    for (int d = 0; d < HD; d++) qo[d] = q8_val(o[d], id);
    p.out_d[row * (D / QK) + h] = f2h(dsc);
    if (p.out_f32) {
#pragma unroll
        for (int d = 0; d < HD; d++) p.out_f32[row * D + h * HD + d] = o[d];
    }
}

void launch_prefill_attention(const PrefAttnParams& p, cudaStream_t s) {
    if (p.n_tiles == 0) return;
    dim3 grid(NH, p.n_tiles);
    k_prefill_attn<<<grid, PREF_QTILE, 0, s>>>(p);
}

}  // namespace gsvcu
