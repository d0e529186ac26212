// attention.cu -- decode (split-KV flash decoding over paged KV) and prefix-masked prefill attention.
//
// Both follow ggml flash_attn_ext's arithmetic as the reference uses it (src/gsv_ar.cpp:257,331,404):
// score = (float)(sum_d (double)(q_d * k_d)) * (1/sqrt(32)), masked keys skipped, online softmax with
// expf, S = S*ms + vs and VKQ = VKQ*ms + v*vs, output VKQ * (1/S), then Q8_0-quantized (one head
// = one 32-value block) for the out-projection GEMM.
#include <cfloat>

#include "kernels.h"

namespace gsvcu {

// ------------------------------------------------------------------ decode
// Work item = (slot, head, chunk of ATT_CHUNK keys), one warp each, 4 heads per CTA.
// K/V rows of one head are 32 contiguous elements inside a 64-token page, so a warp reads
// 8 tokens x 64 B (F16) per 128-bit load instruction; 4 loads of K and 4 of V are in flight per lane.
// Chunks of one (slot, head) are merged by the last warp to finish (atomic ticket, no waiting).
template <typename KT>
__global__ void __launch_bounds__(128) k_decode_attn(const DecAttnParams p) {
    constexpr int EPL = 16 / sizeof(KT);     // elements per lane per load
    constexpr int LPT = HD / EPL;            // lanes per token
    constexpr int TPI = 32 / LPT;            // tokens per warp-load
    constexpr int U = 4;                     // loads in flight per lane (per K and per V)
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

    float m = -INFINITY, l = 0.0f, o[EPL];
#pragma unroll
    for (int e = 0; e < EPL; e++) o[e] = 0.0f;

    for (int base = k0; base < k1; base += TPI * U) {
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
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int kk = base + u * TPI + tk;
            float kf[EPL], vf[EPL];
            if (sizeof(KT) == 2) {
                const __half2* k2 = (const __half2*)&kr[u];
                const __half2* v2 = (const __half2*)&vr[u];
#pragma unroll
                for (int e = 0; e < EPL / 2; e++) {
                    const float2 a = __half22float2(k2[e]), b = __half22float2(v2[e]);
                    kf[2 * e] = a.x; kf[2 * e + 1] = a.y;
                    vf[2 * e] = b.x; vf[2 * e + 1] = b.y;
                }
            } else {
                const float* k4 = (const float*)&kr[u];
                const float* v4 = (const float*)&vr[u];
#pragma unroll
                for (int e = 0; e < EPL; e++) { kf[e] = k4[e]; vf[e] = v4[e]; }
            }
            double dot = 0.0;
#pragma unroll
            for (int e = 0; e < EPL; e++) dot += (double)__fmul_rn(q[e], kf[e]);
#pragma unroll
            for (int off = 1; off < LPT; off <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
            if (kk < k1) {
                const float s = __fmul_rn((float)dot, p.scale);
                if (s > m) {
                    const float ms = expf(__fsub_rn(m, s));
                    m = s;
#pragma unroll
                    for (int e = 0; e < EPL; e++) o[e] = __fadd_rn(__fmul_rn(o[e], ms), vf[e]);
                    l = fmaf(l, ms, 1.0f);
                } else {
                    const float vs = expf(__fsub_rn(s, m));
#pragma unroll
                    for (int e = 0; e < EPL; e++) o[e] = fmaf(vf[e], vs, o[e]);
                    l = __fadd_rn(l, vs);
                }
            }
        }
    }
    // merge the TPI token groups of the warp
#pragma unroll
    for (int off = LPT; off < 32; off <<= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
        const float l2 = __shfl_xor_sync(0xffffffffu, l, off);
        const float mn = fmaxf(m, m2);
        const float a = m == -INFINITY ? 0.0f : expf(__fsub_rn(m, mn));
        const float b = m2 == -INFINITY ? 0.0f : expf(__fsub_rn(m2, mn));
#pragma unroll
        for (int e = 0; e < EPL; e++) {
            const float o2 = __shfl_xor_sync(0xffffffffu, o[e], off);
            o[e] = fmaf(o2, b, __fmul_rn(o[e], a));
        }
        l = fmaf(l2, b, __fmul_rn(l, a));
        m = mn;
    }

    if (nch > 1) {
        float* part = p.part + (((size_t)slot * NH + h) * p.max_chunks) * (2 + HD);
        if (tk == 0) {
#pragma unroll
            for (int e = 0; e < EPL; e++) part[(size_t)chunk * (2 + HD) + 2 + sub * EPL + e] = o[e];
            if (sub == 0) {
                part[(size_t)chunk * (2 + HD) + 0] = m;
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
        float M = -INFINITY;
        for (int c = 0; c < nch; c++) M = fmaxf(M, __ldcg(part + (size_t)c * (2 + HD)));
        l = 0.0f;
#pragma unroll
        for (int e = 0; e < EPL; e++) o[e] = 0.0f;
        for (int c = 0; c < nch; c++) {
            const float mc = __ldcg(part + (size_t)c * (2 + HD));
            const float lc = __ldcg(part + (size_t)c * (2 + HD) + 1);
            const float w = mc == -INFINITY ? 0.0f : expf(__fsub_rn(mc, M));
            l = fmaf(lc, w, l);
#pragma unroll
            for (int e = 0; e < EPL; e++) o[e] = fmaf(__ldcg(part + (size_t)c * (2 + HD) + 2 + sub * EPL + e), w, o[e]);
        }
        if (lane == 0) p.counter[(size_t)slot * NH + h] = 0;   // ready for the next launch
    }

    // finalize and quantize the head's 32 values (one Q8_0 block)
    const float inv = l == 0.0f ? 0.0f : __fdiv_rn(1.0f, l);
    float out[EPL], amax = 0.0f;
#pragma unroll
    for (int e = 0; e < EPL; e++) {
        out[e] = __fmul_rn(o[e], inv);
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
// One thread per query row of one head; keys visited in order, so the online-softmax sequence is
// the same as the reference's per-row loop. Key/value tiles of 64 rows are staged in shared memory
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
    for (int d = 0; d < HD; d++) {
        q[d] = valid ? p.qkv[(size_t)(start + qi) * 3 * D + h * HD + d] : 0.0f;
        o[d] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;
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
                const float ms = expf(__fsub_rn(m, s));
                m = s;
#pragma unroll
                for (int d = 0; d < HD; d++) o[d] = __fadd_rn(__fmul_rn(o[d], ms), Vs[j][d]);
                l = fmaf(l, ms, 1.0f);
            } else {
                const float vs = expf(__fsub_rn(s, m));
#pragma unroll
                for (int d = 0; d < HD; d++) o[d] = fmaf(Vs[j][d], vs, o[d]);
                l = __fadd_rn(l, vs);
            }
        }
    }
    if (!valid) return;
    const float inv = l == 0.0f ? 0.0f : __fdiv_rn(1.0f, l);
    float amax = 0.0f;
#pragma unroll
    for (int d = 0; d < HD; d++) {
        o[d] = __fmul_rn(o[d], inv);
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
