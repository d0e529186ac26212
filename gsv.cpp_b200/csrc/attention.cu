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
// Work item = (slot, head, 64-key page), one warp each, 4 heads (warps) per CTA. Lane 0 stages the
// head's K and V rows of the page into shared memory with two TMA bulk copies (cp.async.bulk, no
// multicast) completing on one mbarrier; the warp then reads them from shared memory.
//
// Arithmetic: a fixed float evaluation order, restated operation for operation by the CPU oracle
// (decode_attention_canonical), so the two agree bit for bit. Lane l = 4*g + s owns dims 8s..8s+7 and
// the keys t = 8u + g (u = 0..7) of its page ("token group" g):
//   score    D_s = fma chain over the lane's 8 dims from 0; dot = (D0 + D1) + (D2 + D3); s_t = dot*scale
//   page max m = max_t s_t;  p_t = exp_canon(s_t - m)   (own float exp, common.cuh; same on the CPU)
//   sums     L_g = sum over u of p_t (ascending u), O_g[d] = fma chain p_t * v_t[d] (ascending u), then
//            l = ((L0+L1)+(L2+L3))+((L4+L5)+(L6+L7)), o[d] likewise
//   merge    over the pages c = 0..n-1 in order: M = max m_c, w = exp_canon(m_c - M),
//            L = fma(w, l_c, L), O[d] = fma(w, o_c[d], O[d]); out = O / L.
// Pages of one (slot, head) are merged by the last warp to finish (atomic ticket, no waiting).

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// Bulk global -> shared copy completing on an mbarrier (no multicast). K/V rows are read once per
// layer-step: they are marked evict-first in L2, so the streamed pages do not push out what the step
// reuses (weights, slot state, page partials).
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    const uint64_t pol = l2_evict_first();
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(pol)
        : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for phase 0 of an mbarrier; warp-uniform result (false: `limit` polls went by).
constexpr uint32_t MBAR_POLL_LIMIT = 1u << 22;
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t limit) {
    uint32_t it = 0;
    while (!mbar_try_wait(bar, 0)) {
        if (++it == limit) break;
    }
    return __all_sync(0xffffffffu, it < limit);
}

// 8 consecutive values of a K/V row slice from shared memory, as floats.
template <typename KT>
__device__ __forceinline__ void load8(const uint8_t* p, float (&f)[8]) {
    if (sizeof(KT) == 2) {
        const uint4 r = *(const uint4*)p;
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            f[2 * i] = __half2float(__ushort_as_half((unsigned short)(w[i] & 0xffffu)));
            f[2 * i + 1] = __half2float(__ushort_as_half((unsigned short)(w[i] >> 16)));
        }
    } else {
        const float4 a = *(const float4*)p, b = *(const float4*)(p + 16);
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
        f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    }
}

// Out = o / l for the head, quantized to one Q8_0 block (the head's 32 values); lane (g, s) holds dims
// 8s..8s+7, group g = 0 writes.
__device__ __forceinline__ void decode_write_out(const DecAttnParams& p, int slot, int h, int g, int sub,
                                                 const float (&o)[8], float l) {
    float out[8], amax = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; e++) {
        out[e] = __fdiv_rn(o[e], l);
        amax = fmaxf(amax, fabsf(out[e]));
    }
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    float dsc, id;
    q8_scale(amax, dsc, id);
    if (g == 0) {
        int8_t* qo = p.out_q + (size_t)slot * D + h * HD + sub * 8;
        uint32_t w0 = 0, w1 = 0;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            w0 |= (uint32_t)(uint8_t)q8_val(out[e], id) << (8 * e);
            w1 |= (uint32_t)(uint8_t)q8_val(out[e + 4], id) << (8 * e);
        }
        *(uint2*)qo = make_uint2(w0, w1);
        if (sub == 0) p.out_d[(size_t)slot * (D / QK) + h] = l == l ? f2h(dsc) : (uint16_t)0x7e00u;
        if (p.out_f32) {
            float4* of = (float4*)(p.out_f32 + (size_t)slot * D + h * HD + sub * 8);
            of[0] = make_float4(out[0], out[1], out[2], out[3]);
            of[1] = make_float4(out[4], out[5], out[6], out[7]);
        }
    }
}

__device__ __forceinline__ bool decode_slot(const DecAttnParams& p, int slot, int& kvpos) {
    if (p.st) {
        kvpos = p.st[slot].kvpos;
        return p.st[slot].decode_now != 0;
    }
    kvpos = p.kvpos[slot];
    return p.active[slot] != 0;
}

template <typename KT> struct DecShape {
    static constexpr int ROWB = HD * (int)sizeof(KT);   // bytes per token row of one head
    static constexpr int PGB = PAGE * ROWB;             // K (or V) bytes of one head in one page
    static constexpr int WARPB = 2 * PGB;               // K + V rows of one warp
    static constexpr size_t SMEM = (size_t)4 * WARPB + 4 * 8;   // 4 warps + 4 mbarriers
};

// One warp: the pinned-order softmax of one head over one staged page (n keys of K rows ks, V rows vs)
// for query q (lane (g, s) holds dims 8s..8s+7); returns the page max m, sum l and o (lane's 8 dims).
// FULL: n == PAGE, so no key needs the bound test (straight-line code for the common, full pages).
template <typename KT, bool FULL>
__device__ __forceinline__ void page_softmax(const uint8_t* ks, const uint8_t* vs, int n, const float (&q)[8],
                                             float scale, float& m_out, float& l_out, float (&o)[8]) {
    using S = DecShape<KT>;
    const int lane = threadIdx.x & 31, sub = lane & 3, g = lane >> 2;
    // scores of the lane's 8 keys t = 8u + g
    float sc[8], m = -INFINITY;
#pragma unroll
    for (int u = 0; u < 8; u++) {
        const int t = 8 * u + g;
        float d = 0.0f;
        if (FULL || t < n) {
            float kf[8];
            load8<KT>(ks + (size_t)t * S::ROWB + sub * 8 * sizeof(KT), kf);
#pragma unroll
            for (int e = 0; e < 8; e++) d = fmaf(q[e], kf[e], d);
        }
        d = __fadd_rn(d, __shfl_xor_sync(0xffffffffu, d, 1));
        d = __fadd_rn(d, __shfl_xor_sync(0xffffffffu, d, 2));
        sc[u] = (FULL || t < n) ? __fmul_rn(d, scale) : -INFINITY;
        m = fmaxf(m, sc[u]);
    }
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    // weights: lane (g, s) evaluates keys u = s and u = s + 4 of its group, then they are shared
    float sa = sc[0], sb = sc[4];
#pragma unroll
    for (int u = 1; u < 4; u++)
        if (sub == u) { sa = sc[u]; sb = sc[u + 4]; }
    const float pa = exp_canon(sa - m), pb = exp_canon(sb - m);   // exp_canon(-inf) = 0 for keys past the end
    float l = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; e++) o[e] = 0.0f;
#pragma unroll
    for (int u = 0; u < 8; u++) {
        const float pu = __shfl_sync(0xffffffffu, u < 4 ? pa : pb, 4 * g + (u & 3));
        const int t = 8 * u + g;
        if (FULL || t < n) {
            float vf[8];
            load8<KT>(vs + (size_t)t * S::ROWB + sub * 8 * sizeof(KT), vf);
            l = __fadd_rn(l, pu);
#pragma unroll
            for (int e = 0; e < 8; e++) o[e] = fmaf(pu, vf[e], o[e]);
        }
    }
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
        l = __fadd_rn(l, __shfl_xor_sync(0xffffffffu, l, off));
#pragma unroll
        for (int e = 0; e < 8; e++) o[e] = __fadd_rn(o[e], __shfl_xor_sync(0xffffffffu, o[e], off));
    }
    m_out = m;
    l_out = l;
}

// One CTA per (4-head group, page, slot); warp = head. Pages of sequences longer than one page leave a
// partial {m, l, -, -, o[32]} for k_decode_merge; one-page sequences are finished here.
template <typename KT>
__global__ void __launch_bounds__(128) k_decode_attn(const DecAttnParams p) {
    using S = DecShape<KT>;
    extern __shared__ __align__(128) uint8_t sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // In the decode step (p.st set) the slot state, the page list and every KV row but this step's are
    // at least two kernels old, so they are read before griddep_wait; op-entry inputs may come from the
    // previous kernel and are read after it.
    const bool early = p.st != nullptr;
    if (!early) {
        griddep_wait();
        griddep_launch();
    }
    int slot, chunk, h, kvpos, ppage = -1;   // ppage: physical page when the list carries it
    bool act;
    if (p.work) {   // compacted list: CTA = (item, head group), trailing CTAs past the list exit
        const int item = p.work_base[p.group] + (int)(blockIdx.x >> 2);
        h = (int)(blockIdx.x & 3) * 4 + warp;
        act = item < p.work_base[p.group + 1];
        slot = 0; chunk = 0; kvpos = 0;
        if (act) {
            const int4 w = p.work[item];
            slot = w.x;
            chunk = w.y & 0xff;
            kvpos = w.y >> 8;
            ppage = w.z;
        }
    } else {
        slot = p.slot0 + blockIdx.z;
        chunk = blockIdx.y;
        h = blockIdx.x * 4 + warp;
        act = decode_slot(p, slot, kvpos);
    }
    const int nkeys = kvpos + 1, k0 = chunk * PAGE;
    if (!act || k0 >= nkeys) {
        if (early) griddep_wait();
        return;
    }
    const int n = min(PAGE, nkeys - k0);
    const int sub = lane & 3, g = lane >> 2;

    uint8_t* ks = sm + (size_t)warp * S::WARPB;
    uint8_t* vs = ks + S::PGB;
    const uint32_t bar = smem_u32((uint64_t*)(sm + 4 * S::WARPB) + warp);
    const bool fresh = chunk == kvpos / PAGE;   // holds the key the previous kernel wrote this step
    auto stage = [&]() {
        const int page = ppage >= 0 ? ppage : p.block_table[(size_t)slot * p.max_pages + chunk];
        const KT* kp = (const KT*)p.pool + (size_t)page * p.n_layer * 2 * NH * PAGE * HD +
                       ((size_t)p.layer * 2 * NH + h) * PAGE * HD;
        const uint32_t bytes = (uint32_t)n * S::ROWB;
        mbar_expect_tx(bar, 2 * bytes + p.fault_extra_tx);   // fault_extra_tx: 0 except under a test's fault
        bulk_g2s(smem_u32(ks), kp, bytes, bar);
        bulk_g2s(smem_u32(vs), kp + (size_t)NH * PAGE * HD, bytes, bar);
    };
    if (lane == 0) {
        mbar_init(bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        if (!(early && fresh)) stage();
    }
    if (early) {
        griddep_wait();
        griddep_launch();
        if (fresh && lane == 0) stage();
    }
    float q[8];
    {
        const float4* qp = (const float4*)(p.q + (size_t)slot * p.q_stride + h * HD + sub * 8);
        const float4 a = qp[0], b = qp[1];
        q[0] = a.x; q[1] = a.y; q[2] = a.z; q[3] = a.w;
        q[4] = b.x; q[5] = b.y; q[6] = b.z; q[7] = b.w;
    }
    __syncwarp();
    const uint32_t limit = p.poll_limit ? p.poll_limit : MBAR_POLL_LIMIT;
    if (!mbar_wait_bounded(bar, limit)) {   // the page never arrived: flag it, wait (bounded) for the copies
        if (lane == 0 && p.err) atomicExch(p.err, 1);
        (void)mbar_wait_bounded(bar, limit);
    }

    float m, l, o[8];
    if (n == PAGE) page_softmax<KT, true>(ks, vs, n, q, p.scale, m, l, o);
    else page_softmax<KT, false>(ks, vs, n, q, p.scale, m, l, o);
    if (nkeys <= PAGE && !p.partials_only) {
        decode_write_out(p, slot, h, g, sub, o, l);
        return;
    }
    if (g == 0) {
        const size_t item = ((size_t)slot * NH + h) * p.max_chunks + chunk;
        float* po = p.part + item * HD + sub * 8;
        __stcg((float4*)po, make_float4(o[0], o[1], o[2], o[3]));
        __stcg((float4*)(po + 4), make_float4(o[4], o[5], o[6], o[7]));
        if (sub == 0) __stcg((float2*)p.part_ml + item, make_float2(m, l));
    }
}

// Merge of the page partials of sequences longer than one page: warp per (slot, head), pages in
// order (M = max m, w = exp_canon(m - M), L = fma(w, l, L), O = fma(w, o, O)), 32 pages per batch staged
// in shared memory by lane-parallel loads.
__global__ void __launch_bounds__(128) k_decode_merge(const DecAttnParams p) {
    __shared__ __align__(16) float sbuf[4][64 + 32 * 32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int item = blockIdx.x * 4 + warp;
    griddep_wait();
    griddep_launch();
    if (item >= p.B * NH) return;
    const int slot = p.slot0 + item / NH, h = item % NH;
    int kvpos;
    if (!decode_slot(p, slot, kvpos)) return;
    const int nch = min((kvpos + PAGE) / PAGE, p.max_chunks);   // the page grid covers max_chunks pages
    if (nch <= 1) return;
    const int sub = lane & 3, g = lane >> 2;
    const size_t item0 = ((size_t)slot * NH + h) * p.max_chunks;
    const float* po = p.part + item0 * HD;
    const float2* pml = (const float2*)p.part_ml + item0;
    float M = -INFINITY;
    for (int c = lane; c < nch; c += 32) M = fmaxf(M, __ldcg((const float*)(pml + c)));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    float* sw = sbuf[warp];          // [32] page weights
    float* sl = sbuf[warp] + 32;     // [32] page sums
    float* so = sbuf[warp] + 64;     // [32][32] page outputs
    float L = 0.0f, O[8];
#pragma unroll
    for (int e = 0; e < 8; e++) O[e] = 0.0f;
    for (int c0 = 0; c0 < nch; c0 += 32) {
        const int cnt = min(32, nch - c0);
        if (lane < cnt) {
            const float2 ml = __ldcg(pml + c0 + lane);
            sw[lane] = exp_canon(ml.x - M);
            sl[lane] = ml.y;
        }
        for (int i = lane; i < cnt * 8; i += 32) {
            const int c = i >> 3, j = i & 7;
            *(float4*)(so + c * 32 + j * 4) = __ldcg((const float4*)(po + (size_t)(c0 + c) * HD + j * 4));
        }
        __syncwarp();
        for (int c = 0; c < cnt; c++) {
            const float w = sw[c];
            L = fmaf(w, sl[c], L);
            const float4 a = *(const float4*)(so + c * 32 + sub * 8), b = *(const float4*)(so + c * 32 + sub * 8 + 4);
            O[0] = fmaf(w, a.x, O[0]); O[1] = fmaf(w, a.y, O[1]); O[2] = fmaf(w, a.z, O[2]); O[3] = fmaf(w, a.w, O[3]);
            O[4] = fmaf(w, b.x, O[4]); O[5] = fmaf(w, b.y, O[5]); O[6] = fmaf(w, b.z, O[6]); O[7] = fmaf(w, b.w, O[7]);
        }
        __syncwarp();
    }
    decode_write_out(p, slot, h, g, sub, O, L);
}

cudaError_t prefill_attn_init_device();   // below, after the prefill kernels

cudaError_t attention_init_device() {
    cudaError_t e = cudaFuncSetAttribute(k_decode_attn<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)DecShape<__half>::SMEM);
    if (e != cudaSuccess) return e;
    if ((e = prefill_attn_init_device()) != cudaSuccess) return e;
    return cudaFuncSetAttribute(k_decode_attn<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)DecShape<float>::SMEM);
}

// One CTA of 1024 threads: slot-major exclusive prefix of the slots' page counts, then the items.
__global__ void __launch_bounds__(1024) k_page_list(const SlotState* st, int M, int split, const int32_t* block_table,
                                                   int max_pages, int4* work, int32_t* base) {
    griddep_wait();
    griddep_launch();
    __shared__ int wsum[32];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int C = (M + 1023) / 1024;   // slots per thread (<= 4)
    int np[4], kp[4], cnt = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int slot = t * C + i;
        np[i] = 0;
        kp[i] = 0;
        if (i < C && slot < M && st[slot].decode_now) {
            kp[i] = st[slot].kvpos;
            np[i] = kp[i] / PAGE + 1;
        }
        cnt += np[i];
    }
    int x = cnt;   // inclusive scan over the block
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += y;
    }
    if (lane == 31) wsum[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = wsum[lane];
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, off);
            if (lane >= off) w += y;
        }
        wsum[lane] = w;
    }
    __syncthreads();
    int off = x - cnt + (warp ? wsum[warp - 1] : 0);   // exclusive prefix of this thread's first slot
    if (t == 0) base[0] = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int slot = t * C + i;
        if (i < C && slot == split) base[1] = off;
        for (int pg = 0; pg < np[i]; pg++)
            work[off + pg] = make_int4(slot, pg | (kp[i] << 8), block_table[(size_t)slot * max_pages + pg], 0);
        off += np[i];
    }
    if (t == 1023) {
        base[2] = off;
        if (split >= M) base[1] = off;
    }
}

void launch_page_list(const SlotState* st, int M, int split, const int32_t* block_table, int max_pages, int4* work,
                      int32_t* base, cudaStream_t s) {
    launch_pdl(k_page_list, dim3(1), dim3(1024), 0, s, st, M, split, block_table, max_pages, work, base);
}

int launch_decode_attention(const DecAttnParams& p, cudaStream_t s) {
    dim3 grid(NH / 4, p.max_chunks, p.B);
    if (p.work) grid = dim3(4 * p.B * p.max_chunks);
    if (p.kv_f32) launch_pdl(k_decode_attn<float>, grid, dim3(128), DecShape<float>::SMEM, s, p);
    else launch_pdl(k_decode_attn<__half>, grid, dim3(128), DecShape<__half>::SMEM, s, p);
    if (p.max_chunks <= 1 || p.partials_only) return 1;
    launch_pdl(k_decode_merge, dim3((p.B * NH + 3) / 4), dim3(128), 0, s, p);
    return 2;
}

// ------------------------------------------------------------------ prefill
// Mask (src/gsv_ar.cpp:215-223): a text query (qi < T) sees the text keys [0, T); a semantic query
// sees the keys [0, qi].
// Prefill attention on the FP64 tensor cores (mma.sync m8n8k4 .f64). Scores q.k are products exact in
// double summed in double, rounded to float and scaled in float (ggml's order); the softmax weights
// exp(s - m) and their sums and the weighted sum of V are carried in double and rounded once. The
// running maximum is taken per 64-key tile; in double the result differs from a key-by-key running
// maximum only at the 1e-16 level, so it rounds to the same float (except at a rounding tie, as any
// change of double summation order).
// CTA = 64 queries of one head of one sequence (one PrefillTile), 8 warps of 8 queries.
// Per 64-key tile, staged in shared memory as double: warp w computes its 8 x 64 score block as 8
// n-tiles of 8 keys (8 k-steps of 4 dims each), lane holding S[row = lane / 4][key = 8t + 2 (lane % 4)
// + i]. That is exactly the A operand of P.V when k-step (t, i) takes keys 8t + 2k + i (k = 0..3): the
// weights never move between lanes, and the V operand is read in that key order.
constexpr int PA_KSTR = HD + 4;   // doubles per staged K / V row: the fragment loads are conflict-free
constexpr size_t PA_SMEM = (size_t)4 * PREF_QTILE * PA_KSTR * 8;   // K and V, two tiles each

__device__ __forceinline__ void dmma884(double& d0, double& d1, double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
                 : "+d"(d0), "+d"(d1)
                 : "d"(a), "d"(b));
}

__global__ void __launch_bounds__(256) k_prefill_attn_mma(const PrefAttnParams p) {
    // two key tiles: the next tile's K / V rows are loaded into registers while this one is used
    extern __shared__ __align__(16) double pa_sm[];
    double(*Ks)[PREF_QTILE][PA_KSTR] = (double(*)[PREF_QTILE][PA_KSTR])pa_sm;
    double(*Vs)[PREF_QTILE][PA_KSTR] = (double(*)[PREF_QTILE][PA_KSTR])(pa_sm + 2 * PREF_QTILE * PA_KSTR);
    const int h = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r = lane >> 2, c = lane & 3;   // fragment row (query) and column group
    griddep_wait();
    griddep_launch();
    const PrefillTile tile = p.tiles[blockIdx.y];
    const int sq = tile.seq, q0 = tile.q0;
    const int start = p.seq_start[sq], S = p.seq_len[sq], T = p.text_len[sq];
    const int qi = q0 + warp * 8 + r;   // this lane's query row
    const bool valid = qi < S;
    const int kend = (q0 + PREF_QTILE <= T) ? T : max(T, min(S, q0 + PREF_QTILE));
    // thread tid stages float4 number tid and tid + 256 of the tile's 64 keys x 8 float4 (K and V)
    float4 kr[2], vr[2];
    auto fetch = [&](int kt) {
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int i = tid + 256 * u, key = i >> 3, d4 = (i & 7) * 4;
            kr[u] = vr[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (kt + key < S) {
                const float* src = p.qkv + (size_t)(start + kt + key) * 3 * D + D + h * HD + d4;
                kr[u] = *(const float4*)src;
                vr[u] = *(const float4*)(src + D);
            }
        }
    };
    auto put = [&](int b) {
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int i = tid + 256 * u, key = i >> 3, d4 = (i & 7) * 4;
            *(double2*)&Ks[b][key][d4] = make_double2(kr[u].x, kr[u].y);
            *(double2*)&Ks[b][key][d4 + 2] = make_double2(kr[u].z, kr[u].w);
            *(double2*)&Vs[b][key][d4] = make_double2(vr[u].x, vr[u].y);
            *(double2*)&Vs[b][key][d4 + 2] = make_double2(vr[u].z, vr[u].w);
        }
    };
    fetch(0);
    double qa[HD / 4];                   // A fragments of Q: Q[qi][4 ks + c]
#pragma unroll
    for (int ks = 0; ks < HD / 4; ks++)
        qa[ks] = valid ? (double)p.qkv[(size_t)(start + qi) * 3 * D + h * HD + 4 * ks + c] : 0.0;
    float m = -INFINITY;
    double lp = 0.0;                     // this lane's share of the row's weight sum
    double o[HD / 8][2];                 // O[qi][8 dn + 2c + e]
#pragma unroll
    for (int dn = 0; dn < HD / 8; dn++) o[dn][0] = o[dn][1] = 0.0;
    put(0);
    int b = 0;
    for (int kt = 0; kt < kend; kt += PREF_QTILE, b ^= 1) {
        __syncthreads();   // tile b staged; every warp is done with tile b ^ 1
        if (kt + PREF_QTILE < kend) fetch(kt + PREF_QTILE);
        // scores: n-tile t = keys kt + 8t .. +7
        float sc[8][2];
        float tmax = -INFINITY;
#pragma unroll
        for (int t = 0; t < 8; t++) {
            double d0 = 0.0, d1 = 0.0;
#pragma unroll
            for (int ks = 0; ks < HD / 4; ks++) dmma884(d0, d1, qa[ks], Ks[b][8 * t + r][4 * ks + c]);
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int key = kt + 8 * t + 2 * c + e;
                const bool vis = valid && key < kend && (qi < T ? key < T : key <= qi);
                const float sv = __fmul_rn((float)(e ? d1 : d0), p.scale);
                sc[t][e] = vis ? sv : -INFINITY;
                tmax = fmaxf(tmax, sc[t][e]);
            }
        }
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
        const float mn = fmaxf(m, tmax);
        if (mn > m && m != -INFINITY) {   // rescale the row's sums to the new maximum
            const double rs = exp((double)m - (double)mn);
            lp *= rs;
#pragma unroll
            for (int dn = 0; dn < HD / 8; dn++) {
                o[dn][0] *= rs;
                o[dn][1] *= rs;
            }
        }
        m = mn;
        // weights and O += P.V
#pragma unroll
        for (int t = 0; t < 8; t++) {
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const double pw = sc[t][e] == -INFINITY ? 0.0 : exp((double)sc[t][e] - (double)m);
                lp += pw;
#pragma unroll
                for (int dn = 0; dn < HD / 8; dn++)
                    dmma884(o[dn][0], o[dn][1], pw, Vs[b][8 * t + 2 * c + e][8 * dn + r]);
            }
        }
        if (kt + PREF_QTILE < kend) put(b ^ 1);
    }
    double l = lp;
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    float of[HD / 8][2], amax = 0.0f;
#pragma unroll
    for (int dn = 0; dn < HD / 8; dn++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
            of[dn][e] = l > 0.0 ? (float)(o[dn][e] / l) : 0.0f;
            amax = fmaxf(amax, fabsf(of[dn][e]));
        }
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    if (!valid) return;
    float dsc, id;
    q8_scale(amax, dsc, id);
    const size_t row = (size_t)(start + qi);
    int8_t* qo = p.out_q + row * D + h * HD;
#pragma unroll
    for (int dn = 0; dn < HD / 8; dn++)
#pragma unroll
        for (int e = 0; e < 2; e++) qo[8 * dn + 2 * c + e] = q8_val(of[dn][e], id);
    if (c == 0) p.out_d[row * (D / QK) + h] = f2h(dsc);
    if (p.out_f32) {
#pragma unroll
        for (int dn = 0; dn < HD / 8; dn++)
#pragma unroll
            for (int e = 0; e < 2; e++) p.out_f32[row * D + h * HD + 8 * dn + 2 * c + e] = of[dn][e];
    }
}

cudaError_t prefill_attn_init_device() {
    return cudaFuncSetAttribute(k_prefill_attn_mma, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PA_SMEM);
}

void launch_prefill_attention(const PrefAttnParams& p, cudaStream_t s) {
    if (p.n_tiles == 0) return;
    dim3 grid(NH, p.n_tiles);
    launch_pdl(k_prefill_attn_mma, grid, dim3(256), PA_SMEM, s, p);
}

}  // namespace gsvcu
