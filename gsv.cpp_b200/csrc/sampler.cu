// sampler.cu -- on-device sampler (replaces the host sampler of reference src/gsv_sampler.cpp and the
// per-step loop body of src/gsv_ar.cpp:764-785). One CTA per sequence slot.
//
// Order and arithmetic follow gsv_logits_to_probs / gsv_sample exactly:
//   EOS masked while step < 11; repetition penalty applied once per occurrence in the window of the
//   last 4096 tokens (a token seen c times is multiplied (negative) or divided (positive) c times);
//   top-p over a stable descending order with a serial softmax/cumulative sum; temperature division;
//   top-k pivot = k-th largest value (ties kept); softmax with a serial float sum in index order;
//   draws q_i = -logf(1 - U_i), U_i = (xorshift64*() >> 40) / 2^24, i = 0..V-1 in order, and the
//   first index maximising p_i / q_i over p_i > 0 (0 elsewhere).
// The V sequential xorshift draws are split over the 32 lanes of a warp: lane j jumps to draw j*dpl
// with a precomputed GF(2) matrix T^(j*dpl) (xorshift64 is linear over GF(2)) and steps from there.
#include <cfloat>

#include "kernels.h"

namespace gsvcu {

constexpr int SAMP_T = 256;
constexpr int VMAX = 1280;
constexpr int SORT_N = 2048;

__device__ __forceinline__ uint32_t f2key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
    const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(u);
}

// expf / logf of the reference sampler (glibc, near correctly rounded) evaluated through double and
// rounded once: equal to glibc's results except in the rare inputs where those are not correctly rounded.
__device__ __forceinline__ float exp_f(float x) { return (float)exp((double)x); }
__device__ __forceinline__ float log_f(float x) { return (float)log((double)x); }

__device__ __forceinline__ uint64_t xs_step(uint64_t s) {
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    return s;
}

__global__ void __launch_bounds__(SAMP_T) k_sampler(const SamplerParams p) {
    const int slot = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // Before the wait for the logits: the jump matrices (constant since initialisation), transposed to
    // [bit][lane] so that the 32 lanes read 32 consecutive words, and the slot's state and repetition
    // counts, which the previous step's sampler and step preparation wrote (two or more kernels ago).
    __shared__ uint64_t jmp[64 * 32];
    for (int e = tid; e < 64 * 32; e += SAMP_T) jmp[(e & 63) * 32 + (e >> 6)] = p.jump[e];
    SlotState* st = p.st + slot;
    if (!st->active) {
        griddep_wait();
        return;
    }
    const int V = p.V;
    const int top_k = st->top_k;
    const float top_p = st->top_p, temperature = st->temperature, rep = st->rep;
    const uint16_t* cnt_row = p.counts + (size_t)slot * V;
    int cnt4[(VMAX + SAMP_T - 1) / SAMP_T];   // this thread's counts, i = tid + SAMP_T * j
#pragma unroll
    for (int j = 0; j < (VMAX + SAMP_T - 1) / SAMP_T; j++) {
        const int i = tid + SAMP_T * j;
        cnt4[j] = (rep != 1.0f && i < V) ? cnt_row[i] : 0;
    }
    griddep_wait();
    griddep_launch();
    __shared__ float lg[VMAX];
    __shared__ float pr[VMAX];
    __shared__ float sv[SORT_N];
    __shared__ int16_t si[SORT_N];
    __shared__ uint32_t hist[256];
    __shared__ float red[SAMP_T / 32];
    __shared__ uint32_t sel_prefix, sel_krem;
    __shared__ int s_tok;
    const int idx = st->n_samp;

    for (int i = tid; i < VMAX; i += SAMP_T) lg[i] = i < V ? p.logits[(size_t)slot * V + i] : -INFINITY;
    __syncthreads();
    if (tid == 0 && idx < 11) lg[p.eos] = -INFINITY;   // src/gsv_ar.cpp:768
    __syncthreads();

    // 1) repetition penalty
    if (rep != 1.0f) {
#pragma unroll
        for (int j = 0; j < (VMAX + SAMP_T - 1) / SAMP_T; j++) {
            const int i = tid + SAMP_T * j, c = cnt4[j];
            if (c) {
                float l = lg[i];
                for (int r = 0; r < c; r++) l = l < 0.0f ? __fmul_rn(l, rep) : __fdiv_rn(l, rep);
                lg[i] = l;
            }
        }
        __syncthreads();
    }

    // 2) top-p (nucleus) over a stable descending order
    if (top_p < 1.0f) {
        for (int i = tid; i < SORT_N; i += SAMP_T) {
            sv[i] = i < V ? lg[i] : -INFINITY;
            si[i] = (int16_t)i;
        }
        for (int size = 2; size <= SORT_N; size <<= 1) {
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                __syncthreads();
                for (int e = tid; e < SORT_N / 2; e += SAMP_T) {
                    const int i = 2 * e - (e & (stride - 1));
                    const int j = i + stride;
                    const float vi = sv[i], vj = sv[j];
                    const int ii = si[i], ij = si[j];
                    // "i before j" in the final order: larger value, or equal value and smaller index
                    const bool before = vi > vj || (vi == vj && ii < ij);
                    const bool desc = (i & size) == 0;
                    if (desc != before) {
                        sv[i] = vj; sv[j] = vi;
                        si[i] = (int16_t)ij; si[j] = (int16_t)ii;
                    }
                }
            }
        }
        __syncthreads();
        const float mx = sv[0];
        for (int k = tid; k < V; k += SAMP_T) pr[k] = exp_f(__fsub_rn(sv[k], mx));
        __syncthreads();
        if (tid == 0) {
            float sum = 0.0f;
            for (int k = 0; k < V; k++) sum = __fadd_rn(sum, pr[k]);
            const float inv_sum = __fdiv_rn(1.0f, sum);
            float cum = 0.0f;
            for (int k = 0; k < V; k++) {
                cum = fmaf(pr[k], inv_sum, cum);
                if (k > 0 && cum > top_p) lg[si[k]] = -INFINITY;
            }
        }
        __syncthreads();
    }

    // 3) temperature
    {
        const float t = fmaxf(temperature, 1e-5f);
        for (int i = tid; i < V; i += SAMP_T) lg[i] = __fdiv_rn(lg[i], t);
        __syncthreads();
    }

    // 4) top-k: exact k-th largest value by 4-pass radix select on order-preserving keys
    if (top_k > 0 && top_k < V) {
        if (tid == 0) { sel_prefix = 0u; sel_krem = (uint32_t)top_k; }
        for (int pass = 0; pass < 4; pass++) {
            const int shift = 24 - 8 * pass;
            const uint32_t mask = pass == 0 ? 0u : (0xffffffffu << (shift + 8));
            hist[tid] = 0u;
            __syncthreads();
            const uint32_t prefix = sel_prefix;
            for (int i = tid; i < V; i += SAMP_T) {
                const uint32_t key = f2key(lg[i]);
                if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
            }
            __syncthreads();
            if (warp == 0) {
                // lane l owns digits 255-8l .. 248-8l (descending)
                uint32_t c[8], tot = 0;
#pragma unroll
                for (int j = 0; j < 8; j++) { c[j] = hist[255 - 8 * lane - j]; tot += c[j]; }
                uint32_t incl = tot;
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const uint32_t v = __shfl_up_sync(0xffffffffu, incl, off);
                    if (lane >= off) incl += v;
                }
                const uint32_t excl = incl - tot;
                const uint32_t krem = sel_krem;
                __syncwarp();
                if (excl < krem && krem <= incl) {
                    uint32_t run = excl;
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        if (run + c[j] >= krem) {
                            sel_prefix = prefix | ((uint32_t)(255 - 8 * lane - j) << shift);
                            sel_krem = krem - run;
                            break;
                        }
                        run += c[j];
                    }
                }
            }
            __syncthreads();
        }
        const float pivot = key2f(sel_prefix);
        for (int i = tid; i < V; i += SAMP_T)
            if (lg[i] < pivot) lg[i] = -INFINITY;
        __syncthreads();
    }

    // 5) softmax
    float mx = -INFINITY;
    for (int i = tid; i < V; i += SAMP_T) mx = fmaxf(mx, lg[i]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int w = 1; w < SAMP_T / 32; w++) mx = fmaxf(mx, red[w]);
    for (int i = tid; i < VMAX; i += SAMP_T) pr[i] = (i < V && lg[i] != -INFINITY) ? exp_f(__fsub_rn(lg[i], mx)) : 0.0f;
    __syncthreads();

    if (warp == 0) {
        // serial sum in index order (zeros do not change a float sum), via ballots
        float sum = 0.0f;
        for (int base = 0; base < V; base += 32) {
            const float v = pr[base + lane];
            unsigned bal = __ballot_sync(0xffffffffu, v != 0.0f);
            while (bal) {
                const int b = __ffs(bal) - 1;
                sum = __fadd_rn(sum, pr[base + b]);
                bal &= bal - 1;
            }
        }
        const float inv = __fdiv_rn(1.0f, sum);

        // draws: lane j covers draws [j*dpl, min(V, (j+1)*dpl))
        const int dpl = p.draws_per_lane;
        const uint64_t s0 = st->rng;
        uint64_t s = 0;
#pragma unroll
        for (int b = 0; b < 64; b++) s ^= ((s0 >> b) & 1ull) ? jmp[b * 32 + lane] : 0ull;
        float best_v = -INFINITY;
        int best_i = 0x7fffffff;
        const int i0 = lane * dpl, i1 = min(V, i0 + dpl);
        for (int i = i0; i < i1; i++) {
            s = xs_step(s);
            // U = (xorshift64*() >> 40) / 2^24: a 24-bit integer times 2^-24, exact in float; only
            // entries of non-zero probability need it (a zero weight gives v = 0)
            const float pv = pr[i];
            float v = 0.0f;
            if (pv != 0.0f) {
                const float pi = __fmul_rn(pv, inv);
                if (pi > 0.0f) {
                    const uint64_t out = s * 0x2545F4914F6CDD1Dull;
                    const float U = __fmul_rn(__uint2float_rn((uint32_t)(out >> 40)), 1.0f / 16777216.0f);
                    const float q = -log_f(__fsub_rn(1.0f, U));
                    v = __fdiv_rn(pi, q);
                }
            }
            if (best_i == 0x7fffffff || v > best_v) {   // first element of the range, then strict >
                best_v = v;
                best_i = i;
            }
        }
        const int last_lane = (V - 1) / dpl;
        const uint64_t s_end = __shfl_sync(0xffffffffu, s, last_lane);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best_v, off);
            const int oi = __shfl_xor_sync(0xffffffffu, best_i, off);
            if (ov > best_v || (ov == best_v && oi < best_i)) { best_v = ov; best_i = oi; }
        }
        if (lane == 0) {
            int tok = best_i;
            if (best_v == -INFINITY) tok = 0;   // every candidate -inf: the reference keeps index 0
            if (idx < st->n_forced) tok = p.forced[(size_t)slot * p.forced_cap + idx];   // src/gsv_ar.cpp:778
            st->rng = s_end;
            s_tok = tok;
        }
    }
    __syncthreads();
    if (tid == 0) {
        const int tok = s_tok;
        p.out_tokens[(size_t)slot * p.tok_cap + idx] = tok;
        st->n_samp = idx + 1;
        // repetition window: append tok, drop the oldest beyond HIST
        if (tok >= 0 && tok < V) {
            uint16_t* cnt = p.counts + (size_t)slot * V;
            int32_t* h = p.hist + (size_t)slot * HIST;
            if (st->hist_len < HIST) {
                h[(st->hist_head + st->hist_len) % HIST] = tok;
                st->hist_len = st->hist_len + 1;
            } else {
                const int old = h[st->hist_head];
                if (old >= 0 && old < V) cnt[old] = (uint16_t)(cnt[old] - 1);
                h[st->hist_head] = tok;
                st->hist_head = (st->hist_head + 1) % HIST;
            }
            cnt[tok] = (uint16_t)(cnt[tok] + 1);
        }
    }
}

void launch_sampler(const SamplerParams& p, cudaStream_t s) {
    if (p.nslots <= 0) return;
    launch_pdl(k_sampler, dim3(p.nslots), dim3(SAMP_T), 0, s, p);
}

}  // namespace gsvcu
