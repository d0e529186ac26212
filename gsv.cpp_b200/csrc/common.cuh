// common.cuh -- shared constants and device helpers of the gsvcu kernels.
//
// Numerics: the library is compiled with --fmad=false; every fused multiply-add is written out
// with fmaf() where the reference's ggml CPU op (built with -mavx2 -mfma) fuses it, and no other
// product is fused. Divisions and square roots are IEEE (no fast-math).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gsvcu {

constexpr int D = 512;        // hidden size (ar.hidden_dim)
constexpr int NH = 16;        // heads (ar.head)
constexpr int HD = 32;        // head dim = one Q8_0 block
constexpr int FF = 2048;      // FFN width (4 D)
constexpr int QK = 32;        // Q8_0 block
constexpr int PAGE = 64;      // tokens per KV page
constexpr int HIST = 4096;    // repetition-penalty window (src/gsv_ar.cpp:769-771)

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

// Q8_0 quantization of one 32-value block given its absolute maximum (quantize_row_q8_0_ref):
// d = amax / 127, id = 1/d (0 when d == 0), q = roundf(x * id) (ties away from zero), d stored fp16.
__device__ __forceinline__ void q8_scale(float amax, float& d, float& id) {
    d = __fdiv_rn(amax, 127.0f);
    id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
}
__device__ __forceinline__ int8_t q8_val(float x, float id) { return (int8_t)(int)roundf(__fmul_rn(x, id)); }

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Programmatic dependent launch. Every kernel of the library calls griddep_wait() before it reads
// anything the previous kernel in the stream may have written (and before it exits), then
// griddep_launch() to let the next kernel start its own prologue. Because no kernel triggers its
// dependents before its own wait returned, a kernel's prologue (the code before griddep_wait) may read
// data written two or more kernels earlier, never the immediately preceding kernel's output. Without a
// programmatic predecessor both are no-ops.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Packed pairs of f32: two IEEE operations per instruction, each lane rounded as the scalar operation
// (fma.rn / mul.rn / add.rn .f32x2), so results equal the scalar code's bit for bit.
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
    return ((uint64_t)__float_as_uint(hi) << 32) | (uint64_t)__float_as_uint(lo);
}
__device__ __forceinline__ float f2lo(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2hi(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// Read-only 128-bit load that does not allocate in L1 (streamed weights / KV).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// exp(x) for x <= 0 in float, the decode-attention softmax and page-merge exponential: Cody-Waite reduction x = n*ln2 + r (ln2 split into a 15-bit head and a
// float tail, so n*head is exact) and the degree-7 Taylor polynomial of exp(r), |r| <= ln2/2, by Horner
// with fma; result p * 2^n. Max error ~1.2 ulp. x < -87 (or -inf) gives 0.
__device__ __forceinline__ float exp_canon(float x) {
    if (!(x >= -87.0f)) return 0.0f;
    const float n = rintf(__fmul_rn(x, 0x1.715476p+0f));   // x / ln2, to nearest even
    float r = fmaf(-n, 0x1.62e4p-1f, x);
    r = fmaf(-n, 0x1.7f7d1cp-20f, r);
    float p = 0x1.a01a02p-13f;                              // 1/7!
    p = fmaf(p, r, 0x1.6c16c2p-10f);                        // 1/6!
    p = fmaf(p, r, 0x1.111112p-7f);                         // 1/5!
    p = fmaf(p, r, 0x1.555556p-5f);                         // 1/4!
    p = fmaf(p, r, 0x1.555556p-3f);                         // 1/3!
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    return __fmul_rn(p, __int_as_float(((int)n + 127) << 23));
}

// Per-slot decode state (device), one entry per sequence slot.
struct SlotState {
    int32_t active;       // 1 while the sequence is in flight
    int32_t kvlen;        // keys stored in the KV cache
    int32_t kvpos;        // position of the token decoded in the current step
    int32_t prompt_len;   // PE offset of generated tokens (src/gsv_ar.cpp:803)
    int32_t n_samp;       // tokens sampled so far
    int32_t max_steps;
    int32_t early_stop;   // -1 off; else stop the group once its first member sampled > early_stop
    int32_t group_first;  // slot of the group's first sequence (early-stop rule keys on it)
    int32_t finish_kind;  // -1 running, 0 EOS, 1 early stop, 2 max_steps
    int32_t finish_idx;   // step index at which the sequence finished
    int32_t hist_len;     // tokens in the repetition window (<= HIST)
    int32_t hist_head;    // ring position of the oldest token
    int32_t n_forced;     // teacher-forced tokens available
    int32_t decode_now;   // 1 when this step decodes the slot
    // the sequence's sampler settings (gsv_sampler_cfg, src/gsv_sampler.h:18-23): sequences with
    // different settings share one running batch
    int32_t top_k;
    float top_p, temperature, rep;
    uint64_t rng;         // xorshift64* state (src/gsv_sampler.h:33-42)
};

}  // namespace gsvcu
