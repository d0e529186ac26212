// tc_common.cuh -- device wrappers shared by the tensor-core kernels (gemm_tc.cu, dit.cu): bounded
// mbarrier waits, TMA tile copies (no multicast), tcgen05.mma kind::f16 with its shared-memory and
// instruction descriptors, TMEM loads; and the host-side tensor-map encoder (cuTensorMapEncodeTiled,
// resolved through the runtime's driver entry point).
#pragma once
#include <cuda.h>

#include <cstdint>

#include "kernels.h"

namespace gsvcu {
namespace tc {

// Bounded waits: each poll suspends the thread until the phase completes or TC_SUSPEND_NS elapse
// (so a waiting role takes almost no issue slots from the epilogue warps beside it), at most
// TC_POLL_LIMIT polls (~1.6 s) before the wait gives up.
constexpr uint32_t TC_POLL_LIMIT = 1u << 14;
constexpr uint32_t TC_SUSPEND_NS = 100000;

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
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(b), "r"(parity), "r"(TC_SUSPEND_NS)
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
// TMEM loads): every lane runs the same polls (one barrier access per poll for the warp, no divergent
// branch), and the outcome is taken from lane 0. A completed phase stays complete until the next one,
// which needs this warp's own arrival first, so once lane 0 saw it every lane may use the buffer.
__device__ __forceinline__ bool bar_wait_warp(uint32_t b, uint32_t parity, volatile int* abort_flag) {
    bool ok = bar_test(b, parity);
    for (uint32_t it = 0; !__shfl_sync(0xffffffffu, (int)ok, 0) && it < TC_POLL_LIMIT; it++) {
        if (*abort_flag) return __shfl_sync(0xffffffffu, 0, 0) != 0;
        ok = bar_try(b, parity);
    }
    return __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
}

// Short waits (a phase expected within microseconds): mbarrier.try_wait without a suspend-time hint, which
// returns after a short system-dependent window, so a completed phase is seen at once; bounded by
// TC_SPIN_LIMIT polls.
constexpr uint32_t TC_SPIN_LIMIT = 1u << 22;
__device__ __forceinline__ bool bar_try_short(uint32_t b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(b), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool bar_wait_short(uint32_t b, uint32_t parity, volatile int* abort_flag) {
    for (uint32_t it = 0; it < TC_SPIN_LIMIT; it++) {
        if (bar_try_short(b, parity)) return true;
        if (*abort_flag) return false;
    }
    return false;
}
// The same for a whole warp (warp-uniform result from lane 0's polls).
__device__ __forceinline__ bool bar_wait_short_warp(uint32_t b, uint32_t parity, volatile int* abort_flag) {
    bool ok = false;
    for (uint32_t it = 0; it < TC_SPIN_LIMIT; it++) {
        ok = __shfl_sync(0xffffffffu, (int)bar_try_short(b, parity), 0) != 0;
        if (ok || *abort_flag) break;
    }
    return ok;
}

// 2D TMA tile store from shared memory (bulk-group completion); c0 = innermost coordinate (elements).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int c0, int c1) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"((uint64_t)map),
                 "r"(c0), "r"(c1), "r"(src)
                 : "memory");
}

// 2D TMA tile load (no multicast) completing on an mbarrier; c0 = innermost coordinate (elements).
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
// 3D TMA tile load (no multicast) completing on an mbarrier; c0 = innermost coordinate (elements).
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
            "r"(dst), "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
        : "memory");
}
// Instruction descriptor, kind::f16: D f32 (bits 4-5 = 1), A and B f16 (0), both K-major, N >> 3 at bit
// 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) { return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24); }

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive TMEM columns of this warp's 32 lanes (lane l gets row lane base + l, columns c..c+15).
// Asynchronous: the registers hold the values only after tmem_wait_ld (which waits for every load this
// thread issued) and tmem_bind, which ties the values to that point for the compiler.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=f"(r[0]), "=f"(r[1]), "=f"(r[2]), "=f"(r[3]), "=f"(r[4]), "=f"(r[5]), "=f"(r[6]), "=f"(r[7]), "=f"(r[8]),
          "=f"(r[9]), "=f"(r[10]), "=f"(r[11]), "=f"(r[12]), "=f"(r[13]), "=f"(r[14]), "=f"(r[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 16 consecutive TMEM columns of this warp's 32 lanes from registers (the inverse of tmem_ld16); complete
// for this thread after tmem_wait_st.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "f"(r[0]), "f"(r[1]), "f"(r[2]), "f"(r[3]), "f"(r[4]), "f"(r[5]), "f"(r[6]), "f"(r[7]), "f"(r[8]), "f"(r[9]),
        "f"(r[10]), "f"(r[11]), "f"(r[12]), "f"(r[13]), "f"(r[14]), "f"(r[15])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_bind(float (&r)[16]) {
    asm volatile(""
                 : "+f"(r[0]), "+f"(r[1]), "+f"(r[2]), "+f"(r[3]), "+f"(r[4]), "+f"(r[5]), "+f"(r[6]), "+f"(r[7]),
                   "+f"(r[8]), "+f"(r[9]), "+f"(r[10]), "+f"(r[11]), "+f"(r[12]), "+f"(r[13]), "+f"(r[14]), "+f"(r[15])
                 :
                 : "memory");
}
// Shared-memory loads by shared-window address.

// ---------------------------------------------------------------- host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled, or null when the driver does not provide it.
inline EncodeTiledFn encode_fn() {
    static const EncodeTiledFn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return (EncodeTiledFn)f;
        cudaGetLastError();
        return (EncodeTiledFn) nullptr;
    }();
    return fn;
}

}  // namespace tc
}  // namespace gsvcu
