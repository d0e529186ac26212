// noalloc.cu -- decode attention for callers that must not allocate device memory.
//
// Some callers cannot call cudaMalloc at the point where they run attention: code that runs while a
// framework's caching allocator owns the whole device, code inside a real-time audio callback that
// must not block on the driver's allocator, or embedders that forbid allocations after start-up.
// gsvcu_op_decode_attention grows its split-KV scratch with cudaMalloc on first use; this variant runs
// the same kernels with their scratch (the per-page partial results) in a fixed array that is part of
// the library image. Every GPU that loads the library holds this array (about 2.3 MiB) until the
// process exits.
#include <cstdio>
#include <mutex>

#include "../../include/gsvcu.h"
#include "kernels.h"

namespace gsvcu {
namespace {

constexpr int kItems = GSVCU_NOALLOC_MAX_ITEMS;                       // (sequence, KV page) pairs
constexpr size_t kPartFloats = (size_t)kItems * NH * PART_STRIDE;    // partials: o[32], {m, l} per head

// Scratch shared by every call on a device.
struct NoallocScratch {
    float part[kPartFloats];
    int32_t err;   // set by the kernels when a bounded wait for staged K/V gave up; cleared by every call
};
static __device__ __align__(256) NoallocScratch g_scratch;

// Device address of g_scratch per device. In host code `g_scratch` is only a stand-in symbol; the
// address a kernel may use comes from cudaGetSymbolAddress, taken once per device with it current.
constexpr int kMaxDevices = 64;
std::mutex g_mu;
NoallocScratch* g_addr[kMaxDevices] = {};

int scratch_for_current_device(NoallocScratch** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return GSVCU_ERR_DEVICE;
    }
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            return GSVCU_ERR_CUDA;
        }
        if (attention_init_device() != cudaSuccess) {
            cudaGetLastError();
            return GSVCU_ERR_CUDA;
        }
        g_addr[dev] = (NoallocScratch*)p;
    }
    *out = g_addr[dev];
    return GSVCU_OK;
}

}  // namespace
}  // namespace gsvcu

using namespace gsvcu;

extern "C" int gsvcu_op_decode_attention_noalloc(void* stream, const float* q_dev, int32_t q_stride,
                                                 const void* pool_dev, int32_t kv_dtype, int32_t n_layer,
                                                 int32_t layer, const int32_t* block_table_dev, int32_t max_pages,
                                                 const int32_t* kvpos_dev, const int32_t* active_dev, int32_t B,
                                                 int8_t* out_q_dev, uint16_t* out_d_dev, float* out_f32_dev) {
    if (!q_dev || !pool_dev || !block_table_dev || !kvpos_dev || !active_dev || !out_q_dev || !out_d_dev || B <= 0 ||
        max_pages <= 0 || n_layer <= 0 || layer < 0 || layer >= n_layer || q_stride < D ||
        (kv_dtype != GSVCU_KV_F16 && kv_dtype != GSVCU_KV_F32) ||
        !decode_attention_aligned(q_dev, q_stride, pool_dev, out_q_dev, out_f32_dev))
        return GSVCU_ERR_ARG;
    const int max_chunks = decode_chunks(max_pages * PAGE);
    if ((int64_t)B * max_chunks > kItems) {
        std::fprintf(stderr,
                     "gsvcu_op_decode_attention_noalloc: B (%d) x max_pages (%d) exceeds the fixed scratch of %d "
                     "sequence-pages (GSVCU_NOALLOC_MAX_ITEMS); use gsvcu_op_decode_attention\n",
                     B, max_pages, kItems);
        return GSVCU_ERR_ARG;
    }
    NoallocScratch* s = nullptr;
    const int rc = scratch_for_current_device(&s);
    if (rc != GSVCU_OK) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    DecAttnParams a;
    a.q = q_dev; a.q_stride = q_stride; a.pool = pool_dev; a.kv_f32 = kv_dtype; a.n_layer = n_layer; a.layer = layer;
    a.block_table = block_table_dev; a.max_pages = max_pages; a.kvpos = kvpos_dev; a.active = active_dev; a.B = B;
    a.max_chunks = max_chunks; a.scale = 1.0f / sqrtf((float)HD); a.out_q = out_q_dev; a.out_d = out_d_dev;
    a.out_f32 = out_f32_dev; a.part = s->part; a.err = &s->err;
    a.part_ml = part_ml_of(s->part, (size_t)B * NH * max_chunks);
    // the status word starts every call at zero; after the kernels it is read back (one 4-byte copy into
    // this stack frame, then the stream is synchronised), so a wait that gave up fails this call
    if (cudaMemsetAsync(&s->err, 0, sizeof(int32_t), st) != cudaSuccess) return GSVCU_ERR_CUDA;
    launch_decode_attention(a, st);
    if (cudaGetLastError() != cudaSuccess) return GSVCU_ERR_CUDA;
    int32_t err = 0;
    if (cudaMemcpyAsync(&err, &s->err, sizeof(err), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return GSVCU_ERR_CUDA;
    if (err) {
        std::fprintf(stderr, "gsvcu_op_decode_attention_noalloc: staged K/V never arrived (bounded wait gave up)\n");
        return GSVCU_ERR_CUDA;
    }
    return GSVCU_OK;
}
