// kernels.h -- host-side launchers of the gsvcu kernels (internal to the library).
#pragma once
#include <utility>

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace gsvcu {

// Launch with programmatic stream serialization allowed (see griddep_wait in common.cuh): the kernel
// may become resident while its predecessor finishes, and waits for it in griddep_wait().
template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ------------------------------------------------------------ Q8_0 GEMM
// Activation planes: xq int8 [M][K] row-major, xd fp16 [M][K/32].
// Weight planes: wq = fragment order [N/16][K/32][32 lanes][16 B] (mma.m16n8k32 A operand),
//                wd = fp16 [N][K/32].
enum { EPI_BIAS = 0, EPI_RESID = 1, EPI_RELU_Q8 = 2 };

struct KvWrite {             // optional store of K/V columns (features [D, 3D)) into KV pages
    void* pool = nullptr;    // [page][n_layer][2][NH][PAGE][HD] elements
    int kv_f32 = 0;
    int n_layer = 0, layer = 0;
    const int32_t* block_table = nullptr;   // [slot][max_pages]
    int max_pages = 0;
    const int32_t* tok_slot = nullptr;      // prefill: slot of each row
    const int32_t* tok_pos = nullptr;       // prefill: position of each row (nullptr = decode)
    const SlotState* st = nullptr;          // decode: row = slot, pos = st.kvpos, only if decode_now
};

struct GemmQ8Params {
    const int8_t* xq = nullptr;
    const uint16_t* xd = nullptr;
    int M = 0;
    const uint4* wq = nullptr;
    const uint16_t* wd = nullptr;
    int N = 0, K = 0;
    const float* bias = nullptr;
    const float* resid = nullptr;   // [M][N]
    float* y = nullptr;             // [M][N]
    int ldy = 0;                    // EPI_BIAS: row stride of y (0: N)
    int n_store = 0;                // EPI_BIAS: columns of y stored (0: N); N may carry zero padding rows
    int8_t* yq = nullptr;           // [M][N]   (EPI_RELU_Q8)
    uint16_t* yd = nullptr;         // [M][N/32]
    KvWrite kv;
    // tensor-core path (gemm_tc.cu): W's Q8_0 integers as fp16 numbers [N][K] row-major, and a device
    // scratch area of tc_scratch_bytes(M, N, K) bytes (128-byte aligned) for the activation side; when
    // both are given and the shape allows, launch_gemm_q8 runs k_tc_prep + k_gemm_q8_tc
    const __half* w16 = nullptr;
    void* tc_scratch = nullptr;
    size_t tc_scratch_n = 0;
    int32_t* err = nullptr;         // set to 1 if a bounded wait of k_gemm_q8_tc gave up (may be null)
};

void launch_gemm_q8(const GemmQ8Params& p, int epi, cudaStream_t s);
// tcgen05 / TMEM / TMA Q8_0 GEMM (prefill): scratch it needs, usable for this call, and its launch (two
// kernels; false: not launched)
size_t tc_scratch_bytes(int M, int N, int K);
bool gemm_tc_usable(const GemmQ8Params& p);
bool launch_gemm_q8_tc(const GemmQ8Params& p, int epi, cudaStream_t s);
cudaError_t gemm_tc_init_device();
// Raise the dynamic shared-memory limit of every GEMM instantiation on the current device.
cudaError_t gemm_q8_init_device();

// Host-side repack of raw GGUF Q8_0 blocks [N][K/32] x 34 B into the two planes.
void pack_q8_0_host(const uint8_t* raw, int N, int K, uint8_t* wq_out, uint16_t* wd_out);

// ------------------------------------------------------------ F32 / F16 weight GEMM (gemm_fx.cu)
// y[m][n] = sum_k w[n][k] * x(m, k) for F32 / F16 / BF16 layer matrices and an F16 / BF16 predict, in
// the order of ggml's FMA-vectorised dot: x rounded to F16 / BF16 for an F16 / BF16 w (round to nearest
// even), 32 float FMA chains (chain c takes
// k = c, c + 32, ...) added pairwise as chains c^16, ^8, ^4, ^1, ^2. K % 64 == 0; w row-major [N][K];
// x, w and every row of both 16-byte aligned (ldx * 4 and K * element size multiples of 16).
enum { FX_F32 = 0, FX_F16 = 1, FX_BF16 = 2, FX_QM = 3, FX_QK = 4 };   // Q4_1 / Q5_1 (k_gemm_qm), K-quants (k_gemm_qk)
enum { FXE_BIAS = 0, FXE_RESID = 1, FXE_RELU = 2 };   // y = acc + b (+ K/V store); (r + acc) + b; relu(acc + b)
struct GemmFxParams {
    const float* x = nullptr;
    int ldx = 0;
    int M = 0;
    const void* w = nullptr;        // FX_QM: the unsigned 4- / 5-bit values as bytes [N][K]; FX_QK: int16
                                    //   scale * value [N][K/256][lane 8][32] (value e of a super-block at
                                    //   (e % 8) * 32 + e / 8)
    const uint16_t* wd = nullptr;   // FX_QM: fp16 d per 32-value block [N][K/32]; FX_QK: d [N][K/256]
    const uint16_t* wm = nullptr;   // FX_QM: fp16 m per block [N][K/32]; FX_QK: dmin [N][K/256] (Q4_K / Q5_K)
    const uint8_t* wmins = nullptr; // FX_QK: the 8 sub-block mins of each super-block (Q4_K / Q5_K)
    int wtype = FX_F32;
    int N = 0, K = 0;
    const float* bias = nullptr;
    const float* resid = nullptr;   // FXE_RESID: [M][N]
    float* y = nullptr;             // [M][ldy] (FXE_BIAS) or [M][N]
    int ldy = 0;                    // FXE_BIAS: row stride of y (0: N)
    int n_store = 0;                // FXE_BIAS: columns of y stored (0: N)
    KvWrite kv;                     // FXE_BIAS: optional K/V store of columns [D, 3D)
    // FX_QK / FX_QM: device scratch for the rows quantized to Q8_K (values [M][K] lane-major per
    // super-block, d [M][K/256], int32 sums of 16 [M][K/16]) or to Q8_1 (values [M][K], d [M][K/32], f32 s
    // [M][K/32]); sized for the larger of the two
    int8_t* qx_q = nullptr;
    float* qx_d = nullptr;
    void* qx_s = nullptr;
};
void launch_gemm_fx(const GemmFxParams& p, int epi, cudaStream_t s);
cudaError_t gemm_fx_init_device();   // shared-memory attributes of the Q4_1 / Q5_1 and K-quant GEMMs

// ------------------------------------------------------------ F32 GEMM, double accumulation
// y[m][n] = (float) sum_k (double)w[n][k] * (double)x(m, k)  (+ add[m][n]); x(m,k) = x[m*ldx + k], or,
// for the BERT projection, gathered from per-sequence [1024][T] feature blocks with an implicit
// trailing 1 (see F32Gather).
struct F32Gather {          // x(m, k): k < bert_dim -> feat[row_off + k*T], k == bert_dim -> 1; row_T < 0 -> 0
    const float* feat = nullptr;      // concatenated per-sequence [bert_dim][T_s] blocks
    const int64_t* row_off = nullptr; // [M] offset of feat[0*T + t] for row m
    const int32_t* row_T = nullptr;   // [M] T of the row's sequence, -1 for rows without features
    int bert_dim = 0;
};
cudaError_t logits_init_device();   // shared-memory attribute of the K = 512 logits kernel
void launch_gemm_f32d(const float* x, int ldx, const F32Gather* gather, int M, const float* w, int N, int K,
                      const float* add, int ldadd, float* y, int ldy, cudaStream_t s);

// ------------------------------------------------------------ LayerNorm + Q8_0, quantize
void launch_layernorm_q8(const float* v, int rows, const float* w, const float* b, float* y, int8_t* yq,
                         uint16_t* yd, cudaStream_t s);
void launch_quantize_q8(const float* x, int rows, int K, int8_t* q, uint16_t* d, cudaStream_t s);

// ------------------------------------------------------------ attention
struct DecAttnParams {
    const float* q = nullptr;
    int q_stride = 0;
    const void* pool = nullptr;
    int kv_f32 = 0;
    int n_layer = 0, layer = 0;
    const int32_t* block_table = nullptr;
    int max_pages = 0;
    const int32_t* kvpos = nullptr;      // op entry: plain arrays
    const int32_t* active = nullptr;
    const SlotState* st = nullptr;       // engine: slot state (kvpos, decode_now)
    int B = 0;
    int max_chunks = 0;
    float scale = 0.f;
    int8_t* out_q = nullptr;
    uint16_t* out_d = nullptr;
    float* out_f32 = nullptr;
    float* part = nullptr;               // scratch: page outputs o [items][HD], see part_ml_of
    float* part_ml = nullptr;            // scratch: page {max, sum} [items] f32x2
    int partials_only = 0;               // 1: every page leaves its partial (the fused layer tail merges)
    int slot0 = 0;                       // first slot of this launch: slots slot0 .. slot0 + B - 1
    // compacted work list of the decode step (k_page_list): item i = {slot, chunk | kvpos << 8, physical
    // page, 0}; this launch serves items work_base[group] .. work_base[group + 1] - 1 (null: rectangular grid)
    const int4* work = nullptr;
    const int32_t* work_base = nullptr;
    int group = 0;
    int32_t* err = nullptr;              // set to 1 if a bounded wait gave up (may be null)
    // fault injection for the failure-path tests (gsvcu_set_wait_fault): bytes each page's mbarrier expects
    // beyond what is staged (so the wait runs out), and the wait's poll limit (0: the default)
    uint32_t fault_extra_tx = 0;
    uint32_t poll_limit = 0;
};
// Split-KV work items of decode attention: one per 64-key page. Page partials of item
// (slot * NH + head) * max_chunks + page: o, HD floats (a 128-byte row), in one array, and {m, l} in a
// second one that follows it; PART_STRIDE floats per item are allocated for both.
inline int decode_chunks(int max_tokens) { return (max_tokens + PAGE - 1) / PAGE; }
constexpr int PART_STRIDE = 4 + HD;
inline float* part_ml_of(float* part, size_t items) { return part + items * HD; }
// Alignment the decode-attention kernel relies on: 16-byte q rows (float4 loads), pool (TMA bulk
// copies) and f32 output (float4 stores), 8-byte Q8_0 output rows (8-byte stores).
inline bool decode_attention_aligned(const float* q, int q_stride, const void* pool, const int8_t* out_q,
                                     const float* out_f32) {
    return ((uintptr_t)q & 15) == 0 && (q_stride & 3) == 0 && ((uintptr_t)pool & 15) == 0 &&
           ((uintptr_t)out_q & 7) == 0 && ((uintptr_t)out_f32 & 15) == 0;
}
// Returns the number of kernels launched (2 when sequences may span several pages: pages + merge;
// 1 with partials_only, where the caller merges).
int launch_decode_attention(const DecAttnParams& p, cudaStream_t s);
// Raise the dynamic shared-memory limit of the decode-attention kernels on the current device.
cudaError_t attention_init_device();
// Build the decode step's (slot, page) list of the M slots (slots decoding this step), slot-major;
// base[0] = 0, base[1] = items of slots < split, base[2] = all items. M <= 4096.
void launch_page_list(const SlotState* st, int M, int split, const int32_t* block_table, int max_pages, int4* work,
                      int32_t* base, cudaStream_t s);

// ------------------------------------------------------------ fused decode layer tail (dense.cu)
// Page merge -> out-projection + residual -> LayerNorm 1 -> FFN1 (ReLU) -> FFN2 + residual ->
// LayerNorm 2 [-> next layer's QKV with the K/V page store], one 16-CTA cluster per 16 slots.
struct DenseParams {
    int slot0 = 0;                      // first slot (row) of this launch
    int M = 0;                          // slots (rows) of this launch: slot0 .. slot0 + M - 1
    const SlotState* st = nullptr;
    const float* part = nullptr;        // attention partials of this layer (partials_only launch)
    const float* part_ml = nullptr;
    int max_chunks = 0;
    const uint4* w_out = nullptr; const uint16_t* d_out = nullptr; const float* b_out = nullptr;
    const float* n1w = nullptr; const float* n1b = nullptr;
    const uint4* w_f1 = nullptr; const uint16_t* d_f1 = nullptr; const float* b_f1 = nullptr;
    const uint4* w_f2 = nullptr; const uint16_t* d_f2 = nullptr; const float* b_f2 = nullptr;
    const float* n2w = nullptr; const float* n2b = nullptr;
    float* x = nullptr;                 // [M][D] residual stream: this layer's input in, its output out
    const uint4* w_qkv = nullptr;       // next layer's QKV (nullptr: last layer)
    const uint16_t* d_qkv = nullptr; const float* b_qkv = nullptr;
    float* q = nullptr;                 // next layer's q, row stride q_stride
    int q_stride = 0;
    KvWrite kv;                         // next layer's K/V page store (decode: st)
    int32_t* err = nullptr;             // set to 1 if a bounded wait gave up
};
// Set the kernel attributes on the current device; *usable = a 16-CTA cluster of it can be resident.
cudaError_t dense_init_device(bool* usable);
void launch_dense_layer(const DenseParams& p, cudaStream_t s);

struct PrefillTile { int32_t seq, q0; };
struct PrefAttnParams {
    const float* qkv = nullptr;          // [M][3D]
    const int32_t* seq_start = nullptr;  // device
    const int32_t* seq_len = nullptr;
    const int32_t* text_len = nullptr;
    const PrefillTile* tiles = nullptr;  // device, n_tiles
    int n_tiles = 0;
    float scale = 0.f;
    int8_t* out_q = nullptr;
    uint16_t* out_d = nullptr;
    float* out_f32 = nullptr;
};
constexpr int PREF_QTILE = 64;
void launch_prefill_attention(const PrefAttnParams& p, cudaStream_t s);

// ------------------------------------------------------------ embeddings
// Prefill: row m -> text (phone id, PE t) or prompt (code, PE t); x = emb + alpha * pe (FMA).
struct PrefEmbedParams {
    const int32_t* ids = nullptr;        // [M]
    const int32_t* pe_pos = nullptr;     // [M]
    const int32_t* is_text = nullptr;    // [M]
    const float* text_emb = nullptr;
    const float* audio_emb = nullptr;
    const float* pe = nullptr;
    float text_alpha = 1.f, audio_alpha = 1.f;
    int M = 0;
    float* x = nullptr;                  // [M][D]
};
void launch_prefill_embed(const PrefEmbedParams& p, cudaStream_t s);

// ------------------------------------------------------------ sampler and step control
struct SamplerParams {
    const float* logits = nullptr;       // [nslots][V]
    int V = 0, eos = 0, nslots = 0;
    SlotState* st = nullptr;             // per slot: sampler settings, RNG, step, repetition window size
    uint16_t* counts = nullptr;          // [nslots][V]
    int32_t* hist = nullptr;             // [nslots][HIST] ring of the repetition window
    int32_t* out_tokens = nullptr;       // [nslots][tok_cap]
    int tok_cap = 0;
    const int32_t* forced = nullptr;     // [nslots][forced_cap] teacher-forced tokens
    int forced_cap = 0;
    const uint64_t* jump = nullptr;      // [32][64] xorshift jump matrices (columns)
    int draws_per_lane = 0;
};
void launch_sampler(const SamplerParams& p, cudaStream_t s);

// Group stop rules + next-token embedding (+ Q8_0) + KV position bump.
struct StepPrepParams {
    SlotState* st = nullptr;
    int nslots = 0;
    int eos = 0;
    const int32_t* out_tokens = nullptr;
    int tok_cap = 0;
    const float* audio_emb = nullptr;
    const float* pe = nullptr;
    float audio_alpha = 1.f;
    float* x = nullptr;                  // [nslots][D]
    int8_t* xq = nullptr;
    uint16_t* xd = nullptr;
};
void launch_step_prep(const StepPrepParams& p, cudaStream_t s);

// dst[didx[r]] = src[sidx[r]] for rows of `width` floats (index arrays may be null = identity).
void launch_copy_rows(float* dst, const int32_t* didx, const float* src, const int32_t* sidx, int nrows, int width,
                      cudaStream_t s);

}  // namespace gsvcu
