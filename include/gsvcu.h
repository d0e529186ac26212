/* gsvcu.h -- C ABI of the B200 (sm_100a) library for gsv.cpp's AR semantic-token hot path.
 *
 * The reference path lives in gsv.cpp's src/gsv_ar.{h,cpp} (class gsv_ar) on top of ggml graphs.
 * This library replaces its internals: a C++ host shim (gsv.cpp_b200/csrc/gsv_ar.cpp) implements
 * the unchanged `class gsv_ar` API on these entry points, and any FFI (ctypes, cgo, JNI) can bind
 * them directly. Plain C types only: pointers, sizes, status codes.
 *
 * Conventions
 *   - Every function returns GSVCU_OK (0) or a negative GSVCU_ERR_* code; the message of the last
 *     failure of a context is gsvcu_last_error(ctx). Nothing calls exit().
 *   - A context owns one CUDA device and one stream; use it from one host thread at a time
 *     (the reference serialises gsv_ar calls the same way, tools/svc_core.h:628,1312).
 *   - "host" pointers are CPU memory; "dev" pointers are device memory on the context's device.
 */
#ifndef GSVCU_H
#define GSVCU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    GSVCU_OK = 0,
    GSVCU_ERR_ARG = -1,      /* invalid argument (null pointer, size or id out of range) */
    GSVCU_ERR_CUDA = -2,     /* a CUDA call failed */
    GSVCU_ERR_OOM = -3,      /* device memory or KV page pool exhausted */
    GSVCU_ERR_IO = -4,       /* file could not be opened or read */
    GSVCU_ERR_FORMAT = -5,   /* GGUF content is not a supported AR model */
    GSVCU_ERR_STATE = -6,    /* call made in the wrong state (e.g. no model loaded) */
    GSVCU_ERR_DEVICE = -7    /* device is not an sm_100 GPU or does not exist */
};

enum { GSVCU_KV_F16 = 0, GSVCU_KV_F32 = 1 };

typedef struct gsvcu_ctx gsvcu_ctx;

/* Model dimensions, as read from the GGUF KV pairs (reference src/gsv_ar.cpp:571-582). */
typedef struct {
    int32_t hidden_dim, n_head, head_dim, n_layer, vocab_size, phoneme_vocab_size, eos, bert_dim, ffn_dim;
    float text_pe_alpha, audio_pe_alpha;
} gsvcu_hparams;

/* Sampler settings; same fields and defaults as gsv_sampler_cfg (reference src/gsv_sampler.h:18-23):
 * top_k 15 (<=0 off), top_p 1.0 (>=1 off), temperature 1.0, repetition_penalty 1.35. */
typedef struct {
    int32_t top_k;
    float top_p, temperature, repetition_penalty;
} gsvcu_sampler_cfg;

/* One sequence (gsv_ar_request, reference src/gsv_ar.h:13-17): phone ids, BERT features laid out
 * [bert_dim][n_phones] (bert[k * n_phones + t]), reference prompt semantic codes. phones and prompt
 * are host memory; bert may be host or device memory of the context's device. */
typedef struct {
    const int32_t* phones;
    int32_t n_phones;
    const float* bert;
    const int32_t* prompt;
    int32_t n_prompt;
} gsvcu_request;

/* Called after each block of decode steps with the number of steps completed so far; the C++ shim
 * forwards it to gsvprog::tick() (reference src/gsv_ar.cpp:761-763). May be NULL. */
typedef void (*gsvcu_progress_fn)(void* user, int32_t steps_done);

/* ---------------------------------------------------------------- context and model */

/* Open a context on CUDA device `device` (what gsv_device_parse selects, reference src/gsv_device.h:19-37). */
int gsvcu_create(int device, gsvcu_ctx** out);
void gsvcu_destroy(gsvcu_ctx* ctx);
const char* gsvcu_last_error(const gsvcu_ctx* ctx);

/* Load an AR GGUF file (replaces gsv_ar::load, reference src/gsv_ar.cpp:490-705): tensor names of
 * tools/export_gguf/convert_ar.py:106-130. Attention / FFN matrices and predict of any type the
 * exporter (--spec attn=.., ffn=.., predict=..) or tools/quantize_gguf.cpp writes: Q8_0, Q4_0, Q4_1,
 * Q5_0, Q5_1, Q4_K, Q5_K, Q6_K, IQ4_NL, F32, F16, BF16 (ffn1_w and ffn2_w of a layer both Q8_0 / Q4_0 /
 * Q5_0 / IQ4_NL or both of the others); embeddings F32, F16 or BF16 (widened on load); bert_proj,
 * norms and biases F32. Q8_0 matrices, and Q4_0 / Q5_0 / IQ4_NL ones as the Q8_0 blocks of the same
 * values, are repacked into tensor-core fragment order on the device; Q4_1 / Q5_1 are unpacked to value
 * bytes and d / m planes, K-quants to scaled int16 values and d / dmin / min planes; F32 / F16 / BF16
 * matrices are kept as stored. Other ggml types are refused (GSVCU_ERR_FORMAT). */
int gsvcu_load_gguf(gsvcu_ctx* ctx, const char* path);
int gsvcu_get_hparams(const gsvcu_ctx* ctx, gsvcu_hparams* out);

/* Size the paged KV pool and the per-step buffers: up to `max_slots` sequences in flight, each
 * with at most `max_ctx` tokens of context (prefix + generated), KV element type GSVCU_KV_F16 or
 * GSVCU_KV_F32. Replaces alloc_cache (reference src/gsv_ar.cpp:94-118). Called implicitly with
 * defaults by the calls below when needed. */
int gsvcu_kv_reserve(gsvcu_ctx* ctx, int32_t max_slots, int32_t max_ctx, int32_t kv_dtype);
/* Free the KV pool and per-step buffers (gsv_ar::release_cache, reference src/gsv_ar.cpp:826). */
int gsvcu_release_cache(gsvcu_ctx* ctx);

/* Parse and validate an AR GGUF file on the host only (no device): KV hyper-parameters and every
 * tensor's name, shape and type, as gsvcu_load_gguf requires (reference src/gsv_ar.cpp:545-662).
 * err (may be NULL) receives the reason of a failure. */
int gsvcu_inspect_gguf(const char* path, gsvcu_hparams* out, char* err, int32_t err_cap);

/* ---------------------------------------------------------------- reference-facing path */

/* Prefill only; host logits_out [B][vocab] of each sequence's last position
 * (gsv_ar::first_logits, reference src/gsv_ar.cpp:707-717). */
int gsvcu_first_logits(gsvcu_ctx* ctx, const gsvcu_request* reqs, int32_t B, float* logits_out);

/* Prefill + KV-cached decode + on-device sampling with the stop rules of gsv_ar::generate
 * (reference src/gsv_ar.cpp:719-824): per-sequence seeds (seeds[b], or seed_base + 0x9E3779B9*b),
 * EOS masked while step < 11, repetition window of the last 4096 tokens, optional teacher forcing
 * (oracle_tokens, same token for every sequence), EOS finish, early stop keyed on sequence 0,
 * max_steps. Outputs (host):
 *   tokens_out [B][cap]   prompt + generated tokens, without the token that stopped the sequence
 *   n_tokens_out [B]      number of valid entries per row (may exceed cap: then rows are truncated)
 *   lens_out [B]          generated counts in the order the sequences finished (gsv_ar_result::lens) */
int gsvcu_generate(gsvcu_ctx* ctx, const gsvcu_request* reqs, int32_t B, const gsvcu_sampler_cfg* sampler,
                   uint64_t seed_base, int32_t early_stop_num, int32_t max_steps, const int32_t* oracle_tokens,
                   int32_t n_oracle, const uint64_t* seeds, int32_t n_seeds, int32_t* tokens_out,
                   int32_t* n_tokens_out, int32_t* lens_out, int32_t cap, gsvcu_progress_fn progress, void* user);

/* Teacher-forced trace for parity checks (the reference's GSV_AR_PROB_DUMP / oracle_tokens
 * diagnostics, src/gsv_ar.cpp:775-778): prefill, then decode `n_steps` forced tokens per sequence
 * (forced [B][n_steps], host). logits_out [n_steps + 1][B][vocab] (row 0 = prefill). dump (may be
 * NULL) [n_steps + 1][B][n_layer][4][hidden]: per layer, for the last position of the step, the
 * attention output, LN1 output, (n1 + W2 h) + b2 and the layer output. */
int gsvcu_debug_trace(gsvcu_ctx* ctx, const gsvcu_request* reqs, int32_t B, const int32_t* forced, int32_t n_steps,
                      float* logits_out, float* dump);

/* ---------------------------------------------------------------- continuous batching
 * The batched entry behind gsv_engine::ar_generate_batch / svc::ArBatcher (reference
 * tools/svc_core.h:1244-1340) generalised to refill: sequences are admitted into free slots while
 * others decode. */

typedef struct {
    int32_t slot;          /* slot that ran the sequence */
    int32_t tag;           /* caller tag given at admission */
    int32_t finish_kind;   /* 0 EOS, 1 early stop, 2 max_steps */
    int32_t n_generated;   /* generated tokens (gsv_ar_result::lens value) */
    int32_t n_tokens;      /* tokens copied to the caller buffer (prompt excluded) */
} gsvcu_finished;

/* Admit sequences into free slots (prefill runs immediately). seeds[i] seeds sequence i; tags are
 * returned with its completion. Every admitted sequence keeps `sampler` (NULL: the reference defaults)
 * for its whole life, so sequences with different sampler settings share the running batch. Fails
 * with GSVCU_ERR_OOM if slots or KV pages are short. */
int gsvcu_serve_admit(gsvcu_ctx* ctx, const gsvcu_request* reqs, int32_t n, const gsvcu_sampler_cfg* sampler,
                      const uint64_t* seeds, const int32_t* tags, int32_t max_steps, int32_t early_stop_num);
/* Run `n_steps` decode steps for every slot in flight, then report the sequences that finished:
 * up to max_done records in done[], their generated tokens concatenated in tokens (host, capacity
 * tok_cap; may be NULL). Returns the number of records (>= 0) or an error. */
int gsvcu_serve_step(gsvcu_ctx* ctx, int32_t n_steps, gsvcu_finished* done, int32_t max_done, int32_t* tokens,
                     int32_t tok_cap);
/* Serving lookahead (no counterpart in the reference; an extension of this library's serving API).
 * on = 1: gsvcu_serve_step(n) first reports the chunk of steps started by the previous call, then
 * starts the next n steps before it returns, so the GPU keeps decoding while the caller handles the
 * results and admits new sequences (they join from the chunk started by the following call). The
 * first call only starts a chunk (returns 0); a final call with n = 0 collects the last chunk.
 * Tokens of every sequence are the same as without lookahead. Default 0. */
int gsvcu_set_serve_lookahead(gsvcu_ctx* ctx, int32_t on);
/* Drop every sequence in flight (cancellation): slots and KV pages return to the pool, nothing is
 * reported. */
int gsvcu_serve_reset(gsvcu_ctx* ctx);
/* Slots currently in flight. */
int gsvcu_serve_active(const gsvcu_ctx* ctx);
/* Generated tokens produced so far: finished sequences plus the tokens sampled so far by the
 * sequences in flight (as of the last gsvcu_serve_step). */
int64_t gsvcu_serve_tokens_total(const gsvcu_ctx* ctx);

/* ---------------------------------------------------------------- kernel-level entry points
 * Device pointers, the context's stream. Used by the parity tests and microbenchmarks. */

/* Activation quantization to Q8_0 planes: x [rows][K] f32 -> q int8 [rows][K], d fp16 bits [rows][K/32]
 * (ggml quantize_row_q8_0 semantics, the src1 conversion of the Q8_0 mul_mat at src/gsv_ar.cpp:244). */
int gsvcu_op_quantize_q8_0(gsvcu_ctx* ctx, const float* x_dev, int32_t rows, int32_t K, int8_t* q_dev,
                           uint16_t* d_dev);

/* Repack raw GGUF Q8_0 blocks (host, [N][K/32] x 34 bytes) into device fragment planes. wq_dev needs
 * N*K bytes, wd_dev N*K/32 fp16. N % 32 == 0, K % 32 == 0. (Weight upload of src/gsv_ar.cpp:549-570.) */
int gsvcu_op_pack_q8_0(gsvcu_ctx* ctx, const uint8_t* raw_host, int32_t N, int32_t K, void* wq_dev, void* wd_dev);

/* Y = W . X^T over Q8_0 planes (ggml Q8_0 mul_mat semantics, src/gsv_ar.cpp:244,260,262,263) with an epilogue:
 *   epi 0: y = acc + bias                        (bias may be NULL)
 *   epi 1: y = (resid + acc) + bias              (pre-LayerNorm sum, src/gsv_ar.cpp:261,264)
 *   epi 2: y = relu(acc + bias) quantized to Q8_0 into yq_dev / yd_dev (src/gsv_ar.cpp:262)
 * xq/xd: activation planes with M rows (row stride K). y_dev [M][N] f32 for epi 0/1. */
int gsvcu_op_q8_gemm(gsvcu_ctx* ctx, const int8_t* xq_dev, const uint16_t* xd_dev, int32_t M, const void* wq_dev,
                     const void* wd_dev, int32_t N, int32_t K, const float* bias_dev, const float* resid_dev,
                     int32_t epi, float* y_dev, int8_t* yq_dev, uint16_t* yd_dev);

/* The tensor-core form of gsvcu_op_q8_gemm (the prefill GEMM of the layers, src/gsv_ar.cpp:244,260,262,263):
 * the same semantics and results bit for bit, computed with tcgen05.mma (fp16 operands holding the
 * Q8_0 integers, fp32 accumulators in tensor memory, per-block float chains on the CUDA cores). w16_dev
 * holds the weight integers as fp16 [N][K] (gsvcu_op_pack_q8_0_f16), wd_dev their scales [N][K/32]. N a
 * multiple of 128, K a multiple of 64 up to 2048, xq_dev and w16_dev 16-byte aligned. Scratch for the
 * fp16 copy of X is owned by the context (grown on demand). */
int gsvcu_op_q8_gemm_tc(gsvcu_ctx* ctx, const int8_t* xq_dev, const uint16_t* xd_dev, int32_t M, const void* w16_dev,
                        const void* wd_dev, int32_t N, int32_t K, const float* bias_dev, const float* resid_dev,
                        int32_t epi, float* y_dev, int8_t* yq_dev, uint16_t* yd_dev);
/* Raw GGUF Q8_0 blocks (host, [N][K/32] x 34 bytes) -> their integers as fp16 [N][K] on the device
 * (w16_dev: N*K*2 bytes), the weight operand of gsvcu_op_q8_gemm_tc. */
int gsvcu_op_pack_q8_0_f16(gsvcu_ctx* ctx, const uint8_t* raw_host, int32_t N, int32_t K, void* w16_dev);

/* Fused LayerNorm (layernorm_affine, P:1535-1585; ln_affine src/gsv_ar.cpp:157-165) over rows of 512
 * already summed as (x + r) + bias, writing f32 and Q8_0 planes. */
int gsvcu_op_layernorm_q8(gsvcu_ctx* ctx, const float* v_dev, int32_t rows, const float* w_dev, const float* b_dev,
                          float* y_dev, int8_t* yq_dev, uint16_t* yd_dev);

/* Y[M][N] = W[N][K] . X[M][K]^T in f32 with double accumulation (ggml F32 mul_mat, src/gsv_ar.cpp:241,266),
 * optional add. */
int gsvcu_op_f32_gemm(gsvcu_ctx* ctx, const float* x_dev, int32_t M, const float* w_dev, int32_t N, int32_t K,
                      const float* add_dev, float* y_dev);

/* Y[M][N] = W[N][K] . X[M][K]^T (+ bias[N], may be NULL) for an F32 (wtype 0), F16 (wtype 1) or BF16
 * (wtype 2) layer matrix (ggml F32 / F16 / BF16 mul_mat, src/gsv_ar.cpp:244,260,262,263) in the order of
 * ggml's FMA-vectorised dot: X rounded to F16 / BF16 for an F16 / BF16 W, 32 float FMA chains (chain c
 * over k = c, c + 32, ...) added
 * pairwise as chains c^16, ^8, ^4, ^1, ^2. K a multiple of 256; x_dev and w_dev 16-byte aligned. */
int gsvcu_op_fx_gemm(gsvcu_ctx* ctx, const float* x_dev, int32_t M, const void* w_dev, int32_t wtype, int32_t N,
                     int32_t K, const float* bias_dev, float* y_dev);

/* Split-KV decode attention over a paged KV pool, 16 heads x 32 dims (flash_attn_ext over the cache,
 * src/gsv_ar.cpp:402-405).
 *   q_dev [B][q_stride] f32 (head h at h*32), pool_dev KV pages, block_table_dev [B][max_pages] int32,
 *   kvpos_dev [B]: index of the newest key (keys 0..kvpos attend), active_dev [B] (0 = skip).
 *   Page layout: [page][n_layer][K,V][16 heads][64 tokens][32] of kv_dtype elements.
 *   Output: Q8_0 planes out_q [B][512], out_d [B][16]; out_f32 [B][512] optional (may be NULL).
 *   Alignment: q_dev, pool_dev and out_f32_dev 16-byte aligned, q_stride a multiple of 4, out_q_dev
 *   8-byte aligned (else GSVCU_ERR_ARG); kvpos < max_pages * 64.
 * One split-KV work item per 64-key page; the pages' partial results live in scratch memory owned by
 * the context (grown on demand). */
int gsvcu_op_decode_attention(gsvcu_ctx* ctx, const float* q_dev, int32_t q_stride, const void* pool_dev,
                              int32_t kv_dtype, int32_t n_layer, int32_t layer, const int32_t* block_table_dev,
                              int32_t max_pages, const int32_t* kvpos_dev, const int32_t* active_dev, int32_t B,
                              int8_t* out_q_dev, uint16_t* out_d_dev, float* out_f32_dev);

/* A page wait of this entry that gives up (bounded, see gsvcu_set_wait_fault) is reported by the next
 * gsvcu_sync of the context as GSVCU_ERR_CUDA, once. kvpos at or beyond max_pages * 64 is clamped to the
 * last page of the block table. */

/* Decode attention that allocates nothing (no counterpart in the reference; added for callers of
 * this library that may not allocate device memory where they run attention -- e.g. code running
 * while a framework's caching allocator owns the device, a real-time callback that must not block
 * in the driver's allocator, or an embedder that forbids allocations after start-up).
 * Same inputs, outputs and results as gsvcu_op_decode_attention, on the caller's `stream`
 * (cudaStream_t, NULL = legacy default stream) of the current device, without a context. The split-KV
 * scratch is a fixed array inside the library (about 2.3 MiB held on every GPU that loads it, until
 * the process exits), sized for B * max_pages <= GSVCU_NOALLOC_MAX_ITEMS (one split-KV work item per
 * 64-key page); larger calls return GSVCU_ERR_ARG with a message on stderr. The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress); make that first call before any stream capture.
 * All calls share the array: calls that overlap on the GPU (other streams, other threads) race.
 * The call returns once its kernels have finished on `stream` (it reads back their status word): a
 * bounded wait for staged K/V that gave up returns GSVCU_ERR_CUDA instead of GSVCU_OK. */
#define GSVCU_NOALLOC_MAX_ITEMS 1024
int gsvcu_op_decode_attention_noalloc(void* stream, const float* q_dev, int32_t q_stride, const void* pool_dev,
                                      int32_t kv_dtype, int32_t n_layer, int32_t layer,
                                      const int32_t* block_table_dev, int32_t max_pages, const int32_t* kvpos_dev,
                                      const int32_t* active_dev, int32_t B, int8_t* out_q_dev, uint16_t* out_d_dev,
                                      float* out_f32_dev);

/* Prefix-masked prefill attention over packed sequences (src/gsv_ar.cpp:215-223, 257): qkv_dev
 * [M][1536] rows (q|k|v), sequence s = rows [start_s, start_s + len_s) whose first text_len_s rows are
 * text (bidirectional among text), the rest semantic (causal, full view of the text).
 * seq_start/seq_len/text_len are host arrays of n_seq entries. */
int gsvcu_op_prefill_attention(gsvcu_ctx* ctx, const float* qkv_dev, int32_t n_seq, const int32_t* seq_start,
                               const int32_t* seq_len, const int32_t* text_len, int8_t* out_q_dev,
                               uint16_t* out_d_dev, float* out_f32_dev);

/* One sampling step per row (gsv_logits_to_probs + gsv_sample, reference src/gsv_sampler.cpp:8-89,
 * with the step < 11 EOS mask of src/gsv_ar.cpp:768): logits_dev [B][V] f32; prev_host [B][prev_stride]
 * repetition windows of n_prev_host[b] tokens (NULL = none); step_host [B] step index; rng_host [B]
 * xorshift64* states, advanced in place; tokens_host [B] out. */
int gsvcu_op_sample(gsvcu_ctx* ctx, const float* logits_dev, int32_t B, int32_t V, int32_t eos,
                    const gsvcu_sampler_cfg* cfg, const int32_t* prev_host, const int32_t* n_prev_host,
                    int32_t prev_stride, const int32_t* step_host, uint64_t* rng_host, int32_t* tokens_host);

/* ---------------------------------------------------------------- BERT feature producer
 * gsv.cpp's gsv_bert (reference src/gsv_bert.{h,cpp}, chinese-roberta-wwm-ext-large up to
 * hidden_states[-3]) on the same device, producing the AR path's `bert` input. A BERT context owns its
 * weights, stream and buffers; use it from one host thread at a time. */
typedef struct gsvcu_bert gsvcu_bert;
typedef struct {
    int32_t hidden, n_head, inter, layers_used, vocab, max_pos;
    float ln_eps;
} gsvcu_bert_hparams;

/* Load a BERT GGUF of tools/export_gguf/convert_bert.py (gsv_bert::load, src/gsv_bert.cpp:311-420):
 * attention / FFN matrices F32, F16, BF16 or Q8_0 (others GSVCU_ERR_FORMAT), embeddings and norms F32 /
 * F16; hidden a multiple of 128 up to 1024, head dim 64. */
int gsvcu_bert_load(int device, const char* path, gsvcu_bert** out);
void gsvcu_bert_destroy(gsvcu_bert* ctx);
const char* gsvcu_bert_last_error(const gsvcu_bert* ctx);
int gsvcu_bert_get_hparams(const gsvcu_bert* ctx, gsvcu_bert_hparams* out);
/* gsv_bert::encode / encode_layers (src/gsv_bert.cpp:207-236): ids [T] with [CLS] / [SEP], T <= max_pos;
 * out (host) [hidden][T] after the first n_layers layers (n_layers < 0: all layers_used; 0: the embedding
 * LayerNorm). */
int gsvcu_bert_encode(gsvcu_bert* ctx, const int32_t* ids, int32_t T, int32_t n_layers, float* out);
/* gsv_bert::encode_feat_batch (src/gsv_bert.cpp:271-301; encode_feat is B = 1): B sequences, sequence b
 * the first lens[b] ids of the slot ids_flat[b * Tmax ..], 3 <= Tmax <= max_pos, 1 <= lens[b] <= Tmax.
 * out gets, for every sequence with lens[b] > 2 and in order, its features without [CLS] / [SEP] as
 * [hidden][lens[b] - 2], concatenated; out is host memory, or device memory of the context's device
 * when out_on_device != 0 (then it can be handed to gsvcu_request.bert directly). Each sequence's
 * features equal those of its own call. */
int gsvcu_bert_encode_feat_batch(gsvcu_bert* ctx, int32_t B, const int32_t* ids_flat, const int32_t* lens,
                                 int32_t Tmax, float* out, int32_t out_on_device);

/* ---------------------------------------------------------------- DiT / CFM velocity estimator
 * gsv.cpp's gsv_dit (reference src/gsv_dit.{h,cpp}: F5-style DiT, 22 blocks of 1024 / 16 heads x 64,
 * CFM Euler sampling with classifier-free guidance) on the same device. A DiT context owns its weights,
 * stream and buffers; use it from one host thread at a time. Arrays are host memory in the reference's
 * torch layouts: mel [100][T] (index c * T + t), condition rows [T][1024]. */
typedef struct gsvcu_dit gsvcu_dit;
typedef struct {
    int32_t dim, depth, heads, dim_head, ff_mult, mel_dim, text_dim;
} gsvcu_dit_hparams;

/* Load a DiT GGUF of tools/export_gguf/convert_dit.py (gsv_dit::load, src/gsv_dit.cpp:640-750): 2D weights
 * F32 or F16 (held as F16 on the device), biases / norms / inv_freq F32; dims 1024 / 16 x 64 / FFN 2048 /
 * mel 100, any depth. */
int gsvcu_dit_load(int device, const char* path, gsvcu_dit** out);
void gsvcu_dit_destroy(gsvcu_dit* ctx);
const char* gsvcu_dit_last_error(const gsvcu_dit* ctx);
int gsvcu_dit_get_hparams(const gsvcu_dit* ctx, gsvcu_dit_hparams* out);
/* The static cache of gsv_dit::prepare (src/gsv_dit.cpp:771-830): `cond` and `neg` are the condition and
 * negative-condition rows [T][1024] (input_embed.proj of [prompt_x | text_embed] and [0 | text_embed], with
 * its bias), x_lens the valid frames (<= 0: T). Also sets the RoPE tables. */
int gsvcu_dit_set_condition(gsvcu_dit* ctx, const float* cond, const float* neg, int32_t T, int32_t x_lens);
/* gsv_dit::prepare (src/gsv_dit.cpp:771-830, cache graph :486-531): the static cache from prompt_mel [100][T]
 * (the prompt frames, zeros after them) and mu [512][T]: text path (mu^T + freqs_cis, 4 ConvNeXtV2 blocks),
 * condition = proj_ctx([prompt_x | text]) + bias, negative = proj_ctx([0 | text]) + bias. Needs the file's
 * text_embed and proj.weight_ctx tensors (else GSVCU_ERR_FORMAT); T <= 4096; x_lens <= 0: T. */
int gsvcu_dit_prepare(gsvcu_dit* ctx, const float* prompt_mel, const float* mu, int32_t T, int32_t x_lens);
/* gsv_dit::velocity (src/gsv_dit.cpp:1325-1338): one estimator pass at time t; x_mel and vel [100][T]. */
int gsvcu_dit_velocity(gsvcu_dit* ctx, const float* x_mel, float t, int32_t negative, float* vel);
/* gsv_dit::sample's CFM loop (src/gsv_dit.cpp:1410-1478) on the set condition: x0 [100][T] the initial
 * noise, the first P frames zeroed, `steps` Euler steps t = j / steps of which the first skip_steps leave x
 * unchanged, guidance v + (v - v_neg) * cfg when cfg > 1e-5 (both branches in one batch); mel_out
 * [100][T - P]. */
int gsvcu_dit_sample(gsvcu_dit* ctx, const float* x0, int32_t P, int32_t steps, float cfg, int32_t skip_steps,
                     float* mel_out);
/* gsv_dit::sample (src/gsv_dit.cpp:1410-1478) in full: prompt [100][P] into the first P of T frames, prepare
 * with mu [512][T], initial noise x0 [100][T] or, when x0 is null, randn * 0.875 from gsv_rng(seed) as the
 * reference draws it; mel_out [100][T - P]. */
int gsvcu_dit_sample_full(gsvcu_dit* ctx, const float* mu, const float* prompt, int32_t P, int32_t T, int32_t steps,
                          float cfg, uint64_t seed, const float* x0, int32_t skip_steps, float* mel_out);
/* gsv_dit::synthesize (src/gsv_dit.cpp:1480-1581): the reference frames (the last 500 of min(mel_ref_T, R))
 * of mel_ref [100][mel_ref_T] and fea_ref [512][R] as prompt, fea_todo [512][N] cut into chunks of 640 frames
 * (block_override > 0: that many; reference + chunk <= 1000), each chunk after the first prompted with the
 * reference frames whose last 32 are the previous chunk's last generated frames; chunk i samples with seed
 * LCG^i(seed) and, when i < n_x0, initial noise x0_chunks[i] ([100][reference + chunk]); skip_steps applies to
 * the first chunk; mel_out [100][N]. */
int gsvcu_dit_synthesize(gsvcu_dit* ctx, const float* fea_ref, int32_t R, const float* fea_todo, int32_t N,
                         const float* mel_ref, int32_t mel_ref_T, int32_t steps, float cfg, uint64_t seed,
                         int32_t block_override, const float* const* x0_chunks, int32_t n_x0, int32_t skip_steps,
                         float* mel_out);
/* gsv_dit::time_sin (src/gsv_dit.cpp:755-769): SinusPositionEmbedding(256) of t, host only. */
void gsvcu_dit_time_sin(float t, float* out256);
/* The checkpoint's RoPE inverse frequencies [32] (gsv_dit::debug_tables' angles are n * inv_freq[i]). */
int gsvcu_dit_get_inv_freq(const gsvcu_dit* ctx, float* out32);
/* cache-dit (DBCache) of gsv_dit (gsv_dit_cfg::dbcache_*, set_dbcache; src/gsv_dit.cpp:1124-1323): with
 * fn > 0 (and < depth) every velocity runs the trunk and the first fn blocks, compares their residual with the
 * one of its branch's last full step (relative L1 over the reference's downsampled view), and, when the gates
 * allow (not a warmup step, the difference below threshold, max_cached / max_cont / max_accum), adds the
 * middle blocks' residual of that last full step instead of running them. Changing fn or downsample resets
 * the cache state; sample() resets the gates and counters. */
int gsvcu_dit_set_dbcache(gsvcu_dit* ctx, int32_t fn, float threshold, int32_t warmup, int32_t warmup_interval,
                          int32_t max_cached, int32_t max_cont, float max_accum, int32_t downsample);
/* The diffusion step the gates see (sample() sets it per step; velocity() callers set it). */
int gsvcu_dit_db_set_step(gsvcu_dit* ctx, int32_t step);
/* Counters per branch [2] (conditional, unconditional) since the last reset. */
int gsvcu_dit_db_get_stats(const gsvcu_dit* ctx, int32_t* steps, int32_t* hits2, int32_t* misses2, float* last_fd2,
                           float* acc2);
/* gsv_dit::set_alg / alg (src/gsv_dit.h:46-49, the loop src/gsv_dit.cpp:1449-1468): uncond_reuse 0 computes
 * the negative branch every guided step; 1 reuses the last computed one on odd steps; 2 extrapolates
 * 2 neg[k-1] - neg[k-2] on odd steps (once two exist). Values outside 0..2 mean 0. */
int gsvcu_dit_set_alg(gsvcu_dit* ctx, int32_t uncond_reuse);
int gsvcu_dit_get_alg(const gsvcu_dit* ctx, int32_t* uncond_reuse);
/* Test entry: the condition rows [2][T][1024] (condition, negative) of the last set_condition / prepare. */
int gsvcu_dit_op_condition(gsvcu_dit* ctx, float* out);
/* Test entry: the hidden state [2T][1024] (rows [0, T) conditioned, [T, 2T) negative) after the trunk and
 * the first n_blocks blocks at time t. */
int gsvcu_dit_op_hidden(gsvcu_dit* ctx, const float* x_mel, float t, int32_t n_blocks, float* hidden);
/* The context's CUDA stream (cudaStream_t), for timing. */
int gsvcu_dit_stream(gsvcu_dit* ctx, void** out);

/* ---------------------------------------------------------------- profiling (GSV_AR_PROFILE buckets,
 * reference src/gsv_ar.cpp:18-42) */

/* Kernel classes of one decode step, indices of ms_by_class. */
enum {
    GSVCU_PROF_SAMPLER = 0, GSVCU_PROF_STEP_PREP, GSVCU_PROF_QKV_GEMM, GSVCU_PROF_DECODE_ATTN, GSVCU_PROF_OUT_GEMM,
    GSVCU_PROF_LAYERNORM, GSVCU_PROF_FFN1_GEMM, GSVCU_PROF_FFN2_GEMM, GSVCU_PROF_PREDICT,
    GSVCU_PROF_DENSE,   /* fused layer tail: page merge, out, LN1, FFN1, FFN2, LN2, next QKV */
    GSVCU_PROF_CLASSES
};
/* Run n_steps decode steps of the slots in flight without the graph, timing every kernel class with
 * CUDA events on the context's stream; ms_by_class [GSVCU_PROF_CLASSES] gets the summed milliseconds
 * (with the fused decode step: sampler, step prep, layer 0's QKV, decode attention, fused layer tail
 * and predict; otherwise one class per unfused kernel),
 * attn_bytes (may be NULL) the algorithmic K/V + q/out bytes the attention launches read and wrote. */
int gsvcu_step_profile(gsvcu_ctx* ctx, int32_t n_steps, float* ms_by_class, int64_t* attn_bytes);
/* Decode-step variant (no counterpart in the reference; an implementation switch of this library).
 * mode 1 (default): each layer after attention runs as one 16-CTA cluster kernel (page merge,
 * out-projection, LayerNorm, FFN, LayerNorm, next layer's QKV), when the device can hold such a
 * cluster; mode 2: the same with >= 32 slots (a multiple of 32) split into two groups on forked
 * streams, so one group's layer tail may overlap the other's attention (measured on B200: no gain,
 * the clusters wait for whole SMs); mode 0: one kernel per operation. Results are identical. Returns GSVCU_OK (GSVCU_ERR_ARG for
 * another mode); gsvcu_fused_decode returns the mode in use (0 when the cluster does not fit, or
 * when the model has F32 / F16 layer matrices: the fused tail reads Q8_0 weights only). */
int gsvcu_set_fused_decode(gsvcu_ctx* ctx, int32_t mode);
/* Prefill GEMM variant (no counterpart in the reference; an implementation switch of this library) for
 * Q8_0-class matrices at 128 rows or more: mode 1 (default) runs them on the tcgen05 tensor cores (TMA
 * tiles, TMEM accumulators, the per-block float chains on CUDA cores), mode 0 on mma.sync tiles. Results
 * are identical bit for bit. */
int gsvcu_set_prefill_gemm(gsvcu_ctx* ctx, int32_t mode);
int gsvcu_fused_decode(const gsvcu_ctx* ctx);
/* Number of kernels this context has launched (graph replays count their kernels). */
int64_t gsvcu_kernel_launches(const gsvcu_ctx* ctx);
/* The context's CUDA stream (cudaStream_t), for callers that order their own work after it or time
 * it with events. */
void* gsvcu_stream(const gsvcu_ctx* ctx);

/* Synchronise the context's stream. Also reports (GSVCU_ERR_CUDA, once) a bounded wait of
 * gsvcu_op_decode_attention that gave up since the last call. */
int gsvcu_sync(gsvcu_ctx* ctx);

/* Failure-path testing (no counterpart in the reference, whose KV allocation failure exits the process,
 * src/gsv_ar.cpp:111). on = 1: every decode-attention launch of this context declares 16 bytes more on
 * its page mbarrier than it stages and gives up after 4096 polls, so its bounded wait runs out: the
 * next status read of generate / serve (or gsvcu_sync after an op call) returns GSVCU_ERR_CUDA with
 * "staged K/V never arrived", and the context stays usable. Nothing faults: the staged copies all
 * complete, only the expected count is never reached. on = 0 (default) restores normal operation. */
int gsvcu_set_wait_fault(gsvcu_ctx* ctx, int32_t on);

#ifdef __cplusplus
}
#endif

#endif /* GSVCU_H */
