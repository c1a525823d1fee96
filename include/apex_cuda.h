/*
 * apex_cuda.h -- C ABI of the B200 (sm_100a) attention hot path.
 *
 * The drop-in boundary for the reference's attention stage: per-head QK RMSNorm + RoPE fused
 * into grouped-query attention over a KV cache.  Plain pointers and sizes only.  Every
 * pointer argument named as a tensor is a DEVICE pointer unless stated otherwise; `stream`
 * is a cudaStream_t passed as void* (NULL = legacy default stream).  Calls only enqueue work;
 * they return before the GPU finishes, like the reference's Backend::run
 * (src/backend/backend.h:55-56), and report launch-time errors as a nonzero status.
 *
 * Reference interfaces replaced (paths inside the spotta85/apex tree):
 *   apex_head_norm_rope_f32   kernel head_norm_rope_f32 (shaders/head_norm_rope.metal:5-20),
 *                             launched by apex::headNormRope (src/ops.h:88-122) through
 *                             Backend::run (src/backend/backend.h:55-56)
 *   apex_attention_f32        kernel attention_f32 (docs/B6_3_attention.md:282-295), launched
 *                             by apex::attention (docs/B6_3_attention.md:424-431)
 *   apex_head_norm_rope_bf16, apex_attn_decode_bf16, apex_attn_decode_partial_bf16,
 *   apex_attn_merge_partials, apex_attn_prefill_bf16
 *                             the bf16 KV-cache path the reference plans (f16 cache,
 *                             docs/B6_3_attention.md:99-102) with the steps of
 *                             apex::attentionBlock between its projections
 *                             (docs/B6_3_attention.md:444-454) fused per call.
 */
#ifndef APEX_CUDA_H
#define APEX_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define APEX_API __attribute__((visibility("default")))
#else
#define APEX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define APEX_OK 0
#define APEX_ERR_INVALID_ARGUMENT 1 /* a size, pointer, alignment or stride was rejected */
#define APEX_ERR_UNSUPPORTED 2      /* valid request this build has no kernel for */
#define APEX_ERR_CUDA 3             /* a CUDA runtime call failed */
#define APEX_ERR_WORKSPACE 4        /* workspace missing or too small */
#define APEX_ERR_DEVICE_TIMEOUT 5   /* a kernel's bounded wait gave up (see apex_cuda_device_status) */

/* Attention geometry and numerics of one layer: the reference's AttentionShape
 * (docs/B6_3_attention.md:365-372) plus the knobs the bf16 configurations need.
 *   scale    softmax scale (the reference model uses 1.0, docs/B6_3_attention.md:27)
 *   qk_norm  1: RMSNorm q and k over head_dim (weights optional), 0: no norm
 *   v_norm   1: weightless RMSNorm of v (the reference model, docs/B6_3_attention.md:25)
 *   window   0 = global causal; else key j is visible to the query at position p iff
 *            p - window < j <= p (docs/B6_3_attention.md:42)
 *   ring     see the field                                                                 */
typedef struct apex_attn_params {
    uint32_t q_heads;
    uint32_t kv_heads;
    uint32_t head_dim;
    uint32_t rope_pairs; /* pairs (i, i + head_dim/2) rotated, 0 = no RoPE */
    float rope_base;
    uint32_t window;
    float scale;
    float eps;
    uint32_t qk_norm;
    uint32_t v_norm;
    uint32_t ring;       /* decode only: 1 = the cache is a ring of `capacity` slots, position p at slot
                            p % capacity (the reference's planned sliding-layer cache,
                            docs/B6_3_attention.md:99-102); needs 0 < window <= capacity.  0 = linear. */
} apex_attn_params;

/* Message of the last failing call on this host thread ("" if none). */
APEX_API const char *apex_cuda_last_error(void);
/* ABI version of this library (major * 100 + minor). */
APEX_API int apex_cuda_abi_version(void);
/* Reads and clears the device-side status word written by kernels whose bounded waits gave
 * up; synchronises `stream`.  Returns APEX_OK or APEX_ERR_DEVICE_TIMEOUT. */
APEX_API int apex_cuda_device_status(void *stream);

/* ------------------------------------------------------------------ f32 drop-ins */

/* Per (token, head): RMSNorm over head_dim with an optional bf16 weight, then RoPE on the
 * first rope_pairs pairs (i, i + head_dim/2) at position abs_pos + token, written to
 * output[token * out_token_stride + head * out_head_stride + d].  input is
 * [tokens][heads][head_dim] f32; weight is head_dim raw bf16 bits (read iff has_weight).
 * input == output is allowed when the strides equal the input layout.  head_dim <= 512,
 * even.  Same arguments, in the same order, as src/ops.h:88-122. */
APEX_API int apex_head_norm_rope_f32(const float *input, const uint16_t *weight, float *output,
                            uint32_t tokens, uint32_t heads, uint32_t head_dim,
                            uint32_t has_weight, uint32_t rope_pairs, float rope_base,
                            uint32_t abs_pos, uint32_t out_token_stride,
                            uint32_t out_head_stride, float eps, void *stream);

/* Softmax over keys for every (token, q head), scale 1.0, as attention_f32.
 * q, out [tokens][q_heads][head_dim]; K, V [kv_heads][capacity][head_dim] f32; the query of
 * token t sits at position pos0 + t and sees keys per `window`.  head_dim <= 512. */
APEX_API int apex_attention_f32(const float *q, const float *K, const float *V, float *out,
                       uint32_t tokens, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                       uint32_t capacity, uint32_t pos0, uint32_t window, void *stream);

/* apex_attention_f32 with an explicit softmax scale. */
APEX_API int apex_attention_f32_scaled(const float *q, const float *K, const float *V, float *out,
                              uint32_t tokens, uint32_t q_heads, uint32_t kv_heads,
                              uint32_t head_dim, uint32_t capacity, uint32_t pos0,
                              uint32_t window, float scale, void *stream);

/* ------------------------------------------------------------------ bf16 hot path */

/* apex_head_norm_rope_f32 on bf16 input/output (the K/V cache append of the bf16 path).
 * All bf16 tensors are raw uint16 bits. */
APEX_API int apex_head_norm_rope_bf16(const uint16_t *input, const uint16_t *weight, uint16_t *output,
                             uint32_t tokens, uint32_t heads, uint32_t head_dim,
                             uint32_t has_weight, uint32_t rope_pairs, float rope_base,
                             uint32_t abs_pos, uint32_t out_token_stride,
                             uint32_t out_head_stride, float eps, void *stream);

/* Workspace bytes apex_attn_decode_bf16 needs for up to `batch` sequences of at most
 * max_seq_len keys (split-KV partials + per-(sequence, kv head) counters). */
APEX_API size_t apex_attn_decode_workspace_bytes(const apex_attn_params *p, uint32_t batch,
                                        uint32_t max_seq_len);
/* Zero the workspace's counters; required once before the first decode call that uses it
 * (every call leaves them zero again). */
APEX_API int apex_attn_decode_workspace_init(void *workspace, size_t workspace_bytes, void *stream);

/* One decode step of `batch` sequences, fused: for each sequence b with seq_lens[b] keys
 * (the new token included, at position seq_lens[b]-1):
 *   q    = rope(rmsnorm(q_raw[b], q_norm_w))                      -- in registers
 *   K[b][:, L-1] = rope(rmsnorm(k_new[b], k_norm_w)), V[b][:, L-1] = [rmsnorm](v_new[b])
 *   out[b] = softmax(scale * q K^T) V over the visible keys          (split-KV, LSE merge)
 * q_raw [B][Hq][D]; k_new, v_new [B][Hkv][D]; caches [B][Hkv][capacity][D]; seq_lens is a
 * DEVICE int32 [B] with 1 <= seq_lens[b] <= max_seq_len <= capacity (a ring cache: any max_seq_len,
 * window <= capacity); out [B][Hq][D].  Norm weights are bf16 [D] or NULL (weight 1.0).
 * head_dim 256 with Hq / Hkv = 2 (split-KV kernel; short contexts of small batches as thread-block
 * clusters), or head_dim 256 / 512 with 1..8 q heads per kv head (tensor-core decode of the
 * reference model's global layers; linear caches). */
APEX_API int apex_attn_decode_bf16(const apex_attn_params *p, const uint16_t *q_raw,
                          const uint16_t *k_new, const uint16_t *v_new,
                          const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                          uint16_t *k_cache, uint16_t *v_cache, uint32_t capacity,
                          const int32_t *seq_lens, uint32_t batch, uint32_t max_seq_len,
                          uint16_t *out, void *workspace, size_t workspace_bytes,
                          void *stream);

/* apex_attn_decode_bf16 for callers that cannot allocate device memory: an engine that keeps
 * all of its device memory under its own fixed budget, or a decode loop that cannot take
 * cudaMalloc's implicit synchronisation.  Same arguments minus the workspace.  It has no
 * counterpart in the reference.
 *   - Scratch is a static 8 MiB device array inside this library, reserved on every GPU the
 *     library is used on until the process exits.  Requests that need more (the size
 *     apex_attn_decode_workspace_bytes reports for batch x max_seq_len; all five benchmark
 *     configurations fit) fail with APEX_ERR_WORKSPACE and launch nothing.
 *   - The first call on each device looks up the array's device address (once per device);
 *     make that first call before any stream capture.
 *   - Allocates nothing: no cudaMalloc, no cudaFree, no allocating library routine.  Each
 *     call clears the scratch counters it needs on `stream` before the kernel.  Every argument
 *     is checked first: a rejected call queues nothing on `stream`.
 *   - Every call shares the one array: calls whose execution overlaps on the GPU (other
 *     streams, other host threads) race and corrupt each other's results; serialise them. */
APEX_API int apex_attn_decode_bf16_noalloc(const apex_attn_params *p, const uint16_t *q_raw,
                                           const uint16_t *k_new, const uint16_t *v_new,
                                           const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                                           uint16_t *k_cache, uint16_t *v_cache, uint32_t capacity,
                                           const int32_t *seq_lens, uint32_t batch,
                                           uint32_t max_seq_len, uint16_t *out, void *stream);

/* Ring caches (apex_attn_params.ring): copies the last min(length, ring_capacity) positions of a linear
 * cache [batch][kv_heads][linear_capacity][head_dim] (e.g. what a prefill wrote) into a ring
 * [batch][kv_heads][ring_capacity][head_dim], position p at slot p % ring_capacity -- the reference's
 * planned 1024-entry sliding-layer cache (docs/B6_3_attention.md:99-102).  bf16 bits; 16-byte aligned. */
APEX_API int apex_kv_ring_store(const uint16_t *k_linear, const uint16_t *v_linear, uint16_t *k_ring, uint16_t *v_ring,
                                uint32_t batch, uint32_t kv_heads, uint32_t head_dim, uint32_t linear_capacity,
                                uint32_t ring_capacity, uint32_t length, void *stream);

/* KV-sequence-split decode: this caller holds global key positions [kv_begin, kv_end) of
 * every sequence, stored at local cache index (position - kv_begin).  Same fused step as
 * apex_attn_decode_bf16 restricted to those keys (the new token is appended here only if
 * seq_lens[b]-1 falls in the range), producing one partial per (b, q head):
 *   partial[(b*Hq + h)*(D+2) + d] = o_d (normalised),  [.. + D] = m (log2 units),
 *   [.. + D+1] = l, with m = max_j s_j*scale*log2(e), l = sum_j 2^(s_j*scale*log2e - m).
 * A sequence with no keys in the range gets l = 0.  max_seq_len bounds the GLOBAL length. */
APEX_API int apex_attn_decode_partial_bf16(const apex_attn_params *p, const uint16_t *q_raw,
                                  const uint16_t *k_new, const uint16_t *v_new,
                                  const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                                  uint16_t *k_cache, uint16_t *v_cache, uint32_t capacity,
                                  const int32_t *seq_lens, uint32_t batch,
                                  uint32_t max_seq_len, uint32_t kv_begin, uint32_t kv_end,
                                  float *partial, void *workspace, size_t workspace_bytes,
                                  void *stream);

/* ------------------------------------------------------------------ KV split over GPUs, fused
 * The reference runs on one device, so nothing here has a counterpart in it.  A KV range split
 * over the GPUs of one NVLink domain is merged inside the decode kernel: each rank writes its
 * partial (the apex_attn_decode_partial_bf16 record) straight into every rank's gather buffer
 * over NVLink, each value as one 8-byte word that carries the step number beside it, waits until
 * its words of every rank carry this step (bounded: on expiry the device status word reports a
 * timeout) and merges.  One launch per step, no collective call, no flag and no fence.
 *
 * Buffers (per rank, zero-initialised, e.g. by apex_device_alloc; shared with the other ranks by
 * apex_ipc_get_handle / apex_ipc_open_handle):
 *   gather  [2][world][batch*q_heads][head_dim+2] uint64 (step << 32 | f32 bits; two slots,
 *                                                         alternating by step)
 *   flags   [world][batch*kv_heads] uint32               (a rank's poison mark, set on failure)
 *   seq     [batch*kv_heads] uint32                      (this rank's step counters)
 * Every rank must call apex_attn_decode_kvsplit_bf16 the same number of times with the same
 * batch and the same world; calls on one rank are serialised (one stream).
 *
 * Failure: the wait for the other ranks' partials gives up after wait_ns (0 = one second).  The
 * step then leaves `out` unwritten for that (sequence, kv head), the device status word reports
 * a timeout (apex_cuda_device_status returns APEX_ERR_DEVICE_TIMEOUT), and the pair's step counter
 * and this rank's flag on every peer are poisoned: every later step of that pair, on every rank,
 * reports a timeout and publishes and merges nothing (a rank that went on after a failed wait
 * could otherwise overwrite a gather slot a slow peer still reads).  After APEX_ERR_DEVICE_TIMEOUT
 * all ranks must stop and build new, zeroed exchange buffers before the next KV-split step. */
typedef struct apex_peer_exchange {
    uint32_t rank, world;       /* 1 <= world <= 8, rank < world */
    float *gather[8];           /* gather[r]: rank r's gather buffer as mapped in this process, 16-byte aligned */
    uint32_t *flags[8];         /* flags[r]: rank r's flag array as mapped in this process */
    uint32_t *seq;              /* this rank's step counters */
    uint64_t wait_ns;           /* bound of the wait for the other ranks, in ns; 0 = 1 s */
} apex_peer_exchange;

/* Bytes of the three buffers above for `batch` sequences over `world` ranks. */
APEX_API int apex_attn_peer_exchange_bytes(const apex_attn_params *p, uint32_t batch, uint32_t world,
                                           size_t *gather_bytes, size_t *flag_bytes, size_t *seq_bytes);

/* apex_attn_decode_partial_bf16 on this rank's key range [kv_begin, kv_end), then the exchange
 * and merge above: out [B][Hq][D] bf16 holds the full decode output on every rank. */
APEX_API int apex_attn_decode_kvsplit_bf16(const apex_attn_params *p, const uint16_t *q_raw,
                                           const uint16_t *k_new, const uint16_t *v_new,
                                           const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                                           uint16_t *k_cache, uint16_t *v_cache, uint32_t capacity,
                                           const int32_t *seq_lens, uint32_t batch, uint32_t max_seq_len,
                                           uint32_t kv_begin, uint32_t kv_end, const apex_peer_exchange *x,
                                           uint16_t *out, void *workspace, size_t workspace_bytes,
                                           void *stream);

/* Zeroed device memory from cudaMalloc (for buffers shared by CUDA IPC, which needs the base of
 * an allocation), and its release.  No counterpart in the reference. */
APEX_API int apex_device_alloc(size_t bytes, void **ptr);
APEX_API int apex_device_free(void *ptr);
/* CUDA IPC: a 64-byte handle for an apex_device_alloc pointer, the same memory opened in another
 * process (peer access enabled on demand), and closing it.  No counterpart in the reference. */
APEX_API int apex_ipc_get_handle(const void *ptr, void *handle64);
APEX_API int apex_ipc_open_handle(const void *handle64, void **ptr);
APEX_API int apex_ipc_close_handle(void *ptr);

/* Log-sum-exp merge of num_partials partial sets laid out [num_partials][rows][D+2] (the
 * apex_attn_decode_partial_bf16 format, e.g. after an all-gather) into out [rows][D] bf16. */
APEX_API int apex_attn_merge_partials(const float *partials, uint32_t num_partials, uint32_t rows,
                             uint32_t head_dim, uint16_t *out, void *stream);

/* Workspace bytes apex_attn_prefill_bf16 needs: the normalised, head-major Q plus 256 bytes
 * of scheduler state for the persistent attention kernel. */
APEX_API size_t apex_attn_prefill_workspace_bytes(const apex_attn_params *p, uint32_t batch,
                                         uint32_t tokens);

/* The first stage of apex_attn_prefill_bf16 on its own: q/k norm + RoPE, K/V appended to the
 * caches at pos0, normalised q written head-major into the workspace ([B][Hq][T][D] bf16 at its
 * start), and the attention stage's scheduler state reset.  workspace: as for
 * apex_attn_prefill_bf16. */
APEX_API int apex_attn_prefill_prep_bf16(const apex_attn_params *p, const uint16_t *q_raw,
                                         const uint16_t *k_raw, const uint16_t *v_raw,
                                         const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                                         uint16_t *k_cache, uint16_t *v_cache, uint32_t capacity,
                                         uint32_t batch, uint32_t tokens, uint32_t pos0,
                                         void *workspace, size_t workspace_bytes, void *stream);

/* The second stage on its own: tcgen05 attention of the normalised q held in the workspace
 * (written by apex_attn_prefill_prep_bf16 for the same batch / tokens / pos0) over cache
 * positions [0, pos0+tokens) -> out [B][T][Hq][D].  Persistent: one CTA per SM. */
APEX_API int apex_attn_prefill_attend_bf16(const apex_attn_params *p, void *workspace,
                                           size_t workspace_bytes, const uint16_t *k_cache,
                                           const uint16_t *v_cache, uint32_t capacity,
                                           uint32_t batch, uint32_t tokens, uint32_t pos0,
                                           uint16_t *out, void *stream);

/* Causal (optionally sliding-window) prefill of `tokens` new tokens per sequence at
 * positions pos0 .. pos0+tokens-1, fused: q/k norm + RoPE, K/V appended to the caches, then
 * attention over cache positions [0, pos0+tokens) on tcgen05 tensor cores.
 * q_raw [B][T][Hq][D]; k_raw, v_raw [B][T][Hkv][D]; caches [B][Hkv][capacity][D] with
 * positions < pos0 already filled; out [B][T][Hq][D].  head_dim 256; 16-byte aligned
 * pointers. */
APEX_API int apex_attn_prefill_bf16(const apex_attn_params *p, const uint16_t *q_raw,
                           const uint16_t *k_raw, const uint16_t *v_raw,
                           const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                           uint16_t *k_cache, uint16_t *v_cache, uint32_t capacity,
                           uint32_t batch, uint32_t tokens, uint32_t pos0, uint16_t *out,
                           void *workspace, size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------ projections and norm
 * The calls either side of the attention path in the reference's attention block
 * (docs/B6_3_attention.md:15-28): q/k/v projections before it, o projection and the
 * post-attention RMSNorm after it.  NVFP4 matrix W [w_rows][hidden_dim]: codes uint32
 * [w_rows][hidden_dim/8] (8 E2M1 codes per word, low nibble first, sign in bit 3) and E4M3 scales
 * uint8 [w_rows][hidden_dim/16] (src/nvfp4.h:11-43).  hidden_dim a multiple of 16; codes 8-byte
 * and input 16-byte aligned. */

/* matmul_nvfp4 (shaders/matmul.metal:4-53, launched by apex::matmulNvfp4, src/ops.h:34-46), buffers
 * in the reference's order: output[t][r] = W[r] . input[t], input [tokens][hidden_dim] f32,
 * output [tokens][w_rows] f32. */
APEX_API int apex_matmul_nvfp4_f32(const float *input, const uint32_t *codes, const uint8_t *scales, float *output,
                                   uint32_t hidden_dim, uint32_t w_rows, uint32_t tokens, void *stream);
/* The same with bf16 input and / or bf16 output (raw bits) for the bf16 attention path: e.g. the raw
 * q/k/v rows apex_attn_decode_bf16 takes, or o_proj over its bf16 output. */
APEX_API int apex_matmul_nvfp4(const void *input, int input_bf16, const uint32_t *codes, const uint8_t *scales,
                               void *output, int output_bf16, uint32_t hidden_dim, uint32_t w_rows, uint32_t tokens,
                               void *stream);
/* Up to four projections of the same input in one launch (q, k and v of a layer: the reference's
 * three matmulNvfp4 calls on one normed hidden state, src/ops.h:34-46): matrix m is codes[m] /
 * scales[m] with w_rows[m] rows of hidden_dim, written to outputs[m] ([tokens][w_rows[m]]); every
 * output is what apex_matmul_nvfp4 would write.  Arrays are host arrays of count entries. */
APEX_API int apex_matmul_nvfp4_multi(const void *input, int input_bf16, uint32_t count, const uint32_t *const *codes,
                                     const uint8_t *const *scales, void *const *outputs, const uint32_t *w_rows,
                                     int output_bf16, uint32_t hidden_dim, uint32_t tokens, void *stream);
/* rms_norm_f32 (shaders/norm.metal:36-81, apex::rmsNorm, src/ops.h:18-27): result[r] =
 * input[r] * rsqrt(mean(input[r]^2) + eps) * weight, rows of hidden_dim f32, weight bf16 bits. */
APEX_API int apex_rms_norm_f32(const float *input, const uint16_t *weight, float *result, uint32_t rows,
                               uint32_t hidden_dim, float eps, void *stream);
/* Workspace bytes of apex_matmul_nvfp4_rms_norm (zeroed once before first use, e.g. with
 * apex_attn_decode_workspace_init; every call leaves it ready for the next). */
APEX_API size_t apex_matmul_nvfp4_rms_norm_workspace_bytes(uint32_t w_rows, uint32_t tokens);
/* o_proj with the post-attention RMSNorm fused into its epilogue: output[t] = rmsnorm(W . input[t],
 * norm_weight) (attn_out of docs/B6_3_attention.md:27-28), and when residual_out is given also
 * residual_out[t] = residual[t] + output[t] (residual may be NULL: zero).  output [tokens][w_rows]
 * f32.  Up to 16 tokens it is one launch (the last CTA normalises); more tokens run the norm as a
 * second launch. */
APEX_API int apex_matmul_nvfp4_rms_norm(const void *input, int input_bf16, const uint32_t *codes, const uint8_t *scales,
                                        const uint16_t *norm_weight, const float *residual, float *output,
                                        float *residual_out, uint32_t hidden_dim, uint32_t w_rows, uint32_t tokens,
                                        float eps, void *workspace, size_t workspace_bytes, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* APEX_CUDA_H */
