// ops.h -- host operators of the attention path over apex::Backend, keeping the reference's
// signatures (src/ops.h:88-122 for headNormRope; docs/B6_3_attention.md:365-431 for
// AttentionShape, KvCache and attention) so engine code written against them runs unchanged
// on CudaBackend, plus the bf16 operators of the B200 path.
#pragma once

#include <cmath>
#include <cstdint>

#include "../../include/apex_cuda.h"
#include "backend/backend.h"

namespace apex {

// Per-layer attention geometry (docs/B6_3_attention.md:365-372).
struct AttentionShape {
    uint32_t q_heads;
    uint32_t kv_heads;
    uint32_t head_dim;
    uint32_t rope_pairs;
    float rope_base;
    uint32_t window;  // 0 = full attention
};

// One layer's f32 KV cache: K and V are [kv_heads][capacity][head_dim]
// (docs/B6_3_attention.md:394-398).
struct KvCache {
    Buffer *k;
    Buffer *v;
    uint32_t capacity;
};

// Queue RMSNorm (+ optional weight, + optional RoPE) per (token, head) with explicit output
// strides in elements; offsets in bytes.  Same signature and argument order as the reference.
inline void headNormRope(Backend &backend, Buffer *input, Buffer *weights, size_t weights_offset,
                         bool has_weights, Buffer *output, size_t output_offset, uint32_t tokens,
                         uint32_t heads, uint32_t head_dim, uint32_t rope_pairs, float rope_base,
                         uint32_t abs_pos, uint32_t out_token_stride, uint32_t out_head_stride,
                         float eps) {
    const uint32_t weight_flag = has_weights ? 1u : 0u;
    backend.run("head_norm_rope_f32",
                {Arg::buf(input), Arg::buf(weights, weights_offset), Arg::buf(output, output_offset),
                 Arg::val(heads), Arg::val(head_dim), Arg::val(weight_flag), Arg::val(rope_pairs),
                 Arg::val(rope_base), Arg::val(abs_pos), Arg::val(out_token_stride),
                 Arg::val(out_head_stride), Arg::val(eps)},
                Dim3{tokens, heads}, Dim3{256});
}

// An NVFP4 matrix [w_rows, hidden_dim] in device memory: codes and scales may live in the same
// buffer (core.bin) at different offsets (src/ops.h:8-16).
struct Nvfp4Matrix {
    Buffer *weights;
    size_t weights_offset;  // uint32 [w_rows, hidden_dim/8]
    Buffer *scales;
    size_t scales_offset;   // uint8 [w_rows, hidden_dim/16]
    uint32_t w_rows;
    uint32_t hidden_dim;
};

// Queue RMSNorm of f32 rows with bf16 weights (src/ops.h:18-27, kernel rms_norm_f32).
inline void rmsNorm(Backend &backend, Buffer *input, Buffer *weights, size_t weight_offset, Buffer *result,
                    uint32_t rows, uint32_t hidden_dim, float eps) {
    backend.run("rms_norm_f32",
                {Arg::buf(input), Arg::buf(weights, weight_offset), Arg::buf(result), Arg::val(hidden_dim),
                 Arg::val(eps)},
                Dim3{rows}, Dim3{256});
}

// Queue output[t] = W . input[t] for an NVFP4 matrix (src/ops.h:34-46, kernel matmul_nvfp4).
inline void matmulNvfp4(Backend &backend, Buffer *input, const Nvfp4Matrix &W, Buffer *output, uint32_t tokens) {
    const uint32_t row_groups = (W.w_rows + 7) / 8;
    backend.run("matmul_nvfp4",
                {Arg::buf(input), Arg::buf(W.weights, W.weights_offset), Arg::buf(W.scales, W.scales_offset),
                 Arg::buf(output), Arg::val(W.hidden_dim), Arg::val(W.w_rows)},
                Dim3{row_groups, tokens}, Dim3{256});
}

// Queue the softmax over keys for every (token, q head), scale 1.0, f32 cache
// (docs/B6_3_attention.md:424-431).
inline void attention(Backend &backend, Buffer *q, const KvCache &cache, Buffer *output,
                      const AttentionShape &s, uint32_t tokens, uint32_t pos0) {
    backend.run("attention_f32",
                {Arg::buf(q), Arg::buf(cache.k), Arg::buf(cache.v), Arg::buf(output),
                 Arg::val(s.q_heads), Arg::val(s.kv_heads), Arg::val(s.head_dim),
                 Arg::val(cache.capacity), Arg::val(pos0), Arg::val(s.window)},
                Dim3{tokens, s.q_heads}, Dim3{256});
}

// The steps of the reference's attentionBlock between its projections
// (docs/B6_3_attention.md:444-454), on f32 buffers: q normed + roped in place; K normed +
// roped into the cache at pos0; V weightless-normed into the cache; attention into o.
// k_raw doubles as v_raw on full-attention layers (docs/B6_3_attention.md:21, 441).
inline void attentionAfterProjections(Backend &backend, Buffer *q, Buffer *k_raw, Buffer *v_raw,
                                      Buffer *norms, size_t q_norm_offset, size_t k_norm_offset,
                                      const AttentionShape &s, KvCache &cache, Buffer *o,
                                      uint32_t tokens, uint32_t pos0, float eps) {
    const uint32_t hd = s.head_dim;
    headNormRope(backend, q, norms, q_norm_offset, true, q, 0, tokens, s.q_heads, hd, s.rope_pairs,
                 s.rope_base, pos0, s.q_heads * hd, hd, eps);
    const size_t cache_offset = size_t(pos0) * hd * sizeof(float);
    headNormRope(backend, k_raw, norms, k_norm_offset, true, cache.k, cache_offset, tokens, s.kv_heads,
                 hd, s.rope_pairs, s.rope_base, pos0, hd, cache.capacity * hd, eps);
    headNormRope(backend, v_raw, norms, k_norm_offset, false, cache.v, cache_offset, tokens, s.kv_heads,
                 hd, 0, s.rope_base, pos0, hd, cache.capacity * hd, eps);
    attention(backend, q, cache, o, s, tokens, pos0);
}

// ---------------------------------------------------------------- bf16 path (B200)

// bf16 cache for a batch: K, V [batch][kv_heads][capacity][head_dim].
struct KvCacheBf16 {
    Buffer *k;
    Buffer *v;
    uint32_t capacity;
};

// Numerics of the bf16 operators (apex_attn_params); scale defaults to 1/sqrt(head_dim).
inline apex_attn_params attnParams(const AttentionShape &s, float scale, float eps, bool qk_norm,
                                   bool v_norm, bool ring = false) {
    return apex_attn_params{s.q_heads, s.kv_heads, s.head_dim, s.rope_pairs, s.rope_base, s.window,
                            scale, eps, qk_norm ? 1u : 0u, v_norm ? 1u : 0u, ring ? 1u : 0u};
}

// Bytes of the workspace attentionDecodeBf16 / attentionPrefillBf16 need.
inline size_t decodeWorkspaceBytes(const apex_attn_params &p, uint32_t batch, uint32_t max_seq_len) {
    return apex_attn_decode_workspace_bytes(&p, batch, max_seq_len);
}
inline size_t prefillWorkspaceBytes(const apex_attn_params &p, uint32_t batch, uint32_t tokens) {
    return apex_attn_prefill_workspace_bytes(&p, batch, tokens);
}

// One fused decode step for `batch` sequences (apex_attn_decode_bf16).  The workspace's
// counters must be zero before its first use (allocate() memory is not zeroed: memset it once).
inline void attentionDecodeBf16(Backend &backend, const apex_attn_params &p, Buffer *q_raw, Buffer *k_new,
                                Buffer *v_new, Buffer *q_norm_w, Buffer *k_norm_w, KvCacheBf16 &cache,
                                Buffer *seq_lens, uint32_t batch, uint32_t max_seq_len, Buffer *out,
                                Buffer *workspace) {
    backend.run("attention_decode_bf16",
                {Arg::buf(q_raw), Arg::buf(k_new), Arg::buf(v_new), Arg::buf(q_norm_w), Arg::buf(k_norm_w),
                 Arg::buf(cache.k), Arg::buf(cache.v), Arg::buf(seq_lens), Arg::buf(out), Arg::buf(workspace),
                 Arg::val(p), Arg::val(cache.capacity), Arg::val(max_seq_len)},
                Dim3{batch}, Dim3{160});
}

// Fused prefill of `tokens` tokens per sequence at pos0 (apex_attn_prefill_bf16).
inline void attentionPrefillBf16(Backend &backend, const apex_attn_params &p, Buffer *q_raw, Buffer *k_raw,
                                 Buffer *v_raw, Buffer *q_norm_w, Buffer *k_norm_w, KvCacheBf16 &cache,
                                 uint32_t batch, uint32_t tokens, uint32_t pos0, Buffer *out,
                                 Buffer *workspace) {
    backend.run("attention_prefill_bf16",
                {Arg::buf(q_raw), Arg::buf(k_raw), Arg::buf(v_raw), Arg::buf(q_norm_w), Arg::buf(k_norm_w),
                 Arg::buf(cache.k), Arg::buf(cache.v), Arg::buf(out), Arg::buf(workspace), Arg::val(p),
                 Arg::val(cache.capacity), Arg::val(pos0)},
                Dim3{tokens, batch}, Dim3{256});
}

// LSE merge of [num_partials][rows][head_dim+2] partials into out [rows][head_dim] bf16.
inline void mergePartials(Backend &backend, Buffer *partials, uint32_t num_partials, uint32_t rows,
                          uint32_t head_dim, Buffer *out) {
    backend.run("attention_merge_partials",
                {Arg::buf(partials), Arg::buf(out), Arg::val(num_partials), Arg::val(head_dim)}, Dim3{rows},
                Dim3{256});
}

}  // namespace apex
