// ref_shim.cpp -- C entry points over the reference's OWN CPU code for this path.
//
// TEST INFRASTRUCTURE ONLY (built into oracle/_ref/, which git ignores).  Compiled against
// the reference's sources where they lie:
//   - src/tests/cpu_ref.h            rmsNormCpu (:14-25), diff (:28-46)
//   - docs/B6_3_attention.md §5      ropeCpu (:471-481), attentionRowCpu (:483-501), taken
//                                    verbatim from the doc's code block into
//                                    oracle/_ref/doc_cpu_ref_additions.h by build_ref.py
// and composed the way the doc's attentionCpu composes them (docs/B6_3_attention.md:643-670).
// This file only adapts calling conventions; all arithmetic is the reference's.
//
// The tree's rmsNormCpu has no "nullptr weight" mode yet (the doc asks for it at :468), so a
// weightless norm passes an all-ones bf16 weight (0x3F80), which is the same arithmetic.
// The reference softmax has no scale (scale 1.0, doc :27); a scale s is applied by
// multiplying q by s first, which is exact when s is a power of two (1.0 and 1/16 here).
#include <cstdint>
#include <cstring>
#include <vector>

#include "cpu_ref.h"                  // reference: src/tests/cpu_ref.h
#include "doc_cpu_ref_additions.h"    // reference: docs/B6_3_attention.md §5 code block

namespace {
const uint16_t* ones_bf16(size_t n) {
    static thread_local std::vector<uint16_t> ones;
    if (ones.size() < n) ones.assign(n, 0x3F80);
    return ones.data();
}
uint32_t first_visible(uint32_t pos, uint32_t window) {
    return (window && pos + 1 > window) ? pos + 1 - window : 0;
}
}  // namespace

extern "C" {

void ref_rms_norm(const float* x, const uint16_t* w, float* y, size_t n, float eps) {
    rmsNormCpu(x, w ? w : ones_bf16(n), y, n, eps);
}

void ref_rope(float* x, size_t head_dim, size_t pairs, float base, uint32_t pos) {
    ropeCpu(x, head_dim, pairs, base, pos);
}

void ref_attention_row(const float* q, const float* K, const float* V, float* out,
                       size_t head_dim, size_t first, size_t last) {
    attentionRowCpu(q, K, V, out, head_dim, first, last);
}

// matvecNvfp4Cpu (src/tests/cpu_ref.h:48-63): output[t, :] = W . input[t, :], NVFP4 W [rows][n].
void ref_matvec_nvfp4(const uint32_t* codes, const uint8_t* scales, const float* input, float* output,
                      size_t tokens, size_t rows, size_t n) {
    matvecNvfp4Cpu(codes, scales, input, output, tokens, rows, n);
}

// rms_norm_f32 semantics (shaders/norm.metal:36-81) through rmsNormCpu, one row at a time, as the
// reference's test-norm computes its CPU answer (src/tests/test_norm.cpp:74-79).
void ref_rms_norm_rows(const float* input, const uint16_t* w, float* output, size_t rows, size_t n, float eps) {
    for (size_t r = 0; r < rows; ++r) rmsNormCpu(input + r * n, w ? w : ones_bf16(n), output + r * n, n, eps);
}

void ref_diff(const float* a, const float* b, size_t n, double* max_abs, double* rel_l2) {
    const Diff d = diff(a, b, n);
    *max_abs = d.max_abs;
    *rel_l2 = d.rel_l2;
}

// head_norm_rope_f32 semantics (shaders/head_norm_rope.metal:5-74) through the CPU ops, the
// way attentionCpu normalises and ropes each head (docs/B6_3_attention.md:647-658).
void ref_head_norm_rope_f32(const float* input, const uint16_t* weight, float* output,
                            uint32_t tokens, uint32_t heads, uint32_t head_dim,
                            uint32_t has_weight, uint32_t rope_pairs, float rope_base,
                            uint32_t abs_pos, uint32_t out_token_stride,
                            uint32_t out_head_stride, float eps) {
    std::vector<float> tmp(head_dim);
#pragma omp parallel for firstprivate(tmp) schedule(static)
    for (long long th = 0; th < (long long)tokens * heads; ++th) {
        const uint32_t t = uint32_t(th / heads), h = uint32_t(th % heads);
        rmsNormCpu(input + (size_t(t) * heads + h) * head_dim,
                   has_weight ? weight : ones_bf16(head_dim), tmp.data(), head_dim, eps);
        ropeCpu(tmp.data(), head_dim, rope_pairs, rope_base, abs_pos + t);
        std::memcpy(output + size_t(t) * out_token_stride + size_t(h) * out_head_stride,
                    tmp.data(), head_dim * sizeof(float));
    }
}

// The softmax-over-keys loop of attentionCpu (docs/B6_3_attention.md:661-670) for queries at
// positions pos0 + t over the cache layout [Hkv][capacity][hd] (doc :90-92).  rows selects
// query indices (nullptr = all tokens); out is [n_rows][Hq][hd].
void ref_attention(const float* q, const float* K, const float* V, float* out, uint32_t tokens,
                   uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim, uint32_t capacity,
                   uint32_t pos0, uint32_t window, float scale, const int32_t* rows,
                   uint32_t n_rows) {
    if (!rows) n_rows = tokens;
    const uint32_t group = q_heads / kv_heads;
    std::vector<float> qs(head_dim);
#pragma omp parallel for firstprivate(qs) schedule(dynamic, 1)
    for (long long rh = 0; rh < (long long)n_rows * q_heads; ++rh) {
        const uint32_t r = uint32_t(rh / q_heads), h = uint32_t(rh % q_heads);
        const uint32_t t = rows ? uint32_t(rows[r]) : r;
        const uint32_t pos = pos0 + t, kvh = h / group;
        const float* qrow = q + (size_t(t) * q_heads + h) * head_dim;
        for (uint32_t d = 0; d < head_dim; ++d) qs[d] = qrow[d] * scale;
        const size_t base = size_t(kvh) * capacity * head_dim;
        attentionRowCpu(qs.data(), K + base, V + base, out + (size_t(r) * q_heads + h) * head_dim,
                        head_dim, first_visible(pos, window), pos);
    }
}

}  // extern "C"
