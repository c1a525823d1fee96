/*
 * apex_oracle.c -- CPU oracle for the attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product path (apex_b200/, include/) links,
 * loads or calls this file.  It is imported by tests/, by __graft_entry__.smoke() as the
 * checker, and by bench.py's cpu_baseline / --impl reference legs as the timed CPU path.
 *
 * A plain-C restatement of the reference's CPU arithmetic for this path, written from the
 * reference's own CPU code and design spec (paths are relative to the spotta85/apex tree):
 *   - orc_rms_norm        src/tests/cpu_ref.h:14-25  (double sum of squares, f32 scale);
 *                         docs/B6_3_attention.md:468 (a NULL weight means weight 1.0)
 *   - orc_rope            docs/B6_3_attention.md:471-481, shaders/head_norm_rope.metal:54-68
 *                         (rotate-half pairs (i, i+hd/2), angle = pos * base^(-2i/hd) in f32,
 *                         exponent over the FULL head_dim)
 *   - orc_head_norm_rope_f32  shaders/head_norm_rope.metal:5-74 launched by
 *                         src/ops.h:88-122 (strides in elements, position abs_pos + token)
 *   - orc_attention_row   docs/B6_3_attention.md:483-501 (exact softmax, double accumulation)
 *   - orc_attention_f32   docs/B6_3_attention.md:282-344 (GQA map h/(Hq/Hkv), window rule
 *                         first = window && pos+1 > window ? pos+1-window : 0) and the CPU
 *                         loop of docs/B6_3_attention.md:661-670
 *   - orc_e2m1 / orc_e4m3  src/nvfp4.h:11-28 (E2M1 table with sign in bit 3; finite E4M3,
 *                         exponent bias 7, e == 0 subnormal m/512)
 *   - orc_matvec_nvfp4    src/tests/cpu_ref.h:48-63 with src/nvfp4.h:31-43: every weight row
 *                         decoded (code i of a 16-weight group at word 2g + i/8, nibble i%8, times
 *                         the group's E4M3 scale), then dotted with each token in double
 *   - orc_rms_norm_rows   shaders/norm.metal:36-81 on rows of a [rows][n] matrix with the
 *                         arithmetic of orc_rms_norm (cpu_ref.h:14-25)
 * plus compositions for the bf16 configurations (prefill with K/V cache append, ragged
 * decode, split-KV partials and their log-sum-exp merge), a bf16 rounding helper and the
 * seeded synthetic-input generator shared by the tests and the golden fixtures.
 *
 * The only departure from the reference is the softmax scale argument: the reference uses
 * scale 1.0 (docs/B6_3_attention.md:27,37); the benchmark configurations use 1/sqrt(hd).
 * Passing scale = 1.0 reproduces the reference exactly.
 *
 * Build with -ffp-contract=off so no multiply-add is fused (the reference oracle is plain
 * IEEE float/double arithmetic).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------- bf16 helpers */

float orc_bf16_to_f32(uint16_t h) {
    uint32_t b = (uint32_t)h << 16;
    float f;
    memcpy(&f, &b, 4);
    return f;
}

/* Round to nearest even; NaN stays NaN. */
uint16_t orc_f32_to_bf16(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    if ((b & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((b >> 16) | 0x40u);
    b += 0x7fffu + ((b >> 16) & 1u);
    return (uint16_t)(b >> 16);
}

static inline float bf16_round(float f) { return orc_bf16_to_f32(orc_f32_to_bf16(f)); }

void orc_round_bf16_inplace(float *x, size_t n) {
    for (size_t i = 0; i < n; ++i) x[i] = bf16_round(x[i]);
}

void orc_bf16_to_f32_array(const uint16_t *in, float *out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = orc_bf16_to_f32(in[i]);
}

void orc_f32_to_bf16_array(const float *in, uint16_t *out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = orc_f32_to_bf16(in[i]);
}

/* ---------------------------------------------------------------- threads */

void orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ---------------------------------------------------------------- synthetic inputs
 * Counter-based generator: every element is a pure function of (seed, stream, index), so
 * any slice of a tensor can be regenerated on its own.  splitmix64 finaliser for the bits,
 * Box-Muller (cosine branch only) in double for N(0,1), then mean + std * z rounded to bf16.
 */
static inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static inline uint64_t rng_bits(uint64_t key, uint64_t i) {
    return mix64(key ^ (i * 0xD1B54A32D192ED03ull));
}

static inline uint64_t rng_key(uint64_t seed, uint64_t stream) {
    return mix64(mix64(seed) ^ (stream * 0xA0761D6478BD642Full));
}

static inline double rng_unit(uint64_t bits) { /* (0, 1) */
    return ((double)(bits >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}

void orc_fill_normal_bf16(uint16_t *out, size_t n, uint64_t seed, uint64_t stream,
                          uint64_t offset, float mean, float std) {
    const uint64_t key = rng_key(seed, stream);
    const double two_pi = 6.283185307179586476925286766559;
#pragma omp parallel for schedule(static)
    for (long long k = 0; k < (long long)n; ++k) {
        const uint64_t i = offset + (uint64_t)k;
        const double u1 = rng_unit(rng_bits(key, 2 * i));
        const double u2 = rng_unit(rng_bits(key, 2 * i + 1));
        const double z = sqrt(-2.0 * log(u1)) * cos(two_pi * u2);
        out[k] = orc_f32_to_bf16((float)((double)mean + (double)std * z));
    }
}

/* Integers uniform in [lo, hi] (inclusive). */
void orc_fill_uniform_int(int32_t *out, size_t n, uint64_t seed, uint64_t stream,
                          int32_t lo, int32_t hi) {
    const uint64_t key = rng_key(seed, stream);
    const uint64_t span = (uint64_t)((int64_t)hi - (int64_t)lo + 1);
    for (size_t i = 0; i < n; ++i) out[i] = lo + (int32_t)(rng_bits(key, i) % span);
}

/* ---------------------------------------------------------------- per-head math */

/* src/tests/cpu_ref.h:14-25; w == NULL means weight 1.0 (docs/B6_3_attention.md:468).
 * Reads all of x before writing y, so x == y is allowed (docs/B6_3_attention.md:675-677). */
void orc_rms_norm(const float *x, const uint16_t *w, float *y, size_t n, float eps) {
    double ss = 0.0;
    for (size_t i = 0; i < n; ++i) ss += (double)x[i] * x[i];
    const float inv = 1.0f / sqrtf((float)(ss / (double)n) + eps);
    for (size_t i = 0; i < n; ++i) {
        const float wf = w ? orc_bf16_to_f32(w[i]) : 1.0f;
        y[i] = x[i] * inv * wf;
    }
}

/* docs/B6_3_attention.md:471-481; shaders/head_norm_rope.metal:54-68. */
void orc_rope(float *x, size_t hd, size_t pairs, float base, uint32_t pos) {
    const size_t half = hd / 2;
    for (size_t i = 0; i < pairs; ++i) {
        const float angle = (float)pos * powf(base, -2.0f * (float)i / (float)hd);
        const float c = cosf(angle), s = sinf(angle);
        const float a = x[i], b = x[half + i];
        x[i] = a * c - b * s;
        x[half + i] = a * s + b * c;
    }
}

/* shaders/head_norm_rope.metal:5-74 as launched by src/ops.h:88-122: one (token, head)
 * slice at a time; output element d of (t, h) at output[t*ots + h*ohs + d]. */
void orc_head_norm_rope_f32(const float *input, const uint16_t *weight, float *output,
                            uint32_t tokens, uint32_t heads, uint32_t head_dim,
                            uint32_t has_weight, uint32_t rope_pairs, float rope_base,
                            uint32_t abs_pos, uint32_t out_token_stride,
                            uint32_t out_head_stride, float eps) {
#pragma omp parallel for schedule(static)
    for (long long th = 0; th < (long long)tokens * heads; ++th) {
        const uint32_t t = (uint32_t)(th / heads), h = (uint32_t)(th % heads);
        float tmp[1024];
        orc_rms_norm(input + ((size_t)t * heads + h) * head_dim, has_weight ? weight : NULL, tmp,
                     head_dim, eps);
        orc_rope(tmp, head_dim, rope_pairs, rope_base, abs_pos + t);
        float *o = output + (size_t)t * out_token_stride + (size_t)h * out_head_stride;
        for (uint32_t d = 0; d < head_dim; ++d) o[d] = tmp[d];
    }
}

/* docs/B6_3_attention.md:483-501: softmax_j(scale * q.K_j) V_j over keys first..last,
 * double accumulation, exact softmax.  Key j of K/V starts at element j * hd. */
void orc_attention_row(const float *q, const float *K, const float *V, float *out, size_t hd,
                       size_t first, size_t last, double scale) {
    const size_t n = last - first + 1;
    double *score = (double *)malloc(n * sizeof(double));
    double m = -INFINITY;
    for (size_t j = first; j <= last; ++j) {
        double s = 0.0;
        const float *k = K + j * hd;
        for (size_t d = 0; d < hd; ++d) s += (double)q[d] * k[d];
        s *= scale;
        score[j - first] = s;
        if (s > m) m = s;
    }
    double l = 0.0;
    for (size_t j = 0; j < n; ++j) {
        score[j] = exp(score[j] - m);
        l += score[j];
    }
    for (size_t d = 0; d < hd; ++d) {
        double acc = 0.0;
        for (size_t j = first; j <= last; ++j) acc += score[j - first] * V[j * hd + d];
        out[d] = (float)(acc / l);
    }
    free(score);
}

/* First visible key for the query at position pos (docs/B6_3_attention.md:42, 299). */
static inline uint32_t first_visible(uint32_t pos, uint32_t window) {
    return (window && pos + 1 > window) ? pos + 1 - window : 0;
}

/* The designed attention_f32 (docs/B6_3_attention.md:282-344): q [T][Hq][hd];
 * K, V [Hkv][capacity][hd]; out [T][Hq][hd]. */
void orc_attention_f32(const float *q, const float *K, const float *V, float *out,
                       uint32_t tokens, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                       uint32_t capacity, uint32_t pos0, uint32_t window, float scale) {
    const uint32_t group = q_heads / kv_heads;
#pragma omp parallel for schedule(dynamic, 1)
    for (long long th = 0; th < (long long)tokens * q_heads; ++th) {
        const uint32_t t = (uint32_t)(th / q_heads), h = (uint32_t)(th % q_heads);
        const uint32_t kvh = h / group, pos = pos0 + t;
        const size_t base = (size_t)kvh * capacity * head_dim;
        orc_attention_row(q + ((size_t)t * q_heads + h) * head_dim, K + base, V + base,
                          out + ((size_t)t * q_heads + h) * head_dim, head_dim,
                          first_visible(pos, window), pos, (double)scale);
    }
}

/* ---------------------------------------------------------------- bf16-path compositions
 * The bf16 configurations run the reference's attentionBlock steps between the projections
 * (docs/B6_3_attention.md:444-454): q norm+rope, K norm+rope into the cache at pos0, V into
 * the cache (weightless norm when v_norm is set), then attention.  Inputs are f32 arrays that
 * hold bf16 values.  round_bf16 = 1 rounds the normalised q/K/V to bf16 the way the GPU
 * stores them; 0 keeps them in f32 (the fp32 reference the tolerance is stated against).
 */

/* raw [T][H][D] -> cache [H][cap][D] at positions pos0 .. pos0+T-1. */
void orc_kv_append(const float *raw, const uint16_t *w, int norm, uint32_t rope_pairs,
                   float rope_base, float eps, float *cache, uint32_t cap, uint32_t pos0,
                   uint32_t T, uint32_t H, uint32_t D, int round_bf16) {
#pragma omp parallel for schedule(static)
    for (long long th = 0; th < (long long)T * H; ++th) {
        const uint32_t t = (uint32_t)(th / H), h = (uint32_t)(th % H);
        float tmp[1024];
        const float *src = raw + ((size_t)t * H + h) * D;
        if (norm) orc_rms_norm(src, w, tmp, D, eps);
        else memcpy(tmp, src, D * sizeof(float));
        if (rope_pairs) orc_rope(tmp, D, rope_pairs, rope_base, pos0 + t);
        float *dst = cache + ((size_t)h * cap + pos0 + t) * D;
        for (uint32_t d = 0; d < D; ++d) dst[d] = round_bf16 ? bf16_round(tmp[d]) : tmp[d];
    }
}

/* Prefill of T tokens at positions pos0.. of one sequence: appends K/V to the cache
 * [Hkv][cap][D], then attends causally (window 0 = global).  rows lists the query token
 * indices to compute (NULL = all T); out is [n_rows][Hq][D]. */
void orc_prefill(const float *q_raw, const float *k_raw, const float *v_raw,
                 const uint16_t *q_w, const uint16_t *k_w, int qk_norm, int v_norm,
                 uint32_t rope_pairs, float rope_base, float eps, float scale, uint32_t window,
                 float *Kc, float *Vc, uint32_t cap, uint32_t pos0, uint32_t T, uint32_t Hq,
                 uint32_t Hkv, uint32_t D, const int32_t *rows, uint32_t n_rows, float *out,
                 int round_bf16) {
    orc_kv_append(k_raw, k_w, qk_norm, rope_pairs, rope_base, eps, Kc, cap, pos0, T, Hkv, D,
                  round_bf16);
    orc_kv_append(v_raw, NULL, v_norm, 0, rope_base, eps, Vc, cap, pos0, T, Hkv, D, round_bf16);
    if (!rows) n_rows = T;
    const uint32_t group = Hq / Hkv;
#pragma omp parallel for schedule(dynamic, 1)
    for (long long rh = 0; rh < (long long)n_rows * Hq; ++rh) {
        const uint32_t r = (uint32_t)(rh / Hq), h = (uint32_t)(rh % Hq);
        const uint32_t t = rows ? (uint32_t)rows[r] : r;
        const uint32_t pos = pos0 + t, kvh = h / group;
        float qn[1024];
        const float *src = q_raw + ((size_t)t * Hq + h) * D;
        if (qk_norm) orc_rms_norm(src, q_w, qn, D, eps);
        else memcpy(qn, src, D * sizeof(float));
        if (rope_pairs) orc_rope(qn, D, rope_pairs, rope_base, pos);
        if (round_bf16) orc_round_bf16_inplace(qn, D);
        const size_t base = (size_t)kvh * cap * D;
        orc_attention_row(qn, Kc + base, Vc + base, out + ((size_t)r * Hq + h) * D, D,
                          first_visible(pos, window), pos, (double)scale);
    }
}

/* One decode step for B sequences.  Sequence b holds lens[b]-1 cached positions; its new
 * token (q_raw[b], k_new[b], v_new[b]) sits at position lens[b]-1 and is appended to the
 * cache [B][Hkv][cap][D] before attending over [first, lens[b]-1].  out is [B][Hq][D]. */
void orc_decode(const float *q_raw, const float *k_new, const float *v_new,
                const uint16_t *q_w, const uint16_t *k_w, int qk_norm, int v_norm,
                uint32_t rope_pairs, float rope_base, float eps, float scale, uint32_t window,
                float *Kc, float *Vc, uint32_t cap, const int32_t *lens, uint32_t B,
                uint32_t Hq, uint32_t Hkv, uint32_t D, float *out, int round_bf16) {
    const size_t seq_stride = (size_t)Hkv * cap * D;
    for (uint32_t b = 0; b < B; ++b) {
        const uint32_t pos = (uint32_t)lens[b] - 1;
        orc_kv_append(k_new + (size_t)b * Hkv * D, k_w, qk_norm, rope_pairs, rope_base, eps,
                      Kc + b * seq_stride, cap, pos, 1, Hkv, D, round_bf16);
        orc_kv_append(v_new + (size_t)b * Hkv * D, NULL, v_norm, 0, rope_base, eps,
                      Vc + b * seq_stride, cap, pos, 1, Hkv, D, round_bf16);
    }
    const uint32_t group = Hq / Hkv;
#pragma omp parallel for schedule(dynamic, 1)
    for (long long bh = 0; bh < (long long)B * Hq; ++bh) {
        const uint32_t b = (uint32_t)(bh / Hq), h = (uint32_t)(bh % Hq);
        const uint32_t pos = (uint32_t)lens[b] - 1, kvh = h / group;
        float qn[1024];
        const float *src = q_raw + ((size_t)b * Hq + h) * D;
        if (qk_norm) orc_rms_norm(src, q_w, qn, D, eps);
        else memcpy(qn, src, D * sizeof(float));
        if (rope_pairs) orc_rope(qn, D, rope_pairs, rope_base, pos);
        if (round_bf16) orc_round_bf16_inplace(qn, D);
        const size_t base = b * seq_stride + (size_t)kvh * cap * D;
        orc_attention_row(qn, Kc + base, Vc + base, out + ((size_t)b * Hq + h) * D, D,
                          first_visible(pos, window), pos, (double)scale);
    }
}

/* Split-KV partial of one query row over keys [lo, hi) (hi > lo), in the log2 domain the
 * GPU path uses: m2 = max_j s_j * scale * log2(e), l = sum_j 2^(s_j*scale*log2e - m2),
 * o = (sum_j 2^(...) V_j) / l.  Writes o[D], then m2, l (D + 2 floats). */
void orc_partial_row(const float *q, const float *K, const float *V, size_t D, size_t lo,
                     size_t hi, double scale, float *out) {
    const double log2e = 1.4426950408889634073599246810019;
    const size_t n = hi - lo;
    double *s = (double *)malloc(n * sizeof(double));
    double m = -INFINITY;
    for (size_t j = 0; j < n; ++j) {
        double acc = 0.0;
        const float *k = K + (lo + j) * D;
        for (size_t d = 0; d < D; ++d) acc += (double)q[d] * k[d];
        s[j] = acc * scale * log2e;
        if (s[j] > m) m = s[j];
    }
    double l = 0.0;
    for (size_t j = 0; j < n; ++j) {
        s[j] = exp2(s[j] - m);
        l += s[j];
    }
    for (size_t d = 0; d < D; ++d) {
        double acc = 0.0;
        for (size_t j = 0; j < n; ++j) acc += s[j] * V[(lo + j) * D + d];
        out[d] = (float)(acc / l);
    }
    out[D] = (float)m;
    out[D + 1] = (float)l;
    free(s);
}

/* Log-sum-exp merge of R partials (each D + 2 floats as written by orc_partial_row; a
 * partial with l == 0 holds no keys and is skipped) into one output row. */
void orc_merge_partials(const float *parts, uint32_t R, size_t D, float *out) {
    double M = -INFINITY;
    for (uint32_t r = 0; r < R; ++r) {
        const float *p = parts + (size_t)r * (D + 2);
        if (p[D + 1] > 0.0f && p[D] > M) M = p[D];
    }
    double den = 0.0;
    for (uint32_t r = 0; r < R; ++r) {
        const float *p = parts + (size_t)r * (D + 2);
        if (p[D + 1] > 0.0f) den += exp2((double)p[D] - M) * p[D + 1];
    }
    for (size_t d = 0; d < D; ++d) {
        double num = 0.0;
        for (uint32_t r = 0; r < R; ++r) {
            const float *p = parts + (size_t)r * (D + 2);
            if (p[D + 1] > 0.0f) num += exp2((double)p[D] - M) * p[D + 1] * p[d];
        }
        out[d] = (float)(num / den);
    }
}

/* ---------------------------------------------------------------- NVFP4 projections */

/* src/nvfp4.h:11-16 */
float orc_e2m1(uint32_t code) {
    static const float table[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    const float v = table[code & 7u];
    return (code & 8u) ? -v : v;
}

/* src/nvfp4.h:18-28 */
float orc_e4m3(uint8_t byte) {
    const uint32_t e = (byte >> 3) & 0xFu, m = byte & 7u;
    const float v = e == 0 ? (float)m * (1.0f / 512.0f) : ldexpf(1.0f + (float)m * 0.125f, (int)e - 7);
    return (byte & 0x80u) ? -v : v;
}

/* output[t * rows + r] = W[r] . input[t] for W [rows][n] in NVFP4: codes uint32 [rows][n/8]
 * (8 codes per word, low nibble first), scales E4M3 [rows][n/16].  src/tests/cpu_ref.h:48-63. */
void orc_matvec_nvfp4(const uint32_t *codes, const uint8_t *scales, const float *input, float *output,
                      size_t tokens, size_t rows, size_t n) {
#pragma omp parallel
    {
        float *w = (float *)malloc(n * sizeof(float));
#pragma omp for schedule(static)
        for (long long r = 0; r < (long long)rows; ++r) {
            const uint32_t *cr = codes + (size_t)r * (n / 8);
            const uint8_t *sr = scales + (size_t)r * (n / 16);
            for (size_t g = 0; g < n / 16; ++g) {
                const float sc = orc_e4m3(sr[g]);
                for (size_t i = 0; i < 16; ++i) {
                    const uint32_t word = cr[2 * g + i / 8];
                    w[g * 16 + i] = orc_e2m1((word >> (4 * (i % 8))) & 0xFu) * sc;
                }
            }
            for (size_t t = 0; t < tokens; ++t) {
                double acc = 0.0;
                for (size_t i = 0; i < n; ++i) acc += (double)w[i] * input[t * n + i];
                output[t * rows + (size_t)r] = (float)acc;
            }
        }
        free(w);
    }
}

/* shaders/norm.metal:36-81 (one row per threadgroup) with cpu_ref.h:14-25 arithmetic. */
void orc_rms_norm_rows(const float *input, const uint16_t *w, float *output, size_t rows, size_t n, float eps) {
    for (size_t r = 0; r < rows; ++r) orc_rms_norm(input + r * n, w, output + r * n, n, eps);
}

/* Raw 32-bit words of the seeded generator (codes of synthetic NVFP4 matrices). */
void orc_fill_u32(uint32_t *out, size_t n, uint64_t seed, uint64_t stream) {
    const uint64_t key = rng_key(seed, stream);
    for (size_t i = 0; i < n; ++i) out[i] = (uint32_t)(rng_bits(key, i) >> 16);
}
