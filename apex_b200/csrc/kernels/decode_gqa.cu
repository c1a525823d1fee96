// decode_gqa.cu -- fused single-token decode for wide GQA groups and head_dim 512: the reference
// model's global ("full attention") layers, 16 q heads over 2 kv heads of head_dim 512, RoPE on the
// first 64 of 256 pairs, theta 1e6, weightless RMSNorm of V, V taken from the raw k projection
// (docs/B6_3_attention.md:46-60, 17-33).  Semantics as apex_attn_decode_bf16 (same entry point; this
// form serves head_dim 256 or 512 with 1 to 8 q heads per kv head, except 256 / 2 which the split-KV
// kernel of decode_splitkv.cu serves).
//
// B200 design.  Still HBM-bound, but at 8 q heads per kv head every K/V byte feeds 4 multiply-adds,
// about 70 % of the SMs' FP32 FMA rate at full HBM bandwidth -- so the two products run on the
// tensor cores with mma.sync (m16n8k16, bf16 in, f32 accumulate), the heads on the N side:
//   S^T [16 keys x 8 heads] = K [16 x D] . Q^T      (A = K rows, ldmatrix from shared memory;
//                                                     Q split into bf16 hi + lo planes: two MMAs, so
//                                                     the scores keep ~16 mantissa bits of q)
//   O^T [D x 8 heads]     += V^T [D x 16] . P^T     (A = V rows through ldmatrix.trans; P^T from the
//                                                     S^T accumulator by two movmatrix.trans)
// A CTA = 4 consumer warps + 1 producer warp.  The producer copies each 16-key stage of K and of V
// with ONE tiled TMA copy each: a 3-D view of the cache -- 64-element (128-byte) chunks of a row,
// rows, chunks -- with box {64, 16, D/64} lands chunk-major in shared memory ([chunk][key][128 B]),
// and the 128-byte swizzle then XORs a key's 16-byte columns with key & 7, so the 8 rows an ldmatrix
// reads at one column sit in 8 different bank groups.  (Per-row 1 KB bulk copies into padded rows
// were tried first: 32 copies per stage capped the kernel at ~0.6 of HBM.)  Each consumer warp takes
// whole stages and keeps its own online softmax (log2 domain) with O^T in registers (D/16
// accumulator tiles).  Warps merge through
// shared memory, splits through the workspace, the last CTA of a (sequence, kv head) merging them.
// tcgen05 would need M >= 64 rows of one operand in shared memory per MMA and a TMEM round trip per
// 16-key tile for the softmax; at 8 heads per step the tensor work is ~2 % of the tensor peak, so
// the register-resident mma.sync form is the one with the shortest dependency chain here.
#include <algorithm>
#include <string>

#include "common.cuh"
#include "internal.h"
#include "mma_sync.cuh"

namespace apex {
namespace {

constexpr int kHeads = 8;          // MMA N: q heads of one kv head (padded with zero heads)
constexpr int kStagePos = 16;      // keys per stage (MMA M)
constexpr int kWarps = 4;          // consumer warps
constexpr int kThreads = (kWarps + 1) * 32;
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint32_t kMaxSplits = 4096;
constexpr uint32_t kGroup = 8;         // splits merged by the last CTA of each group

struct GqaArgs {
    const uint16_t *q_raw, *k_new, *v_new, *q_w, *k_w;
    uint16_t *k_cache, *v_cache;
    const int32_t *seq_lens;
    uint16_t *out;
    float *ws_part;      // [B][Hq][max_splits][D + 4]
    unsigned *ws_count;  // [B][Hkv] splits (or groups of splits) done
    unsigned *ws_gcount; // [B][Hkv][max_groups] splits of each group done
    unsigned *status;
    uint32_t capacity, q_heads, kv_heads, group, rope_pairs, window, qk_norm, v_norm;
    uint32_t chunk, max_splits, max_groups, max_seq_len;
    float eps, scale_log2;
    RopeTable rope;
};

template <int D>
struct GqaSmem {
    static constexpr int kTile = kStagePos * D * 2;             // one operand's 16 keys, swizzled
    static constexpr int kStageBytes = 2 * kTile;               // K tile then V tile
    static constexpr int kStages = D == 512 ? 4 : 8;            // 128 KB of K/V in flight
    alignas(1024) uint8_t ring[kStages][kStageBytes];
    alignas(1024) uint8_t tail[kStageBytes];      // the new token (key 0) and 15 zero keys
    uint16_t q[2][kHeads][D + 8];                 // bf16 hi / lo planes of the scaled q, padded rows
    float rope_cs[256], rope_sn[256];
    float red_m[kWarps][kHeads], red_l[kWarps][kHeads];
    uint64_t full[kStages], empty[kStages];
    int is_last;
};
// The merges stage up to kHeads x (kGroup + 1) partial records at once in the ring and the tail
// (contiguous), and keep the batch's weights beside them in q's space.
static_assert(offsetof(GqaSmem<512>, tail) == sizeof(GqaSmem<512>::ring) &&
                  offsetof(GqaSmem<256>, tail) == sizeof(GqaSmem<256>::ring),
              "ring and tail are one staging area");
static_assert(sizeof(GqaSmem<512>::ring) + sizeof(GqaSmem<512>::tail) >= kHeads * (kGroup + 1) * (512 + 4) * 4 &&
                  sizeof(GqaSmem<256>::ring) + sizeof(GqaSmem<256>::tail) >= kHeads * (kGroup + 1) * (256 + 4) * 4,
              "a batch of partial records fits the staging area");
static_assert(sizeof(GqaSmem<256>::q) >= kHeads * (kGroup + 1 + 2) * 4, "batch weights fit q's space");

__device__ __forceinline__ void gqa_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kWarps * 32) : "memory"); }

// RMSNorm (optional weight) and rotate-half RoPE of one D-wide row held E = D/32 contiguous elements
// per lane (lane l: [E*l, E*l + E)); the pair (i, i + D/2) meets across lanes l and l ^ 16.
template <int D>
__device__ __forceinline__ void norm_rope_row(float (&x)[D / 32], uint32_t lane, bool norm, const uint16_t *w,
                                              float eps, uint32_t rope_pairs, const float *cs, const float *sn) {
    constexpr int E = D / 32;
    if (norm) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) ss += x[e] * x[e];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = rsqrtf(ss * (1.0f / static_cast<float>(D)) + eps);
#pragma unroll
        for (int e = 0; e < E; ++e)
            x[e] = x[e] * inv * (w ? __uint_as_float(static_cast<uint32_t>(w[E * lane + e]) << 16) : 1.0f);
    }
    if (rope_pairs) {
        const bool low = lane < 16;
#pragma unroll
        for (int e = 0; e < E; ++e) {
            const uint32_t i = E * (lane & 15) + e;
            const float other = __shfl_xor_sync(0xffffffffu, x[e], 16);
            if (i < rope_pairs) x[e] = low ? (x[e] * cs[i] - other * sn[i]) : (other * sn[i] + x[e] * cs[i]);
        }
    }
}

template <int D>
__device__ __forceinline__ void load_row(const uint16_t *src, uint32_t lane, float (&x)[D / 32]) {
    constexpr int E = D / 32;
#pragma unroll
    for (int k = 0; k < E / 8; ++k) {
        const uint4 v = *reinterpret_cast<const uint4 *>(src + E * lane + 8 * k);
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            x[8 * k + 2 * j] = bf16lo(u[j]);
            x[8 * k + 2 * j + 1] = bf16hi(u[j]);
        }
    }
}

// Shared-memory byte offset of key `key`, 16-byte column `col` (of D/8) in a swizzled 16-key tile:
// chunk-major [col / 8][key][128 B] with the 16-byte column inside the chunk XORed with key & 7.
__device__ __forceinline__ uint32_t tile_off(uint32_t key, uint32_t col) {
    return (col >> 3) * (kStagePos * 128) + key * 128 + (((col & 7) ^ (key & 7)) << 4);
}

// One 16-key tile of this warp: scores, online softmax, O^T += V^T P^T.  kbase / vbase: shared
// addresses of the tile's swizzled K / V keys; nvalid keys valid (the V keys past it are zero).
template <int D>
__device__ __forceinline__ void gqa_tile(uint32_t kbase, uint32_t vbase, int nvalid, uint32_t lane, uint32_t qhi,
                                         uint32_t qlo, float (&m)[2], float (&l)[2], float (&o)[D / 16][4]) {
    const uint32_t g = lane >> 2;
    const uint32_t mi = lane >> 3, r = lane & 7;
    // A = K keys: matrix mi covers keys r + 8*(mi & 1), the 16-byte column 2*kk + (mi >> 1) of step kk
    const uint32_t a_key = r + 8 * (mi & 1), a_col = mi >> 1;
    // B = q rows (heads): matrix (lane >> 3) & 1 covers dims 8*((lane >> 3) & 1)
    const uint32_t b_off = (lane & 7) * ((D + 8) * 2) + 16 * ((lane >> 3) & 1);
    // four independent accumulator pairs (hi, lo) over the 16-dim steps: eight short MMA chains
    constexpr int kChains = 4;
    float s[kChains][2][4];
#pragma unroll
    for (int ch = 0; ch < kChains; ++ch)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[ch][0][j] = s[ch][1][j] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; kk += kChains) {
#pragma unroll
        for (int ch = 0; ch < kChains; ++ch) {
            uint32_t a[4], bh0, bh1, bl0, bl1;
            ldsm_x4(kbase + tile_off(a_key, 2 * (kk + ch) + a_col), a);
            ldsm_x2(qhi + b_off + (kk + ch) * 32, bh0, bh1);
            ldsm_x2(qlo + b_off + (kk + ch) * 32, bl0, bl1);
            mma_bf16(s[ch][0], a, bh0, bh1);
            mma_bf16(s[ch][1], a, bl0, bl1);
        }
    }
    // scores: key g (j < 2) or g + 8 (j >= 2), head 2c + (j & 1)
    float p[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int key = static_cast<int>(g) + (j >= 2 ? 8 : 0);
        float v = 0.f;
#pragma unroll
        for (int ch = 0; ch < kChains; ++ch) v += s[ch][0][j] + s[ch][1][j];
        p[j] = key < nvalid ? v : -INFINITY;
    }
    float mx[2] = {fmaxf(p[0], p[2]), fmaxf(p[1], p[3])};
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], off));
    float alpha[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const float mn = fmaxf(m[h], mx[h]);
        alpha[h] = fast_exp2(m[h] - mn);  // 0 when m was -inf
        m[h] = mn;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) p[j] = fast_exp2(p[j] - m[j & 1]);  // 0 for masked keys
    l[0] = l[0] * alpha[0] + p[0] + p[2];
    l[1] = l[1] * alpha[1] + p[1] + p[3];
    if (__any_sync(0xffffffffu, alpha[0] != 1.f || alpha[1] != 1.f)) {
#pragma unroll
        for (int t = 0; t < D / 16; ++t) {
            o[t][0] *= alpha[0];
            o[t][1] *= alpha[1];
            o[t][2] *= alpha[0];
            o[t][3] *= alpha[1];
        }
    }
    // P^T as the B operand: keys 0-7 and 8-15 transposed into (key = 2c.., head = g)
    const uint32_t b0 = movmatrix_t(pack_bf16(p[0], p[1]));
    const uint32_t b1 = movmatrix_t(pack_bf16(p[2], p[3]));
    // A = V^T: matrix mi covers keys r + 8*(mi >> 1), the 16-byte column 2*t + (mi & 1) of dim tile t
    const uint32_t v_key = r + 8 * (mi >> 1), v_col = mi & 1;
#pragma unroll
    for (int t = 0; t < D / 16; ++t) {
        uint32_t a[4];
        ldsm_x4_t(vbase + tile_off(v_key, 2 * t + v_col), a);
        mma_bf16(o[t], a, b0, b1);
    }
}

// Merges n partial records of every head -- head h's record i at part + ((rows_b + h) * max_splits +
// first + i * stride) * (D + 4): o normalised by its l, then m (log2 units) and l -- staged kGroup + 1
// at a time in the ring and tail by cp.async (one round trip per batch), with the running max and
// weight sum of each head rescaled from batch to batch.  final_out: o / sum to bf16 out; otherwise
// the merged record (o normalised, m, l = the weight sum) replaces record `first`.  Thread t owns
// float4 column t % (D/4) of heads t / (D/4), + 128 / (D/4), ...
template <int D>
__device__ void merge_records(GqaSmem<D> &sm, const GqaArgs &a, float *part, uint64_t rows_b, uint32_t G,
                              uint32_t first, uint32_t stride, uint32_t n, bool final_out, uint32_t tid) {
    constexpr uint32_t kRec = D + 4;
    constexpr uint32_t kCols = D / 4;
    constexpr uint32_t kHStep = kWarps * 32 / kCols;
    constexpr uint32_t kHpt = kHeads / kHStep;
    constexpr uint32_t kBatch = kGroup + 1;
    const uint32_t warp = tid >> 5, lane = tid & 31;
    const uint32_t col = tid % kCols, h0 = tid / kCols;
    float *stage = reinterpret_cast<float *>(sm.ring[0]);    // [head][kBatch][kRec]
    float *wts = reinterpret_cast<float *>(&sm.q[0][0][0]);  // [head][kBatch]
    float *scl = wts + kHeads * kBatch;                      // [head] rescale of the running sums
    float *den = scl + kHeads;                               // [head] running weight sum
    float *mrun = den + kHeads;                              // [head] running max
    float acc[kHpt][4];
#pragma unroll
    for (uint32_t k = 0; k < kHpt; ++k) acc[k][0] = acc[k][1] = acc[k][2] = acc[k][3] = 0.f;
    if (tid < kHeads) {
        den[tid] = 0.f;
        mrun[tid] = -INFINITY;
    }
    for (uint32_t i0 = 0; i0 < n; i0 += kBatch) {
        const uint32_t cnt = min(kBatch, n - i0);
        const uint32_t per_h = cnt * (kRec / 4);  // 16-byte pieces of one head's records
        for (uint32_t q = tid; q < G * per_h; q += kWarps * 32) {
            const uint32_t h = q / per_h, rem = q % per_h, i = rem / (kRec / 4), w16 = rem % (kRec / 4);
            const float *src = part + ((rows_b + h) * a.max_splits + first + (i0 + i) * stride) * kRec + 4 * w16;
            cp_async16(smem_u32(stage + (h * kBatch + i) * kRec + 4 * w16), src);
        }
        cp_async_commit();
        cp_async_wait<0>();
        gqa_sync();
        for (uint32_t h = warp; h < G; h += kWarps) {  // weights of the batch; lane i: record i
            const bool has = lane < cnt;
            const float *rec = stage + (h * kBatch + (has ? lane : 0)) * kRec;
            const float mi = has ? rec[D] : -INFINITY, li = has ? rec[D + 1] : 0.f;
            float M = li > 0.f ? mi : -INFINITY;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
            const float m_old = mrun[h];
            const float Mn = fmaxf(m_old, M);
            const float wt = li > 0.f ? fast_exp2(mi - Mn) * li : 0.f;
            float sum = wt;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            if (has) wts[h * kBatch + lane] = wt;
            __syncwarp();
            if (lane == 0) {
                const float sc = m_old == -INFINITY ? 0.f : fast_exp2(m_old - Mn);
                scl[h] = sc;
                den[h] = den[h] * sc + sum;
                mrun[h] = Mn;
            }
        }
        gqa_sync();
#pragma unroll
        for (uint32_t k = 0; k < kHpt; ++k) {
            const uint32_t h = h0 + k * kHStep;
            if (h >= G) continue;
            const float sc = scl[h];
            float r[4] = {acc[k][0] * sc, acc[k][1] * sc, acc[k][2] * sc, acc[k][3] * sc};
            const float *srec = stage + h * kBatch * kRec + 4 * col;
            for (uint32_t i = 0; i < cnt; ++i) {
                const float wt = wts[h * kBatch + i];
                const float4 v = *reinterpret_cast<const float4 *>(srec + i * kRec);
                r[0] += wt * v.x;
                r[1] += wt * v.y;
                r[2] += wt * v.z;
                r[3] += wt * v.w;
            }
            acc[k][0] = r[0];
            acc[k][1] = r[1];
            acc[k][2] = r[2];
            acc[k][3] = r[3];
        }
        gqa_sync();  // the staging area is free for the next batch
    }
#pragma unroll
    for (uint32_t k = 0; k < kHpt; ++k) {
        const uint32_t h = h0 + k * kHStep;
        if (h >= G) continue;
        const float dn = den[h];
        const float inv = dn > 0.f ? 1.0f / dn : 0.f;
        if (final_out) {
            uint2 pk;
            pk.x = pack_bf16(acc[k][0] * inv, acc[k][1] * inv);
            pk.y = pack_bf16(acc[k][2] * inv, acc[k][3] * inv);
            *reinterpret_cast<uint2 *>(a.out + (rows_b + h) * D + 4 * col) = pk;
        } else {
            float *dst = part + ((rows_b + h) * a.max_splits + first) * kRec;
            *reinterpret_cast<float4 *>(dst + 4 * col) =
                make_float4(acc[k][0] * inv, acc[k][1] * inv, acc[k][2] * inv, acc[k][3] * inv);
            if (col == 0) {
                dst[D] = mrun[h];
                dst[D + 1] = dn;
            }
        }
    }
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1) decode_gqa_kernel(const __grid_constant__ GqaArgs a,
                                                                 const __grid_constant__ CUtensorMap tk,
                                                                 const __grid_constant__ CUtensorMap tv) {
    using Smem = GqaSmem<D>;
    constexpr int E = D / 32;
    constexpr int kTile = Smem::kTile;
    constexpr int ST = Smem::kStages;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    // the 128-byte swizzle repeats every 1024 bytes: stage tiles start on 1024-byte boundaries
    Smem &sm = *reinterpret_cast<Smem *>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023));
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const uint32_t G = a.group;

    const int32_t L = a.seq_lens[b];
    const bool bad = L < 0 || static_cast<uint32_t>(L) > a.max_seq_len;
    const uint32_t Lu = bad ? 0u : static_cast<uint32_t>(L);
    const uint32_t pos_new = Lu - 1;
    const uint32_t first = (a.window && Lu > a.window) ? Lu - a.window : 0;
    const uint32_t n_keys = Lu > first ? Lu - first : 0;
    const uint32_t nsplit = n_keys ? (n_keys + a.chunk - 1) / a.chunk : 1;
    if (bad && split == 0 && tid == 0 && kvh == 0) atomicOr(a.status, kStatusBadLength);
    if (split >= nsplit) return;
    if (nsplit > a.max_splits) {
        if (tid == 0) atomicOr(a.status, kStatusBadLength);
        return;
    }
    const uint32_t lo = first + split * a.chunk;
    const uint32_t hi = n_keys ? min(lo + a.chunk, Lu) : lo;
    const bool has_new = n_keys && pos_new >= lo && pos_new < hi;
    const uint32_t n_cached = (has_new ? pos_new : hi) > lo ? (has_new ? pos_new : hi) - lo : 0;
    const uint32_t n_stages = (n_cached + kStagePos - 1) / kStagePos;
    const uint64_t head_base = (static_cast<uint64_t>(b) * a.kv_heads + kvh) * a.capacity * D;

    if (tid == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(smem_u32(&sm.full[s]), 1);
            mbar_init(smem_u32(&sm.empty[s]), 1);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kWarps) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            prefetch_tensormap(&tk);
            prefetch_tensormap(&tv);
            // row index of this split's first key in the [B * Hkv * capacity] rows of the cache
            const int32_t row0 = static_cast<int32_t>((static_cast<uint64_t>(b) * a.kv_heads + kvh) * a.capacity + lo);
            for (uint32_t s = 0; s < n_stages; ++s) {
                const uint32_t slot = s % ST;
                if (s >= ST && !mbar_wait(smem_u32(&sm.empty[slot]), ((s / ST) - 1) & 1, a.status)) break;
                const uint32_t full = smem_u32(&sm.full[slot]);
                // 16 whole keys every stage (keys past the split are masked; past the cache, zero)
                mbar_arrive_expect_tx(full, 2 * kTile);
                const uint32_t dst = smem_u32(sm.ring[slot]);
                tma_load_3d(dst, &tk, 0, row0 + static_cast<int32_t>(s * kStagePos), 0, full);
                tma_load_3d(dst + kTile, &tv, 0, row0 + static_cast<int32_t>(s * kStagePos), 0, full);
            }
        }
        return;
    }

    // -------------------------------------------------------------------- consumers
    // zero the q planes (heads >= G stay zero) and the tail tile; RoPE table of the new position
    for (uint32_t i = tid; i < sizeof(sm.q) / 16; i += kWarps * 32) reinterpret_cast<uint4 *>(sm.q)[i] = make_uint4(0, 0, 0, 0);
    for (uint32_t i = tid; i < sizeof(sm.tail) / 16; i += kWarps * 32)
        reinterpret_cast<uint4 *>(sm.tail)[i] = make_uint4(0, 0, 0, 0);
    const float pos_f = static_cast<float>(pos_new);
    for (uint32_t i = tid; i < a.rope_pairs; i += kWarps * 32)
        rope_sincos(pos_f * a.rope.inv_freq[i], sm.rope_sn[i], sm.rope_cs[i]);
    gqa_sync();
    // q rows: warp w takes heads w, w + 4 of this kv head's group (norm + RoPE, scaled for exp2,
    // split into bf16 hi + lo)
    for (uint32_t hh = warp; hh < G; hh += kWarps) {
        float x[E];
        load_row<D>(a.q_raw + (static_cast<uint64_t>(b) * a.q_heads + kvh * G + hh) * D, lane, x);
        norm_rope_row<D>(x, lane, a.qk_norm, a.q_w, a.eps, a.rope_pairs, sm.rope_cs, sm.rope_sn);
#pragma unroll
        for (int e = 0; e < E; ++e) {
            const float v = x[e] * a.scale_log2;
            const float vh = bf16_round(v);
            sm.q[0][hh][E * lane + e] = static_cast<uint16_t>(pack_bf16(vh, 0.f) & 0xFFFFu);
            sm.q[1][hh][E * lane + e] = static_cast<uint16_t>(pack_bf16(v - vh, 0.f) & 0xFFFFu);
        }
    }
    if (has_new && warp >= 2) {
        // new k (warp 2: norm + RoPE) and new v (warp 3: optional weightless norm): rounded to bf16
        // once, written to the cache at pos_new and to row 0 of the tail tile
        const bool is_k = warp == 2;
        float x[E];
        load_row<D>((is_k ? a.k_new : a.v_new) + (static_cast<uint64_t>(b) * a.kv_heads + kvh) * D, lane, x);
        if (is_k)
            norm_rope_row<D>(x, lane, a.qk_norm, a.k_w, a.eps, a.rope_pairs, sm.rope_cs, sm.rope_sn);
        else
            norm_rope_row<D>(x, lane, a.v_norm, nullptr, a.eps, 0, sm.rope_cs, sm.rope_sn);
        uint16_t *dst = (is_k ? a.k_cache : a.v_cache) + head_base + static_cast<uint64_t>(pos_new) * D;
        uint8_t *ttile = sm.tail + (is_k ? 0 : kTile);
#pragma unroll
        for (int k = 0; k < E / 8; ++k) {
            uint4 pk;
            pk.x = pack_bf16(x[8 * k], x[8 * k + 1]);
            pk.y = pack_bf16(x[8 * k + 2], x[8 * k + 3]);
            pk.z = pack_bf16(x[8 * k + 4], x[8 * k + 5]);
            pk.w = pack_bf16(x[8 * k + 6], x[8 * k + 7]);
            *reinterpret_cast<uint4 *>(dst + E * lane + 8 * k) = pk;
            *reinterpret_cast<uint4 *>(ttile + tile_off(0, (E * lane + 8 * k) / 8)) = pk;  // key 0
        }
    }
    gqa_sync();

    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    float o[D / 16][4];
#pragma unroll
    for (int t = 0; t < D / 16; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;
    const uint32_t qhi = smem_u32(&sm.q[0][0][0]), qlo = smem_u32(&sm.q[1][0][0]);
    for (uint32_t s = warp; s < n_stages; s += kWarps) {
        const uint32_t slot = s % ST;
        if (!mbar_wait(smem_u32(&sm.full[slot]), (s / ST) & 1, a.status)) break;
        const int n = static_cast<int>(min(static_cast<uint32_t>(kStagePos), n_cached - s * kStagePos));
        uint8_t *st = sm.ring[slot];
        if (n < kStagePos) {  // keys past the split's (other positions, or unwritten memory): zero V's
            for (uint32_t i = lane; i < static_cast<uint32_t>(kStagePos - n) * (D / 8); i += 32) {
                const uint32_t key = n + i / (D / 8), col = i % (D / 8);
                *reinterpret_cast<uint4 *>(st + kTile + tile_off(key, col)) = make_uint4(0, 0, 0, 0);
            }
            __syncwarp();
        }
        gqa_tile<D>(smem_u32(st), smem_u32(st + kTile), n, lane, qhi, qlo, m, l, o);
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&sm.empty[slot]));
    }
    if (has_new && warp == 0)
        gqa_tile<D>(smem_u32(sm.tail), smem_u32(sm.tail + kTile), 1, lane, qhi, qlo, m, l, o);

    // ---- per-warp totals: l summed over the lanes that share heads (2c, 2c+1)
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) l[h] += __shfl_xor_sync(0xffffffffu, l[h], off);
    gqa_sync();  // every warp is done with the ring: reuse it for the warp merge
    float *wacc = reinterpret_cast<float *>(sm.ring[0]);  // [warp][head 8][D]
    const uint32_t g8 = lane >> 2, c = lane & 3;
    if (lane < 4) {
        sm.red_m[warp][2 * c] = m[0];
        sm.red_m[warp][2 * c + 1] = m[1];
        sm.red_l[warp][2 * c] = l[0];
        sm.red_l[warp][2 * c + 1] = l[1];
    }
#pragma unroll
    for (int t = 0; t < D / 16; ++t) {  // o[t][j]: dim 16t + g8 (+8 for j >= 2), head 2c + (j & 1)
        float *w0 = wacc + (static_cast<uint64_t>(warp) * kHeads) * D;
        w0[(2 * c) * D + 16 * t + g8] = o[t][0];
        w0[(2 * c + 1) * D + 16 * t + g8] = o[t][1];
        w0[(2 * c) * D + 16 * t + g8 + 8] = o[t][2];
        w0[(2 * c + 1) * D + 16 * t + g8 + 8] = o[t][3];
    }
    gqa_sync();

    // ---- CTA merge: thread t takes (head, 4 dims) chunks h * D/4 + q for t, t + 128, ...
    const uint64_t rows_b = static_cast<uint64_t>(b) * a.q_heads + kvh * G;
    float *part = a.ws_part;  // [B][Hq][max_splits][D + 4]
    for (uint32_t ch = tid; ch < G * (D / 4); ch += kWarps * 32) {
        const uint32_t h = ch / (D / 4), d0 = (ch % (D / 4)) * 4;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarps; ++w)
            if (sm.red_l[w][h] > 0.f) M = fmaxf(M, sm.red_m[w][h]);
        float den = 0.f, acc4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            if (!(sm.red_l[w][h] > 0.f)) continue;
            const float wt = fast_exp2(sm.red_m[w][h] - M);
            den += wt * sm.red_l[w][h];
            const float4 v = *reinterpret_cast<const float4 *>(wacc + (static_cast<uint64_t>(w) * kHeads + h) * D + d0);
            acc4[0] += wt * v.x;
            acc4[1] += wt * v.y;
            acc4[2] += wt * v.z;
            acc4[3] += wt * v.w;
        }
        const float inv = den > 0.f ? 1.0f / den : 0.f;
        if (nsplit == 1) {
            uint2 pk;
            pk.x = pack_bf16(acc4[0] * inv, acc4[1] * inv);
            pk.y = pack_bf16(acc4[2] * inv, acc4[3] * inv);
            *reinterpret_cast<uint2 *>(a.out + (rows_b + h) * D + d0) = pk;
        } else {
            float *dst = part + ((rows_b + h) * a.max_splits + split) * (D + 4);
            *reinterpret_cast<float4 *>(dst + d0) = make_float4(acc4[0] * inv, acc4[1] * inv, acc4[2] * inv, acc4[3] * inv);
            if (d0 == 0) {
                dst[D] = M;
                dst[D + 1] = den;
            }
        }
    }
    if (nsplit == 1) return;
    // ---- splits in groups of kGroup: the last CTA of a group merges the group into the group's first
    // record, and the last group's merger merges the groups into out (one level for <= kGroup splits).
    // Each merger stages its records by cp.async in one or a few round trips, so no single CTA reads
    // hundreds of partials one load at a time.
    const uint32_t ngroups = (nsplit + kGroup - 1) / kGroup;
    if (ngroups > 1) {
        const uint32_t grp = split / kGroup, gsize = min(kGroup, nsplit - grp * kGroup);
        gqa_sync();
        if (tid == 0) {
            __threadfence();
            unsigned *gc = a.ws_gcount + (static_cast<uint64_t>(b) * a.kv_heads + kvh) * a.max_groups + grp;
            const unsigned prev = atomicAdd(gc, 1u);
            const int last = prev == gsize - 1;
            if (last) *gc = 0;
            sm.is_last = last;
        }
        gqa_sync();
        if (!sm.is_last) return;
        __threadfence();
        if (gsize > 1) merge_records<D>(sm, a, part, rows_b, G, grp * kGroup, 1, gsize, false, tid);
    }
    gqa_sync();
    if (tid == 0) {
        __threadfence();
        unsigned *counter = a.ws_count + static_cast<uint64_t>(b) * a.kv_heads + kvh;
        const unsigned prev = atomicAdd(counter, 1u);
        const int last = prev == (ngroups > 1 ? ngroups : nsplit) - 1;
        if (last) *counter = 0;
        sm.is_last = last;
    }
    gqa_sync();
    if (!sm.is_last) return;
    __threadfence();
    if (ngroups > 1)
        merge_records<D>(sm, a, part, rows_b, G, 0, kGroup, ngroups, true, tid);
    else
        merge_records<D>(sm, a, part, rows_b, G, 0, 1, nsplit, true, tid);
}

uint32_t gqa_max_splits(uint32_t batch, uint32_t kv_heads, uint32_t max_len) {
    const uint64_t by_len = (static_cast<uint64_t>(max_len) + 63) / 64;
    const uint64_t by_grid = static_cast<uint64_t>(sm_count()) * 4 / std::max<uint64_t>(1, uint64_t(batch) * kv_heads) + 2;
    return static_cast<uint32_t>(std::max<uint64_t>(1, std::min({by_len, by_grid, uint64_t(kMaxSplits)})));
}

// Keys per split: whole waves of CTAs (one per SM) with every (sequence, kv head) cut into the same
// number of splits, so no wave runs a handful of CTAs (8 x 2 pairs of 32768 keys: 9 splits each, 144
// CTAs, instead of 10 splits and a second wave of 12); at least 64 keys (4 stages) per split.
uint32_t gqa_chunk(uint32_t batch, uint32_t kv_heads, uint32_t len) {
    const uint64_t pairs = std::max<uint64_t>(1, static_cast<uint64_t>(batch) * kv_heads);
    const uint64_t sms = static_cast<uint64_t>(sm_count());
    const uint64_t waves = (pairs + sms - 1) / sms;
    const uint64_t per = std::max<uint64_t>(1, waves * sms / pairs);
    uint64_t c = (std::max<uint32_t>(len, 1) + per - 1) / per;
    c = std::max<uint64_t>(c, 64);
    c = (c + kStagePos - 1) / kStagePos * kStagePos;
    return static_cast<uint32_t>(std::min<uint64_t>(c, 1u << 24));
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

}  // namespace

bool gqa_decode_form(const apex_attn_params *p) {
    if (!p || p->kv_heads == 0 || p->q_heads % p->kv_heads) return false;
    const uint32_t g = p->q_heads / p->kv_heads;
    if (p->head_dim == 256 && g == 2) return false;  // the split-KV kernel's shape
    return (p->head_dim == 256 || p->head_dim == 512) && g >= 1 && g <= kHeads;
}

// Workspace: partial records [B][Hq][max_splits][D + 4] f32, then the counters: [B][Hkv] splits or
// groups done, then [B][Hkv][max_groups] splits of each group done.
size_t gqa_workspace_bytes(const apex_attn_params *p, uint32_t batch, uint32_t max_len) {
    const uint32_t max_splits = gqa_max_splits(batch, p->kv_heads, max_len);
    const size_t parts = static_cast<size_t>(batch) * p->q_heads * max_splits * (p->head_dim + 4) * sizeof(float);
    const size_t max_groups = (max_splits + kGroup - 1) / kGroup;
    return align256(parts) + align256(static_cast<size_t>(batch) * p->kv_heads * sizeof(unsigned)) +
           align256(static_cast<size_t>(batch) * p->kv_heads * max_groups * sizeof(unsigned));
}

int launch_gqa_decode(const apex_attn_params *p, const uint16_t *q_raw, const uint16_t *k_new, const uint16_t *v_new,
                      const uint16_t *q_w, const uint16_t *k_w, uint16_t *k_cache, uint16_t *v_cache,
                      uint32_t capacity, const int32_t *seq_lens, uint32_t batch, uint32_t max_seq_len,
                      uint16_t *out, void *workspace, size_t workspace_bytes_given, void *stream, const char *name) {
    if (p->ring) return fail(APEX_ERR_UNSUPPORTED, std::string(name) + ": ring caches are served for head_dim 256, group 2");
    if (batch == 0) return ok();
    if (batch > 65535 || p->kv_heads > 65535) return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": batch or kv_heads too large");
    if (p->rope_pairs > p->head_dim / 2)
        return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": rope_pairs > head_dim / 2");
    if (!q_raw || !k_new || !v_new || !k_cache || !v_cache || !seq_lens || !out)
        return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": null tensor");
    for (const void *ptr : {(const void *)q_raw, (const void *)k_new, (const void *)v_new, (const void *)k_cache,
                            (const void *)v_cache})
        if (!aligned16(ptr)) return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": tensors must be 16-byte aligned");
    if (max_seq_len == 0 || max_seq_len > capacity)
        return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": need 1 <= max_seq_len <= capacity");
    const size_t need = gqa_workspace_bytes(p, batch, max_seq_len);
    if (!workspace || workspace_bytes_given < need || !aligned16(workspace))
        return fail(APEX_ERR_WORKSPACE, std::string(name) + ": workspace of " + std::to_string(need) + " bytes required");
    GqaArgs a{};
    a.q_raw = q_raw; a.k_new = k_new; a.v_new = v_new; a.q_w = q_w; a.k_w = k_w;
    a.k_cache = k_cache; a.v_cache = v_cache; a.seq_lens = seq_lens; a.out = out;
    const uint32_t max_splits = gqa_max_splits(batch, p->kv_heads, max_seq_len);
    a.ws_part = static_cast<float *>(workspace);
    a.ws_count = reinterpret_cast<unsigned *>(static_cast<uint8_t *>(workspace) +
                                              align256(static_cast<size_t>(batch) * p->q_heads * max_splits *
                                                       (p->head_dim + 4) * sizeof(float)));
    a.ws_gcount = reinterpret_cast<unsigned *>(reinterpret_cast<uint8_t *>(a.ws_count) +
                                               align256(static_cast<size_t>(batch) * p->kv_heads * sizeof(unsigned)));
    a.max_groups = (max_splits + kGroup - 1) / kGroup;
    a.status = device_status_ptr();
    if (!a.status) return fail(APEX_ERR_CUDA, std::string(name) + ": device status word unavailable");
    a.capacity = capacity; a.q_heads = p->q_heads; a.kv_heads = p->kv_heads; a.group = p->q_heads / p->kv_heads;
    a.rope_pairs = p->rope_pairs; a.window = p->window; a.qk_norm = p->qk_norm; a.v_norm = p->v_norm;
    a.max_splits = max_splits; a.max_seq_len = max_seq_len;
    a.eps = p->eps; a.scale_log2 = p->scale * kLog2e;
    const uint32_t range = std::min(max_seq_len, p->window ? p->window : max_seq_len);
    a.chunk = gqa_chunk(batch, p->kv_heads, range);
    uint32_t grid_x = (range + a.chunk - 1) / a.chunk;
    while (grid_x > max_splits) {  // keep within the workspace's split count
        a.chunk *= 2;
        grid_x = (range + a.chunk - 1) / a.chunk;
    }
    rope_table(a.rope.inv_freq, p->rope_pairs, p->head_dim, p->rope_base);
    // the caches as {64 elements, rows, D/64 chunks} with byte strides {D*2, 128}: one box = 16 keys
    // of one operand, chunk-major in shared memory
    const uint64_t rows = static_cast<uint64_t>(batch) * p->kv_heads * capacity;
    if (rows > 0x7fffffffull) return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": cache too large");
    const uint64_t dims[3] = {64, rows, p->head_dim / 64u};
    const uint64_t strides[2] = {p->head_dim * 2ull, 128};
    const uint32_t box[3] = {64, static_cast<uint32_t>(kStagePos), p->head_dim / 64u};
    CUtensorMap tk, tv;
    int rc = make_tensor_map_bf16_3d_box(&tk, k_cache, dims, strides, box);
    if (rc) return rc;
    rc = make_tensor_map_bf16_3d_box(&tv, v_cache, dims, strides, box);
    if (rc) return rc;
    const dim3 grid(grid_x, p->kv_heads, batch);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (p->head_dim == 512) {
        rc = check_cuda(cudaFuncSetAttribute(decode_gqa_kernel<512>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(sizeof(GqaSmem<512>) + 1024)),
                        name);
        if (rc) return rc;
        decode_gqa_kernel<512><<<grid, kThreads, sizeof(GqaSmem<512>) + 1024, s>>>(a, tk, tv);
    } else {
        rc = check_cuda(cudaFuncSetAttribute(decode_gqa_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(sizeof(GqaSmem<256>) + 1024)),
                        name);
        if (rc) return rc;
        decode_gqa_kernel<256><<<grid, kThreads, sizeof(GqaSmem<256>) + 1024, s>>>(a, tk, tv);
    }
    rc = check_cuda(cudaGetLastError(), name);
    return rc ? rc : ok();
}

}  // namespace apex
