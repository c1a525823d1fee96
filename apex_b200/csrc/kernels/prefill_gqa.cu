// prefill_gqa.cu -- bf16 prefill for head_dim 512: the reference model's global ("full attention")
// layers, 16 q heads over 2 kv heads of head_dim 512, RoPE on the first 64 of 256 pairs, weightless
// RMSNorm of V, V taken from the raw k projection (docs/B6_3_attention.md:46-60, 17-33).  Semantics
// as apex_attn_prefill_bf16 (same entry points; this form serves head_dim 512).
//
// Preparation: q (norm + partial RoPE) into the head-major workspace [B][Hq][T][512], k (norm +
// partial RoPE) and v (weightless norm, or a plain copy) into the caches at pos0, by the bf16
// head_norm_rope kernel with the caches' strides.
//
// Attention.  GQA groups of 1, 2, 4 and 8 (the global layers' 8 among them) run on the tensor cores
// (prefill_wide.cu: a CTA pair splitting the head dimension).  Other groups take the form here, on
// mma.sync m16n8k16 (bf16 in, f32 accumulate) with the head dimension split over warps: a CTA takes
// 16 queries of two q heads
// of one GQA group; warp (head, slice) keeps its 16 x 128 slice of Q in registers, computes the
// partial scores of its slice against each 32-key tile, the four slice warps of a head add their
// partials through shared memory in a fixed order (so all four hold the same scores, bit for bit, and
// the same softmax), and each accumulates its 128-dim slice of O in registers with P kept in
// registers as the A operand (the score accumulator layout is the next A fragment's).  One producer
// warp streams each tile's K and V with one tiled TMA copy each: the cache viewed as {64-element
// chunks, keys (cut at pos0 + T, so keys past the prefill read as zeros), chunks, kv rows} lands
// chunk-major with the 128-byte swizzle, whose XOR of a key's 16-byte columns with key & 7 keeps
// ldmatrix conflict-free.  Scores in the log2 domain, online softmax per row, causal and window
// masks by position.
#include <cuda_runtime.h>

#include <algorithm>
#include <string>

#include "common.cuh"
#include "internal.h"
#include "mma_sync.cuh"

namespace apex {
namespace {

constexpr int kD = 512;
constexpr int kQ = 16;                             // queries per CTA (MMA M)
constexpr int kHeadsPerCta = 2;                    // q heads of one GQA group per CTA
constexpr int kSlices = 4;                         // warps per head
constexpr int kSliceDims = kD / kSlices;           // 128
constexpr int kConsumers = kHeadsPerCta * kSlices; // 8
constexpr int kThreads = (kConsumers + 1) * 32;    // + producer warp
constexpr int kKeys = 32;                          // keys per tile
constexpr int kStages = 3;
constexpr uint32_t kTileBytes = kKeys * kD * 2;    // 32 KB: K or V of one tile
constexpr uint32_t kStageBytes = 2 * kTileBytes;
constexpr uint32_t kRedFloats = kHeadsPerCta * kSlices * 16 * 32;  // one tile's partial scores
constexpr uint32_t kOffRed = kStages * kStageBytes;
constexpr uint32_t kOffBar = kOffRed + 2 * kRedFloats * 4;
constexpr uint32_t kSmemBytes = kOffBar + 8 * 2 * kStages + 1024;  // + alignment slack of the dynamic base
static_assert(kSmemBytes <= 232448, "shared memory budget");
constexpr float kLog2e = 1.4426950408889634f;

struct GqaPrefillArgs {
    const uint16_t *q_ws;  // [B][Hq][T][512] normalised, roped q
    uint16_t *out;         // [B][T][Hq][512]
    unsigned *status;
    uint32_t T, pos0, q_heads, kv_heads, group, window, head_pairs, n_qtiles;
    float scale_log2;
};

// Byte offset of key `key`, 16-byte column `col` (of 64) in a tile: chunk-major [col / 8][key][128 B],
// the column inside its chunk XORed with key & 7 (the 128-byte swizzle of the TMA copy).
__device__ __forceinline__ uint32_t tile_off(uint32_t key, uint32_t col) {
    return (col >> 3) * (kKeys * 128) + key * 128 + (((col & 7) ^ (key & 7)) << 4);
}

__device__ __forceinline__ void head_sync(uint32_t head_slot) {  // the four slice warps of one head
    asm volatile("bar.sync %0, %1;" ::"r"(1 + head_slot), "n"(kSlices * 32) : "memory");
}

__global__ void __launch_bounds__(kThreads, 1) prefill_gqa_kernel(const __grid_constant__ GqaPrefillArgs a,
                                                                  const __grid_constant__ CUtensorMap tk,
                                                                  const __grid_constant__ CUtensorMap tv) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t *base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const uint32_t sb = smem_u32(base);
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // blocks in launch order take the query tiles from the last (most keys) to the first, every
    // (kv head, head pair) of a tile in turn, so that the short causal tiles fill the tail
    const uint32_t rows_y = a.kv_heads * a.head_pairs;
    const uint32_t yy = blockIdx.x % rows_y;
    const uint32_t b = blockIdx.z, kvh = yy / a.head_pairs, hp = yy % a.head_pairs;
    const uint32_t t0 = (a.n_qtiles - 1 - blockIdx.x / rows_y) * kQ;
    const uint32_t pos_first = a.pos0 + t0, pos_last = a.pos0 + min(a.T, t0 + kQ) - 1;
    const uint32_t kv_lo = (a.window && pos_first + 1 > a.window) ? pos_first + 1 - a.window : 0;
    const uint32_t j0 = kv_lo / kKeys * kKeys;
    const uint32_t n_tiles = (pos_last - j0) / kKeys + 1;
    auto full = [&](uint32_t s) { return sb + kOffBar + 8 * s; };
    auto empty = [&](uint32_t s) { return sb + kOffBar + 8 * (kStages + s); };

    if (tid == 0) {
        prefetch_tensormap(&tk);
        prefetch_tensormap(&tv);
        for (uint32_t s = 0; s < kStages; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), kConsumers);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kConsumers) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            uint32_t issued = 0;
            for (uint32_t j = 0; j < n_tiles; ++j) {
                const uint32_t s = j % kStages;
                if (j >= kStages && !mbar_wait(empty(s), ((j / kStages) - 1) & 1, a.status)) break;
                mbar_arrive_expect_tx(full(s), kStageBytes);
                const int32_t key = static_cast<int32_t>(j0 + j * kKeys);
                const int32_t row = static_cast<int32_t>(b * a.kv_heads + kvh);
                tma_load_4d(sb + s * kStageBytes, &tk, 0, key, 0, row, full(s));
                tma_load_4d(sb + s * kStageBytes + kTileBytes, &tv, 0, key, 0, row, full(s));
                issued = j + 1;
            }
            // the block's shared memory outlives every copy: the last copies' phases are each stage's
            // latest (consumers that gave up on a wait no longer see them)
            for (uint32_t j = issued > kStages ? issued - kStages : 0; j < issued; ++j)
                if (!mbar_wait(full(j % kStages), (j / kStages) & 1, a.status)) break;
        }
        return;
    }

    // -------------------------------------------------------------------- consumers
    const uint32_t hs = warp / kSlices, w = warp % kSlices;       // head slot, 128-dim slice
    const uint32_t hg = 2 * hp + hs;                              // head inside the GQA group
    const bool head_ok = hg < a.group;
    const uint32_t h = kvh * a.group + (head_ok ? hg : 0);
    const uint32_t g = lane >> 2, c = lane & 3;                   // MMA fragment row / column pair
    // Q slice in registers: A fragments of the 8 16-dim steps of dims [128w, 128w + 128)
    uint32_t qa[8][4];
    {
        const uint16_t *qrow = a.q_ws + (static_cast<uint64_t>(b) * a.q_heads + h) * a.T * kD;
        const bool r0 = head_ok && t0 + g < a.T, r1 = head_ok && t0 + g + 8 < a.T;
        const uint32_t *q0 = reinterpret_cast<const uint32_t *>(qrow + static_cast<uint64_t>(r0 ? t0 + g : 0) * kD);
        const uint32_t *q1 = reinterpret_cast<const uint32_t *>(qrow + static_cast<uint64_t>(r1 ? t0 + g + 8 : 0) * kD);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            const uint32_t d = (kSliceDims * w + 16 * kk + 2 * c) / 2;  // u32 index of dims (d, d + 1)
            qa[kk][0] = r0 ? q0[d] : 0u;
            qa[kk][1] = r1 ? q1[d] : 0u;
            qa[kk][2] = r0 ? q0[d + 4] : 0u;
            qa[kk][3] = r1 ? q1[d + 4] : 0u;
        }
    }
    float o[16][4];  // O slice: 16 n-tiles of 8 dims, rows g and g + 8
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;     // rows g, g + 8 (log2 units)
    const int pos0r = static_cast<int>(pos_first + g), pos1r = pos0r + 8;
    float *red = reinterpret_cast<float *>(base + kOffRed);
    bool alive = true;
    // K: matrix (lane >> 3) covers keys (lane & 7) + 8 (lane >> 4), dims + 8 ((lane >> 3) & 1) of a
    // 16-key, 16-dim block; V (transposed): keys (lane & 7) + 8 ((lane >> 3) & 1), dims + 8 (lane >> 4)
    const uint32_t k_key = (lane & 7) + 8 * (lane >> 4), k_col = (lane >> 3) & 1;
    const uint32_t v_key = (lane & 7) + 8 * ((lane >> 3) & 1), v_col = lane >> 4;

    for (uint32_t j = 0; j < n_tiles; ++j) {
        const uint32_t s = j % kStages;
        // a failed wait leaves the scores at zero but keeps every warp in step (the slice warps
        // meet at a barrier every tile)
        alive = alive && __all_sync(0xffffffffu, mbar_wait(full(s), (j / kStages) & 1, a.status));
        const uint32_t kbase = sb + s * kStageBytes, vbase = kbase + kTileBytes;
        // ---- partial scores of this slice: S[16 queries][32 keys] over dims [128w, 128w + 128)
        float sp[4][4];
#pragma unroll
        for (int n = 0; n < 4; ++n) sp[n][0] = sp[n][1] = sp[n][2] = sp[n][3] = 0.f;
        if (alive) {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
                for (int np = 0; np < 2; ++np) {  // keys 16np .. 16np + 15: two n-tiles
                    uint32_t r[4];
                    ldsm_x4(kbase + tile_off(16 * np + k_key, 16 * w + 2 * kk + k_col), r);
                    mma_bf16(sp[2 * np], qa[kk], r[0], r[1]);
                    mma_bf16(sp[2 * np + 1], qa[kk], r[2], r[3]);
                }
            }
        }
        // ---- the four slices' partials, added in slice order by every slice warp
        float *mine = red + (j & 1) * kRedFloats + ((hs * kSlices + w) * 16) * 32;
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) mine[(4 * n + e) * 32 + lane] = sp[n][e];
        head_sync(hs);
        float sc[4][4];
        {
            const float *part = red + (j & 1) * kRedFloats + (hs * kSlices * 16) * 32;
#pragma unroll
            for (int n = 0; n < 4; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    float v = part[(4 * n + e) * 32 + lane];
#pragma unroll
                    for (int q = 1; q < kSlices; ++q) v += part[(q * 16 + 4 * n + e) * 32 + lane];
                    sc[n][e] = v;
                }
        }
        // ---- masks (causal, window) and the online softmax of rows g and g + 8
        const int key0 = static_cast<int>(j0 + j * kKeys);
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = key0 + 8 * n + 2 * c + (e & 1);
                const int pos = e < 2 ? pos0r : pos1r;
                const bool vis = key <= pos && (!a.window || key > pos - static_cast<int>(a.window));
                const float x = vis ? sc[n][e] * a.scale_log2 : -INFINITY;
                sc[n][e] = x;
                if (e < 2) mx0 = fmaxf(mx0, x); else mx1 = fmaxf(mx1, x);
            }
#pragma unroll
        for (int off = 1; off < 4; off <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
        }
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float al0 = mn0 == -INFINITY ? 1.f : fast_exp2(m0 - mn0);  // 0 when m was -inf
        const float al1 = mn1 == -INFINITY ? 1.f : fast_exp2(m1 - mn1);
        const float sub0 = mn0 == -INFINITY ? 0.f : mn0, sub1 = mn1 == -INFINITY ? 0.f : mn1;
        m0 = mn0;
        m1 = mn1;
        float ps0 = 0.f, ps1 = 0.f;
        uint32_t pa[2][4];  // P as the A operand of the two 16-key steps
#pragma unroll
        for (int n = 0; n < 4; ++n) {
            const float p0 = fast_exp2(sc[n][0] - sub0), p1 = fast_exp2(sc[n][1] - sub0);
            const float p2 = fast_exp2(sc[n][2] - sub1), p3 = fast_exp2(sc[n][3] - sub1);
            ps0 += p0 + p1;
            ps1 += p2 + p3;
            pa[n >> 1][(n & 1) * 2] = pack_bf16(p0, p1);      // row g, keys 8n + 2c, + 1
            pa[n >> 1][(n & 1) * 2 + 1] = pack_bf16(p2, p3);  // row g + 8
        }
        l0 = l0 * al0 + ps0;
        l1 = l1 * al1 + ps1;
        if (__any_sync(0xffffffffu, al0 != 1.f || al1 != 1.f)) {
#pragma unroll
            for (int n = 0; n < 16; ++n) {
                o[n][0] *= al0;
                o[n][1] *= al0;
                o[n][2] *= al1;
                o[n][3] *= al1;
            }
        }
        // ---- O slice += P V[:, 128w .. 128w + 128)
        if (alive) {
#pragma unroll
            for (int ks = 0; ks < 2; ++ks) {
#pragma unroll
                for (int dn = 0; dn < 8; ++dn) {  // dims 16dn .. 16dn + 15 of the slice: two n-tiles
                    uint32_t r[4];
                    ldsm_x4_t(vbase + tile_off(16 * ks + v_key, 16 * w + 2 * dn + v_col), r);
                    mma_bf16(o[2 * dn], pa[ks], r[0], r[1]);
                    mma_bf16(o[2 * dn + 1], pa[ks], r[2], r[3]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty(s));
    }

    // -------------------------------------------------------------------- O / l -> bf16
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, off);
        l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    if (!alive || !head_ok) return;
    const float inv0 = l0 > 0.f ? 1.0f / l0 : 0.f, inv1 = l1 > 0.f ? 1.0f / l1 : 0.f;
    const uint64_t row_stride = static_cast<uint64_t>(a.q_heads) * kD;
    uint16_t *out0 = a.out + (static_cast<uint64_t>(b) * a.T + t0 + g) * row_stride + static_cast<uint64_t>(h) * kD +
                     kSliceDims * w + 2 * c;
    const bool w0 = t0 + g < a.T, w1 = t0 + g + 8 < a.T;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
        if (w0) *reinterpret_cast<uint32_t *>(out0 + 8 * n) = pack_bf16(o[n][0] * inv0, o[n][1] * inv0);
        if (w1) *reinterpret_cast<uint32_t *>(out0 + 8 * row_stride + 8 * n) = pack_bf16(o[n][2] * inv1, o[n][3] * inv1);
    }
}

}  // namespace

size_t prefill_gqa_workspace_bytes(uint32_t batch, uint32_t tokens, uint32_t q_heads) {
    return static_cast<size_t>(batch) * q_heads * tokens * kD * 2;
}

int launch_prefill_gqa_prep(const apex_attn_params *p, const uint16_t *q_raw, const uint16_t *k_raw,
                            const uint16_t *v_raw, const uint16_t *q_w, const uint16_t *k_w, uint16_t *k_cache,
                            uint16_t *v_cache, uint32_t capacity, uint32_t batch, uint32_t tokens, uint32_t pos0,
                            void *workspace, cudaStream_t s) {
    uint16_t *q_ws = static_cast<uint16_t *>(workspace);
    const uint64_t D = kD, Hq = p->q_heads, Hkv = p->kv_heads;
    for (uint32_t b = 0; b < batch; ++b) {
        const uint64_t tok = static_cast<uint64_t>(b) * tokens;
        // q: [T][Hq][512] -> [Hq][T][512] of the workspace (token stride 512, head stride T * 512)
        int rc = apex_head_norm_rope_bf16(q_raw + tok * Hq * D, q_w, q_ws + static_cast<uint64_t>(b) * Hq * tokens * D,
                                          tokens, p->q_heads, kD, q_w != nullptr, p->rope_pairs, p->rope_base, pos0,
                                          kD, tokens * kD, p->eps, s);
        if (rc) return rc;
        uint16_t *kc = k_cache + (static_cast<uint64_t>(b) * Hkv * capacity + pos0) * D;
        uint16_t *vc = v_cache + (static_cast<uint64_t>(b) * Hkv * capacity + pos0) * D;
        rc = apex_head_norm_rope_bf16(k_raw + tok * Hkv * D, k_w, kc, tokens, p->kv_heads, kD, k_w != nullptr,
                                      p->rope_pairs, p->rope_base, pos0, kD, capacity * kD, p->eps, s);
        if (rc) return rc;
        if (p->v_norm) {
            rc = apex_head_norm_rope_bf16(v_raw + tok * Hkv * D, nullptr, vc, tokens, p->kv_heads, kD, 0, 0,
                                          p->rope_base, pos0, kD, capacity * kD, p->eps, s);
            if (rc) return rc;
        } else {
            for (uint32_t hh = 0; hh < p->kv_heads; ++hh) {
                rc = check_cuda(cudaMemcpy2DAsync(vc + static_cast<uint64_t>(hh) * capacity * D, D * 2,
                                                  v_raw + (tok * Hkv + hh) * D, Hkv * D * 2, D * 2, tokens,
                                                  cudaMemcpyDeviceToDevice, s),
                                "prefill (head_dim 512): v copy");
                if (rc) return rc;
            }
        }
    }
    return APEX_OK;
}

int launch_prefill_gqa_attend(const apex_attn_params *p, const void *workspace, const uint16_t *k_cache,
                              const uint16_t *v_cache, uint32_t capacity, uint32_t batch, uint32_t tokens,
                              uint32_t pos0, uint16_t *out, cudaStream_t s) {
    if (prefill_wide_applies(p))
        return launch_prefill_wide_attend(p, workspace, k_cache, v_cache, capacity, batch, tokens, pos0, out, s);
    const uint64_t kv_len = static_cast<uint64_t>(pos0) + tokens;
    const uint64_t row = kD * 2ull;
    // caches [B*Hkv][capacity][512] as {64-element chunks, keys (cut at pos0 + T), 8 chunks, kv rows}:
    // one box = 32 keys x 512 dims, chunk-major
    CUtensorMap tk, tv;
    int rc = make_tensor_map_bf16_4d(&tk, k_cache, {64, kv_len, kD / 64, static_cast<uint64_t>(batch) * p->kv_heads},
                                     {row, 128, row * capacity}, {64, static_cast<uint32_t>(kKeys), kD / 64, 1}, true);
    if (rc) return rc;
    rc = make_tensor_map_bf16_4d(&tv, v_cache, {64, kv_len, kD / 64, static_cast<uint64_t>(batch) * p->kv_heads},
                                 {row, 128, row * capacity}, {64, static_cast<uint32_t>(kKeys), kD / 64, 1}, true);
    if (rc) return rc;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        rc = check_cuda(cudaFuncSetAttribute(prefill_gqa_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kSmemBytes)),
                        "prefill (head_dim 512) smem attribute");
        if (rc) return rc;
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    GqaPrefillArgs a{};
    a.q_ws = static_cast<const uint16_t *>(workspace);
    a.out = out;
    a.status = device_status_ptr();
    if (!a.status) return fail(APEX_ERR_CUDA, "prefill (head_dim 512): device status word unavailable");
    a.T = tokens;
    a.pos0 = pos0;
    a.q_heads = p->q_heads;
    a.kv_heads = p->kv_heads;
    a.group = p->q_heads / p->kv_heads;
    a.window = p->window;
    a.head_pairs = (a.group + kHeadsPerCta - 1) / kHeadsPerCta;
    a.n_qtiles = (tokens + kQ - 1) / kQ;
    a.scale_log2 = p->scale * kLog2e;
    const dim3 grid(a.n_qtiles * p->kv_heads * a.head_pairs, 1, batch);
    prefill_gqa_kernel<<<grid, kThreads, kSmemBytes, s>>>(a, tk, tv);
    return check_cuda(cudaGetLastError(), "prefill (head_dim 512) launch");
}

}  // namespace apex
