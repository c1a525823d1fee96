// prefill_tc.cu -- fused causal (optionally sliding-window) prefill on tcgen05 tensor cores.
//
// Reference semantics (docs/B6_3_attention.md:444-454 and :296-343): q and k are RMS-normed
// with their bf16 weights and roped at position pos0 + t, v optionally weightless-normed; K and
// V are appended to the cache [kv_heads][capacity][hd] at pos0 (the reference's f32 cache
// becomes bf16, its planned format, docs/B6_3_attention.md:99-102); then for every query
// o = softmax(scale * q K^T) V over keys p - window < j <= p (or j <= p), GQA map h/(Hq/Hkv).
//
// Two launches per call:
//  1. prep: one warp per 256-wide row, 16-byte loads; q -> a head-major workspace
//     [B][Hq][T][256] so a 128-query tile is one 3-D TMA box; k, v -> the caches.
//  2. attention: one CTA per (128-query tile, q head), 8 warps:
//       warp 0  TMA producer: Q tile once (64 KB), then K and V as 64-key half tiles (32 KB)
//               through a 4-slot ring; 3-D tensor maps bound keys at pos0+T so keys past the
//               cache end read as zeros (never uninitialised memory).
//       warp 1  tcgen05.mma issuer (one thread) and TMEM owner (512 columns):
//               S_j = Q K_j^T  (M=128, N=64 x 2, K=16 x 16, bf16 -> f32) into S[j%2],
//               O  += P_j V_j  (M=128, N=256, K=16 x 8; V is the MN-major B operand).
//               S_{j+1} is issued before PV_j, so the tensor pipe computes the next scores
//               while the softmax warps work on the current ones.
//       warps 4-7  softmax and epilogue, one query row per thread (TMEM lane = row):
//               tcgen05.ld of the S row, causal/window mask only on boundary tiles, online
//               softmax in the log2 domain with lazy rescaling (O is rescaled in TMEM only
//               when the row max grows by more than 2^8), P written as bf16 into shared memory
//               in the 128-byte-swizzled K-major layout the PV MMA reads.
//     TMEM: O = columns [0, 256), S0 = [256, 384), S1 = [384, 512).
//     Tiles of 128 keys; only tiles that intersect the causal/window band are visited.
#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "row256.cuh"

namespace apex {
namespace {

constexpr int kD = 256;
constexpr int kBM = 128;                          // queries per CTA
constexpr int kBN = 128;                          // keys per tile
constexpr int kSlotKeys = 64;                     // keys per ring slot
constexpr int kSlots = 4;
constexpr uint32_t kQChunk = kBM * 128;           // 64 dims of 128 rows, 128 B per row
constexpr uint32_t kSlotChunk = kSlotKeys * 128;  // 64 dims of 64 keys
constexpr uint32_t kPChunk = kBM * 128;           // 64 keys of 128 rows
constexpr uint32_t kQBytes = kBM * kD * 2;        // 65536
constexpr uint32_t kSlotBytes = kSlotKeys * kD * 2;  // 32768
constexpr uint32_t kPBytes = kBM * kBN * 2;       // 32768
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffSlots = kOffQ + kQBytes;
constexpr uint32_t kOffP = kOffSlots + kSlots * kSlotBytes;
constexpr uint32_t kOffBar = kOffP + kPBytes;
constexpr uint32_t kOffTmem = kOffBar + 128;
constexpr uint32_t kSmemBytes = kOffTmem + 128 + 1024;  // + slack to align the base to 1024
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 0, kColS = 256;
constexpr int kThreads = 256;
constexpr float kTau = 8.0f;                      // lazy-rescale threshold (log2 units)
constexpr float kLog2e = 1.4426950408889634f;

static_assert(kSmemBytes <= 232448, "shared memory budget");

// barrier indices (8 bytes each at kOffBar)
constexpr int kBarQ = 0, kBarFull = 1, kBarEmpty = 5, kBarS = 9, kBarP = 11, kBarO = 12;

struct PrefillArgs {
    uint16_t *out;  // [B][T][Hq][D]
    unsigned *status;  // device status word
    uint32_t T, pos0, q_heads, kv_heads, window, n_qtiles;
    float scale_log2;
};

__device__ __forceinline__ bool visible(uint32_t key, uint32_t pos, uint32_t window) {
    return key <= pos && (window == 0 || key + window > pos);
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const PrefillArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sb = smem_u32(base);
    auto bar = [&](int i) { return sb + kOffBar + 8u * i; };
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(base + kOffTmem);

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t bh = blockIdx.x;
    const uint32_t h = bh % a.q_heads, b = bh / a.q_heads;
    const uint32_t kvh = h / (a.q_heads / a.kv_heads);
    const uint32_t qt = a.n_qtiles - 1 - blockIdx.y;  // heaviest tiles first
    const uint32_t t0 = qt * kBM;
    const uint32_t rows_valid = min(static_cast<uint32_t>(kBM), a.T - t0);
    const uint32_t pos_first = a.pos0 + t0, pos_last = pos_first + rows_valid - 1;
    const uint32_t kv_lo = (a.window && pos_first + 1 > a.window) ? pos_first + 1 - a.window : 0;
    const uint32_t j_start = (kv_lo / kBN) * kBN;
    const uint32_t n_tiles = (pos_last - j_start) / kBN + 1;

    if (tid == 0) {
        mbar_init(bar(kBarQ), 1);
        for (int i = 0; i < kSlots; ++i) {
            mbar_init(bar(kBarFull + i), 1);
            mbar_init(bar(kBarEmpty + i), 1);
        }
        mbar_init(bar(kBarS + 0), 1);
        mbar_init(bar(kBarS + 1), 1);
        mbar_init(bar(kBarP), kBM);
        mbar_init(bar(kBarO), 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_holder), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            prefetch_tensormap(&tm_q);
            prefetch_tensormap(&tm_k);
            prefetch_tensormap(&tm_v);
            mbar_arrive_expect_tx(bar(kBarQ), kQBytes);
            for (int c = 0; c < 4; ++c)
                tma_load_3d(sb + kOffQ + c * kQChunk, &tm_q, c * 64, static_cast<int32_t>(t0),
                            static_cast<int32_t>(b * a.q_heads + h), bar(kBarQ));
            uint32_t n = 0;
            bool alive = true;
            for (uint32_t j = 0; j < n_tiles && alive; ++j) {
                const uint32_t key0 = j_start + j * kBN;
                for (int which = 0; which < 2 && alive; ++which) {
                    const CUtensorMap *map = which == 0 ? &tm_k : &tm_v;
                    for (int half = 0; half < 2; ++half, ++n) {
                        const uint32_t slot = n % kSlots;
                        if (n >= kSlots && !mbar_wait(bar(kBarEmpty + slot), ((n / kSlots) - 1) & 1, a.status)) {
                            alive = false;
                            break;
                        }
                        mbar_arrive_expect_tx(bar(kBarFull + slot), kSlotBytes);
                        const uint32_t dst = sb + kOffSlots + slot * kSlotBytes;
                        for (int c = 0; c < 4; ++c)
                            tma_load_3d(dst + c * kSlotChunk, map, c * 64,
                                        static_cast<int32_t>(key0 + half * kSlotKeys),
                                        static_cast<int32_t>(b * a.kv_heads + kvh), bar(kBarFull + slot));
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idS = idesc_bf16_f32(kBM, kSlotKeys, 0, 0);
            constexpr uint32_t idPV = idesc_bf16_f32(kBM, kD, 0, 1);
            bool alive = mbar_wait(bar(kBarQ), 0, a.status);
            auto issue_pv = [&](uint32_t i) {
                if (!alive) return;
                alive = mbar_wait(bar(kBarP), i & 1, a.status) && mbar_wait(bar(kBarFull + 2), i & 1, a.status) &&
                        mbar_wait(bar(kBarFull + 3), i & 1, a.status);
                if (!alive) return;
                tc_fence_after();
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) {
                    const uint64_t ad = smem_desc_sw128(sb + kOffP + (ks / 4) * kPChunk + (ks % 4) * 32, 16, 1024);
                    const uint32_t vslot = 2 + ks / 4;
                    const uint64_t bd = smem_desc_sw128(sb + kOffSlots + vslot * kSlotBytes + (ks % 4) * 2048,
                                                        kSlotChunk, 1024);
                    tc_mma_ss(tmem + kColO, ad, bd, idPV, (i > 0 || ks > 0) ? 1u : 0u);
                }
                tc_commit(bar(kBarO));
                tc_commit(bar(kBarEmpty + 2));
                tc_commit(bar(kBarEmpty + 3));
            };
            for (uint32_t j = 0; j < n_tiles && alive; ++j) {
                alive = mbar_wait(bar(kBarFull + 0), j & 1, a.status) && mbar_wait(bar(kBarFull + 1), j & 1, a.status);
                if (!alive) break;
                tc_fence_after();
                const uint32_t s_col = kColS + (j & 1) * 128;
#pragma unroll
                for (int ks = 0; ks < 16; ++ks) {
                    const uint64_t ad = smem_desc_sw128(sb + kOffQ + (ks / 4) * kQChunk + (ks % 4) * 32, 16, 1024);
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const uint64_t bd = smem_desc_sw128(
                            sb + kOffSlots + half * kSlotBytes + (ks / 4) * kSlotChunk + (ks % 4) * 32, 16, 1024);
                        tc_mma_ss(tmem + s_col + half * kSlotKeys, ad, bd, idS, ks > 0 ? 1u : 0u);
                    }
                }
                tc_commit(bar(kBarS + (j & 1)));
                tc_commit(bar(kBarEmpty + 0));
                tc_commit(bar(kBarEmpty + 1));
                if (j >= 1) issue_pv(j - 1);
            }
            issue_pv(n_tiles - 1);
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------ softmax + epilogue
        const uint32_t r = tid - 128;              // query row == TMEM lane
        const uint32_t lane_base = tmem + ((32u * (warp - 4)) << 16);
        const uint32_t t = t0 + r;
        const uint32_t pos = a.pos0 + t;
        const bool row_valid = r < rows_valid;
        float m_run = -INFINITY, l_run = 0.f;
        bool alive = true;
        for (uint32_t j = 0; j < n_tiles; ++j) {
            if (!__all_sync(0xffffffffu, mbar_wait(bar(kBarS + (j & 1)), (j >> 1) & 1, a.status))) {
                alive = false;  // warp-uniform: the tcgen05.ld below is warp-collective
                break;
            }
            tc_fence_after();
            uint32_t sv[4][32];
            const uint32_t s_addr = lane_base + kColS + (j & 1) * 128;
#pragma unroll
            for (int c = 0; c < 4; ++c) tmem_ld32(s_addr + c * 32, sv[c]);
            tc_wait_ld();
            const uint32_t key0 = j_start + j * kBN;
            const bool need_mask = (key0 + kBN - 1 > pos_first) || (a.window && key0 + a.window <= pos_last);
            float mt = -INFINITY;
#pragma unroll
            for (int c = 0; c < 4; ++c)
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    float x = __uint_as_float(sv[c][i]) * a.scale_log2;
                    if (need_mask && !visible(key0 + c * 32 + i, pos, a.window)) x = -INFINITY;
                    sv[c][i] = __float_as_uint(x);
                    mt = fmaxf(mt, x);
                }
            float alpha = 1.f;
            bool rescale = false;
            if (mt > m_run + kTau) {
                alpha = fast_exp2(m_run - mt);  // 0 when m_run = -inf
                rescale = j > 0;
                m_run = mt;
            }
            const float m_use = m_run == -INFINITY ? 0.f : m_run;
            float rowsum = 0.f;
            uint32_t packed[4][16];
#pragma unroll
            for (int c = 0; c < 4; ++c)
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float p0 = fast_exp2(__uint_as_float(sv[c][2 * i]) - m_use);
                    const float p1 = fast_exp2(__uint_as_float(sv[c][2 * i + 1]) - m_use);
                    rowsum += p0 + p1;
                    packed[c][i] = pack_bf16(p0, p1);
                }
            l_run = l_run * alpha + rowsum;
            if (j >= 1 && !__all_sync(0xffffffffu, mbar_wait(bar(kBarO), (j - 1) & 1, a.status))) {
                alive = false;
                break;
            }
            // tcgen05.ld/st are warp-collective: the whole warp rescales if any of its rows
            // must, with factor 1 for the rows that need not.
            if (__any_sync(0xffffffffu, rescale)) {
                const float f = rescale ? alpha : 1.0f;
                tc_fence_after();
#pragma unroll 1
                for (int c = 0; c < 8; ++c) {
                    uint32_t o[32];
                    tmem_ld32(lane_base + kColO + c * 32, o);
                    tc_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
                    tmem_st32(lane_base + kColO + c * 32, o);
                }
                tc_wait_st();
            }
            // P row r -> 128-byte-swizzled K-major tile: 16-byte unit u of key chunk c at
            // chunk + r*128 + ((u ^ (r & 7)) * 16).
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint8_t *rowp = base + kOffP + c * kPChunk + r * 128;
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int w0 = (c * 64 + u * 8) / 2;  // packed index of the unit's first pair
                    uint4 v;
                    v.x = packed[w0 / 16][w0 % 16];
                    v.y = packed[(w0 + 1) / 16][(w0 + 1) % 16];
                    v.z = packed[(w0 + 2) / 16][(w0 + 2) % 16];
                    v.w = packed[(w0 + 3) / 16][(w0 + 3) % 16];
                    *reinterpret_cast<uint4 *>(rowp + ((u ^ (r & 7)) * 16)) = v;
                }
            }
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(bar(kBarP));
        }
        // epilogue: O / l -> bf16 out[b][t][h][:]
        if (__all_sync(0xffffffffu, alive && mbar_wait(bar(kBarO), (n_tiles - 1) & 1, a.status))) {
            tc_fence_after();
            const float inv_l = l_run > 0.f ? 1.0f / l_run : 0.f;
            uint16_t *orow = a.out + ((static_cast<uint64_t>(b) * a.T + t) * a.q_heads + h) * kD;
#pragma unroll 1
            for (int c = 0; c < 8; ++c) {
                uint32_t o[32];
                tmem_ld32(lane_base + kColO + c * 32, o);
                tc_wait_ld();
                if (row_valid) {
                    uint4 *dst = reinterpret_cast<uint4 *>(orow + c * 32);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        uint4 v;
                        v.x = pack_bf16(__uint_as_float(o[8 * q + 0]) * inv_l, __uint_as_float(o[8 * q + 1]) * inv_l);
                        v.y = pack_bf16(__uint_as_float(o[8 * q + 2]) * inv_l, __uint_as_float(o[8 * q + 3]) * inv_l);
                        v.z = pack_bf16(__uint_as_float(o[8 * q + 4]) * inv_l, __uint_as_float(o[8 * q + 5]) * inv_l);
                        v.w = pack_bf16(__uint_as_float(o[8 * q + 6]) * inv_l, __uint_as_float(o[8 * q + 7]) * inv_l);
                        dst[q] = v;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---------------------------------------------------------------- prep: norm + rope + append
struct PrepArgs {
    const uint16_t *q_raw, *k_raw, *v_raw, *q_w, *k_w;
    uint16_t *q_ws, *k_cache, *v_cache;
    uint32_t B, T, pos0, q_heads, kv_heads, capacity, rope_pairs, qk_norm, v_norm;
    float rope_base, eps;
};

__global__ void __launch_bounds__(256) prefill_prep_kernel(const PrepArgs a) {
    __shared__ float inv_freq[kD / 2];
    for (uint32_t i = threadIdx.x; i < a.rope_pairs; i += blockDim.x)
        inv_freq[i] = rope_inv_freq(i, kD, a.rope_base);
    __syncthreads();
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t nq = static_cast<uint64_t>(a.B) * a.T * a.q_heads;
    const uint64_t nk = static_cast<uint64_t>(a.B) * a.T * a.kv_heads;
    const uint64_t total = nq + 2 * nk;
    const uint64_t warps = static_cast<uint64_t>(gridDim.x) * (blockDim.x >> 5);
    for (uint64_t r = static_cast<uint64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < total;
         r += warps) {
        const uint16_t *src;
        uint16_t *dst;
        const uint16_t *w;
        bool norm;
        uint32_t pairs, t;
        if (r < nq) {
            const uint32_t hq = static_cast<uint32_t>(r % a.q_heads);
            const uint64_t bt = r / a.q_heads;
            t = static_cast<uint32_t>(bt % a.T);
            const uint32_t bb = static_cast<uint32_t>(bt / a.T);
            src = a.q_raw + r * kD;
            dst = a.q_ws + ((static_cast<uint64_t>(bb) * a.q_heads + hq) * a.T + t) * kD;
            w = a.q_w;
            norm = a.qk_norm;
            pairs = a.rope_pairs;
        } else {
            const bool is_k = r < nq + nk;
            const uint64_t rr = r - nq - (is_k ? 0 : nk);
            const uint32_t hk = static_cast<uint32_t>(rr % a.kv_heads);
            const uint64_t bt = rr / a.kv_heads;
            t = static_cast<uint32_t>(bt % a.T);
            const uint32_t bb = static_cast<uint32_t>(bt / a.T);
            src = (is_k ? a.k_raw : a.v_raw) + rr * kD;
            dst = (is_k ? a.k_cache : a.v_cache) +
                  ((static_cast<uint64_t>(bb) * a.kv_heads + hk) * a.capacity + a.pos0 + t) * kD;
            w = is_k ? a.k_w : nullptr;
            norm = is_k ? a.qk_norm : a.v_norm;
            pairs = is_k ? a.rope_pairs : 0;
        }
        float x[8];
        unpack8(*reinterpret_cast<const uint4 *>(src + 8 * lane), x);
        norm_rope_row(x, lane, norm, w, a.eps, pairs, inv_freq, static_cast<float>(a.pos0 + t));
        *reinterpret_cast<uint4 *>(dst + 8 * lane) = pack8(x);
    }
}

size_t q_ws_bytes(uint32_t batch, uint32_t tokens, uint32_t q_heads) {
    return static_cast<size_t>(batch) * tokens * q_heads * kD * 2;
}

}  // namespace
}  // namespace apex

namespace apex {
namespace {

int validate_prefill(const apex_attn_params *p, uint32_t capacity, uint32_t batch, uint32_t tokens,
                     uint32_t pos0, std::initializer_list<const void *> tensors, const char *name) {
    const std::string n(name);
    if (!p) return fail(APEX_ERR_INVALID_ARGUMENT, n + ": null params");
    if (p->head_dim != kD) return fail(APEX_ERR_UNSUPPORTED, n + ": this build supports head_dim 256");
    if (p->kv_heads == 0 || p->q_heads == 0 || p->q_heads % p->kv_heads)
        return fail(APEX_ERR_INVALID_ARGUMENT, n + ": q_heads must be a multiple of kv_heads");
    if (p->rope_pairs > kD / 2) return fail(APEX_ERR_INVALID_ARGUMENT, n + ": rope_pairs > head_dim / 2");
    if (batch == 0 || tokens == 0) return APEX_OK;
    for (const void *ptr : tensors) {
        if (!ptr) return fail(APEX_ERR_INVALID_ARGUMENT, n + ": null tensor");
        if (!aligned16(ptr)) return fail(APEX_ERR_INVALID_ARGUMENT, n + ": tensors must be 16-byte aligned");
    }
    if (static_cast<uint64_t>(pos0) + tokens > capacity)
        return fail(APEX_ERR_INVALID_ARGUMENT, n + ": pos0 + tokens exceeds capacity");
    if ((tokens + kBM - 1) / kBM > 65535 || static_cast<uint64_t>(batch) * p->q_heads > 0x7fffffffu)
        return fail(APEX_ERR_INVALID_ARGUMENT, n + ": problem too large for one launch");
    return APEX_OK;
}

int launch_prep(const apex_attn_params *p, const uint16_t *q_raw, const uint16_t *k_raw, const uint16_t *v_raw,
                const uint16_t *q_w, const uint16_t *k_w, uint16_t *k_cache, uint16_t *v_cache,
                uint32_t capacity, uint32_t batch, uint32_t tokens, uint32_t pos0, uint16_t *q_normed,
                cudaStream_t s) {
    PrepArgs pa{q_raw, k_raw, v_raw, q_w, k_w, q_normed, k_cache, v_cache, batch, tokens, pos0, p->q_heads,
                p->kv_heads, capacity, p->rope_pairs, p->qk_norm, p->v_norm, p->rope_base, p->eps};
    const uint64_t rows = static_cast<uint64_t>(batch) * tokens * (p->q_heads + 2ull * p->kv_heads);
    const uint32_t grid = static_cast<uint32_t>(std::min<uint64_t>((rows + 7) / 8, 16ull * sm_count()));
    prefill_prep_kernel<<<grid, 256, 0, s>>>(pa);
    return check_cuda(cudaGetLastError(), "prefill prep launch");
}

int launch_attend(const apex_attn_params *p, const uint16_t *q_normed, const uint16_t *k_cache,
                  const uint16_t *v_cache, uint32_t capacity, uint32_t batch, uint32_t tokens, uint32_t pos0,
                  uint16_t *out, cudaStream_t s) {
    CUtensorMap tq, tk, tv;
    int rc = make_tensor_map_bf16_3d(&tq, q_normed, kD, tokens, static_cast<uint64_t>(batch) * p->q_heads,
                                     kD * 2ull, static_cast<uint64_t>(tokens) * kD * 2, 64, kBM);
    if (rc) return rc;
    const uint64_t kv_len = static_cast<uint64_t>(pos0) + tokens;
    rc = make_tensor_map_bf16_3d(&tk, k_cache, kD, kv_len, static_cast<uint64_t>(batch) * p->kv_heads, kD * 2ull,
                                 static_cast<uint64_t>(capacity) * kD * 2, 64, kSlotKeys);
    if (rc) return rc;
    rc = make_tensor_map_bf16_3d(&tv, v_cache, kD, kv_len, static_cast<uint64_t>(batch) * p->kv_heads, kD * 2ull,
                                 static_cast<uint64_t>(capacity) * kD * 2, 64, kSlotKeys);
    if (rc) return rc;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_set[dev]) {
        rc = check_cuda(cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kSmemBytes)),
                        "prefill smem attribute");
        if (rc) return rc;
        attr_set[dev] = true;
    }
    unsigned *status = device_status_ptr();
    if (!status) return fail(APEX_ERR_CUDA, "prefill: device status word unavailable");
    const uint32_t n_qtiles = (tokens + kBM - 1) / kBM;
    PrefillArgs fa{out, status, tokens, pos0, p->q_heads, p->kv_heads, p->window, n_qtiles, p->scale * kLog2e};
    const dim3 grid(batch * p->q_heads, n_qtiles);
    prefill_tc_kernel<<<grid, kThreads, kSmemBytes, s>>>(tq, tk, tv, fa);
    return check_cuda(cudaGetLastError(), "prefill attention launch");
}

}  // namespace
}  // namespace apex

extern "C" size_t apex_attn_prefill_workspace_bytes(const apex_attn_params *p, uint32_t batch,
                                                    uint32_t tokens) {
    if (!p) return 0;
    return apex::q_ws_bytes(batch, tokens, p->q_heads);
}

extern "C" int apex_attn_prefill_prep_bf16(const apex_attn_params *p, const uint16_t *q_raw,
                                           const uint16_t *k_raw, const uint16_t *v_raw,
                                           const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                                           uint16_t *k_cache, uint16_t *v_cache, uint32_t capacity,
                                           uint32_t batch, uint32_t tokens, uint32_t pos0,
                                           uint16_t *q_normed, void *stream) {
    using namespace apex;
    int rc = validate_prefill(p, capacity, batch, tokens, pos0, {q_raw, k_raw, v_raw, k_cache, v_cache, q_normed},
                              "apex_attn_prefill_prep_bf16");
    if (rc || batch == 0 || tokens == 0) return rc ? rc : ok();
    rc = launch_prep(p, q_raw, k_raw, v_raw, q_norm_w, k_norm_w, k_cache, v_cache, capacity, batch, tokens, pos0,
                     q_normed, static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

extern "C" int apex_attn_prefill_attend_bf16(const apex_attn_params *p, const uint16_t *q_normed,
                                             const uint16_t *k_cache, const uint16_t *v_cache,
                                             uint32_t capacity, uint32_t batch, uint32_t tokens,
                                             uint32_t pos0, uint16_t *out, void *stream) {
    using namespace apex;
    int rc = validate_prefill(p, capacity, batch, tokens, pos0, {q_normed, k_cache, v_cache, out},
                              "apex_attn_prefill_attend_bf16");
    if (rc || batch == 0 || tokens == 0) return rc ? rc : ok();
    rc = launch_attend(p, q_normed, k_cache, v_cache, capacity, batch, tokens, pos0, out,
                       static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

extern "C" int apex_attn_prefill_bf16(const apex_attn_params *p, const uint16_t *q_raw,
                                      const uint16_t *k_raw, const uint16_t *v_raw,
                                      const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                                      uint16_t *k_cache, uint16_t *v_cache, uint32_t capacity,
                                      uint32_t batch, uint32_t tokens, uint32_t pos0,
                                      uint16_t *out, void *workspace, size_t workspace_bytes,
                                      void *stream) {
    using namespace apex;
    int rc = validate_prefill(p, capacity, batch, tokens, pos0, {q_raw, k_raw, v_raw, k_cache, v_cache, out},
                              "apex_attn_prefill_bf16");
    if (rc || batch == 0 || tokens == 0) return rc ? rc : ok();
    const size_t need = q_ws_bytes(batch, tokens, p->q_heads);
    if (!workspace || workspace_bytes < need)
        return fail(APEX_ERR_WORKSPACE, "apex_attn_prefill_bf16: workspace of " + std::to_string(need) + " bytes required");
    if (!aligned16(workspace)) return fail(APEX_ERR_INVALID_ARGUMENT, "apex_attn_prefill_bf16: tensors must be 16-byte aligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint16_t *qn = static_cast<uint16_t *>(workspace);
    rc = launch_prep(p, q_raw, k_raw, v_raw, q_norm_w, k_norm_w, k_cache, v_cache, capacity, batch, tokens, pos0, qn, s);
    if (rc) return rc;
    rc = launch_attend(p, qn, k_cache, v_cache, capacity, batch, tokens, pos0, out, s);
    return rc ? rc : ok();
}
