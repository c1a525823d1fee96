// prefill_wide.cu -- tcgen05 attention of the head_dim-512 prefill (the reference model's global
// layers: 16 q heads over 2 kv heads of head_dim 512, docs/B6_3_attention.md:46-60) for GQA groups
// of 1, 2, 4 or 8.  The preparation (q norm + RoPE into the workspace, k and v into the caches) is
// prefill_gqa.cu's; other groups take prefill_gqa.cu's mma.sync attention.
//
// One work item = the 128 query rows {G heads of one kv head} x {128 / G consecutive queries}, so
// every key tile serves all heads of the group.  A 128 x 512 f32 O fills all of TMEM, so the item
// runs on a CTA pair (a cluster of two) that splits the head dimension: CTA c owns dims
// [256c, 256c + 256) of Q, K, V and O and issues its own cta_group::1 MMAs.
//   S_c = Q_c K_c^T   (M=128 rows, N=32 keys, K=256): Q_c in TMEM (A operand, loaded once by the
//                     softmax warps), this CTA's half of the key tile in shared memory, K-major
//   S = S_0 + S_1     the softmax warps swap their 128 x 32 f32 partials through distributed
//                     shared memory each tile; f32 addition commutes, so both CTAs hold the same
//                     scores bit for bit, the same softmax, and the same P
//   O_c += P V_c      (M=128, N=256 dims, K=32 keys): P in TMEM (bf16 pairs over the tile's S
//                     columns), this CTA's half of the V tile in shared memory, MN-major
// TMEM (each CTA, lane = row): O [0, 256), Q [256, 384), S/P of tile j in [384 + 32 (j % 3), +32).
// Per CTA, 8 warps: warp 0 TMA producer (K and V half-tiles of 32 keys, one tiled copy each),
// warp 1 TMEM owner and MMA issuer (S(j+2) before PV(j)), warps 2-3 idle, warps 4-7 softmax (thread
// = row; tile j+1's partial goes to the peer before tile j's softmax; log2-domain online softmax,
// masks only on tiles crossing the causal / window band, O rescaled in TMEM only when a row max
// grows by more than 2^8) and the epilogue.
#include <cuda_runtime.h>

#include <algorithm>
#include <string>

#include "common.cuh"
#include "internal.h"

namespace apex {
namespace {

constexpr int kD = 512;
constexpr int kRows = 128;                           // TMEM lanes: group heads x queries
constexpr int kKeys = 32;                            // keys per tile
constexpr int kStages = 5;
constexpr int kSBufs = 3;                            // S/P buffers in TMEM: the issuer runs two tiles ahead
constexpr int kXBufs = 4;                            // score-partial buffers: the peer runs up to three ahead
constexpr uint32_t kKvChunk = kKeys * 128;           // 4 KB: 32 keys x 64 dims, 128-byte swizzle
constexpr uint32_t kTileBytes = 4 * kKvChunk;        // 16 KB: this CTA's 256 dims of 32 keys
constexpr uint32_t kStageBytes = 2 * kTileBytes;     // K tile, then V tile
constexpr uint32_t kXBytes = kRows * kKeys * 4;      // 16 KB: one tile's score partials
constexpr uint32_t kOffStages = 0;
constexpr uint32_t kOffX = kOffStages + kStages * kStageBytes;
// barriers: Full/Empty per stage; QReady (Q in TMEM); S (scores of tile j in buffer j % 3); X (the
// peer's partial of tile j arrived in buffer j % 4); P (P of tile j in TMEM); O (PV of tile parity
// done); OFinal (every MMA done)
constexpr int kBarFull = 0, kBarEmpty = kBarFull + kStages, kBarQ = kBarEmpty + kStages, kBarS = kBarQ + 1,
              kBarX = kBarS + kSBufs, kBarP = kBarX + kXBufs, kBarO = kBarP + kSBufs, kBarOFinal = kBarO + 2,
              kNumBars = kBarOFinal + 1;
constexpr uint32_t kOffBar = kOffX + kXBufs * kXBytes;
constexpr uint32_t kOffTmem = kOffBar + 8 * kNumBars;
constexpr uint32_t kSmemBytes = kOffTmem + 16 + 1024;  // + alignment slack of the dynamic base
static_assert(kSmemBytes <= 232448, "shared memory budget");
constexpr int kThreads = 256;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 0, kColQ = 256, kColS = 384;
constexpr float kTau = 8.0f;  // lazy-rescale threshold (log2 units)
constexpr float kLog2e = 1.4426950408889634f;

struct WideArgs {
    const uint16_t *q_ws;  // [B][Hq][T][512] normalised, roped q
    uint16_t *out;         // [B][T][Hq][512]
    unsigned *status;
    uint32_t T, pos0, q_heads, kv_heads, group, qt, window, n_qtiles, kv_rows;
    float scale_log2;
};

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    prefill_wide_kernel(const __grid_constant__ WideArgs a, const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    // the same padding in both CTAs (same kernel, same static layout), so mapa of a local address
    // names the same variable in the peer
    uint8_t *base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const uint32_t sb = smem_u32(base);
    auto bar = [&](int i) { return sb + kOffBar + 8u * i; };
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(base + kOffTmem);
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_rank(), peer = rank ^ 1u;

    // item: heaviest query tiles first across every (sequence, kv head)
    const uint32_t item = blockIdx.x >> 1;
    const uint32_t qt = a.n_qtiles - 1 - item / a.kv_rows, bkv = item % a.kv_rows;
    const uint32_t b = bkv / a.kv_heads, kvh = bkv % a.kv_heads;
    const uint32_t t0 = qt * a.qt;
    const uint32_t rows_valid = min(a.qt, a.T - t0);  // queries of this tile inside the call
    const uint32_t pos_first = a.pos0 + t0, pos_last = pos_first + rows_valid - 1;
    const uint32_t kv_lo = (a.window && pos_first + 1 > a.window) ? pos_first + 1 - a.window : 0;
    const uint32_t j0 = kv_lo / kKeys * kKeys;
    const uint32_t n_tiles = (pos_last - j0) / kKeys + 1;

    if (tid == 0) {
        prefetch_tensormap(&tk);
        prefetch_tensormap(&tv);
        for (int s = 0; s < kStages; ++s) {
            mbar_init(bar(kBarFull + s), 1);
            mbar_init(bar(kBarEmpty + s), 1);
        }
        mbar_init(bar(kBarQ), 4);
        for (int i = 0; i < kSBufs; ++i) {
            mbar_init(bar(kBarS + i), 1);
            mbar_init(bar(kBarP + i), 4);
        }
        for (int i = 0; i < kXBufs; ++i) mbar_init(bar(kBarX + i), 4);  // armed by the four softmax warps
        for (int i = 0; i < 2; ++i) mbar_init(bar(kBarO + i), 1);
        mbar_init(bar(kBarOFinal), 1);
        // the score buffers of tiles 0-3 armed for the four softmax warps before the peer can send
        for (uint32_t jj = 0; jj < kXBufs && jj < n_tiles; ++jj)
            for (int w = 0; w < 4; ++w) mbar_arrive_expect_tx(bar(kBarX + jj), 32 * 128);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_holder), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    cluster_sync();  // both CTAs' barriers exist before either arrives on the other's
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            const int32_t row = static_cast<int32_t>(b * a.kv_heads + kvh);
            uint32_t issued = 0;
            for (uint32_t j = 0; j < n_tiles; ++j) {
                const uint32_t s = j % kStages;
                if (j >= kStages && !mbar_wait(bar(kBarEmpty + s), ((j / kStages) - 1) & 1, a.status)) break;
                mbar_arrive_expect_tx(bar(kBarFull + s), kStageBytes);
                const int32_t key = static_cast<int32_t>(j0 + j * kKeys);
                const uint32_t dst = sb + kOffStages + s * kStageBytes;
                // {64-element chunk, key, chunk, kv row}: this CTA's four chunks of 32 keys
                tma_load_4d(dst, &tk, 0, key, static_cast<int32_t>(4 * rank), row, bar(kBarFull + s));
                tma_load_4d(dst + kTileBytes, &tv, 0, key, static_cast<int32_t>(4 * rank), row, bar(kBarFull + s));
                issued = j + 1;
            }
            // every copy lands before the block's shared memory can be released
            for (uint32_t j = issued > kStages ? issued - kStages : 0; j < issued; ++j)
                if (!mbar_wait(bar(kBarFull + j % kStages), (j / kStages) & 1, a.status)) break;
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idS = idesc_bf16_f32(kRows, kKeys, 0, 0);
            constexpr uint32_t idPV = idesc_bf16_f32(kRows, 256, 0, 1);
            const uint64_t k_desc = smem_desc_sw128(sb + kOffStages, 16, 1024);
            const uint64_t v_desc = smem_desc_sw128(sb + kOffStages + kTileBytes, kKvChunk, 1024);
            bool alive = mbar_wait(bar(kBarQ), 0, a.status);
            tc_fence_after();
            // S(j) goes two tiles ahead of PV(j - 2): the softmax finds S(j + 1) done when it starts
            // tile j, and the score buffer S(j) overwrites held P(j - 3), read by PV(j - 3) before
            for (uint32_t j = 0; j < n_tiles + 2 && alive; ++j) {
                if (j < n_tiles) {  // S(j) = Q K(j)^T over this CTA's 256 dims
                    const uint32_t s = j % kStages;
                    if (!mbar_wait(bar(kBarFull + s), (j / kStages) & 1, a.status)) {
                        alive = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t s_col = tmem + kColS + (j % kSBufs) * kKeys;
#pragma unroll
                    for (int k = 0; k < 4; ++k)
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks)  // 16-dim step: 8 Q columns, 32 bytes of a K row
                            tc_mma_ts(s_col, tmem + kColQ + (4 * k + ks) * 8,
                                      k_desc + ((s * kStageBytes + k * kKvChunk + ks * 32) >> 4), idS,
                                      (k | ks) ? 1u : 0u);
                    tc_commit(bar(kBarS + j % kSBufs));
                }
                if (j >= 2) {  // O += P(j-2) V(j-2)
                    const uint32_t jp = j - 2, sp = jp % kStages;
                    if (!mbar_wait(bar(kBarP + jp % kSBufs), (jp / kSBufs) & 1, a.status)) {
                        alive = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int ks = 0; ks < 2; ++ks)  // 16 keys: 8 P columns, 2 KB of the V tile
                        tc_mma_ts(tmem + kColO, tmem + kColS + (jp % kSBufs) * kKeys + ks * 8,
                                  v_desc + ((sp * kStageBytes + ks * 2048) >> 4), idPV, (jp | ks) ? 1u : 0u);
                    tc_commit(bar(kBarEmpty + sp));
                    tc_commit(bar(kBarO + (jp & 1)));
                }
            }
            // completes once every MMA issued above is done (also on a failed wait, so that the
            // TMEM is never released under a running MMA)
            tc_commit(bar(kBarOFinal));
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------ softmax + epilogue
        const uint32_t quad = warp - 4, r = quad * 32 + lane;  // row == TMEM lane
        const uint32_t lane_base = tmem + ((32u * quad) << 16);
        const uint32_t hh = r / a.qt, qq = r % a.qt;          // head of the group, query of the tile
        const uint32_t h = kvh * a.group + hh, t = t0 + qq;
        const bool row_ok = qq < rows_valid;
        const int pos = static_cast<int>(a.pos0 + t);
        bool alive = true;
        // Q: this CTA's 256 dims of the row into TMEM (zeros past the call's tokens)
        {
            const uint4 *src = reinterpret_cast<const uint4 *>(
                a.q_ws + ((static_cast<uint64_t>(b) * a.q_heads + h) * a.T + (row_ok ? t : t0)) * kD + 256 * rank);
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                uint32_t v[32];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint4 x = row_ok ? __ldg(src + 8 * c + i) : make_uint4(0u, 0u, 0u, 0u);
                    v[4 * i] = x.x;
                    v[4 * i + 1] = x.y;
                    v[4 * i + 2] = x.z;
                    v[4 * i + 3] = x.w;
                }
                tmem_st32(lane_base + kColQ + 32 * c, v);
            }
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kBarQ));
        }
        // score partials: row r of a tile's buffer holds 32 floats as eight 16-byte chunks, chunk c
        // at (c ^ (r & 7)) -- a warp's eight-lane phases hit distinct banks
        const uint32_t x_row = sb + kOffX + r * 128;
        const uint32_t x_peer = mapa(x_row, peer);
        const uint32_t swz = r & 7;
        // this CTA's scores of tile jj from TMEM
        auto load_s = [&](uint32_t jj, uint32_t(&v)[32]) {
            if (!__all_sync(0xffffffffu, mbar_wait(bar(kBarS + jj % kSBufs), (jj / kSBufs) & 1, a.status)))
                return false;
            tc_fence_after();
            tmem_ld32(lane_base + kColS + (jj % kSBufs) * kKeys, v);
            tc_wait_ld(v);
            return true;
        };
        // ... into the peer's buffer of tile jj by asynchronous stores that count their bytes on the
        // peer's barrier of that buffer (no fence on this side)
        auto send = [&](uint32_t jj, const uint32_t(&v)[32]) {
            const uint32_t xb = (jj % kXBufs) * kXBytes, xbar = mapa(bar(kBarX + jj % kXBufs), peer);
#pragma unroll
            for (int c = 0; c < 8; ++c)
                st_async_v4(x_peer + xb + 16 * (c ^ swz), v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3], xbar);
        };
        // A buffer's barrier completes a phase when this CTA's four warps have armed it (each for its
        // 32 rows' 4 KB) and the peer's 16 KB have landed.  A warp arms buffer j % 4 for tile j + 4
        // once it has read tile j (tiles 0-3 were armed at set-up), so no phase completes before the
        // slowest warp has read the buffer's last tile, and the peer's bytes for tile j + 4 -- sent
        // only after all of this CTA's partials of tile j + 2 arrived -- always find the buffer armed.
        auto arm = [&](uint32_t jj) {
            if (lane == 0 && jj < n_tiles) mbar_arrive_expect_tx(bar(kBarX + jj % kXBufs), 32 * 128);
        };
        float m_run = -INFINITY, l_sum = 0.f;
        uint32_t sv[32];
        alive = load_s(0, sv);
        if (alive) send(0, sv);
        // Tile j: tile j + 1's scores go to the peer first, so the exchange of the next tile overlaps
        // this tile's softmax.  The peer can then be up to three tiles ahead in its sends: four
        // buffers keep its writes off the buffer read here.
        for (uint32_t j = 0; j < n_tiles && alive; ++j) {
            uint32_t nv[32];
            if (j + 1 < n_tiles) {
                if (!load_s(j + 1, nv)) {
                    alive = false;
                    break;
                }
                send(j + 1, nv);
            }
            if (!__all_sync(0xffffffffu, mbar_wait_cluster(bar(kBarX + j % kXBufs), (j / kXBufs) & 1, a.status))) {
                alive = false;
                break;
            }
            float sc[32];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const float4 o = *reinterpret_cast<const float4 *>(base + kOffX + (j % kXBufs) * kXBytes + r * 128 +
                                                                   16 * (c ^ swz));
                sc[4 * c] = __uint_as_float(sv[4 * c]) + o.x;
                sc[4 * c + 1] = __uint_as_float(sv[4 * c + 1]) + o.y;
                sc[4 * c + 2] = __uint_as_float(sv[4 * c + 2]) + o.z;
                sc[4 * c + 3] = __uint_as_float(sv[4 * c + 3]) + o.w;
            }
            __syncwarp();  // every lane has read its row of the buffer
            arm(j + kXBufs);
#pragma unroll
            for (int k = 0; k < 32; ++k) sv[k] = nv[k];
            // masks: only tiles that cross the causal or window band
            const uint32_t key0 = j0 + j * kKeys;
            const bool need_mask = key0 + kKeys - 1 > pos_first || (a.window && key0 + a.window <= pos_last);
            if (need_mask) {
#pragma unroll
                for (int k = 0; k < 32; ++k) {
                    const int key = static_cast<int>(key0) + k;
                    const bool vis = key <= pos && (!a.window || key > pos - static_cast<int>(a.window));
                    sc[k] = vis ? sc[k] : -INFINITY;
                }
            }
            float mx = -INFINITY;
#pragma unroll
            for (int k = 0; k < 32; ++k) mx = fmaxf(mx, sc[k]);
            const float mt = mx * a.scale_log2;
            float alpha = 1.f;
            bool rescale = false;
            if (mt > m_run + kTau) {
                alpha = fast_exp2(m_run - mt);          // 0 when m_run = -inf
                rescale = m_run != -INFINITY;           // O holds only zeros while m_run = -inf
                m_run = mt;
            }
            l_sum *= alpha;
            if (__any_sync(0xffffffffu, rescale)) {
                // O rows of this warp scaled in TMEM once PV(j-1), the last one issued, is done
                const uint32_t jp = j - 1;
                if (!__all_sync(0xffffffffu, mbar_wait(bar(kBarO + (jp & 1)), (jp >> 1) & 1, a.status))) {
                    alive = false;
                    break;
                }
                tc_fence_after();
                const float f = rescale ? alpha : 1.f;
#pragma unroll 1
                for (int c = 0; c < 8; ++c) {
                    uint32_t ov[32];
                    tmem_ld32(lane_base + kColO + 32 * c, ov);
                    tc_wait_ld(ov);
#pragma unroll
                    for (int k = 0; k < 32; ++k) ov[k] = __float_as_uint(__uint_as_float(ov[k]) * f);
                    tmem_st32(lane_base + kColO + 32 * c, ov);
                }
                tc_wait_st();
            }
            const float neg_m = m_run == -INFINITY ? 0.f : -m_run;
            uint32_t pk[16];
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const float p0 = fast_exp2(fmaf(sc[2 * k], a.scale_log2, neg_m));
                const float p1 = fast_exp2(fmaf(sc[2 * k + 1], a.scale_log2, neg_m));
                l_sum += p0 + p1;
                pk[k] = pack_bf16(p0, p1);
            }
            tmem_st16(lane_base + kColS + (j % kSBufs) * kKeys, pk);
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kBarP + j % kSBufs));
        }
        // epilogue: O / l -> bf16, this CTA's 256 dims of the row
        if (alive && __all_sync(0xffffffffu, mbar_wait(bar(kBarOFinal), 0, a.status))) {
            tc_fence_after();
            const float inv = l_sum > 0.f ? 1.0f / l_sum : 0.f;
            uint4 *dst = reinterpret_cast<uint4 *>(
                a.out + ((static_cast<uint64_t>(b) * a.T + (row_ok ? t : t0)) * a.q_heads + h) * kD + 256 * rank);
#pragma unroll 1
            for (int c = 0; c < 8; ++c) {
                uint32_t ov[32];
                tmem_ld32(lane_base + kColO + 32 * c, ov);
                tc_wait_ld(ov);
                if (row_ok) {
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        dst[4 * c + i] = make_uint4(
                            pack_bf16(__uint_as_float(ov[8 * i]) * inv, __uint_as_float(ov[8 * i + 1]) * inv),
                            pack_bf16(__uint_as_float(ov[8 * i + 2]) * inv, __uint_as_float(ov[8 * i + 3]) * inv),
                            pack_bf16(__uint_as_float(ov[8 * i + 4]) * inv, __uint_as_float(ov[8 * i + 5]) * inv),
                            pack_bf16(__uint_as_float(ov[8 * i + 6]) * inv, __uint_as_float(ov[8 * i + 7]) * inv));
                }
            }
        }
    }

    // teardown: no MMA runs and neither CTA touches the other's shared memory any more
    __syncwarp();  // the single-lane roles rejoin their warps before the aligned cluster barrier
    if (warp == 1) mbar_wait(bar(kBarOFinal), 0, a.status);
    tc_fence_before();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace

bool prefill_wide_applies(const apex_attn_params *p) {
    if (!p || p->head_dim != static_cast<uint32_t>(kD) || p->kv_heads == 0) return false;
    const uint32_t g = p->q_heads / p->kv_heads;
    return g == 1 || g == 2 || g == 4 || g == 8;
}

int launch_prefill_wide_attend(const apex_attn_params *p, const void *workspace, const uint16_t *k_cache,
                               const uint16_t *v_cache, uint32_t capacity, uint32_t batch, uint32_t tokens,
                               uint32_t pos0, uint16_t *out, cudaStream_t s) {
    const uint64_t kv_len = static_cast<uint64_t>(pos0) + tokens;
    const uint64_t row = kD * 2ull;
    const uint64_t kv_rows = static_cast<uint64_t>(batch) * p->kv_heads;
    // caches [B*Hkv][capacity][512] as {64-element chunks, keys (cut at pos0 + T), 8 chunks, kv rows}:
    // one box = 32 keys x 4 chunks (one CTA's 256 dims), chunk-major
    CUtensorMap tk, tv;
    int rc = make_tensor_map_bf16_4d(&tk, k_cache, {64, kv_len, kD / 64, kv_rows}, {row, 128, row * capacity},
                                     {64, static_cast<uint32_t>(kKeys), 4, 1}, true);
    if (rc) return rc;
    rc = make_tensor_map_bf16_4d(&tv, v_cache, {64, kv_len, kD / 64, kv_rows}, {row, 128, row * capacity},
                                 {64, static_cast<uint32_t>(kKeys), 4, 1}, true);
    if (rc) return rc;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        rc = check_cuda(cudaFuncSetAttribute(prefill_wide_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kSmemBytes)),
                        "prefill (head_dim 512, tcgen05) smem attribute");
        if (rc) return rc;
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    WideArgs a{};
    a.q_ws = static_cast<const uint16_t *>(workspace);
    a.out = out;
    a.status = device_status_ptr();
    if (!a.status) return fail(APEX_ERR_CUDA, "prefill (head_dim 512): device status word unavailable");
    a.T = tokens;
    a.pos0 = pos0;
    a.q_heads = p->q_heads;
    a.kv_heads = p->kv_heads;
    a.group = p->q_heads / p->kv_heads;
    a.qt = kRows / a.group;
    a.window = p->window;
    a.n_qtiles = (tokens + a.qt - 1) / a.qt;
    a.kv_rows = static_cast<uint32_t>(kv_rows);
    a.scale_log2 = p->scale * kLog2e;
    const uint64_t items = static_cast<uint64_t>(a.n_qtiles) * kv_rows;
    if (2 * items > 0x7fffffffull) return fail(APEX_ERR_INVALID_ARGUMENT, "prefill (head_dim 512): problem too large");
    prefill_wide_kernel<<<static_cast<uint32_t>(2 * items), kThreads, kSmemBytes, s>>>(a, tk, tv);
    return check_cuda(cudaGetLastError(), "prefill (head_dim 512, tcgen05) launch");
}

}  // namespace apex
