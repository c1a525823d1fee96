// prefill_tc.cu -- fused causal (optionally sliding-window) prefill on tcgen05 tensor cores.
//
// Reference semantics (docs/B6_3_attention.md:444-454 and :296-343): q and k are RMS-normed
// with their bf16 weights and roped at position pos0 + t, v optionally weightless-normed; K and
// V are appended to the cache [kv_heads][capacity][hd] at pos0 (the reference's f32 cache
// becomes bf16, its planned format, docs/B6_3_attention.md:99-102); then for every query
// o = softmax(scale * q K^T) V over keys p - window < j <= p (or j <= p), GQA map h/(Hq/Hkv).
//
// Two launches per call:
//  1. prep: one warp per (sequence, token): the token's RoPE cos/sin are computed once and
//     reused for its Hq + Hkv rows; every row is one 16-byte load and store per lane.  q goes
//     to a head-major workspace [B][Hq][T][256] (one 3-D TMA box per 128-query tile), k and v
//     to the caches.  It also zeroes the attention kernel's scheduler counters.
//  2. attention: a persistent kernel, one CTA per SM, pulling work items (128-query tile x q
//     head) from an atomic counter, heaviest tiles first (items are ordered by query tile,
//     last first).  Per CTA, 12 warps:
//       warp 0  scheduler + TMA producer: K and V as 64-key tiles (32 KB each) through a
//               7-slot ring; 3-D tensor maps end at pos0+T, so keys past the valid cache read
//               as zeros, never as uninitialised memory.
//       warp 1  TMEM owner (512 columns) and tcgen05.mma issuer (one thread), both products in
//               the A-from-TMEM form of .kind::f16, so shared memory only feeds B:
//               S_t = Q K_t^T (M=128, N=64, K=16 x 16), Q in TMEM, K K-major in smem;
//               O += P_t V_t  (M=128, N=256, K=16 x 4), P in TMEM, V MN-major in smem.
//               S_{t+1} is issued before PV_t, and the next item's S MMAs run while the
//               current item's epilogue drains O.
//       warps 4-11  two warpgroups per 128 query rows (TMEM lane = row; half 0 takes keys
//               0-31 of each tile and dims 0-127, half 1 keys 32-63 and dims 128-255): they put
//               each item's normalised q into TMEM, run the online softmax (log2 domain, mask
//               only on tiles crossing the causal/window band, lazy rescaling of O when a row
//               max grows by more than 2^8, row max and sum exchanged between the halves), store
//               P as bf16 pairs over their S columns, and write the epilogue.
//     TMEM: O = columns [0, 256), Q = [256, 384), S0/P0 = [384, 448), S1/P1 = [448, 512).
#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "row256.cuh"

namespace apex {
namespace {

constexpr int kD = 256;
constexpr int kBM = 128;                             // queries per item
constexpr int kBN = 64;                              // keys per tile (one ring slot of K, one of V)
constexpr int kSlots = 7;
constexpr uint32_t kSlotChunk = kBN * 128;           // 64 dims x 64 keys, 128 B per key row
constexpr uint32_t kSlotBytes = kBN * kD * 2;        // 32768
constexpr uint32_t kOffSlots = 0;
constexpr uint32_t kOffBar = kOffSlots + kSlots * kSlotBytes;
constexpr uint32_t kNumBars = 40;
constexpr uint32_t kOffItems = kOffBar + 8 * kNumBars;
constexpr uint32_t kItemRing = 8;
constexpr uint32_t kOffRed = kOffItems + 4 * kItemRing;  // float [2 parity][2 half][128]
constexpr uint32_t kOffTmem = kOffRed + 2 * 2 * 128 * 4;
constexpr uint32_t kSmemBytes = kOffTmem + 16;  // the dynamic shared memory base is 1024-aligned
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 0, kColQ = 256, kColS = 384;  // O f32 [0,256), Q bf16 pairs [256,384), S 2 x 64
constexpr int kThreads = 384;                        // 12 warps: 0 TMA, 1 MMA, 4-11 softmax
constexpr float kTau = 8.0f;                         // lazy-rescale threshold (log2 units)
constexpr float kLog2e = 1.4426950408889634f;

static_assert(kSmemBytes <= 232448, "shared memory budget");

// barrier indices (8 bytes each at kOffBar)
constexpr int kBarQFull = 0, kBarQEmpty = 1, kBarFull = 2, kBarEmpty = kBarFull + kSlots,
              kBarS = kBarEmpty + kSlots, kBarP = kBarS + 2, kBarO = kBarP + 2, kBarOFree = kBarO + 2,
              kBarItem = kBarOFree + 1, kBarRed = kBarItem + kItemRing;
static_assert(kBarRed + 2 <= kNumBars, "barrier budget");

struct PrefillArgs {
    uint16_t *out;        // [B][T][Hq][D]
    const uint16_t *q;    // normalised q [B][Hq][T][D] (the workspace)
    unsigned *status;     // device status word
    unsigned *sched;      // [0] next item, [1] CTAs done (zeroed by the prep kernel)
    uint32_t batch, T, pos0, q_heads, kv_heads, window, n_qtiles, n_items;
    float scale_log2;
};

struct Item {
    uint32_t b, h, kvh, t0, rows_valid, pos_first, pos_last, j_start, n_tiles;
};

__device__ __forceinline__ Item item_geometry(uint32_t idx, const PrefillArgs &a) {
    Item it;
    const uint32_t bh_count = a.batch * a.q_heads;
    const uint32_t qt = a.n_qtiles - 1 - idx / bh_count;  // last query tiles (most keys) first
    const uint32_t bh = idx % bh_count;
    it.b = bh / a.q_heads;
    it.h = bh % a.q_heads;
    it.kvh = it.h / (a.q_heads / a.kv_heads);
    it.t0 = qt * kBM;
    it.rows_valid = min(static_cast<uint32_t>(kBM), a.T - it.t0);
    it.pos_first = a.pos0 + it.t0;
    it.pos_last = it.pos_first + it.rows_valid - 1;
    const uint32_t kv_lo = (a.window && it.pos_first + 1 > a.window) ? it.pos_first + 1 - a.window : 0;
    it.j_start = (kv_lo / kBN) * kBN;
    it.n_tiles = (it.pos_last - it.j_start) / kBN + 1;
    return it;
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                      const PrefillArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *base = smem_raw;
    const uint32_t sb = smem_u32(base);
    if (sb & 1023u) {  // the swizzled tiles need 1024-byte alignment; never expected to fire
        if (threadIdx.x == 0) atomicOr(a.status, kStatusTimeout);
        return;
    }
    auto bar = [&](int i) { return sb + kOffBar + 8u * i; };
    volatile int *items = reinterpret_cast<volatile int *>(base + kOffItems);
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(base + kOffTmem);

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid == 0) {
        mbar_init(bar(kBarQFull), 2 * kBM);   // Q in TMEM, written by the softmax threads
        mbar_init(bar(kBarQEmpty), 1);        // the item's last S MMA done with Q
        for (int i = 0; i < kSlots; ++i) {
            mbar_init(bar(kBarFull + i), 1);
            mbar_init(bar(kBarEmpty + i), 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar(kBarS + i), 1);
            mbar_init(bar(kBarP + i), 2 * kBM);
            mbar_init(bar(kBarRed + i), 2 * kBM);
        }
        mbar_init(bar(kBarO + 0), 1);
        mbar_init(bar(kBarO + 1), 1);
        mbar_init(bar(kBarOFree), 2 * kBM);
        for (uint32_t i = 0; i < kItemRing; ++i) mbar_init(bar(kBarItem + i), 1);
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
        // ------------------------------------------------------------ scheduler + TMA producer
        if (lane == 0) {
            prefetch_tensormap(&tm_k);
            prefetch_tensormap(&tm_v);
            uint32_t kv_n = 0;
            bool alive = true;
            for (uint32_t it = 0;; ++it) {
                int idx = static_cast<int>(atomicAdd(a.sched, 1u));
                if (static_cast<uint32_t>(idx) >= a.n_items || !alive) idx = -1;
                items[it % kItemRing] = idx;
                mbar_arrive(bar(kBarItem + it % kItemRing));
                if (idx < 0) break;
                const Item g = item_geometry(static_cast<uint32_t>(idx), a);
                for (uint32_t j = 0; j < g.n_tiles && alive; ++j) {
                    const uint32_t key0 = g.j_start + j * kBN;
                    for (int which = 0; which < 2; ++which, ++kv_n) {  // K then V
                        const uint32_t slot = kv_n % kSlots;
                        if (kv_n >= kSlots &&
                            !mbar_wait(bar(kBarEmpty + slot), ((kv_n / kSlots) - 1) & 1, a.status)) {
                            alive = false;
                            break;
                        }
                        mbar_arrive_expect_tx(bar(kBarFull + slot), kSlotBytes);
                        const uint32_t dst = sb + kOffSlots + slot * kSlotBytes;
                        const CUtensorMap *map = which == 0 ? &tm_k : &tm_v;
                        for (int c = 0; c < 4; ++c)
                            tma_load_3d(dst + c * kSlotChunk, map, c * 64, static_cast<int32_t>(key0),
                                        static_cast<int32_t>(g.b * a.kv_heads + g.kvh), bar(kBarFull + slot));
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idS = idesc_bf16_f32(kBM, kBN, 0, 0);
            constexpr uint32_t idPV = idesc_bf16_f32(kBM, kD, 0, 1);
            uint32_t gt = 0, kv_n = 0;
            bool alive = true;
            auto wait_full = [&](uint32_t n) { return mbar_wait(bar(kBarFull + n % kSlots), (n / kSlots) & 1, a.status); };
            // O += P_t V_t for global tile t; V at ring position nv; P in TMEM over S buffer t%2
            auto issue_pv = [&](uint32_t t, uint32_t nv, bool first, uint32_t it) {
                if (!alive) return;
                alive = mbar_wait(bar(kBarP + (t & 1)), (t >> 1) & 1, a.status);
                if (alive && first && it >= 1) alive = mbar_wait(bar(kBarOFree), (it - 1) & 1, a.status);
                alive = alive && wait_full(nv);
                if (!alive) return;
                tc_fence_after();
                const uint32_t p_col = tmem + kColS + (t & 1) * kBN;
                const uint32_t vslot = nv % kSlots;
#pragma unroll
                for (int ks = 0; ks < kBN / 16; ++ks) {
                    const uint64_t bd =
                        smem_desc_sw128(sb + kOffSlots + vslot * kSlotBytes + ks * 2048, kSlotChunk, 1024);
                    tc_mma_ts(tmem + kColO, p_col + ks * 8, bd, idPV, (!first || ks > 0) ? 1u : 0u);
                }
                tc_commit(bar(kBarO + (t & 1)));
                tc_commit(bar(kBarEmpty + vslot));
            };
            for (uint32_t it = 0; alive; ++it) {
                if (!mbar_wait(bar(kBarItem + it % kItemRing), (it / kItemRing) & 1, a.status)) break;
                const int idx = items[it % kItemRing];
                if (idx < 0) break;
                if (!mbar_wait(bar(kBarQFull), it & 1, a.status)) break;  // Q of this item in TMEM
                tc_fence_after();
                const Item g = item_geometry(static_cast<uint32_t>(idx), a);
                for (uint32_t j = 0; j < g.n_tiles && alive; ++j) {
                    const uint32_t t = gt + j, nk = kv_n + 2 * j;
                    alive = wait_full(nk);
                    if (!alive) break;
                    tc_fence_after();
                    const uint32_t s_col = tmem + kColS + (t & 1) * kBN;
                    const uint32_t kslot = nk % kSlots;
#pragma unroll
                    for (int ks = 0; ks < kD / 16; ++ks) {
                        const uint64_t bd = smem_desc_sw128(
                            sb + kOffSlots + kslot * kSlotBytes + (ks / 4) * kSlotChunk + (ks % 4) * 32, 16, 1024);
                        tc_mma_ts(s_col, tmem + kColQ + ks * 8, bd, idS, ks > 0 ? 1u : 0u);
                    }
                    tc_commit(bar(kBarS + (t & 1)));
                    tc_commit(bar(kBarEmpty + kslot));
                    if (j + 1 == g.n_tiles) tc_commit(bar(kBarQEmpty));  // Q is free once these finish
                    if (j >= 1) issue_pv(t - 1, kv_n + 2 * (j - 1) + 1, j - 1 == 0, it);
                }
                issue_pv(gt + g.n_tiles - 1, kv_n + 2 * (g.n_tiles - 1) + 1, g.n_tiles == 1, it);
                gt += g.n_tiles;
                kv_n += 2 * g.n_tiles;
            }
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------ Q loader, softmax, epilogue
        // Two warpgroups share each query row: half 0 owns S columns [0, 32) of each 64-key tile,
        // q/O dims [0, 128); half 1 owns S columns [32, 64), dims [128, 256).  The row max (every
        // tile) and the row sum (every item) are exchanged through shared memory with an
        // mbarrier handshake, so every wait stays bounded.
        const uint32_t half = (warp - 4) >> 2, quad = warp & 3;
        const uint32_t r = quad * 32 + lane;                  // query row == TMEM lane
        const uint32_t lane_base = tmem + ((32u * quad) << 16);
        float *red = reinterpret_cast<float *>(base + kOffRed);  // [2 parity][2 half][128]
        uint32_t gt = 0, xchg = 0;
        bool alive = true;
        // Wait for PV of global tile t.  o_done is a ring of two barriers indexed by tile parity:
        // when this runs (after S(t+1) or S(t) completed), PV(t-2) is already complete (it was
        // issued before those S MMAs) and PV(t+2) cannot have started, so the parity is
        // unambiguous without observing every phase.
        auto wait_pv = [&](uint32_t t) {
            alive = alive && __all_sync(0xffffffffu, mbar_wait(bar(kBarO + (t & 1)), (t >> 1) & 1, a.status));
        };
        // The handshake also orders TMEM: each half has finished reading its S columns before it
        // arrives, and half 1 overwrites some of half 0's S columns with P only after the wait.
        auto exchange = [&](float mine, float &theirs) {
            const uint32_t slot = xchg & 1;
            red[(slot * 2 + half) * kBM + r] = mine;
            tc_fence_before();
            mbar_arrive(bar(kBarRed + slot));
            const bool ok = __all_sync(0xffffffffu, mbar_wait(bar(kBarRed + slot), (xchg >> 1) & 1, a.status));
            tc_fence_after();
            theirs = red[(slot * 2 + (half ^ 1)) * kBM + r];
            ++xchg;
            return ok;
        };
        // This row's q (this half's 128 dims) -> TMEM columns [kColQ + 64*half, +64) as bf16 pairs.
        auto load_q = [&](const Item &g, uint32_t it) {
            if (it >= 1 && !__all_sync(0xffffffffu, mbar_wait(bar(kBarQEmpty), (it - 1) & 1, a.status))) {
                alive = false;
                return;
            }
            const uint32_t t = g.t0 + r;
            const uint16_t *src = a.q + ((static_cast<uint64_t>(g.b) * a.q_heads + g.h) * a.T + t) * kD + half * 128;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t w[32];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const uint4 v = r < g.rows_valid ? *reinterpret_cast<const uint4 *>(src + c * 64 + u * 8)
                                                     : make_uint4(0u, 0u, 0u, 0u);
                    w[4 * u + 0] = v.x;
                    w[4 * u + 1] = v.y;
                    w[4 * u + 2] = v.z;
                    w[4 * u + 3] = v.w;
                }
                tmem_st32(lane_base + kColQ + half * 64 + c * 32, w);
            }
            tc_wait_st();
            tc_fence_before();
            mbar_arrive(bar(kBarQFull));
        };
        int idx = -1;
        Item g{};
        // item 0's q
        if (__all_sync(0xffffffffu, mbar_wait(bar(kBarItem), 0, a.status))) {
            idx = items[0];
            if (idx >= 0) {
                g = item_geometry(static_cast<uint32_t>(idx), a);
                load_q(g, 0);
            }
        } else {
            alive = false;
        }
        for (uint32_t it = 0; alive && idx >= 0; ++it) {
            const uint32_t t = g.t0 + r;
            const int pos = static_cast<int>(a.pos0 + t);
            float m_run = -INFINITY, l_part = 0.f;
            for (uint32_t j = 0; j < g.n_tiles && alive; ++j) {
                const uint32_t tt = gt + j;
                bool ok = __all_sync(0xffffffffu, mbar_wait(bar(kBarS + (tt & 1)), (tt >> 1) & 1, a.status));
                tc_fence_after();
                uint32_t sv[32];
                const uint32_t s_addr = lane_base + kColS + (tt & 1) * kBN + half * 32;
                if (ok) {
                    tmem_ld32(s_addr, sv);
                    tc_wait_ld();
                }
                const uint32_t tile0 = g.j_start + j * kBN;
                const bool need_mask = (tile0 + kBN - 1 > g.pos_first) || (a.window && tile0 + a.window <= g.pos_last);
                if (need_mask) {
                    // visible keys of this row relative to this half's first key: [lo, hi]
                    const int key0 = static_cast<int>(tile0 + half * 32);
                    const int hi = pos - key0;
                    const int lo = a.window ? pos + 1 - static_cast<int>(a.window) - key0 : -(1 << 30);
#pragma unroll
                    for (int k = 0; k < 32; ++k)
                        if (k > hi || k < lo) sv[k] = 0xff800000u;  // -inf
                }
                float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                for (int k = 0; k < 32; ++k) mx[k & 3] = fmaxf(mx[k & 3], __uint_as_float(sv[k]));
                const float mine = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
                float other;
                ok = exchange(mine, other) && ok;
                if (!ok) {
                    alive = false;
                    break;
                }
                const float mt = fmaxf(mine, other) * a.scale_log2;
                float alpha = 1.f;
                bool rescale = false;
                if (mt > m_run + kTau) {
                    alpha = fast_exp2(m_run - mt);  // 0 when m_run = -inf
                    rescale = j > 0;
                    m_run = mt;
                }
                const float neg_m = m_run == -INFINITY ? 0.f : -m_run;
                float sum[4] = {0.f, 0.f, 0.f, 0.f};
                uint32_t packed[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float p0 = fast_exp2(fmaf(__uint_as_float(sv[2 * i]), a.scale_log2, neg_m));
                    const float p1 = fast_exp2(fmaf(__uint_as_float(sv[2 * i + 1]), a.scale_log2, neg_m));
                    sum[i & 3] += p0 + p1;
                    packed[i] = pack_bf16(p0, p1);
                }
                l_part = l_part * alpha + ((sum[0] + sum[1]) + (sum[2] + sum[3]));
                // tcgen05.ld/st are warp-collective: the whole warp rescales if any row must, after
                // PV of the previous tile has finished accumulating into O.
                if (__any_sync(0xffffffffu, rescale)) {
                    wait_pv(tt - 1);
                    if (!alive) break;
                    tc_fence_after();
                    const float f = rescale ? alpha : 1.0f;
#pragma unroll 1
                    for (int c = 0; c < 4; ++c) {
                        uint32_t o[32];
                        const uint32_t oa = lane_base + kColO + half * 128 + c * 32;
                        tmem_ld32(oa, o);
                        tc_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
                        tmem_st32(oa, o);
                    }
                }
                // P (bf16 pairs): this half's 32 keys -> columns [16*half, 16*half + 16) of the S buffer
                tmem_st16(lane_base + kColS + (tt & 1) * kBN + half * 16, packed);
                tc_wait_st();
                tc_fence_before();
                mbar_arrive(bar(kBarP + (tt & 1)));
            }
            if (!alive) break;
            // the next item's q goes into TMEM now, so its S MMAs overlap this epilogue
            const Item cur = g;
            const uint32_t cur_n = g.n_tiles;
            if (!__all_sync(0xffffffffu, mbar_wait(bar(kBarItem + (it + 1) % kItemRing), ((it + 1) / kItemRing) & 1,
                                                   a.status))) {
                alive = false;
                break;
            }
            idx = items[(it + 1) % kItemRing];
            if (idx >= 0) {
                g = item_geometry(static_cast<uint32_t>(idx), a);
                load_q(g, it + 1);
                if (!alive) break;
            }
            // epilogue: O / l -> bf16 out[b][t][h][half*128 ...]
            wait_pv(gt + cur_n - 1);
            float l_other;
            if (!exchange(l_part, l_other) || !alive) {
                alive = false;
                break;
            }
            tc_fence_after();
            const float l_run = l_part + l_other;
            const float inv_l = l_run > 0.f ? 1.0f / l_run : 0.f;
            const bool row_valid = r < cur.rows_valid;
            uint16_t *orow =
                a.out + ((static_cast<uint64_t>(cur.b) * a.T + t) * a.q_heads + cur.h) * kD + half * 128;
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                uint32_t o[32];
                tmem_ld32(lane_base + kColO + half * 128 + c * 32, o);
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
            tc_fence_before();
            mbar_arrive(bar(kBarOFree));
            gt += cur_n;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    if (tid == 0) {
        // the last CTA to finish resets the scheduler for the next launch
        __threadfence();
        if (atomicAdd(a.sched + 1, 1u) == gridDim.x - 1) {
            a.sched[0] = 0;
            a.sched[1] = 0;
        }
    }
}

// ---------------------------------------------------------------- prep: norm + rope + append
struct PrepArgs {
    const uint16_t *q_raw, *k_raw, *v_raw, *q_w, *k_w;
    uint16_t *q_ws, *k_cache, *v_cache;
    unsigned *sched;
    uint32_t B, T, pos0, q_heads, kv_heads, capacity, rope_pairs, qk_norm, v_norm;
    float eps;
    RopeTable rope;
};

// RMSNorm (optional, weight in registers) + RoPE with this lane's precomputed cos/sin of one
// 256-wide row held 8 dims per lane; pairs (i, i+128) meet across lanes l and l^16.
__device__ __forceinline__ void norm_rope_cs(float (&x)[8], uint32_t lane, bool norm, const float (&w)[8],
                                             float eps, bool rope, uint32_t rope_pairs, const float (&cs)[8],
                                             const float (&sn)[8]) {
    if (norm) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += x[e] * x[e];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = 1.0f / sqrtf(ss / static_cast<float>(kD) + eps);
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = x[e] * inv * w[e];
    }
    if (rope) {
        const bool low = lane < 16;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float other = __shfl_xor_sync(0xffffffffu, x[e], 16);
            if (8 * (lane & 15) + e < rope_pairs)
                x[e] = low ? (x[e] * cs[e] - other * sn[e]) : (other * sn[e] + x[e] * cs[e]);
        }
    }
}

// Work unit = (position, group): groups [0, nqg) are 8 q heads each, groups [nqg, nqg + nkg)
// are 4 kv heads each (k and v); a warp issues all loads of its unit before any math, so one
// HBM round trip covers 8 rows and many units are in flight per SM.
__global__ void __launch_bounds__(256) prefill_prep_kernel(const __grid_constant__ PrepArgs a) {
    const uint32_t lane = threadIdx.x & 31;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        a.sched[0] = 0;
        a.sched[1] = 0;
    }
    const uint32_t nqg = (a.q_heads + 7) / 8, nkg = (a.kv_heads + 3) / 4, groups = nqg + nkg;
    const uint64_t units = static_cast<uint64_t>(a.B) * a.T * groups;
    const uint64_t warps = static_cast<uint64_t>(gridDim.x) * (blockDim.x >> 5);
    for (uint64_t u = static_cast<uint64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); u < units;
         u += warps) {
        const uint64_t bt = u / groups;
        const uint32_t grp = static_cast<uint32_t>(u % groups);
        const uint32_t b = static_cast<uint32_t>(bt / a.T), t = static_cast<uint32_t>(bt % a.T);
        const bool is_q = grp < nqg;
        const uint32_t h0 = is_q ? grp * 8 : (grp - nqg) * 4;
        const uint32_t n = is_q ? min(8u, a.q_heads - h0) : min(4u, a.kv_heads - h0);
        uint4 raw[8];
        if (is_q) {
            const uint16_t *src = a.q_raw + (bt * a.q_heads + h0) * kD + 8 * lane;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (static_cast<uint32_t>(i) < n) raw[i] = *reinterpret_cast<const uint4 *>(src + i * kD);
        } else {
            const uint16_t *ks = a.k_raw + (bt * a.kv_heads + h0) * kD + 8 * lane;
            const uint16_t *vs = a.v_raw + (bt * a.kv_heads + h0) * kD + 8 * lane;
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (static_cast<uint32_t>(i) < n) {
                    raw[i] = *reinterpret_cast<const uint4 *>(ks + i * kD);
                    raw[4 + i] = *reinterpret_cast<const uint4 *>(vs + i * kD);
                }
        }
        const float pos = static_cast<float>(a.pos0 + t);
        float cs[8], sn[8], w[8], ones[8];
        const uint16_t *wsrc = is_q ? a.q_w : a.k_w;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const uint32_t i = 8 * (lane & 15) + e;
            if (i < a.rope_pairs) sincos_angle(pos * a.rope.inv_freq[i], sn[e], cs[e]);
            else cs[e] = 1.f, sn[e] = 0.f;
            w[e] = wsrc ? __uint_as_float(static_cast<uint32_t>(wsrc[8 * lane + e]) << 16) : 1.0f;
            ones[e] = 1.0f;
        }
        if (is_q) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if (static_cast<uint32_t>(i) >= n) break;
                float x[8];
                unpack8(raw[i], x);
                norm_rope_cs(x, lane, a.qk_norm, w, a.eps, a.rope_pairs != 0, a.rope_pairs, cs, sn);
                uint16_t *dst = a.q_ws + ((static_cast<uint64_t>(b) * a.q_heads + h0 + i) * a.T + t) * kD;
                *reinterpret_cast<uint4 *>(dst + 8 * lane) = pack8(x);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                if (static_cast<uint32_t>(i) >= n) break;
                const uint64_t off = ((static_cast<uint64_t>(b) * a.kv_heads + h0 + i) * a.capacity + a.pos0 + t) * kD;
                float x[8], y[8];
                unpack8(raw[i], x);
                unpack8(raw[4 + i], y);
                norm_rope_cs(x, lane, a.qk_norm, w, a.eps, a.rope_pairs != 0, a.rope_pairs, cs, sn);
                norm_rope_cs(y, lane, a.v_norm, ones, a.eps, false, 0, cs, sn);
                *reinterpret_cast<uint4 *>(a.k_cache + off + 8 * lane) = pack8(x);
                *reinterpret_cast<uint4 *>(a.v_cache + off + 8 * lane) = pack8(y);
            }
        }
    }
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

size_t q_ws_bytes(uint32_t batch, uint32_t tokens, uint32_t q_heads) {
    return static_cast<size_t>(batch) * tokens * q_heads * kD * 2;
}

size_t ws_bytes(uint32_t batch, uint32_t tokens, uint32_t q_heads) {
    return align256(q_ws_bytes(batch, tokens, q_heads)) + 256;  // + scheduler counters
}

unsigned *sched_ptr(void *workspace, uint32_t batch, uint32_t tokens, uint32_t q_heads) {
    return reinterpret_cast<unsigned *>(static_cast<uint8_t *>(workspace) +
                                        align256(q_ws_bytes(batch, tokens, q_heads)));
}

int validate_prefill(const apex_attn_params *p, uint32_t capacity, uint32_t batch, uint32_t tokens,
                     uint32_t pos0, std::initializer_list<const void *> tensors, void *workspace,
                     size_t workspace_bytes, const char *name) {
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
    const uint64_t items = static_cast<uint64_t>(batch) * p->q_heads * ((tokens + kBM - 1) / kBM);
    if (items > 0x7fffffffull) return fail(APEX_ERR_INVALID_ARGUMENT, n + ": problem too large for one launch");
    const size_t need = ws_bytes(batch, tokens, p->q_heads);
    if (!workspace || workspace_bytes < need)
        return fail(APEX_ERR_WORKSPACE, n + ": workspace of " + std::to_string(need) + " bytes required");
    if (!aligned16(workspace)) return fail(APEX_ERR_INVALID_ARGUMENT, n + ": tensors must be 16-byte aligned");
    return APEX_OK;
}

int launch_prep(const apex_attn_params *p, const uint16_t *q_raw, const uint16_t *k_raw, const uint16_t *v_raw,
                const uint16_t *q_w, const uint16_t *k_w, uint16_t *k_cache, uint16_t *v_cache,
                uint32_t capacity, uint32_t batch, uint32_t tokens, uint32_t pos0, void *workspace,
                cudaStream_t s) {
    PrepArgs pa{};
    pa.q_raw = q_raw; pa.k_raw = k_raw; pa.v_raw = v_raw; pa.q_w = q_w; pa.k_w = k_w;
    pa.q_ws = static_cast<uint16_t *>(workspace); pa.k_cache = k_cache; pa.v_cache = v_cache;
    pa.sched = sched_ptr(workspace, batch, tokens, p->q_heads);
    pa.B = batch; pa.T = tokens; pa.pos0 = pos0; pa.q_heads = p->q_heads; pa.kv_heads = p->kv_heads;
    pa.capacity = capacity; pa.rope_pairs = p->rope_pairs; pa.qk_norm = p->qk_norm; pa.v_norm = p->v_norm;
    pa.eps = p->eps;
    rope_table(pa.rope.inv_freq, p->rope_pairs, kD, p->rope_base);
    const uint64_t units = static_cast<uint64_t>(batch) * tokens * ((p->q_heads + 7) / 8 + (p->kv_heads + 3) / 4);
    const uint32_t grid = static_cast<uint32_t>(std::max<uint64_t>(1, std::min<uint64_t>((units + 7) / 8, 32ull * sm_count())));
    prefill_prep_kernel<<<grid, 256, 0, s>>>(pa);
    return check_cuda(cudaGetLastError(), "prefill prep launch");
}

int launch_attend(const apex_attn_params *p, void *workspace, const uint16_t *k_cache, const uint16_t *v_cache,
                  uint32_t capacity, uint32_t batch, uint32_t tokens, uint32_t pos0, uint16_t *out,
                  cudaStream_t s) {
    CUtensorMap tk, tv;
    const uint64_t kv_len = static_cast<uint64_t>(pos0) + tokens;
    int rc = make_tensor_map_bf16_3d(&tk, k_cache, kD, kv_len, static_cast<uint64_t>(batch) * p->kv_heads, kD * 2ull,
                                     static_cast<uint64_t>(capacity) * kD * 2, 64, kBN);
    if (rc) return rc;
    rc = make_tensor_map_bf16_3d(&tv, v_cache, kD, kv_len, static_cast<uint64_t>(batch) * p->kv_heads, kD * 2ull,
                                 static_cast<uint64_t>(capacity) * kD * 2, 64, kBN);
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
    PrefillArgs fa{};
    fa.out = out;
    fa.q = static_cast<const uint16_t *>(workspace);
    fa.status = device_status_ptr();
    if (!fa.status) return fail(APEX_ERR_CUDA, "prefill: device status word unavailable");
    fa.sched = sched_ptr(workspace, batch, tokens, p->q_heads);
    fa.batch = batch; fa.T = tokens; fa.pos0 = pos0; fa.q_heads = p->q_heads; fa.kv_heads = p->kv_heads;
    fa.window = p->window;
    fa.n_qtiles = (tokens + kBM - 1) / kBM;
    fa.n_items = batch * p->q_heads * fa.n_qtiles;
    fa.scale_log2 = p->scale * kLog2e;
    const uint32_t grid = std::min<uint32_t>(fa.n_items, static_cast<uint32_t>(sm_count()));
    prefill_tc_kernel<<<grid, kThreads, kSmemBytes, s>>>(tk, tv, fa);
    return check_cuda(cudaGetLastError(), "prefill attention launch");
}

}  // namespace
}  // namespace apex

extern "C" size_t apex_attn_prefill_workspace_bytes(const apex_attn_params *p, uint32_t batch,
                                                    uint32_t tokens) {
    if (!p) return 0;
    return apex::ws_bytes(batch, tokens, p->q_heads);
}

extern "C" int apex_attn_prefill_prep_bf16(const apex_attn_params *p, const uint16_t *q_raw,
                                           const uint16_t *k_raw, const uint16_t *v_raw,
                                           const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                                           uint16_t *k_cache, uint16_t *v_cache, uint32_t capacity,
                                           uint32_t batch, uint32_t tokens, uint32_t pos0,
                                           void *workspace, size_t workspace_bytes, void *stream) {
    using namespace apex;
    int rc = validate_prefill(p, capacity, batch, tokens, pos0, {q_raw, k_raw, v_raw, k_cache, v_cache}, workspace,
                              workspace_bytes, "apex_attn_prefill_prep_bf16");
    if (rc || batch == 0 || tokens == 0) return rc ? rc : ok();
    rc = launch_prep(p, q_raw, k_raw, v_raw, q_norm_w, k_norm_w, k_cache, v_cache, capacity, batch, tokens, pos0,
                     workspace, static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

extern "C" int apex_attn_prefill_attend_bf16(const apex_attn_params *p, void *workspace,
                                             size_t workspace_bytes, const uint16_t *k_cache,
                                             const uint16_t *v_cache, uint32_t capacity,
                                             uint32_t batch, uint32_t tokens, uint32_t pos0,
                                             uint16_t *out, void *stream) {
    using namespace apex;
    int rc = validate_prefill(p, capacity, batch, tokens, pos0, {k_cache, v_cache, out}, workspace, workspace_bytes,
                              "apex_attn_prefill_attend_bf16");
    if (rc || batch == 0 || tokens == 0) return rc ? rc : ok();
    rc = launch_attend(p, workspace, k_cache, v_cache, capacity, batch, tokens, pos0, out,
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
                              workspace, workspace_bytes, "apex_attn_prefill_bf16");
    if (rc || batch == 0 || tokens == 0) return rc ? rc : ok();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    rc = launch_prep(p, q_raw, k_raw, v_raw, q_norm_w, k_norm_w, k_cache, v_cache, capacity, batch, tokens, pos0,
                     workspace, s);
    if (rc) return rc;
    rc = launch_attend(p, workspace, k_cache, v_cache, capacity, batch, tokens, pos0, out, s);
    return rc ? rc : ok();
}
