// prefill_tc.cu -- fused causal (optionally sliding-window) prefill on tcgen05 tensor cores.
//
// Reference semantics (docs/B6_3_attention.md:444-454 and :296-343): q and k are RMS-normed
// with their bf16 weights and roped at position pos0 + t, v optionally weightless-normed; K and
// V are appended to the cache [kv_heads][capacity][hd] at pos0 (the reference's f32 cache
// becomes bf16, its planned format, docs/B6_3_attention.md:99-102); then for every query
// o = softmax(scale * q K^T) V over keys p - window < j <= p (or j <= p), GQA map h/(Hq/Hkv).
//
// Two launches per call:
//  1. prep: a persistent grid (two blocks per SM) streams each token's q, k and v rows into a
//     4-stage shared-memory ring with 1-D TMA bulk copies (one producer warp, which also writes
//     the token's RoPE cos/sin); eight consumer warps norm, rope and store the rows, one 16-byte
//     load and store per lane per row.  q goes to a head-major workspace [B][Hq][T][256] (one
//     3-D TMA box per 128-query tile), k and v to the caches.  It also zeroes the attention
//     kernel's scheduler counters.
//  2. attention: a persistent kernel of CTA pairs (clusters of two on two SMs).  A pair takes
//     its first work item by its cluster index and later ones from an atomic counter, heaviest
//     first: 256 query rows = the same 128 queries for the two q heads of a GQA group (head
//     2i+r in CTA r) when the group size is even, else 256 consecutive queries of one head (rows
//     128r.. in CTA r).  Both products are
//     M=256 tcgen05.mma.cta_group::2.kind::f16 issued by one thread of CTA 0:
//       S_t = Q K_t^T  (N=128 keys, K=256): Q (128 rows x 256, this CTA's) and this CTA's half
//                      of the key tile (64 keys x 256) in shared memory, K-major;
//       O += P_t V_t   (N=256 dims, K=128 keys): P in TMEM, this CTA's half of V (128 keys x
//                      128 dims) in shared memory, MN-major.
//     so each SM streams half of every K/V tile that serves 256 query rows.  Per CTA, 12 warps:
//       warp 0  TMA producer (CTA 0's also takes items and sends them to CTA 1): 16 KB ring
//               slots in consumption order K(0) K(1) V(0) K(2) V(1) ...; all copies of the pair
//               complete on CTA 0's barriers; tensor maps end at pos0+T (keys past the valid
//               cache read as zeros).
//       warp 1  TMEM owner (512 columns, allocated for the pair); in CTA 0, the MMA issuer: the
//               whole warp runs the issue loop and one elected lane issues, so the descriptors
//               stay in uniform registers and 64-cycle MMAs go back to back.  S_{t+1} is issued
//               before PV_t.
//       warps 4-11  two warpgroups per 128 query rows (TMEM lane = row; half 0 takes keys
//               0-63 of each tile and dims 0-127, half 1 keys 64-127 and dims 128-255): online
//               softmax in the log2 domain (mask only on tiles crossing the causal/window
//               band; O rescaled in TMEM only when a row max grows by more than 2^8).  Each
//               half reads all 128 scores of its row for the max, so both halves reach the same
//               max with no exchange; the row sums meet once per item.  P goes as bf16 pairs over
//               the first 32 of the half's own S columns; then the epilogue.
//     TMEM (each CTA, its 128 rows): O = columns [0, 256), S0/P0 = [256, 384), S1/P1 = [384, 512).
#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "row256.cuh"

namespace apex {
namespace {

constexpr int kD = 256;
constexpr int kBM = 128;                             // query rows per CTA
constexpr int kBN = 128;                             // keys per tile (both CTAs)
constexpr int kSlots = 10;
constexpr uint32_t kChunk = 64 * 128;                // 64 rows x 128 B (one TMA box)
constexpr uint32_t kSlotBytes = 2 * kChunk;          // 16 KB
constexpr uint32_t kQBytes = kBM * kD * 2;           // 64 KB
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffSlots = kQBytes;
// The epilogue stages each item's output in four ring slots (one per epilogue warp: its 32 rows
// as four [32 rows][128 B] tiles, 128-byte swizzle), taken in ring order right after the item's
// last V tile and handed back once the output stores have read them.
constexpr uint32_t kBoxBytes = 32 * 128;             // one output store: 32 rows x 64 dims
constexpr uint32_t kStageSlots = 4;                  // ring slots per item's output
static_assert(kSlotBytes == 4 * kBoxBytes, "one epilogue warp's 32 rows fill one slot");
constexpr uint32_t kOffBar = kOffSlots + kSlots * kSlotBytes;
constexpr uint32_t kNumBars = 48;
constexpr uint32_t kOffItems = kOffBar + 8 * kNumBars;
constexpr uint32_t kItemRing = 8;
constexpr uint32_t kOffStageSlot = kOffItems + 4 * kItemRing;  // uint32 [2 item parity][4 warps]
constexpr uint32_t kOffRed = kOffStageSlot + 4 * 2 * kStageSlots;  // row sums, float [2 item parity][2 half][128]
constexpr uint32_t kOffFlag = kOffRed + 2 * 2 * 128 * 4;
constexpr uint32_t kOffTmem = kOffFlag + 16;
constexpr uint32_t kSmemBytes = kOffTmem + 16;  // the dynamic shared memory base is 1024-aligned
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 0, kColS = 256;
constexpr int kThreads = 512;                        // 16 warps: 0 TMA, 1 TMEM/MMA, 4-11 softmax, 12-15 epilogue
constexpr float kTau = 8.0f;                         // lazy-rescale threshold (log2 units)
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint32_t kHalfWarps = 8;                   // one softmax half of both CTAs
constexpr uint32_t kSoftmaxThreads = 256;            // softmax threads of one CTA
constexpr uint32_t kEpiThreads = 128;                // epilogue threads of one CTA
constexpr uint32_t kEpiPairWarps = 8;                // epilogue warps of both CTAs
// Registers per thread after setmaxnreg, per warpgroup (0: TMA + MMA, 1-2: softmax, 3: epilogue).
// The launch gives each warpgroup 128 x 128; the split must add up to the same total.
constexpr uint32_t kRegsTmaMma = 64, kRegsSoftmax = 168, kRegsEpilogue = 112;
static_assert(kRegsTmaMma + 2 * kRegsSoftmax + kRegsEpilogue == 4 * (65536 / kThreads), "register split");

static_assert(kSmemBytes <= 232448, "shared memory budget");
static_assert(kOffSlots % 1024 == 0 && kSlotBytes % 1024 == 0, "swizzled tiles need 1024-byte slots");

// barrier indices (8 bytes each at kOffBar).  CTA 0's copies of QFull, Full, P and OFree count
// the pair; Empty, QEmpty, S and O are signalled in both CTAs by multicast commits.  P is one
// barrier per (softmax half, tile parity), so PV can start on the first 64 keys early.  L (row
// sums written, by item parity) and LFree (row sums read) pass the row sums from the softmax
// warps to the epilogue warps of the same CTA.  OItem completes once per item, when its last PV
// is done: the epilogue waits on it rather than on O, whose phase may lag two behind.  Stage (by
// item parity, each CTA its own) tells the epilogue warps that the producer has taken the item's
// four staging slots; they hand each slot back on the slot's Empty barrier of their own CTA.
constexpr int kBarQFull = 0, kBarQEmpty = 1, kBarFull = 2, kBarEmpty = kBarFull + kSlots,
              kBarS = kBarEmpty + kSlots, kBarP = kBarS + 2, kBarO = kBarP + 4, kBarOFree = kBarO + 2,
              kBarItem = kBarOFree + 1, kBarL = kBarItem + kItemRing, kBarLFree = kBarL + 2,
              kBarOItem = kBarLFree + 2, kBarStage = kBarOItem + 1;
static_assert(kBarStage + 2 <= kNumBars, "barrier budget");

struct PrefillArgs {
    uint16_t *out;        // [B][T][Hq][D]
    unsigned *status;     // device status word
    unsigned *sched;      // [0] next item, [1] CTAs done (zeroed by the prep kernel)
    uint32_t batch, T, pos0, kv_len, q_heads, kv_heads, window, n_qtiles, n_items, pair_heads;
    uint32_t group_major;  // items ordered (sequence, heads) first, so concurrent pairs share K/V in L2
    float scale_log2;
};

struct Item {
    uint32_t b, h, kvh, t0, rows_valid, q_row;  // this CTA's head, first query, valid rows, q box row
    uint32_t pos_first, pos_last;               // positions of this CTA's rows
    uint32_t j_start, n_tiles;                  // key tiles of the pair
};

// Item order: heaviest query tiles (most keys) first across all (sequence, heads) when the
// launch's K/V fits in L2 many times over; otherwise (sequence, heads) major with the query tiles
// of one group taken together, heaviest first, so the pairs that run at once stream the same keys.
__device__ __forceinline__ void split_item(uint32_t idx, uint32_t groups, const PrefillArgs &a, uint32_t &qt,
                                           uint32_t &grp) {
    if (a.group_major) {
        grp = idx / a.n_qtiles;
        qt = a.n_qtiles - 1 - idx % a.n_qtiles;
    } else {
        qt = a.n_qtiles - 1 - idx / groups;
        grp = idx % groups;
    }
}

// Bit k set for k in [lo, hi] (bounds relative to a 32-key chunk; empty when hi < lo).
__device__ __forceinline__ uint32_t visible_bits(int lo, int hi) {
    lo = max(lo, 0);
    hi = min(hi, 31);
    if (hi < lo) return 0u;
    const uint32_t upto_hi = hi == 31 ? 0xffffffffu : ((2u << hi) - 1u);
    return upto_hi & ~((1u << lo) - 1u);
}

// Masks one 32-key chunk of a warp's 32 rows (bit k of vis: key k visible in this lane's row).  The
// masked band crosses a chunk in at most one warp of four, so the common cases are decided for the
// whole warp at once.  Returns false when no row of the warp sees any key of the chunk (all -inf).
__device__ __forceinline__ bool mask_chunk(uint32_t (&x)[32], uint32_t vis) {
    if (__all_sync(0xffffffffu, vis == 0xffffffffu)) return true;
    if (__all_sync(0xffffffffu, vis == 0u)) {
#pragma unroll
        for (int k = 0; k < 32; ++k) x[k] = 0xff800000u;  // -inf
        return false;
    }
    // branch-free (a lane-dependent `if` per key costs the warp a divergent branch each): keep is
    // all ones where key k is visible, and the rest becomes -inf
#pragma unroll
    for (int k = 0; k < 32; ++k) {
        const uint32_t keep = static_cast<uint32_t>(static_cast<int32_t>(vis << (31 - k)) >> 31);
        x[k] = (x[k] & keep) | (0xff800000u & ~keep);
    }
    return true;
}

__device__ __forceinline__ Item item_geometry(uint32_t idx, const PrefillArgs &a, uint32_t rank) {
    Item it;
    uint32_t t0_pair, span, qt, bp;
    if (a.pair_heads) {  // two heads of one GQA group, same 128 queries
        const uint32_t pairs = a.q_heads / 2;
        split_item(idx, a.batch * pairs, a, qt, bp);
        it.b = bp / pairs;
        it.h = 2 * (bp % pairs) + rank;
        t0_pair = qt * kBM;
        it.t0 = t0_pair;
        span = kBM;
    } else {  // one head, 256 consecutive queries
        split_item(idx, a.batch * a.q_heads, a, qt, bp);
        it.b = bp / a.q_heads;
        it.h = bp % a.q_heads;
        t0_pair = qt * 2 * kBM;
        it.t0 = t0_pair + rank * kBM;
        span = 2 * kBM;
    }
    it.kvh = it.h / (a.q_heads / a.kv_heads);
    it.rows_valid = a.T > it.t0 ? min(static_cast<uint32_t>(kBM), a.T - it.t0) : 0u;
    it.q_row = min(it.t0, a.T - 1);  // a q box always starts inside the workspace
    it.pos_first = a.pos0 + it.t0;
    it.pos_last = it.pos_first + (it.rows_valid ? it.rows_valid - 1 : 0u);
    const uint32_t pair_first = a.pos0 + t0_pair;
    const uint32_t pair_last = a.pos0 + min(a.T, t0_pair + span) - 1;
    const uint32_t kv_lo = (a.window && pair_first + 1 > a.window) ? pair_first + 1 - a.window : 0;
    it.j_start = (kv_lo / kBN) * kBN;
    it.n_tiles = (pair_last - it.j_start) / kBN + 1;
    return it;
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    prefill_pair_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                        const PrefillArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *base = smem_raw;
    const uint32_t sb = smem_u32(base);
    if (sb & 1023u) {  // same layout in both CTAs: both leave before any pair operation
        if (threadIdx.x == 0) atomicOr(a.status, kStatusTimeout);
        return;
    }
    auto bar = [&](int i) { return sb + kOffBar + 8u * i; };
    volatile int *items = reinterpret_cast<volatile int *>(base + kOffItems);
    volatile uint32_t *err_flag = reinterpret_cast<volatile uint32_t *>(base + kOffFlag);
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(base + kOffTmem);
    float *red = reinterpret_cast<float *>(base + kOffRed);  // row sums [2 item parity][2 half][128]

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;

    if (tid == 0) {
        // the descriptors' first fetch takes about a microsecond: start it before the set-up
        prefetch_tensormap(&tm_q);
        prefetch_tensormap(&tm_k);
        prefetch_tensormap(&tm_v);
        prefetch_tensormap(&tm_o);
        mbar_init(bar(kBarQFull), 1);
        mbar_init(bar(kBarQEmpty), 1);
        for (int i = 0; i < kSlots; ++i) {
            mbar_init(bar(kBarFull + i), 1);
            mbar_init(bar(kBarEmpty + i), 1);
        }
        for (int i = 0; i < 4; ++i) mbar_init(bar(kBarP + i), kHalfWarps);
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar(kBarS + i), 1);
            mbar_init(bar(kBarO + i), 1);
            mbar_init(bar(kBarL + i), kSoftmaxThreads);
            mbar_init(bar(kBarLFree + i), kEpiThreads);
        }
        mbar_init(bar(kBarOFree), kEpiPairWarps);
        mbar_init(bar(kBarOItem), 1);
        for (int i = 0; i < 2; ++i) mbar_init(bar(kBarStage + i), 1);
        for (uint32_t i = 0; i < kItemRing; ++i) mbar_init(bar(kBarItem + i), 1);
        *err_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(tmem_holder), kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    bool alive = true;

    // Both the TMA producer and the MMA issuer walk one stream of key tiles across items: K(t) /
    // S(t) come before V(t-1) / PV(t-1) also when tile t opens the next item, so the next item's
    // first scores are under way while the softmax still works on the previous item's last tile.
    if (warp < 4) {
        reg_dealloc<kRegsTmaMma>();
        if (warp == 0 && lane == 0) {
            // -------------------------------------------------------- TMA producer (+ scheduler in CTA 0)
            // Everything above overlapped the preceding kernel (the prep); from here on this
            // thread reads its outputs (scheduler counters, q, K, V), and every other role only
            // acts on items and data this thread hands on.
            griddep_wait();
            uint32_t n = 0;  // ring position (same sequence in both CTAs and the MMA issuer)
            auto next_slot = [&](uint32_t &dst, uint32_t &full) {
                const uint32_t slot = n % kSlots;
                if (n >= kSlots && !mbar_wait(bar(kBarEmpty + slot), ((n / kSlots) - 1) & 1, a.status))
                    return false;
                if (leader) mbar_arrive_expect_tx(bar(kBarFull + slot), 2 * kSlotBytes);
                dst = sb + kOffSlots + slot * kSlotBytes;
                full = mapa(bar(kBarFull + slot), 0);
                ++n;
                return true;
            };
            // a box never starts past the cache end; the keys it then holds are masked
            auto key_row = [&](uint32_t key) { return static_cast<int32_t>(min(key, a.kv_len - 1)); };
            bool pend = false;  // V of the previous tile, loaded after the next tile's K
            uint32_t pend_key = 0;
            int32_t pend_row = 0;
            auto load_v = [&]() {  // this CTA's 128 dims, keys [0,64) then [64,128)
                for (int s = 0; s < 2 && alive; ++s) {
                    uint32_t dst, full;
                    if (!next_slot(dst, full)) {
                        alive = false;
                        break;
                    }
                    for (int c = 0; c < 2; ++c)
                        tma_load_3d_pair(dst + c * kChunk, &tm_v, 128 * rank + 64 * c, key_row(pend_key + 64 * s),
                                         pend_row, full);
                }
                pend = false;
            };
            // the next four ring positions become item `item`'s output staging: each waits for its
            // slot like a load, completes its Full phase with no bytes (CTA 0), and goes to the
            // epilogue warp of its index; the MMA issuer passes over the same four positions
            uint32_t *stage_slot = reinterpret_cast<uint32_t *>(base + kOffStageSlot);
            auto reserve_stage = [&](uint32_t item) {
                for (uint32_t q = 0; q < kStageSlots; ++q) {
                    const uint32_t slot = n % kSlots;
                    if (n >= kSlots && !mbar_wait(bar(kBarEmpty + slot), ((n / kSlots) - 1) & 1, a.status)) {
                        alive = false;
                        return;
                    }
                    if (leader) mbar_arrive(bar(kBarFull + slot));
                    stage_slot[(item & 1) * kStageSlots + q] = slot;
                    ++n;
                }
                mbar_arrive(bar(kBarStage + (item & 1)));
            };
            uint32_t taken = 0;  // items this pair took
            for (uint32_t it = 0; alive; ++it) {
                const uint32_t is = it % kItemRing;
                int idx;
                if (leader) {
                    // each pair's first item is its cluster index (no round trip to a counter that
                    // every pair hits at once); later items come from the counter, past those
                    const uint32_t pairs = gridDim.x / 2;
                    const uint32_t claimed = it == 0 ? blockIdx.x / 2 : pairs + atomicAdd(a.sched, 1u);
                    idx = claimed < a.n_items ? static_cast<int>(claimed) : -1;
                    items[is] = idx;
                    st_cluster_u32(mapa(sb + kOffItems + 4 * is, 1), static_cast<uint32_t>(idx));
                    mbar_arrive(bar(kBarItem + is));
                    mbar_arrive_cluster(mapa(bar(kBarItem + is), 1));
                } else {
                    if (!mbar_wait_cluster(bar(kBarItem + is), (it / kItemRing) & 1, a.status)) {
                        alive = false;
                        break;
                    }
                    idx = items[is];
                }
                if (idx < 0) break;
                taken = it + 1;
                const Item g = item_geometry(static_cast<uint32_t>(idx), a, rank);
                const int32_t kv_row = static_cast<int32_t>(g.b * a.kv_heads + g.kvh);
                for (uint32_t j = 0; j < g.n_tiles && alive; ++j) {
                    // K(j): this CTA's 64 keys, dims [0,128) then [128,256)
                    const uint32_t key = g.j_start + j * kBN + 64 * rank;
                    for (int s = 0; s < 2 && alive; ++s) {
                        uint32_t dst, full;
                        if (!next_slot(dst, full)) {
                            alive = false;
                            break;
                        }
                        for (int c = 0; c < 2; ++c)
                            tma_load_3d_pair(dst + c * kChunk, &tm_k, 128 * s + 64 * c, key_row(key), kv_row, full);
                    }
                    if (pend && alive) load_v();
                    if (j == 0 && alive) {  // Q, once the previous item's S MMAs are done with it
                        if (it >= 1 && !mbar_wait(bar(kBarQEmpty), (it - 1) & 1, a.status)) {
                            alive = false;
                            break;
                        }
                        if (leader) mbar_arrive_expect_tx(bar(kBarQFull), 2 * kQBytes);
                        const uint32_t full = mapa(bar(kBarQFull), 0);
                        for (int c = 0; c < 4; ++c)
                            tma_load_3d_pair(sb + kOffQ + c * (kQBytes / 4), &tm_q, 64 * c,
                                             static_cast<int32_t>(g.q_row),
                                             static_cast<int32_t>(g.b * a.q_heads + g.h), full);
                        if (it >= 1) reserve_stage(it - 1);  // the previous item's last V is in the ring
                    }
                    pend = true;
                    pend_key = g.j_start + j * kBN;
                    pend_row = kv_row;
                }
            }
            if (pend && alive) {
                load_v();
                if (alive) reserve_stage(taken - 1);
            }
        } else if (warp == 1 && leader) {
            // -------------------------------------------------------- MMA issuer (CTA 0)
            // The whole warp runs the loop (its values stay warp-uniform) and one elected lane issues
            // each tcgen05 instruction; the waits poll with test_wait (mbar_wait_spin).
            auto wait_all = [&](uint32_t b, uint32_t parity) {
                return __all_sync(0xffffffffu, mbar_wait_spin(b, parity, a.status));
            };
            constexpr uint32_t idS = idesc_bf16_f32(2 * kBM, kBN, 0, 0);
            constexpr uint32_t idPV = idesc_bf16_f32(2 * kBM, kD, 0, 1);
            // Descriptors of the first K-step; every other step is a byte offset added to the
            // start-address field (address >> 4, all offsets stay inside shared memory).
            const uint64_t q_desc = smem_desc_sw128(sb + kOffQ, 16, 1024);
            const uint64_t k_desc = smem_desc_sw128(sb + kOffSlots, 16, 1024);
            const uint64_t v_desc = smem_desc_sw128(sb + kOffSlots, kChunk, 1024);
            uint32_t gt = 0, n = 0;
            auto wait_full = [&](uint32_t m) { return wait_all(bar(kBarFull + m % kSlots), (m / kSlots) & 1); };
            auto issue_pv = [&](uint32_t t, bool first, bool last, uint32_t it) {
                if (!alive) return;
                if (first && it >= 1) alive = wait_all(bar(kBarOFree), (it - 1) & 1);
                const uint32_t p_col = tmem + kColS + (t & 1) * kBN;
                for (int s = 0; s < 2 && alive; ++s) {
                    if (!wait_all(bar(kBarP + 2 * s + (t & 1)), (t >> 1) & 1)) {
                        alive = false;
                        return;
                    }
                    if (!wait_full(n)) {
                        alive = false;
                        return;
                    }
                    tc_fence_after();
                    const uint32_t slot = n % kSlots;
                    const uint64_t vd = v_desc + ((slot * kSlotBytes) >> 4);
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        tc_mma_ts_pair(tmem + kColO, p_col + s * 64 + ks * 8, vd + ((ks * 2048) >> 4), idPV,
                                       (!first || s > 0 || ks > 0) ? 1u : 0u);
                    tc_commit_pair_both(bar(kBarEmpty + slot));
                    ++n;
                }
                tc_commit_pair_both(bar(kBarO + (t & 1)));
                if (last) {
                    tc_commit_pair_both(bar(kBarOItem));
                    // the item's four output-staging positions: no MMA reads them
                    for (uint32_t q = 0; q < kStageSlots && alive; ++q) {
                        alive = wait_full(n);
                        ++n;
                    }
                }
            };
            bool pend = false, pend_first = false, pend_last = false;  // PV of the previous tile, issued after the next S
            uint32_t pend_t = 0, pend_it = 0;
            for (uint32_t it = 0; alive; ++it) {
                if (!wait_all(bar(kBarItem + it % kItemRing), (it / kItemRing) & 1)) {
                    alive = false;
                    break;
                }
                const int idx = items[it % kItemRing];
                if (idx < 0) break;
                const Item g = item_geometry(static_cast<uint32_t>(idx), a, 0);
                if (!wait_all(bar(kBarQFull), it & 1)) {
                    alive = false;
                    break;
                }
                tc_fence_after();
                for (uint32_t j = 0; j < g.n_tiles && alive; ++j) {
                    const uint32_t t = gt + j;
                    const uint32_t s_col = tmem + kColS + (t & 1) * kBN;
                    for (int s = 0; s < 2 && alive; ++s) {  // K(j) dims [128s, 128s+128)
                        if (!wait_full(n)) {
                            alive = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t slot = n % kSlots;
                        const uint64_t kd = k_desc + ((slot * kSlotBytes) >> 4);
                        const uint64_t qd = q_desc + ((s * 2 * (kQBytes / 4)) >> 4);
#pragma unroll
                        for (int ks = 0; ks < 8; ++ks) {  // 16-dim step 8s + ks of the 256 dims
                            const uint32_t off = ((ks / 4) * (kQBytes / 4) + (ks % 4) * 32) >> 4;
                            const uint32_t koff = ((ks / 4) * kChunk + (ks % 4) * 32) >> 4;
                            tc_mma_ss_pair(s_col, qd + off, kd + koff, idS, (s | ks) ? 1u : 0u);
                        }
                        tc_commit_pair_both(bar(kBarEmpty + slot));
                        ++n;
                    }
                    if (!alive) break;
                    tc_commit_pair_both(bar(kBarS + (t & 1)));
                    if (j + 1 == g.n_tiles) tc_commit_pair_both(bar(kBarQEmpty));  // Q free once these finish
                    if (pend) issue_pv(pend_t, pend_first, pend_last, pend_it);
                    pend = true;
                    pend_t = t;
                    pend_first = j == 0;
                    pend_last = j + 1 == g.n_tiles;
                    pend_it = it;
                }
                gt += g.n_tiles;
            }
            if (pend && alive) issue_pv(pend_t, pend_first, pend_last, pend_it);
        }
    } else if (warp < 12) {
        // ------------------------------------------------------------ softmax (both CTAs)
        reg_alloc<kRegsSoftmax>();
        const uint32_t half = (warp - 4) >> 2, quad = warp & 3;
        const uint32_t r = quad * 32 + lane;                  // query row == TMEM lane
        const uint32_t lane_base = tmem + ((32u * quad) << 16);
        const uint32_t p_bar0 = mapa(bar(kBarP + 2 * half), 0), p_bar1 = mapa(bar(kBarP + 2 * half + 1), 0);
        uint32_t gt = 0;
        // Wait for PV of global tile t.  o_done is a ring of two barriers indexed by tile parity:
        // when this runs (after S(t+1) or S(t) completed), PV(t-2) is already complete (it was
        // issued before those S MMAs) and PV(t+2) cannot have started, so the parity is
        // unambiguous without observing every phase.
        auto wait_pv = [&](uint32_t t) {
            alive = alive && __all_sync(0xffffffffu, mbar_wait(bar(kBarO + (t & 1)), (t >> 1) & 1, a.status));
        };
        // one elected lane per warp reports to CTA 0 after the warp's TMEM accesses are done
        auto warp_arrive = [&](uint32_t cluster_bar) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(cluster_bar);
        };
        for (uint32_t it = 0; alive; ++it) {
            if (!__all_sync(0xffffffffu, mbar_wait_cluster(bar(kBarItem + it % kItemRing), (it / kItemRing) & 1,
                                                            a.status))) {
                alive = false;
                break;
            }
            const int idx = items[it % kItemRing];
            if (idx < 0) break;
            const Item g = item_geometry(static_cast<uint32_t>(idx), a, rank);
            const uint32_t t = g.t0 + r;
            const int pos = static_cast<int>(a.pos0 + t);
            float m_run = -INFINITY, l_part = 0.f;
            for (uint32_t j = 0; j < g.n_tiles && alive; ++j) {
                const uint32_t tt = gt + j;
                if (!__all_sync(0xffffffffu, mbar_wait(bar(kBarS + (tt & 1)), (tt >> 1) & 1, a.status))) {
                    alive = false;
                    break;
                }
                tc_fence_after();
                const uint32_t s_row = lane_base + kColS + (tt & 1) * kBN;
                const uint32_t s_addr = s_row + half * 64;
                const uint32_t o_addr = s_row + (half ^ 1) * 64;
                uint32_t sv[64];
                float mx;
                {
                    const uint32_t tile0 = g.j_start + j * kBN;
                    const bool need_mask = g.rows_valid && ((tile0 + kBN - 1 > g.pos_first) ||
                                                            (a.window && tile0 + a.window <= g.pos_last));
                    // visible keys of this row relative to the tile's first key: [lo, hi]
                    const int hi = pos - static_cast<int>(tile0);
                    const int lo = a.window ? pos + 1 - static_cast<int>(a.window) - static_cast<int>(tile0) : -(1 << 30);
                    const int own = static_cast<int>(half) * 64, oth = static_cast<int>(half ^ 1) * 64;
                    uint32_t ov[32];
                    mx = -INFINITY;
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        uint32_t(&sc)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sv[32 * c]);
                        tmem_ld32(s_addr + 32 * c, sc);
                        tmem_ld32(o_addr + 32 * c, ov);
                        tc_wait_ld(sc, ov);
                        bool sc_live = true, ov_live = true;
                        if (need_mask) {
                            sc_live = mask_chunk(sc, visible_bits(lo - own - 32 * c, hi - own - 32 * c));
                            ov_live = mask_chunk(ov, visible_bits(lo - oth - 32 * c, hi - oth - 32 * c));
                        }
                        if (ov_live) {
#pragma unroll
                            for (int k = 0; k < 32; k += 2) mx = fmax3(mx, __uint_as_float(ov[k]), __uint_as_float(ov[k + 1]));
                        }
                        if (sc_live) {
#pragma unroll
                            for (int k = 0; k < 32; k += 2) mx = fmax3(mx, __uint_as_float(sc[k]), __uint_as_float(sc[k + 1]));
                        }
                    }
                }
                const float mt = mx * a.scale_log2;
                float alpha = 1.f;
                bool rescale = false;
                if (mt > m_run + kTau) {
                    alpha = fast_exp2(m_run - mt);  // 0 when m_run = -inf
                    rescale = j > 0 && m_run != -INFINITY;  // O holds only zeros while m_run = -inf
                    m_run = mt;
                }
                const float neg_m = m_run == -INFINITY ? 0.f : -m_run;
                // p = 2^(s * scale - m) in packed f32x2 arithmetic; 12 of the 64 exponentials run as a
                // polynomial on the FMA pipe, the rest on MUFU (which alone would bound this loop)
                uint64_t sum2[2] = {0ull, 0ull};
                uint32_t packed[32];
                const uint64_t scale2 = f32x2(a.scale_log2, a.scale_log2), neg_m2 = f32x2(neg_m, neg_m);
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const uint64_t x2 = fma_f32x2(f32x2(__uint_as_float(sv[2 * i]), __uint_as_float(sv[2 * i + 1])),
                                                  scale2, neg_m2);
                    float p0, p1;
                    if (i % 5 == 2 && i < 30) {
                        exp2_poly_x2(x2, p0, p1);
                    } else {
                        float x0, x1;
                        f32x2_split(x2, x0, x1);
                        p0 = fast_exp2(x0);
                        p1 = fast_exp2(x1);
                    }
                    sum2[i & 1] = add_f32x2(sum2[i & 1], f32x2(p0, p1));
                    packed[i] = pack_bf16(p0, p1);
                }
                float s0, s1, s2, s3;
                f32x2_split(sum2[0], s0, s1);
                f32x2_split(sum2[1], s2, s3);
                l_part = l_part * alpha + ((s0 + s1) + (s2 + s3));
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
                        tc_wait_ld(o);
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
                        tmem_st32(oa, o);
                    }
                }
                tmem_st32(s_addr, packed);  // P over the first 32 of this half's own S columns
                tc_wait_st();
                warp_arrive((tt & 1) ? p_bar1 : p_bar0);
            }
            if (!alive) break;
            // this half's row sums go to the epilogue warps (slot it % 2, free once item it - 2's
            // epilogue has read it)
            if (it >= 2 && !__all_sync(0xffffffffu, mbar_wait(bar(kBarLFree + (it & 1)), ((it >> 1) - 1) & 1, a.status))) {
                alive = false;
                break;
            }
            red[((it & 1) * 2 + half) * kBM + r] = l_part;
            mbar_arrive(bar(kBarL + (it & 1)));
            gt += g.n_tiles;
        }
    } else {
        // ------------------------------------------------------------ epilogue (both CTAs)
        // O / l -> bf16 out[b][t][h][...] for this CTA's 128 rows, once the item's last PV is done.
        // Warp q stages its 32 rows in the ring slot the producer took for it (four [32 rows][128 B]
        // tiles, 128-byte swizzle: 16-byte piece c of row x at ((c ^ (x & 7)) * 16)), so the
        // four 64-column rounds never wait for a store to read a tile: O goes back to the next
        // item's PV as soon as its last columns are in registers.  Then one TMA store per tile (rows
        // at or past T clipped by the tensor map) and, once they have read the slot, the slot goes
        // back to the producer on its Empty barrier.
        reg_dealloc<kRegsEpilogue>();
        const uint32_t quad = warp & 3;
        const uint32_t r = quad * 32 + lane;
        const uint32_t lane_base = tmem + ((32u * quad) << 16);
        const uint32_t ofree_bar = mapa(bar(kBarOFree), 0);
        const uint32_t *stage_slot = reinterpret_cast<const uint32_t *>(base + kOffStageSlot);
        for (uint32_t it = 0; alive; ++it) {
            if (!__all_sync(0xffffffffu, mbar_wait_cluster(bar(kBarItem + it % kItemRing), (it / kItemRing) & 1,
                                                            a.status))) {
                alive = false;
                break;
            }
            const int idx = items[it % kItemRing];
            if (idx < 0) break;
            const Item g = item_geometry(static_cast<uint32_t>(idx), a, rank);
            // the item's last PV (OItem completes once per item; the next item's PVs wait for this
            // warp's O release, so the barrier cannot run a phase ahead), its row sums, its slots
            if (!__all_sync(0xffffffffu, mbar_wait(bar(kBarOItem), it & 1, a.status)) ||
                !__all_sync(0xffffffffu, mbar_wait(bar(kBarL + (it & 1)), (it >> 1) & 1, a.status)) ||
                !__all_sync(0xffffffffu, mbar_wait(bar(kBarStage + (it & 1)), (it >> 1) & 1, a.status))) {
                alive = false;
                break;
            }
            tc_fence_after();
            const float l_run = red[((it & 1) * 2) * kBM + r] + red[((it & 1) * 2 + 1) * kBM + r];
            mbar_arrive(bar(kBarLFree + (it & 1)));
            const float inv_l = l_run > 0.f ? 1.0f / l_run : 0.f;
            const bool any_rows = quad * 32 < g.rows_valid;
            const uint32_t slot = stage_slot[(it & 1) * kStageSlots + quad];
            const uint32_t stg = sb + kOffSlots + slot * kSlotBytes;  // 1024-aligned
            const uint32_t row_base = stg + lane * 128 + ((lane & 7) << 4);
            // 64 columns per TMEM load; each is packed to bf16 and staged while the next is in flight
            uint32_t raw[64];
            uint32_t(&raw_lo)[32] = *reinterpret_cast<uint32_t(*)[32]>(&raw[0]);
            uint32_t(&raw_hi)[32] = *reinterpret_cast<uint32_t(*)[32]>(&raw[32]);
            tmem_ld64(lane_base + kColO, raw);
            tc_wait_ld(raw_lo, raw_hi);
#pragma unroll
            for (int pr = 0; pr < 4; ++pr) {
                uint32_t pk[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) pk[i] = scale_pack_bf16(raw[2 * i], raw[2 * i + 1], inv_l);
                if (pr < 3) tmem_ld64(lane_base + kColO + 64 * (pr + 1), raw);
#pragma unroll
                for (int c = 0; c < 8; ++c)  // piece c of row `lane` at (c ^ (lane & 7)) * 16
                    st_shared_v4((row_base ^ (c << 4)) + pr * kBoxBytes,
                                 make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]));
                if (pr < 3) tc_wait_ld(raw_lo, raw_hi);
                if (pr == 2) {  // all of O is in registers: the next item's first PV may overwrite it
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_remote(ofree_bar);
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                if (any_rows) {
#pragma unroll
                    for (int b4 = 0; b4 < 4; ++b4)
                        tma_store_4d(&tm_o, stg + b4 * kBoxBytes, static_cast<int32_t>(64 * b4), static_cast<int32_t>(g.h),
                                     static_cast<int32_t>(g.t0 + quad * 32), static_cast<int32_t>(g.b));
                    bulk_commit_group();
                    bulk_wait_read_all();  // the stores have read the slot
                }
                mbar_arrive(bar(kBarEmpty + slot));
            }
        }
        if (lane == 0) bulk_wait_all();
    }
    // Teardown.  The epilogue's TMA stores have finished (above).  After a failed wait, copies or
    // MMAs of this pair may still be in flight: give them time to land (bounded) before the pair
    // releases TMEM and shared memory.
    if (!alive) *err_flag = 1u;
    __syncwarp();
    tc_fence_before();
    cluster_sync();
    if (tid == 0 && *err_flag) {
        const long long start = clock64();
        while (clock64() - start < 400000ll) __nanosleep(1000);
    }
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, kTmemCols);
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
    unsigned *status;     // device status word
    uint32_t B, T, pos0, q_heads, kv_heads, capacity, rope_pairs, qk_norm, v_norm;
    float eps;
    RopeTable rope;
};

// A persistent grid of two blocks per SM walks the tokens (block i: tokens i, i + grid, ...).  Per
// token, one producer warp copies the token's q rows, then k rows, then v rows (three contiguous
// runs in the [B][T][heads][256] inputs, 16 KB at Hq = 16, Hkv = 8) into the next stage of a
// 4-stage shared-memory ring with 1-D TMA bulk copies, and writes the token's RoPE cos/sin beside
// it; eight consumer warps take rows w, w+8, ... of the stage: RMS norm (weights held in
// registers), RoPE, bf16, one 16-byte load and store per lane per row.  Loads of later tokens
// stay in flight while earlier ones are computed and stored.
// Lane l holds dims [4l, 4l+4) and [128+4l, 128+4l+4) of a row: both members of its four RoPE pairs,
// so rotation needs no shuffles.
constexpr int kPrepConsumers = 8;
constexpr int kPrepThreads = (kPrepConsumers + 1) * 32;
constexpr int kPrepStages = 4;
constexpr uint32_t kRowBytes = kD * 2;
constexpr uint32_t kPrepMaxRows = 96;  // q + k + v rows of one token (shared memory: 4 x 48 KB)

uint32_t prep_smem_bytes(uint32_t rows) { return kPrepStages * (rows * kRowBytes + kD * 4) + 2 * kPrepStages * 8; }

__device__ __forceinline__ void unpack4(uint2 v, float (&x)[4]) {
    x[0] = bf16lo(v.x); x[1] = bf16hi(v.x); x[2] = bf16lo(v.y); x[3] = bf16hi(v.y);
}
__device__ __forceinline__ uint2 pack4(const float (&x)[4]) { return make_uint2(pack_bf16(x[0], x[1]), pack_bf16(x[2], x[3])); }

__global__ void __launch_bounds__(kPrepThreads, 2) prefill_prep_kernel(const __grid_constant__ PrepArgs a) {
    extern __shared__ __align__(128) uint8_t psm[];
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) griddep_launch_dependents();  // the attention kernel's set-up may start
    if (blockIdx.x == 0 && tid == 0) {
        a.sched[0] = 0;
        a.sched[1] = 0;
    }
    const uint32_t Hq = a.q_heads, Hkv = a.kv_heads, rows = Hq + 2 * Hkv;
    const uint32_t stage_bytes = rows * kRowBytes;
    float *tab = reinterpret_cast<float *>(psm + kPrepStages * stage_bytes);  // [stage][cos 128 | sin 128]
    const uint32_t bars = smem_u32(psm + kPrepStages * (stage_bytes + kD * 4));
    auto full = [&](uint32_t s) { return bars + 8u * s; };
    auto empty = [&](uint32_t s) { return bars + 8u * (kPrepStages + s); };
    if (tid == 0) {
        for (int s = 0; s < kPrepStages; ++s) {
            mbar_init(full(s), 32);  // the producer warp's lanes (after their cos/sin) + the copies' bytes
            mbar_init(empty(s), kPrepConsumers);
        }
        fence_mbar_init();
    }
    __syncthreads();
    const uint32_t ntok = a.B * a.T, G = gridDim.x;
    if (warp == kPrepConsumers) {
        // ---------------------------------------------------------------- producer warp
        uint32_t n = 0;
        for (uint32_t tok = blockIdx.x; tok < ntok; tok += G, ++n) {
            const uint32_t s = n % kPrepStages;
            if (n >= kPrepStages &&
                !__all_sync(0xffffffffu, mbar_wait(empty(s), ((n / kPrepStages) - 1) & 1, a.status)))
                break;
            const uint32_t t = tok % a.T;
            uint8_t *st = psm + s * stage_bytes;
            if (lane == 0) {
                mbar_expect_tx(full(s), stage_bytes);
                tma_bulk_load(smem_u32(st), a.q_raw + static_cast<uint64_t>(tok) * Hq * kD, Hq * kRowBytes, full(s));
                tma_bulk_load(smem_u32(st + Hq * kRowBytes), a.k_raw + static_cast<uint64_t>(tok) * Hkv * kD,
                              Hkv * kRowBytes, full(s));
                tma_bulk_load(smem_u32(st + (Hq + Hkv) * kRowBytes), a.v_raw + static_cast<uint64_t>(tok) * Hkv * kD,
                              Hkv * kRowBytes, full(s));
            }
            const float pos = static_cast<float>(a.pos0 + t);
            float *cs = tab + s * kD;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint32_t i = 4 * lane + e;
                float c = 1.f, sn = 0.f;
                if (i < a.rope_pairs) rope_sincos(pos * a.rope.inv_freq[i], sn, c);
                cs[i] = c;
                cs[kD / 2 + i] = sn;
            }
            mbar_arrive(full(s));
        }
        return;
    }
    // -------------------------------------------------------------------- consumer warps
    const uint32_t d_lo = 4 * lane, d_hi = kD / 2 + 4 * lane;
    float wq[8], wk[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        wq[e] = a.q_w ? bf16lo(static_cast<uint32_t>(a.q_w[d_lo + e])) : 1.f;
        wq[4 + e] = a.q_w ? bf16lo(static_cast<uint32_t>(a.q_w[d_hi + e])) : 1.f;
        wk[e] = a.k_w ? bf16lo(static_cast<uint32_t>(a.k_w[d_lo + e])) : 1.f;
        wk[4 + e] = a.k_w ? bf16lo(static_cast<uint32_t>(a.k_w[d_hi + e])) : 1.f;
    }
    uint32_t n = 0;
    for (uint32_t tok = blockIdx.x; tok < ntok; tok += G, ++n) {
        const uint32_t s = n % kPrepStages;
        if (!__all_sync(0xffffffffu, mbar_wait(full(s), (n / kPrepStages) & 1, a.status))) break;
        const uint32_t b = tok / a.T, t = tok - b * a.T;
        const uint8_t *st = psm + s * stage_bytes;
        const float *cs_tab = tab + s * kD;
        float cs[4], sn[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            cs[e] = cs_tab[d_lo + e];
            sn[e] = cs_tab[kD / 2 + d_lo + e];
        }
        // rows warp, warp + 8, warp + 16, warp + 24 together (their RMS reductions interleave)
        for (uint32_t base = warp; base < rows; base += 4 * kPrepConsumers) {
            uint2 raw[4][2];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t r = base + i * kPrepConsumers;
                if (r < rows) {
                    raw[i][0] = *reinterpret_cast<const uint2 *>(st + r * kRowBytes + 8 * lane);
                    raw[i][1] = *reinterpret_cast<const uint2 *>(st + r * kRowBytes + kRowBytes / 2 + 8 * lane);
                } else {
                    raw[i][0] = raw[i][1] = make_uint2(0u, 0u);
                }
            }
            float lo[4][4], hi[4][4], ss[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                unpack4(raw[i][0], lo[i]);
                unpack4(raw[i][1], hi[i]);
                ss[i] = 0.f;
#pragma unroll
                for (int e = 0; e < 4; ++e) ss[i] += lo[i][e] * lo[i][e] + hi[i][e] * hi[i][e];
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                for (int i = 0; i < 4; ++i) ss[i] += __shfl_xor_sync(0xffffffffu, ss[i], o);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t r = base + i * kPrepConsumers;
                if (r >= rows) continue;
                const bool is_q = r < Hq, is_v = r >= Hq + Hkv;
                const bool norm = is_v ? a.v_norm != 0 : a.qk_norm != 0;
                const float inv = norm ? rsqrtf(ss[i] * (1.0f / kD) + a.eps) : 1.0f;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    lo[i][e] *= inv * (is_v ? 1.0f : (is_q ? wq[e] : wk[e]));
                    hi[i][e] *= inv * (is_v ? 1.0f : (is_q ? wq[4 + e] : wk[4 + e]));
                }
                if (!is_v) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float l = lo[i][e], h = hi[i][e];
                        lo[i][e] = l * cs[e] - h * sn[e];
                        hi[i][e] = h * cs[e] + l * sn[e];
                    }
                }
                uint16_t *dst =
                    is_q ? a.q_ws + ((static_cast<uint64_t>(b) * Hq + r) * a.T + t) * kD
                         : (is_v ? a.v_cache : a.k_cache) +
                               ((static_cast<uint64_t>(b) * Hkv + (r - Hq - (is_v ? Hkv : 0u))) * a.capacity + a.pos0 + t) * kD;
                *reinterpret_cast<uint2 *>(dst + d_lo) = pack4(lo[i]);
                *reinterpret_cast<uint2 *>(dst + d_hi) = pack4(hi[i]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty(s));  // this warp is done reading the stage
    }
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

size_t q_ws_bytes(uint32_t batch, uint32_t tokens, uint32_t q_heads) {
    return static_cast<size_t>(batch) * tokens * q_heads * kD * 2;
}

size_t ws_bytes(uint32_t batch, uint32_t tokens, uint32_t q_heads) {
    return align256(q_ws_bytes(batch, tokens, q_heads)) + 256;  // + scheduler counters
}

constexpr uint32_t kWideD = 512;  // the global layers' head_dim (prefill_gqa.cu)

size_t ws_bytes_for(const apex_attn_params *p, uint32_t batch, uint32_t tokens) {
    return p->head_dim == kWideD ? prefill_gqa_workspace_bytes(batch, tokens, p->q_heads)
                                 : ws_bytes(batch, tokens, p->q_heads);
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
    const bool wide = p->head_dim == kWideD;
    if (p->head_dim != kD && !wide) return fail(APEX_ERR_UNSUPPORTED, n + ": this build supports head_dim 256 and 512");
    if (wide && !p->qk_norm)
        return fail(APEX_ERR_UNSUPPORTED, n + ": head_dim 512 prefill normalises q and k (qk_norm = 1)");
    if (p->ring) return fail(APEX_ERR_UNSUPPORTED, n + ": prefill writes a linear cache (copy its last keys into a ring with apex_kv_ring_store)");
    if (p->kv_heads == 0 || p->q_heads == 0 || p->q_heads % p->kv_heads)
        return fail(APEX_ERR_INVALID_ARGUMENT, n + ": q_heads must be a multiple of kv_heads");
    if (p->rope_pairs > p->head_dim / 2) return fail(APEX_ERR_INVALID_ARGUMENT, n + ": rope_pairs > head_dim / 2");
    if (batch == 0 || tokens == 0) return APEX_OK;
    for (const void *ptr : tensors) {
        if (!ptr) return fail(APEX_ERR_INVALID_ARGUMENT, n + ": null tensor");
        if (!aligned16(ptr)) return fail(APEX_ERR_INVALID_ARGUMENT, n + ": tensors must be 16-byte aligned");
    }
    if (static_cast<uint64_t>(pos0) + tokens > capacity)
        return fail(APEX_ERR_INVALID_ARGUMENT, n + ": pos0 + tokens exceeds capacity");
    if (wide) {
        // grid (ceil(T / 16) x kv heads x ceil(group / 2), 1, batch); the norm-and-RoPE launches take
        // strides of tokens x 512 and capacity x 512 elements as 32-bit values
        const uint64_t gx = static_cast<uint64_t>(p->kv_heads) * ((p->q_heads / p->kv_heads + 1) / 2) *
                            ((tokens + 15) / 16);
        if (gx > 0x7fffffffull || batch > 65535 || static_cast<uint64_t>(capacity) * kWideD > 0xffffffffull)
            return fail(APEX_ERR_INVALID_ARGUMENT, n + ": problem too large for one launch");
    } else {
        const uint64_t items = static_cast<uint64_t>(batch) * p->q_heads * ((tokens + kBM - 1) / kBM);
        if (items > 0x7fffffffull) return fail(APEX_ERR_INVALID_ARGUMENT, n + ": problem too large for one launch");
        if (p->q_heads + 2 * p->kv_heads > kPrepMaxRows)
            return fail(APEX_ERR_UNSUPPORTED, n + ": more than 96 q + k + v heads per token");
    }
    if (static_cast<uint64_t>(batch) * tokens > 0xffffffffull)
        return fail(APEX_ERR_INVALID_ARGUMENT, n + ": problem too large for one launch");
    const size_t need = ws_bytes_for(p, batch, tokens);
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
    pa.status = device_status_ptr();
    if (!pa.status) return fail(APEX_ERR_CUDA, "prefill prep: device status word unavailable");
    const uint32_t rows = p->q_heads + 2 * p->kv_heads;
    const uint32_t smem = prep_smem_bytes(rows);
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_set[dev]) {
        const int rc = check_cuda(cudaFuncSetAttribute(prefill_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                       static_cast<int>(prep_smem_bytes(kPrepMaxRows))),
                                  "prefill prep smem attribute");
        if (rc) return rc;
        attr_set[dev] = true;
    }
    const uint64_t ntok = static_cast<uint64_t>(batch) * tokens;
    const uint32_t grid = static_cast<uint32_t>(std::max<uint64_t>(1, std::min<uint64_t>(ntok, 2ull * sm_count())));
    prefill_prep_kernel<<<grid, kPrepThreads, smem, s>>>(pa);
    return check_cuda(cudaGetLastError(), "prefill prep launch");
}

// Clusters of two that fit on the device at once with this kernel's shared memory (some GPCs
// have an odd number of SMs); queried once per device.
uint32_t max_active_pairs() {
    static int cached[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && cached[dev]) return static_cast<uint32_t>(cached[dev]);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * static_cast<uint32_t>(sm_count() / 2), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmemBytes;
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, prefill_pair_kernel, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();  // clear the query's error; fall back to one pair per two SMs
        n = sm_count() / 2;
    }
    if (dev < 64) cached[dev] = n;
    return static_cast<uint32_t>(n);
}

int launch_attend(const apex_attn_params *p, void *workspace, const uint16_t *k_cache, const uint16_t *v_cache,
                  uint32_t capacity, uint32_t batch, uint32_t tokens, uint32_t pos0, uint16_t *out,
                  cudaStream_t s) {
    CUtensorMap tq, tk, tv;
    const uint64_t kv_len = static_cast<uint64_t>(pos0) + tokens;
    const uint64_t kv_rows = static_cast<uint64_t>(batch) * p->kv_heads;
    // normalised q [B*Hq][T][256]: one box = 128 queries x 64 dims
    int rc = make_tensor_map_bf16_3d(&tq, workspace, kD, tokens, static_cast<uint64_t>(batch) * p->q_heads, kD * 2ull,
                                     static_cast<uint64_t>(tokens) * kD * 2, 64, kBM);
    if (rc) return rc;
    // caches [B*Hkv][capacity][256] cut at pos0+T: one box = 64 keys x 64 dims
    rc = make_tensor_map_bf16_3d(&tk, k_cache, kD, kv_len, kv_rows, kD * 2ull, static_cast<uint64_t>(capacity) * kD * 2,
                                 64, 64);
    if (rc) return rc;
    rc = make_tensor_map_bf16_3d(&tv, v_cache, kD, kv_len, kv_rows, kD * 2ull, static_cast<uint64_t>(capacity) * kD * 2,
                                 64, 64);
    if (rc) return rc;
    // output [B][T][Hq][256] as {256, Hq, T, B}: one box = 64 dims x 1 head x 32 queries
    CUtensorMap to;
    const uint64_t row = static_cast<uint64_t>(kD) * 2;
    rc = make_tensor_map_bf16_4d(&to, out, {static_cast<uint64_t>(kD), p->q_heads, tokens, batch},
                                 {row, row * p->q_heads, row * p->q_heads * tokens}, {64, 1, 32, 1}, true);
    if (rc) return rc;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_set[dev]) {
        rc = check_cuda(cudaFuncSetAttribute(prefill_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kSmemBytes)),
                        "prefill smem attribute");
        if (rc) return rc;
        attr_set[dev] = true;
    }
    PrefillArgs fa{};
    fa.out = out;
    fa.status = device_status_ptr();
    if (!fa.status) return fail(APEX_ERR_CUDA, "prefill: device status word unavailable");
    fa.sched = sched_ptr(workspace, batch, tokens, p->q_heads);
    fa.batch = batch; fa.T = tokens; fa.pos0 = pos0; fa.kv_len = static_cast<uint32_t>(kv_len);
    fa.q_heads = p->q_heads; fa.kv_heads = p->kv_heads; fa.window = p->window;
    fa.pair_heads = (p->q_heads / p->kv_heads) % 2 == 0;
    if (fa.pair_heads) {
        fa.n_qtiles = (tokens + kBM - 1) / kBM;
        fa.n_items = batch * (p->q_heads / 2) * fa.n_qtiles;
    } else {
        fa.n_qtiles = (tokens + 2 * kBM - 1) / (2 * kBM);
        fa.n_items = batch * p->q_heads * fa.n_qtiles;
    }
    fa.scale_log2 = p->scale * kLog2e;
    // K and V of the whole launch: beyond ~3/8 of L2, order items so that pairs share keys
    const uint64_t kv_bytes = kv_rows * kv_len * kD * 2 * 2;
    fa.group_major = kv_bytes > (48ull << 20);
    const uint32_t pairs = std::min<uint32_t>(fa.n_items, max_active_pairs());
    // Programmatic stream serialization: the pairs' set-up (barriers, TMEM, tensor maps) overlaps
    // the tail of the preceding kernel; the producers wait for it before touching its outputs.
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * pairs, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return check_cuda(cudaLaunchKernelEx(&cfg, prefill_pair_kernel, tq, tk, tv, to, fa), "prefill attention launch");
}

}  // namespace
}  // namespace apex

extern "C" size_t apex_attn_prefill_workspace_bytes(const apex_attn_params *p, uint32_t batch,
                                                    uint32_t tokens) {
    if (!p) return 0;
    return apex::ws_bytes_for(p, batch, tokens);
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
    rc = p->head_dim == kWideD
             ? launch_prefill_gqa_prep(p, q_raw, k_raw, v_raw, q_norm_w, k_norm_w, k_cache, v_cache, capacity, batch,
                                       tokens, pos0, workspace, static_cast<cudaStream_t>(stream))
             : launch_prep(p, q_raw, k_raw, v_raw, q_norm_w, k_norm_w, k_cache, v_cache, capacity, batch, tokens,
                           pos0, workspace, static_cast<cudaStream_t>(stream));
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
    rc = p->head_dim == kWideD
             ? launch_prefill_gqa_attend(p, workspace, k_cache, v_cache, capacity, batch, tokens, pos0, out,
                                         static_cast<cudaStream_t>(stream))
             : launch_attend(p, workspace, k_cache, v_cache, capacity, batch, tokens, pos0, out,
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
    if (p->head_dim == kWideD) {
        rc = launch_prefill_gqa_prep(p, q_raw, k_raw, v_raw, q_norm_w, k_norm_w, k_cache, v_cache, capacity, batch,
                                     tokens, pos0, workspace, s);
        if (rc) return rc;
        rc = launch_prefill_gqa_attend(p, workspace, k_cache, v_cache, capacity, batch, tokens, pos0, out, s);
        return rc ? rc : ok();
    }
    rc = launch_prep(p, q_raw, k_raw, v_raw, q_norm_w, k_norm_w, k_cache, v_cache, capacity, batch, tokens, pos0,
                     workspace, s);
    if (rc) return rc;
    rc = launch_attend(p, workspace, k_cache, v_cache, capacity, batch, tokens, pos0, out, s);
    return rc ? rc : ok();
}
