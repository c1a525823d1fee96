// decode_splitkv.cu -- fused single-token decode over a bf16 KV cache (split-KV), plus the
// log-sum-exp merge of per-GPU partials.
//
// Reference semantics: the new token's q is normalised and roped (shaders/head_norm_rope.metal,
// called on q at docs/B6_3_attention.md:445-446), its k/v are normalised (k also roped) and
// written into the cache at position L-1 (docs/B6_3_attention.md:448-452), then the softmax
// over the visible keys is taken per q head with the GQA map h / (Hq/Hkv) and the window rule
// (attention_f32, docs/B6_3_attention.md:296-343).  Decode is T = 1 of that same kernel
// (docs/B6_3_attention.md:95-97).
//
// B200 design (HBM-bound): work item = (sequence b, kv head, split of `chunk` positions).
// One CTA = 4 consumer warps + 1 producer warp.  The producer streams contiguous runs of K
// and V rows ([pos][256] bf16, 512 B each) with 1-D TMA bulk copies into a 3-stage ring of
// 32 positions (16 KB K + 16 KB V per stage), so every byte of the cache is read once, in
// 16 KB bursts, by the copy engine.  Each consumer warp owns 8 positions of a stage and keeps
// a private online softmax for BOTH q heads of the GQA group (the K/V row is read once for
// both): lane l holds dims [8l, 8l+8) of q and of the accumulators; one 128-bit shared load
// per lane reads a whole 512 B row; the 16 partial dot products (8 positions x 2 heads) are
// reduced with a 16-shuffle transposed butterfly that leaves one finished score per lane.
// Scores live in the log2 domain (q is pre-scaled by scale*log2(e)), so exponentials are
// single ex2 instructions.  Warps merge once per CTA; the last CTA of each (b, kv head)
// (atomic counter, no spin) merges the split partials and writes bf16 -- one launch per step.
#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "row256.cuh"

namespace apex {
namespace {

constexpr int kD = 256;                 // head_dim
constexpr int kG = 2;                   // q heads per kv head (GQA group)
constexpr int kPosPerWarp = 8;          // positions one consumer warp takes from a stage
constexpr int kRowBytes = kD * 2;
// Split-KV form: 4 consumer warps, stages of 32 positions, a 3-stage ring, 2 CTAs per SM.
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kStagePos = kConsumerWarps * kPosPerWarp;
constexpr int kStages = 3;
// Cluster form (short contexts): 8 consumer warps, stages of 64 positions, a 1- or 2-stage ring; the
// splits of one (sequence, kv head) form one thread-block cluster and merge in the leader CTA's
// shared memory.
constexpr int kShortWarps = 8;
constexpr int kShortStagePos = kShortWarps * kPosPerWarp;
constexpr uint32_t kMaxCluster = 16;
constexpr uint32_t kShortMaxLen = 4096;  // longest context the cluster form is chosen for
constexpr int kPart = kD + 2;           // public partial record: o[D], m, l
constexpr int kWsRec = kD + 4;          // workspace record: o[D], m, l, pad (16-byte multiple)
constexpr int kLLRec = kD + 2;          // peer gather record: o[D], m, l as 8-byte (step, value) words
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint32_t kMaxPeers = 8;       // GPUs of one NVLink domain that share a KV range

struct DecodeArgs {
    const uint16_t *q_raw, *k_new, *v_new, *q_w, *k_w;
    uint16_t *k_cache, *v_cache;
    const int32_t *seq_lens;
    uint16_t *out;       // [B][Hq][D] bf16 (full mode)
    float *partial_out;  // [B][Hq][D+2]   (partial mode)
    float *ws_part;      // [B][Hq][max_splits][D+4]
    unsigned *ws_count;  // [B][Hkv]
    unsigned *status;    // device status word
    uint32_t capacity, q_heads, kv_heads, rope_pairs, window, qk_norm, v_norm;
    uint32_t chunk, max_splits, kv_begin, kv_end, max_seq_len;
    uint32_t ring;       // 1: position p of the cache is slot p % capacity (window <= capacity)
    float rope_base, eps, scale_log2;
    int partial_mode;
    // peer mode (a KV range split over `world` GPUs): this rank's partial goes straight into every
    // rank's gather buffer over NVLink, a per-step sequence flag follows it, and the rank merges
    // all partials itself once every rank's flag has arrived (no collective launch, no merge launch)
    int peer_mode;
    uint32_t rank, world;
    float *peer_gather[kMaxPeers];    // rank r's [2 step parity][world][B*Hq][D+2] (step, f32) words, mapped here
    unsigned *peer_flags[kMaxPeers];  // rank r's [world][B*Hkv] last published step
    unsigned *peer_seq;               // this rank's [B*Hkv] step counters
    unsigned long long peer_wait_ns;  // bound of the wait for the other ranks' flags
    RopeTable rope;      // inv_freq[i] = rope_base^(-2i/256)
};

// Peer mode: a step counter or flag with this bit set is poisoned -- some rank's wait for this
// (sequence, kv head) gave up, so the two-slot ordering of the gather buffers no longer holds.
// Every later step of that pair on every rank reports a timeout and writes nothing.
constexpr unsigned kPeerPoison = 0x80000000u;
constexpr unsigned long long kPeerWaitDefaultNs = 1000000000ull;  // one second

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

template <int CW, int ST, bool CL>
struct __align__(16) DecodeSmemT {
    uint8_t k[ST][CW * kPosPerWarp * kRowBytes];
    uint8_t v[ST][CW * kPosPerWarp * kRowBytes];
    float q[kG][kD];
    uint16_t new_k[kD];
    uint16_t new_v[kD];
    float rope_cs[kD / 2], rope_sn[kD / 2];  // cos, sin of the new position per pair
    float wm[CW][kG], wl[CW][kG];
    float red[CW][kG];
    float parts[CL ? kMaxCluster : 1][kG][kWsRec];  // cluster form: every split's partial (leader)
    uint64_t full[ST], empty[ST];
    uint64_t gather;                                 // cluster form: one arrival per split (leader)
    int is_last;
};
using DecodeSmem = DecodeSmemT<kConsumerWarps, kStages, false>;

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Relaxed system-scope access to the poison flags (the data words carry their own step number).
__device__ __forceinline__ unsigned ld_relaxed_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
template <int CW = kConsumerWarps>
__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(CW * 32) : "memory");
}
// Cluster barrier halves (not warp-aligned: the producer warp's lanes diverge).
__device__ __forceinline__ void cluster_wait_acquire() { asm volatile("barrier.cluster.wait.acquire;" ::: "memory"); }
// Store two floats into another CTA's shared memory (cluster address), counted in bytes on that
// CTA's mbarrier (complete_tx): the receiver's wait on the barrier is all the ordering needed.
__device__ __forceinline__ void st_async_f32x2(uint32_t addr, float x, float y, uint32_t remote_bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(addr),
                 "f"(x), "f"(y), "r"(remote_bar)
                 : "memory");
}
__device__ __forceinline__ void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory"); }

// Online-softmax update of one warp with up to 8 key/value rows (row j at kbase/vbase +
// j*512 bytes in shared memory).  State: m[g] (log2 units, warp-uniform), lpart (this lane's
// share of l for head (lane>>1)&1), acc[g][8] (dims [8l, 8l+8) of head g).
__device__ __forceinline__ void warp_step(const uint8_t *kbase, const uint8_t *vbase, int nvalid,
                                          uint32_t lane, const float (&qf)[kG][8],
                                          float (&m)[kG], float &lpart, float (&acc)[kG][8]) {
    float part[16];
#pragma unroll
    for (int j = 0; j < kPosPerWarp; ++j) {
        if (j < nvalid) {
            const uint4 raw = *reinterpret_cast<const uint4 *>(kbase + j * kRowBytes + lane * 16);
            float kf[8];
            unpack8(raw, kf);
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                s0 = fmaf(qf[0][e], kf[e], s0);
                s1 = fmaf(qf[1][e], kf[e], s1);
            }
            part[2 * j] = s0;
            part[2 * j + 1] = s1;
        } else {
            part[2 * j] = 0.f;
            part[2 * j + 1] = 0.f;
        }
    }
    // Transposed butterfly: after the 5 rounds lane l holds the full score of value index
    // l >> 1 = 2*j + g, i.e. position j = l >> 2 and head g = (l >> 1) & 1.
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4, b1 = lane & 2;
    float r1[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float keep = b4 ? part[i + 8] : part[i];
        const float send = b4 ? part[i] : part[i + 8];
        r1[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    float r2[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float keep = b3 ? r1[i + 4] : r1[i];
        const float send = b3 ? r1[i] : r1[i + 4];
        r2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    float r3[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float keep = b2 ? r2[i + 2] : r2[i];
        const float send = b2 ? r2[i] : r2[i + 2];
        r3[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    float s = (b1 ? r3[1] : r3[0]) + __shfl_xor_sync(0xffffffffu, b1 ? r3[0] : r3[1], 2);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    const int my_j = lane >> 2;
    const int my_g = (lane >> 1) & 1;
    if (my_j >= nvalid) s = -INFINITY;

    float mx = s;
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
    const float mo = __shfl_xor_sync(0xffffffffu, mx, 2);
    float m_new[kG], alpha[kG];
    m_new[0] = fmaxf(m[0], my_g == 0 ? mx : mo);
    m_new[1] = fmaxf(m[1], my_g == 0 ? mo : mx);
#pragma unroll
    for (int g = 0; g < kG; ++g) alpha[g] = fast_exp2(m[g] - m_new[g]);  // 0 when m = -inf
    // selects, not m_new[my_g] / alpha[my_g]: a lane-dependent index would put the arrays on the stack
    const float p = fast_exp2(s - (my_g ? m_new[1] : m_new[0]));         // 0 for invalid rows
    lpart = lpart * (my_g ? alpha[1] : alpha[0]) + p;
#pragma unroll
    for (int g = 0; g < kG; ++g) {
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g][e] *= alpha[g];
        m[g] = m_new[g];
    }
    // Every probability and V row first (independent shuffles and shared loads in flight together),
    // then the accumulation.  Rows past nvalid read as zero (their p is 0; stale shared memory
    // could hold non-finite bits).
    float p0[kPosPerWarp], p1[kPosPerWarp];
    uint4 vraw[kPosPerWarp];
#pragma unroll
    for (int j = 0; j < kPosPerWarp; ++j) {
        p0[j] = __shfl_sync(0xffffffffu, p, 4 * j);
        p1[j] = __shfl_sync(0xffffffffu, p, 4 * j + 2);
        vraw[j] = j < nvalid ? *reinterpret_cast<const uint4 *>(vbase + j * kRowBytes + lane * 16)
                             : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int j = 0; j < kPosPerWarp; ++j) {
        float vf[8];
        unpack8(vraw[j], vf);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            acc[0][e] = fmaf(p0[j], vf[e], acc[0][e]);
            acc[1][e] = fmaf(p1[j], vf[e], acc[1][e]);
        }
    }
}

// Max (or sum) over the 128 consumer threads of one value per head, using red[][] in shared
// memory; every consumer thread gets the result.
template <bool kMax, int CW = kConsumerWarps>
__device__ __forceinline__ void consumer_reduce(float (&v)[kG], float (&red)[CW][kG], uint32_t warp,
                                                uint32_t lane) {
#pragma unroll
    for (int g = 0; g < kG; ++g) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float t = __shfl_xor_sync(0xffffffffu, v[g], o);
            v[g] = kMax ? fmaxf(v[g], t) : v[g] + t;
        }
        if (lane == 0) red[warp][g] = v[g];
    }
    consumer_sync();
#pragma unroll
    for (int g = 0; g < kG; ++g) {
        float r = red[0][g];
#pragma unroll
        for (int w = 1; w < CW; ++w) r = kMax ? fmaxf(r, red[w][g]) : r + red[w][g];
        v[g] = r;
    }
    consumer_sync<CW>();
}

// Peer mode: publish this rank's partial of (b, kv head) -- thread t holds head g = t / 64, dims
// [d0, d0+4) of the normalised o, and (m, l) when d0 = 0 -- to every rank, then merge all ranks'
// partials into bf16 out.  Every value travels as one 8-byte word (step << 32 | float bits) written
// with 16-byte stores of two words; an aligned 8-byte word is written and read as a whole, so a
// reader that polls its own words until their step matches this step has the data without any
// flag or fence (a system-scope fence per published partial, which waits for the NVLink stores to
// be acknowledged, cost more than the wait itself).  Steps alternate between two gather slots, so a
// rank that runs ahead never overwrites data a slower peer is still merging (it cannot start step
// k+2 before it has read every peer's step k+1, which each peer publishes only after finishing step
// k).  The wait is bounded (a.peer_wait_ns): on expiry, or when a peer's poison flag is set, the
// status word gets kStatusTimeout, the output is left unwritten, and this pair's counter and this
// rank's poison flag on every peer are set, so that no rank publishes into or merges from the
// gather slots again (the ordering above assumed a wait that succeeded).
__device__ __forceinline__ void st_sys_v2(uint64_t *p, uint64_t x, uint64_t y) {
    asm volatile("st.relaxed.sys.global.v2.b64 [%0], {%1, %2};" ::"l"(p), "l"(x), "l"(y) : "memory");
}
__device__ __forceinline__ void ld_sys_v2(const uint64_t *p, uint64_t &x, uint64_t &y) {
    asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(x), "=l"(y) : "l"(p) : "memory");
}
__device__ __forceinline__ uint64_t ll_word(unsigned seq, float v) {
    return (static_cast<uint64_t>(seq) << 32) | __float_as_uint(v);
}
__device__ __forceinline__ float ll_value(uint64_t w) { return __uint_as_float(static_cast<unsigned>(w)); }
__device__ __forceinline__ bool ll_is(uint64_t w, unsigned seq) { return static_cast<unsigned>(w >> 32) == seq; }

__device__ void peer_publish_merge(const DecodeArgs &a, DecodeSmem &sm, uint32_t b, uint32_t kvh, uint32_t tid,
                                   uint32_t g, uint32_t d0, const float (&o)[4], float m, float l) {
    const uint32_t bhkv = gridDim.z * a.kv_heads, bkv = b * a.kv_heads + kvh;
    const uint64_t rows = static_cast<uint64_t>(gridDim.z) * a.q_heads;
    const uint64_t row = static_cast<uint64_t>(b) * a.q_heads + kvh * kG + g;
    const unsigned prev = *reinterpret_cast<volatile unsigned *>(a.peer_seq + bkv);
    if (prev & kPeerPoison) {  // an earlier step gave up: publish nothing, merge nothing
        if (tid == 0) atomicOr(a.status, kStatusTimeout);
        return;
    }
    const unsigned seq = prev + 1u;
    const uint32_t par = seq & 1u;
    for (uint32_t p = 0; p < a.world; ++p) {
        uint64_t *dst = reinterpret_cast<uint64_t *>(a.peer_gather[p]) +
                        ((static_cast<uint64_t>(par) * a.world + a.rank) * rows + row) * kLLRec;
        st_sys_v2(dst + d0, ll_word(seq, o[0]), ll_word(seq, o[1]));
        st_sys_v2(dst + d0 + 2, ll_word(seq, o[2]), ll_word(seq, o[3]));
        if (d0 == 0) st_sys_v2(dst + kD, ll_word(seq, m), ll_word(seq, l));
    }
    // every thread waits for its own words (and the head's m, l) of every rank
    const uint64_t *base = reinterpret_cast<const uint64_t *>(a.peer_gather[a.rank]) +
                           static_cast<uint64_t>(par) * a.world * rows * kLLRec;
    float ov[kMaxPeers][4], mr[kMaxPeers], lr[kMaxPeers];
    bool ok = true;
    const unsigned long long start = globaltimer_ns();
#pragma unroll
    for (uint32_t r = 0; r < kMaxPeers; ++r) {
        mr[r] = -INFINITY;
        lr[r] = 0.f;
        if (r >= a.world || !ok) continue;
        const uint64_t *src = base + (r * rows + row) * kLLRec;
        for (;;) {
            uint64_t w0, w1, w2, w3, w4, w5;
            ld_sys_v2(src + d0, w0, w1);
            ld_sys_v2(src + d0 + 2, w2, w3);
            ld_sys_v2(src + kD, w4, w5);
            if (ll_is(w0, seq) && ll_is(w1, seq) && ll_is(w2, seq) && ll_is(w3, seq) && ll_is(w4, seq) &&
                ll_is(w5, seq)) {
                ov[r][0] = ll_value(w0);
                ov[r][1] = ll_value(w1);
                ov[r][2] = ll_value(w2);
                ov[r][3] = ll_value(w3);
                mr[r] = ll_value(w4);
                lr[r] = ll_value(w5);
                break;
            }
            if ((ld_relaxed_sys(a.peer_flags[a.rank] + r * bhkv + bkv) & kPeerPoison) ||  // that rank gave up
                globaltimer_ns() - start > a.peer_wait_ns) {
                ok = false;
                break;
            }
            __nanosleep(32);
        }
    }
    if (tid == 0) sm.is_last = 1;
    consumer_sync();
    if (!ok) sm.is_last = 0;
    consumer_sync();
    if (!sm.is_last) {
        if (tid == 0) {
            atomicOr(a.status, kStatusTimeout);
            a.peer_seq[bkv] = seq | kPeerPoison;
            for (uint32_t p = 0; p < a.world; ++p)
                st_release_sys(a.peer_flags[p] + a.rank * bhkv + bkv, seq | kPeerPoison);
        }
        return;
    }
    if (tid == 0) a.peer_seq[bkv] = seq;
    // log-sum-exp merge over the ranks (each partial: o normalised by its l, l relative to its m)
    float M = -INFINITY;
#pragma unroll
    for (uint32_t r = 0; r < kMaxPeers; ++r)
        if (lr[r] > 0.f) M = fmaxf(M, mr[r]);
    float den = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (uint32_t r = 0; r < kMaxPeers; ++r) {
        if (!(lr[r] > 0.f)) continue;
        const float wt = fast_exp2(mr[r] - M) * lr[r];
        den += wt;
        acc[0] += wt * ov[r][0];
        acc[1] += wt * ov[r][1];
        acc[2] += wt * ov[r][2];
        acc[3] += wt * ov[r][3];
    }
    const float inv = den > 0.f ? 1.0f / den : 0.f;
    uint2 packed;
    packed.x = pack_bf16(acc[0] * inv, acc[1] * inv);
    packed.y = pack_bf16(acc[2] * inv, acc[3] * inv);
    *reinterpret_cast<uint2 *>(a.out + row * kD + d0) = packed;
}

// The decode step, in two forms.
//   CL = false (CW = 4, ST = 3): split-KV.  Any number of splits per (b, kv head); the last CTA of
//     each (found with an atomic counter, no spinning) merges the split partials from the
//     workspace.  Also the partial and peer (KV split over GPUs) modes.
//   CL = true (CW = 8, ST = 1 or 2): the splits of one (b, kv head) are one thread-block cluster
//     of gridDim.x <= 16 CTAs.  Every split pushes its partial into the leader CTA's shared memory
//     with asynchronous distributed-shared-memory stores counted on the leader's mbarrier, and the
//     leader merges -- no workspace round trip, no fence + atomic, no second pass through L2, which
//     at short contexts is most of the step.  No CTA returns before its pushes are issued.
// Global attention (window 0): a split's first stage does not depend on the sequence length, so the
// producer requests it before anything else -- before the length load -- and the consumers mask the
// rows past the length (the cache holds `capacity` positions, so the extra rows are in bounds).
template <int CW, int ST, bool CL>
__global__ void __launch_bounds__((CW + 1) * 32, (CL && ST > 1) ? 1 : 2)
    decode_kernel(const __grid_constant__ DecodeArgs a) {
    using Smem = DecodeSmemT<CW, ST, CL>;
    constexpr int SP = CW * kPosPerWarp;          // positions per stage
    constexpr int DPT = kG * kD / (CW * 32);      // output dims per consumer thread in the merges
    static_assert(CL || CW == kConsumerWarps, "the split-KV form has 4 consumer warps");
    static_assert(!CL || DPT == 2, "the cluster form pushes two dims per thread");
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Smem &sm = *reinterpret_cast<Smem *>(smem_raw);

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const uint32_t Hq = a.q_heads;
    const uint64_t head_base =
        (static_cast<uint64_t>(b) * a.kv_heads + kvh) * a.capacity * kD;  // element offset

    // ---- barriers and the speculative first stage, by the producer lane, before the length load
    const uint32_t spec_off = split * a.chunk;  // local cache index of this split's first key (window 0)
    const uint32_t spec_rows = (a.window == 0 && spec_off < a.capacity) ? min(static_cast<uint32_t>(SP), a.capacity - spec_off) : 0u;
    if (warp == CW && lane == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(smem_u32(&sm.full[s]), 1);
            mbar_init(smem_u32(&sm.empty[s]), CW);
        }
        if constexpr (CL) mbar_init(smem_u32(&sm.gather), 1);
        fence_mbar_init();
        if (spec_rows) {
            const uint32_t full = smem_u32(&sm.full[0]);
            mbar_arrive_expect_tx(full, 2 * spec_rows * kRowBytes);
            tma_bulk_load(smem_u32(sm.k[0]), a.k_cache + head_base + static_cast<uint64_t>(spec_off) * kD,
                          spec_rows * kRowBytes, full);
            tma_bulk_load(smem_u32(sm.v[0]), a.v_cache + head_base + static_cast<uint64_t>(spec_off) * kD,
                          spec_rows * kRowBytes, full);
        }
        // cluster form, leader: every split's partial (two heads x (D + 2) floats) is expected here
        if constexpr (CL)
            if (split == 0) mbar_arrive_expect_tx(smem_u32(&sm.gather), gridDim.x * kG * (kD + 2) * 4);
    }
    __syncthreads();
    // cluster form: every CTA's barriers are initialised before any CTA reaches the pushes below
    if constexpr (CL) cluster_arrive_relaxed();

    // ---- key range of this (b, kv head) and of this split (global positions)
    const int32_t L = a.seq_lens[b];
    const bool bad = L < 0 || static_cast<uint32_t>(L) > a.max_seq_len ||
                     (!a.ring && L > 0 && static_cast<uint32_t>(L) - 1 >= a.kv_begin + a.capacity &&
                      static_cast<uint32_t>(L) - 1 < a.kv_end);
    const uint32_t Lu = bad ? 0u : static_cast<uint32_t>(L);
    const uint32_t pos_new = Lu - 1;  // only meaningful when Lu >= 1
    const uint32_t first = (a.window && Lu > a.window) ? Lu - a.window : 0;
    const uint32_t kb = max(first, a.kv_begin);
    const uint32_t ke = min(Lu, a.kv_end);
    const uint32_t n_keys = ke > kb ? ke - kb : 0;
    const uint32_t nsplit = n_keys ? (n_keys + a.chunk - 1) / a.chunk : 1;
    if (bad && split == 0 && tid == 0 && kvh == 0) atomicOr(a.status, kStatusBadLength);
    // A cluster split without keys still takes part: it pushes an empty partial (l = 0).
    bool idle = split >= nsplit;
    if constexpr (!CL) {
        if (idle || nsplit > a.max_splits) {  // the second cannot happen for lengths <= max_seq_len
            if (!idle && tid == 0) atomicOr(a.status, kStatusBadLength);
            // the speculative copy lands before the CTA leaves
            if (spec_rows && tid == 0) mbar_wait(smem_u32(&sm.full[0]), 0, a.status);
            return;
        }
    } else if (nsplit > gridDim.x) {  // cannot happen for lengths <= max_seq_len
        if (split == 0 && tid == 0) atomicOr(a.status, kStatusBadLength);
        idle = true;
    }
    const uint32_t lo = kb + split * a.chunk;
    const uint32_t hi = (n_keys && !idle) ? min(lo + a.chunk, ke) : lo;
    const bool has_new = n_keys && !idle && pos_new >= lo && pos_new < hi;
    const uint32_t cache_hi = has_new ? pos_new : hi;
    const uint32_t n_cached = cache_hi > lo ? cache_hi - lo : 0;
    const uint32_t n_stages = (n_cached + SP - 1) / SP;
    const uint32_t n_wait = max(n_stages, spec_rows ? 1u : 0u);  // stages whose copies land here

    const uint16_t *kc = a.k_cache + head_base + static_cast<uint64_t>(lo - a.kv_begin) * kD;
    const uint16_t *vc = a.v_cache + head_base + static_cast<uint64_t>(lo - a.kv_begin) * kD;
    const uint32_t new_slot = a.ring ? pos_new % a.capacity : pos_new - a.kv_begin;

    if (warp == CW) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            for (uint32_t s = spec_rows ? 1u : 0u; s < n_stages; ++s) {
                const uint32_t slot = s % ST;
                if (s >= ST && !mbar_wait(smem_u32(&sm.empty[slot]), ((s / ST) - 1) & 1, a.status)) break;
                const uint32_t p0 = s * SP;
                const uint32_t n = min(static_cast<uint32_t>(SP), n_cached - p0);
                const uint32_t bytes = n * kRowBytes;
                const uint32_t full = smem_u32(&sm.full[slot]);
                mbar_arrive_expect_tx(full, 2 * bytes);
                if (!a.ring) {
                    tma_bulk_load(smem_u32(sm.k[slot]), kc + static_cast<uint64_t>(p0) * kD, bytes, full);
                    tma_bulk_load(smem_u32(sm.v[slot]), vc + static_cast<uint64_t>(p0) * kD, bytes, full);
                } else {  // slots (lo + p0) % capacity onward, in two runs where the ring wraps
                    const uint32_t i0 = (lo + p0) % a.capacity, n1 = min(n, a.capacity - i0);
                    const uint16_t *kr = a.k_cache + head_base, *vr = a.v_cache + head_base;
                    tma_bulk_load(smem_u32(sm.k[slot]), kr + static_cast<uint64_t>(i0) * kD, n1 * kRowBytes, full);
                    tma_bulk_load(smem_u32(sm.v[slot]), vr + static_cast<uint64_t>(i0) * kD, n1 * kRowBytes, full);
                    if (n1 < n) {
                        tma_bulk_load(smem_u32(sm.k[slot]) + n1 * kRowBytes, kr, (n - n1) * kRowBytes, full);
                        tma_bulk_load(smem_u32(sm.v[slot]) + n1 * kRowBytes, vr, (n - n1) * kRowBytes, full);
                    }
                }
            }
        }
        if constexpr (CL) {  // both cluster barrier phases, like every thread of the cluster
            cluster_wait_acquire();
            cluster_arrive_relaxed();
            cluster_wait_acquire();
        }
        return;
    }

    // -------------------------------------------------------------------- consumers
    // This warp's row (q of head kvh*G + warp for warps 0..G-1; the new k / v for warps G, G+1 of
    // the split that owns the new position) and its norm weights are loaded first, so their latency
    // overlaps the cos/sin table below.
    const bool row_q = warp < kG, row_kv = warp >= kG && warp < kG + 2 && has_new, is_k = warp == kG;
    uint4 raw = make_uint4(0u, 0u, 0u, 0u);
    float wv[8];
    {
        const uint16_t *src = row_q ? a.q_raw + (static_cast<uint64_t>(b) * Hq + kvh * kG + warp) * kD
                                    : (is_k ? a.k_new : a.v_new) + (static_cast<uint64_t>(b) * a.kv_heads + kvh) * kD;
        const uint16_t *w = row_q ? a.q_w : (is_k ? a.k_w : nullptr);
        if (row_q || row_kv) raw = *reinterpret_cast<const uint4 *>(src + 8 * lane);
#pragma unroll
        for (int e = 0; e < 8; ++e)
            wv[e] = w && (row_q || row_kv) ? __uint_as_float(static_cast<uint32_t>(w[8 * lane + e]) << 16) : 1.0f;
    }
    // cos/sin of the new position, one pair per consumer thread
    const float pos_f = static_cast<float>(pos_new);
    for (uint32_t i = tid; i < a.rope_pairs; i += CW * 32)
        rope_sincos(pos_f * a.rope.inv_freq[i], sm.rope_sn[i], sm.rope_cs[i]);
    consumer_sync<CW>();
    if (row_q) {
        // q: norm + rope at the new position, pre-scaled for exp2
        float x[8];
        unpack8(raw, x);
        norm_rope_row_tab(x, lane, a.qk_norm, wv, a.eps, a.rope_pairs, sm.rope_cs, sm.rope_sn);
#pragma unroll
        for (int e = 0; e < 8; ++e) sm.q[warp][8 * lane + e] = x[e] * a.scale_log2;
    } else if (row_kv) {
        // new k: norm + rope; new v: optional weightless norm.  Both are rounded to bf16 once, stored
        // to the cache and kept in shared memory for this split.
        float x[8];
        unpack8(raw, x);
        if (is_k)
            norm_rope_row_tab(x, lane, a.qk_norm, wv, a.eps, a.rope_pairs, sm.rope_cs, sm.rope_sn);
        else
            norm_rope_row_tab(x, lane, a.v_norm, wv, a.eps, 0, sm.rope_cs, sm.rope_sn);
        const uint4 packed = pack8(x);
        *reinterpret_cast<uint4 *>((is_k ? sm.new_k : sm.new_v) + 8 * lane) = packed;
        uint16_t *dst = (is_k ? a.k_cache : a.v_cache) + head_base + static_cast<uint64_t>(new_slot) * kD;
        *reinterpret_cast<uint4 *>(dst + 8 * lane) = packed;
    }
    consumer_sync<CW>();

    float qf[kG][8];
#pragma unroll
    for (int g = 0; g < kG; ++g)
#pragma unroll
        for (int e = 0; e < 8; ++e) qf[g][e] = sm.q[g][8 * lane + e];

    float m[kG] = {-INFINITY, -INFINITY};
    float lpart = 0.f;
    float acc[kG][8];
#pragma unroll
    for (int g = 0; g < kG; ++g)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g][e] = 0.f;

    for (uint32_t s = 0; s < n_wait; ++s) {
        const uint32_t slot = s % ST;
        if (!mbar_wait(smem_u32(&sm.full[slot]), (s / ST) & 1, a.status)) break;
        const int n = s < n_stages ? static_cast<int>(min(static_cast<uint32_t>(SP), n_cached - s * SP)) : 0;
        const int nvalid = min(max(n - static_cast<int>(warp) * kPosPerWarp, 0), kPosPerWarp);
        if (nvalid > 0)
            warp_step(sm.k[slot] + warp * kPosPerWarp * kRowBytes,
                      sm.v[slot] + warp * kPosPerWarp * kRowBytes, nvalid, lane, qf, m, lpart, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&sm.empty[slot]));
    }
    if (has_new && warp == 0)
        warp_step(reinterpret_cast<const uint8_t *>(sm.new_k),
                  reinterpret_cast<const uint8_t *>(sm.new_v), 1, lane, qf, m, lpart, acc);

    // ---- per-warp l: sum this lane's share over the 8 positions of its head
    float lt = lpart;
    lt += __shfl_xor_sync(0xffffffffu, lt, 4);
    lt += __shfl_xor_sync(0xffffffffu, lt, 8);
    lt += __shfl_xor_sync(0xffffffffu, lt, 16);
    const float lother = __shfl_xor_sync(0xffffffffu, lt, 2);
    const int my_g = (lane >> 1) & 1;
    consumer_sync<CW>();  // every warp is done with the stage buffers: reuse them for the merge
    float *wacc = reinterpret_cast<float *>(sm.k[0]);  // [warps][G][D] f32
    if (lane == 0) {
        sm.wm[warp][0] = m[0];
        sm.wm[warp][1] = m[1];
        sm.wl[warp][0] = my_g == 0 ? lt : lother;
        sm.wl[warp][1] = my_g == 0 ? lother : lt;
    }
#pragma unroll
    for (int g = 0; g < kG; ++g)
#pragma unroll
        for (int e = 0; e < 8; ++e) wacc[(warp * kG + g) * kD + 8 * lane + e] = acc[g][e];
    consumer_sync<CW>();

    // ---- CTA merge: thread t owns head g, dims [d0, d0 + DPT)
    const uint32_t g = tid / (kD / DPT), d0 = (tid % (kD / DPT)) * DPT;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < CW; ++w)
        if (sm.wl[w][g] > 0.f) M = fmaxf(M, sm.wm[w][g]);
    float den = 0.f, o[DPT];
#pragma unroll
    for (int e = 0; e < DPT; ++e) o[e] = 0.f;
#pragma unroll
    for (int w = 0; w < CW; ++w) {
        if (!(sm.wl[w][g] > 0.f)) continue;
        const float wt = fast_exp2(sm.wm[w][g] - M);
        den += wt * sm.wl[w][g];
#pragma unroll
        for (int e = 0; e < DPT; ++e) o[e] += wt * wacc[(w * kG + g) * kD + d0 + e];
    }
    const float inv_den = den > 0.f ? 1.0f / den : 0.f;
#pragma unroll
    for (int e = 0; e < DPT; ++e) o[e] *= inv_den;
    const uint32_t h = kvh * kG + g;
    const uint64_t row = static_cast<uint64_t>(b) * Hq + h;

    if constexpr (CL) {
        // ---- push this split's partial into the leader's shared memory (counted on its barrier)
        cluster_wait_acquire();  // the leader's barrier and buffer are initialised
        const uint32_t leader_rec = mapa(smem_u32(&sm.parts[split][g][0]), 0);
        const uint32_t leader_bar = mapa(smem_u32(&sm.gather), 0);
        st_async_f32x2(leader_rec + d0 * 4, o[0], o[1], leader_bar);
        if (d0 == 0) st_async_f32x2(leader_rec + kD * 4, M, den, leader_bar);
        // The second cluster barrier phase keeps every CTA resident until the leader has merged
        // (so the pushes of a CTA that is done have certainly landed before it exits).
        if (split != 0 || !mbar_wait_cluster(smem_u32(&sm.gather), 0, a.status)) {
            cluster_arrive_relaxed();
            cluster_wait_acquire();
            return;
        }
        // ---- leader: log-sum-exp merge of the cluster's partials
        float Mx = -INFINITY;
        for (uint32_t s = 0; s < gridDim.x; ++s) {
            const float *p = sm.parts[s][g];
            if (p[kD + 1] > 0.f) Mx = fmaxf(Mx, p[kD]);
        }
        float dt = 0.f, r[DPT];
#pragma unroll
        for (int e = 0; e < DPT; ++e) r[e] = 0.f;
        for (uint32_t s = 0; s < gridDim.x; ++s) {
            const float *p = sm.parts[s][g];
            if (!(p[kD + 1] > 0.f)) continue;
            const float wt = fast_exp2(p[kD] - Mx) * p[kD + 1];
            dt += wt;
#pragma unroll
            for (int e = 0; e < DPT; ++e) r[e] += wt * p[d0 + e];
        }
        const float inv = dt > 0.f ? 1.0f / dt : 0.f;
#pragma unroll
        for (int e = 0; e < DPT; e += 2)
            *reinterpret_cast<uint32_t *>(a.out + row * kD + d0 + e) = pack_bf16(r[e] * inv, r[e + 1] * inv);
        cluster_arrive_relaxed();
        cluster_wait_acquire();
        return;
    } else {
        if (nsplit == 1) {
            if (a.peer_mode) {
                peer_publish_merge(a, sm, b, kvh, tid, g, d0, o, M, den);
            } else if (a.partial_mode) {
                float *dst = a.partial_out + row * kPart;
#pragma unroll
                for (int e = 0; e < 4; ++e) dst[d0 + e] = o[e];
                if (d0 == 0) {
                    dst[kD] = M;
                    dst[kD + 1] = den;
                }
            } else {
                uint2 packed;
                packed.x = pack_bf16(o[0], o[1]);
                packed.y = pack_bf16(o[2], o[3]);
                *reinterpret_cast<uint2 *>(a.out + row * kD + d0) = packed;
            }
            return;
        }

        // ---- split partial -> workspace; the last CTA of (b, kv head) merges all splits
        float *mine = a.ws_part + (row * a.max_splits + split) * kWsRec;
#pragma unroll
        for (int e = 0; e < 4; ++e) mine[d0 + e] = o[e];
        if (d0 == 0) {
            mine[kD] = M;
            mine[kD + 1] = den;
        }
        consumer_sync();
        if (tid == 0) {
            // the barrier orders every consumer's partial before this thread's release fence, which
            // then publishes them all to the CTA that sees the count complete
            __threadfence();
            unsigned *counter = a.ws_count + static_cast<uint64_t>(b) * a.kv_heads + kvh;
            const unsigned prev = atomicAdd(counter, 1u);
            const int last = prev == nsplit - 1;
            if (last) *counter = 0;  // ready for the next call
            sm.is_last = last;
        }
        consumer_sync();
        if (!sm.is_last) return;
        __threadfence();
        // Parallel log-sum-exp merge of the nsplit partials of both heads: per-split (m, l) staged in
        // shared memory (the stage buffers are free), block reductions for the max and the sum,
        // then each thread accumulates its 4 dims over the splits with independent 16-byte loads.
        const float *parts0 = a.ws_part + (static_cast<uint64_t>(b) * Hq + kvh * kG) * a.max_splits * kWsRec;
        float *ms = reinterpret_cast<float *>(sm.v[0]);  // [G][nsplit] m, then the weights
        float *ls = ms + kG * nsplit;                      // [G][nsplit] l
        float mx[kG] = {-INFINITY, -INFINITY};
        for (uint32_t s = tid; s < nsplit; s += kConsumerWarps * 32) {
#pragma unroll
            for (int gg = 0; gg < kG; ++gg) {
                const float *p = parts0 + (static_cast<uint64_t>(gg) * a.max_splits + s) * kWsRec;
                const float2 ml = __ldcg(reinterpret_cast<const float2 *>(p + kD));
                ms[gg * nsplit + s] = ml.x;
                ls[gg * nsplit + s] = ml.y;
                if (ml.y > 0.f) mx[gg] = fmaxf(mx[gg], ml.x);
            }
        }
        consumer_reduce<true>(mx, sm.red, warp, lane);
        float dsum[kG] = {0.f, 0.f};
        for (uint32_t s = tid; s < nsplit; s += kConsumerWarps * 32) {
#pragma unroll
            for (int gg = 0; gg < kG; ++gg) {
                const float l_s = ls[gg * nsplit + s];
                const float wt = l_s > 0.f ? fast_exp2(ms[gg * nsplit + s] - mx[gg]) * l_s : 0.f;
                ms[gg * nsplit + s] = wt;
                dsum[gg] += wt;
            }
        }
        consumer_reduce<false>(dsum, sm.red, warp, lane);  // its barriers also publish the weights
        const float *pg = parts0 + static_cast<uint64_t>(g) * a.max_splits * kWsRec + d0;
        const float *wg = ms + g * nsplit;
        float r[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t s = 0;
        for (; s + 8 <= nsplit; s += 8) {  // 8 independent 16-byte loads in flight per thread
            float4 ov[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) ov[u] = __ldcg(reinterpret_cast<const float4 *>(pg + (s + u) * kWsRec));
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const float wt = wg[s + u];
                r[0] += wt * ov[u].x;
                r[1] += wt * ov[u].y;
                r[2] += wt * ov[u].z;
                r[3] += wt * ov[u].w;
            }
        }
        for (; s < nsplit; ++s) {
            const float4 ov = __ldcg(reinterpret_cast<const float4 *>(pg + s * kWsRec));
            const float wt = wg[s];
            r[0] += wt * ov.x;
            r[1] += wt * ov.y;
            r[2] += wt * ov.z;
            r[3] += wt * ov.w;
        }
        const float Mx = g ? mx[1] : mx[0], dtot = g ? dsum[1] : dsum[0];  // selects keep both in registers
        const float inv = dtot > 0.f ? 1.0f / dtot : 0.f;
        if (a.peer_mode) {
            const float on[4] = {r[0] * inv, r[1] * inv, r[2] * inv, r[3] * inv};
            peer_publish_merge(a, sm, b, kvh, tid, g, d0, on, Mx, dtot);
        } else if (a.partial_mode) {
            // A rank partial stores l relative to its own max Mx: l_rank = sum_s 2^(m_s - Mx) l_s.
            float *dst = a.partial_out + row * kPart;
#pragma unroll
            for (int e = 0; e < 4; ++e) dst[d0 + e] = r[e] * inv;
            if (d0 == 0) {
                dst[kD] = Mx;
                dst[kD + 1] = dtot;
            }
        } else {
            uint2 packed;
            packed.x = pack_bf16(r[0] * inv, r[1] * inv);
            packed.y = pack_bf16(r[2] * inv, r[3] * inv);
            *reinterpret_cast<uint2 *>(a.out + row * kD + d0) = packed;
        }
    }
}

__global__ void merge_partials_kernel(const float *__restrict__ parts, uint32_t num_parts,
                                      uint32_t rows, uint32_t head_dim, uint16_t *__restrict__ out) {
    const uint32_t row = blockIdx.x;
    const uint64_t rec = head_dim + 2;
    float M = -INFINITY;
    for (uint32_t r = 0; r < num_parts; ++r) {
        const float *p = parts + (static_cast<uint64_t>(r) * rows + row) * rec;
        if (p[head_dim + 1] > 0.f) M = fmaxf(M, p[head_dim]);
    }
    for (uint32_t d = threadIdx.x; d < head_dim; d += blockDim.x) {
        float den = 0.f, num = 0.f;
        for (uint32_t r = 0; r < num_parts; ++r) {
            const float *p = parts + (static_cast<uint64_t>(r) * rows + row) * rec;
            const float l = p[head_dim + 1];
            if (!(l > 0.f)) continue;
            const float wt = fast_exp2(p[head_dim] - M) * l;
            den += wt;
            num += wt * p[d];
        }
        __nv_bfloat16 v = __float2bfloat16_rn(den > 0.f ? num / den : 0.f);
        out[static_cast<uint64_t>(row) * head_dim + d] = *reinterpret_cast<uint16_t *>(&v);
    }
}

// ---------------------------------------------------------------- host-side planning
uint32_t target_ctas() { return 16u * static_cast<uint32_t>(sm_count()); }  // 8 waves x 2/SM

// Splits.  About 8 waves of CTAs balance a batch of unequal lengths, but every CTA pays a fixed
// prologue (q norm + RoPE, first loads) and the merge reads one partial per split.  So a split gets
// at least this many positions (2 x 512 KB of K and V) whenever the splits still fill one wave,
// and a single sequence -- all of whose splits are equal -- is cut into exactly one wave
// (measured on 131072 positions: 81 % of HBM with 8 waves, 87 % with 1024-position splits, 97 %
// with one wave; a 64-sequence ragged batch is unchanged at 1024 and loses 7 % at one wave).
constexpr uint64_t kMinChunkPos = 1024;

uint32_t choose_chunk(uint32_t batch, uint32_t kv_heads, uint32_t range_len) {
    const uint64_t rows = static_cast<uint64_t>(batch) * kv_heads * std::max<uint32_t>(range_len, 1);
    uint64_t c = (rows + target_ctas() - 1) / target_ctas();
    const uint64_t one_wave = 2ull * static_cast<uint64_t>(sm_count());
    const uint64_t wave_chunk = (rows + one_wave - 1) / one_wave;
    c = std::max<uint64_t>(c, batch == 1 ? wave_chunk : std::min<uint64_t>(wave_chunk, kMinChunkPos));
    c = (c + kStagePos - 1) / kStagePos * kStagePos;
    return static_cast<uint32_t>(std::min<uint64_t>(std::max<uint64_t>(c, kStagePos), 1u << 24));
}

// Splits of a KV split's partial modes, where every sequence covers the same key range (each rank
// holds the same positions of every sequence), so a plan launches exactly batch * kv_heads * splits
// CTAs.  The split size is the one with the least modelled time -- whole waves of two CTAs per SM,
// each as long as a split plus a fixed per-CTA cost -- among sizes of at least the floor above
// (ties keep the larger split).  A last wave that is half empty costs as much as a full one: at 8
// GPUs a batch of 8 sequences of 131072 keys gives each rank 16384 keys per sequence, which
// 1024-key splits cut into 3.46 waves; 9 splits per (sequence, kv head) fill two.
constexpr uint64_t kCtaCostPos = 64;  // per-CTA set-up and merge, in key positions of streaming

uint32_t choose_chunk_equal(uint32_t batch, uint32_t kv_heads, uint32_t range_len) {
    const uint64_t pairs = static_cast<uint64_t>(batch) * kv_heads;
    const uint64_t len = std::max<uint32_t>(range_len, 1);
    const uint64_t one_wave = 2ull * static_cast<uint64_t>(sm_count());
    const uint64_t wave_chunk = (pairs * len + one_wave - 1) / one_wave;
    const uint64_t floor_c = batch == 1 ? wave_chunk : std::min<uint64_t>(wave_chunk, kMinChunkPos);
    uint64_t best_c = 0, best_cost = ~0ull;
    for (uint64_t s = 1; s <= len; ++s) {
        const uint64_t c = ((len + s - 1) / s + kStagePos - 1) / kStagePos * kStagePos;
        if (c < floor_c) break;
        const uint64_t ctas = pairs * ((len + c - 1) / c);
        const uint64_t cost = (ctas + one_wave - 1) / one_wave * (c + kCtaCostPos);
        if (cost < best_cost) {
            best_cost = cost;
            best_c = c;
        }
    }
    if (!best_c || best_c > (1u << 24)) return choose_chunk(batch, kv_heads, range_len);
    return static_cast<uint32_t>(best_c);
}

uint32_t max_splits_for(uint32_t batch, uint32_t kv_heads, uint32_t max_len) {
    const uint64_t by_len = (static_cast<uint64_t>(max_len) + kStagePos - 1) / kStagePos;
    const uint64_t by_target = target_ctas() / std::max<uint64_t>(1, static_cast<uint64_t>(batch) * kv_heads) + 2;
    // the last-CTA merge stages 2 * G * splits floats in the 48 KB of V stage buffers
    return static_cast<uint32_t>(std::max<uint64_t>(1, std::min({by_len, by_target, uint64_t(3072)})));
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

size_t workspace_bytes(uint32_t batch, uint32_t q_heads, uint32_t kv_heads, uint32_t max_len) {
    const size_t parts = static_cast<size_t>(batch) * q_heads * max_splits_for(batch, kv_heads, max_len) *
                         kWsRec * sizeof(float);
    return align256(parts) + align256(static_cast<size_t>(batch) * kv_heads * sizeof(unsigned));
}

int check_params(const apex_attn_params *p, const char *name) {
    if (!p) return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": null params");
    if (p->head_dim != kD)
        return fail(APEX_ERR_UNSUPPORTED, std::string(name) + ": this build supports head_dim 256");
    if (p->kv_heads == 0 || p->q_heads != p->kv_heads * kG)
        return fail(APEX_ERR_UNSUPPORTED, std::string(name) + ": this build supports q_heads = 2 * kv_heads");
    if (p->rope_pairs > kD / 2)
        return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": rope_pairs > head_dim / 2");
    if (p->kv_heads > 65535) return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": too many kv heads");
    return APEX_OK;
}

// A validated decode launch: arguments and grid, or empty (batch 0: nothing to launch).  cluster > 0
// selects the cluster form (grid.x == cluster CTAs per (sequence, kv head)).
struct DecodePlan {
    DecodeArgs a{};
    dim3 grid;
    uint32_t cluster = 0;
    int stages = 0;  // cluster form: ring stages (1 or 2)
    bool empty = false;
};

using ShortSmem1 = DecodeSmemT<kShortWarps, 1, true>;
using ShortSmem2 = DecodeSmemT<kShortWarps, 2, true>;

template <int ST>
size_t short_smem_bytes() { return ST == 1 ? sizeof(ShortSmem1) : sizeof(ShortSmem2); }

// How many clusters of `size` CTAs of the cluster form (ring of ST stages) can be resident at once
// on the current device; sets the kernel's attributes first (once per device).
template <int ST>
int active_clusters(uint32_t size) {
    static std::mutex mu;
    static std::vector<std::vector<int>> cache;  // [device][size]: -1 unknown
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    std::lock_guard<std::mutex> lock(mu);
    if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1);
    auto &row = cache[dev];
    if (row.empty()) {
        auto *kernel = decode_kernel<kShortWarps, ST, true>;
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(short_smem_bytes<ST>())) != cudaSuccess ||
            cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
            cudaGetLastError();
            row.assign(kMaxCluster + 1, 0);
            return 0;
        }
        row.assign(kMaxCluster + 1, -1);
    }
    if (row[size] < 0) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(size, 1, 1);
        cfg.blockDim = dim3((kShortWarps + 1) * 32, 1, 1);
        cfg.dynamicSmemBytes = short_smem_bytes<ST>();
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = size;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, decode_kernel<kShortWarps, ST, true>, &cfg) != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        row[size] = n;
    }
    return row[size];
}

// Cluster size for a short-context decode of `batch` sequences, or 0 for the split-KV form.  The
// cluster form is taken when every (sequence, kv head) gets a cluster of at least two splits and
// all the clusters are resident at once (one wave); at short contexts the step is latency, and
// merging in distributed shared memory saves the workspace round trip and the second pass.  Splits
// of one 64-position stage use a one-stage ring (about 100 KB of shared memory, two CTAs per SM).
uint32_t short_cluster(uint32_t batch, uint32_t kv_heads, uint32_t range_len, uint32_t &chunk, int &stages) {
    const uint64_t pairs = static_cast<uint64_t>(batch) * kv_heads;
    const uint64_t most = std::min<uint64_t>(kMaxCluster, (range_len + kShortStagePos - 1) / kShortStagePos);
    for (uint64_t c = most; c >= 2; --c) {
        uint64_t ch = (range_len + c - 1) / c;
        ch = (ch + kShortStagePos - 1) / kShortStagePos * kShortStagePos;
        const uint64_t used = (range_len + ch - 1) / ch;
        if (used < 2 || used != c) continue;
        const int st = ch == kShortStagePos ? 1 : 2;
        const int fit = st == 1 ? active_clusters<1>(static_cast<uint32_t>(used))
                                : active_clusters<2>(static_cast<uint32_t>(used));
        if (static_cast<uint64_t>(fit) >= pairs) {
            chunk = static_cast<uint32_t>(ch);
            stages = st;
            return static_cast<uint32_t>(used);
        }
    }
    return 0;
}

// Checks every argument of a decode call and fills `plan`; queues nothing.
int plan_decode(const apex_attn_params *p, const uint16_t *q_raw, const uint16_t *k_new,
                const uint16_t *v_new, const uint16_t *q_w, const uint16_t *k_w,
                uint16_t *k_cache, uint16_t *v_cache, uint32_t capacity,
                const int32_t *seq_lens, uint32_t batch, uint32_t max_seq_len,
                uint32_t kv_begin, uint32_t kv_end, bool partial_mode, uint16_t *out,
                float *partial_out, void *workspace, size_t workspace_bytes_given,
                const char *name, const apex_peer_exchange *peer, DecodePlan &plan) {
    int rc = check_params(p, name);
    if (rc) return rc;
    if (batch == 0) {
        plan.empty = true;
        return APEX_OK;
    }
    if (batch > 65535) return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": batch > 65535");
    if (!q_raw || !k_new || !v_new || !k_cache || !v_cache || !seq_lens ||
        (partial_mode && !peer ? !partial_out : !out))
        return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": null tensor");
    if (peer) {
        if (peer->world < 1 || peer->world > kMaxPeers || peer->rank >= peer->world)
            return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": need 1 <= world <= 8 and rank < world");
        if (!peer->seq) return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": null step counters");
        // one CTA per (sequence, kv head) waits for the other ranks while holding its SM slot; at
        // most one per SM keeps every rank's remaining CTAs schedulable
        if (static_cast<uint64_t>(batch) * p->kv_heads > static_cast<uint64_t>(sm_count()))
            return fail(APEX_ERR_UNSUPPORTED, std::string(name) + ": batch * kv_heads above the SM count");
        for (uint32_t r = 0; r < peer->world; ++r)
            if (!peer->gather[r] || !peer->flags[r] || !aligned16(peer->gather[r]))
                return fail(APEX_ERR_INVALID_ARGUMENT,
                            std::string(name) + ": every rank's gather buffer (16-byte aligned) and flags are needed");
    }
    for (const void *ptr : {(const void *)q_raw, (const void *)k_new, (const void *)v_new,
                            (const void *)k_cache, (const void *)v_cache})
        if (!aligned16(ptr)) return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": tensors must be 16-byte aligned");
    if (max_seq_len == 0) return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": max_seq_len must be >= 1");
    if (kv_end <= kv_begin) return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": empty kv range");
    const bool ring = p->ring != 0;
    if (ring && (partial_mode || peer))
        return fail(APEX_ERR_UNSUPPORTED, std::string(name) + ": ring caches are served by the one-GPU decode only");
    if (ring && (p->window == 0 || p->window > capacity))
        return fail(APEX_ERR_INVALID_ARGUMENT,
                    std::string(name) + ": a ring cache needs 0 < window <= capacity (it holds the last capacity keys)");
    uint32_t range_len = std::min<uint32_t>(kv_end, max_seq_len) - std::min(kv_begin, max_seq_len);
    if (!partial_mode && p->window) range_len = std::min(range_len, p->window);  // keys one query can see
    if (!ring && (partial_mode ? static_cast<uint64_t>(kv_end) - kv_begin : max_seq_len) > capacity)
        return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": key range exceeds cache capacity");
    const size_t need = workspace_bytes(batch, p->q_heads, p->kv_heads, max_seq_len);
    if (!workspace || workspace_bytes_given < need)
        return fail(APEX_ERR_WORKSPACE, std::string(name) + ": workspace of " + std::to_string(need) +
                                            " bytes required");
    if (!aligned16(workspace)) return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": workspace must be 16-byte aligned");

    DecodeArgs &a = plan.a;
    a = DecodeArgs{};
    a.q_raw = q_raw; a.k_new = k_new; a.v_new = v_new; a.q_w = q_w; a.k_w = k_w;
    a.k_cache = k_cache; a.v_cache = v_cache; a.seq_lens = seq_lens;
    a.out = out; a.partial_out = partial_out;
    const uint32_t max_splits = max_splits_for(batch, p->kv_heads, max_seq_len);
    a.ws_part = static_cast<float *>(workspace);
    a.ws_count = reinterpret_cast<unsigned *>(
        static_cast<uint8_t *>(workspace) +
        align256(static_cast<size_t>(batch) * p->q_heads * max_splits * kWsRec * sizeof(float)));
    a.capacity = capacity; a.q_heads = p->q_heads; a.kv_heads = p->kv_heads;
    a.rope_pairs = p->rope_pairs; a.window = p->window; a.qk_norm = p->qk_norm; a.v_norm = p->v_norm;
    a.chunk = partial_mode ? choose_chunk_equal(batch, p->kv_heads, range_len)
                           : choose_chunk(batch, p->kv_heads, range_len);
    a.max_splits = max_splits;
    a.kv_begin = kv_begin; a.kv_end = kv_end; a.max_seq_len = max_seq_len;
    a.ring = ring ? 1u : 0u;
    a.rope_base = p->rope_base; a.eps = p->eps; a.scale_log2 = p->scale * kLog2e;
    a.partial_mode = partial_mode ? 1 : 0;
    if (peer) {
        a.peer_mode = 1;
        a.rank = peer->rank;
        a.world = peer->world;
        for (uint32_t r = 0; r < peer->world; ++r) {
            a.peer_gather[r] = peer->gather[r];
            a.peer_flags[r] = peer->flags[r];
        }
        a.peer_seq = peer->seq;
        a.peer_wait_ns = peer->wait_ns ? peer->wait_ns : kPeerWaitDefaultNs;
    }
    rope_table(a.rope.inv_freq, p->rope_pairs, kD, p->rope_base);
    a.status = device_status_ptr();
    if (!a.status) return fail(APEX_ERR_CUDA, std::string(name) + ": device status word unavailable");
    uint32_t grid_x = std::max<uint32_t>(1, (std::max<uint32_t>(range_len, 1) + a.chunk - 1) / a.chunk);
    if (grid_x > max_splits)
        return fail(APEX_ERR_WORKSPACE, std::string(name) + ": internal split plan exceeds workspace");
    if (!partial_mode && !peer && max_seq_len <= kShortMaxLen) {
        uint32_t chunk = 0;
        int stages = 0;
        const uint32_t c = short_cluster(batch, p->kv_heads, range_len, chunk, stages);
        if (c) {
            a.chunk = chunk;
            grid_x = c;
            plan.cluster = c;
            plan.stages = stages;
        }
    }
    plan.grid = dim3(grid_x, p->kv_heads, batch);
    return APEX_OK;
}

// Queues the planned decode kernel on `stream`.
int run_decode_plan(const DecodePlan &plan, void *stream, const char *name) {
    if (plan.empty) return ok();
    if (plan.cluster) {  // attributes were set when the plan was made (active_clusters)
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = plan.grid;
        cfg.blockDim = dim3((kShortWarps + 1) * 32, 1, 1);
        cfg.dynamicSmemBytes = plan.stages == 1 ? short_smem_bytes<1>() : short_smem_bytes<2>();
        cfg.stream = static_cast<cudaStream_t>(stream);
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = plan.cluster;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const int rc = check_cuda(plan.stages == 1
                                      ? cudaLaunchKernelEx(&cfg, decode_kernel<kShortWarps, 1, true>, plan.a)
                                      : cudaLaunchKernelEx(&cfg, decode_kernel<kShortWarps, 2, true>, plan.a),
                                  name);
        return rc ? rc : ok();
    }
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    auto *kernel = decode_kernel<kConsumerWarps, kStages, false>;
    if (dev < 64 && !attr_set[dev]) {
        const int rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                       static_cast<int>(sizeof(DecodeSmem))),
                                  "decode smem attribute");
        if (rc) return rc;
        attr_set[dev] = true;
    }
    kernel<<<plan.grid, kThreads, sizeof(DecodeSmem), static_cast<cudaStream_t>(stream)>>>(plan.a);
    const int rc = check_cuda(cudaGetLastError(), name);
    return rc ? rc : ok();
}

int launch_decode(const apex_attn_params *p, const uint16_t *q_raw, const uint16_t *k_new,
                  const uint16_t *v_new, const uint16_t *q_w, const uint16_t *k_w,
                  uint16_t *k_cache, uint16_t *v_cache, uint32_t capacity,
                  const int32_t *seq_lens, uint32_t batch, uint32_t max_seq_len,
                  uint32_t kv_begin, uint32_t kv_end, bool partial_mode, uint16_t *out,
                  float *partial_out, void *workspace, size_t workspace_bytes_given, void *stream,
                  const char *name, const apex_peer_exchange *peer = nullptr) {
    DecodePlan plan;
    const int rc = plan_decode(p, q_raw, k_new, v_new, q_w, k_w, k_cache, v_cache, capacity, seq_lens, batch,
                               max_seq_len, kv_begin, kv_end, partial_mode, out, partial_out, workspace,
                               workspace_bytes_given, name, peer, plan);
    return rc ? rc : run_decode_plan(plan, stream, name);
}

}  // namespace
}  // namespace apex

extern "C" size_t apex_attn_decode_workspace_bytes(const apex_attn_params *p, uint32_t batch,
                                                   uint32_t max_seq_len) {
    if (!p || p->kv_heads == 0) return 0;
    if (apex::gqa_decode_form(p)) return apex::gqa_workspace_bytes(p, batch, std::max<uint32_t>(max_seq_len, 1));
    return apex::workspace_bytes(batch, p->q_heads, p->kv_heads, std::max<uint32_t>(max_seq_len, 1));
}

extern "C" int apex_attn_decode_workspace_init(void *workspace, size_t workspace_bytes,
                                               void *stream) {
    if (!workspace) return apex::fail(APEX_ERR_WORKSPACE, "apex_attn_decode_workspace_init: null workspace");
    const int rc = apex::check_cuda(
        cudaMemsetAsync(workspace, 0, workspace_bytes, static_cast<cudaStream_t>(stream)),
        "apex_attn_decode_workspace_init");
    return rc ? rc : apex::ok();
}

extern "C" int apex_attn_decode_bf16(const apex_attn_params *p, const uint16_t *q_raw,
                                     const uint16_t *k_new, const uint16_t *v_new,
                                     const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                                     uint16_t *k_cache, uint16_t *v_cache, uint32_t capacity,
                                     const int32_t *seq_lens, uint32_t batch,
                                     uint32_t max_seq_len, uint16_t *out, void *workspace,
                                     size_t workspace_bytes, void *stream) {
    if (apex::gqa_decode_form(p))
        return apex::launch_gqa_decode(p, q_raw, k_new, v_new, q_norm_w, k_norm_w, k_cache, v_cache, capacity,
                                       seq_lens, batch, max_seq_len, out, workspace, workspace_bytes, stream,
                                       "apex_attn_decode_bf16");
    return apex::launch_decode(p, q_raw, k_new, v_new, q_norm_w, k_norm_w, k_cache, v_cache,
                               capacity, seq_lens, batch, max_seq_len, 0, 0xffffffffu, false, out,
                               nullptr, workspace, workspace_bytes, stream, "apex_attn_decode_bf16");
}

extern "C" int apex_attn_decode_partial_bf16(const apex_attn_params *p, const uint16_t *q_raw,
                                             const uint16_t *k_new, const uint16_t *v_new,
                                             const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                                             uint16_t *k_cache, uint16_t *v_cache,
                                             uint32_t capacity, const int32_t *seq_lens,
                                             uint32_t batch, uint32_t max_seq_len,
                                             uint32_t kv_begin, uint32_t kv_end, float *partial,
                                             void *workspace, size_t workspace_bytes,
                                             void *stream) {
    return apex::launch_decode(p, q_raw, k_new, v_new, q_norm_w, k_norm_w, k_cache, v_cache,
                               capacity, seq_lens, batch, max_seq_len, kv_begin, kv_end, true,
                               nullptr, partial, workspace, workspace_bytes, stream,
                               "apex_attn_decode_partial_bf16");
}

extern "C" int apex_attn_peer_exchange_bytes(const apex_attn_params *p, uint32_t batch, uint32_t world,
                                             size_t *gather_bytes, size_t *flag_bytes, size_t *seq_bytes) {
    using namespace apex;
    int rc = check_params(p, "apex_attn_peer_exchange_bytes");
    if (rc) return rc;
    if (world < 1 || world > kMaxPeers)
        return fail(APEX_ERR_INVALID_ARGUMENT, "apex_attn_peer_exchange_bytes: need 1 <= world <= 8");
    if (!gather_bytes || !flag_bytes || !seq_bytes)
        return fail(APEX_ERR_INVALID_ARGUMENT, "apex_attn_peer_exchange_bytes: null output");
    *gather_bytes = 2ull * world * batch * p->q_heads * kLLRec * sizeof(uint64_t);  // 16-byte multiples
    *flag_bytes = static_cast<size_t>(world) * batch * p->kv_heads * sizeof(uint32_t);
    *seq_bytes = static_cast<size_t>(batch) * p->kv_heads * sizeof(uint32_t);
    return ok();
}

extern "C" int apex_attn_decode_kvsplit_bf16(const apex_attn_params *p, const uint16_t *q_raw,
                                             const uint16_t *k_new, const uint16_t *v_new,
                                             const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                                             uint16_t *k_cache, uint16_t *v_cache, uint32_t capacity,
                                             const int32_t *seq_lens, uint32_t batch, uint32_t max_seq_len,
                                             uint32_t kv_begin, uint32_t kv_end, const apex_peer_exchange *x,
                                             uint16_t *out, void *workspace, size_t workspace_bytes,
                                             void *stream) {
    if (!x) return apex::fail(APEX_ERR_INVALID_ARGUMENT, "apex_attn_decode_kvsplit_bf16: null peer exchange");
    return apex::launch_decode(p, q_raw, k_new, v_new, q_norm_w, k_norm_w, k_cache, v_cache, capacity, seq_lens,
                               batch, max_seq_len, kv_begin, kv_end, true, out, nullptr, workspace,
                               workspace_bytes, stream, "apex_attn_decode_kvsplit_bf16", x);
}

extern "C" int apex_attn_merge_partials(const float *partials, uint32_t num_partials,
                                        uint32_t rows, uint32_t head_dim, uint16_t *out,
                                        void *stream) {
    using namespace apex;
    if (rows == 0) return ok();
    if (!partials || !out) return fail(APEX_ERR_INVALID_ARGUMENT, "apex_attn_merge_partials: null tensor");
    if (num_partials == 0 || head_dim == 0)
        return fail(APEX_ERR_INVALID_ARGUMENT, "apex_attn_merge_partials: empty partial set");
    merge_partials_kernel<<<rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(partials, num_partials,
                                                                              rows, head_dim, out);
    const int rc = check_cuda(cudaGetLastError(), "apex_attn_merge_partials");
    return rc ? rc : ok();
}

// ---------------------------------------------------------------- ring caches
namespace apex {
namespace {

// Rows [first, length) of linear [B][H][lin_cap][D] into ring [B][H][ring_cap][D] at slot p % ring_cap;
// one 16-byte piece per thread.
__global__ void kv_ring_store_kernel(const uint4 *__restrict__ k_lin, const uint4 *__restrict__ v_lin,
                                     uint4 *__restrict__ k_ring, uint4 *__restrict__ v_ring, uint32_t heads,
                                     uint32_t pieces, uint32_t lin_cap, uint32_t ring_cap, uint32_t first,
                                     uint32_t n) {
    const uint64_t total = static_cast<uint64_t>(heads) * n * pieces;  // this block row's sequence: blockIdx.y
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t c = static_cast<uint32_t>(i % pieces);
        const uint64_t rest = i / pieces;
        const uint32_t j = static_cast<uint32_t>(rest % n);
        const uint64_t bh = static_cast<uint64_t>(blockIdx.y) * heads + rest / n;
        const uint32_t pos = first + j;
        const uint64_t src = (bh * lin_cap + pos) * pieces + c, dst = (bh * ring_cap + pos % ring_cap) * pieces + c;
        k_ring[dst] = k_lin[src];
        v_ring[dst] = v_lin[src];
    }
}

}  // namespace
}  // namespace apex

extern "C" int apex_kv_ring_store(const uint16_t *k_linear, const uint16_t *v_linear, uint16_t *k_ring,
                                  uint16_t *v_ring, uint32_t batch, uint32_t kv_heads, uint32_t head_dim,
                                  uint32_t linear_capacity, uint32_t ring_capacity, uint32_t length, void *stream) {
    using namespace apex;
    const char *name = "apex_kv_ring_store";
    if (batch == 0 || kv_heads == 0 || length == 0) return ok();
    if (!k_linear || !v_linear || !k_ring || !v_ring) return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": null tensor");
    if (head_dim == 0 || head_dim % 8) return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": head_dim a multiple of 8");
    if (ring_capacity == 0 || length > linear_capacity)
        return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": need ring_capacity > 0 and length <= linear_capacity");
    for (const void *ptr : {(const void *)k_linear, (const void *)v_linear, (const void *)k_ring, (const void *)v_ring})
        if (!aligned16(ptr)) return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": tensors must be 16-byte aligned");
    if (batch > 65535) return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": batch > 65535");
    const uint32_t first = length > ring_capacity ? length - ring_capacity : 0;
    const uint32_t n = length - first;
    const uint64_t per_seq = static_cast<uint64_t>(kv_heads) * n * (head_dim / 8);
    const uint32_t blocks = static_cast<uint32_t>(std::min<uint64_t>((per_seq + 255) / 256, 65535));
    kv_ring_store_kernel<<<dim3(blocks, batch), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const uint4 *>(k_linear), reinterpret_cast<const uint4 *>(v_linear),
        reinterpret_cast<uint4 *>(k_ring), reinterpret_cast<uint4 *>(v_ring), kv_heads, head_dim / 8, linear_capacity,
        ring_capacity, first, n);
    const int rc = check_cuda(cudaGetLastError(), name);
    return rc ? rc : ok();
}

// ---------------------------------------------------------------- allocation-free variant
// Some callers cannot call cudaMalloc for the decode workspace: an engine that owns all of
// its device memory under a fixed budget (the design of the engine this path comes from) has
// nowhere to put a library allocation, and a latency-critical decode loop cannot pay for
// cudaMalloc's implicit device synchronisation.  apex_attn_decode_bf16_noalloc serves them
// from this file-scope device array instead.  It is a fixed 8 MiB: every GPU the library is
// used on holds it until the process exits.  The decode kernel receives its address; host
// code only names it to look that address up.
namespace apex {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
static __device__ __align__(256) uint8_t g_decode_scratch[kNoAllocScratchBytes];

// Device address of g_decode_scratch on the current device, looked up once per device (the
// symbol's host-side name is only a stand-in, never a device address).
int noalloc_scratch(void **ptr) {
    static std::mutex mu;
    static std::vector<void *> cache;
    int dev = 0;
    int rc = check_cuda(cudaGetDevice(&dev), "apex_attn_decode_bf16_noalloc: cudaGetDevice");
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(mu);
    if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1, nullptr);
    if (!cache[dev]) {
        void *p = nullptr;
        rc = check_cuda(cudaGetSymbolAddress(&p, g_decode_scratch),
                        "apex_attn_decode_bf16_noalloc: cudaGetSymbolAddress");
        if (rc) return rc;
        cache[dev] = p;
    }
    *ptr = cache[dev];
    return APEX_OK;
}

}  // namespace
}  // namespace apex

extern "C" int apex_attn_decode_bf16_noalloc(const apex_attn_params *p, const uint16_t *q_raw,
                                             const uint16_t *k_new, const uint16_t *v_new,
                                             const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                                             uint16_t *k_cache, uint16_t *v_cache,
                                             uint32_t capacity, const int32_t *seq_lens,
                                             uint32_t batch, uint32_t max_seq_len, uint16_t *out,
                                             void *stream) {
    using namespace apex;
    const char *name = "apex_attn_decode_bf16_noalloc";
    int rc = check_params(p, name);
    if (rc) return rc;
    if (batch == 0) return ok();
    const uint32_t msl = std::max<uint32_t>(max_seq_len, 1);
    const size_t need = workspace_bytes(batch, p->q_heads, p->kv_heads, msl);
    if (need > kNoAllocScratchBytes)
        return fail(APEX_ERR_WORKSPACE,
                    std::string(name) + ": batch " + std::to_string(batch) + " x max_seq_len " +
                        std::to_string(msl) + " needs " + std::to_string(need) +
                        " bytes of scratch; the static scratch holds " +
                        std::to_string(kNoAllocScratchBytes) + " (use apex_attn_decode_bf16)");
    void *scratch = nullptr;
    rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    // Every argument is checked before anything is queued, so a rejected call leaves nothing on
    // `stream` (no counter clear on the shared array either).
    DecodePlan plan;
    rc = plan_decode(p, q_raw, k_new, v_new, q_norm_w, k_norm_w, k_cache, v_cache, capacity, seq_lens, batch,
                     max_seq_len, 0, 0xffffffffu, false, out, nullptr, scratch, kNoAllocScratchBytes, name,
                     nullptr, plan);
    if (rc) return rc;
    // The split counters must start at zero; the array keeps whatever the last call left.
    rc = check_cuda(cudaMemsetAsync(plan.a.ws_count, 0, static_cast<size_t>(batch) * p->kv_heads * sizeof(unsigned),
                                    static_cast<cudaStream_t>(stream)),
                    "apex_attn_decode_bf16_noalloc: clear counters");
    if (rc) return rc;
    return run_decode_plan(plan, stream, name);
}
