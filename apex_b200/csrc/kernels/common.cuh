// common.cuh -- device helpers shared by the sm_100a kernels: bf16 packing, RoPE frequencies,
// mbarriers with bounded waits, TMA (bulk and tensor) copies, tcgen05 / TMEM wrappers.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace apex {

// Device status word bits (the word itself lives in capi_common.cu; kernels receive its
// address as an argument and apex_cuda_device_status reads and clears it).
constexpr unsigned kStatusTimeout = 1u;    // a bounded wait gave up
constexpr unsigned kStatusBadLength = 2u;  // a sequence length outside the caller's bounds
// Bounded waits give up after this many SM clock cycles (about one second at 1.9 GHz).
constexpr long long kWaitBudgetCycles = 2000000000ll;

// ------------------------------------------------------------------ bf16 <-> f32
__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}
// bf16 pair (low half a * s, high half b * s), the two products in one packed f32x2 multiply
// (sm_100) and both rounded to nearest even in one conversion.
__device__ __forceinline__ uint32_t scale_pack_bf16(uint32_t a, uint32_t b, float s) {
    uint32_t r;
    asm("{\n\t.reg .b64 x, y, sc;\n\t.reg .b32 lo, hi;\n\t"
        "mov.b64 x, {%1, %2};\n\t"
        "mov.b64 sc, {%3, %3};\n\t"
        "mul.rn.f32x2 y, x, sc;\n\t"
        "mov.b64 {lo, hi}, y;\n\t"
        "cvt.rn.bf16x2.f32 %0, hi, lo;\n\t}"
        : "=r"(r)
        : "r"(a), "r"(b), "r"(__float_as_uint(s)));
    return r;
}
__device__ __forceinline__ float bf16_round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
}

// RoPE inverse frequencies inv_freq[i] = base^(-2i/hd) for i < pairs, computed once on the host
// (rope_table) and passed by value; kernels stage the table in shared memory.
constexpr int kMaxRopePairs = 256;
struct RopeTable {
    float inv_freq[kMaxRopePairs];
};

// cos and sin of the f32 angle of a RoPE pair (the angle itself is the f32 product pos * inv_freq,
// as the reference computes it).  The angle is reduced to [-pi, pi] in double precision
// (r = angle - k * 2pi, k = rint(angle / 2pi); for |angle| < 2^24 the reduction error is below
// 1e-9), then the hardware sine/cosine, whose absolute error on [-pi, pi] is about 2^-21, is
// applied to r.  Exact enough for bf16 outputs and for the f32 drop-in's 1e-5 relative gate, and
// a handful of instructions instead of a full-range library call per pair.
__device__ __forceinline__ void rope_sincos(float angle, float &s, float &c) {
    constexpr double kTwoPi = 6.283185307179586476925286766559;
    constexpr double kInvTwoPi = 0.15915494309189533576888376337251;
    const double a = static_cast<double>(angle);
    const double k = rint(a * kInvTwoPi);
    const float r = static_cast<float>(fma(-k, kTwoPi, a));
    __sincosf(r, &s, &c);
}

// max of three floats in one instruction (sm_100)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ------------------------------------------------------------------ packed f32x2 arithmetic (sm_100)
__device__ __forceinline__ uint64_t f32x2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f32x2_split(uint64_t v, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t sub_f32x2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
// 2^x0 and 2^x1 on the FMA pipe (x <= 8; x is clamped at -126, so -inf gives 2^-126 or a denormal,
// never a wrapped exponent: the cubic's value is in [0.7, 1.5]), to take part of a softmax's
// exponentials off the MUFU pipe.  Cody-Waite style reduction x = j + f, j = rint(x) by the
// 1.5 * 2^23 shift, f in [-1/2, 1/2]; 2^f by a cubic whose coefficients are the least-squares fit
// of 2^f on 2001 equally spaced points of [-1/2, 1/2] (maximum relative error 1.9e-4 over
// [-30, 0], well below the 2^-9 of the bf16 P it feeds); 2^j is added to the exponent field.
__device__ __forceinline__ void exp2_poly_x2(uint64_t x2, float &p0, float &p1) {
    float x0, x1;
    f32x2_split(x2, x0, x1);
    const uint64_t x = f32x2(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
    const uint64_t shift = f32x2(12582912.0f, 12582912.0f);
    const uint64_t t = add_f32x2(x, shift);
    const uint64_t f = sub_f32x2(x, sub_f32x2(t, shift));
    uint64_t q = fma_f32x2(f32x2(0.0558758713f, 0.0558758713f), f, f32x2(0.242296502f, 0.242296502f));
    q = fma_f32x2(q, f, f32x2(0.693127215f, 0.693127215f));
    q = fma_f32x2(q, f, f32x2(0.999948144f, 0.999948144f));
    float q0, q1, t0, t1;
    f32x2_split(q, q0, q1);
    f32x2_split(t, t0, t1);
    // unsigned: the shift moves j's low bits (two's complement) into the exponent field and wraps
    p0 = __uint_as_float(__float_as_uint(q0) + (__float_as_uint(t0) << 23));
    p1 = __uint_as_float(__float_as_uint(q1) + (__float_as_uint(t1) << 23));
}

// ------------------------------------------------------------------ shared-memory addresses
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarriers
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Raise the transaction count of the current phase without arriving.
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Non-blocking: has the phase with the given parity completed?
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Waits for the phase with the given parity to complete.  Gives up after kWaitBudgetCycles,
// sets kStatusTimeout in *status and returns false.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned *status) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long start = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - start > kWaitBudgetCycles) {
            atomicOr(status, kStatusTimeout);
            return false;
        }
    }
    return true;
}
// Same contract as mbar_wait, for a thread that issues tcgen05.mma: checks first with the
// non-blocking test_wait.  On B200 a try_wait or a clock read on the issuing thread costs about 90
// cycles even when the phase has already completed, and the tensor pipe runs dry meanwhile; a
// test_wait does not stall it.  A phase still open is waited for with try_wait, which suspends
// the warp instead of taking issue slots from the warps that share its scheduler.
__device__ __forceinline__ bool mbar_wait_spin(uint32_t bar, uint32_t parity, unsigned *status) {
    if (mbar_test_wait(bar, parity)) return true;
    return mbar_wait(bar, parity, status);
}

// ------------------------------------------------------------------ TMA
// 1-D bulk copy global -> shared, completion counted in bytes on `bar`.  src, dst 16-byte
// aligned, bytes a multiple of 16.
__device__ __forceinline__ void tma_bulk_load(uint32_t dst, const void *src, uint32_t bytes,
                                              uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}
// 3-D tiled tensor load (no multicast).  c0 is the innermost coordinate in elements; it must
// be a multiple of 16 bytes / element size.
// 2-D tiled load global -> shared (this CTA), completing on `bar`; no multicast.  c0 * element size
// must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int32_t c0, int32_t c1,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, int32_t c0,
                                            int32_t c1, int32_t c2, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
        "%3, %4}], [%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
        : "memory");
}
// 4-D tiled load global -> shared (this CTA), completing on `bar`; no multicast.  c0 * element size
// must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap *map, int32_t c0, int32_t c1, int32_t c2,
                                            int32_t c3, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
        : "memory");
}
// 4-D tiled store shared -> global (bulk async group; no multicast).  Elements outside the
// tensor are not written.  c0 * element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap *map, uint32_t src, int32_t c0, int32_t c1, int32_t c2,
                                             int32_t c3) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until this thread's committed bulk stores have finished reading their shared memory.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Wait until this thread's committed bulk stores are complete.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// At most one committed bulk group of this thread may still be reading its shared-memory source.
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
// 16-byte asynchronous global -> shared copy through L2 (both addresses 16-byte aligned), its
// group commit, and the wait until at most N of this thread's groups are still in flight.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// 16-byte shared store by shared-window address.
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// Make generic-proxy shared-memory writes visible to the async proxy (TMA, tensor cores).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------ tcgen05 / TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t holder_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(holder_smem),
                 "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (bf16 inputs, f32 accumulate).
__device__ __forceinline__ void tc_mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// D[tmem] (+)= A[tmem] * B[smem desc], kind::f16; A is M x 16 bf16 in TMEM (lane = row, two
// elements per 32-bit column, 8 columns per MMA), K-major.
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// Arrive once on `bar` when all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// tcgen05.wait::ld that also names the 32 registers a preceding tcgen05.ld wrote, so the compiler
// cannot schedule any use of them before the wait.
__device__ __forceinline__ void tc_wait_ld(uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}
// The same for two 32-register loads waited together.
__device__ __forceinline__ void tc_wait_ld(uint32_t (&a)[32], uint32_t (&b)[32]) {
    tc_wait_ld(a);
    asm volatile(""
                 : "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7]),
                   "+r"(b[8]), "+r"(b[9]), "+r"(b[10]), "+r"(b[11]), "+r"(b[12]), "+r"(b[13]), "+r"(b[14]),
                   "+r"(b[15]), "+r"(b[16]), "+r"(b[17]), "+r"(b[18]), "+r"(b[19]), "+r"(b[20]), "+r"(b[21]),
                   "+r"(b[22]), "+r"(b[23]), "+r"(b[24]), "+r"(b[25]), "+r"(b[26]), "+r"(b[27]), "+r"(b[28]),
                   "+r"(b[29]), "+r"(b[30]), "+r"(b[31])
                 :
                 : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 consecutive 32-bit TMEM columns of this warp's 32 lanes -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
        "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// ------------------------------------------------------------------ programmatic dependent launch
// In a kernel launched with programmatic stream serialization: block until the preceding
// kernel in the stream has completed and its memory is visible (a no-op otherwise).
// Per-warpgroup register budget (all 128 threads of a warpgroup execute the same one).  inc waits
// until other warpgroups have released enough registers: the block's split must not exceed the
// registers it was launched with.
template <uint32_t N>
__device__ __forceinline__ void reg_alloc() {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void reg_dealloc() {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel in the stream (if launched with programmatic stream serialization) be
// scheduled once every block of this grid has executed this or exited.
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------------ CTA pairs (cluster of 2)
// A pair of CTAs on two SMs runs one M=256 tcgen05.mma (.cta_group::2): each CTA supplies
// half of A's rows and half of B's N columns from the same shared-memory offsets and receives
// its 128 rows of D in its own TMEM.  Rank 0 (the leader) issues the MMAs.
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Address of the same shared variable in CTA `rank` of this cluster (shared::cluster window).
__device__ __forceinline__ uint32_t mapa(uint32_t smem_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void st_cluster_u32(uint32_t cluster_addr, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}
// Asynchronous 16-byte store into a cluster peer's shared memory whose completion counts 16 bytes on
// the peer's mbarrier (complete_tx): the receiver arms that barrier with expect_tx and waits on it;
// the sender needs no fence.
__device__ __forceinline__ void st_async_v4(uint32_t cluster_addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d,
                                            uint32_t cluster_bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                     cluster_addr),
                 "r"(a), "r"(b), "r"(c), "r"(d), "r"(cluster_bar)
                 : "memory");
}
__device__ __forceinline__ void st_cluster_v4(uint32_t cluster_addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(cluster_addr), "r"(a), "r"(b), "r"(c),
                 "r"(d)
                 : "memory");
}
// Arrive on an mbarrier given by its shared::cluster address (this CTA's or the peer's), with
// release at cluster scope: the arriving thread's earlier shared-memory writes (e.g. with
// st_cluster_u32) are visible to a waiter that acquires at cluster scope.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// Arrive on an mbarrier given by its shared::cluster address, release at CTA scope only: for
// hand-offs whose data is tensor memory, ordered by tcgen05.wait + tcgen05.fence around the
// barrier rather than by the memory model.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait with cluster-scope acquire (for barriers that the peer CTA arrives on).
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, unsigned *status) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const long long start = clock64();
    while (!mbar_try_wait_cluster(bar, parity)) {
        if (clock64() - start > kWaitBudgetCycles) {
            atomicOr(status, kStatusTimeout);
            return false;
        }
    }
    return true;
}
// 3-D tiled load into this CTA's shared memory whose completion is counted on an mbarrier that
// may live in either CTA of the pair (no multicast).
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap *map, int32_t c0, int32_t c1,
                                                 int32_t c2, uint32_t cluster_bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
        "%3, %4}], [%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(cluster_bar)
        : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t holder_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(holder_smem),
                 "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
// Pair MMAs and commits are called by all 32 lanes of a converged warp and issued by the lane
// that elect.sync picks (the same lane every time, so a commit tracks that lane's MMAs).  The warp
// computes the descriptors together: values it holds uniformly stay in uniform registers, which
// keeps the issue loop short enough to feed 64-cycle MMAs back to back.
__device__ __forceinline__ void tc_mma_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void tc_mma_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// Arrive once on the mbarrier at offset `bar` in both CTAs of the pair when all previously
// issued pair MMAs of the elected lane complete.
__device__ __forceinline__ void tc_commit_pair_both(uint32_t bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n\t}" ::"r"(bar),
        "h"(static_cast<uint16_t>(3))
        : "memory");
}
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[64]) {
    uint32_t(&lo)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[0]);
    uint32_t(&hi)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[32]);
    tmem_ld32(taddr, lo);
    tmem_ld32(taddr + 32, hi);
}

// Shared-memory matrix descriptor for tcgen05.mma, 128-byte swizzle (sm_100 format):
// start address >> 4 in bits [0,14), leading byte offset >> 4 in [16,30), stride byte offset
// >> 4 in [32,46), version 1 in [46,48), layout type 2 (SWIZZLE_128B) in [61,64).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B and f32 D: D format bits [4,6) = 1,
// A format [7,10) = 1 (bf16), B format [10,13) = 1, A major bit 15, B major bit 16
// (0 = K-major, 1 = MN-major), N >> 3 in [17,23), M >> 4 in [24,29).
__host__ __device__ constexpr uint32_t idesc_bf16_f32(uint32_t M, uint32_t N, uint32_t a_mn_major,
                                                      uint32_t b_mn_major) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (a_mn_major << 15) | (b_mn_major << 16) |
           ((N >> 3) << 17) | ((M >> 4) << 24);
}

}  // namespace apex
