// nvfp4.cu -- the projections either side of the attention path (NVFP4 weights) and RMSNorm.
//
// Reference semantics:
//   matmul_nvfp4 (shaders/matmul.metal:4-53, launched by apex::matmulNvfp4, src/ops.h:34-46):
//     output[t][r] = sum_g e4m3(scales[r][g]) * sum_{i<16} e2m1(code_{r,16g+i}) * input[t][16g+i]
//     with codes uint32 [rows][n/8] (8 codes per word, low nibble first) and E4M3 scales
//     [rows][n/16] (src/nvfp4.h:11-43; CPU form src/tests/cpu_ref.h:48-63).
//   rms_norm_f32 (shaders/norm.metal:36-81, apex::rmsNorm, src/ops.h:18-27):
//     y = x * rsqrt(mean(x^2) + eps) * w, w raw bf16 bits.
//   The attention block ends with out = W_o . o and attn_out = rmsnorm(out, post_attention_norm)
//   (docs/B6_3_attention.md:15-28); apex_matmul_nvfp4_rms_norm fuses the two.
//
// B200 design.  A decode projection is a matrix-vector product over a few tokens: HBM-bound on the
// 0.5625 bytes per weight, with ~3 instructions per weight to decode, so the kernel keeps the decode
// off the critical resources: the E2M1 pairs and the E4M3 scale go through the sm_100 hardware
// conversions (cvt e2m1x2 -> f16x2, e4m3 -> f16; every E2M1 x E4M3 value is exact in f16 and f32),
// each warp owns 2 weight rows so one 16-wide input chunk serves both, every lane keeps 8 groups of
// both rows' codes (64 B) in flight, and a token chunk of 4 reuses each decoded weight 4 times.  Sums
// are f32 (the reference's per-group partial, then scale, then a warp reduction -- its order).
// Inputs are f32 or bf16 (the attention output), outputs f32 or bf16 (raw q/k/v for the bf16 path).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>

#include <algorithm>
#include <string>
#include <type_traits>

#include "common.cuh"
#include "internal.h"

namespace apex {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRowsPerWarp = 2;
constexpr int kRowsPerCta = kWarps * kRowsPerWarp;
constexpr int kTok = 4;         // tokens per pass over the weights
constexpr int kBatch = 8;       // groups of 16 weights per lane in flight
constexpr uint32_t kFusedMaxTokens = 16;  // above this the fused norm runs as a second launch

struct NormEpilogue {
    const uint16_t *weight = nullptr;  // bf16 [rows]; null = no fused norm
    const float *residual = nullptr;   // optional [tokens][rows]
    float *residual_out = nullptr;     // optional: residual + normalised output
    float *ws_sumsq = nullptr;         // [ctas][tokens] per-CTA sums of squares
    unsigned *ws_count = nullptr;      // CTAs done
    float eps = 0.f;
};

__device__ __forceinline__ float e4m3_to_f32(uint8_t b) {
    const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(b), __NV_E4M3);
    return __half2float(__half(h));
}

// 16 weights of one group: byte k of the 8 code bytes holds weights 2k (low nibble) and 2k+1.
__device__ __forceinline__ void decode_group(uint2 c, float (&w)[16]) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const uint32_t word = k < 4 ? c.x : c.y;
        const __half2_raw h = __nv_cvt_fp4x2_to_halfraw2(static_cast<__nv_fp4x2_storage_t>((word >> (8 * (k & 3))) & 0xFFu),
                                                       __NV_E2M1);
        const float2 f = __half22float2(__half2(h));
        w[2 * k] = f.x;
        w[2 * k + 1] = f.y;
    }
}

__device__ __forceinline__ void load16(const float *p, float (&x)[16]) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float4 v = __ldg(reinterpret_cast<const float4 *>(p) + k);
        x[4 * k] = v.x;
        x[4 * k + 1] = v.y;
        x[4 * k + 2] = v.z;
        x[4 * k + 3] = v.w;
    }
}
__device__ __forceinline__ void load16(const __nv_bfloat16 *p, float (&x)[16]) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const uint4 v = __ldg(reinterpret_cast<const uint4 *>(p) + k);
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            x[8 * k + 2 * e] = bf16lo(u[e]);
            x[8 * k + 2 * e + 1] = bf16hi(u[e]);
        }
    }
}

__device__ __forceinline__ void store(float *p, float v) { *p = v; }
__device__ __forceinline__ void store(__nv_bfloat16 *p, float v) { *p = __float2bfloat16_rn(v); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// One CTA = 8 warps x 2 rows.  With a fused norm (ep.weight), TOut is f32 and `out` receives the
// normalised rows: each CTA writes its rows before the norm, its per-token sums of squares to the
// workspace, and the last CTA to finish (atomic counter, no spinning) sums them in CTA order and
// rescales every row.
template <typename TIn, typename TOut>
__global__ void __launch_bounds__(kThreads) nvfp4_matvec_kernel(const TIn *__restrict__ input,
                                                               const uint32_t *__restrict__ codes,
                                                               const uint8_t *__restrict__ scales,
                                                               TOut *__restrict__ out, uint32_t tokens,
                                                               uint32_t rows, uint32_t n, NormEpilogue ep) {
    __shared__ float s_sq[kWarps][kFusedMaxTokens];
    __shared__ int s_last;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t row0 = (blockIdx.x * kWarps + warp) * kRowsPerWarp;
    const uint32_t G = n / 16, wpr = n / 8;
    const bool fused = ep.weight != nullptr;
    // per-token sums of squares of this warp's rows, kept by lane 0 in shared memory (a register
    // array indexed by the runtime token would live on the stack)
    if (lane == 0)
        for (uint32_t t = 0; t < kFusedMaxTokens; ++t) s_sq[warp][t] = 0.f;

    for (uint32_t t0 = 0; t0 < tokens; t0 += kTok) {
        const uint32_t tc = min(static_cast<uint32_t>(kTok), tokens - t0);
        float acc[kRowsPerWarp][kTok];
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
            for (int t = 0; t < kTok; ++t) acc[r][t] = 0.f;

        for (uint32_t gb = 0; gb < G; gb += 32 * kBatch) {
            // this lane's groups gb + lane + 32k: both rows' codes and scales requested together
            uint2 cw[kBatch][kRowsPerWarp];
            uint8_t sc[kBatch][kRowsPerWarp];
#pragma unroll
            for (int k = 0; k < kBatch; ++k) {
                const uint32_t g = gb + lane + 32u * k;
#pragma unroll
                for (int r = 0; r < kRowsPerWarp; ++r) {
                    const uint32_t row = row0 + r;
                    const bool ok = g < G && row < rows;
                    cw[k][r] = ok ? __ldg(reinterpret_cast<const uint2 *>(codes + static_cast<uint64_t>(row) * wpr) + g)
                                  : make_uint2(0u, 0u);
                    sc[k][r] = ok ? __ldg(scales + static_cast<uint64_t>(row) * G + g) : 0;
                }
            }
#pragma unroll
            for (int k = 0; k < kBatch; ++k) {
                const uint32_t g = gb + lane + 32u * k;
                if (g >= G) break;
                float x[kTok][16];
#pragma unroll
                for (int t = 0; t < kTok; ++t) {
                    if (t < static_cast<int>(tc)) {
                        load16(input + static_cast<uint64_t>(t0 + t) * n + 16u * g, x[t]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j) x[t][j] = 0.f;
                    }
                }
#pragma unroll
                for (int r = 0; r < kRowsPerWarp; ++r) {
                    float w[16];
                    decode_group(cw[k][r], w);
                    const float s = e4m3_to_f32(sc[k][r]);
#pragma unroll
                    for (int t = 0; t < kTok; ++t) {
                        float part = 0.f;  // the reference's order: weights j and 8 + j in turn
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            part = fmaf(w[j], x[t][j], part);
                            part = fmaf(w[8 + j], x[t][8 + j], part);
                        }
                        acc[r][t] = fmaf(s, part, acc[r][t]);
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r) {
            const uint32_t row = row0 + r;
#pragma unroll
            for (int t = 0; t < kTok; ++t) {
                const float v = warp_sum(acc[r][t]);
                if (row < rows && t < static_cast<int>(tc)) {
                    if (lane == 0) {
                        store(out + static_cast<uint64_t>(t0 + t) * rows + row, v);
                        if (fused) s_sq[warp][t0 + t] += v * v;  // t0 + t < kFusedMaxTokens when fused
                    }
                }
            }
        }
    }
    if (!fused) return;

    // ---- fused RMSNorm epilogue (tokens <= kFusedMaxTokens; TOut is float)
    __syncthreads();
    if (threadIdx.x < tokens) {
        float v = 0.f;
        for (int w = 0; w < kWarps; ++w) v += s_sq[w][threadIdx.x];
        ep.ws_sumsq[static_cast<uint64_t>(blockIdx.x) * tokens + threadIdx.x] = v;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();  // this CTA's rows and partial sums before its count
        const unsigned prev = atomicAdd(ep.ws_count, 1u);
        s_last = prev == gridDim.x - 1;
        if (s_last) *ep.ws_count = 0;  // ready for the next call
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    __shared__ float s_inv[kFusedMaxTokens];
    if (threadIdx.x < tokens) {
        float total = 0.f;  // CTA order: the same sum on every run
        for (uint32_t c = 0; c < gridDim.x; ++c) total += __ldcg(ep.ws_sumsq + static_cast<uint64_t>(c) * tokens + threadIdx.x);
        s_inv[threadIdx.x] = rsqrtf(total / static_cast<float>(rows) + ep.eps);
    }
    __syncthreads();
    float *o = reinterpret_cast<float *>(out);
    for (uint64_t i = threadIdx.x; i < static_cast<uint64_t>(tokens) * rows; i += kThreads) {
        const uint32_t t = static_cast<uint32_t>(i / rows), r = static_cast<uint32_t>(i % rows);
        const float y = __ldcg(o + i) * s_inv[t] * __uint_as_float(static_cast<uint32_t>(ep.weight[r]) << 16);
        o[i] = y;
        if (ep.residual_out) ep.residual_out[i] = (ep.residual ? ep.residual[i] : 0.f) + y;
    }
}

// The streaming form: a persistent grid of CTAs, each walking 16-row tiles of the matrix.  One
// producer warp copies a tile's codes and scales (each one contiguous run: the rows of a tile are
// adjacent) into a ring of shared-memory stages with 1-D TMA bulk copies; eight consumer warps take
// two rows each, decode from shared memory and accumulate.  The ring keeps 2-4 tiles (50-150 KB)
// in flight per CTA without holding them in registers.
constexpr int kTileRows = 16;
constexpr int kMaxStages = 4;
constexpr uint32_t kStageBudget = 200u * 1024u;

struct TileArgs {
    uint32_t tokens, n, tiles, stages;  // tiles: of all matrices
    uint32_t code_bytes, scale_bytes, stage_bytes;  // per tile / per stage
    unsigned *status;
};

// Up to four matrices of the same width over the same input (q, k and v of one layer): one launch
// walks the tiles of all of them, matrix m owning tiles [tile0[m], tile0[m + 1]).
constexpr int kMaxMats = 4;
struct StreamMats {
    const uint32_t *codes[kMaxMats];
    const uint8_t *scales[kMaxMats];
    void *out[kMaxMats];
    uint32_t rows[kMaxMats];
    uint32_t tile0[kMaxMats + 1];
    uint32_t count;
};

__device__ __forceinline__ uint32_t mat_of(const StreamMats &m, uint32_t tile) {
    uint32_t i = 0;
#pragma unroll
    for (int j = 1; j < kMaxMats; ++j)
        if (static_cast<uint32_t>(j) < m.count && tile >= m.tile0[j]) i = j;
    return i;
}

template <typename TIn, typename TOut, int TK>
__global__ void __launch_bounds__(kThreads + 32, TK == 1 ? 2 : 1) nvfp4_stream_kernel(const TIn *__restrict__ input,
                                                                        const __grid_constant__ StreamMats mats,
                                                                        const TileArgs ta, NormEpilogue ep) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[kMaxStages], empty[kMaxStages];
    __shared__ float s_sq[kWarps][kFusedMaxTokens];
    __shared__ int s_last;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t n = ta.n, G = n / 16;
    const bool fused = ep.weight != nullptr;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < ta.stages; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), kWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kWarps) {  // ------------------------------------------------ producer
        if (lane == 0) {
            uint32_t k = 0;
            for (uint32_t tile = blockIdx.x; tile < ta.tiles; tile += gridDim.x, ++k) {
                const uint32_t slot = k % ta.stages;
                if (k >= ta.stages && !mbar_wait(smem_u32(&empty[slot]), ((k / ta.stages) - 1) & 1, ta.status)) break;
                const uint32_t m = mat_of(mats, tile), local = tile - mats.tile0[m];
                const uint32_t nrows = min(static_cast<uint32_t>(kTileRows), mats.rows[m] - local * kTileRows);
                const uint32_t cb = nrows * (n / 2), sb = nrows * G;
                uint8_t *st = smem + static_cast<size_t>(slot) * ta.stage_bytes;
                const uint32_t fb = smem_u32(&full[slot]);
                // both runs are multiples of 16 bytes at 16-byte offsets (the host checks n and rows)
                mbar_arrive_expect_tx(fb, cb + sb);
                tma_bulk_load(smem_u32(st),
                              reinterpret_cast<const uint8_t *>(mats.codes[m]) + static_cast<uint64_t>(local) * ta.code_bytes,
                              cb, fb);
                tma_bulk_load(smem_u32(st + ta.code_bytes), mats.scales[m] + static_cast<uint64_t>(local) * ta.scale_bytes,
                              sb, fb);
            }
        }
        return;
    }

    // ---------------------------------------------------------------------- consumers
    // per-token sums of squares of this warp's rows, kept by lane 0 in shared memory
    if (lane == 0)
        for (uint32_t t = 0; t < kFusedMaxTokens; ++t) s_sq[warp][t] = 0.f;
    uint32_t k = 0;
    for (uint32_t tile = blockIdx.x; tile < ta.tiles; tile += gridDim.x, ++k) {
        const uint32_t slot = k % ta.stages;
        if (!mbar_wait(smem_u32(&full[slot]), (k / ta.stages) & 1, ta.status)) break;
        const uint8_t *st = smem + static_cast<size_t>(slot) * ta.stage_bytes;
        const uint32_t m = mat_of(mats, tile);
        const uint32_t rows = mats.rows[m];
        TOut *out = static_cast<TOut *>(mats.out[m]);
        const uint32_t rbase = (tile - mats.tile0[m]) * kTileRows;
        const uint32_t lr0 = warp * kRowsPerWarp;  // rows lr0, lr0+1 of the tile
        for (uint32_t t0 = 0; t0 < ta.tokens; t0 += TK) {
            const uint32_t tc = min(static_cast<uint32_t>(TK), ta.tokens - t0);
            float acc[kRowsPerWarp][TK];
#pragma unroll
            for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
                for (int t = 0; t < TK; ++t) acc[r][t] = 0.f;
            for (uint32_t g = lane; g < G; g += 32) {
                float x[TK][16];
#pragma unroll
                for (int t = 0; t < TK; ++t) {
                    if (t < static_cast<int>(tc)) {
                        load16(input + static_cast<uint64_t>(t0 + t) * n + 16u * g, x[t]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j) x[t][j] = 0.f;
                    }
                }
#pragma unroll
                for (int r = 0; r < kRowsPerWarp; ++r) {
                    const uint32_t lr = lr0 + r;
                    if (rbase + lr >= rows) break;
                    const uint2 cw = *reinterpret_cast<const uint2 *>(st + static_cast<size_t>(lr) * (n / 2) + 8u * g);
                    const float s = e4m3_to_f32(st[ta.code_bytes + static_cast<size_t>(lr) * G + g]);
                    float w[16];
                    decode_group(cw, w);
#pragma unroll
                    for (int t = 0; t < TK; ++t) {
                        float part = 0.f;  // the reference's order: weights j and 8 + j in turn
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            part = fmaf(w[j], x[t][j], part);
                            part = fmaf(w[8 + j], x[t][8 + j], part);
                        }
                        acc[r][t] = fmaf(s, part, acc[r][t]);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < kRowsPerWarp; ++r) {
                const uint32_t row = rbase + lr0 + r;
#pragma unroll
                for (int t = 0; t < TK; ++t) {
                    const float v = warp_sum(acc[r][t]);
                    if (row < rows && t < static_cast<int>(tc) && lane == 0) {
                        store(out + static_cast<uint64_t>(t0 + t) * rows + row, v);
                        if (fused) s_sq[warp][t0 + t] += v * v;
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&empty[slot]));
    }
    if (!fused) return;

    // ---- fused RMSNorm epilogue (as in nvfp4_matvec_kernel), among the consumer warps
    asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory");
    if (threadIdx.x < ta.tokens) {
        float v = 0.f;
        for (int w = 0; w < kWarps; ++w) v += s_sq[w][threadIdx.x];
        ep.ws_sumsq[static_cast<uint64_t>(blockIdx.x) * ta.tokens + threadIdx.x] = v;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory");
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(ep.ws_count, 1u);
        s_last = prev == gridDim.x - 1;
        if (s_last) *ep.ws_count = 0;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory");
    if (!s_last) return;
    __threadfence();
    __shared__ float s_inv[kFusedMaxTokens];
    if (threadIdx.x < ta.tokens) {
        float total = 0.f;
        for (uint32_t c = 0; c < gridDim.x; ++c) total += __ldcg(ep.ws_sumsq + static_cast<uint64_t>(c) * ta.tokens + threadIdx.x);
        s_inv[threadIdx.x] = rsqrtf(total / static_cast<float>(mats.rows[0]) + ep.eps);
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory");
    // the fused norm runs with one matrix (the host checks)
    const uint32_t rows0 = mats.rows[0];
    float *o = static_cast<float *>(mats.out[0]);
    for (uint64_t i = threadIdx.x; i < static_cast<uint64_t>(ta.tokens) * rows0; i += kThreads) {
        const uint32_t t = static_cast<uint32_t>(i / rows0), r = static_cast<uint32_t>(i % rows0);
        const float y = __ldcg(o + i) * s_inv[t] * __uint_as_float(static_cast<uint32_t>(ep.weight[r]) << 16);
        o[i] = y;
        if (ep.residual_out) ep.residual_out[i] = (ep.residual ? ep.residual[i] : 0.f) + y;
    }
}

// rms_norm_f32: one CTA per row; sum of squares in f32 over a strided pass, block reduction, then
// y = x * rsqrt(mean + eps) * w (shaders/norm.metal:36-81).  Optional residual add into a second
// output (h = residual + y).
__global__ void __launch_bounds__(256) rms_norm_kernel(const float *__restrict__ input, const uint16_t *__restrict__ w,
                                                       float *__restrict__ result, const float *__restrict__ residual,
                                                       float *__restrict__ residual_out, uint32_t n, float eps) {
    __shared__ float part[8];
    const uint64_t base = static_cast<uint64_t>(blockIdx.x) * n;
    const float *x = input + base;
    const bool vec = (n % 4 == 0) && ((reinterpret_cast<uintptr_t>(input) & 15) == 0);
    float ss = 0.f;
    if (vec) {
        for (uint32_t i = threadIdx.x; i < n / 4; i += blockDim.x) {
            const float4 v = reinterpret_cast<const float4 *>(x)[i];
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
    } else {
        for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) ss += x[i] * x[i];
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (uint32_t k = 0; k < blockDim.x / 32; ++k) tot += part[k];
    const float inv = rsqrtf(tot / static_cast<float>(n) + eps);
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float y = x[i] * inv * __uint_as_float(static_cast<uint32_t>(w[i]) << 16);
        result[base + i] = y;
        if (residual_out) residual_out[base + i] = (residual ? residual[base + i] : 0.f) + y;
    }
}

int check_matvec(const void *input, const uint32_t *codes, const uint8_t *scales, const void *output, uint32_t n,
                 uint32_t rows, uint32_t tokens, bool in_bf16, const char *name) {
    if (!input || !codes || !scales || !output) return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": null tensor");
    if (n == 0 || n % 16)
        return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": hidden_dim must be a positive multiple of 16");
    if (rows == 0 || tokens == 0) return APEX_OK;
    if ((reinterpret_cast<uintptr_t>(codes) & 7) || (reinterpret_cast<uintptr_t>(input) & 15))
        return fail(APEX_ERR_INVALID_ARGUMENT,
                    std::string(name) + ": codes must be 8-byte and input 16-byte aligned");
    (void)in_bf16;
    return APEX_OK;
}

// ---------------------------------------------------------------- tensor-core form (prefill sizes)
// For bf16 input and at least kTcMinTokens tokens the projection is a GEMM: D[r][t] = sum_k W[r][k]
// x[t][k], M = weight rows, N = tokens, K = hidden_dim, run on CTA pairs (tcgen05.mma.cta_group::2,
// M = 256: each CTA dequantises its own 128 weight rows).  A tile is 256 rows x 512 tokens: every
// dequantised 64-wide K step of the weights feeds two N = 256 MMAs (the weights' dequantisation, not
// the tensor cores, is the scarcer resource), and each CTA loads 256 of the 512 tokens (128 of each
// MMA), so an SM streams 32 KB of activations and 4 KB of codes per K step.  Weights stay NVFP4 in
// HBM; eight warps per CTA dequantise each 128 x 64 tile exactly into bf16 (an E2M1 value times its
// E4M3 scale has at most 6 significant bits, so the bf16 product is exact) and write it in the
// 128-byte-swizzled K-major layout a TMA copy would produce; x tiles and the codes come by TMA.
// CTA 0's MMA warp issues tcgen05.mma kind::f16 (f32 accumulate in TMEM, all 512 columns); four
// epilogue warps per CTA read each tile back (TMEM lane = weight row, column c = token tok0 + c;
// each store writes 32 consecutive rows of one token).  The grid is persistent (pairs take tiles
// round-robin, weight-row major so concurrent pairs share weight rows in L2).  Sums are f32 over
// exact products (the order differs from the per-group reference order by f32 rounding only).
// No TMA multicast.
// Three rings per CTA: x halves (B, freed by the MMAs), dequantised weights (A, written by the
// dequantising warps, freed by the MMAs) and raw codes (freed by the dequantising warps as soon as
// they have read them, so the codes run far ahead of the MMAs and a dequantisation never waits for a
// load issued after the MMA that freed its A slot).  The dequantising warps hand each A tile to CTA
// 0's barrier after an async-proxy fence with a CTA-scope arrival (a cluster-scope release per warp
// and step halved the kernel's rate).
constexpr uint32_t kTcBM = 128, kTcBN = 512, kTcBK = 64;  // BM per CTA, BN per pair (two N = 256 MMAs)
constexpr uint32_t kTcSB = 3, kTcSA = 4, kTcSR = 8;       // ring depths: x, A, codes
constexpr uint32_t kTcMinTokens = 32;
constexpr uint32_t kTcABytes = kTcBM * kTcBK * 2;            // 16 KB dequantised weights
constexpr uint32_t kTcBBytes = (kTcBN / 2) * kTcBK * 2;      // 32 KB: this CTA's half of the x tile
constexpr uint32_t kTcBHalf = kTcBBytes / 2;                 // its 128 tokens of one N = 256 MMA
constexpr uint32_t kTcRawBytes = kTcBM * (kTcBK / 2);        // 4 KB codes
constexpr uint32_t kTcOffA = 0, kTcOffB = kTcSA * kTcABytes, kTcOffRaw = kTcOffB + kTcSB * kTcBBytes;
constexpr uint32_t kTcOffBar = kTcOffRaw + kTcSR * kTcRawBytes;
constexpr uint32_t kTcNumBars = 2 * (kTcSB + kTcSA + kTcSR) + 2;
constexpr uint32_t kTcOffTmem = kTcOffBar + 8 * kTcNumBars;
constexpr uint32_t kTcSmem = kTcOffTmem + 16 + 1024;         // + alignment slack of the dynamic base
// warp 0 x loads, 1 MMA, 2-9 dequantise (two threads per row), 10-13 epilogue, 14 code loads
constexpr int kTcThreads = 480;
constexpr uint32_t kTcDqWarps = 8, kTcEpiWarps = 4, kTcCodeWarp = 14;
static_assert(kTcSmem <= 232448, "shared memory budget");

struct TcArgs {
    const uint8_t *scales;
    void *out;
    unsigned *status;
    uint32_t rows, n, tokens, tiles_n, tiles;
};

template <typename TOut>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kTcThreads, 1)
    nvfp4_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_codes,
                    const TcArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t *base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const uint32_t sb = smem_u32(base);
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const uint32_t nk = a.n / kTcBK;
    // CTA 0's b_full, a_full and acc_empty count the pair; the others are each CTA's own
    auto bar_at = [&](uint32_t i) { return sb + kTcOffBar + 8 * i; };
    auto b_full = [&](uint32_t s) { return bar_at(s); };                                   // x halves landed
    auto b_empty = [&](uint32_t s) { return bar_at(kTcSB + s); };                          // MMAs done with them
    auto a_full = [&](uint32_t s) { return bar_at(2 * kTcSB + s); };                       // A tiles written
    auto a_empty = [&](uint32_t s) { return bar_at(2 * kTcSB + kTcSA + s); };              // MMAs done with it
    auto raw_full = [&](uint32_t s) { return bar_at(2 * (kTcSB + kTcSA) + s); };           // codes landed
    auto raw_empty = [&](uint32_t s) { return bar_at(2 * (kTcSB + kTcSA) + kTcSR + s); };  // codes read
    const uint32_t acc_full = bar_at(2 * (kTcSB + kTcSA + kTcSR));
    const uint32_t acc_empty = bar_at(2 * (kTcSB + kTcSA + kTcSR) + 1);
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(base + kTcOffTmem);
    __shared__ int err;

    if (tid == 0) {
        prefetch_tensormap(&tm_x);
        prefetch_tensormap(&tm_codes);
        for (uint32_t s = 0; s < kTcSB; ++s) {
            mbar_init(b_full(s), 1);
            mbar_init(b_empty(s), 1);
        }
        for (uint32_t s = 0; s < kTcSA; ++s) {
            mbar_init(a_full(s), 2 * kTcDqWarps);
            mbar_init(a_empty(s), 1);
        }
        for (uint32_t s = 0; s < kTcSR; ++s) {
            mbar_init(raw_full(s), 1);
            mbar_init(raw_empty(s), kTcDqWarps);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 2 * kTcEpiWarps);
        err = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(tmem_holder), kTcBN);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    bool alive = true;
    // the pair's tiles: pair, + pairs, ...; tile t = (256 weight rows t / tiles_n, 256 tokens t % tiles_n)
    const uint32_t pair = blockIdx.x / 2, pairs = gridDim.x / 2;
    auto tile_row0 = [&](uint32_t t) { return (t / a.tiles_n) * (2 * kTcBM) + rank * kTcBM; };  // this CTA's rows
    auto tile_tok0 = [&](uint32_t t) { return (t % a.tiles_n) * kTcBN; };
    if (warp == 0) {
        // ------------------------------------------------------------ x loads (each CTA its half)
        if (lane == 0) {
            uint32_t g = 0;  // step counter over all tiles
            const uint32_t bf0 = mapa(b_full(0), 0);
            for (uint32_t t = pair; t < a.tiles && alive; t += pairs) {
                // this CTA's 128 tokens of each N = 256 half: tok0 + 128 rank and tok0 + 256 + 128 rank
                const int32_t x0 = static_cast<int32_t>(tile_tok0(t) + rank * 128);
                for (uint32_t kb = 0; kb < nk; ++kb, ++g) {
                    const uint32_t s = g % kTcSB;
                    if (g >= kTcSB && !mbar_wait(b_empty(s), ((g / kTcSB) - 1) & 1, a.status)) {
                        alive = false;
                        break;
                    }
                    // both CTAs' halves complete on CTA 0's barrier (full boxes: tokens past the end
                    // read as zeros)
                    if (leader) mbar_arrive_expect_tx(b_full(s), 2 * kTcBBytes);
                    for (uint32_t h = 0; h < 2; ++h)
                        tma_load_3d_pair(sb + kTcOffB + s * kTcBBytes + h * kTcBHalf, &tm_x, static_cast<int32_t>(kb * kTcBK),
                                         x0 + static_cast<int32_t>(256 * h), 0, bf0 + 8 * s);
                }
            }
        }
    } else if (warp == kTcCodeWarp) {
        // ------------------------------------------------------------ code loads (each CTA its rows)
        if (lane == 0) {
            uint32_t g = 0;
            for (uint32_t t = pair; t < a.tiles && alive; t += pairs) {
                const int32_t r0 = static_cast<int32_t>(tile_row0(t));
                for (uint32_t kb = 0; kb < nk; ++kb, ++g) {
                    const uint32_t s = g % kTcSR;
                    if (g >= kTcSR && !mbar_wait(raw_empty(s), ((g / kTcSR) - 1) & 1, a.status)) {
                        alive = false;
                        break;
                    }
                    mbar_arrive_expect_tx(raw_full(s), kTcRawBytes);
                    tma_load_2d(sb + kTcOffRaw + s * kTcRawBytes, &tm_codes, static_cast<int32_t>(kb * (kTcBK / 2)), r0,
                                raw_full(s));
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (CTA 0, whole warp)
        if (leader) {
            auto wait_all = [&](uint32_t b, uint32_t parity) {  // polls with test_wait (no suspend)
                return __all_sync(0xffffffffu, mbar_wait_spin(b, parity, a.status));
            };
            constexpr uint32_t idesc = idesc_bf16_f32(2 * kTcBM, 256, 0, 0);
            const uint64_t a_desc = smem_desc_sw128(sb + kTcOffA, 16, 1024);
            const uint64_t b_desc = smem_desc_sw128(sb + kTcOffB, 16, 1024);
            uint32_t g = 0, i = 0;
            for (uint32_t t = pair; t < a.tiles && alive; t += pairs, ++i) {
                // both CTAs' epilogues have read the previous tile's accumulator
                if (i >= 1 && !wait_all(acc_empty, (i - 1) & 1)) {
                    alive = false;
                    break;
                }
                tc_fence_after();
                for (uint32_t kb = 0; kb < nk; ++kb, ++g) {
                    const uint32_t sbb = g % kTcSB, sa = g % kTcSA;
                    if (!wait_all(b_full(sbb), (g / kTcSB) & 1) || !wait_all(a_full(sa), (g / kTcSA) & 1)) {
                        alive = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (uint32_t kk = 0; kk < kTcBK / 16; ++kk)  // K = 16 per MMA: +32 bytes inside the swizzle atom
#pragma unroll
                        for (uint32_t h = 0; h < 2; ++h)  // the A tile serves both 256-token halves
                            tc_mma_ss_pair(tmem + 256 * h, a_desc + ((sa * kTcABytes + kk * 32) >> 4),
                                           b_desc + ((sbb * kTcBBytes + h * kTcBHalf + kk * 32) >> 4), idesc,
                                           (kb | kk) ? 1u : 0u);
                    tc_commit_pair_both(b_empty(sbb));
                    tc_commit_pair_both(a_empty(sa));
                }
                if (alive) tc_commit_pair_both(acc_full);
            }
        }
    } else if (warp < 2 + kTcDqWarps) {
        // ------------------------------------------------------------ dequantise (each CTA its rows)
        const uint32_t d = (tid - 64) >> 1, hf = tid & 1;  // row of the tile, half of its 64 weights
        const uint32_t fa0 = mapa(a_full(0), 0);
        uint32_t g = 0;
        for (uint32_t t = pair; t < a.tiles && alive; t += pairs) {
            const uint32_t grow = tile_row0(t) + d;
            const bool row_ok = grow < a.rows;
            const uint8_t *srow = a.scales + static_cast<uint64_t>(row_ok ? grow : 0) * (a.n / 16);
            // the 4 scales of a 64-wide step are one aligned 32-bit word; the next step's is loaded ahead
            uint32_t sc_next = row_ok ? __ldg(reinterpret_cast<const uint32_t *>(srow)) : 0u;
            for (uint32_t kb = 0; kb < nk; ++kb, ++g) {
                const uint32_t sr = g % kTcSR, s = g % kTcSA;
                const uint32_t sc = sc_next;
                if (kb + 1 < nk) sc_next = row_ok ? __ldg(reinterpret_cast<const uint32_t *>(srow + 4 * (kb + 1))) : 0u;
                if (!mbar_wait(raw_full(sr), (g / kTcSR) & 1, a.status)) {
                    alive = false;
                    break;
                }
                // this thread's 32 weights: groups 2hf, 2hf + 1 of the row
                const uint4 c = *reinterpret_cast<const uint4 *>(base + kTcOffRaw + sr * kTcRawBytes + d * (kTcBK / 2) +
                                                                 16 * hf);
                __syncwarp();
                if (lane == 0) mbar_arrive(raw_empty(sr));  // the codes are in registers
                if (g >= kTcSA && !mbar_wait(a_empty(s), ((g / kTcSA) - 1) & 1, a.status)) {
                    alive = false;
                    break;
                }
                const uint32_t words[4] = {c.x, c.y, c.z, c.w};
                const uint32_t arow = sb + kTcOffA + s * kTcABytes + d * 128;  // 1024-aligned tile: row d's 128 B
#pragma unroll
                for (int q = 0; q < 2; ++q) {  // 16 weights per group, its E4M3 scale
                    const uint32_t grp = 2 * hf + q;
                    float w[16];
                    decode_group(make_uint2(words[2 * q], words[2 * q + 1]), w);
                    const float scale = e4m3_to_f32(static_cast<uint8_t>((sc >> (8 * grp)) & 0xFFu));
                    uint32_t pk[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) pk[e] = pack_bf16(w[2 * e] * scale, w[2 * e + 1] * scale);
#pragma unroll
                    for (int h = 0; h < 2; ++h)  // 16-byte chunk c of the row at (c ^ (row & 7)) * 16
                        st_shared_v4(arow + (((2 * grp + h) ^ (d & 7)) << 4),
                                     make_uint4(pk[4 * h], pk[4 * h + 1], pk[4 * h + 2], pk[4 * h + 3]));
                }
                // the tensor cores read the tile through the async proxy; the hand-off to CTA 0's
                // barrier follows the proxy fence (as a TMA-written tile's completion would)
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive_remote(fa0 + 8 * s);
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue (each CTA its rows)
        const uint32_t qd = warp & 3;  // TMEM lanes 32qd.. (this CTA's weight rows 32qd.. of the tile)
        const uint32_t ae0 = mapa(acc_empty, 0);
        TOut *out = static_cast<TOut *>(a.out);
        uint32_t i = 0;
        for (uint32_t t = pair; t < a.tiles && alive; t += pairs, ++i) {
            if (!__all_sync(0xffffffffu, mbar_wait(acc_full, i & 1, a.status))) {
                alive = false;
                break;
            }
            tc_fence_after();
            const uint32_t row = tile_row0(t) + 32 * qd + lane, tok0 = tile_tok0(t);
            const uint32_t taddr = tmem + ((32u * qd) << 16);  // column c = token tok0 + c
#pragma unroll 1
            for (uint32_t j = 0; j < kTcBN / 32; ++j) {
                if (tok0 + 32 * j >= a.tokens) break;  // warp-uniform
                uint32_t v[32];
                tmem_ld32(taddr + 32 * j, v);
                tc_wait_ld(v);
                if (row < a.rows) {
                    const uint32_t n_tok = min(32u, a.tokens - (tok0 + 32 * j));
                    TOut *dst = out + static_cast<uint64_t>(tok0 + 32 * j) * a.rows + row;
#pragma unroll
                    for (int e = 0; e < 32; ++e) {
                        if (static_cast<uint32_t>(e) < n_tok) store(dst, __uint_as_float(v[e]));
                        dst += a.rows;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(ae0);
        }
    }
    // Teardown: after a failed wait copies or MMAs of the pair may still be in flight: give them time
    // to land (bounded) before the pair releases TMEM and shared memory.
    if (!alive) err = 1;
    __syncwarp();
    tc_fence_before();
    cluster_sync();
    if (tid == 0 && err) {
        const long long start = clock64();
        while (clock64() - start < 400000ll) __nanosleep(1000);
    }
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, kTcBN);
    }
}

// Clusters of two that fit on the device at once with this kernel's shared memory; queried once
// per device.
template <typename TOut>
uint32_t tc_max_pairs() {
    static int cached[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && cached[dev]) return static_cast<uint32_t>(cached[dev]);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * static_cast<uint32_t>(sm_count() / 2), 1, 1);
    cfg.blockDim = dim3(kTcThreads, 1, 1);
    cfg.dynamicSmemBytes = kTcSmem;
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, nvfp4_tc_kernel<TOut>, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();  // clear the query's error; fall back to one pair per two SMs
        n = sm_count() / 2;
    }
    if (dev >= 0 && dev < 64) cached[dev] = n;
    return static_cast<uint32_t>(n);
}

template <typename TOut>
int launch_tc(const void *input, const uint32_t *codes, const uint8_t *scales, void *output, uint32_t n, uint32_t rows,
              uint32_t tokens, void *stream, const char *name) {
    CUtensorMap tx, tcodes;
    // x [tokens][n] bf16: one box = 128 tokens x 64 elements (128-byte swizzle, K-major): a CTA's
    // share of one N = 256 MMA
    int rc = make_tensor_map_bf16_3d(&tx, input, n, tokens, 1, n * 2ull, n * 2ull * tokens, kTcBK, 128);
    if (rc) return rc;
    // codes [rows][n/2] bytes: one box = 128 rows x 32 bytes (64 weights)
    rc = make_tensor_map_u8_2d(&tcodes, codes, n / 2, rows, n / 2, kTcBK / 2, kTcBM);
    if (rc) return rc;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        rc = check_cuda(cudaFuncSetAttribute(nvfp4_tc_kernel<TOut>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kTcSmem)),
                        name);
        if (rc) return rc;
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    TcArgs ta{};
    ta.scales = scales;
    ta.out = output;
    ta.status = device_status_ptr();
    if (!ta.status) return fail(APEX_ERR_CUDA, std::string(name) + ": device status word unavailable");
    ta.rows = rows;
    ta.n = n;
    ta.tokens = tokens;
    ta.tiles_n = (tokens + kTcBN - 1) / kTcBN;
    ta.tiles = ((rows + 2 * kTcBM - 1) / (2 * kTcBM)) * ta.tiles_n;
    const uint32_t grid = 2 * std::min<uint32_t>(ta.tiles, tc_max_pairs<TOut>());  // one CTA pair per two SMs
    nvfp4_tc_kernel<TOut><<<grid, kTcThreads, kTcSmem, static_cast<cudaStream_t>(stream)>>>(tx, tcodes, ta);
    rc = check_cuda(cudaGetLastError(), name);
    return rc ? rc : ok();
}

// The tensor-core form applies to bf16 input from kTcMinTokens tokens, hidden_dim a multiple of 64,
// 16-byte aligned input and codes and 4-byte aligned scales.
bool tc_applies(bool in_bf16, const void *input, const uint32_t *codes, const uint8_t *scales, uint32_t n,
                uint32_t tokens, uint32_t rows) {
    return in_bf16 && tokens >= kTcMinTokens && n % kTcBK == 0 && rows > 0 &&
           static_cast<uint64_t>((rows + kTcBM - 1) / kTcBM) * ((tokens + kTcBN - 1) / kTcBN) < (1ull << 31) &&
           !(reinterpret_cast<uintptr_t>(input) & 15) && !(reinterpret_cast<uintptr_t>(codes) & 15) &&
           !(reinterpret_cast<uintptr_t>(scales) & 3);
}

// The streaming form applies when every tile's codes and scales are whole 16-byte runs at 16-byte
// offsets (n a multiple of 32, and of 256 unless the rows fill whole tiles) and two stages fit.
bool stream_plan(const StreamMats &mats, uint32_t n, uint32_t tokens, TileArgs &ta, uint32_t &grid, size_t &smem) {
    if (n % 32) return false;
    for (uint32_t m = 0; m < mats.count; ++m)
        if ((n % 256 && mats.rows[m] % kTileRows) || (reinterpret_cast<uintptr_t>(mats.codes[m]) & 15) ||
            (reinterpret_cast<uintptr_t>(mats.scales[m]) & 15))
            return false;
    ta.tokens = tokens;
    ta.n = n;
    ta.tiles = mats.tile0[mats.count];
    ta.code_bytes = kTileRows * (n / 2);
    ta.scale_bytes = kTileRows * (n / 16);
    ta.stage_bytes = (ta.code_bytes + ta.scale_bytes + 127) & ~127u;
    ta.stages = std::min<uint32_t>(kMaxStages, kStageBudget / ta.stage_bytes);
    if (ta.stages < 2) return false;
    ta.stages = std::min<uint32_t>(ta.stages, std::max<uint32_t>(2, ta.tiles));
    smem = static_cast<size_t>(ta.stages) * ta.stage_bytes;
    const uint32_t per_sm = smem <= 100u * 1024u ? 2u : 1u;
    grid = std::min<uint32_t>(ta.tiles, per_sm * static_cast<uint32_t>(sm_count()));
    ta.status = device_status_ptr();
    return ta.status != nullptr;
}

StreamMats one_matrix(const uint32_t *codes, const uint8_t *scales, void *output, uint32_t rows) {
    StreamMats m{};
    m.codes[0] = codes;
    m.scales[0] = scales;
    m.out[0] = output;
    m.rows[0] = rows;
    m.tile0[1] = (rows + kTileRows - 1) / kTileRows;
    m.count = 1;
    return m;
}

template <typename TIn, typename TOut>
int launch_stream(const void *input, const StreamMats &mats, const TileArgs &ta, uint32_t grid, size_t smem,
                  const NormEpilogue &ep, void *stream, const char *name) {
    auto *kernel = ta.tokens == 1 ? nvfp4_stream_kernel<TIn, TOut, 1> : nvfp4_stream_kernel<TIn, TOut, kTok>;
    int rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kStageBudget)),
                        name);
    if (rc) return rc;
    kernel<<<grid, kThreads + 32, smem, static_cast<cudaStream_t>(stream)>>>(static_cast<const TIn *>(input), mats,
                                                                             ta, ep);
    rc = check_cuda(cudaGetLastError(), name);
    return rc ? rc : ok();
}

template <typename TIn, typename TOut>
int launch_matvec(const void *input, const uint32_t *codes, const uint8_t *scales, void *output, uint32_t n,
                  uint32_t rows, uint32_t tokens, const NormEpilogue &ep, void *stream, const char *name) {
    TileArgs ta{};
    uint32_t grid = 0;
    size_t smem = 0;
    if (!ep.weight && tc_applies(std::is_same<TIn, __nv_bfloat16>::value, input, codes, scales, n, tokens, rows))
        return launch_tc<TOut>(input, codes, scales, output, n, rows, tokens, stream, name);
    const StreamMats mats = one_matrix(codes, scales, output, rows);
    if (stream_plan(mats, n, tokens, ta, grid, smem))
        return launch_stream<TIn, TOut>(input, mats, ta, grid, smem, ep, stream, name);
    const uint32_t ctas = (rows + kRowsPerCta - 1) / kRowsPerCta;
    nvfp4_matvec_kernel<TIn, TOut><<<ctas, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const TIn *>(input), codes, scales, static_cast<TOut *>(output), tokens, rows, n, ep);
    const int rc = check_cuda(cudaGetLastError(), name);
    return rc ? rc : ok();
}

}  // namespace
}  // namespace apex

extern "C" int apex_matmul_nvfp4(const void *input, int input_bf16, const uint32_t *codes, const uint8_t *scales,
                                 void *output, int output_bf16, uint32_t hidden_dim, uint32_t w_rows,
                                 uint32_t tokens, void *stream) {
    using namespace apex;
    const char *name = "apex_matmul_nvfp4";
    int rc = check_matvec(input, codes, scales, output, hidden_dim, w_rows, tokens, input_bf16 != 0, name);
    if (rc) return rc;
    if (w_rows == 0 || tokens == 0) return ok();
    const NormEpilogue none{};
    if (input_bf16)
        return output_bf16 ? launch_matvec<__nv_bfloat16, __nv_bfloat16>(input, codes, scales, output, hidden_dim, w_rows,
                                                                           tokens, none, stream, name)
                           : launch_matvec<__nv_bfloat16, float>(input, codes, scales, output, hidden_dim, w_rows, tokens,
                                                                  none, stream, name);
    return output_bf16 ? launch_matvec<float, __nv_bfloat16>(input, codes, scales, output, hidden_dim, w_rows, tokens,
                                                              none, stream, name)
                       : launch_matvec<float, float>(input, codes, scales, output, hidden_dim, w_rows, tokens, none,
                                                     stream, name);
}

extern "C" int apex_matmul_nvfp4_f32(const float *input, const uint32_t *codes, const uint8_t *scales, float *output,
                                     uint32_t hidden_dim, uint32_t w_rows, uint32_t tokens, void *stream) {
    return apex_matmul_nvfp4(input, 0, codes, scales, output, 0, hidden_dim, w_rows, tokens, stream);
}

extern "C" int apex_rms_norm_f32(const float *input, const uint16_t *weight, float *result, uint32_t rows,
                                 uint32_t hidden_dim, float eps, void *stream) {
    using namespace apex;
    if (rows == 0) return ok();
    if (!input || !weight || !result) return fail(APEX_ERR_INVALID_ARGUMENT, "apex_rms_norm_f32: null tensor");
    if (hidden_dim == 0) return fail(APEX_ERR_INVALID_ARGUMENT, "apex_rms_norm_f32: hidden_dim 0");
    rms_norm_kernel<<<rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(input, weight, result, nullptr, nullptr,
                                                                        hidden_dim, eps);
    const int rc = check_cuda(cudaGetLastError(), "apex_rms_norm_f32");
    return rc ? rc : ok();
}

extern "C" size_t apex_matmul_nvfp4_rms_norm_workspace_bytes(uint32_t w_rows, uint32_t tokens) {
    // one partial per CTA of whichever form runs (the streaming grid never exceeds the tile count)
    const size_t ctas = (static_cast<size_t>(w_rows) + apex::kRowsPerCta - 1) / apex::kRowsPerCta;
    return ((ctas * std::max<uint32_t>(tokens, 1) * sizeof(float) + 255) & ~static_cast<size_t>(255)) + 256;
}

extern "C" int apex_matmul_nvfp4_rms_norm(const void *input, int input_bf16, const uint32_t *codes,
                                          const uint8_t *scales, const uint16_t *norm_weight, const float *residual,
                                          float *output, float *residual_out, uint32_t hidden_dim, uint32_t w_rows,
                                          uint32_t tokens, float eps, void *workspace, size_t workspace_bytes,
                                          void *stream) {
    using namespace apex;
    const char *name = "apex_matmul_nvfp4_rms_norm";
    int rc = check_matvec(input, codes, scales, output, hidden_dim, w_rows, tokens, input_bf16 != 0, name);
    if (rc) return rc;
    if (w_rows == 0 || tokens == 0) return ok();
    if (!norm_weight) return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": null norm weight");
    if (tokens > kFusedMaxTokens) {  // prefill-sized: the projection, then the norm as its own launch
        rc = apex_matmul_nvfp4(input, input_bf16, codes, scales, output, 0, hidden_dim, w_rows, tokens, stream);
        if (rc) return rc;
        rms_norm_kernel<<<tokens, 256, 0, static_cast<cudaStream_t>(stream)>>>(output, norm_weight, output, residual,
                                                                              residual_out, w_rows, eps);
        rc = check_cuda(cudaGetLastError(), name);
        return rc ? rc : ok();
    }
    const size_t need = apex_matmul_nvfp4_rms_norm_workspace_bytes(w_rows, tokens);
    if (!workspace || workspace_bytes < need)
        return fail(APEX_ERR_WORKSPACE, std::string(name) + ": workspace of " + std::to_string(need) + " bytes required");
    NormEpilogue ep;
    ep.weight = norm_weight;
    ep.residual = residual;
    ep.residual_out = residual_out;
    ep.ws_sumsq = static_cast<float *>(workspace);
    ep.ws_count = reinterpret_cast<unsigned *>(static_cast<uint8_t *>(workspace) + need - 256);
    ep.eps = eps;
    return input_bf16 ? launch_matvec<__nv_bfloat16, float>(input, codes, scales, output, hidden_dim, w_rows, tokens, ep,
                                                            stream, name)
                      : launch_matvec<float, float>(input, codes, scales, output, hidden_dim, w_rows, tokens, ep,
                                                    stream, name);
}

extern "C" int apex_matmul_nvfp4_multi(const void *input, int input_bf16, uint32_t count,
                                       const uint32_t *const *codes, const uint8_t *const *scales,
                                       void *const *outputs, const uint32_t *w_rows, int output_bf16,
                                       uint32_t hidden_dim, uint32_t tokens, void *stream) {
    using namespace apex;
    const char *name = "apex_matmul_nvfp4_multi";
    if (count == 0) return ok();
    if (count > static_cast<uint32_t>(kMaxMats))
        return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": at most 4 matrices");
    if (!codes || !scales || !outputs || !w_rows) return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": null array");
    StreamMats mats{};
    mats.count = count;
    for (uint32_t m = 0; m < count; ++m) {
        const int rc = check_matvec(input, codes[m], scales[m], outputs[m], hidden_dim, w_rows[m], tokens,
                                    input_bf16 != 0, name);
        if (rc) return rc;
        mats.codes[m] = codes[m];
        mats.scales[m] = scales[m];
        mats.out[m] = outputs[m];
        mats.rows[m] = w_rows[m];
        mats.tile0[m + 1] = mats.tile0[m] + (w_rows[m] + kTileRows - 1) / kTileRows;
    }
    if (tokens == 0 || mats.tile0[count] == 0) return ok();
    TileArgs ta{};
    uint32_t grid = 0;
    size_t smem = 0;
    bool empty_matrix = false, tensor_core = true;
    for (uint32_t m = 0; m < count; ++m) {
        empty_matrix = empty_matrix || w_rows[m] == 0;
        tensor_core = tensor_core && tc_applies(input_bf16 != 0, input, codes[m], scales[m], hidden_dim, tokens, w_rows[m]);
    }
    // prefill sizes: one tensor-core GEMM per matrix (below) instead of the streaming walk
    if (!empty_matrix && !tensor_core && stream_plan(mats, hidden_dim, tokens, ta, grid, smem)) {
        const NormEpilogue none{};
        if (input_bf16)
            return output_bf16 ? launch_stream<__nv_bfloat16, __nv_bfloat16>(input, mats, ta, grid, smem, none, stream, name)
                               : launch_stream<__nv_bfloat16, float>(input, mats, ta, grid, smem, none, stream, name);
        return output_bf16 ? launch_stream<float, __nv_bfloat16>(input, mats, ta, grid, smem, none, stream, name)
                           : launch_stream<float, float>(input, mats, ta, grid, smem, none, stream, name);
    }
    // prefill sizes, or shapes the streaming form does not take: one launch per matrix
    for (uint32_t m = 0; m < count; ++m) {
        const int rc = apex_matmul_nvfp4(input, input_bf16, codes[m], scales[m], outputs[m], output_bf16, hidden_dim,
                                         w_rows[m], tokens, stream);
        if (rc) return rc;
    }
    return ok();
}
