// head_norm_rope.cu -- per-(token, head) RMSNorm + optional bf16 weight + rotate-half RoPE,
// written with caller-chosen strides.  The f32 entry point is the drop-in for the reference
// kernel head_norm_rope_f32 (shaders/head_norm_rope.metal:5-74, launched by src/ops.h:88-122);
// the bf16 entry point is the same operation on bf16 tensors (the bf16 KV-cache append).
//
// B200 layout: one warp per (token, head) row instead of the reference's 256-thread group.
// The row is staged once in shared memory (so input == output is safe: every read of the
// row happens before its writes), the sum of squares is a warp shuffle reduction, and the
// RoPE inverse frequencies are computed once per block into shared memory.
#include "common.cuh"
#include "internal.h"

namespace apex {
namespace {

constexpr int kRowsPerBlock = 8;  // warps per block
constexpr int kMaxHeadDim = 512;  // the reference stages rows in row[512]

template <typename T>
__device__ __forceinline__ float load_elem(const T *p);
template <>
__device__ __forceinline__ float load_elem<float>(const float *p) { return *p; }
template <>
__device__ __forceinline__ float load_elem<uint16_t>(const uint16_t *p) {
    return __uint_as_float(static_cast<uint32_t>(*p) << 16);
}
template <typename T>
__device__ __forceinline__ void store_elem(T *p, float v);
template <>
__device__ __forceinline__ void store_elem<float>(float *p, float v) { *p = v; }
template <>
__device__ __forceinline__ void store_elem<uint16_t>(uint16_t *p, float v) {
    __nv_bfloat16 b = __float2bfloat16_rn(v);
    *p = *reinterpret_cast<uint16_t *>(&b);
}

template <typename T>
__global__ void __launch_bounds__(kRowsPerBlock * 32)
    head_norm_rope_kernel(const T *input, const uint16_t *__restrict__ weight,
                          T *output, uint32_t tokens, uint32_t heads, uint32_t head_dim,
                          uint32_t has_weight, uint32_t rope_pairs, float rope_base,
                          uint32_t abs_pos, uint32_t out_token_stride, uint32_t out_head_stride,
                          float eps, const __grid_constant__ RopeTable rope) {
    __shared__ float inv_freq[kMaxHeadDim / 2];
    __shared__ float rows[kRowsPerBlock][kMaxHeadDim];
    for (uint32_t i = threadIdx.x; i < rope_pairs; i += blockDim.x) inv_freq[i] = rope.inv_freq[i];
    __syncthreads();

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float *row = rows[warp];
    const uint32_t half = head_dim / 2;
    const uint64_t total = static_cast<uint64_t>(tokens) * heads;
    for (uint64_t r = static_cast<uint64_t>(blockIdx.x) * kRowsPerBlock + warp; r < total;
         r += static_cast<uint64_t>(gridDim.x) * kRowsPerBlock) {
        const uint32_t token = static_cast<uint32_t>(r / heads);
        const uint32_t head = static_cast<uint32_t>(r % heads);
        const T *in = input + r * head_dim;
        float ss = 0.f;
        for (uint32_t i = lane; i < head_dim; i += 32) {
            const float x = load_elem(in + i);
            row[i] = x;
            ss += x * x;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = 1.0f / sqrtf(ss / static_cast<float>(head_dim) + eps);
        for (uint32_t i = lane; i < head_dim; i += 32) {
            const float w = has_weight ? __uint_as_float(static_cast<uint32_t>(weight[i]) << 16) : 1.0f;
            row[i] = row[i] * inv * w;
        }
        __syncwarp();
        const float pos = static_cast<float>(abs_pos + token);
        for (uint32_t i = lane; i < rope_pairs; i += 32) {
            float s, c;
            rope_sincos(pos * inv_freq[i], s, c);
            const float a = row[i], b = row[half + i];
            row[i] = a * c - b * s;
            row[half + i] = a * s + b * c;
        }
        __syncwarp();
        T *out = output + static_cast<uint64_t>(token) * out_token_stride +
                 static_cast<uint64_t>(head) * out_head_stride;
        for (uint32_t i = lane; i < head_dim; i += 32) store_elem(out + i, row[i]);
        __syncwarp();
    }
}

template <typename T>
int launch(const T *input, const uint16_t *weight, T *output, uint32_t tokens, uint32_t heads,
           uint32_t head_dim, uint32_t has_weight, uint32_t rope_pairs, float rope_base,
           uint32_t abs_pos, uint32_t out_token_stride, uint32_t out_head_stride, float eps,
           void *stream, const char *name) {
    if (tokens == 0 || heads == 0) return ok();
    if (!input || !output) return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": null tensor");
    if (has_weight && !weight) return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": null weight");
    if (head_dim == 0 || head_dim > kMaxHeadDim || (head_dim & 1))
        return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": head_dim must be even and <= 512");
    if (rope_pairs > head_dim / 2)
        return fail(APEX_ERR_INVALID_ARGUMENT, std::string(name) + ": rope_pairs > head_dim / 2");
    const uint64_t rows = static_cast<uint64_t>(tokens) * heads;
    const uint64_t want = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
    const uint32_t grid = static_cast<uint32_t>(std::min<uint64_t>(want, 16ull * sm_count()));
    RopeTable rope{};
    rope_table(rope.inv_freq, rope_pairs, head_dim, rope_base);
    head_norm_rope_kernel<T><<<grid, kRowsPerBlock * 32, 0, static_cast<cudaStream_t>(stream)>>>(
        input, weight, output, tokens, heads, head_dim, has_weight, rope_pairs, rope_base, abs_pos,
        out_token_stride, out_head_stride, eps, rope);
    const int rc = check_cuda(cudaGetLastError(), name);
    return rc ? rc : ok();
}

}  // namespace
}  // namespace apex

extern "C" int apex_head_norm_rope_f32(const float *input, const uint16_t *weight, float *output,
                                       uint32_t tokens, uint32_t heads, uint32_t head_dim,
                                       uint32_t has_weight, uint32_t rope_pairs, float rope_base,
                                       uint32_t abs_pos, uint32_t out_token_stride,
                                       uint32_t out_head_stride, float eps, void *stream) {
    return apex::launch<float>(input, weight, output, tokens, heads, head_dim, has_weight,
                               rope_pairs, rope_base, abs_pos, out_token_stride, out_head_stride,
                               eps, stream, "apex_head_norm_rope_f32");
}

extern "C" int apex_head_norm_rope_bf16(const uint16_t *input, const uint16_t *weight,
                                        uint16_t *output, uint32_t tokens, uint32_t heads,
                                        uint32_t head_dim, uint32_t has_weight,
                                        uint32_t rope_pairs, float rope_base, uint32_t abs_pos,
                                        uint32_t out_token_stride, uint32_t out_head_stride,
                                        float eps, void *stream) {
    return apex::launch<uint16_t>(input, weight, output, tokens, heads, head_dim, has_weight,
                                  rope_pairs, rope_base, abs_pos, out_token_stride,
                                  out_head_stride, eps, stream, "apex_head_norm_rope_bf16");
}
