// attention_f32.cu -- drop-in for the reference's designed attention_f32 kernel
// (docs/B6_3_attention.md:282-344, launched by apex::attention, :424-431): for every
// (query token t, q head h), softmax over the visible keys of the f32 cache
// [kv_heads][capacity][head_dim], GQA head map kv = h / (q_heads / kv_heads), window rule
// first = window && pos+1 > window ? pos+1-window : 0 with pos = pos0 + t.
//
// B200 layout: one block of 8 warps per (t, h).  Each warp streams its own subset of keys
// with a private online softmax (no block barrier per key chunk, unlike the reference's six
// barriers per 256-key chunk); the eight (m, l, acc) states are merged once at the end.
// Each lane owns head_dim/32 output dims, so K and V rows are read with coalesced loads.
#include "common.cuh"
#include "internal.h"

namespace apex {
namespace {

constexpr int kWarps = 8;
constexpr int kMaxHeadDim = 512;
constexpr int kPerLane = kMaxHeadDim / 32;

__global__ void __launch_bounds__(kWarps * 32)
    attention_f32_kernel(const float *__restrict__ q, const float *__restrict__ K,
                         const float *__restrict__ V, float *__restrict__ out, uint32_t q_heads,
                         uint32_t kv_heads, uint32_t head_dim, uint32_t capacity, uint32_t pos0,
                         uint32_t window, float scale) {
    __shared__ float s_m[kWarps], s_l[kWarps];
    __shared__ float s_acc[kWarps][kMaxHeadDim];

    const uint32_t token = blockIdx.x, head = blockIdx.y;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t kv_head = head / (q_heads / kv_heads);
    const uint32_t pos = pos0 + token;
    const uint32_t first = (window && pos + 1 > window) ? pos + 1 - window : 0;

    const float *qrow = q + (static_cast<uint64_t>(token) * q_heads + head) * head_dim;
    const float *Kh = K + static_cast<uint64_t>(kv_head) * capacity * head_dim;
    const float *Vh = V + static_cast<uint64_t>(kv_head) * capacity * head_dim;

    float qr[kPerLane], acc[kPerLane];
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
        const uint32_t d = lane + 32 * i;
        qr[i] = d < head_dim ? qrow[d] * scale : 0.f;
        acc[i] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    for (uint32_t j = first + warp; j <= pos; j += kWarps) {
        const float *k = Kh + static_cast<uint64_t>(j) * head_dim;
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < kPerLane; ++i) {
            const uint32_t d = lane + 32 * i;
            if (d < head_dim) s += qr[i] * k[d];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        const float m_new = fmaxf(m, s);
        const float alpha = expf(m - m_new);  // 0 on the first key (m = -inf)
        const float p = expf(s - m_new);
        l = l * alpha + p;
        const float *v = Vh + static_cast<uint64_t>(j) * head_dim;
#pragma unroll
        for (int i = 0; i < kPerLane; ++i) {
            const uint32_t d = lane + 32 * i;
            acc[i] = acc[i] * alpha + (d < head_dim ? p * v[d] : 0.f);
        }
        m = m_new;
    }
    if (lane == 0) {
        s_m[warp] = m;
        s_l[warp] = l;
    }
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
        const uint32_t d = lane + 32 * i;
        if (d < head_dim) s_acc[warp][d] = acc[i];
    }
    __syncthreads();
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, s_m[w]);
    float wgt[kWarps], den = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
        wgt[w] = s_l[w] > 0.f ? expf(s_m[w] - M) : 0.f;
        den += wgt[w] * s_l[w];
    }
    float *orow = out + (static_cast<uint64_t>(token) * q_heads + head) * head_dim;
    for (uint32_t d = threadIdx.x; d < head_dim; d += blockDim.x) {
        float num = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) num += wgt[w] * s_acc[w][d];
        orow[d] = num / den;
    }
}

}  // namespace
}  // namespace apex

extern "C" int apex_attention_f32_scaled(const float *q, const float *K, const float *V,
                                         float *out, uint32_t tokens, uint32_t q_heads,
                                         uint32_t kv_heads, uint32_t head_dim, uint32_t capacity,
                                         uint32_t pos0, uint32_t window, float scale,
                                         void *stream) {
    using namespace apex;
    if (tokens == 0) return ok();
    if (!q || !K || !V || !out) return fail(APEX_ERR_INVALID_ARGUMENT, "apex_attention_f32: null tensor");
    if (head_dim == 0 || head_dim > kMaxHeadDim)
        return fail(APEX_ERR_INVALID_ARGUMENT, "apex_attention_f32: head_dim must be in 1..512");
    if (kv_heads == 0 || q_heads == 0 || q_heads % kv_heads)
        return fail(APEX_ERR_INVALID_ARGUMENT, "apex_attention_f32: q_heads must be a multiple of kv_heads");
    if (static_cast<uint64_t>(pos0) + tokens > capacity)
        return fail(APEX_ERR_INVALID_ARGUMENT, "apex_attention_f32: pos0 + tokens exceeds capacity");
    if (q_heads > 65535) return fail(APEX_ERR_INVALID_ARGUMENT, "apex_attention_f32: too many heads");
    const dim3 grid(tokens, q_heads);
    attention_f32_kernel<<<grid, kWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
        q, K, V, out, q_heads, kv_heads, head_dim, capacity, pos0, window, scale);
    const int rc = check_cuda(cudaGetLastError(), "apex_attention_f32");
    return rc ? rc : ok();
}

extern "C" int apex_attention_f32(const float *q, const float *K, const float *V, float *out,
                                  uint32_t tokens, uint32_t q_heads, uint32_t kv_heads,
                                  uint32_t head_dim, uint32_t capacity, uint32_t pos0,
                                  uint32_t window, void *stream) {
    return apex_attention_f32_scaled(q, K, V, out, tokens, q_heads, kv_heads, head_dim, capacity,
                                     pos0, window, 1.0f, stream);
}
