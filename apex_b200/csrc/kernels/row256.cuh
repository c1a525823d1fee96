// row256.cuh -- one 256-wide bf16 head row held by a warp, 8 dims per lane (lane l owns dims
// [8l, 8l+8), one 16-byte load or store per lane): unpacking, and the per-head RMSNorm +
// rotate-half RoPE of shaders/head_norm_rope.metal:28-68, where the RoPE pair (i, i+128)
// meets across lanes l and l^16.
#pragma once

#include "common.cuh"

namespace apex {

constexpr int kRowDim = 256;

__device__ __forceinline__ void unpack8(const uint4 v, float (&f)[8]) {
    f[0] = bf16lo(v.x); f[1] = bf16hi(v.x); f[2] = bf16lo(v.y); f[3] = bf16hi(v.y);
    f[4] = bf16lo(v.z); f[5] = bf16hi(v.z); f[6] = bf16lo(v.w); f[7] = bf16hi(v.w);
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
    uint4 v;
    v.x = pack_bf16(f[0], f[1]);
    v.y = pack_bf16(f[2], f[3]);
    v.z = pack_bf16(f[4], f[5]);
    v.w = pack_bf16(f[6], f[7]);
    return v;
}

// RMSNorm (optional; this lane's 8 weights `w`, already loaded) and RoPE of one 256-wide row held 8
// dims per lane; pair (i, i + 128) meets across lanes l and l ^ 16.  cos/sin of every pair come from
// tables (cs[i], sn[i] for i < rope_pairs) computed beforehand.
__device__ __forceinline__ void norm_rope_row_tab(float (&x)[8], uint32_t lane, bool norm, const float (&w)[8],
                                                  float eps, uint32_t rope_pairs, const float *cs, const float *sn) {
    if (norm) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += x[e] * x[e];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = rsqrtf(ss * (1.0f / static_cast<float>(kRowDim)) + eps);
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = x[e] * inv * w[e];
    }
    if (rope_pairs) {
        const bool low = lane < 16;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const uint32_t i = 8 * (lane & 15) + e;
            const float other = __shfl_xor_sync(0xffffffffu, x[e], 16);
            if (i < rope_pairs) x[e] = low ? (x[e] * cs[i] - other * sn[i]) : (other * sn[i] + x[e] * cs[i]);
        }
    }
}

}  // namespace apex
