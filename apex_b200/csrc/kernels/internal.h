// internal.h -- host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <string>

#include "../../../include/apex_cuda.h"

namespace apex {

// Records `msg` as this thread's last error and returns `code`.
int fail(int code, const std::string &msg);
// Checks a CUDA runtime result; on failure records it and returns APEX_ERR_CUDA.
int check_cuda(cudaError_t e, const char *what);
// Clears this thread's last error and returns APEX_OK.
int ok();

// Number of SMs of the current device (cached per device).
int sm_count();
// Device address of the current device's status word (see kStatusTimeout), or null.
unsigned *device_status_ptr();

// A 3-D bf16 tensor map with 128-byte swizzle: dims {d0 (innermost, elements), d1, d2},
// byte strides of dims 1 and 2, box {box0, box1, 1}.  Out-of-range elements read as zero.
int make_tensor_map_bf16_3d(CUtensorMap *map, const void *base, uint64_t d0, uint64_t d1,
                            uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes,
                            uint32_t box0, uint32_t box1);

// A 2-D byte tensor map, no swizzle: dims {d0 (innermost, bytes), d1}, byte stride of dim 1, box
// {box0, box1} (box0 a multiple of 16 bytes).
int make_tensor_map_u8_2d(CUtensorMap *map, const void *base, uint64_t d0, uint64_t d1, uint64_t stride1_bytes,
                          uint32_t box0, uint32_t box1);

// A 3-D bf16 tensor map with 128-byte swizzle and a full 3-D box: dims {d0 (innermost, elements),
// d1, d2}, byte strides of dims 1 and 2 (any order), box {box0, box1, box2}.  Out-of-range elements read
// as zero.
int make_tensor_map_bf16_3d_box(CUtensorMap *map, const void *base, const uint64_t (&dims)[3],
                                const uint64_t (&strides_bytes)[2], const uint32_t (&box)[3]);

// A 4-D bf16 tensor map for tiled stores, 128-byte swizzle (rows of up to 64 elements) or 64-byte
// swizzle (up to 32): dims {d0 (innermost), d1, d2, d3}, byte strides of dims 1..3, box {box0, box1,
// box2, box3}.  Elements outside the tensor are not written.
int make_tensor_map_bf16_4d(CUtensorMap *map, const void *base, const uint64_t (&dims)[4],
                            const uint64_t (&strides_bytes)[3], const uint32_t (&box)[4], bool swizzle128);

// inv_freq[i] = base^(-2i/head_dim) (f32 exponent, double-precision power rounded to f32) for
// i < pairs, the frequencies of shaders/head_norm_rope.metal:59.
void rope_table(float *inv_freq, uint32_t pairs, uint32_t head_dim, float base);

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Decode for wide GQA groups / head_dim 512 (decode_gqa.cu): whether `p` takes that form, its
// workspace size, and the launch (same arguments as apex_attn_decode_bf16).
bool gqa_decode_form(const apex_attn_params *p);
size_t gqa_workspace_bytes(const apex_attn_params *p, uint32_t batch, uint32_t max_len);
int launch_gqa_decode(const apex_attn_params *p, const uint16_t *q_raw, const uint16_t *k_new, const uint16_t *v_new,
                      const uint16_t *q_w, const uint16_t *k_w, uint16_t *k_cache, uint16_t *v_cache,
                      uint32_t capacity, const int32_t *seq_lens, uint32_t batch, uint32_t max_seq_len,
                      uint16_t *out, void *workspace, size_t workspace_bytes_given, void *stream, const char *name);

// Prefill for head_dim 512 (prefill_gqa.cu), arguments validated by the caller: the q workspace
// [B][Hq][T][512] it needs, the preparation (q into the workspace; k and v into the caches at pos0)
// and the attention over the caches.
size_t prefill_gqa_workspace_bytes(uint32_t batch, uint32_t tokens, uint32_t q_heads);
int launch_prefill_gqa_prep(const apex_attn_params *p, const uint16_t *q_raw, const uint16_t *k_raw,
                            const uint16_t *v_raw, const uint16_t *q_w, const uint16_t *k_w, uint16_t *k_cache,
                            uint16_t *v_cache, uint32_t capacity, uint32_t batch, uint32_t tokens, uint32_t pos0,
                            void *workspace, cudaStream_t s);
int launch_prefill_gqa_attend(const apex_attn_params *p, const void *workspace, const uint16_t *k_cache,
                              const uint16_t *v_cache, uint32_t capacity, uint32_t batch, uint32_t tokens,
                              uint32_t pos0, uint16_t *out, cudaStream_t s);
// Its tcgen05 attention (prefill_wide.cu) for GQA groups of 1, 2, 4 or 8, over the same workspace.
bool prefill_wide_applies(const apex_attn_params *p);
int launch_prefill_wide_attend(const apex_attn_params *p, const void *workspace, const uint16_t *k_cache,
                               const uint16_t *v_cache, uint32_t capacity, uint32_t batch, uint32_t tokens,
                               uint32_t pos0, uint16_t *out, cudaStream_t s);

}  // namespace apex
