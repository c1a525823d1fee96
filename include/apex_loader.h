/*
 * apex_loader.h -- C ABI of the packed-weights loader: the checkpoint layout the reference's
 * packer writes (core.bin + layer_NN.bin + manifest.json, tools/repack.py:1-36), read into B200
 * device memory.
 *
 * Reference interfaces replaced (paths inside the spotta85/apex tree):
 *   apex_model_open / apex_model_summary / apex_model_tensor / apex_model_expert_piece
 *                        apex::ModelInfo::load, ModelInfo::getTensor, expert_pieces
 *                        (src/model_info.h:92-207)
 *   apex_model_upload_core  mapFile + Backend::wrapNoCopy of core.bin (src/file.h:27-73,
 *                        src/main.cpp:12-21): on a B200 the bytes are copied once into HBM at the
 *                        manifest's offsets instead of being mapped
 *   apex_model_load_expert  "one pread at a computed offset, straight into a GPU-visible buffer"
 *                        (tools/repack.py:17-23)
 *   apex_model_verify    `repack.py verify` (tools/repack.py:262-287): SHA-256 of every core tensor
 *                        and expert slot against the manifest
 * Status codes are those of apex_cuda.h plus APEX_ERR_FORMAT; the message of a failing call is
 * apex_cuda_last_error().  Device pointers are cudaMalloc'd by the caller.
 */
#ifndef APEX_LOADER_H
#define APEX_LOADER_H

#include <stddef.h>
#include <stdint.h>

#include "apex_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

#define APEX_ERR_FORMAT 6 /* a manifest, file size, offset or digest does not match */

typedef struct apex_model apex_model;

typedef struct apex_model_summary {
    uint64_t core_size;          /* bytes of core.bin */
    uint64_t alignment;          /* every core tensor starts on a multiple of this */
    uint64_t expert_slot_size;   /* stride of one expert slot in a layer file */
    uint32_t core_tensors;
    uint32_t layer_files;
    uint32_t num_hidden_layers;
    uint32_t hidden_size;
    uint32_t num_attention_heads;
    uint32_t num_key_value_heads;
    uint32_t head_dim;
    uint32_t global_head_dim;
    uint32_t num_global_key_value_heads;
    uint32_t sliding_window;
    uint32_t num_experts;
    uint32_t quant_group_size;
    uint32_t quant_bits;
    float rms_norm_eps;
    float rope_theta_sliding;
    float rope_theta_full;
    float partial_rotary_factor_full;
} apex_model_summary;

/* Parses dir/manifest.json and checks it against the files beside it (sizes, bounds,
 * alignment).  *model must be released with apex_model_close. */
APEX_API int apex_model_open(const char *dir, apex_model **model);
APEX_API void apex_model_close(apex_model *model);
APEX_API int apex_model_summary_get(const apex_model *model, apex_model_summary *out);
/* Offset and size in core.bin of a core tensor (e.g. "layers.0.self_attn.q_proj.weight"). */
APEX_API int apex_model_tensor(const apex_model *model, const char *name, uint64_t *offset, uint64_t *nbytes);
/* Offset within an expert slot and size of a piece (e.g. "gate_proj.weight"). */
APEX_API int apex_model_expert_piece(const apex_model *model, const char *name, uint64_t *offset, uint64_t *nbytes);
/* Host-only digest check of every core tensor and expert slot. */
APEX_API int apex_model_verify(const apex_model *model);
/* Copies core.bin into device_dst (>= core_size bytes) at the manifest's offsets, overlapping
 * disk reads with host-to-device copies on `stream`; returns when the copy is complete.  With
 * verify != 0 every tensor's digest is checked on the way.  *seconds (may be NULL) = wall time. */
APEX_API int apex_model_upload_core(const apex_model *model, void *device_dst, size_t capacity, int verify,
                                    void *stream, double *seconds);
/* Copies expert slot `expert` of `layer` (expert_slot_size bytes) into device_dst; returns when
 * the copy is complete. */
APEX_API int apex_model_load_expert(const apex_model *model, uint32_t layer, uint32_t expert, void *device_dst,
                                    size_t capacity, int verify, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* APEX_LOADER_H */
