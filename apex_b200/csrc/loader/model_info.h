// model_info.h -- the packed checkpoint's description (manifest.json) and its loading into B200
// device memory.
//
// The reference reads the same manifest into apex::ModelInfo (src/model_info.h:45-207), maps
// core.bin and hands the mapping to the GPU without a copy (src/file.h:27-73, Apple unified
// memory).  A B200 has its own HBM, so here core.bin is copied ONCE into one device allocation at
// the manifest's offsets (a tensor is `device base + TensorInfo::offset`, exactly the reference's
// `Buffer* + offset` addressing), with disk reads and host-to-device copies overlapped through a
// ring of pinned staging buffers; an expert slot of a layer file is one read at its computed
// offset straight into a caller's device buffer.  Digests (SHA-256 per core tensor and per expert
// slot, tools/repack.py:262-287) can be checked on the bytes as they pass through.
//
// Same type and member names as the reference where it has them, so code written against
// src/model_info.h compiles against this header.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <string>
#include <vector>

#if defined(__GNUC__)
#define APEX_LOADER_API __attribute__((visibility("default")))
#else
#define APEX_LOADER_API
#endif

namespace apex {

// One tensor of core.bin (src/model_info.h:45-51) plus its digest.
struct TensorInfo {
    std::string dtype;             // "BF16", "U32", "U8", "F32", ...
    std::vector<std::int64_t> shape;
    std::uint64_t offset = 0;      // bytes from the start of core.bin
    std::uint64_t nbytes = 0;
    std::string sha256;            // hex digest of the tensor's bytes ("" if absent)
};

// One piece of an expert slot (src/model_info.h:54-60); offset is within the slot.
struct ExpertPiece {
    std::string name;
    std::string dtype;
    std::vector<std::int64_t> shape;
    std::uint64_t offset = 0;
    std::uint64_t nbytes = 0;
};

// The model configuration the loader reads (src/model_info.h:63-87).
struct ModelConfig {
    int hidden_size = 0;
    int intermediate_size = 0;
    int moe_intermediate_size = 0;
    int num_attention_heads = 0;
    int num_key_value_heads = 0;
    int head_dim = 0;
    int num_hidden_layers = 0;
    int num_experts = 0;
    int top_k_experts = 0;
    int vocab_size = 0;
    int sliding_window = 0;
    double rms_norm_eps = 0;
    double final_logit_softcapping = 0;
    std::vector<std::string> layer_types;
    int global_head_dim = 0;
    int num_global_key_value_heads = 0;
    bool attention_k_eq_v = false;
    double rope_theta_sliding = 0;
    double rope_theta_full = 0;
    double partial_rotary_factor_full = 0;
};

// One layer_NN.bin: num_experts slots of `stride` bytes.
struct LayerFile {
    int layer = 0;
    std::string file;
    std::uint64_t size = 0;
    std::uint64_t stride = 0;
    int num_experts = 0;
    std::vector<std::string> expert_sha256;
};

struct APEX_LOADER_API ModelInfo {
    std::string dir;
    ModelConfig config;
    int quant_group_size = 0;
    int quant_bits = 0;
    std::string quant_mode;
    std::uint64_t alignment = 0;   // every core tensor starts on a multiple of this
    std::uint64_t core_size = 0;
    std::map<std::string, TensorInfo> core;
    std::uint64_t expert_slot_size = 0;
    std::map<std::string, ExpertPiece> expert_pieces;
    std::vector<LayerFile> layers;

    const TensorInfo &getTensor(const std::string &name) const;
    std::string layer_file(int layer) const;

    // Parses dir/manifest.json and checks it against itself and the files beside it: every core
    // tensor inside core.bin and aligned, core.bin of the stated size, every layer file of
    // num_experts * stride bytes with its pieces inside the stride.  Throws std::runtime_error.
    static ModelInfo load(const std::string &dir);
};

// Result of a copy into device memory.
struct LoadStats {
    std::uint64_t bytes = 0;
    double seconds = 0;
    std::string mismatch;          // name of the first tensor / slot whose digest differed, or ""
};

// Copies core.bin into `dst` (device memory of at least info.core_size bytes) at the manifest's
// offsets; waits for the copies on `stream` before returning.  With verify, every tensor's
// SHA-256 is checked on the way (LoadStats::mismatch names the first that differs).
APEX_LOADER_API LoadStats uploadCore(const ModelInfo &info, void *dst, std::uint64_t capacity, bool verify,
                                     cudaStream_t stream);

// Copies expert slot `expert` of `layer` (stride bytes) into `dst`; waits for the copy.
APEX_LOADER_API LoadStats loadExpert(const ModelInfo &info, int layer, int expert, void *dst,
                                     std::uint64_t capacity, bool verify, cudaStream_t stream);

// Host-only check of every digest in the manifest against the files (tools/repack.py:262-287).
// Returns "" or the first mismatching tensor / slot.
APEX_LOADER_API std::string verifyFiles(const ModelInfo &info);

}  // namespace apex
