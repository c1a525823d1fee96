// loader.cpp -- manifest parsing and checks, core.bin upload into HBM, expert-slot loads, and the
// C ABI of include/apex_loader.h.
//
// Reference: apex::ModelInfo::load (src/model_info.h:123-207) reads the same manifest fields;
// mapFile / touchAll (src/file.h:27-73) map core.bin for a no-copy GPU buffer; the packer's
// verify (tools/repack.py:262-287) re-hashes tensors and slots.
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <fstream>
#include <memory>
#include <sstream>
#include <stdexcept>

#include "../../../include/apex_loader.h"
#include "../kernels/internal.h"
#include "json.h"
#include "model_info.h"
#include "sha256.h"

namespace apex {
namespace {

uint64_t dtype_bytes(const std::string &dt) {
    if (dt == "BF16" || dt == "F16" || dt == "I16" || dt == "U16") return 2;
    if (dt == "F32" || dt == "U32" || dt == "I32") return 4;
    if (dt == "U8" || dt == "I8" || dt == "F8_E4M3" || dt == "BOOL") return 1;
    if (dt == "F64" || dt == "I64" || dt == "U64") return 8;
    return 0;  // unknown: size not checked
}

std::vector<int64_t> shape_of(const json::Value &v) {
    std::vector<int64_t> s;
    for (const auto &d : v.as_array()) s.push_back(d.as_int());
    return s;
}

void check_size(const std::string &what, const std::string &dtype, const std::vector<int64_t> &shape,
                uint64_t nbytes) {
    const uint64_t eb = dtype_bytes(dtype);
    if (!eb) return;
    uint64_t n = 1;
    for (int64_t d : shape) {
        if (d < 0) throw std::runtime_error(what + ": negative dimension");
        n *= static_cast<uint64_t>(d);
    }
    if (n * eb != nbytes)
        throw std::runtime_error(what + ": shape x " + dtype + " is " + std::to_string(n * eb) + " bytes, manifest says " +
                                 std::to_string(nbytes));
}

uint64_t file_size(const std::string &path) {
    struct stat st {};
    if (stat(path.c_str(), &st) != 0) throw std::runtime_error("cannot stat " + path);
    return static_cast<uint64_t>(st.st_size);
}

struct Fd {
    int fd = -1;
    explicit Fd(const std::string &path) : fd(open(path.c_str(), O_RDONLY)) {
        if (fd < 0) throw std::runtime_error("cannot open " + path);
    }
    ~Fd() {
        if (fd >= 0) close(fd);
    }
    void read_at(void *dst, uint64_t n, uint64_t off, const std::string &path) const {
        auto *p = static_cast<uint8_t *>(dst);
        while (n) {
            const ssize_t r = pread(fd, p, n, static_cast<off_t>(off));
            if (r <= 0) throw std::runtime_error("short read of " + path + " at byte " + std::to_string(off));
            p += r;
            off += static_cast<uint64_t>(r);
            n -= static_cast<uint64_t>(r);
        }
    }
};

// Pinned host staging buffers, reused across calls (per process).
struct Staging {
    static constexpr uint64_t kChunk = 32ull << 20;
    static constexpr int kBuffers = 3;
    void *buf[kBuffers] = {};
    cudaEvent_t done[kBuffers] = {};
    bool ok = false;
    Staging() {
        ok = true;
        for (int i = 0; i < kBuffers; ++i) {
            ok = ok && cudaHostAlloc(&buf[i], kChunk, cudaHostAllocDefault) == cudaSuccess &&
                 cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming) == cudaSuccess;
        }
    }
    static Staging &get() {
        static Staging s;
        if (!s.ok) throw std::runtime_error("cannot allocate pinned staging buffers");
        return s;
    }
};

void cuda_or_throw(cudaError_t e, const char *what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace

const TensorInfo &ModelInfo::getTensor(const std::string &name) const {
    auto it = core.find(name);
    if (it == core.end()) throw std::runtime_error("tensor not found: " + name);
    return it->second;
}

std::string ModelInfo::layer_file(int layer) const {
    char name[32];
    std::snprintf(name, sizeof name, "/layer_%02d.bin", layer);
    return dir + name;
}

ModelInfo ModelInfo::load(const std::string &dir) {
    std::ifstream in(dir + "/manifest.json", std::ios::binary);
    if (!in) throw std::runtime_error("ModelInfo: cannot open " + dir + "/manifest.json");
    std::stringstream ss;
    ss << in.rdbuf();
    const json::Value j = json::parse(ss.str());

    ModelInfo m;
    m.dir = dir;
    const auto &tc = j.at("text_config");
    ModelConfig &c = m.config;
    c.hidden_size = static_cast<int>(tc.at("hidden_size").as_int());
    c.intermediate_size = static_cast<int>(tc.at("intermediate_size").as_int());
    c.moe_intermediate_size = static_cast<int>(tc.at("moe_intermediate_size").as_int());
    c.num_attention_heads = static_cast<int>(tc.at("num_attention_heads").as_int());
    c.num_key_value_heads = static_cast<int>(tc.at("num_key_value_heads").as_int());
    c.head_dim = static_cast<int>(tc.at("head_dim").as_int());
    c.num_hidden_layers = static_cast<int>(tc.at("num_hidden_layers").as_int());
    c.num_experts = static_cast<int>(tc.at("num_experts").as_int());
    c.top_k_experts = static_cast<int>(tc.at("top_k_experts").as_int());
    c.vocab_size = static_cast<int>(tc.at("vocab_size").as_int());
    c.sliding_window = static_cast<int>(tc.at("sliding_window").as_int());
    c.rms_norm_eps = tc.at("rms_norm_eps").as_double();
    c.final_logit_softcapping = tc.at("final_logit_softcapping").as_double();
    for (const auto &t : tc.at("layer_types").as_array()) c.layer_types.push_back(t.as_string());
    c.global_head_dim = static_cast<int>(tc.at("global_head_dim").as_int());
    c.num_global_key_value_heads = static_cast<int>(tc.at("num_global_key_value_heads").as_int());
    c.attention_k_eq_v = tc.at("attention_k_eq_v").as_bool();
    const auto &rp = tc.at("rope_parameters");
    c.rope_theta_sliding = rp.at("sliding_attention").at("rope_theta").as_double();
    c.rope_theta_full = rp.at("full_attention").at("rope_theta").as_double();
    c.partial_rotary_factor_full = rp.at("full_attention").at("partial_rotary_factor").as_double();

    const auto &q = j.at("quantization");
    m.quant_group_size = static_cast<int>(q.at("group_size").as_int());
    m.quant_bits = static_cast<int>(q.at("bits").as_int());
    m.quant_mode = q.at("mode").as_string();
    m.alignment = j.has("alignment") ? j.at("alignment").as_u64() : 1;
    if (m.alignment == 0) throw std::runtime_error("manifest: alignment 0");

    const auto &core = j.at("core");
    m.core_size = core.at("size").as_u64();
    const std::string core_path = dir + "/" + (core.has("file") ? core.at("file").as_string() : "core.bin");
    const uint64_t core_file = file_size(core_path);
    if (core_file != m.core_size)
        throw std::runtime_error("core.bin is " + std::to_string(core_file) + " bytes, manifest says " +
                                 std::to_string(m.core_size));
    for (const auto &t : core.at("tensors").as_array()) {
        TensorInfo info;
        const std::string name = t.at("name").as_string();
        info.dtype = t.at("dtype").as_string();
        info.shape = shape_of(t.at("shape"));
        info.offset = t.at("offset").as_u64();
        info.nbytes = t.at("nbytes").as_u64();
        if (t.has("sha256")) info.sha256 = t.at("sha256").as_string();
        if (info.offset % m.alignment)
            throw std::runtime_error("tensor " + name + ": offset " + std::to_string(info.offset) +
                                     " not a multiple of the alignment " + std::to_string(m.alignment));
        if (info.offset > m.core_size || info.nbytes > m.core_size - info.offset)
            throw std::runtime_error("tensor " + name + ": bytes beyond the end of core.bin");
        check_size("tensor " + name, info.dtype, info.shape, info.nbytes);
        if (!m.core.emplace(name, std::move(info)).second) throw std::runtime_error("tensor " + name + " listed twice");
    }

    const auto &layers = j.at("layers").as_array();
    for (const auto &l : layers) {
        LayerFile lf;
        lf.layer = static_cast<int>(l.at("layer").as_int());
        lf.file = l.at("file").as_string();
        lf.size = l.at("size").as_u64();
        lf.stride = l.at("stride").as_u64();
        lf.num_experts = static_cast<int>(l.at("num_experts").as_int());
        if (l.has("expert_sha256"))
            for (const auto &h : l.at("expert_sha256").as_array()) lf.expert_sha256.push_back(h.as_string());
        if (lf.num_experts < 0 || lf.size != static_cast<uint64_t>(lf.num_experts) * lf.stride)
            throw std::runtime_error(lf.file + ": size is not num_experts x stride");
        const uint64_t fs = file_size(dir + "/" + lf.file);
        if (fs != lf.size)
            throw std::runtime_error(lf.file + " is " + std::to_string(fs) + " bytes, manifest says " +
                                     std::to_string(lf.size));
        m.layers.push_back(std::move(lf));
    }
    if (!layers.empty()) {
        // every layer shares the slot layout; read it from the first (as the reference does)
        const auto &l0 = layers.front();
        m.expert_slot_size = l0.at("stride").as_u64();
        for (const auto &p : l0.at("pieces").as_array()) {
            ExpertPiece piece;
            piece.name = p.at("name").as_string();
            piece.dtype = p.at("dtype").as_string();
            piece.shape = shape_of(p.at("shape"));
            piece.offset = p.at("offset").as_u64();
            piece.nbytes = p.at("nbytes").as_u64();
            if (piece.offset > m.expert_slot_size || piece.nbytes > m.expert_slot_size - piece.offset)
                throw std::runtime_error("expert piece " + piece.name + ": bytes beyond the slot");
            const std::string name = piece.name;
            m.expert_pieces.emplace(name, std::move(piece));
        }
        for (const auto &lf : m.layers)
            if (lf.stride != m.expert_slot_size) throw std::runtime_error(lf.file + ": stride differs from layer 0");
    }
    return m;
}

namespace {

// Digest state of the core tensors while core.bin streams past in order.
struct TensorHasher {
    struct Item {
        uint64_t begin, end;
        const std::string *name, *want;
    };
    std::vector<Item> items;  // by offset
    size_t next = 0;          // first tensor not finished
    std::vector<Sha256> sha;
    std::string mismatch;

    explicit TensorHasher(const ModelInfo &info) {
        for (const auto &kv : info.core)
            if (!kv.second.sha256.empty())
                items.push_back({kv.second.offset, kv.second.offset + kv.second.nbytes, &kv.first, &kv.second.sha256});
        std::sort(items.begin(), items.end(), [](const Item &a, const Item &b) { return a.begin < b.begin; });
        sha.resize(items.size());
    }
    // Bytes [off, off + n) of core.bin at p.
    void feed(const uint8_t *p, uint64_t off, uint64_t n) {
        const uint64_t end = off + n;
        for (size_t i = next; i < items.size() && items[i].begin < end; ++i) {
            const uint64_t a = std::max(items[i].begin, off), b = std::min(items[i].end, end);
            if (a < b) sha[i].update(p + (a - off), b - a);
            if (items[i].end <= end) {
                if (mismatch.empty() && sha[i].hex() != *items[i].want) mismatch = *items[i].name;
                if (i == next) ++next;
            }
        }
        while (next < items.size() && items[next].end <= end) ++next;
    }
};

std::string slot_digest(const Fd &fd, const std::string &path, uint64_t off, uint64_t n, uint8_t *tmp, uint64_t tmp_n) {
    Sha256 h;
    for (uint64_t done = 0; done < n;) {
        const uint64_t k = std::min(tmp_n, n - done);
        fd.read_at(tmp, k, off + done, path);
        h.update(tmp, k);
        done += k;
    }
    return h.hex();
}

uint64_t slot_bytes(const ModelInfo &info) {
    uint64_t n = 0;
    for (const auto &kv : info.expert_pieces) n = std::max(n, kv.second.offset + kv.second.nbytes);
    return n;
}

}  // namespace

LoadStats uploadCore(const ModelInfo &info, void *dst, uint64_t capacity, bool verify, cudaStream_t stream) {
    if (!dst) throw std::runtime_error("uploadCore: null destination");
    if (capacity < info.core_size)
        throw std::runtime_error("uploadCore: destination holds " + std::to_string(capacity) + " bytes, core.bin is " +
                                 std::to_string(info.core_size));
    const auto t0 = std::chrono::steady_clock::now();
    const std::string path = info.dir + "/core.bin";
    Fd fd(path);
    Staging &st = Staging::get();
    TensorHasher hasher(info);
    uint64_t off = 0;
    int k = 0;
    while (off < info.core_size) {
        const int slot = k % Staging::kBuffers;
        if (k >= Staging::kBuffers) cuda_or_throw(cudaEventSynchronize(st.done[slot]), "uploadCore: staging reuse");
        const uint64_t n = std::min<uint64_t>(Staging::kChunk, info.core_size - off);
        fd.read_at(st.buf[slot], n, off, path);
        if (verify) hasher.feed(static_cast<const uint8_t *>(st.buf[slot]), off, n);
        cuda_or_throw(cudaMemcpyAsync(static_cast<uint8_t *>(dst) + off, st.buf[slot], n, cudaMemcpyHostToDevice, stream),
                      "uploadCore: copy");
        cuda_or_throw(cudaEventRecord(st.done[slot], stream), "uploadCore: event");
        off += n;
        ++k;
    }
    cuda_or_throw(cudaStreamSynchronize(stream), "uploadCore: synchronize");
    LoadStats s;
    s.bytes = info.core_size;
    s.seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (verify) s.mismatch = hasher.mismatch;
    return s;
}

LoadStats loadExpert(const ModelInfo &info, int layer, int expert, void *dst, uint64_t capacity, bool verify,
                     cudaStream_t stream) {
    if (!dst) throw std::runtime_error("loadExpert: null destination");
    const LayerFile *lf = nullptr;
    for (const auto &l : info.layers)
        if (l.layer == layer) lf = &l;
    if (!lf) throw std::runtime_error("loadExpert: no layer " + std::to_string(layer));
    if (expert < 0 || expert >= lf->num_experts) throw std::runtime_error("loadExpert: expert out of range");
    if (capacity < lf->stride) throw std::runtime_error("loadExpert: destination smaller than a slot");
    const auto t0 = std::chrono::steady_clock::now();
    const std::string path = info.dir + "/" + lf->file;
    Fd fd(path);
    Staging &st = Staging::get();
    const uint64_t base = static_cast<uint64_t>(expert) * lf->stride;
    const uint64_t used = slot_bytes(info);
    Sha256 h;
    uint64_t off = 0;
    int k = 0;
    while (off < lf->stride) {
        const int slot = k % Staging::kBuffers;
        if (k >= Staging::kBuffers) cuda_or_throw(cudaEventSynchronize(st.done[slot]), "loadExpert: staging reuse");
        const uint64_t n = std::min<uint64_t>(Staging::kChunk, lf->stride - off);
        fd.read_at(st.buf[slot], n, base + off, path);
        if (verify && off < used) h.update(st.buf[slot], std::min(n, used - off));
        cuda_or_throw(cudaMemcpyAsync(static_cast<uint8_t *>(dst) + off, st.buf[slot], n, cudaMemcpyHostToDevice, stream),
                      "loadExpert: copy");
        cuda_or_throw(cudaEventRecord(st.done[slot], stream), "loadExpert: event");
        off += n;
        ++k;
    }
    cuda_or_throw(cudaStreamSynchronize(stream), "loadExpert: synchronize");
    LoadStats s;
    s.bytes = lf->stride;
    s.seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (verify && static_cast<size_t>(expert) < lf->expert_sha256.size() && h.hex() != lf->expert_sha256[expert])
        s.mismatch = lf->file + " expert " + std::to_string(expert);
    return s;
}

std::string verifyFiles(const ModelInfo &info) {
    std::vector<uint8_t> tmp(8u << 20);
    {
        const std::string path = info.dir + "/core.bin";
        Fd fd(path);
        std::vector<std::pair<uint64_t, const std::string *>> order;
        for (const auto &kv : info.core)
            if (!kv.second.sha256.empty()) order.emplace_back(kv.second.offset, &kv.first);
        std::sort(order.begin(), order.end());
        for (const auto &o : order) {
            const TensorInfo &t = info.core.at(*o.second);
            if (slot_digest(fd, path, t.offset, t.nbytes, tmp.data(), tmp.size()) != t.sha256) return *o.second;
        }
    }
    const uint64_t used = slot_bytes(info);
    for (const auto &lf : info.layers) {
        const std::string path = info.dir + "/" + lf.file;
        Fd fd(path);
        for (size_t e = 0; e < lf.expert_sha256.size(); ++e)
            if (slot_digest(fd, path, e * lf.stride, used, tmp.data(), tmp.size()) != lf.expert_sha256[e])
                return lf.file + " expert " + std::to_string(e);
    }
    return "";
}

}  // namespace apex

struct apex_model {
    apex::ModelInfo info;
};

extern "C" {

int apex_model_open(const char *dir, apex_model **model) {
    if (!dir || !model) return apex::fail(APEX_ERR_INVALID_ARGUMENT, "apex_model_open: null argument");
    *model = nullptr;
    try {
        auto m = std::make_unique<apex_model>();
        m->info = apex::ModelInfo::load(dir);
        *model = m.release();
    } catch (const std::exception &e) {
        return apex::fail(APEX_ERR_FORMAT, std::string("apex_model_open: ") + e.what());
    }
    return apex::ok();
}

void apex_model_close(apex_model *model) { delete model; }

int apex_model_summary_get(const apex_model *model, apex_model_summary *out) {
    if (!model || !out) return apex::fail(APEX_ERR_INVALID_ARGUMENT, "apex_model_summary_get: null argument");
    const auto &m = model->info;
    const auto &c = m.config;
    *out = apex_model_summary{};
    out->core_size = m.core_size;
    out->alignment = m.alignment;
    out->expert_slot_size = m.expert_slot_size;
    out->core_tensors = static_cast<uint32_t>(m.core.size());
    out->layer_files = static_cast<uint32_t>(m.layers.size());
    out->num_hidden_layers = static_cast<uint32_t>(c.num_hidden_layers);
    out->hidden_size = static_cast<uint32_t>(c.hidden_size);
    out->num_attention_heads = static_cast<uint32_t>(c.num_attention_heads);
    out->num_key_value_heads = static_cast<uint32_t>(c.num_key_value_heads);
    out->head_dim = static_cast<uint32_t>(c.head_dim);
    out->global_head_dim = static_cast<uint32_t>(c.global_head_dim);
    out->num_global_key_value_heads = static_cast<uint32_t>(c.num_global_key_value_heads);
    out->sliding_window = static_cast<uint32_t>(c.sliding_window);
    out->num_experts = static_cast<uint32_t>(c.num_experts);
    out->quant_group_size = static_cast<uint32_t>(m.quant_group_size);
    out->quant_bits = static_cast<uint32_t>(m.quant_bits);
    out->rms_norm_eps = static_cast<float>(c.rms_norm_eps);
    out->rope_theta_sliding = static_cast<float>(c.rope_theta_sliding);
    out->rope_theta_full = static_cast<float>(c.rope_theta_full);
    out->partial_rotary_factor_full = static_cast<float>(c.partial_rotary_factor_full);
    return apex::ok();
}

int apex_model_tensor(const apex_model *model, const char *name, uint64_t *offset, uint64_t *nbytes) {
    if (!model || !name || !offset || !nbytes) return apex::fail(APEX_ERR_INVALID_ARGUMENT, "apex_model_tensor: null argument");
    auto it = model->info.core.find(name);
    if (it == model->info.core.end()) return apex::fail(APEX_ERR_INVALID_ARGUMENT, std::string("tensor not found: ") + name);
    *offset = it->second.offset;
    *nbytes = it->second.nbytes;
    return apex::ok();
}

int apex_model_expert_piece(const apex_model *model, const char *name, uint64_t *offset, uint64_t *nbytes) {
    if (!model || !name || !offset || !nbytes)
        return apex::fail(APEX_ERR_INVALID_ARGUMENT, "apex_model_expert_piece: null argument");
    auto it = model->info.expert_pieces.find(name);
    if (it == model->info.expert_pieces.end())
        return apex::fail(APEX_ERR_INVALID_ARGUMENT, std::string("expert piece not found: ") + name);
    *offset = it->second.offset;
    *nbytes = it->second.nbytes;
    return apex::ok();
}

int apex_model_verify(const apex_model *model) {
    if (!model) return apex::fail(APEX_ERR_INVALID_ARGUMENT, "apex_model_verify: null model");
    try {
        const std::string bad = apex::verifyFiles(model->info);
        if (!bad.empty()) return apex::fail(APEX_ERR_FORMAT, "digest mismatch: " + bad);
    } catch (const std::exception &e) {
        return apex::fail(APEX_ERR_FORMAT, std::string("apex_model_verify: ") + e.what());
    }
    return apex::ok();
}

int apex_model_upload_core(const apex_model *model, void *device_dst, size_t capacity, int verify, void *stream,
                           double *seconds) {
    if (!model) return apex::fail(APEX_ERR_INVALID_ARGUMENT, "apex_model_upload_core: null model");
    try {
        const apex::LoadStats s =
            apex::uploadCore(model->info, device_dst, capacity, verify != 0, static_cast<cudaStream_t>(stream));
        if (seconds) *seconds = s.seconds;
        if (!s.mismatch.empty()) return apex::fail(APEX_ERR_FORMAT, "digest mismatch: " + s.mismatch);
    } catch (const std::exception &e) {
        return apex::fail(APEX_ERR_FORMAT, std::string("apex_model_upload_core: ") + e.what());
    }
    return apex::ok();
}

int apex_model_load_expert(const apex_model *model, uint32_t layer, uint32_t expert, void *device_dst, size_t capacity,
                           int verify, void *stream) {
    if (!model) return apex::fail(APEX_ERR_INVALID_ARGUMENT, "apex_model_load_expert: null model");
    try {
        const apex::LoadStats s = apex::loadExpert(model->info, static_cast<int>(layer), static_cast<int>(expert),
                                                   device_dst, capacity, verify != 0, static_cast<cudaStream_t>(stream));
        if (!s.mismatch.empty()) return apex::fail(APEX_ERR_FORMAT, "digest mismatch: " + s.mismatch);
    } catch (const std::exception &e) {
        return apex::fail(APEX_ERR_FORMAT, std::string("apex_model_load_expert: ") + e.what());
    }
    return apex::ok();
}

}  // extern "C"
