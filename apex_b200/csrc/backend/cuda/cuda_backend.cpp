// cuda_backend.cpp -- CudaBackend: the reference's Backend contract on CUDA (see the header).
#include "cuda_backend.h"

#include <chrono>
#include <cstdio>
#include <cstring>
#include <functional>
#include <stdexcept>
#include <vector>

#include "../../../../include/apex_cuda.h"

namespace apex {

// ------------------------------------------------------------------ ledger and phase table
MemoryLedger &MemoryLedger::get() {
    static MemoryLedger m;
    return m;
}
void MemoryLedger::add(const std::string &category, size_t bytes) {
    std::lock_guard<std::mutex> lock(mu_);
    bytes_[category] += bytes;
    current_ += bytes;
    if (current_ > peak_) peak_ = current_;
}
void MemoryLedger::remove(const std::string &category, size_t bytes) {
    std::lock_guard<std::mutex> lock(mu_);
    size_t &b = bytes_[category];
    b = b > bytes ? b - bytes : 0;
    current_ = current_ > bytes ? current_ - bytes : 0;
}
size_t MemoryLedger::current() const {
    std::lock_guard<std::mutex> lock(mu_);
    return current_;
}
size_t MemoryLedger::peak() const {
    std::lock_guard<std::mutex> lock(mu_);
    return peak_;
}
void MemoryLedger::print(FILE *out) const {
    std::lock_guard<std::mutex> lock(mu_);
    std::fprintf(out, "%-24s %14s\n", "category", "bytes");
    for (const auto &[name, b] : bytes_) std::fprintf(out, "%-24s %14zu\n", name.c_str(), b);
    std::fprintf(out, "%-24s %14zu\n%-24s %14zu\n", "total", current_, "peak", peak_);
}

PhaseTable &PhaseTable::get() {
    static PhaseTable t;
    return t;
}
void PhaseTable::add(const std::string &phase, double ms) {
    std::lock_guard<std::mutex> lock(mu_);
    Stats &s = stats_[phase];
    s.total_ms += ms;
    s.calls++;
    if (ms > s.max_ms) s.max_ms = ms;
}
void PhaseTable::print(FILE *out) const {
    std::lock_guard<std::mutex> lock(mu_);
    std::fprintf(out, "%-24s %10s %8s %10s %10s\n", "phase", "total ms", "calls", "avg ms", "max ms");
    for (const auto &[name, s] : stats_)
        std::fprintf(out, "%-24s %10.2f %8ld %10.3f %10.3f\n", name.c_str(), s.total_ms, s.calls,
                     s.total_ms / s.calls, s.max_ms);
}

// ------------------------------------------------------------------ helpers
namespace {

void cuda_check(cudaError_t e, const char *what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

void apex_check(int rc, const char *kernel) {
    if (rc != APEX_OK)
        throw std::runtime_error(std::string(kernel) + ": " + apex_cuda_last_error());
}

// Device pointer of a buffer argument (null buffer -> null pointer).
template <class T>
T *ptr(const Arg &a, const char *kernel, size_t index) {
    if (a.bytes) throw std::runtime_error(std::string(kernel) + ": argument " + std::to_string(index) +
                                          " must be a buffer");
    if (!a.buffer) return nullptr;
    if (a.offset > a.buffer->length)
        throw std::runtime_error(std::string(kernel) + ": offset beyond buffer " + std::to_string(index));
    return reinterpret_cast<T *>(static_cast<uint8_t *>(a.buffer->ptr) + a.offset);
}

size_t bytes_after(const Arg &a) { return a.buffer ? a.buffer->length - a.offset : 0; }

template <class T>
T val(const Arg &a, const char *kernel, size_t index) {
    if (!a.bytes || a.size != sizeof(T))
        throw std::runtime_error(std::string(kernel) + ": argument " + std::to_string(index) +
                                 " must be a " + std::to_string(sizeof(T)) + "-byte value");
    T v;
    std::memcpy(&v, a.bytes, sizeof(T));
    return v;
}

using Launcher = std::function<void(const std::vector<Arg> &, Dim3, cudaStream_t)>;

void need_args(const std::vector<Arg> &a, size_t n, const char *kernel) {
    if (a.size() != n)
        throw std::runtime_error(std::string(kernel) + ": expected " + std::to_string(n) + " arguments, got " +
                                 std::to_string(a.size()));
}

// Arguments in the reference's buffer-index order (src/ops.h:106-120).
void launch_head_norm_rope(const std::vector<Arg> &a, Dim3 g, cudaStream_t s, bool bf16, const char *k) {
    need_args(a, 12, k);
    const uint32_t heads = val<uint32_t>(a[3], k, 3);
    if (g.y != heads) throw std::runtime_error(std::string(k) + ": grid.y must equal heads");
    const uint32_t tokens = g.x;
    if (bf16) {
        apex_check(apex_head_norm_rope_bf16(ptr<const uint16_t>(a[0], k, 0), ptr<const uint16_t>(a[1], k, 1),
                                            ptr<uint16_t>(a[2], k, 2), tokens, heads, val<uint32_t>(a[4], k, 4),
                                            val<uint32_t>(a[5], k, 5), val<uint32_t>(a[6], k, 6),
                                            val<float>(a[7], k, 7), val<uint32_t>(a[8], k, 8),
                                            val<uint32_t>(a[9], k, 9), val<uint32_t>(a[10], k, 10),
                                            val<float>(a[11], k, 11), s),
                   k);
    } else {
        apex_check(apex_head_norm_rope_f32(ptr<const float>(a[0], k, 0), ptr<const uint16_t>(a[1], k, 1),
                                           ptr<float>(a[2], k, 2), tokens, heads, val<uint32_t>(a[4], k, 4),
                                           val<uint32_t>(a[5], k, 5), val<uint32_t>(a[6], k, 6),
                                           val<float>(a[7], k, 7), val<uint32_t>(a[8], k, 8),
                                           val<uint32_t>(a[9], k, 9), val<uint32_t>(a[10], k, 10),
                                           val<float>(a[11], k, 11), s),
                   k);
    }
}

// docs/B6_3_attention.md:426-430 order: q, K, V, out, q_heads, kv_heads, head_dim, capacity,
// pos0, window [, scale]; grid {tokens, q_heads}.
void launch_attention_f32(const std::vector<Arg> &a, Dim3 g, cudaStream_t s, const char *k) {
    if (a.size() != 10 && a.size() != 11) need_args(a, 10, k);
    const uint32_t q_heads = val<uint32_t>(a[4], k, 4);
    if (g.y != q_heads) throw std::runtime_error(std::string(k) + ": grid.y must equal q_heads");
    const float scale = a.size() == 11 ? val<float>(a[10], k, 10) : 1.0f;
    apex_check(apex_attention_f32_scaled(ptr<const float>(a[0], k, 0), ptr<const float>(a[1], k, 1),
                                         ptr<const float>(a[2], k, 2), ptr<float>(a[3], k, 3), g.x, q_heads,
                                         val<uint32_t>(a[5], k, 5), val<uint32_t>(a[6], k, 6),
                                         val<uint32_t>(a[7], k, 7), val<uint32_t>(a[8], k, 8),
                                         val<uint32_t>(a[9], k, 9), scale, s),
               k);
}

// q_raw, k_new, v_new, q_norm_w, k_norm_w, k_cache, v_cache, seq_lens, out, workspace,
// params, capacity, max_seq_len; grid {batch}.
void launch_decode(const std::vector<Arg> &a, Dim3 g, cudaStream_t s, const char *k) {
    need_args(a, 13, k);
    const apex_attn_params p = val<apex_attn_params>(a[10], k, 10);
    apex_check(apex_attn_decode_bf16(&p, ptr<const uint16_t>(a[0], k, 0), ptr<const uint16_t>(a[1], k, 1),
                                     ptr<const uint16_t>(a[2], k, 2), ptr<const uint16_t>(a[3], k, 3),
                                     ptr<const uint16_t>(a[4], k, 4), ptr<uint16_t>(a[5], k, 5),
                                     ptr<uint16_t>(a[6], k, 6), val<uint32_t>(a[11], k, 11),
                                     ptr<const int32_t>(a[7], k, 7), g.x, val<uint32_t>(a[12], k, 12),
                                     ptr<uint16_t>(a[8], k, 8), ptr<void>(a[9], k, 9), bytes_after(a[9]), s),
               k);
}

// q_raw, k_raw, v_raw, q_norm_w, k_norm_w, k_cache, v_cache, out, workspace, params,
// capacity, pos0; grid {tokens, batch}.
void launch_prefill(const std::vector<Arg> &a, Dim3 g, cudaStream_t s, const char *k) {
    need_args(a, 12, k);
    const apex_attn_params p = val<apex_attn_params>(a[9], k, 9);
    apex_check(apex_attn_prefill_bf16(&p, ptr<const uint16_t>(a[0], k, 0), ptr<const uint16_t>(a[1], k, 1),
                                      ptr<const uint16_t>(a[2], k, 2), ptr<const uint16_t>(a[3], k, 3),
                                      ptr<const uint16_t>(a[4], k, 4), ptr<uint16_t>(a[5], k, 5),
                                      ptr<uint16_t>(a[6], k, 6), val<uint32_t>(a[10], k, 10), g.y, g.x,
                                      val<uint32_t>(a[11], k, 11), ptr<uint16_t>(a[7], k, 7),
                                      ptr<void>(a[8], k, 8), bytes_after(a[8]), s),
               k);
}

// partials, out, num_partials, head_dim; grid {rows}.
void launch_merge(const std::vector<Arg> &a, Dim3 g, cudaStream_t s, const char *k) {
    need_args(a, 4, k);
    apex_check(apex_attn_merge_partials(ptr<const float>(a[0], k, 0), val<uint32_t>(a[2], k, 2), g.x,
                                        val<uint32_t>(a[3], k, 3), ptr<uint16_t>(a[1], k, 1), s),
               k);
}

// src/ops.h:39-44 order: input, weights(+offset), scales(+offset), output, hidden_dim, w_rows;
// grid {row groups of 8, tokens}.
void launch_matmul_nvfp4(const std::vector<Arg> &a, Dim3 g, cudaStream_t s, const char *k) {
    need_args(a, 6, k);
    const uint32_t w_rows = val<uint32_t>(a[5], k, 5);
    if (g.x * 8 < w_rows) throw std::runtime_error(std::string(k) + ": grid.x must cover w_rows in groups of 8");
    apex_check(apex_matmul_nvfp4_f32(ptr<const float>(a[0], k, 0), ptr<const uint32_t>(a[1], k, 1),
                                     ptr<const uint8_t>(a[2], k, 2), ptr<float>(a[3], k, 3),
                                     val<uint32_t>(a[4], k, 4), w_rows, g.y, s),
               k);
}

// src/ops.h:21-26 order: input, weights(+offset), result, hidden_dim, eps; grid {rows}.
void launch_rms_norm(const std::vector<Arg> &a, Dim3 g, cudaStream_t s, const char *k) {
    need_args(a, 5, k);
    apex_check(apex_rms_norm_f32(ptr<const float>(a[0], k, 0), ptr<const uint16_t>(a[1], k, 1),
                                 ptr<float>(a[2], k, 2), g.x, val<uint32_t>(a[3], k, 3), val<float>(a[4], k, 4), s),
               k);
}

const std::map<std::string, Launcher> &launchers() {
    static const std::map<std::string, Launcher> table = {
        {"head_norm_rope_f32", [](auto &a, Dim3 g, cudaStream_t s) { launch_head_norm_rope(a, g, s, false, "head_norm_rope_f32"); }},
        {"head_norm_rope_bf16", [](auto &a, Dim3 g, cudaStream_t s) { launch_head_norm_rope(a, g, s, true, "head_norm_rope_bf16"); }},
        {"attention_f32", [](auto &a, Dim3 g, cudaStream_t s) { launch_attention_f32(a, g, s, "attention_f32"); }},
        {"attention_decode_bf16", [](auto &a, Dim3 g, cudaStream_t s) { launch_decode(a, g, s, "attention_decode_bf16"); }},
        {"attention_prefill_bf16", [](auto &a, Dim3 g, cudaStream_t s) { launch_prefill(a, g, s, "attention_prefill_bf16"); }},
        {"attention_merge_partials", [](auto &a, Dim3 g, cudaStream_t s) { launch_merge(a, g, s, "attention_merge_partials"); }},
        {"matmul_nvfp4", [](auto &a, Dim3 g, cudaStream_t s) { launch_matmul_nvfp4(a, g, s, "matmul_nvfp4"); }},
        {"rms_norm_f32", [](auto &a, Dim3 g, cudaStream_t s) { launch_rms_norm(a, g, s, "rms_norm_f32"); }},
    };
    return table;
}

}  // namespace

// ------------------------------------------------------------------ CudaBackend
CudaBackend::CudaBackend(int device) : device_(device) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= device)
        throw std::runtime_error("CudaBackend: no CUDA device " + std::to_string(device));
    cuda_check(cudaSetDevice(device), "CudaBackend: cudaSetDevice");
    cudaDeviceProp prop{};
    cuda_check(cudaGetDeviceProperties(&prop, device), "CudaBackend: device properties");
    name_ = prop.name;
    cuda_check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "CudaBackend: stream");
}

CudaBackend::~CudaBackend() {
    if (stream_) {
        cudaStreamSynchronize(stream_);
        cudaStreamDestroy(stream_);
    }
}

Buffer *CudaBackend::wrapNoCopy(void *cpu_ptr, size_t bytes) {
    const size_t page = 4096;
    if (reinterpret_cast<uintptr_t>(cpu_ptr) % page || bytes % page)
        throw std::runtime_error("wrapNoCopy: pointer and length must be page multiples");
    cuda_check(cudaSetDevice(device_), "wrapNoCopy: cudaSetDevice");
    cuda_check(cudaHostRegister(cpu_ptr, bytes, cudaHostRegisterMapped | cudaHostRegisterReadOnly),
               "wrapNoCopy: cudaHostRegister");
    void *dev = nullptr;
    cuda_check(cudaHostGetDevicePointer(&dev, cpu_ptr, 0), "wrapNoCopy: cudaHostGetDevicePointer");
    return new Buffer{dev, cpu_ptr, bytes, "", true};
}

Buffer *CudaBackend::allocate(size_t bytes, const char *category) {
    cuda_check(cudaSetDevice(device_), "allocate: cudaSetDevice");
    void *p = nullptr;
    cuda_check(cudaMallocManaged(&p, bytes ? bytes : 1), "allocate: cudaMallocManaged");
    const std::string cat = category && *category ? category : "uncategorized";
    MemoryLedger::get().add(cat, bytes);
    return new Buffer{p, p, bytes, cat, false};
}

void *CudaBackend::contents(Buffer *buffer) { return buffer ? buffer->host : nullptr; }

void CudaBackend::release(Buffer *buffer) {
    if (!buffer) return;
    if (buffer->wrapped) {
        cudaHostUnregister(buffer->host);
    } else {
        MemoryLedger::get().remove(buffer->category, buffer->length);
        cudaFree(buffer->ptr);
    }
    delete buffer;
}

void CudaBackend::run(const char *kernel, std::initializer_list<Arg> args, Dim3 threadgroups,
                      Dim3 threads_per_group) {
    const auto &table = launchers();
    auto it = table.find(kernel ? kernel : "");
    if (it == table.end()) throw std::runtime_error(std::string("CudaBackend: no kernel named ") + (kernel ? kernel : "(null)"));
    if (threads_per_group.total() > 1024) throw std::runtime_error(std::string(kernel) + ": threadgroup too large");
    cuda_check(cudaSetDevice(device_), "run: cudaSetDevice");
    it->second(std::vector<Arg>(args), threadgroups, stream_);
}

void CudaBackend::sync() {
    const auto t0 = std::chrono::steady_clock::now();
    cuda_check(cudaStreamSynchronize(stream_), "sync");
    PhaseTable::get().add("gpu_sync", std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count());
    apex_check(apex_cuda_device_status(stream_), "sync");
}

}  // namespace apex
