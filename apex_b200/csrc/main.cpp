// main.cpp -- command-line tool over CudaBackend, in the style of the reference's CLI
// (src/main.cpp:58-72): one subcommand per action, exit code = failure count.
//
//   apex_cuda_cli device
//   apex_cuda_cli bench-attn prefill <tokens> <window> [steps]
//   apex_cuda_cli bench-attn decode <context> <batch> [steps]
//   apex_cuda_cli manifest <packed_dir>       (the reference's `apex manifest`, src/main.cpp:36-49)
//   apex_cuda_cli load <packed_dir>           (core.bin into HBM with digest checks, timed)
//
// bench-attn runs the bf16 operators of ops.h on synthetic inputs through the Backend
// interface (allocate / run / sync) and prints the phase table and the memory ledger.
#include <chrono>
#include <functional>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "backend/cuda/cuda_backend.h"
#include "loader/model_info.h"
#include "ops.h"

namespace {

uint16_t to_bf16(float f) {
    uint32_t b;
    std::memcpy(&b, &f, 4);
    b += 0x7fffu + ((b >> 16) & 1u);
    return static_cast<uint16_t>(b >> 16);
}

void fill_normal(apex::Backend &backend, apex::Buffer *buf, size_t count, uint32_t seed, float mean = 0.f,
                 float std = 1.f) {
    std::mt19937 rng(seed);
    std::normal_distribution<float> nd(mean, std);
    auto *p = static_cast<uint16_t *>(backend.contents(buf));
    for (size_t i = 0; i < count; ++i) p[i] = to_bf16(nd(rng));
}

int run_device() {
    apex::CudaBackend backend;
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    std::printf("device: %s, %d SMs, ABI %d\n", backend.deviceName(), sms, apex_cuda_abi_version());
    return 0;
}

int run_bench(const std::string &kind, uint32_t a, uint32_t b, int steps) {
    apex::CudaBackend backend;
    std::printf("device: %s\n", backend.deviceName());
    const uint32_t Hq = 16, Hkv = 8, D = 256;
    const apex::AttentionShape s{Hq, Hkv, D, D / 2, kind == "prefill" ? 1e4f : 1e6f,
                                 kind == "prefill" ? b : 0u};
    const apex_attn_params p = apex::attnParams(s, 1.0f / std::sqrt(float(D)), 1e-6f, true, false);
    auto *qw = backend.allocate(D * 2, "weights");
    auto *kw = backend.allocate(D * 2, "weights");
    fill_normal(backend, qw, D, 1, 1.f, 0.1f);
    fill_normal(backend, kw, D, 2, 1.f, 0.1f);
    double work = 0;  // FLOPs (prefill) or bytes (decode) per step
    std::vector<apex::Buffer *> bufs{qw, kw};
    auto alloc = [&](size_t bytes, const char *cat) {
        bufs.push_back(backend.allocate(bytes, cat));
        return bufs.back();
    };
    std::function<void()> step;
    if (kind == "prefill") {
        const uint32_t T = a, window = b;
        auto *q = alloc(size_t(T) * Hq * D * 2, "activations");
        auto *k = alloc(size_t(T) * Hkv * D * 2, "activations");
        auto *v = alloc(size_t(T) * Hkv * D * 2, "activations");
        auto *o = alloc(size_t(T) * Hq * D * 2, "activations");
        apex::KvCacheBf16 cache{alloc(size_t(Hkv) * T * D * 2, "kv_cache"), alloc(size_t(Hkv) * T * D * 2, "kv_cache"), T};
        auto *ws = alloc(apex::prefillWorkspaceBytes(p, 1, T), "scratch");
        fill_normal(backend, q, size_t(T) * Hq * D, 3);
        fill_normal(backend, k, size_t(T) * Hkv * D, 4);
        fill_normal(backend, v, size_t(T) * Hkv * D, 5);
        for (uint32_t t = 0; t < T; ++t) {
            const uint32_t first = (window && t + 1 > window) ? t + 1 - window : 0;
            work += 4.0 * Hq * D * (t - first + 1);
        }
        step = [&, q, k, v, o, ws, cache]() mutable {
            apex::attentionPrefillBf16(backend, p, q, k, v, qw, kw, cache, 1, T, 0, o, ws);
        };
    } else {
        const uint32_t L = a, B = b;
        auto *q = alloc(size_t(B) * Hq * D * 2, "activations");
        auto *k = alloc(size_t(B) * Hkv * D * 2, "activations");
        auto *v = alloc(size_t(B) * Hkv * D * 2, "activations");
        auto *o = alloc(size_t(B) * Hq * D * 2, "activations");
        apex::KvCacheBf16 cache{alloc(size_t(B) * Hkv * L * D * 2, "kv_cache"),
                                alloc(size_t(B) * Hkv * L * D * 2, "kv_cache"), L};
        auto *lens = alloc(size_t(B) * 4, "activations");
        const size_t wsb = apex::decodeWorkspaceBytes(p, B, L);
        auto *ws = alloc(wsb, "scratch");
        std::memset(backend.contents(ws), 0, wsb);
        fill_normal(backend, q, size_t(B) * Hq * D, 3);
        fill_normal(backend, k, size_t(B) * Hkv * D, 4);
        fill_normal(backend, v, size_t(B) * Hkv * D, 5);
        fill_normal(backend, cache.k, size_t(B) * Hkv * L * D, 6);
        fill_normal(backend, cache.v, size_t(B) * Hkv * L * D, 7);
        auto *lp = static_cast<int32_t *>(backend.contents(lens));
        for (uint32_t i = 0; i < B; ++i) lp[i] = static_cast<int32_t>(L);
        work = double(B) * (2.0 * Hkv * L * D * 2 + 2.0 * Hq * D * 2);
        step = [&, q, k, v, o, ws, lens, cache]() mutable {
            apex::attentionDecodeBf16(backend, p, q, k, v, qw, kw, cache, lens, B, L, o, ws);
        };
    }
    for (int i = 0; i < 3; ++i) step();
    backend.sync();
    const auto t0 = std::chrono::steady_clock::now();
    for (int i = 0; i < steps; ++i) step();
    backend.sync();
    const double s_total = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    const double per = s_total / steps;
    if (kind == "prefill")
        std::printf("prefill: %.3f ms/step, %.1f TFLOP/s (wall clock incl. launch)\n", per * 1e3, work / per / 1e12);
    else
        std::printf("decode: %.3f ms/step, %.1f GB/s (wall clock incl. launch)\n", per * 1e3, work / per / 1e9);
    apex::PhaseTable::get().print(stdout);
    apex::MemoryLedger::get().print(stdout);
    for (auto *buf : bufs) backend.release(buf);
    return 0;
}

// Prints the packed model's metadata without reading weight files.
int run_manifest(const std::string &dir) {
    const apex::ModelInfo m = apex::ModelInfo::load(dir);
    std::printf("core tensors: %zu\n", m.core.size());
    std::printf("core bytes: %llu\n", static_cast<unsigned long long>(m.core_size));
    std::printf("expert stride: %llu\n", static_cast<unsigned long long>(m.expert_slot_size));
    std::printf("layer files: %zu\n", m.layers.size());
    if (m.core.count("norm.weight"))
        std::printf("norm.weight offset: %llu\n", static_cast<unsigned long long>(m.getTensor("norm.weight").offset));
    return 0;
}

// Copies core.bin into one device allocation (checking every tensor's digest on the way) and one
// expert slot of layer 0, and prints the rates.
int run_load(const std::string &dir) {
    const apex::ModelInfo m = apex::ModelInfo::load(dir);
    void *core = nullptr;
    if (cudaMalloc(&core, m.core_size) != cudaSuccess) throw std::runtime_error("cudaMalloc of core.bin failed");
    const apex::LoadStats s = apex::uploadCore(m, core, m.core_size, true, nullptr);
    std::printf("core.bin: %.3f GB in %.3f s (%.2f GB/s)%s%s\n", s.bytes / 1e9, s.seconds, s.bytes / 1e9 / s.seconds,
                s.mismatch.empty() ? "" : ", digest mismatch: ", s.mismatch.c_str());
    int failures = s.mismatch.empty() ? 0 : 1;
    if (!m.layers.empty()) {
        void *slot = nullptr;
        if (cudaMalloc(&slot, m.expert_slot_size) != cudaSuccess) throw std::runtime_error("cudaMalloc of a slot failed");
        const apex::LoadStats e = apex::loadExpert(m, m.layers.front().layer, 0, slot, m.expert_slot_size, true, nullptr);
        std::printf("expert slot: %llu bytes in %.3f ms%s%s\n", static_cast<unsigned long long>(e.bytes), e.seconds * 1e3,
                    e.mismatch.empty() ? "" : ", digest mismatch: ", e.mismatch.c_str());
        failures += e.mismatch.empty() ? 0 : 1;
        cudaFree(slot);
    }
    cudaFree(core);
    return failures;
}

}  // namespace

int main(int argc, char **argv) {
    try {
        if (argc == 2 && std::strcmp(argv[1], "device") == 0) return run_device();
        if (argc == 3 && std::strcmp(argv[1], "manifest") == 0) return run_manifest(argv[2]);
        if (argc == 3 && std::strcmp(argv[1], "load") == 0) return run_load(argv[2]);
        if (argc >= 5 && std::strcmp(argv[1], "bench-attn") == 0) {
            const int steps = argc >= 6 ? std::atoi(argv[5]) : 20;
            return run_bench(argv[2], static_cast<uint32_t>(std::atoi(argv[3])),
                             static_cast<uint32_t>(std::atoi(argv[4])), steps);
        }
    } catch (const std::exception &e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 1;
    }
    std::fprintf(stderr,
                 "usage: apex_cuda_cli device | apex_cuda_cli bench-attn prefill <tokens> <window> [steps] | "
                 "apex_cuda_cli bench-attn decode <context> <batch> [steps] | apex_cuda_cli manifest <packed_dir> | "
                 "apex_cuda_cli load <packed_dir>\n");
    return 2;
}
