// cuda_backend.h -- apex::Backend on a B200: the sibling of the reference's MetalBackend
// (src/backend/metal_backend.h:18-55).  Kernels are looked up by the reference's names and
// launched through the C ABI of include/apex_cuda.h on one CUDA stream.
//
//   allocate    cudaMallocManaged: one pointer valid on host and device, like Metal shared
//               storage (contents() is that pointer; valid after sync()).
//   wrapNoCopy  cudaHostRegister(mapped, read-only) of the caller's pages (the reference
//               wraps mmap'd core.bin the same way, without a copy).
//   run         looks the name up in a launcher table, unpacks the Args in the reference's
//               buffer-index order and enqueues on the backend's stream.  Throws
//               std::runtime_error for an unknown name, a wrong argument count or a failed
//               launch (the reference throws for a missing function or pipeline).
//   sync        cudaStreamSynchronize, timed as "gpu_sync", then a device-status check.
#pragma once

#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <string>

#include "../backend.h"

#if defined(__GNUC__)
#define APEX_CXX_API __attribute__((visibility("default")))
#else
#define APEX_CXX_API
#endif

namespace apex {

struct Buffer {
    void *ptr = nullptr;        // device-accessible pointer (managed, or mapped host)
    void *host = nullptr;       // host pointer (same as ptr for managed memory)
    size_t length = 0;
    std::string category;       // ledger category; empty for wrapped buffers
    bool wrapped = false;
};

// Bytes per category with peak (the reference's MemoryTracker, src/profiling/memory.h:36-94,
// without the macOS task_info comparison).
class APEX_CXX_API MemoryLedger {
  public:
    static MemoryLedger &get();
    void add(const std::string &category, size_t bytes);
    void remove(const std::string &category, size_t bytes);
    size_t current() const;
    size_t peak() const;
    void print(FILE *out) const;

  private:
    mutable std::mutex mu_;
    std::map<std::string, size_t> bytes_;
    size_t current_ = 0, peak_ = 0;
};

// Wall-clock phase table (the reference's Profile/Timer, src/profiling/timer.h:19-80).
class APEX_CXX_API PhaseTable {
  public:
    static PhaseTable &get();
    void add(const std::string &phase, double ms);
    void print(FILE *out) const;

  private:
    struct Stats {
        double total_ms = 0, max_ms = 0;
        long calls = 0;
    };
    mutable std::mutex mu_;
    std::map<std::string, Stats> stats_;
};

class APEX_CXX_API CudaBackend : public Backend {
  public:
    explicit CudaBackend(int device = 0);
    ~CudaBackend() override;
    CudaBackend(const CudaBackend &) = delete;
    CudaBackend &operator=(const CudaBackend &) = delete;

    Buffer *wrapNoCopy(void *cpu_ptr, size_t bytes) override;
    Buffer *allocate(size_t bytes, const char *category) override;
    void *contents(Buffer *buffer) override;
    void release(Buffer *buffer) override;
    void run(const char *kernel, std::initializer_list<Arg> args, Dim3 threadgroups,
             Dim3 threads_per_group) override;
    void sync() override;

    const char *deviceName() const { return name_.c_str(); }
    cudaStream_t stream() const { return stream_; }

  private:
    int device_ = 0;
    cudaStream_t stream_ = nullptr;
    std::string name_;
};

}  // namespace apex
