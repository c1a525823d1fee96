// backend.h -- the engine's GPU interface, identical in shape to the reference's
// src/backend/backend.h:12-63 so that a CUDA backend drops in beside its Metal one: the same
// Buffer / Arg / Dim3 / Backend names, member functions and argument meanings.
//
// A kernel launch is queued by name with ordered arguments, each either a (buffer, byte
// offset) pair or a host value copied at run() time; sync() submits and waits.
#pragma once

#include <cstddef>
#include <cstdint>
#include <initializer_list>

namespace apex {

struct Buffer;  // defined per backend

// One kernel argument: a device buffer plus byte offset, or host bytes copied at run() time.
struct Arg {
    Buffer *buffer = nullptr;
    size_t offset = 0;
    const void *bytes = nullptr;
    size_t size = 0;

    static Arg buf(Buffer *b, size_t offset = 0) { return {b, offset, nullptr, 0}; }
    template <class T>
    static Arg val(const T &v) {
        return {nullptr, 0, &v, sizeof(T)};
    }
};

// Grid (in thread groups) or thread-group shape.
struct Dim3 {
    uint32_t x = 1, y = 1, z = 1;
    Dim3(uint32_t x_, uint32_t y_ = 1, uint32_t z_ = 1) : x(x_), y(y_), z(z_) {}
    uint32_t total() const { return x * y * z; }
};

class Backend {
  public:
    virtual ~Backend() = default;
    // Lets the GPU read host memory without a copy (the mmap'd weights).
    virtual Buffer *wrapNoCopy(void *cpu_ptr, size_t bytes) = 0;
    // Fresh memory visible to both CPU and GPU, recorded under `category`.
    virtual Buffer *allocate(size_t bytes, const char *category) = 0;
    // CPU pointer to the buffer's bytes (valid after sync()).
    virtual void *contents(Buffer *buffer) = 0;
    // Frees a buffer and updates the memory ledger.
    virtual void release(Buffer *buffer) = 0;
    // Queues one launch of the named kernel.
    virtual void run(const char *kernel, std::initializer_list<Arg> args, Dim3 threadgroups,
                     Dim3 threads_per_group) = 0;
    // Submits queued launches and waits for completion.
    virtual void sync() = 0;
};

}  // namespace apex
