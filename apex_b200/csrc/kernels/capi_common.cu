// capi_common.cu -- error reporting, device status word, SM count and tensor-map encoding
// shared by every C-ABI entry point.
#include <cmath>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include <cstring>

#include "internal.h"

namespace apex {

// One status word per device, written by kernels whose bounded waits give up (they receive
// its address) and read and cleared by apex_cuda_device_status.
static __device__ unsigned int g_device_status = 0;

namespace {
thread_local std::string t_last_error;

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}
}  // namespace

int fail(int code, const std::string &msg) {
    t_last_error = msg;
    return code;
}

int check_cuda(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return APEX_OK;
    return fail(APEX_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int ok() {
    t_last_error.clear();
    return APEX_OK;
}

int sm_count() {
    static std::mutex mu;
    static std::vector<int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
    if (cache[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n > 0 ? n : 148;
    }
    return cache[dev];
}

void rope_table(float *inv_freq, uint32_t pairs, uint32_t head_dim, float base) {
    for (uint32_t i = 0; i < pairs; ++i) {
        const float e = -2.0f * static_cast<float>(i) / static_cast<float>(head_dim);
        inv_freq[i] = static_cast<float>(std::pow(static_cast<double>(base), static_cast<double>(e)));
    }
}

unsigned *device_status_ptr() {
    static std::mutex mu;
    static std::vector<unsigned *> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if ((int)cache.size() <= dev) cache.resize(dev + 1, nullptr);
    if (!cache[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
        cache[dev] = static_cast<unsigned *>(p);
    }
    return cache[dev];
}

int make_tensor_map_bf16_3d(CUtensorMap *map, const void *base, uint64_t d0, uint64_t d1,
                            uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes,
                            uint32_t box0, uint32_t box1) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(APEX_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[3] = {d0, d1, d2};
    const cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
    const cuuint32_t box[3] = {box0, box1, 1};
    const cuuint32_t estride[3] = {1, 1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims,
                          strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(APEX_ERR_INVALID_ARGUMENT,
                    "cuTensorMapEncodeTiled rejected the tensor (error " + std::to_string((int)r) +
                        "): base must be 16-byte aligned and strides multiples of 16 bytes");
    return APEX_OK;
}

int make_tensor_map_u8_2d(CUtensorMap *map, const void *base, uint64_t d0, uint64_t d1, uint64_t stride1_bytes,
                          uint32_t box0, uint32_t box1) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(APEX_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[2] = {d0, d1};
    const cuuint64_t strides[1] = {stride1_bytes};
    const cuuint32_t box[2] = {box0, box1};
    const cuuint32_t estride[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estride,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(APEX_ERR_INVALID_ARGUMENT,
                    "cuTensorMapEncodeTiled rejected the tensor (error " + std::to_string((int)r) +
                        "): base must be 16-byte aligned and strides multiples of 16 bytes");
    return APEX_OK;
}

int make_tensor_map_bf16_3d_box(CUtensorMap *map, const void *base, const uint64_t (&dims)[3],
                                const uint64_t (&strides_bytes)[2], const uint32_t (&box)[3]) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(APEX_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
    const cuuint64_t st[2] = {strides_bytes[0], strides_bytes[1]};
    const cuuint32_t bx[3] = {box[0], box[1], box[2]};
    const cuuint32_t estride[3] = {1, 1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), d, st, bx, estride,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(APEX_ERR_INVALID_ARGUMENT,
                    "cuTensorMapEncodeTiled rejected the tensor (error " + std::to_string((int)r) +
                        "): base must be 16-byte aligned and strides multiples of 16 bytes");
    return APEX_OK;
}

int make_tensor_map_bf16_4d(CUtensorMap *map, const void *base, const uint64_t (&dims)[4],
                            const uint64_t (&strides_bytes)[3], const uint32_t (&box)[4], bool swizzle128) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(APEX_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
    const cuuint64_t st[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
    const cuuint32_t bx[4] = {box[0], box[1], box[2], box[3]};
    const cuuint32_t estride[4] = {1, 1, 1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void *>(base), d, st, bx, estride,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                          CU_TENSOR_MAP_L2_PROMOTION_NONE,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(APEX_ERR_INVALID_ARGUMENT,
                    "cuTensorMapEncodeTiled rejected the tensor (error " + std::to_string((int)r) +
                        "): base must be 16-byte aligned and strides multiples of 16 bytes");
    return APEX_OK;
}

}  // namespace apex

extern "C" {

const char *apex_cuda_last_error(void) { return apex::t_last_error.c_str(); }

int apex_cuda_abi_version(void) { return 103; }

int apex_cuda_device_status(void *stream) {
    unsigned int host = 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int rc = apex::check_cuda(
        cudaMemcpyFromSymbolAsync(&host, apex::g_device_status, sizeof(host), 0,
                                  cudaMemcpyDeviceToHost, s),
        "read device status");
    if (rc) return rc;
    rc = apex::check_cuda(cudaStreamSynchronize(s), "synchronize");
    if (rc) return rc;
    if (host) {
        const unsigned int zero = 0;
        rc = apex::check_cuda(cudaMemcpyToSymbolAsync(apex::g_device_status, &zero, sizeof(zero), 0,
                                                      cudaMemcpyHostToDevice, s),
                              "clear device status");
        if (rc) return rc;
        rc = apex::check_cuda(cudaStreamSynchronize(s), "synchronize");
        if (rc) return rc;
        if (host & apex::kStatusTimeout)
            return apex::fail(APEX_ERR_DEVICE_TIMEOUT, "a kernel's bounded wait gave up");
        return apex::fail(APEX_ERR_INVALID_ARGUMENT,
                          "a kernel skipped a sequence whose length exceeded max_seq_len or the cache");
    }
    return apex::ok();
}

int apex_device_alloc(size_t bytes, void **ptr) {
    if (!ptr || bytes == 0) return apex::fail(APEX_ERR_INVALID_ARGUMENT, "apex_device_alloc: null pointer or size 0");
    *ptr = nullptr;
    int rc = apex::check_cuda(cudaMalloc(ptr, bytes), "apex_device_alloc");
    if (rc) return rc;
    rc = apex::check_cuda(cudaMemset(*ptr, 0, bytes), "apex_device_alloc: zero");
    if (rc) {
        cudaFree(*ptr);
        *ptr = nullptr;
        return rc;
    }
    return apex::ok();
}

int apex_device_free(void *ptr) {
    if (!ptr) return apex::ok();
    const int rc = apex::check_cuda(cudaFree(ptr), "apex_device_free");
    return rc ? rc : apex::ok();
}

int apex_ipc_get_handle(const void *ptr, void *handle64) {
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
    if (!ptr || !handle64) return apex::fail(APEX_ERR_INVALID_ARGUMENT, "apex_ipc_get_handle: null pointer");
    cudaIpcMemHandle_t h;
    const int rc = apex::check_cuda(cudaIpcGetMemHandle(&h, const_cast<void *>(ptr)), "apex_ipc_get_handle");
    if (rc) return rc;
    memcpy(handle64, &h, sizeof(h));
    return apex::ok();
}

int apex_ipc_open_handle(const void *handle64, void **ptr) {
    if (!handle64 || !ptr) return apex::fail(APEX_ERR_INVALID_ARGUMENT, "apex_ipc_open_handle: null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle64, sizeof(h));
    *ptr = nullptr;
    const int rc = apex::check_cuda(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess),
                                    "apex_ipc_open_handle");
    return rc ? rc : apex::ok();
}

int apex_ipc_close_handle(void *ptr) {
    if (!ptr) return apex::ok();
    const int rc = apex::check_cuda(cudaIpcCloseMemHandle(ptr), "apex_ipc_close_handle");
    return rc ? rc : apex::ok();
}

}  // extern "C"
