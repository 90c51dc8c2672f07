// Host-side helpers shared by the C-ABI translation units (capi.cu, vae_capi.cu): the context object,
// the thread's last error message, CUDA status conversion, device guards and the arena allocator.
#pragma once
#include "ernie_cuda.h"
#include <cuda_runtime.h>
#include <string>
#include <utility>
#include <vector>

struct ernie_cuda_context
{
    int device = 0;
    cudaStream_t stream = nullptr;
    int num_sms = 148;
    int *error_flag = nullptr; // device-side protocol status of the bounded waits
    int query_rows = 128;
    cudaEvent_t events[16] = {};
};

namespace ernie_b200
{
namespace capi
{
inline thread_local std::string g_last_error;

inline int fail(int code, const std::string &message)
{
    g_last_error = message;
    return code;
}

inline int from_cuda(cudaError_t e, const char *action)
{
    if (e == cudaSuccess) return ERNIE_CUDA_OK;
    const int code = e == cudaErrorMemoryAllocation ? ERNIE_CUDA_OUT_OF_MEMORY : ERNIE_CUDA_ERROR;
    return fail(code, std::string(action) + ": " + cudaGetErrorString(e));
}

inline int from_launch(int e, const char *action) { return from_cuda(static_cast<cudaError_t>(e), action); }

#define ERNIE_TRY(expr)                                                                                             \
    do                                                                                                              \
    {                                                                                                               \
        const int _rc = (expr);                                                                                     \
        if (_rc != ERNIE_CUDA_OK) return _rc;                                                                       \
    } while (0)
#define ERNIE_LAUNCH(expr, what) ERNIE_TRY(from_launch((expr), what))
#define ERNIE_CUDA(expr, what) ERNIE_TRY(from_cuda((expr), what))

inline size_t align256(size_t bytes) { return (bytes + 255) & ~size_t(255); }

// Carves one device allocation into 256-byte aligned sub-buffers.
struct Arena
{
    std::vector<std::pair<void **, size_t>> parts;
    void *base = nullptr;
    template <class T> void add(T **ptr, size_t count) { parts.push_back({reinterpret_cast<void **>(ptr), align256(count * sizeof(T))}); }
    size_t bytes() const
    {
        size_t total = 0;
        for (const auto &p : parts) total += p.second;
        return total;
    }
    cudaError_t allocate()
    {
        const cudaError_t e = cudaMalloc(&base, bytes());
        if (e != cudaSuccess) return e;
        char *cursor = static_cast<char *>(base);
        for (auto &p : parts)
        {
            *p.first = cursor;
            cursor += p.second;
        }
        return cudaSuccess;
    }
};

struct DeviceGuard
{
    int previous = -1;
    explicit DeviceGuard(int device)
    {
        cudaGetDevice(&previous);
        if (previous != device) cudaSetDevice(device);
    }
    ~DeviceGuard()
    {
        int now = -1;
        cudaGetDevice(&now);
        if (previous >= 0 && now != previous) cudaSetDevice(previous);
    }
};

} // namespace capi
} // namespace ernie_b200
