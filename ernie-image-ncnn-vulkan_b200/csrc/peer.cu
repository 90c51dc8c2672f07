// Barrier of a sequence-parallel group over NVLink peer memory (one GPU per process, buffers shared
// through CUDA IPC). Used twice per DiT block: after the QKV GEMM has stored every GPU's heads into
// their owners' memory, and after the attention has stored every token row back into its owner's
// memory. One warp per GPU; arrival stores are release at system scope, the waits acquire at system
// scope and give up after a fixed time (status 21 in the context's error flag). Also the store of one
// buffer into every member's memory (the gather of latent slices and step flags).
#include "kernels.h"
#include "peer_sync.cuh"
#include <algorithm>
#include <cstdint>

namespace ernie_b200
{
namespace
{
constexpr int kErrPeerBarrierTimeout = 21;

__device__ __forceinline__ unsigned long long global_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void store_release_sys(unsigned *p, unsigned v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned load_acquire_sys(const unsigned *p)
{
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void peer_barrier_kernel(PeerBarrier b)
{
    const int lane = threadIdx.x;
    unsigned e = 0;
    if (lane == 0)
    {
        e = *b.epoch + 1;
        *b.epoch = e;
    }
    e = __shfl_sync(0xffffffffu, e, 0);
    // every store of the kernels before this one (stream order) is ordered before the arrival
    __threadfence_system();
    if (lane < b.world)
    {
        unsigned *member = nullptr;
#pragma unroll
        for (int d = 0; d < kMaxDest; ++d)
            if (d == lane) member = b.peer_slots[d];
        store_release_sys(member + b.rank, e);
    }
    bool ok = true;
    if (lane < b.world)
    {
        const unsigned long long start = global_ns();
        // wrap-safe "arrival < e"
        while (static_cast<int>(load_acquire_sys(b.slots + lane) - e) < 0)
        {
            if (global_ns() - start > static_cast<unsigned long long>(b.timeout_ns))
            {
                ok = false;
                break;
            }
            __nanosleep(100);
        }
    }
    if (!ok && b.error_flag) atomicExch(b.error_flag, kErrPeerBarrierTimeout);
    __threadfence_system();
}
} // namespace

int launch_peer_barrier(const PeerBarrier &barrier, cudaStream_t stream)
{
    if (!barrier.slots || !barrier.epoch || barrier.world < 2 || barrier.world > kMaxDest || barrier.rank < 0 ||
        barrier.rank >= barrier.world || barrier.timeout_ns <= 0)
        return cudaErrorInvalidValue;
    for (int d = 0; d < barrier.world; ++d)
        if (!barrier.peer_slots[d]) return cudaErrorInvalidValue;
    peer_barrier_kernel<<<1, 32, 0, stream>>>(barrier);
    return cudaGetLastError();
}

namespace
{
__global__ void peer_signal_kernel(PeerSignal s) { peer_signal_warp(s); }
} // namespace

int launch_peer_signal(const PeerSignal &signal, cudaStream_t stream)
{
    if (!signal.counter || !signal.epoch || signal.members < 1 || signal.members > kMaxDest) return cudaErrorInvalidValue;
    for (int d = 0; d < signal.members; ++d)
        if (!signal.peer_slot[d]) return cudaErrorInvalidValue;
    PeerSignal one = signal;
    one.warps = 1;
    peer_signal_kernel<<<1, 32, 0, stream>>>(one);
    return cudaGetLastError();
}

namespace
{
// dst[d][i] = src[i] for every member d: 16-byte stores when every address allows, else 4-byte ones.
template <class V> __global__ void peer_put_kernel(const V *__restrict__ src, long long count, PeerPut put)
{
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count; i += stride)
    {
        const V value = src[i];
#pragma unroll
        for (int d = 0; d < kMaxDest; ++d)
            if (d < put.members) static_cast<V *>(put.dst[d])[i] = value;
    }
}
} // namespace

int launch_peer_put(const void *src, size_t bytes, const PeerPut &put, cudaStream_t stream)
{
    if (bytes == 0) return cudaSuccess;
    if (!src || bytes % 4 || put.members < 1 || put.members > kMaxDest) return cudaErrorInvalidValue;
    bool wide = bytes % 16 == 0 && reinterpret_cast<uintptr_t>(src) % 16 == 0;
    for (int d = 0; d < put.members; ++d)
    {
        if (!put.dst[d] || reinterpret_cast<uintptr_t>(put.dst[d]) % 4) return cudaErrorInvalidValue;
        wide = wide && reinterpret_cast<uintptr_t>(put.dst[d]) % 16 == 0;
    }
    const long long count = static_cast<long long>(bytes / (wide ? 16 : 4));
    const int blocks = static_cast<int>(std::min<long long>((count + 255) / 256, 1184));
    if (wide)
        peer_put_kernel<uint4><<<blocks, 256, 0, stream>>>(static_cast<const uint4 *>(src), count, put);
    else
        peer_put_kernel<unsigned><<<blocks, 256, 0, stream>>>(static_cast<const unsigned *>(src), count, put);
    return cudaGetLastError();
}
} // namespace ernie_b200
