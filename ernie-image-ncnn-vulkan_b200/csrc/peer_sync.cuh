// Device side of the sequence-parallel completion flags (PeerSignal / PeerWait in kernels.h).
//
// Producer: every arriving warp makes its stores (peer memory included) visible at system scope, then
// counts itself in this GPU's counter; the warp that completes the count publishes epoch + 1 into its
// slot of every member with a system-scope release store and resets the counter for the next launch
// (which is stream-ordered after this one). Consumer: one thread per loading role polls this GPU's
// slots with system-scope acquire loads until each reaches this GPU's own epoch of the producer (whose
// own launch, earlier on this stream, has already counted it), bounded by %globaltimer; then a proxy
// fence orders the peers' generic-proxy stores before the bulk-tensor (async proxy) loads that follow.
// After a failed wait (status 21 in the error flag) later waits return at once, so a lost member costs
// one timeout, not one per wait.
#pragma once
#include "kernels.h"

namespace ernie_b200
{
constexpr int kErrPeerWaitTimeout = 21;

__device__ __forceinline__ unsigned long long sync_global_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void sync_store_release_sys(unsigned *p, unsigned v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned sync_load_acquire_sys(const unsigned *p)
{
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Called by every lane of each arriving warp, after the warp's last store.
__device__ __forceinline__ void peer_signal_warp(const PeerSignal &s)
{
    if (!s.counter) return;
    __threadfence_system();
    __syncwarp();
    if ((threadIdx.x & 31) != 0) return;
    const unsigned done = atomicAdd(s.counter, 1u) + 1u;
    if (done != static_cast<unsigned>(s.warps)) return;
    __threadfence_system();
    const unsigned e = *reinterpret_cast<volatile unsigned *>(s.epoch) + 1u;
    *reinterpret_cast<volatile unsigned *>(s.epoch) = e;
    atomicExch(s.counter, 0u);
#pragma unroll
    for (int p = 0; p < kMaxDest; ++p)
        if (p < s.members) sync_store_release_sys(s.peer_slot[p], e);
}

// Called by one thread before its first bulk load. Returns false after a timeout (or an earlier one).
__device__ __forceinline__ bool peer_wait_all(const PeerWait &w)
{
    if (!w.slots) return true;
    if (w.error_flag && *reinterpret_cast<volatile int *>(w.error_flag) != 0) return false;
    const unsigned e = *reinterpret_cast<const volatile unsigned *>(w.epoch);
    const unsigned long long start = sync_global_ns();
    for (int p = 0; p < w.members; ++p)
        while (static_cast<int>(sync_load_acquire_sys(w.slots + p) - e) < 0) // wrap-safe "slot < e"
        {
            if (sync_global_ns() - start > static_cast<unsigned long long>(w.timeout_ns))
            {
                if (w.error_flag) atomicExch(w.error_flag, kErrPeerWaitTimeout);
                return false;
            }
            __nanosleep(64);
        }
    asm volatile("fence.proxy.async.global;" ::: "memory");
    return true;
}
} // namespace ernie_b200
