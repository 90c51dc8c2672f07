// Non-finite latent check that allocates nothing (ernie_cuda_finite_latent_noalloc).
//
// ernie_cuda_finite_latent allocates a 4-byte device status word on every call. Some embedding
// applications reserve all of their device memory at start-up and then forbid device allocation (a
// fixed memory budget shared with other models, or a rule against cudaMalloc's implicit
// synchronisation in a serving loop); they call this variant, which keeps its scratch in a fixed
// device array instead.
//
// Scratch: one status word per latent channel (128 x 4 bytes = 512 bytes), a file-scope
// __device__ array present on every GPU that loads the library until the process exits. Host code
// never names the array as a device address: every call, with the context's device current, looks
// the address up with cudaGetSymbolAddress (a lookup, no allocation, once the library's device code
// is loaded on that device; the first call on a device may load it). Every call shares the array,
// clears it before use and leaves the last call's per-channel status in it; calls that overlap on
// the GPU (two streams, two host threads on one device) race on it. The call waits for the
// context's stream before it returns.
#include "ernie_cuda.h"
#include <cuda_runtime.h>
#include <string>

namespace
{
constexpr int kStatusWords = 128; // latent channels, the maximum this scratch can hold
__device__ __align__(256) int g_channel_status[kStatusWords];

// One CTA per (channel, slice of the H*W plane); a non-finite value sets that channel's word.
__global__ void finite_channels_kernel(const float *latent, int plane, int *status)
{
    const int channel = blockIdx.y;
    const float *values = latent + static_cast<size_t>(channel) * plane;
    bool ok = true;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < plane; i += gridDim.x * blockDim.x)
        ok = ok && isfinite(values[i]);
    if (__any_sync(0xffffffffu, !ok) && (threadIdx.x % 32) == 0) atomicOr(status + channel, 1);
}

// The device address of g_channel_status on the current device. Looked up on every call rather than
// cached, so a device reset (which reloads the module at a new address) cannot leave a stale pointer.
cudaError_t scratch_address(int **address)
{
    return cudaGetSymbolAddress(reinterpret_cast<void **>(address), g_channel_status);
}
} // namespace

// Defined in capi.cu: records the calling thread's error message and returns `code`.
int ernie_cuda_record_error(int code, const char *message);
int ernie_cuda_context_device_and_stream(ernie_cuda_context *ctx, int *device, cudaStream_t *stream);

extern "C" int ernie_cuda_finite_latent_noalloc(ernie_cuda_context *ctx, const float *latent, int width, int height,
                                                int *finite)
{
    if (!ctx || !latent || !finite) return ernie_cuda_record_error(ERNIE_CUDA_ERROR, "null argument");
    if (width < 1 || height < 1 || width > 256 || height > 256)
        return ernie_cuda_record_error(ERNIE_CUDA_ERROR,
                                       "Expected [128,H,W] latent with 1 <= H,W <= 256 (the static status array "
                                       "holds 128 channels)");
    int device = 0;
    cudaStream_t stream = nullptr;
    if (ernie_cuda_context_device_and_stream(ctx, &device, &stream) != ERNIE_CUDA_OK)
        return ernie_cuda_record_error(ERNIE_CUDA_ERROR, "invalid context");
    int previous = -1;
    cudaGetDevice(&previous);
    if (previous != device) cudaSetDevice(device);
    int *status = nullptr;
    cudaError_t e = scratch_address(&status);
    if (e == cudaSuccess) e = cudaMemsetAsync(status, 0, kStatusWords * sizeof(int), stream);
    if (e == cudaSuccess)
    {
        const int plane = width * height;
        int slices = (plane + 255) / 256;
        if (slices > 8) slices = 8;
        finite_channels_kernel<<<dim3(slices, kStatusWords), 256, 0, stream>>>(latent, plane, status);
        e = cudaGetLastError();
    }
    int host[kStatusWords];
    if (e == cudaSuccess) e = cudaMemcpyAsync(host, status, sizeof(host), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (previous >= 0 && previous != device) cudaSetDevice(previous);
    if (e != cudaSuccess)
        return ernie_cuda_record_error(e == cudaErrorMemoryAllocation ? ERNIE_CUDA_OUT_OF_MEMORY : ERNIE_CUDA_ERROR,
                                       (std::string("finite_latent_noalloc: ") + cudaGetErrorString(e)).c_str());
    int bad = 0;
    for (int c = 0; c < kStatusWords; ++c) bad |= host[c];
    *finite = bad ? 0 : 1;
    return ERNIE_CUDA_OK;
}
