// HBM-bound kernels of the hot path: row statistics + adaLN modulation (the A operand of each
// GEMM), head GEMVs, latent transpose, Euler / finite / VAE unpack, and the stand-alone ERNIE
// layer operators (RMSNorm/LayerNorm, erf-GELU, FP32 residual add). Every kernel reads and writes
// each element once with 16-byte vector accesses where the layout allows.
#include "kernels.h"
#include "ernie_synth.h"
#include "ptx.cuh"

namespace ernie_b200
{
namespace
{
constexpr int kRowThreads = 256;
// Threads per row of the 4096-wide RMSNorm + modulate (the DiT's two norms per block).
#ifndef ERNIE_NORM_THREADS
#define ERNIE_NORM_THREADS 256
#endif
constexpr int kNormThreads = ERNIE_NORM_THREADS;
// Rows per CTA of that norm (1: the one-row kernel; 2 or 4: rms_rows_kernel), a launch-shape knob. Two
// rows per CTA measured 0.0187-0.0188 ms per C2 launch against 0.0210-0.0214 for one (0.024-0.025 against
// 0.027 inside the step); four were slower (0.022).
#ifndef ERNIE_NORM_ROWS
#define ERNIE_NORM_ROWS 2
#endif
constexpr int kNormRows = ERNIE_NORM_ROWS;
static_assert(kNormThreads >= 64 && kNormThreads <= 1024 && 1024 % kNormThreads == 0, "norm threads");

__device__ __forceinline__ float block_sum(float value, float *scratch)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) value += __shfl_xor_sync(0xffffffffu, value, o);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    __syncthreads();
    if (lane == 0) scratch[warp] = value;
    __syncthreads();
    float total = 0.f;
    const int warps = blockDim.x / 32;
    for (int w = 0; w < warps; ++w) total += scratch[w];
    return total;
}

__device__ __forceinline__ void split3(float x, __nv_bfloat16 &hi, __nv_bfloat16 &mid, __nv_bfloat16 &lo)
{
    hi = __float2bfloat16_rn(x);
    const float r1 = x - __bfloat162float(hi);
    mid = __float2bfloat16_rn(r1);
    lo = __float2bfloat16_rn(r1 - __bfloat162float(mid));
}

// One CTA per row of `width` = 4 * VEC * THREADS floats. RMSNorm: x * (mean(x^2) + eps)^(-1/2) * gamma
// (block.ncnn.param rmsn_8 / rmsn_11); LayerNorm: (x - mean) / sqrt(var + eps) (output head ln_1).
// Then y * (1 + scale) + shift (add_0/mul_1/add_2, add_17/mul_18/add_19), stored as BF16 or split-3.
template <int VEC, bool CENTERED, int THREADS = kRowThreads>
__global__ void __launch_bounds__(THREADS) norm_modulate_kernel(const float *__restrict__ x, const float *gamma,
                                                                     const float *scale, const float *shift,
                                                                     float eps, __nv_bfloat16 *out, int split3_out)
{
    constexpr int width = 4 * VEC * THREADS;
    __shared__ float scratch[32];
    const size_t row = blockIdx.x;
    const float4 *xr = reinterpret_cast<const float4 *>(x + row * width);
    float4 v[VEC];
#pragma unroll
    for (int i = 0; i < VEC; ++i) v[i] = xr[threadIdx.x + i * THREADS];
    float mean = 0.f;
    if (CENTERED)
    {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < VEC; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
        mean = block_sum(s, scratch) / float(width);
#pragma unroll
        for (int i = 0; i < VEC; ++i)
        {
            v[i].x -= mean;
            v[i].y -= mean;
            v[i].z -= mean;
            v[i].w -= mean;
        }
    }
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) sq += (v[i].x * v[i].x + v[i].y * v[i].y) + (v[i].z * v[i].z + v[i].w * v[i].w);
    const float inverse = 1.f / sqrtf(block_sum(sq, scratch) / float(width) + eps);
#pragma unroll
    for (int i = 0; i < VEC; ++i)
    {
        const int col = (threadIdx.x + i * THREADS) * 4;
        float y[4] = {v[i].x * inverse, v[i].y * inverse, v[i].z * inverse, v[i].w * inverse};
        if (!CENTERED)
        {
            const float4 g = __ldg(reinterpret_cast<const float4 *>(gamma + col));
            y[0] *= g.x;
            y[1] *= g.y;
            y[2] *= g.z;
            y[3] *= g.w;
        }
        if (scale)
        {
            const float4 sc = __ldg(reinterpret_cast<const float4 *>(scale + col));
            const float4 sh = __ldg(reinterpret_cast<const float4 *>(shift + col));
            y[0] = y[0] * (1.f + sc.x) + sh.x;
            y[1] = y[1] * (1.f + sc.y) + sh.y;
            y[2] = y[2] * (1.f + sc.z) + sh.z;
            y[3] = y[3] * (1.f + sc.w) + sh.w;
        }
        if (!split3_out)
        {
            __nv_bfloat162 *dst = reinterpret_cast<__nv_bfloat162 *>(out + row * width + col);
            dst[0] = __floats2bfloat162_rn(y[0], y[1]);
            dst[1] = __floats2bfloat162_rn(y[2], y[3]);
        }
        else
        {
            __nv_bfloat16 *dst = out + row * (3 * width) + col;
#pragma unroll
            for (int j = 0; j < 4; ++j) split3(y[j], dst[j], dst[width + j], dst[2 * width + j]);
        }
    }
}

// RMSNorm + modulate of ROWS rows per CTA (a launch-shape variant of norm_modulate_kernel<VEC, false>:
// every thread keeps ROWS x VEC float4 loads in flight and the rows share one pair of block barriers).
template <int VEC, int THREADS, int ROWS>
__global__ void __launch_bounds__(THREADS) rms_rows_kernel(const float *__restrict__ x, int rows, const float *gamma,
                                                           const float *scale, const float *shift, float eps,
                                                           __nv_bfloat16 *out, int split3_out)
{
    constexpr int width = 4 * VEC * THREADS, warps = THREADS / 32;
    __shared__ float scratch[warps][ROWS];
    const int row0 = blockIdx.x * ROWS;
    grid_dependency_wait(); // launched programmatically after the GEMM that wrote x
    grid_dependents_launch();
    float4 v[ROWS][VEC];
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
    {
        const float4 *xr = reinterpret_cast<const float4 *>(x + static_cast<size_t>(row0 + r) * width);
#pragma unroll
        for (int i = 0; i < VEC; ++i)
            v[r][i] = row0 + r < rows ? xr[threadIdx.x + i * THREADS] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float sq[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
    {
        sq[r] = 0.f;
#pragma unroll
        for (int i = 0; i < VEC; ++i)
            sq[r] += (v[r][i].x * v[r][i].x + v[r][i].y * v[r][i].y) + (v[r][i].z * v[r][i].z + v[r][i].w * v[r][i].w);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq[r] += __shfl_xor_sync(0xffffffffu, sq[r], o);
    }
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (lane == 0)
#pragma unroll
        for (int r = 0; r < ROWS; ++r) scratch[warp][r] = sq[r];
    __syncthreads();
    float inverse[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
    {
        float total = 0.f;
        for (int w = 0; w < warps; ++w) total += scratch[w][r];
        inverse[r] = 1.f / sqrtf(total / float(width) + eps);
    }
#pragma unroll
    for (int i = 0; i < VEC; ++i)
    {
        const int col = (threadIdx.x + i * THREADS) * 4;
        const float4 g = __ldg(reinterpret_cast<const float4 *>(gamma + col));
        float4 sc = make_float4(0.f, 0.f, 0.f, 0.f), sh = sc;
        if (scale)
        {
            sc = __ldg(reinterpret_cast<const float4 *>(scale + col));
            sh = __ldg(reinterpret_cast<const float4 *>(shift + col));
        }
#pragma unroll
        for (int r = 0; r < ROWS; ++r)
        {
            if (row0 + r >= rows) continue;
            float y[4] = {v[r][i].x * inverse[r] * g.x, v[r][i].y * inverse[r] * g.y, v[r][i].z * inverse[r] * g.z,
                          v[r][i].w * inverse[r] * g.w};
            if (scale)
            {
                y[0] = y[0] * (1.f + sc.x) + sh.x;
                y[1] = y[1] * (1.f + sc.y) + sh.y;
                y[2] = y[2] * (1.f + sc.z) + sh.z;
                y[3] = y[3] * (1.f + sc.w) + sh.w;
            }
            const size_t row = static_cast<size_t>(row0 + r);
            if (!split3_out)
            {
                __nv_bfloat162 *dst = reinterpret_cast<__nv_bfloat162 *>(out + row * width + col);
                dst[0] = __floats2bfloat162_rn(y[0], y[1]);
                dst[1] = __floats2bfloat162_rn(y[2], y[3]);
            }
            else
            {
                __nv_bfloat16 *dst = out + row * (3 * width) + col;
#pragma unroll
                for (int j = 0; j < 4; ++j) split3(y[j], dst[j], dst[width + j], dst[2 * width + j]);
            }
        }
    }
}

// latent [128][tokens] (channel-major, as src/latent_ops.h stores it) -> A operand [tokens][128].
__global__ void latent_to_tokens_kernel(const float *__restrict__ latent, int tokens, int ld, __nv_bfloat16 *out,
                                        int split3_out)
{
    __shared__ float tile[32][33];
    const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y)
    {
        const int t = t0 + threadIdx.x;
        tile[i][threadIdx.x] = t < tokens ? latent[static_cast<size_t>(c0 + i) * ld + t] : 0.f;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y)
    {
        const int t = t0 + i;
        if (t >= tokens) continue;
        const float value = tile[threadIdx.x][i];
        const int c = c0 + threadIdx.x;
        if (!split3_out) out[static_cast<size_t>(t) * kLatent + c] = __float2bfloat16_rn(value);
        else
        {
            __nv_bfloat16 *dst = out + static_cast<size_t>(t) * (3 * kLatent) + c;
            split3(value, dst[0], dst[kLatent], dst[2 * kLatent]);
        }
    }
}

// y[n] = W[n,:] . act(x) + bias[n]: one warp per output row, x staged in shared memory.
// Bandwidth-bound (reads each BF16 weight once); used for the time-embedding MLP, the adaLN
// modulation linear and the output head's scale/shift linear (head.ncnn.param InnerProduct layers).
__global__ void __launch_bounds__(256) gemv_kernel(const __nv_bfloat16 *__restrict__ w, const float *__restrict__ x,
                                                   const float *bias, float *y, int n, int k, int silu_input)
{
    extern __shared__ float xs[];
    for (int i = threadIdx.x; i < k; i += blockDim.x)
    {
        const float value = x[i];
        xs[i] = silu_input ? value / (1.f + expf(-value)) : value;
    }
    __syncthreads();
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int row = blockIdx.x * (blockDim.x / 32) + warp;
    if (row >= n) return;
    const uint4 *wr = reinterpret_cast<const uint4 *>(w + static_cast<size_t>(row) * k);
    float acc = 0.f;
    for (int i = lane; i < k / 8; i += 32)
    {
        const uint4 packed = __ldg(wr + i);
        const __nv_bfloat162 *pair = reinterpret_cast<const __nv_bfloat162 *>(&packed);
        const float *xv = xs + i * 8;
#pragma unroll
        for (int j = 0; j < 4; ++j)
        {
            const float2 f = __bfloat1622float2(pair[j]);
            acc += f.x * xv[2 * j] + f.y * xv[2 * j + 1];
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) y[row] = acc + (bias ? bias[row] : 0.f);
}

// euler_step (src/latent_ops.cpp:72-92; GLSL `precise` at :135-143): change = delta * v,
// out = x + change, each rounded separately.
__global__ void euler_kernel(const float *sample, const float *prediction, float delta, long long count, float *out)
{
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        out[i] = __fadd_rn(sample[i], __fmul_rn(delta, prediction[i]));
}

__global__ void finite_kernel(const float *x, long long count, int *flag)
{
    bool ok = true;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        ok = ok && isfinite(x[i]);
    if (__any_sync(0xffffffffu, !ok) && (threadIdx.x % 32) == 0) atomicOr(flag, 1);
}

// unpack_for_vae (src/latent_ops.cpp:94-124, shader :145-164): z * sqrt(var + 1e-5) + mean,
// channel c -> output channel c/4 at (2y + (c%4)/2, 2x + c%2). One thread per output element, so
// the writes are coalesced.
__global__ void unpack_kernel(const float *packed, const float *mean, const float *variance, int w, int h, float *out)
{
    const long long total = 32LL * (2 * h) * (2 * w);
    const int ow = 2 * w, oh = 2 * h;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
    {
        const int oc = static_cast<int>(i / (static_cast<long long>(oh) * ow));
        const int rem = static_cast<int>(i % (static_cast<long long>(oh) * ow));
        const int oy = rem / ow, ox = rem % ow;
        const int c = oc * 4 + (oy % 2) * 2 + (ox % 2);
        const int y = oy / 2, x = ox / 2;
        const float scale = __fsqrt_rn(__fadd_rn(variance[c], 1e-5f));
        const float scaled = __fmul_rn(packed[static_cast<size_t>(c) * w * h + y * w + x], scale);
        out[i] = __fadd_rn(scaled, mean[c]);
    }
}

__global__ void gelu_kernel(float *data, long long count)
{
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
    {
        const float x = data[i];
        data[i] = 0.5f * x * erfcf(-0.7071067811865475f * x);
    }
}

__global__ void residual_add_kernel(const float *a, const float *b, float *out, long long count)
{
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        out[i] = __fadd_rn(a[i], b[i]);
}

// Stand-alone ErnieNorm layer (RMSNorm widths 128/3072/4096 or LayerNorm 4096), FP32 in and out.
__global__ void rmsnorm_kernel(const float *x, const float *gamma, int width, float eps, int centered, float *out)
{
    __shared__ float scratch[32];
    const size_t row = blockIdx.x;
    const float *xr = x + row * width;
    float mean = 0.f;
    if (centered)
    {
        float s = 0.f;
        for (int i = threadIdx.x; i < width; i += blockDim.x) s += xr[i];
        mean = block_sum(s, scratch) / float(width);
    }
    float sq = 0.f;
    for (int i = threadIdx.x; i < width; i += blockDim.x)
    {
        const float d = xr[i] - mean;
        sq += d * d;
    }
    const float inverse = 1.f / sqrtf(block_sum(sq, scratch) / float(width) + eps);
    for (int i = threadIdx.x; i < width; i += blockDim.x)
    {
        const float y = (xr[i] - mean) * inverse;
        out[row * width + i] = centered ? y : y * gamma[i];
    }
}

__global__ void synth_bf16_kernel(uint64_t seed, uint64_t stream_id, float scale, float offset, long long rows, int cols,
                                  int group, long long group_stride, long long group_offset, __nv_bfloat16 *out)
{
    const long long total = rows * cols;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
    {
        const long long row = i / cols, col = i % cols;
        const long long dst_row = (row / group) * group_stride + group_offset + row % group;
        const uint16_t bits = ernie_synth_weight(seed, stream_id, static_cast<uint64_t>(i), scale, offset);
        out[dst_row * cols + col] = __ushort_as_bfloat16(bits);
    }
}

__global__ void synth_f32_bf16_kernel(uint64_t seed, uint64_t stream_id, float scale, float offset, long long count,
                                      float *out)
{
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        out[i] = ernie_synth_bf16_to_float(ernie_synth_weight(seed, stream_id, static_cast<uint64_t>(i), scale, offset));
}

// FP32 rows -> BF16 GEMM operand (or 3 BF16 planes [rows][3*cols]): text features for text_proj.
__global__ void to_operand_kernel(const float *src, long long rows, int cols, __nv_bfloat16 *out, int split3_out)
{
    const long long total = rows * cols;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
    {
        const long long r = i / cols;
        const int c = static_cast<int>(i % cols);
        if (!split3_out) out[i] = __float2bfloat16_rn(src[i]);
        else
        {
            __nv_bfloat16 *dst = out + r * 3 * cols + c;
            split3(src[i], dst[0], dst[cols], dst[2 * cols]);
        }
    }
}

int grid_for(long long count, int threads = 256)
{
    long long blocks = (count + threads - 1) / threads;
    if (blocks > 148LL * 16) blocks = 148LL * 16;
    return blocks < 1 ? 1 : static_cast<int>(blocks);
}
} // namespace

int launch_norm_modulate(const float *x, int rows, int width, const float *gamma, const float *scale,
                         const float *shift, float eps, int centered, __nv_bfloat16 *out, int split3_out,
                         cudaStream_t stream)
{
    if (rows < 1) return cudaSuccess;
    if (!x || !out || (!centered && !gamma) || (scale == nullptr) != (shift == nullptr)) return cudaErrorInvalidValue;
    const dim3 grid(rows), block(kRowThreads);
    if (width == 4096)
    {
        if (centered) norm_modulate_kernel<4, true><<<grid, block, 0, stream>>>(x, gamma, scale, shift, eps, out, split3_out);
        else if (kNormRows > 1)
        {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((rows + kNormRows - 1) / kNormRows);
            cfg.blockDim = dim3(kNormThreads);
            cfg.stream = stream;
            cudaLaunchAttribute attrs[1];
            cfg.attrs = attrs;
            cfg.numAttrs = add_programmatic_attribute(attrs, 0);
            return cudaLaunchKernelEx(&cfg, rms_rows_kernel<1024 / kNormThreads, kNormThreads, kNormRows>, x, rows, gamma,
                                      scale, shift, eps, out, split3_out);
        }
        else
            norm_modulate_kernel<1024 / kNormThreads, false, kNormThreads>
                <<<grid, kNormThreads, 0, stream>>>(x, gamma, scale, shift, eps, out, split3_out);
    }
    else if (width == 3072)
    {
        if (centered) norm_modulate_kernel<3, true><<<grid, block, 0, stream>>>(x, gamma, scale, shift, eps, out, split3_out);
        else norm_modulate_kernel<3, false><<<grid, block, 0, stream>>>(x, gamma, scale, shift, eps, out, split3_out);
    }
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}

int launch_to_operand(const float *src, long long rows, int cols, __nv_bfloat16 *out, int split3_out,
                      cudaStream_t stream)
{
    if (rows < 1) return cudaSuccess;
    to_operand_kernel<<<grid_for(rows * cols), 256, 0, stream>>>(src, rows, cols, out, split3_out);
    return cudaGetLastError();
}

int launch_latent_to_tokens(const float *latent, int tokens, __nv_bfloat16 *out, int split3_out, cudaStream_t stream,
                            int ld)
{
    if (tokens < 1) return cudaSuccess;
    latent_to_tokens_kernel<<<dim3((tokens + 31) / 32, kLatent / 32), dim3(32, 8), 0, stream>>>(
        latent, tokens, ld > 0 ? ld : tokens, out, split3_out);
    return cudaGetLastError();
}

int launch_gemv(const __nv_bfloat16 *w, const float *x, const float *bias, float *y, int n, int k, int silu_input,
                cudaStream_t stream)
{
    if (k % 8 || k > 12288 || n < 1) return cudaErrorInvalidValue;
    gemv_kernel<<<(n + 7) / 8, 256, k * sizeof(float), stream>>>(w, x, bias, y, n, k, silu_input);
    return cudaGetLastError();
}

int launch_euler(const float *sample, const float *prediction, float delta, long long count, float *out,
                 cudaStream_t stream)
{
    euler_kernel<<<grid_for(count), 256, 0, stream>>>(sample, prediction, delta, count, out);
    return cudaGetLastError();
}

int launch_finite(const float *x, long long count, int *flag, cudaStream_t stream)
{
    finite_kernel<<<grid_for(count), 256, 0, stream>>>(x, count, flag);
    return cudaGetLastError();
}

int launch_unpack_for_vae(const float *packed, const float *mean, const float *variance, int w, int h, float *out,
                          cudaStream_t stream)
{
    unpack_kernel<<<grid_for(32LL * 4 * w * h), 256, 0, stream>>>(packed, mean, variance, w, h, out);
    return cudaGetLastError();
}

int launch_gelu(float *data, long long count, cudaStream_t stream)
{
    gelu_kernel<<<grid_for(count), 256, 0, stream>>>(data, count);
    return cudaGetLastError();
}

int launch_residual_add(const float *a, const float *b, float *out, long long count, cudaStream_t stream)
{
    residual_add_kernel<<<grid_for(count), 256, 0, stream>>>(a, b, out, count);
    return cudaGetLastError();
}

int launch_rmsnorm(const float *x, const float *gamma, long long rows, int width, float eps, int centered, float *out,
                   cudaStream_t stream)
{
    if (rows < 1) return cudaSuccess;
    rmsnorm_kernel<<<static_cast<unsigned>(rows), 128, 0, stream>>>(x, gamma, width, eps, centered, out);
    return cudaGetLastError();
}

int launch_synth_bf16(uint64_t seed, uint64_t stream_id, float scale, float offset, long long rows, int cols, int group,
                      long long group_stride, long long group_offset, __nv_bfloat16 *out, cudaStream_t stream)
{
    synth_bf16_kernel<<<grid_for(rows * cols), 256, 0, stream>>>(seed, stream_id, scale, offset, rows, cols, group,
                                                                 group_stride, group_offset, out);
    return cudaGetLastError();
}

int launch_synth_f32_bf16(uint64_t seed, uint64_t stream_id, float scale, float offset, long long count, float *out,
                          cudaStream_t stream)
{
    synth_f32_bf16_kernel<<<grid_for(count), 256, 0, stream>>>(seed, stream_id, scale, offset, count, out);
    return cudaGetLastError();
}
} // namespace ernie_b200
