// Attention for the ERNIE DiT block (reference: sdpa_22 in block.ncnn.param:58, ErnieSDPA /
// AccurateSDPA in src/ernie_attention.cpp:35-233): softmax(Q K^T / sqrt(128) + mask_row) V over the
// joint image+text sequence, non-causal. Keys at or beyond the valid count (padded text slots,
// mask -1e30 in src/conditioning.cpp:41-42) contribute exactly zero in the reference, so whole key
// tiles past the valid count are skipped here.
//
//  * BF16 mode runs the tcgen05/TMEM flash kernel in flash_tc.cu.
//  * attention_f32_kernel: FP32 scores, FP64 softmax sums and P.V accumulation. Serves the FP32
//    exactness mode, the stand-alone SDPA layer contract (GQA with one K/V head, widths up to 128,
//    row or dense additive masks, mask per head), replacing the reference's Kahan-compensated
//    FP32 shaders (cmake/ErnieAttentionShader.cmake:18-55), the text encoder's causal grouped-query
//    attention (32 query heads over 8 K/V heads), and the prompt enhancer's chunks over its K/V cache
//    (queries at positions causal_offset.., keys 0..kv_len).
#include "kernels.h"
#include <cmath>

namespace ernie_b200
{
namespace
{
constexpr int kDim = 128;

// ------------------------------------------------------------------ FP32 attention, FP64 sums
constexpr int kFQ = 64, kFK = 32, kFThreads = 256;
constexpr int kFSmem = (kFQ * (kDim + 1) + kFK * (kDim + 1) + kFK * kDim + kFQ * (kFK + 1)) * 4;

__device__ __forceinline__ void split3(float x, __nv_bfloat16 &hi, __nv_bfloat16 &mid, __nv_bfloat16 &lo)
{
    hi = __float2bfloat16_rn(x);
    const float r1 = x - __bfloat162float(hi);
    mid = __float2bfloat16_rn(r1);
    lo = __float2bfloat16_rn(r1 - __bfloat162float(mid));
}

__global__ void __launch_bounds__(kFThreads) attention_f32_kernel(AttentionF32Args a)
{
    extern __shared__ float fsm[];
    float *qs = fsm;                         // [64][129]
    float *ks = qs + kFQ * (kDim + 1);       // [32][129]
    float *vs = ks + kFK * (kDim + 1);       // [32][128]
    float *ps = vs + kFK * kDim;             // [64][33]
    const int head = blockIdx.y, q0 = blockIdx.x * kFQ;
    const int kv_head = head / (a.heads / a.kv_heads);
    const int tid = threadIdx.x, qi = tid >> 2, sub = tid & 3;
    const int width = a.width;
    const float scale = 1.f / sqrtf(static_cast<float>(width));
    const float *qh = a.q + head * a.q_head_stride;
    const float *kh = a.k + kv_head * a.kv_head_stride;
    const float *vh = a.v + kv_head * a.kv_head_stride;
    for (int i = tid; i < kFQ * kDim; i += kFThreads)
    {
        const int r = i / kDim, d = i % kDim;
        qs[r * (kDim + 1) + d] = (q0 + r < a.nq && d < width) ? qh[static_cast<size_t>(q0 + r) * width + d] : 0.f;
    }
    const int qrow = q0 + qi;
    const float *mrow = nullptr;
    if (a.mask)
        mrow = a.mask + (static_cast<size_t>(a.mask_heads == 1 ? 0 : head) * a.mask_rows +
                         (a.mask_rows == 1 ? 0 : (qrow < a.nq ? qrow : 0))) *
                            a.nk;
    float m_run = -INFINITY;
    double l_run = 0.0;
    double acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.0;
    // causal: no key past this CTA's last query row (rows start at position causal_offset)
    const int kv_end = a.causal ? min(a.kv_len, q0 + kFQ + a.causal_offset) : a.kv_len;
    const int tiles = (kv_end + kFK - 1) / kFK;
    for (int j = 0; j < tiles; ++j)
    {
        const int key0 = j * kFK;
        __syncthreads();
        for (int i = tid; i < kFK * kDim; i += kFThreads)
        {
            const int r = i / kDim, d = i % kDim;
            const bool in = key0 + r < a.kv_len && d < width;
            ks[r * (kDim + 1) + d] = in ? kh[static_cast<size_t>(key0 + r) * width + d] : 0.f;
            vs[r * kDim + d] = in ? vh[static_cast<size_t>(key0 + r) * width + d] : 0.f;
        }
        __syncthreads();
        float sc[8];
        float tile_max = -INFINITY;
#pragma unroll
        for (int i = 0; i < 8; ++i)
        {
            const int kj = sub + 4 * i;
            const float *qr = qs + qi * (kDim + 1);
            const float *kr = ks + kj * (kDim + 1);
            float dot = 0.f;
#pragma unroll 8
            for (int d = 0; d < kDim; ++d) dot = fmaf(qr[d], kr[d], dot);
            const int key = key0 + kj;
            float x = key < a.kv_len && !(a.causal && key > qrow + a.causal_offset)
                          ? dot * scale + (mrow ? mrow[key] : 0.f)
                          : -INFINITY;
            sc[i] = x;
            tile_max = fmaxf(tile_max, x);
        }
        tile_max = fmaxf(tile_max, __shfl_xor_sync(0xffffffffu, tile_max, 1));
        tile_max = fmaxf(tile_max, __shfl_xor_sync(0xffffffffu, tile_max, 2));
        const float m_new = fmaxf(m_run, tile_max);
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        const double alpha = static_cast<double>(expf(m_run - m_use));
        m_run = m_new;
        double psum = 0.0;
#pragma unroll
        for (int i = 0; i < 8; ++i)
        {
            const float p = expf(sc[i] - m_use);
            ps[qi * (kFK + 1) + sub + 4 * i] = p;
            psum += p;
        }
        psum += __shfl_xor_sync(0xffffffffu, psum, 1);
        psum += __shfl_xor_sync(0xffffffffu, psum, 2);
        l_run = l_run * alpha + psum;
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] *= alpha;
        __syncthreads();
        const float *pr = ps + qi * (kFK + 1);
        for (int kj = 0; kj < kFK; ++kj)
        {
            const double p = pr[kj];
            const float *vr = vs + kj * kDim + sub;
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[i] = fma(p, static_cast<double>(vr[4 * i]), acc[i]);
        }
    }
    if (qrow >= a.nq) return;
    if (a.out_mode == 0)
    {
        float *dst = a.out_f32 + (static_cast<size_t>(head) * a.nq + qrow) * width;
#pragma unroll
        for (int i = 0; i < 32; ++i)
        {
            const int d = sub + 4 * i;
            if (d < width) dst[d] = static_cast<float>(acc[i] / l_run);
        }
    }
    else if (a.out_mode == 2)
    {
        __nv_bfloat16 *dst = a.out_split3 + (static_cast<size_t>(qrow) * a.heads + head) * width;
#pragma unroll
        for (int i = 0; i < 32; ++i)
        {
            const int d = sub + 4 * i;
            if (d < width) dst[d] = __float2bfloat16_rn(static_cast<float>(acc[i] / l_run));
        }
    }
    else
    {
        const size_t plane = static_cast<size_t>(a.heads) * width;
        __nv_bfloat16 *dst = a.out_split3 + static_cast<size_t>(qrow) * 3 * plane + static_cast<size_t>(head) * width;
#pragma unroll
        for (int i = 0; i < 32; ++i)
        {
            const int d = sub + 4 * i;
            if (d < width) split3(static_cast<float>(acc[i] / l_run), dst[d], dst[plane + d], dst[2 * plane + d]);
        }
    }
}
// ------------------------------------------------------------------ decode: a few query rows, many keys
// One CTA per (head, query row); its 8 warps take consecutive groups of 4 keys in turn. Per key a warp forms
// the FP32 score (4 dimensions per lane, reduced across the warp) and updates its own online softmax, the
// total and P.V in FP64 as above; the warps' partial results are merged at the end. Same arithmetic
// contract as attention_f32_kernel: FP32 scores and exponentials, FP64 sums.
constexpr int kDWarps = 8, kDKeys = 4;

__device__ __forceinline__ float warp_sum_f32(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__global__ void __launch_bounds__(kDWarps * 32) attention_decode_kernel(AttentionF32Args a)
{
    __shared__ __align__(16) float qs[kDim];
    __shared__ float wm[kDWarps];
    __shared__ double wl[kDWarps];
    __shared__ double wo[kDWarps][kDim];
    const int head = blockIdx.x, qrow = blockIdx.y;
    const int kv_head = head / (a.heads / a.kv_heads);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const float scale = 1.f / sqrtf(static_cast<float>(kDim));
    if (threadIdx.x < kDim) qs[threadIdx.x] = a.q[head * a.q_head_stride + static_cast<size_t>(qrow) * kDim + threadIdx.x];
    __syncthreads();
    const float4 q4 = *reinterpret_cast<const float4 *>(qs + lane * 4);
    const float *kh = a.k + kv_head * a.kv_head_stride;
    const float *vh = a.v + kv_head * a.kv_head_stride;
    const float *mrow = nullptr;
    if (a.mask)
        mrow = a.mask + (static_cast<size_t>(a.mask_heads == 1 ? 0 : head) * a.mask_rows + (a.mask_rows == 1 ? 0 : qrow)) *
                            a.nk;
    const int offset = a.position ? *a.position : a.causal_offset;
    const int kv_len = a.position ? offset + a.nq : a.kv_len;
    const int kv_end = a.causal ? min(kv_len, qrow + offset + 1) : kv_len;
    float m_w = -INFINITY;
    double l_w = 0.0, o[4] = {0.0, 0.0, 0.0, 0.0};
    for (int key0 = warp * kDKeys; key0 < kv_end; key0 += kDWarps * kDKeys)
    {
        float sc[kDKeys];
        float4 v4[kDKeys];
#pragma unroll
        for (int j = 0; j < kDKeys; ++j)
        {
            const int key = key0 + j;
            float d = 0.f;
            v4[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (key < kv_end)
            {
                const float4 k4 = *reinterpret_cast<const float4 *>(kh + static_cast<size_t>(key) * kDim + lane * 4);
                v4[j] = *reinterpret_cast<const float4 *>(vh + static_cast<size_t>(key) * kDim + lane * 4);
                d = fmaf(q4.w, k4.w, fmaf(q4.z, k4.z, fmaf(q4.y, k4.y, q4.x * k4.x)));
            }
            sc[j] = d;
        }
#pragma unroll
        for (int j = 0; j < kDKeys; ++j) sc[j] = warp_sum_f32(sc[j]);
#pragma unroll
        for (int j = 0; j < kDKeys; ++j)
        {
            const int key = key0 + j;
            if (key >= kv_end) break;
            const float s = sc[j] * scale + (mrow ? mrow[key] : 0.f);
            if (s == -INFINITY) continue;
            const float m_new = fmaxf(m_w, s);
            const double alpha = static_cast<double>(expf(m_w - m_new)); // 0 while m_w is -inf
            const double p = static_cast<double>(expf(s - m_new));
            l_w = l_w * alpha + p;
            o[0] = fma(p, static_cast<double>(v4[j].x), o[0] * alpha);
            o[1] = fma(p, static_cast<double>(v4[j].y), o[1] * alpha);
            o[2] = fma(p, static_cast<double>(v4[j].z), o[2] * alpha);
            o[3] = fma(p, static_cast<double>(v4[j].w), o[3] * alpha);
            m_w = m_new;
        }
    }
    if (lane == 0)
    {
        wm[warp] = m_w;
        wl[warp] = l_w;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) wo[warp][lane * 4 + i] = o[i];
    __syncthreads();
    if (threadIdx.x >= kDim) return;
    const int d = threadIdx.x;
    float m = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDWarps; ++w) m = fmaxf(m, wm[w]);
    double l = 0.0, acc = 0.0;
#pragma unroll
    for (int w = 0; w < kDWarps; ++w)
    {
        if (wm[w] == -INFINITY) continue;
        const double f = static_cast<double>(expf(wm[w] - m));
        l += wl[w] * f;
        acc += wo[w][d] * f;
    }
    const float out = static_cast<float>(acc / l);
    if (a.out_mode == 0)
        a.out_f32[(static_cast<size_t>(head) * a.nq + qrow) * kDim + d] = out;
    else if (a.out_mode == 2)
        a.out_split3[(static_cast<size_t>(qrow) * a.heads + head) * kDim + d] = __float2bfloat16_rn(out);
    else
    {
        const size_t plane = static_cast<size_t>(a.heads) * kDim;
        __nv_bfloat16 *dst = a.out_split3 + static_cast<size_t>(qrow) * 3 * plane + static_cast<size_t>(head) * kDim + d;
        split3(out, dst[0], dst[plane], dst[2 * plane]);
    }
}
} // namespace

int prepare_attention_kernels()
{
    return cudaFuncSetAttribute(attention_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kFSmem);
}

int launch_attention_f32(const AttentionF32Args &args, cudaStream_t stream)
{
    if (args.nq < 1 || args.nk < 1 || args.kv_len < 1 || args.kv_len > args.nk || args.width < 1 ||
        args.width > kDim || args.heads < 1 || args.kv_heads < 1 || args.heads % args.kv_heads ||
        args.out_mode < 0 || args.out_mode > 2 || args.causal_offset < 0 ||
        (args.mask && args.mask_heads != 1 && args.mask_heads != args.heads) ||
        (args.mask && args.mask_rows != 1 && args.mask_rows != args.nq))
        return cudaErrorInvalidValue;
    if (args.decode)
    {
        if (args.nq > 32 || args.width != kDim) return cudaErrorInvalidValue;
        attention_decode_kernel<<<dim3(args.heads, args.nq), kDWarps * 32, 0, stream>>>(args);
        return cudaGetLastError();
    }
    const dim3 grid((args.nq + kFQ - 1) / kFQ, args.heads);
    attention_f32_kernel<<<grid, kFThreads, kFSmem, stream>>>(args);
    return cudaGetLastError();
}
} // namespace ernie_b200
