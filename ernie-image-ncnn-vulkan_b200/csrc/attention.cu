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
    const dim3 grid((args.nq + kFQ - 1) / kFQ, args.heads);
    attention_f32_kernel<<<grid, kFThreads, kFSmem, stream>>>(args);
    return cudaGetLastError();
}
} // namespace ernie_b200
