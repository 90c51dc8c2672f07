// The text encoder's rotary embedding and head split (reference: the Mistral decoder layer the reference
// exports per block, tools/export_text_block.py:50-61, with ExportBlock.rotary's half-split rotation,
// tools/export_dit_block.py:39-47).
#include "kernels.h"

namespace ernie_b200
{
namespace
{
constexpr int kTextQHeads = 32, kTextKvHeads = 8, kTextHeadDim = 128, kTextQkv = (32 + 2 * 8) * 128;

// qkv FP32 [tokens][6144] (q 32 heads, k 8 heads, v 8 heads, 128 each) -> head-major FP32 q [32][tokens][128],
// k, v [8][tokens][128]; q and k rotated: out[:64] = x[:64] cos[:64] - x[64:] sin[:64],
// out[64:] = x[64:] cos[64:] + x[:64] sin[64:] (FP32, no contraction).
__global__ void text_rope_kernel(const float *qkv, const float *cos_t, const float *sin_t, int tokens, float *q,
                                 float *k, float *v)
{
    const int head = blockIdx.y, t = blockIdx.x, d = threadIdx.x; // 64 threads: pairs (d, d + 64)
    if (t >= tokens) return;
    const float *row = qkv + static_cast<size_t>(t) * kTextQkv;
    if (head < kTextQHeads + kTextKvHeads)
    {
        const float *x = row + head * kTextHeadDim;
        const float *c = cos_t + static_cast<size_t>(t) * kTextHeadDim, *s = sin_t + static_cast<size_t>(t) * kTextHeadDim;
        const float first = x[d], second = x[d + 64];
        const float lo = __fsub_rn(__fmul_rn(first, c[d]), __fmul_rn(second, s[d]));
        const float hi = __fadd_rn(__fmul_rn(second, c[d + 64]), __fmul_rn(first, s[d + 64]));
        float *dst = head < kTextQHeads
                         ? q + (static_cast<size_t>(head) * tokens + t) * kTextHeadDim
                         : k + (static_cast<size_t>(head - kTextQHeads) * tokens + t) * kTextHeadDim;
        dst[d] = lo;
        dst[d + 64] = hi;
    }
    else
    {
        const int vh = head - kTextQHeads - kTextKvHeads;
        const float *x = row + (kTextQHeads + kTextKvHeads + vh) * kTextHeadDim;
        float *dst = v + (static_cast<size_t>(vh) * tokens + t) * kTextHeadDim;
        dst[d] = x[d];
        dst[d + 64] = x[d + 64];
    }
}

// BF16 mode: the same rotation written as the tcgen05 attention's operands, q [32][rows_pad][128],
// k [8][rows_pad][128] and v transposed [8][128][rows_pad] (rows past `tokens` left as they are: zero).
// One CTA = 32 tokens x one head, one warp per token at a time with lanes on consecutive dimensions (every
// load and store a whole row segment). V goes through a shared-memory tile so that its transposed rows are
// written 32 tokens at a time.
__global__ void text_rope_bf16_kernel(const float *qkv, const float *cos_t, const float *sin_t, int tokens,
                                      int rows_pad, __nv_bfloat16 *q, __nv_bfloat16 *k, __nv_bfloat16 *vt)
{
    __shared__ __nv_bfloat16 tile[kTextHeadDim][34]; // [dim][token] (+2 padding: row stride 17 banks)
    const int head = blockIdx.y, t0 = blockIdx.x * 32, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool rotate = head < kTextQHeads + kTextKvHeads;
    const int col = rotate ? head * kTextHeadDim : (kTextQHeads + kTextKvHeads) * kTextHeadDim +
                                                       (head - kTextQHeads - kTextKvHeads) * kTextHeadDim;
    for (int tt = warp; tt < 32; tt += 4)
    {
        const int t = t0 + tt;
        if (t >= tokens) break;
        const float *x = qkv + static_cast<size_t>(t) * kTextQkv + col;
        if (rotate)
        {
            const float *c = cos_t + static_cast<size_t>(t) * kTextHeadDim;
            const float *s = sin_t + static_cast<size_t>(t) * kTextHeadDim;
            __nv_bfloat16 *dst = head < kTextQHeads
                                     ? q + (static_cast<size_t>(head) * rows_pad + t) * kTextHeadDim
                                     : k + (static_cast<size_t>(head - kTextQHeads) * rows_pad + t) * kTextHeadDim;
#pragma unroll
            for (int j = 0; j < 2; ++j)
            {
                const int d = lane + 32 * j;
                const float first = x[d], second = x[d + 64];
                dst[d] = __float2bfloat16_rn(__fsub_rn(__fmul_rn(first, c[d]), __fmul_rn(second, s[d])));
                dst[d + 64] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(second, c[d + 64]), __fmul_rn(first, s[d + 64])));
            }
        }
        else
        {
#pragma unroll
            for (int j = 0; j < 4; ++j) tile[lane + 32 * j][tt] = __float2bfloat16_rn(x[lane + 32 * j]);
        }
    }
    if (rotate) return; // uniform per CTA
    __syncthreads();
    // transposed: dimension row d holds tokens t0 .. t0 + 31 (consecutive 64 bytes)
    const int vh = head - kTextQHeads - kTextKvHeads;
    __nv_bfloat16 *base = vt + static_cast<size_t>(vh) * kTextHeadDim * rows_pad + t0;
    for (int i = threadIdx.x; i < kTextHeadDim * 32; i += blockDim.x)
    {
        const int d = i >> 5, tt = i & 31;
        if (t0 + tt < tokens) base[static_cast<size_t>(d) * rows_pad + tt] = tile[d][tt];
    }
}
} // namespace

int launch_text_rope_bf16(const float *qkv, const float *cos_t, const float *sin_t, int tokens, int rows_pad,
                          __nv_bfloat16 *q, __nv_bfloat16 *k, __nv_bfloat16 *vt, cudaStream_t stream)
{
    if (tokens < 1 || rows_pad < tokens) return cudaErrorInvalidValue;
    text_rope_bf16_kernel<<<dim3((tokens + 31) / 32, kTextQHeads + 2 * kTextKvHeads), 128, 0, stream>>>(
        qkv, cos_t, sin_t, tokens, rows_pad, q, k, vt);
    return cudaGetLastError();
}

int launch_text_rope(const float *qkv, const float *cos_t, const float *sin_t, int tokens, float *q, float *k, float *v,
                     cudaStream_t stream)
{
    if (tokens < 1) return cudaErrorInvalidValue;
    text_rope_kernel<<<dim3(tokens, kTextQHeads + 2 * kTextKvHeads), 64, 0, stream>>>(qkv, cos_t, sin_t, tokens, q, k, v);
    return cudaGetLastError();
}
} // namespace ernie_b200
