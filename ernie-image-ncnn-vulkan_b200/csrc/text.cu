// The text encoder's rotary embedding and head split (reference: the Mistral decoder layer the reference
// exports per block, tools/export_text_block.py:51-61, with ExportBlock.rotary's half-split rotation,
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

// ---- decode products (prompt enhancer) -------------------------------------------------------------
// The PE block graph's seven projections (src/pe_graph.cpp:22-28 q/k/v, :62 o_proj, :67-69 gate/up with
// the Swish on the gate, :71 down_proj) for a step of 1..4 token rows, and the LM head's 131072-row
// projection: one warp per weight row, FP32 accumulation against the activation rows staged in FP32.
namespace
{
constexpr int kGemvRows = 4, kGemvWarps = 8, kGemvMaxK = 9216;

__device__ __forceinline__ float warp_sum_f(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// sum_k x[r][k] * w[k] for the block's staged rows, one weight row per warp, 8 BF16 per lane per step
__device__ __forceinline__ void gemv_row(const float *xs, int rows, int k, const __nv_bfloat16 *w, int lane,
                                         float (&acc)[kGemvRows])
{
#pragma unroll
    for (int r = 0; r < kGemvRows; ++r) acc[r] = 0.f;
    // four 16-byte weight loads in flight per lane (k is a multiple of 256)
#pragma unroll 4
    for (int k0 = lane * 8; k0 < k; k0 += 256)
    {
        const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(w + k0));
        const __nv_bfloat162 *p = reinterpret_cast<const __nv_bfloat162 *>(&raw);
        float wv[8];
#pragma unroll
        for (int j = 0; j < 4; ++j)
        {
            const float2 f = __bfloat1622float2(p[j]);
            wv[2 * j] = f.x;
            wv[2 * j + 1] = f.y;
        }
#pragma unroll
        for (int r = 0; r < kGemvRows; ++r)
        {
            if (r >= rows) break;
            const float4 x0 = *reinterpret_cast<const float4 *>(xs + r * k + k0);
            const float4 x1 = *reinterpret_cast<const float4 *>(xs + r * k + k0 + 4);
            float s = acc[r];
            s = fmaf(x0.x, wv[0], s);
            s = fmaf(x0.y, wv[1], s);
            s = fmaf(x0.z, wv[2], s);
            s = fmaf(x0.w, wv[3], s);
            s = fmaf(x1.x, wv[4], s);
            s = fmaf(x1.y, wv[5], s);
            s = fmaf(x1.z, wv[6], s);
            s = fmaf(x1.w, wv[7], s);
            acc[r] = s;
        }
    }
#pragma unroll
    for (int r = 0; r < kGemvRows; ++r) acc[r] = warp_sum_f(acc[r]);
}

__device__ __forceinline__ void store_h(const GemvArgs &a, int r, int i, float v)
{
    if (a.h_split3)
    {
        __nv_bfloat16 *dst = a.h + static_cast<size_t>(r) * 3 * a.ffn + i;
        const __nv_bfloat16 hi = __float2bfloat16_rn(v);
        const float r1 = v - __bfloat162float(hi);
        const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
        dst[0] = hi;
        dst[a.ffn] = mid;
        dst[2 * a.ffn] = __float2bfloat16_rn(r1 - __bfloat162float(mid));
    }
    else
        a.h[static_cast<size_t>(r) * a.ffn + i] = __float2bfloat16_rn(v);
}

__global__ void __launch_bounds__(kGemvWarps * 32) gemv_kernel(GemvArgs a, int epi)
{
    extern __shared__ float xs[]; // [rows][k] FP32
    const int total = a.rows * a.k;
    for (int i = threadIdx.x; i < total; i += blockDim.x)
    {
        const int r = i / a.k, c = i - r * a.k;
        const __nv_bfloat16 *src = a.a + static_cast<size_t>(r) * a.planes * a.k + c;
        float v = __bfloat162float(src[0]);
        if (a.planes == 3) v = (v + __bfloat162float(src[a.k])) + __bfloat162float(src[2 * a.k]);
        xs[i] = v;
    }
    __syncthreads();
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int outputs = epi == static_cast<int>(GemvEpilogue::SwiGLU) ? a.ffn : a.n_rows;
    const int o = blockIdx.x * kGemvWarps + warp;
    if (o >= outputs) return;
    float acc[kGemvRows];
    if (epi == static_cast<int>(GemvEpilogue::SwiGLU))
    {
        // feature o: up row (o / 64) * 128 + o % 64, gate row 64 further
        const int row_up = (o / 64) * 128 + (o % 64);
        float gate[kGemvRows];
        gemv_row(xs, a.rows, a.k, a.w + static_cast<size_t>(row_up + 64) * a.k, lane, gate);
        gemv_row(xs, a.rows, a.k, a.w + static_cast<size_t>(row_up) * a.k, lane, acc);
        if (lane == 0)
            for (int r = 0; r < a.rows; ++r)
            {
                const float g = gate[r];
                const float v = a.h_split3 ? acc[r] * __fdiv_rn(g, 1.f + expf(-g)) : acc[r] * __fdividef(g, 1.f + __expf(-g));
                store_h(a, r, o, v);
            }
        return;
    }
    gemv_row(xs, a.rows, a.k, a.w + static_cast<size_t>(o) * a.k, lane, acc);
    if (lane == 0)
        for (int r = 0; r < a.rows; ++r)
        {
            float *dst = a.out + static_cast<size_t>(r) * a.ldo + o;
            if (epi == static_cast<int>(GemvEpilogue::Resid)) *dst = *dst + acc[r];
            else *dst = acc[r];
        }
}
} // namespace

__global__ void pe_cache_append_kernel(const float *k, const float *v, int rows, float *kc, float *vc, int capacity,
                                       const int *position)
{
    const int r = blockIdx.x, head = blockIdx.y, lane = threadIdx.x; // 32 threads: one float4 each
    const size_t src = (static_cast<size_t>(head) * rows + r) * 128 + lane * 4;
    const size_t dst = (static_cast<size_t>(head) * capacity + *position + r) * 128 + lane * 4;
    *reinterpret_cast<float4 *>(kc + dst) = *reinterpret_cast<const float4 *>(k + src);
    *reinterpret_cast<float4 *>(vc + dst) = *reinterpret_cast<const float4 *>(v + src);
}

__global__ void pe_advance_kernel(int *position, int rows) { *position += rows; }

int launch_pe_cache_append(const float *k, const float *v, int rows, float *k_cache, float *v_cache, int capacity,
                           const int *position, cudaStream_t stream)
{
    if (!k || !v || !k_cache || !v_cache || !position || rows < 1 || capacity < rows) return cudaErrorInvalidValue;
    pe_cache_append_kernel<<<dim3(rows, 8), 32, 0, stream>>>(k, v, rows, k_cache, v_cache, capacity, position);
    return cudaGetLastError();
}

int launch_pe_advance(int *position, int rows, cudaStream_t stream)
{
    if (!position || rows < 1) return cudaErrorInvalidValue;
    pe_advance_kernel<<<1, 1, 0, stream>>>(position, rows);
    return cudaGetLastError();
}

int prepare_gemv_kernels()
{
    return cudaFuncSetAttribute(gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvRows * kGemvMaxK * 4);
}

int launch_gemv(const GemvArgs &a, GemvEpilogue epi, cudaStream_t stream)
{
    if (!a.a || !a.w || a.rows < 1 || a.rows > kGemvRows || a.k < 256 || a.k % 256 || a.k > kGemvMaxK ||
        (a.planes != 1 && a.planes != 3) || a.n_rows < 1)
        return cudaErrorInvalidValue;
    int outputs = a.n_rows;
    if (epi == GemvEpilogue::SwiGLU)
    {
        if (!a.h || a.ffn < 64 || a.ffn % 64 || a.n_rows != 2 * a.ffn) return cudaErrorInvalidValue;
        outputs = a.ffn;
    }
    else if (!a.out || a.ldo < a.n_rows)
        return cudaErrorInvalidValue;
    const size_t smem = static_cast<size_t>(a.rows) * a.k * 4;
    gemv_kernel<<<(outputs + kGemvWarps - 1) / kGemvWarps, kGemvWarps * 32, smem, stream>>>(a, static_cast<int>(epi));
    return cudaGetLastError();
}
} // namespace ernie_b200
