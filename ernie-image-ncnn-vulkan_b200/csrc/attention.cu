// Attention for the ERNIE DiT block (reference: sdpa_22 in block.ncnn.param:58, ErnieSDPA /
// AccurateSDPA in src/ernie_attention.cpp:35-233): softmax(Q K^T / sqrt(128) + mask_row) V over the
// joint image+text sequence, non-causal. Keys at or beyond the valid count (padded text slots,
// mask -1e30 in src/conditioning.cpp:41-42) contribute exactly zero in the reference, so whole key
// tiles past the valid count are skipped here.
//
//  * attention_bf16_kernel: BF16 operands, FP32 online softmax and accumulation (flash form,
//    O(N) memory, no N x N workspace). 128 queries x 64 keys per iteration, 8 warps.
//  * attention_f32_kernel: FP32 scores, FP64 softmax sums and P.V accumulation. Serves the FP32
//    exactness mode and the stand-alone SDPA layer contract (GQA with one K/V head, widths up to 128,
//    row or dense additive masks, mask per head), replacing the reference's Kahan-compensated
//    FP32 shaders (cmake/ErnieAttentionShader.cmake:18-55).
#include "kernels.h"
#include <cmath>

namespace ernie_b200
{
namespace
{
// ------------------------------------------------------------------ BF16 flash attention
constexpr int kQTile = 128, kKTile = 64, kDim = 128, kAttnThreads = 256;
constexpr int kAttnSmem = (kQTile + 4 * kKTile) * kDim * 2;

__device__ __forceinline__ uint32_t swz(int row, int chunk) { return row * kDim + ((chunk ^ (row & 7)) << 3); }

__device__ __forceinline__ void cp_async16(void *dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi)
{
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ void load_rows(__nv_bfloat16 *dst, const __nv_bfloat16 *src, int rows)
{
    for (int i = threadIdx.x; i < rows * 16; i += kAttnThreads)
    {
        const int r = i >> 4, ch = i & 15;
        cp_async16(dst + swz(r, ch), src + static_cast<size_t>(r) * kDim + ch * 8);
    }
}

__global__ void __launch_bounds__(kAttnThreads, 1)
    attention_bf16_kernel(const __nv_bfloat16 *__restrict__ q, const __nv_bfloat16 *__restrict__ k,
                          const __nv_bfloat16 *__restrict__ v, const float *__restrict__ mask, int rows, int rows_pad,
                          int kv_len, int heads, __nv_bfloat16 *__restrict__ out)
{
    extern __shared__ __align__(128) __nv_bfloat16 smem[];
    __nv_bfloat16 *qs = smem;
    __nv_bfloat16 *ks = smem + kQTile * kDim;
    __nv_bfloat16 *vs = ks + 2 * kKTile * kDim;
    const int head = blockIdx.y, q0 = blockIdx.x * kQTile;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const size_t head_off = static_cast<size_t>(head) * rows_pad * kDim;
    const __nv_bfloat16 *qh = q + head_off, *kh = k + head_off, *vh = v + head_off;
    const int tiles = (kv_len + kKTile - 1) / kKTile;

    load_rows(qs, qh + static_cast<size_t>(q0) * kDim, kQTile);
    load_rows(ks, kh, kKTile);
    load_rows(vs, vh, kKTile);
    cp_commit();

    constexpr float kScaleLog2 = 0.08838834764831845f * 1.4426950408889634f;
    constexpr float kLog2e = 1.4426950408889634f;
    uint32_t qf[8][4];
    float o[16][4];
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    const int g = lane >> 2, t = lane & 3;
    const int mat = lane >> 3, r8 = lane & 7;

    for (int j = 0; j < tiles; ++j)
    {
        const int stage = j & 1;
        if (j + 1 < tiles)
        {
            const int ns = stage ^ 1;
            load_rows(ks + ns * kKTile * kDim, kh + static_cast<size_t>(j + 1) * kKTile * kDim, kKTile);
            load_rows(vs + ns * kKTile * kDim, vh + static_cast<size_t>(j + 1) * kKTile * kDim, kKTile);
            cp_commit();
            cp_wait<1>();
        }
        else
            cp_wait<0>();
        __syncthreads();
        if (j == 0)
        {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
            {
                const int row = warp * 16 + r8 + (mat & 1) * 8;
                const int chunk = kk * 2 + (mat >> 1);
                ldsm_x4(static_cast<uint32_t>(__cvta_generic_to_shared(qs + swz(row, chunk))), qf[kk][0], qf[kk][1],
                        qf[kk][2], qf[kk][3]);
            }
        }
        const __nv_bfloat16 *kt = ks + stage * kKTile * kDim;
        const __nv_bfloat16 *vt = vs + stage * kKTile * kDim;
        float s[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
        {
#pragma unroll
            for (int nb2 = 0; nb2 < 4; ++nb2)
            {
                uint32_t b0, b1, b2, b3;
                const int key = nb2 * 16 + r8 + (mat >> 1) * 8;
                const int chunk = kk * 2 + (mat & 1);
                ldsm_x4(static_cast<uint32_t>(__cvta_generic_to_shared(kt + swz(key, chunk))), b0, b1, b2, b3);
                mma_bf16(s[2 * nb2], qf[kk], b0, b1);
                mma_bf16(s[2 * nb2 + 1], qf[kk], b2, b3);
            }
        }
        // scale, mask, online softmax (rows g and g + 8 of this warp's 16)
        const int key0 = j * kKTile;
        float tile_max[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int nb = 0; nb < 8; ++nb)
#pragma unroll
            for (int e = 0; e < 4; ++e)
            {
                const int key = key0 + nb * 8 + 2 * t + (e & 1);
                float x = s[nb][e] * kScaleLog2;
                if (key >= kv_len) x = -INFINITY;
                else if (mask) x += __ldg(mask + key) * kLog2e;
                s[nb][e] = x;
                tile_max[e >> 1] = fmaxf(tile_max[e >> 1], x);
            }
        float alpha[2];
#pragma unroll
        for (int r = 0; r < 2; ++r)
        {
            tile_max[r] = fmaxf(tile_max[r], __shfl_xor_sync(0xffffffffu, tile_max[r], 1));
            tile_max[r] = fmaxf(tile_max[r], __shfl_xor_sync(0xffffffffu, tile_max[r], 2));
            const float m_new = fmaxf(m_run[r], tile_max[r]);
            const float m_use = m_new == -INFINITY ? 0.f : m_new;
            alpha[r] = exp2f(m_run[r] - m_use);
            m_run[r] = m_new;
            tile_max[r] = m_use;
        }
        float row_sum[2] = {0.f, 0.f};
#pragma unroll
        for (int nb = 0; nb < 8; ++nb)
#pragma unroll
            for (int e = 0; e < 4; ++e)
            {
                const float p = exp2f(s[nb][e] - tile_max[e >> 1]);
                s[nb][e] = p;
                row_sum[e >> 1] += p;
            }
#pragma unroll
        for (int r = 0; r < 2; ++r) l_run[r] = l_run[r] * alpha[r] + row_sum[r];
#pragma unroll
        for (int nd = 0; nd < 16; ++nd)
        {
            o[nd][0] *= alpha[0];
            o[nd][1] *= alpha[0];
            o[nd][2] *= alpha[1];
            o[nd][3] *= alpha[1];
        }
        // O += P V
#pragma unroll
        for (int kk2 = 0; kk2 < 4; ++kk2)
        {
            uint32_t pa[4];
            pa[0] = pack_bf16(s[2 * kk2][0], s[2 * kk2][1]);
            pa[1] = pack_bf16(s[2 * kk2][2], s[2 * kk2][3]);
            pa[2] = pack_bf16(s[2 * kk2 + 1][0], s[2 * kk2 + 1][1]);
            pa[3] = pack_bf16(s[2 * kk2 + 1][2], s[2 * kk2 + 1][3]);
#pragma unroll
            for (int nd2 = 0; nd2 < 8; ++nd2)
            {
                uint32_t b0, b1, b2, b3;
                const int key = kk2 * 16 + r8 + (mat & 1) * 8;
                const int chunk = nd2 * 2 + (mat >> 1);
                ldsm_x4_t(static_cast<uint32_t>(__cvta_generic_to_shared(vt + swz(key, chunk))), b0, b1, b2, b3);
                mma_bf16(o[2 * nd2], pa, b0, b1);
                mma_bf16(o[2 * nd2 + 1], pa, b2, b3);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int r = 0; r < 2; ++r)
    {
        l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
        l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
        l_run[r] = 1.f / l_run[r];
    }
    const size_t ld = static_cast<size_t>(heads) * kDim;
#pragma unroll
    for (int r = 0; r < 2; ++r)
    {
        const int row = q0 + warp * 16 + g + r * 8;
        if (row >= rows) continue;
        __nv_bfloat16 *dst = out + static_cast<size_t>(row) * ld + head * kDim + 2 * t;
#pragma unroll
        for (int nd = 0; nd < 16; ++nd)
            *reinterpret_cast<__nv_bfloat162 *>(dst + nd * 8) =
                __floats2bfloat162_rn(o[nd][2 * r] * l_run[r], o[nd][2 * r + 1] * l_run[r]);
    }
}

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
    const int kv_head = a.kv_heads == 1 ? 0 : head;
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
    const int tiles = (a.kv_len + kFK - 1) / kFK;
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
            float x = key < a.kv_len ? dot * scale + (mrow ? mrow[key] : 0.f) : -INFINITY;
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
    cudaError_t e = cudaFuncSetAttribute(attention_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attention_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kFSmem);
    return e;
}

int launch_attention_bf16(const __nv_bfloat16 *q, const __nv_bfloat16 *k, const __nv_bfloat16 *v, const float *mask,
                          int rows, int rows_pad, int kv_len, int heads, __nv_bfloat16 *out, cudaStream_t stream)
{
    if (rows < 1 || kv_len < 1 || kv_len > rows_pad || rows_pad % kQTile || rows > rows_pad || heads < 1)
        return cudaErrorInvalidValue;
    const dim3 grid((rows + kQTile - 1) / kQTile, heads);
    attention_bf16_kernel<<<grid, kAttnThreads, kAttnSmem, stream>>>(q, k, v, mask, rows, rows_pad, kv_len, heads, out);
    return cudaGetLastError();
}

int launch_attention_f32(const AttentionF32Args &args, cudaStream_t stream)
{
    if (args.nq < 1 || args.nk < 1 || args.kv_len < 1 || args.kv_len > args.nk || args.width < 1 ||
        args.width > kDim || args.heads < 1 || (args.kv_heads != 1 && args.kv_heads != args.heads) ||
        (args.mask && args.mask_heads != 1 && args.mask_heads != args.heads) ||
        (args.mask && args.mask_rows != 1 && args.mask_rows != args.nq))
        return cudaErrorInvalidValue;
    const dim3 grid((args.nq + kFQ - 1) / kFQ, args.heads);
    attention_f32_kernel<<<grid, kFThreads, kFSmem, stream>>>(args);
    return cudaGetLastError();
}
} // namespace ernie_b200
