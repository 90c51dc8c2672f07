// FP32-exact attention on the tensor cores (the session's FP32 mode).
//
// Replaces sdpa_22 (block.ncnn.param:58; AccurateSDPA, src/ernie_attention.cpp:35-233) in FP32 mode:
// softmax(Q K^T / sqrt(128) + mask_row) V with FP32-level accuracy. Q, K and V^T arrive from the QKV
// epilogue as three BF16 planes each (x = hi + mid + lo to 24 significant bits), so every product of
// planes is exact on the tensor core:
//   S  = sum over the plane pairs (a, b) with a + b <= 2 of Q_a K_b^T  (6 MMAs of K = 128; the dropped
//        pairs are below 2^-24 of |Q||K|), computed per KV tile of 64 keys into TMEM;
//   p  = expf(S / sqrt(128) + mask - m) in FP32, as the FP32 SIMT path computes it, row sums in FP64;
//   O_j = sum over (a, b), a + b <= 2, of P_a V_b (P split into three BF16 planes in TMEM) into a fresh
//        TMEM accumulator per KV tile: no tensor-core accumulation chain is longer than 6 x 64 products
//        (chain error grows with its length), and the softmax warps add the tiles' O_j into an FP32 sum
//        in TMEM with the online-softmax rescale.
// One CTA = one head x 128 queries, 224 threads:
//   warp 0  TMA producer of Q (once) and K planes (one 64-key tile at a time)
//   warp 1  TMEM allocator + single-thread tcgen05.mma issuer: S(j+1) as soon as softmax has copied S(j)
//           out of TMEM, PV(j) once P(j) is in TMEM
//   warp 2  TMA producer of the V^T planes
//   warps 3..6  softmax, one query row per thread (TMEM lane = row)
// TMEM (512 columns): S [0,64), P planes [64,160) (32 columns of BF16 pairs each), O_j [256,384), the
// running FP32 sum of the O_j [384,512).
// All mbarrier waits are bounded. Every TMA load fills this CTA's own shared memory.
#include "kernels.h"
#include "ptx.cuh"
#include <cudaTypedefs.h>
#include <mutex>

namespace ernie_b200
{
namespace
{
constexpr int kThreads = 224;
constexpr int kRows = 128, kDim = 128, kKeys = 64, kPlanes = 3;
constexpr int kQHalf = kRows * 64 * 2;          // 64 dims of a 128-row plane: 16 KB
constexpr int kQPlane = 2 * kQHalf;             // 32 KB
constexpr int kKHalf = kKeys * 64 * 2;          // 64 dims of a 64-key plane: 8 KB
constexpr int kKPlane = 2 * kKHalf;             // 16 KB
constexpr int kVPlane = kDim * kKeys * 2;       // V^T: 128 dims x 64 keys, 16 KB
constexpr int kSmemBytes = kPlanes * (kQPlane + kKPlane + kVPlane) + 1024 + 256;
constexpr int kTmemCols = 512;
constexpr uint32_t kColS = 0, kColP = 64, kColO = 256, kColAcc = 384;
// plane pairs whose products reach FP32 precision: (hi,hi) (hi,mid) (mid,hi) (hi,lo) (lo,hi) (mid,mid)
__constant__ int kPairA[6] = {0, 0, 1, 0, 2, 1};
__constant__ int kPairB[6] = {0, 1, 0, 2, 0, 1};

enum : int
{
    kErrF32Producer = 31,
    kErrF32Mma = 32,
    kErrF32Softmax = 33,
};

struct F32Args
{
    int rows, rows_pad, kv_len, heads;
    const float *mask;
    __nv_bfloat16 *out; // token-major [rows][3 * heads * 128]: hi, mid, lo planes of the output
    int *error_flag;
};

__device__ __forceinline__ void split3(float x, __nv_bfloat16 &hi, __nv_bfloat16 &mid, __nv_bfloat16 &lo)
{
    hi = __float2bfloat16_rn(x);
    const float r1 = x - __bfloat162float(hi);
    mid = __float2bfloat16_rn(r1);
    lo = __float2bfloat16_rn(r1 - __bfloat162float(mid));
}

__device__ __forceinline__ float plane_of(float x, int p)
{
    __nv_bfloat16 h, m, l;
    split3(x, h, m, l);
    return __bfloat162float(p == 0 ? h : p == 1 ? m : l);
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi)
{
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ void umma_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate)
{
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
                 "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
                 : "memory");
}

__device__ __forceinline__ void tmem_store_32u(uint32_t taddr, const uint32_t *v)
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
                 "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
                 "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
                 "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
                 "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
                 "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
                 "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
                 : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    flash_f32_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                     const __grid_constant__ CUtensorMap map_vt, F32Args a)
{
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *base_ptr = smem_raw + (base - raw);
    auto s_q = [&](int p) { return base + p * kQPlane; };
    auto s_k = [&](int p) { return base + kPlanes * kQPlane + p * kKPlane; };
    auto s_v = [&](int p) { return base + kPlanes * (kQPlane + kKPlane) + p * kVPlane; };
    const uint32_t bars = base + kPlanes * (kQPlane + kKPlane + kVPlane);
    const uint32_t q_full = bars, k_full = bars + 8, k_empty = bars + 16, v_full = bars + 24, v_empty = bars + 32,
                   s_full = bars + 40, s_free = bars + 48, p_full = bars + 56, pv_done = bars + 64;
    const uint32_t slot = bars + 72;

    const int head = blockIdx.y, q0 = blockIdx.x * kRows;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int tiles = (a.kv_len + kKeys - 1) / kKeys;

    if (threadIdx.x == 0)
    {
        mbar_init(q_full, 1);
        mbar_init(k_full, 1);
        mbar_init(k_empty, 1);
        mbar_init(v_full, 1);
        mbar_init(v_empty, 1);
        mbar_init(s_full, 1);
        mbar_init(s_free, 4);
        mbar_init(p_full, 4);
        mbar_init(pv_done, 1);
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0)
    {
        prefetch_tensormap(&map_q);
        prefetch_tensormap(&map_k);
        prefetch_tensormap(&map_vt);
    }
    if (warp == 1)
    {
        tmem_alloc(slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t *>(base_ptr + (slot - base));

    if (warp == 0)
    {
        if (lane == 0)
        {
            mbar_arrive_expect_tx(q_full, kPlanes * kQPlane);
            for (int p = 0; p < kPlanes; ++p)
            {
                const int row = (p * a.heads + head) * a.rows_pad + q0;
                tma_load_2d(s_q(p), &map_q, q_full, 0, row);
                tma_load_2d(s_q(p) + kQHalf, &map_q, q_full, 64, row);
            }
            for (int j = 0; j < tiles; ++j)
            {
                if (!mbar_wait(k_empty, (j & 1) ^ 1u))
                {
                    if (a.error_flag) atomicExch(a.error_flag, kErrF32Producer);
                    break;
                }
                mbar_arrive_expect_tx(k_full, kPlanes * kKPlane);
                for (int p = 0; p < kPlanes; ++p)
                {
                    const int row = (p * a.heads + head) * a.rows_pad + j * kKeys;
                    tma_load_2d(s_k(p), &map_k, k_full, 0, row);
                    tma_load_2d(s_k(p) + kKHalf, &map_k, k_full, 64, row);
                }
            }
        }
    }
    else if (warp == 2)
    {
        if (lane == 0)
        {
            for (int j = 0; j < tiles; ++j)
            {
                if (!mbar_wait(v_empty, (j & 1) ^ 1u))
                {
                    if (a.error_flag) atomicExch(a.error_flag, kErrF32Producer);
                    break;
                }
                mbar_arrive_expect_tx(v_full, kPlanes * kVPlane);
                for (int p = 0; p < kPlanes; ++p)
                    tma_load_2d(s_v(p), &map_vt, v_full, j * kKeys, (p * a.heads + head) * kDim);
            }
        }
    }
    else if (warp == 1)
    {
        if (lane == 0)
        {
            constexpr uint32_t idesc_s = idesc_bf16(kRows, kKeys), idesc_pv = idesc_bf16(kRows, kDim);
            bool ok = mbar_wait(q_full, 0);
            auto issue_s = [&]() {
#pragma unroll 1
                for (int c = 0; c < 6; ++c)
                {
                    const int pa = kPairA[c], pb = kPairB[c];
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                    {
                        const uint64_t ad = smem_desc_sw128(s_q(pa) + (k >> 2) * kQHalf) + 2u * (k & 3);
                        const uint64_t bd = smem_desc_sw128(s_k(pb) + (k >> 2) * kKHalf) + 2u * (k & 3);
                        umma_bf16(tmem_base + kColS, ad, bd, idesc_s, (c > 0 || k > 0) ? 1u : 0u);
                    }
                }
                umma_commit(s_full);
                umma_commit(k_empty);
            };
            if (ok && (ok = mbar_wait(k_full, 0)))
            {
                tc_fence_after();
                issue_s();
            }
            for (int j = 0; j < tiles && ok; ++j)
            {
                if (j + 1 < tiles)
                {
                    if (!mbar_wait(s_free, j & 1) || !mbar_wait(k_full, (j + 1) & 1))
                    {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    issue_s();
                }
                if (!mbar_wait(p_full, j & 1) || !mbar_wait(v_full, j & 1))
                {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll 1
                for (int c = 0; c < 6; ++c)
                {
                    const int pa = kPairA[c], pb = kPairB[c];
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        umma_tmem_a(tmem_base + kColO, tmem_base + kColP + pa * 32 + 8u * k,
                                    smem_desc_sw128(s_v(pb)) + 2u * k, idesc_pv, (c > 0 || k > 0) ? 1u : 0u);
                }
                umma_commit(pv_done);
                umma_commit(v_empty);
            }
            if (!ok && a.error_flag) atomicExch(a.error_flag, kErrF32Mma);
        }
    }
    else
    {
        const int quarter = warp & 3;      // TMEM lane quarter this warp may access
        const int r = quarter * 32 + lane; // query row within the tile == TMEM lane
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        const float scale = 1.f / sqrtf(static_cast<float>(kDim));
        float m_run = -INFINITY;
        double l_run = 0.0;
        bool ok = true;
        for (int j = 0; j < tiles && ok; ++j)
        {
            if (!mbar_wait(s_full, j & 1))
            {
                ok = false;
                break;
            }
            tc_fence_after();
            float x[kKeys];
            tmem_load_32(lane_base + kColS, *reinterpret_cast<float(*)[32]>(x));
            tmem_load_32(lane_base + kColS + 32, *reinterpret_cast<float(*)[32]>(x + 32));
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free); // the MMA warp may compute S(j+1) now
            const int key0 = j * kKeys;
            float tmax = -INFINITY;
#pragma unroll
            for (int k = 0; k < kKeys; ++k)
            {
                const int key = key0 + k;
                x[k] = key < a.kv_len ? x[k] * scale + (a.mask ? __ldg(a.mask + key) : 0.f) : -INFINITY;
                tmax = fmaxf(tmax, x[k]);
            }
            const float m_new = fmaxf(m_run, tmax);
            const float m_use = m_new == -INFINITY ? 0.f : m_new;
            const float alpha = expf(m_run - m_use);
            float psum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int k = 0; k < kKeys; ++k)
            {
                x[k] = expf(x[k] - m_use);
                psum[k & 3] += x[k];
            }
            l_run = l_run * static_cast<double>(alpha) +
                    (static_cast<double>(psum[0]) + psum[1] + static_cast<double>(psum[2]) + psum[3]);
            m_run = m_new;
            // O(j-1) is complete and the P planes are free: fold O(j-1) into the running sum, rescaled
            // to the new max (the sum held the tiles before j-1 relative to the previous max)
            if (j > 0)
            {
                if (!mbar_wait(pv_done, (j - 1) & 1))
                {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll 1
                for (int cc = 0; cc < 4; ++cc)
                {
                    float o[32], acc[32];
                    tmem_load_32(lane_base + kColO + cc * 32, o);
                    if (j > 1)
                        tmem_load_32(lane_base + kColAcc + cc * 32, acc);
                    else
#pragma unroll
                        for (int t = 0; t < 32; ++t) acc[t] = 0.f;
#pragma unroll
                    for (int t = 0; t < 32; ++t) acc[t] = (acc[t] + o[t]) * alpha;
                    tmem_store_32(lane_base + kColAcc + cc * 32, acc);
                }
            }
#pragma unroll 1
            for (int p = 0; p < kPlanes; ++p)
            {
                uint32_t pk[32];
#pragma unroll
                for (int k = 0; k < kKeys; k += 2) pk[k / 2] = pack2(plane_of(x[k], p), plane_of(x[k + 1], p));
                tmem_store_32u(lane_base + kColP + p * 32, pk);
                tmem_store_wait();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
        }
        if (ok && !mbar_wait(pv_done, (tiles - 1) & 1)) ok = false;
        if (!ok)
        {
            if (a.error_flag && lane == 0) atomicExch(a.error_flag, kErrF32Softmax);
        }
        else
        {
            tc_fence_after();
            const int row = q0 + r;
            const size_t plane = static_cast<size_t>(a.heads) * kDim;
            __nv_bfloat16 *dst = a.out + static_cast<size_t>(row) * 3 * plane + static_cast<size_t>(head) * kDim;
            const double inv = 1.0 / l_run;
#pragma unroll 1
            for (int cc = 0; cc < 4; ++cc)
            {
                float o[32], acc[32];
                tmem_load_32(lane_base + kColO + cc * 32, o);
                if (tiles > 1)
                    tmem_load_32(lane_base + kColAcc + cc * 32, acc);
                else
#pragma unroll
                    for (int t = 0; t < 32; ++t) acc[t] = 0.f;
                if (row < a.rows)
                {
#pragma unroll
                    for (int t = 0; t < 32; t += 8)
                    {
                        __align__(16) __nv_bfloat16 h[8], m[8], l[8];
#pragma unroll
                        for (int u = 0; u < 8; ++u)
                            split3(static_cast<float>(static_cast<double>(acc[t + u] + o[t + u]) * inv), h[u], m[u],
                                   l[u]);
                        const int d = cc * 32 + t;
                        *reinterpret_cast<uint4 *>(dst + d) = *reinterpret_cast<const uint4 *>(h);
                        *reinterpret_cast<uint4 *>(dst + plane + d) = *reinterpret_cast<const uint4 *>(m);
                        *reinterpret_cast<uint4 *>(dst + 2 * plane + d) = *reinterpret_cast<const uint4 *>(l);
                    }
                }
            }
        }
    }
    __syncthreads();
    if (warp == 1)
    {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

bool map_2d(CUtensorMap *map, const void *ptr, uint64_t rows, uint64_t cols, uint32_t box_rows)
{
    auto fn = encode_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(ptr) & 15u) || (cols * 2) % 16) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t element_strides[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, element_strides,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
} // namespace

int prepare_flash_f32_kernels()
{
    return cudaFuncSetAttribute(flash_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
}

int launch_flash_f32(const __nv_bfloat16 *q3, const __nv_bfloat16 *k3, const __nv_bfloat16 *vt3, const float *mask,
                     int rows, int rows_pad, int kv_len, int heads, __nv_bfloat16 *out_split3, int *error_flag,
                     cudaStream_t stream)
{
    if (rows < 1 || kv_len < 1 || kv_len > rows_pad || rows_pad % kRows || rows > rows_pad || heads < 1 || !out_split3)
        return cudaErrorInvalidValue;
    CUtensorMap mq, mk, mv;
    const uint64_t plane_rows = static_cast<uint64_t>(kPlanes) * heads * rows_pad;
    if (!map_2d(&mq, q3, plane_rows, kDim, kRows) || !map_2d(&mk, k3, plane_rows, kDim, kKeys) ||
        !map_2d(&mv, vt3, static_cast<uint64_t>(kPlanes) * heads * kDim, static_cast<uint64_t>(rows_pad), kDim))
        return cudaErrorInvalidValue;
    F32Args a{rows, rows_pad, kv_len, heads, mask, out_split3, error_flag};
    const dim3 grid((rows + kRows - 1) / kRows, heads);
    flash_f32_kernel<<<grid, kThreads, kSmemBytes, stream>>>(mq, mk, mv, a);
    return cudaGetLastError();
}
} // namespace ernie_b200
