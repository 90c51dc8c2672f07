// tcgen05 flash attention for the ERNIE DiT block (BF16 mode).
//
// Replaces sdpa_22 (block.ncnn.param:58; ErnieSDPA / AccurateSDPA, src/ernie_attention.cpp:35-233):
// softmax(Q K^T / sqrt(128) + mask_row) V per head over the joint image+text sequence, non-causal,
// keys past the valid count (the -1e30 text padding of src/conditioning.cpp:41-42) skipped.
//
// One CTA = one head x 128 queries; KV tiles of 128 keys.
//   warp 0      TMA producer: Q once, then K and V^T tiles through a 2-stage ring
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer:
//                 S_j = Q K_j^T   (M=128, N=128, K=128) into one of two TMEM S buffers
//                 O  += P_j V_j   (M=128, N=128 dims, K=128 keys) into the TMEM O accumulator
//   warps 2..5  softmax, one query row per thread: tcgen05.ld of S_j, online max/sum in FP32,
//               P_j written as BF16 into one of two 128-byte-swizzled shared tiles (the K-major
//               A operand of the next MMA), final O / l. The running max is only raised (and O in
//               TMEM rescaled) when a tile's max exceeds it by more than 2^8; between raises the
//               stale max is exact because O and l share it, and P stays <= 256.
// Issue order S_0, S_1, PV_0, S_2, PV_1, S_3, ... lets S_{j+1} run while softmax works on S_j,
// and the two P buffers let softmax j+1 write while PV_j is still executing.
// V is stored transposed ([head][dim][token], written by the QKV GEMM epilogue) so both MMAs use
// K-major operands. All mbarrier waits are bounded. Every TMA load fills this CTA's own shared memory.
#include "kernels.h"
#include "ptx.cuh"
#include <cudaTypedefs.h>
#include <mutex>

namespace ernie_b200
{
namespace
{
constexpr int kThreads = 192;
constexpr int kTile = 128;                   // queries per CTA, keys per KV tile, head dim
constexpr int kHalfBytes = kTile * 64 * 2;   // one 64-column half of a 128 x 128 BF16 tile
constexpr int kTileBytes = 2 * kHalfBytes;   // 32 KB
constexpr int kSmemBytes = 7 * kTileBytes + 1024 + 256; // Q, 2 K, 2 V^T, 2 P tiles
constexpr int kTmemCols = 512;               // S buffers at columns 0 and 128, O at 256

enum FlashError : int
{
    kErrFlashProducerTimeout = 11,
    kErrFlashMmaTimeout = 12,
    kErrFlashSoftmaxTimeout = 13,
};

struct FlashArgs
{
    int rows, rows_pad, kv_len;
    const float *mask;
    FlashOutput out;
    int *error_flag;
};

__device__ __forceinline__ float fast_exp2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d)
{
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi)
{
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

__global__ void __launch_bounds__(kThreads, 1)
    flash_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                    const __grid_constant__ CUtensorMap map_vt, FlashArgs a)
{
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *base_ptr = smem_raw + (base - raw);
    const uint32_t s_q = base;
    auto s_k = [&](int s) { return base + (1 + s) * kTileBytes; };
    auto s_v = [&](int s) { return base + (3 + s) * kTileBytes; };
    auto s_p = [&](int b) { return base + (5 + b) * kTileBytes; };
    const uint32_t bars = base + 7 * kTileBytes;
    const uint32_t q_full = bars;
    auto k_full = [&](int s) { return bars + 8u * (1 + s); };
    auto k_empty = [&](int s) { return bars + 8u * (3 + s); };
    auto v_full = [&](int s) { return bars + 8u * (5 + s); };
    auto v_empty = [&](int s) { return bars + 8u * (7 + s); };
    auto s_full = [&](int s) { return bars + 8u * (9 + s); };
    auto p_full = [&](int b) { return bars + 8u * (11 + b); };
    auto p_empty = [&](int b) { return bars + 8u * (13 + b); };
    const uint32_t slot = bars + 8u * 15;

    const int head = blockIdx.y, q0 = blockIdx.x * kTile;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int tiles = (a.kv_len + kTile - 1) / kTile;

    if (threadIdx.x == 0)
    {
        mbar_init(q_full, 1);
        for (int s = 0; s < 2; ++s)
        {
            mbar_init(k_full(s), 1);
            mbar_init(k_empty(s), 1);
            mbar_init(v_full(s), 1);
            mbar_init(v_empty(s), 1);
            mbar_init(s_full(s), 1);
            mbar_init(p_full(s), 4);
            mbar_init(p_empty(s), 1);
        }
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
    const uint32_t o_col = 256;

    if (warp == 0)
    {
        if (lane == 0)
        {
            const int row_q = head * a.rows_pad + q0;
            mbar_arrive_expect_tx(q_full, kTileBytes);
            tma_load_2d(s_q, &map_q, q_full, 0, row_q);
            tma_load_2d(s_q + kHalfBytes, &map_q, q_full, 64, row_q);
            for (int j = 0; j < tiles; ++j)
            {
                const int s = j & 1;
                const uint32_t ph = (j >> 1) & 1;
                const int row_k = head * a.rows_pad + j * kTile;
                if (!mbar_wait(k_empty(s), ph ^ 1u))
                {
                    if (a.error_flag) atomicExch(a.error_flag, kErrFlashProducerTimeout);
                    break;
                }
                mbar_arrive_expect_tx(k_full(s), kTileBytes);
                tma_load_2d(s_k(s), &map_k, k_full(s), 0, row_k);
                tma_load_2d(s_k(s) + kHalfBytes, &map_k, k_full(s), 64, row_k);
                if (!mbar_wait(v_empty(s), ph ^ 1u))
                {
                    if (a.error_flag) atomicExch(a.error_flag, kErrFlashProducerTimeout);
                    break;
                }
                mbar_arrive_expect_tx(v_full(s), kTileBytes);
                tma_load_2d(s_v(s), &map_vt, v_full(s), j * kTile, head * kTile);
                tma_load_2d(s_v(s) + kHalfBytes, &map_vt, v_full(s), j * kTile + 64, head * kTile);
            }
        }
    }
    else if (warp == 1)
    {
        if (lane == 0)
        {
            constexpr uint32_t idesc = idesc_bf16(128, 128);
            bool ok = mbar_wait(q_full, 0);
            auto issue_s = [&](int j) -> bool {
                const int s = j & 1;
                if (!mbar_wait(k_full(s), (j >> 1) & 1)) return false;
                tc_fence_after();
#pragma unroll
                for (int k = 0; k < 8; ++k)
                {
                    const uint64_t ad = smem_desc_sw128(s_q + (k >> 2) * kHalfBytes) + 2u * (k & 3);
                    const uint64_t bd = smem_desc_sw128(s_k(s) + (k >> 2) * kHalfBytes) + 2u * (k & 3);
                    umma_bf16(tmem_base + s * 128, ad, bd, idesc, k > 0 ? 1u : 0u);
                }
                umma_commit(k_empty(s));
                umma_commit(s_full(s));
                return true;
            };
            if (ok) ok = issue_s(0);
            if (ok && tiles > 1) ok = issue_s(1);
            for (int j = 0; j < tiles && ok; ++j)
            {
                const int b = j & 1;
                const uint32_t ph = (j >> 1) & 1;
                if (!mbar_wait(p_full(b), ph) || !mbar_wait(v_full(b), ph))
                {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int k = 0; k < 8; ++k)
                {
                    const uint64_t ad = smem_desc_sw128(s_p(b) + (k >> 2) * kHalfBytes) + 2u * (k & 3);
                    const uint64_t bd = smem_desc_sw128(s_v(b) + (k >> 2) * kHalfBytes) + 2u * (k & 3);
                    umma_bf16(tmem_base + o_col, ad, bd, idesc, (j > 0 || k > 0) ? 1u : 0u);
                }
                umma_commit(v_empty(b));
                umma_commit(p_empty(b));
                if (j + 2 < tiles) ok = issue_s(j + 2);
            }
            if (!ok && a.error_flag) atomicExch(a.error_flag, kErrFlashMmaTimeout);
        }
    }
    else
    {
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane; // row within the query tile == TMEM lane
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        // scores stay in raw units; c folds 1/sqrt(128) and log2(e) into one FFMA per element
        constexpr float c = 0.08838834764831845f * 1.4426950408889634f;
        constexpr float kMaskToRaw = 11.313708498984761f; // log2(e)/c = sqrt(128)
        constexpr float kRescaleLog2 = 8.f;              // rescale O only when the max grows by 2^8
        float m_run = -INFINITY, l_run = 0.f;
        int waited0 = 0, waited1 = 0; // completions of p_empty[0] / p_empty[1] already observed
        bool ok = true;
        auto wait_pv = [&](int i) -> bool { // PV_i complete
            const int b = i & 1, k = i >> 1;
            int &waited = b ? waited1 : waited0;
            if (waited > k) return true;
            if (!mbar_wait(p_empty(b), k & 1)) return false;
            waited = k + 1;
            return true;
        };
        for (int j = 0; j < tiles && ok; ++j)
        {
            const int b = j & 1;
            if (!mbar_wait(s_full(b), (j >> 1) & 1))
            {
                ok = false;
                break;
            }
            tc_fence_after();
            float x[128];
            tmem_load_128(lane_base + b * 128, x);
            const int key0 = j * kTile;
            if (a.mask)
            {
#pragma unroll
                for (int k = 0; k < 128; ++k)
                    if (key0 + k < a.kv_len) x[k] = fmaf(__ldg(a.mask + key0 + k), kMaskToRaw, x[k]);
            }
            if (key0 + kTile > a.kv_len)
            {
#pragma unroll
                for (int k = 0; k < 128; ++k)
                    if (key0 + k >= a.kv_len) x[k] = -INFINITY;
            }
            float tmax = x[0];
#pragma unroll
            for (int k = 1; k < 128; ++k) tmax = fmaxf(tmax, x[k]);
            if (j == 0) m_run = tmax;
            else if (__any_sync(0xffffffffu, (tmax - m_run) * c > kRescaleLog2))
            {
                // the O rescale must land between PV_{j-1} and PV_j
                const float m_new = fmaxf(m_run, tmax);
                const float alpha = fast_exp2((m_run - m_new) * c);
                if (!wait_pv(j - 1))
                {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int cc = 0; cc < 4; ++cc)
                {
                    float o[32];
                    tmem_load_32(lane_base + o_col + cc * 32, o);
#pragma unroll
                    for (int t = 0; t < 32; ++t) o[t] *= alpha;
                    tmem_store_32(lane_base + o_col + cc * 32, o);
                }
                tmem_store_wait();
                l_run *= alpha;
                m_run = m_new;
            }
            const float neg = -m_run * c;
            float row_sum = 0.f;
#pragma unroll
            for (int k = 0; k < 128; ++k)
            {
                x[k] = fast_exp2(fmaf(x[k], c, neg));
                row_sum += x[k];
            }
            l_run += row_sum;
            // P buffer b is free once PV_{j-2} has consumed it
            if (j >= 2 && !wait_pv(j - 2))
            {
                ok = false;
                break;
            }
            // P row r as BF16 into the swizzled K-major tile: half h holds keys 64h..64h+63,
            // 16-byte chunk cc of row r sits at chunk cc ^ (r & 7).
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int cc = 0; cc < 8; ++cc)
                {
                    const float *v = x + h * 64 + cc * 8;
                    const uint32_t addr = s_p(b) + h * kHalfBytes + r * 128 + ((cc ^ (r & 7)) << 4);
                    st_shared_v4(addr, pack2(v[0], v[1]), pack2(v[2], v[3]), pack2(v[4], v[5]), pack2(v[6], v[7]));
                }
            fence_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full(b));
        }
        if (ok && !wait_pv(tiles - 1)) ok = false;
        if (!ok)
        {
            if (a.error_flag && lane == 0) atomicExch(a.error_flag, kErrFlashSoftmaxTimeout);
        }
        else
        {
            tc_fence_after();
            const int row = q0 + r;
            const float inv = 1.f / l_run;
            // output row `row` belongs to destination row / rows_per_dest (its owner GPU in a
            // sequence-parallel group; destination 0 on one GPU)
            const int dest = row / a.out.rows_per_dest, dest_row = row - dest * a.out.rows_per_dest;
            __nv_bfloat16 *dst_base = nullptr;
#pragma unroll
            for (int d = 0; d < kMaxDest; ++d)
                if (d == dest) dst_base = a.out.dst[d];
            __nv_bfloat16 *dst = dst_base + static_cast<size_t>(dest_row) * a.out.ld + a.out.col_offset + head * kTile;
#pragma unroll
            for (int cc = 0; cc < 4; ++cc)
            {
                float o[32];
                tmem_load_32(lane_base + o_col + cc * 32, o);
                if (row < a.rows)
                {
#pragma unroll
                    for (int t = 0; t < 32; t += 8)
                    {
                        uint4 packed;
                        packed.x = pack2(o[t] * inv, o[t + 1] * inv);
                        packed.y = pack2(o[t + 2] * inv, o[t + 3] * inv);
                        packed.z = pack2(o[t + 4] * inv, o[t + 5] * inv);
                        packed.w = pack2(o[t + 6] * inv, o[t + 7] * inv);
                        *reinterpret_cast<uint4 *>(dst + cc * 32 + t) = packed;
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

bool map_2d(CUtensorMap *map, const void *ptr, uint64_t rows, uint64_t cols)
{
    auto fn = encode_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(ptr) & 15u) || (cols * 2) % 16) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {64, 128};
    const cuuint32_t element_strides[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, element_strides,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
} // namespace

int prepare_flash_kernels()
{
    return cudaFuncSetAttribute(flash_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
}

int launch_flash_tc(const __nv_bfloat16 *q, const __nv_bfloat16 *k, const __nv_bfloat16 *vt, const float *mask,
                    int rows, int rows_pad, int kv_len, int heads, const FlashOutput &out, int *error_flag,
                    cudaStream_t stream)
{
    if (rows < 1 || kv_len < 1 || kv_len > rows_pad || rows_pad % kTile || rows > rows_pad || heads < 1 ||
        out.rows_per_dest < 1 || out.ld % 8 || out.col_offset % 8 || out.col_offset + heads * kTile > out.ld)
        return cudaErrorInvalidValue;
    for (int d = 0; d < (rows + out.rows_per_dest - 1) / out.rows_per_dest; ++d)
        if (d >= kMaxDest || !out.dst[d]) return cudaErrorInvalidValue;
    CUtensorMap mq, mk, mv;
    if (!map_2d(&mq, q, static_cast<uint64_t>(heads) * rows_pad, kTile) ||
        !map_2d(&mk, k, static_cast<uint64_t>(heads) * rows_pad, kTile) ||
        !map_2d(&mv, vt, static_cast<uint64_t>(heads) * kTile, static_cast<uint64_t>(rows_pad)))
        return cudaErrorInvalidValue;
    FlashArgs a{rows, rows_pad, kv_len, mask, out, error_flag};
    const dim3 grid((rows + kTile - 1) / kTile, heads);
    flash_tc_kernel<<<grid, kThreads, kSmemBytes, stream>>>(mq, mk, mv, a);
    return cudaGetLastError();
}

int launch_flash_tc(const __nv_bfloat16 *q, const __nv_bfloat16 *k, const __nv_bfloat16 *vt, const float *mask,
                    int rows, int rows_pad, int kv_len, int heads, __nv_bfloat16 *out, int *error_flag,
                    cudaStream_t stream)
{
    FlashOutput o;
    o.dst[0] = out;
    o.rows_per_dest = rows;
    o.ld = heads * kTile;
    o.col_offset = 0;
    return launch_flash_tc(q, k, vt, mask, rows, rows_pad, kv_len, heads, o, error_flag, stream);
}
} // namespace ernie_b200
