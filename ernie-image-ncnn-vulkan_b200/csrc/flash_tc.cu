// tcgen05 flash attention for the ERNIE DiT block (BF16 mode).
//
// Replaces sdpa_22 (block.ncnn.param:58; ErnieSDPA / AccurateSDPA, src/ernie_attention.cpp:35-233):
// softmax(Q K^T / sqrt(128) + mask_row) V per head over the joint image+text sequence, non-causal
// (the prompt encoder's causal grouped-query attention uses the same kernel with `causal` and `kv_group`),
// keys past the valid count (the -1e30 text padding of src/conditioning.cpp:41-42) skipped.
//
// One CTA = one head x 256 queries as two 128-row query tiles A and B that share every K / V^T tile;
// KV tiles of 128 keys. TMEM (512 columns): S_A, S_B, O_A, O_B, 128 columns each. Softmax copies S_g
// into registers and frees it at once, so S_g(j+1) is computed while softmax works on S_g(j); P_g goes
// to a 128-byte-swizzled shared tile (the K-major A operand of the PV MMA). Each softmax warpgroup
// therefore runs tile after tile without waiting for its own PV and next S, and the two groups keep
// the MUFU (16 ex2 per clock per SM, as many per tile as the tensor core's cycles) and the tensor core
// busy together.
//   warp 0      TMA producer of Q_A, Q_B (once) and the K tiles (2-stage ring)
//   warp 2      TMA producer of the V^T tiles (one buffer, refilled once both PVs have read it)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer, per KV tile j:
//                 S_A(j+1), S_B(j+1) (each once softmax has freed S_g(j)), PV_A(j), PV_B(j)
//   warp 3      idle (warpgroup 0 hands its registers to the softmax warpgroups)
//   warps 4..7  softmax of tile A, warps 8..11 softmax of tile B; one query row per thread:
//               tcgen05.ld of S_g(j), online max/sum in FP32 (8 max chains, packed FP32x2 FFMA/FADD),
//               ex2 on the MUFU, P_g(j) as BF16 into its shared tile once PV_g(j-1) has read the
//               previous one, final O / l. The running max is only raised (and O_g rescaled in TMEM,
//               after PV_g(j-1)) when a tile's max exceeds it by more than 2^8; between raises the
//               stale max is exact because O and l share it.
// V is stored transposed ([head][dim][token], written by the QKV GEMM epilogue) so both MMAs use
// K-major operands. All mbarrier waits are bounded. Every TMA load fills this CTA's own shared memory.
#include "kernels.h"
#include "ptx.cuh"
#include "peer_sync.cuh"
#include <cudaTypedefs.h>
#include <mutex>

namespace ernie_b200
{
namespace
{
constexpr int kThreads = 384;               // three warpgroups (register reallocation is per warpgroup)
// Registers per thread after setmaxnreg: warpgroup 0 (producers, MMA, one idle warp) gives registers
// to the two softmax warpgroups. 128 x 88 + 256 x 208 = 64512 = 384 x 168, so the launch must have
// 168 registers per thread, which ptxas assigns at 384 threads; the host refuses to launch otherwise
// (an increase the block cannot satisfy would wait).
constexpr int kRegsControl = 88, kRegsSoftmax = 208, kMinLaunchRegs = 168;
static_assert(128 * kRegsControl + 256 * kRegsSoftmax <= kThreads * kMinLaunchRegs, "register split");
constexpr int kTile = 128;                   // queries per tile, keys per KV tile, head dim
constexpr int kRowsPerCta = 2 * kTile;       // two query tiles
constexpr int kHalfBytes = kTile * 64 * 2;   // one 64-column half of a 128 x 128 BF16 tile
constexpr int kTileBytes = 2 * kHalfBytes;   // 32 KB
constexpr int kSmemBytes = 7 * kTileBytes + 1024 + 256; // Q_A, Q_B, P_A, P_B, 2 K, 1 V^T
constexpr int kTmemCols = 512;               // S_A 0, S_B 128, O_A 256, O_B 384
// One-tile CTAs after all two-tile ones (a launch-order knob; 0 keeps the plain head-major order).
#ifndef ERNIE_FLASH_SHORT_LAST
#define ERNIE_FLASH_SHORT_LAST 1
#endif
constexpr bool kShortLast = ERNIE_FLASH_SHORT_LAST != 0;

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
    int causal = 0;   // key j > query i excluded; key tiles past the CTA's last query skipped
    int kv_group = 1; // query heads per K/V head (grouped-query attention)
    PeerSync sync;    // sequence parallel: wait for every member's Q/K/V rows, signal the stored output rows
};

__device__ __forceinline__ float fast_exp2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// max(a, b, c) in one instruction (the three-input form of max.f32, sm_100)
__device__ __forceinline__ float max3(float a, float b, float c)
{
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
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
    auto s_q = [&](int g) { return base + g * kTileBytes; };
    auto s_p = [&](int g) { return base + (2 + g) * kTileBytes; };
    auto s_k = [&](int s) { return base + (4 + s) * kTileBytes; };
    const uint32_t s_v = base + 6 * kTileBytes;
    const uint32_t bars = base + 7 * kTileBytes;
    const uint32_t q_full = bars;
    auto k_full = [&](int s) { return bars + 8u * (1 + s); };
    auto k_empty = [&](int s) { return bars + 8u * (3 + s); };
    const uint32_t v_full = bars + 8u * 5, v_empty = bars + 8u * 6;
    auto s_full = [&](int g) { return bars + 8u * (7 + g); };
    auto s_free = [&](int g) { return bars + 8u * (9 + g); };
    auto p_full = [&](int g) { return bars + 8u * (11 + g); };
    auto pv_done = [&](int g) { return bars + 8u * (13 + g); };
    const uint32_t tmem_done = bars + 8u * 15;
    const uint32_t slot = bars + 8u * 16;

    // CTA -> (head, query block). Non-causal: when the last query block of each head holds a single tile,
    // those short CTAs take the highest linear indices, after every two-tile CTA, so the grid's final wave
    // can consist of short CTAs only (C4: 1024 two-tile CTAs, then 32 one-tile ones). Rows are computed
    // the same way whichever CTA holds them.
    int head = blockIdx.y, qb = blockIdx.x;
    if (kShortLast && !a.causal && gridDim.x > 1 && (gridDim.x - 1) * kRowsPerCta + kTile >= a.rows)
    {
        const int full = gridDim.x - 1, linear = blockIdx.x + gridDim.x * blockIdx.y, two_tile = full * gridDim.y;
        head = linear < two_tile ? linear / full : linear - two_tile;
        qb = linear < two_tile ? linear % full : full;
    }
    const int q0 = qb * kRowsPerCta, kv_head = head / a.kv_group;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int kv_tiles = (a.kv_len + kTile - 1) / kTile;
    // causal: no key past this CTA's last query row
    const int q_end = min(a.rows, q0 + kRowsPerCta);
    const int tiles = a.causal ? min(kv_tiles, (q_end + kTile - 1) / kTile) : kv_tiles;
    // the second query tile of the last CTA of a head may hold no row at all: then only tile A runs
    const int groups = q0 + kTile < a.rows ? 2 : 1;

    if (threadIdx.x == 0)
    {
        mbar_init(q_full, 1);
        for (int s = 0; s < 2; ++s)
        {
            mbar_init(k_full(s), 1);
            mbar_init(k_empty(s), 1);
            mbar_init(s_full(s), 1);
            mbar_init(s_free(s), 4);
            mbar_init(p_full(s), 4);
            mbar_init(pv_done(s), 1);
        }
        mbar_init(v_full, 1);
        mbar_init(v_empty, 1);
        mbar_init(tmem_done, 8);
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
    grid_dependency_wait(); // the previous kernel's writes (Q, K, V^T, mask, peer flags) are visible from here
    grid_dependents_launch();
    auto s_col = [](int g) { return static_cast<uint32_t>(g * 128); };
    auto o_col = [](int g) { return static_cast<uint32_t>(256 + g * 128); };
    // Each role ends the kernel on its own: the register split differs per warpgroup, so no code
    // after the split is shared. TMEM is freed by warp 1 once all 8 softmax warps are done with it.
    if (warp < 4)
    {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
        if (warp == 0 && lane == 0)
        {
            peer_wait_all(a.sync.wait);
            const int row_q = head * a.rows_pad + q0;
            mbar_arrive_expect_tx(q_full, 2 * kTileBytes);
            for (int g = 0; g < 2; ++g)
            {
                tma_load_2d(s_q(g), &map_q, q_full, 0, row_q + g * kTile);
                tma_load_2d(s_q(g) + kHalfBytes, &map_q, q_full, 64, row_q + g * kTile);
            }
            for (int j = 0; j < tiles; ++j)
            {
                const int s = j & 1;
                const int row_k = kv_head * a.rows_pad + j * kTile;
                if (!mbar_wait(k_empty(s), ((j >> 1) & 1) ^ 1u))
                {
                    if (a.error_flag) atomicExch(a.error_flag, kErrFlashProducerTimeout);
                    break;
                }
                mbar_arrive_expect_tx(k_full(s), kTileBytes);
                tma_load_2d(s_k(s), &map_k, k_full(s), 0, row_k);
                tma_load_2d(s_k(s) + kHalfBytes, &map_k, k_full(s), 64, row_k);
            }
        }
        else if (warp == 2 && lane == 0)
        {
            peer_wait_all(a.sync.wait);
            for (int j = 0; j < tiles; ++j)
            {
                if (!mbar_wait(v_empty, (j & 1) ^ 1u))
                {
                    if (a.error_flag) atomicExch(a.error_flag, kErrFlashProducerTimeout);
                    break;
                }
                mbar_arrive_expect_tx(v_full, kTileBytes);
                tma_load_2d(s_v, &map_vt, v_full, j * kTile, kv_head * kTile);
                tma_load_2d(s_v + kHalfBytes, &map_vt, v_full, j * kTile + 64, kv_head * kTile);
            }
        }
        else if (warp == 1)
        {
            if (lane == 0)
            {
                constexpr uint32_t idesc = idesc_bf16(128, 128);
                bool ok = mbar_wait(q_full, 0);
                auto issue_s = [&](int g, int j) {
                    const int s = j & 1;
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                    {
                        const uint64_t ad = smem_desc_sw128(s_q(g) + (k >> 2) * kHalfBytes) + 2u * (k & 3);
                        const uint64_t bd = smem_desc_sw128(s_k(s) + (k >> 2) * kHalfBytes) + 2u * (k & 3);
                        umma_bf16(tmem_base + s_col(g), ad, bd, idesc, k > 0 ? 1u : 0u);
                    }
                    umma_commit(s_full(g));
                };
                auto issue_pv = [&](int g, int j) {
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                    {
                        const uint64_t ad = smem_desc_sw128(s_p(g) + (k >> 2) * kHalfBytes) + 2u * (k & 3);
                        const uint64_t bd = smem_desc_sw128(s_v + (k >> 2) * kHalfBytes) + 2u * (k & 3);
                        umma_bf16(tmem_base + o_col(g), ad, bd, idesc, (j > 0 || k > 0) ? 1u : 0u);
                    }
                    umma_commit(pv_done(g));
                };
                if (ok && (ok = mbar_wait(k_full(0), 0)))
                {
                    tc_fence_after();
                    issue_s(0, 0);
                    if (groups > 1) issue_s(1, 0);
                    umma_commit(k_empty(0));
                }
                for (int j = 0; j < tiles && ok; ++j)
                {
                    if (j + 1 < tiles)
                    {
                        // S_g(j+1) as soon as softmax g has copied S_g(j) out of TMEM
                        const int n = j + 1;
                        if (!mbar_wait(k_full(n & 1), (n >> 1) & 1))
                        {
                            ok = false;
                            break;
                        }
#pragma unroll
                        for (int g = 0; g < 2; ++g)
                        {
                            if (g >= groups || !ok) continue;
                            if (!mbar_wait(s_free(g), j & 1))
                            {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            issue_s(g, n);
                        }
                        if (!ok) break;
                        umma_commit(k_empty(n & 1));
                    }
                    if (!mbar_wait(v_full, j & 1))
                    {
                        ok = false;
                        break;
                    }
#pragma unroll
                    for (int g = 0; g < 2; ++g)
                    {
                        if (g >= groups || !ok) continue;
                        if (!mbar_wait(p_full(g), j & 1))
                        {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        issue_pv(g, j);
                    }
                    if (!ok) break;
                    umma_commit(v_empty);
                }
                if (!ok && a.error_flag) atomicExch(a.error_flag, kErrFlashMmaTimeout);
            }
            __syncwarp();
            if (!mbar_wait(tmem_done, 0) && a.error_flag && lane == 0) atomicExch(a.error_flag, kErrFlashMmaTimeout);
            tc_fence_after();
            tmem_dealloc(tmem_base, kTmemCols);
        }
    }
    else
    {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
        const int g = (warp - 4) >> 2;    // 0: tile A (warps 4..7), 1: tile B (warps 8..11)
        const bool active = g < groups;
        const int quarter = warp & 3;     // TMEM lane quarter this warp may access
        const int r = quarter * 32 + lane; // row within the query tile == TMEM lane
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        // scores stay in raw units; c folds 1/sqrt(128) and log2(e) into one FFMA per element
        constexpr float c = 0.08838834764831845f * 1.4426950408889634f;
        constexpr float kMaskToRaw = 11.313708498984761f; // log2(e)/c = sqrt(128)
        constexpr float kRescaleLog2 = 8.f;              // rescale O only when the max grows by 2^8
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        for (int j = 0; j < tiles && ok && active; ++j)
        {
            if (!mbar_wait(s_full(g), j & 1))
            {
                ok = false;
                break;
            }
            tc_fence_after();
            float x[128];
            tmem_load_128(lane_base + s_col(g), x);
            // S_g is in registers: the MMA warp may compute S_g(j+1) now
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free(g));
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
            if (a.causal)
            {
                // key0 + k visible iff k <= lim; key tile 0 holds a visible key for every row, so the running
                // max is finite before any fully masked tile
                const int lim = q0 + g * kTile + r - key0;
                if (lim < kTile - 1)
                {
#pragma unroll
                    for (int k = 0; k < 128; ++k)
                        if (k > lim) x[k] = -INFINITY;
                }
            }
            // row max over 8 independent chains, two new scores per three-input max
            float mx[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) mx[k] = x[k];
#pragma unroll
            for (int k = 8; k < 128; k += 2) mx[(k >> 1) & 7] = max3(mx[(k >> 1) & 7], x[k], x[k + 1]);
            const float tmax = fmaxf(max3(mx[0], mx[1], mx[2]), max3(mx[3], mx[4], max3(mx[5], mx[6], mx[7])));
            // PV_g(j-1) has read P_g(j-1) (and added into O_g) before P_g(j) or a rescale may touch them
            if (j > 0)
            {
                if (!mbar_wait(pv_done(g), (j - 1) & 1))
                {
                    ok = false;
                    break;
                }
                tc_fence_after();
            }
            if (j == 0) m_run = tmax;
            else if (__any_sync(0xffffffffu, (tmax - m_run) * c > kRescaleLog2))
            {
                const float m_new = fmaxf(m_run, tmax);
                const float alpha = fast_exp2((m_run - m_new) * c);
#pragma unroll
                for (int cc = 0; cc < 4; ++cc)
                {
                    float o[32];
                    tmem_load_32(lane_base + o_col(g) + cc * 32, o);
#pragma unroll
                    for (int t = 0; t < 32; ++t) o[t] *= alpha;
                    tmem_store_32(lane_base + o_col(g) + cc * 32, o);
                }
                tmem_store_wait();
                l_run *= alpha;
                m_run = m_new;
            }
            // exponent arguments two at a time (packed FP32x2 FFMA), four independent pair sums; P row r
            // as BF16 into the swizzled K-major tile: half h holds keys 64h..64h+63, 16-byte chunk cc of
            // row r sits at chunk cc ^ (r & 7)
            const float2 scale2 = make_float2(c, c), neg2 = make_float2(-m_run * c, -m_run * c);
            float2 sum2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                              make_float2(0.f, 0.f)};
#pragma unroll
            for (int k8 = 0; k8 < 128; k8 += 8)
            {
                uint32_t w[4];
#pragma unroll
                for (int t = 0; t < 8; t += 2)
                {
                    const float2 arg = __ffma2_rn(make_float2(x[k8 + t], x[k8 + t + 1]), scale2, neg2);
                    const float e0 = fast_exp2(arg.x), e1 = fast_exp2(arg.y);
                    sum2[t >> 1] = __fadd2_rn(sum2[t >> 1], make_float2(e0, e1));
                    w[t >> 1] = pack2(e0, e1);
                }
                const int h = k8 >> 6, cc = (k8 & 63) >> 3;
                st_shared_v4(s_p(g) + h * kHalfBytes + r * 128 + ((cc ^ (r & 7)) << 4), w[0], w[1], w[2], w[3]);
            }
            const float2 s01 = __fadd2_rn(sum2[0], sum2[1]), s23 = __fadd2_rn(sum2[2], sum2[3]);
            const float2 s4 = __fadd2_rn(s01, s23);
            l_run += s4.x + s4.y;
            fence_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full(g));
        }
        if (ok && active && !mbar_wait(pv_done(g), (tiles - 1) & 1)) ok = false;
        if (!ok)
        {
            if (a.error_flag && lane == 0) atomicExch(a.error_flag, kErrFlashSoftmaxTimeout);
        }
        else if (active)
        {
            tc_fence_after();
            const int row = q0 + g * kTile + r;
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
                tmem_load_32(lane_base + o_col(g) + cc * 32, o);
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
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tmem_done);
        peer_signal_warp(a.sync.signal); // this warp's output rows are stored
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
    cudaFuncAttributes attr;
    cudaError_t e = cudaFuncGetAttributes(&attr, flash_tc_kernel);
    if (e != cudaSuccess) return e;
    // the register split above needs this many registers per thread at launch
    if (attr.numRegs < kMinLaunchRegs) return cudaErrorInvalidConfiguration;
    return cudaFuncSetAttribute(flash_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
}

int launch_flash_tc(const __nv_bfloat16 *q, const __nv_bfloat16 *k, const __nv_bfloat16 *vt, const float *mask,
                    int rows, int rows_pad, int kv_len, int heads, const FlashOutput &out, int *error_flag,
                    cudaStream_t stream, int causal, int kv_heads, const PeerSync *sync)
{
    if (kv_heads == 0) kv_heads = heads;
    if (rows < 1 || kv_len < 1 || kv_len > rows_pad || rows_pad % kTile || rows > rows_pad || heads < 1 ||
        kv_heads < 1 || heads % kv_heads || out.rows_per_dest < 1 || out.ld % 8 || out.col_offset % 8 ||
        out.col_offset + heads * kTile > out.ld)
        return cudaErrorInvalidValue;
    for (int d = 0; d < (rows + out.rows_per_dest - 1) / out.rows_per_dest; ++d)
        if (d >= kMaxDest || !out.dst[d]) return cudaErrorInvalidValue;
    CUtensorMap mq, mk, mv;
    if (!map_2d(&mq, q, static_cast<uint64_t>(heads) * rows_pad, kTile) ||
        !map_2d(&mk, k, static_cast<uint64_t>(kv_heads) * rows_pad, kTile) ||
        !map_2d(&mv, vt, static_cast<uint64_t>(kv_heads) * kTile, static_cast<uint64_t>(rows_pad)))
        return cudaErrorInvalidValue;
    FlashArgs a{rows, rows_pad, kv_len, mask, out, error_flag};
    a.causal = causal ? 1 : 0;
    a.kv_group = heads / kv_heads;
    const dim3 grid((rows + kRowsPerCta - 1) / kRowsPerCta, heads);
    if (sync)
    {
        a.sync = *sync;
        a.sync.signal.warps = static_cast<int>(grid.x * grid.y) * 8; // the eight softmax warps of each CTA
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attrs[1];
    cfg.attrs = attrs;
    cfg.numAttrs = add_programmatic_attribute(attrs, 0);
    return cudaLaunchKernelEx(&cfg, flash_tc_kernel, mq, mk, mv, a);
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
