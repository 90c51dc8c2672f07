// tcgen05 flash attention for the ERNIE DiT block (BF16 mode).
//
// Replaces sdpa_22 (block.ncnn.param:58; ErnieSDPA / AccurateSDPA, src/ernie_attention.cpp:35-233):
// softmax(Q K^T / sqrt(128) + mask_row) V per head over the joint image+text sequence, non-causal,
// keys past the valid count (the -1e30 text padding of src/conditioning.cpp:41-42) skipped.
//
// One CTA = one head x 256 queries as two 128-row query tiles A and B that share every K / V^T tile;
// KV tiles of 128 keys. TMEM (512 columns): S_A, S_B, O_A, O_B, 128 columns each; P_g (BF16 pairs,
// 64 columns) overwrites the first half of S_g once softmax has read S_g, and is the TMEM A operand
// of the PV MMA, so P never touches shared memory.
//   warp 0      TMA producer: Q_A, Q_B once, then K and V^T tiles through a 2-stage ring
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer, in the order
//                 S_A(j), PV_B(j-1), S_B(j), PV_A(j), S_A(j+1), ...
//               so the tensor core computes one group's MMAs while the other group's softmax runs
//               (MMAs of one thread execute in issue order, so S_g(j+1) overwrites P_g(j) only after
//               PV_g(j) has read it)
//   warps 2, 3  idle (warpgroup 0 hands its registers to the softmax warpgroups)
//   warps 4..7  softmax of tile A, warps 8..11 softmax of tile B; one query row per thread:
//               tcgen05.ld of S_g(j), online max/sum in FP32, P_g(j) stored to TMEM, final O / l.
//               exp2 on the MUFU (a degree-3 polynomial on the FMA pipe for part of the keys was
//               measured slower: at ~9 instructions per element it costs more issue slots than the
//               MUFU's 8 cycles per warp instruction save). Row max over 8 independent chains, the
//               exponent arguments and row sums as packed FP32x2 operations.
//               The running max is only raised (and O_g rescaled in TMEM) when a tile's max exceeds
//               it by more than 2^8; between raises the stale max is exact because O and l share it.
//               The commit of S_g(j) also covers PV_g(j-1), so a rescale never races the PV MMA.
// V is stored transposed ([head][dim][token], written by the QKV GEMM epilogue) so the PV MMA's B
// operand is K-major. All mbarrier waits are bounded. Every TMA load fills this CTA's own shared memory.
#include "kernels.h"
#include "ptx.cuh"
#include <cudaTypedefs.h>
#include <mutex>

namespace ernie_b200
{
namespace
{
constexpr int kThreads = 384;               // three warpgroups (register reallocation is per warpgroup)
// Registers per thread after setmaxnreg: warpgroup 0 (TMA, MMA, two idle warps) gives registers to
// the two softmax warpgroups (216 each: no spills; at 168 the softmax spilled). 128 x 72 + 256 x 216 =
// 64512 = 384 x 168, so the launch must have 168 registers per thread, which ptxas assigns at 384
// threads; the host refuses to launch otherwise (an increase the block cannot satisfy would wait).
constexpr int kRegsControl = 72, kRegsSoftmax = 216, kMinLaunchRegs = 168;
static_assert(128 * kRegsControl + 256 * kRegsSoftmax <= kThreads * kMinLaunchRegs, "register split");
constexpr int kTile = 128;                   // queries per tile, keys per KV tile, head dim
constexpr int kRowsPerCta = 2 * kTile;       // two query tiles
constexpr int kHalfBytes = kTile * 64 * 2;   // one 64-column half of a 128 x 128 BF16 tile
constexpr int kTileBytes = 2 * kHalfBytes;   // 32 KB
constexpr int kSmemBytes = 6 * kTileBytes + 1024 + 256; // Q_A, Q_B, 2 K, 2 V^T tiles
constexpr int kTmemCols = 512;               // S_A 0, S_B 128, O_A 256, O_B 384

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

__device__ __forceinline__ uint32_t pack2(float lo, float hi)
{
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

// O (+)= P V: A = P from TMEM (128 lanes x 16 keys per instruction = 8 columns of BF16 pairs).
__device__ __forceinline__ void umma_bf16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
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
    flash_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                    const __grid_constant__ CUtensorMap map_vt, FlashArgs a)
{
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *base_ptr = smem_raw + (base - raw);
    auto s_q = [&](int g) { return base + g * kTileBytes; };
    auto s_k = [&](int s) { return base + (2 + s) * kTileBytes; };
    auto s_v = [&](int s) { return base + (4 + s) * kTileBytes; };
    const uint32_t bars = base + 6 * kTileBytes;
    const uint32_t q_full = bars;
    auto k_full = [&](int s) { return bars + 8u * (1 + s); };
    auto k_empty = [&](int s) { return bars + 8u * (3 + s); };
    auto v_full = [&](int s) { return bars + 8u * (5 + s); };
    auto v_empty = [&](int s) { return bars + 8u * (7 + s); };
    auto s_full = [&](int g) { return bars + 8u * (9 + g); };
    auto p_full = [&](int g) { return bars + 8u * (11 + g); };
    auto o_full = [&](int g) { return bars + 8u * (13 + g); };
    const uint32_t tmem_done = bars + 8u * 15;
    const uint32_t slot = bars + 8u * 16;

    const int head = blockIdx.y, q0 = blockIdx.x * kRowsPerCta;
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
            mbar_init(o_full(s), 1);
        }
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
    auto s_col = [](int g) { return static_cast<uint32_t>(g * 128); };
    auto o_col = [](int g) { return static_cast<uint32_t>(256 + g * 128); };
    // Each role ends the kernel on its own: the register split differs per warpgroup, so no code
    // after the split is shared. TMEM is freed by warp 1 once all 8 softmax warps are done with it.
    if (warp < 4)
    {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
    if (warp == 0)
    {
        if (lane == 0)
        {
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
            auto issue_s = [&](int g, int s) {
#pragma unroll
                for (int k = 0; k < 8; ++k)
                {
                    const uint64_t ad = smem_desc_sw128(s_q(g) + (k >> 2) * kHalfBytes) + 2u * (k & 3);
                    const uint64_t bd = smem_desc_sw128(s_k(s) + (k >> 2) * kHalfBytes) + 2u * (k & 3);
                    umma_bf16(tmem_base + s_col(g), ad, bd, idesc, k > 0 ? 1u : 0u);
                }
                umma_commit(s_full(g));
            };
            // PV_g(j): waits for P_g(j) and V_j
            auto issue_pv = [&](int g, int j) -> bool {
                const int s = j & 1;
                const uint32_t ph = (j >> 1) & 1;
                if (!mbar_wait(p_full(g), j & 1) || !mbar_wait(v_full(s), ph)) return false;
                tc_fence_after();
#pragma unroll
                for (int k = 0; k < 8; ++k)
                {
                    const uint64_t bd = smem_desc_sw128(s_v(s) + (k >> 2) * kHalfBytes) + 2u * (k & 3);
                    umma_bf16_tmem_a(tmem_base + o_col(g), tmem_base + s_col(g) + 8u * k, bd, idesc,
                                     (j > 0 || k > 0) ? 1u : 0u);
                }
                return true;
            };
            for (int j = 0; j < tiles && ok; ++j)
            {
                const int s = j & 1;
                if (!mbar_wait(k_full(s), (j >> 1) & 1))
                {
                    ok = false;
                    break;
                }
                tc_fence_after();
                issue_s(0, s);
                if (j > 0)
                {
                    if (!issue_pv(1, j - 1))
                    {
                        ok = false;
                        break;
                    }
                    umma_commit(v_empty((j - 1) & 1));
                }
                issue_s(1, s);
                umma_commit(k_empty(s));
                if (!issue_pv(0, j))
                {
                    ok = false;
                    break;
                }
                if (j == tiles - 1) umma_commit(o_full(0));
            }
            if (ok)
            {
                ok = issue_pv(1, tiles - 1);
                if (ok)
                {
                    umma_commit(v_empty((tiles - 1) & 1));
                    umma_commit(o_full(1));
                }
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
        const int quarter = warp & 3;     // TMEM lane quarter this warp may access
        const int r = quarter * 32 + lane; // row within the query tile == TMEM lane
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        // scores stay in raw units; c folds 1/sqrt(128) and log2(e) into one FFMA per element
        constexpr float c = 0.08838834764831845f * 1.4426950408889634f;
        constexpr float kMaskToRaw = 11.313708498984761f; // log2(e)/c = sqrt(128)
        constexpr float kRescaleLog2 = 8.f;              // rescale O only when the max grows by 2^8
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        for (int j = 0; j < tiles && ok; ++j)
        {
            if (!mbar_wait(s_full(g), j & 1))
            {
                ok = false;
                break;
            }
            tc_fence_after();
            float x[128];
            tmem_load_128(lane_base + s_col(g), x);
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
            // row max over 8 independent chains (a single 127-long chain is latency bound)
            float mx[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) mx[k] = x[k];
#pragma unroll
            for (int k = 8; k < 128; ++k) mx[k & 7] = fmaxf(mx[k & 7], x[k]);
            const float tmax = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                     fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
            if (j == 0) m_run = tmax;
            else if (__any_sync(0xffffffffu, (tmax - m_run) * c > kRescaleLog2))
            {
                // PV_g(j-1) is complete: its commit preceded S_g(j)'s
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
                l_run *= alpha;
                m_run = m_new;
            }
            // exponent arguments two at a time (packed FP32x2 FFMA), four independent pair sums
            const float2 scale2 = make_float2(c, c), neg2 = make_float2(-m_run * c, -m_run * c);
            float2 sum2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                              make_float2(0.f, 0.f)};
            uint32_t pk[64];
#pragma unroll
            for (int k = 0; k < 128; k += 2)
            {
                const float2 arg = __ffma2_rn(make_float2(x[k], x[k + 1]), scale2, neg2);
                const float e0 = fast_exp2(arg.x), e1 = fast_exp2(arg.y);
                sum2[(k >> 1) & 3] = __fadd2_rn(sum2[(k >> 1) & 3], make_float2(e0, e1));
                pk[k / 2] = pack2(e0, e1);
            }
            const float2 s01 = __fadd2_rn(sum2[0], sum2[1]), s23 = __fadd2_rn(sum2[2], sum2[3]);
            const float2 s4 = __fadd2_rn(s01, s23);
            l_run += s4.x + s4.y;
            // P_g(j) over the first 64 columns of S_g (the MMA reads it as BF16 pairs, key 2i low)
            tmem_store_32u(lane_base + s_col(g), pk);
            tmem_store_32u(lane_base + s_col(g) + 32, pk + 32);
            tmem_store_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full(g));
        }
        if (ok && !mbar_wait(o_full(g), 0)) ok = false;
        if (!ok)
        {
            if (a.error_flag && lane == 0) atomicExch(a.error_flag, kErrFlashSoftmaxTimeout);
        }
        else
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
    const dim3 grid((rows + kRowsPerCta - 1) / kRowsPerCta, heads);
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
