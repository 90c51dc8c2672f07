// The VAE decoder's kernels for sm_100a: a tcgen05 implicit-GEMM convolution and the bandwidth-bound
// GroupNorm / SiLU / upsample / softmax passes around it.
//
// Replaces the ncnn layers of the reference's decoder graph (AutoencoderKLFlux2 post_quant_conv +
// decoder, exported by tools/export_vae.py and run by src/vae.cpp:18-64):
//   Convolution 3x3 / 1x1     conv_kernel (implicit GEMM: M = pixels, N = output channels, K = taps x Cin)
//   BinaryOp add (residual)   fused into the conv epilogue (out = acc + bias + resid)
//   GroupNorm (ErnieGroupNorm, src/ernie_groupnorm.cpp:33-64)
//                             FP64 partial sums in the producing conv's epilogue -> gn_finalize_kernel
//                             (per-channel scale/shift) -> gn_apply_kernel (+ Swish) writing the next
//                             conv's BF16 operand
//   Interp nearest x2         upsample_kernel (writes the upsampling conv's operand)
//   MultiHeadAttention        1x1-conv projections + score/probability GEMMs on conv_kernel,
//                             softmax_rows_kernel between them
//
// conv_kernel structure (one CTA per SM, persistent over 128-pixel x BN-channel output tiles):
//   warp 0      TMA producer. The A tile of k-block (tap, c0) is a 3D box {64 channels, 128 pixels, 1 row}
//               of the NHWC BF16 operand at (plane*Cin + c0, x0 + dx, y + dy): the tap's shift is a
//               coordinate offset, and TMA's zero fill outside the image is the convolution's
//               zero padding. The B tile is {64, BN} of the [Cout][planes x taps x Cin] weights.
//               Stride-2 mode (the encoder's Downsample2D) reads a space-to-depth operand: tap (ky, kx) is
//               the box at (phase * planes * Cin + plane * Cin + c0, x0 + kx / 2, y + ky / 2), phase =
//               (ky & 1) * 2 + (kx & 1), so the strided taps stay unit-stride boxes.
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer (M=128, N=BN, K=16 per instruction).
//   warps 2..5  epilogue: one TMEM lane (one pixel) per thread; bias, residual, FP32 NHWC store and
//               the GroupNorm partial sums of the written values.
// FP32-exact mode multiplies three BF16 planes (hi, mid, lo) of the operand by one (exact-BF16 weights)
// or three weight planes, keeping the products of total plane order <= 2, and restarts the tensor-core
// accumulator every `group` k-blocks (the partials are summed in FP32 registers), as the DiT GEMM does.
#include "ernie_synth.h"
#include "kernels.h"
#include "ptx.cuh"
#include <cudaTypedefs.h>
#include <mutex>
#include <type_traits>

namespace ernie_b200
{
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

namespace
{
constexpr int CM = 128, CK = 64, kConvThreads = 320, kEpiWarps = 8;
enum : int
{
    kErrConvProducerTimeout = 31,
    kErrConvMmaTimeout = 32,
    kErrConvEpilogueTimeout = 33,
};

// Output tile: MSUB sub-tiles of 128 pixels (128-pixel row segments, consecutive in the flattened
// row-segment order) x BN channels. MSUB = 2 lets two M=128 MMAs share each B tile.
template <int BN, bool PROMOTE, int MSUB> struct ConvCfg
{
    static_assert(BN == 32 || BN == 128 || BN == 256, "tile widths");
    static_assert(MSUB == 1 || (MSUB == 2 && BN <= 128), "two pixel sub-tiles with 32- or 128-channel tiles");
    static_assert(MSUB == 2 || BN >= 128, "every epilogue warp takes a multiple of 32 columns");
    static_assert(!PROMOTE || (BN == 128 && MSUB == 1) || BN == 32, "FP32 promotion: at most 64 running sums");
    static constexpr int kStages = BN == 32 ? 5 : (BN == 256 || MSUB == 2) ? 4 : 6;
    static constexpr int kABytes = MSUB * CM * CK * 2;
    static constexpr int kBBytes = BN * CK * 2;
    static constexpr int kStageBytes = kABytes + kBBytes; // a multiple of 1024 for every configuration
    static constexpr int kAccCols = MSUB * BN;           // one accumulator buffer
    static constexpr int kTmemCols = 2 * kAccCols;
    // columns per epilogue warp: warps 2..5 and 6..9 take the two sub-tiles, or the two column halves
    static constexpr int kWarpCols = MSUB == 2 ? BN : BN / 2;
    static constexpr int kBarrierBytes = 256;
    // per epilogue warp: a [32][20] FP32 staging tile and 32 FP64 (sum, sum of squares) GroupNorm slots
    static constexpr int kStageFloats = 32 * 20;
    static constexpr int kEpilogueOffset = kStages * kStageBytes + kBarrierBytes;
    static constexpr int kEpilogueBytes = kEpiWarps * (kStageFloats * 4 + 32 * 16);
    static constexpr int kSmemBytes = kEpilogueOffset + kEpilogueBytes + 1024;
    static_assert(kSmemBytes <= 232448, "shared memory per CTA");
};

// Plane pair (operand plane, weight plane) of product p: one product in BF16 mode; (0,0) (1,0) (2,0)
// against exact-BF16 weights; the six pairs of total order <= 2 against three weight planes.
__device__ __forceinline__ void plane_pair(int products, int p, int &pa, int &pb)
{
    if (products == 6)
    {
        pa = (0x910 >> (2 * p)) & 3; // 0 0 1 0 1 2
        pb = (0x184 >> (2 * p)) & 3; // 0 1 0 2 1 0
    }
    else
    {
        pa = p;
        pb = 0;
    }
}

__device__ __forceinline__ double warp_sum(double v)
{
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Columns [col, col + 32) of the warp's 32 pixels (thread `lane` holds pixel row `lane` in v), as two 16-column
// halves staged through shared memory and written row-major: lane covers columns + 4*(lane % 4) .. +3 of rows
// 8*i + lane / 4, so 4 lanes store one 64-byte row segment. out = (acc + bias) + resid for the first `limit`
// rows. The thread's GroupNorm partial sums of each half (one group per thread and half) are added to
// s[0..1], q[0..1].
template <typename T>
__device__ __forceinline__ void rows_pair(const float (&v)[32], float *stage, int col, int limit, long long pixel_first,
                                          int lane, const ConvArgs &a, T (&s)[2], T (&q)[2])
{
    const int c4 = (lane & 3) * 4, oct = lane >> 2;
    // the residual loads of both halves first: `out` may alias `resid` (in place), so a load placed after
    // an earlier row's store could not be hoisted above it
    float4 u[2][4];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int i = 0; i < 4; ++i)
        {
            const int r = 8 * i + oct;
            u[h][i] = a.resid && r < limit
                          ? *reinterpret_cast<const float4 *>(a.resid + (pixel_first + r) * a.ldo + col + 16 * h + c4)
                          : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    const bool stats = a.stats != nullptr;
#pragma unroll
    for (int h = 0; h < 2; ++h)
    {
        float4 *mine = reinterpret_cast<float4 *>(stage + lane * 20);
#pragma unroll
        for (int k = 0; k < 4; ++k)
            mine[k] = make_float4(v[16 * h + 4 * k], v[16 * h + 4 * k + 1], v[16 * h + 4 * k + 2], v[16 * h + 4 * k + 3]);
        __syncwarp();
        const float4 b = a.bias ? __ldg(reinterpret_cast<const float4 *>(a.bias + col + 16 * h + c4))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int i = 0; i < 4; ++i)
        {
            const int r = 8 * i + oct;
            float4 t = *reinterpret_cast<const float4 *>(stage + r * 20 + c4);
            // (conv + bias) + residual, the reference graph's Convolution then BinaryOp add
            t.x = (t.x + b.x) + u[h][i].x;
            t.y = (t.y + b.y) + u[h][i].y;
            t.z = (t.z + b.z) + u[h][i].z;
            t.w = (t.w + b.w) + u[h][i].w;
            if (r < limit)
            {
                if (a.out) *reinterpret_cast<float4 *>(a.out + (pixel_first + r) * a.ldo + col + 16 * h + c4) = t;
                if (stats)
                {
                    const T d0 = t.x, d1 = t.y, d2 = t.z, d3 = t.w;
                    s[h] += (d0 + d1) + (d2 + d3);
                    q[h] += (d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3);
                }
            }
        }
        __syncwarp();
    }
}

// The tile's per-thread GroupNorm partials (slot k: columns col0 + 16k .. +16 of the warp's range) summed over
// the lanes of each group in FP64 and added into the warp's group slots `acc` (a fixed order: deterministic).
template <typename T, int SLOTS>
__device__ __forceinline__ void flush_stats(const T (&s)[SLOTS], const T (&q)[SLOTS], int col0, int cpg, int lane,
                                            double2 *acc)
{
    double ds[SLOTS], dq[SLOTS];
#pragma unroll
    for (int k = 0; k < SLOTS; ++k)
    {
        ds[k] = static_cast<double>(s[k]);
        dq[k] = static_cast<double>(q[k]);
    }
    // lanes of one group: the eight row octets, and cpg / 4 neighbouring column quads
#pragma unroll
    for (int o = 4; o <= 16; o <<= 1)
#pragma unroll
        for (int k = 0; k < SLOTS; ++k)
        {
            ds[k] += __shfl_xor_sync(0xffffffffu, ds[k], o);
            dq[k] += __shfl_xor_sync(0xffffffffu, dq[k], o);
        }
    if (cpg >= 8)
#pragma unroll
        for (int k = 0; k < SLOTS; ++k)
        {
            ds[k] += __shfl_xor_sync(0xffffffffu, ds[k], 1);
            dq[k] += __shfl_xor_sync(0xffffffffu, dq[k], 1);
        }
    if (cpg >= 16)
#pragma unroll
        for (int k = 0; k < SLOTS; ++k)
        {
            ds[k] += __shfl_xor_sync(0xffffffffu, ds[k], 2);
            dq[k] += __shfl_xor_sync(0xffffffffu, dq[k], 2);
        }
    if (lane < 4 && (lane & (cpg / 4 - 1)) == 0)
    {
#pragma unroll
        for (int k = 0; k < SLOTS; ++k)
        {
            const int g = (col0 + 16 * k + lane * 4) / cpg;
            acc[g].x += ds[k];
            acc[g].y += dq[k];
        }
    }
    __syncwarp();
}

template <int BN, bool PROMOTE, int MSUB>
__global__ void __launch_bounds__(kConvThreads, 1)
    conv_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, ConvArgs args)
{
    using C = ConvCfg<BN, PROMOTE, MSUB>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *base_ptr = smem_raw + (base - raw);
    const uint32_t bars = base + C::kStages * C::kStageBytes;
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (C::kStages + s); };
    auto tfull_bar = [&](int i) { return bars + 8u * (2 * C::kStages + i); };
    auto tempty_bar = [&](int i) { return bars + 8u * (2 * C::kStages + 2 + i); };
    const uint32_t slot = bars + 8u * (2 * C::kStages + 4);
    auto tile_a = [&](int s, int sub) { return base + s * C::kStageBytes + sub * (CM * CK * 2); };
    auto tile_b = [&](int s) { return base + s * C::kStageBytes + C::kABytes; };

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int tiles_x = (args.width + CM - 1) / CM, segments = args.height * tiles_x;
    const int m_tiles = (segments + MSUB - 1) / MSUB;
    const int n_tiles = args.cout / BN, tiles = m_tiles * n_tiles;
    const int cblk = args.cin / CK, k_blocks = args.taps * cblk;
    const int span = PROMOTE ? args.group : k_blocks; // k-blocks per accumulation chain
    const int products = args.products;

    if (threadIdx.x == 0)
    {
        for (int s = 0; s < C::kStages; ++s)
        {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int i = 0; i < 2; ++i)
        {
            mbar_init(tfull_bar(i), 1);
            mbar_init(tempty_bar(i), kEpiWarps);
        }
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0)
    {
        prefetch_tensormap(&map_a);
        prefetch_tensormap(&map_b);
    }
    if (warp == 1)
    {
        tmem_alloc(slot, C::kTmemCols);
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
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x)
            {
                // output channels fastest: CTAs working at the same time share operand rows in L2
                const int m_blk = tile / n_tiles, n_blk = tile - m_blk * n_tiles;
                int ys[MSUB], xs[MSUB];
#pragma unroll
                for (int sub = 0; sub < MSUB; ++sub)
                {
                    const int seg = m_blk * MSUB + sub; // past the last segment: rows past the image, zero-filled
                    ys[sub] = seg / tiles_x;
                    xs[sub] = (seg - ys[sub] * tiles_x) * CM;
                }
                for (int kb = 0; kb < k_blocks && ok; ++kb)
                {
                    const int tap = kb / cblk, c0 = (kb - tap * cblk) * CK;
                    const int ky = tap / 3, kx = tap - ky * 3;
                    int dy = 0, dx = 0, coff = 0;
                    if (args.stride2)
                    {
                        dy = ky >> 1;
                        dx = kx >> 1;
                        coff = ((ky & 1) * 2 + (kx & 1)) * args.phase_stride;
                    }
                    else if (args.taps == 9)
                    {
                        dy = ky - 1;
                        dx = kx - 1;
                    }
                    for (int p = 0; p < products; ++p)
                    {
                        int pa, pb;
                        plane_pair(products, p, pa, pb);
                        if (!mbar_wait(empty_bar(stage), phase ^ 1u))
                        {
                            if (args.error_flag) atomicExch(args.error_flag, kErrConvProducerTimeout);
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(full_bar(stage), C::kStageBytes);
#pragma unroll
                        for (int sub = 0; sub < MSUB; ++sub)
                            tma_load_3d(tile_a(stage, sub), &map_a, full_bar(stage), coff + pa * args.cin + c0,
                                        xs[sub] + dx, ys[sub] + dy);
                        tma_load_2d(tile_b(stage), &map_b, full_bar(stage), pb * args.taps * args.cin + kb * CK,
                                    n_blk * BN);
                        if (++stage == C::kStages)
                        {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                }
            }
            // On a timeout no drain is needed: the last load was issued before the failed wait began,
            // kWaitLimitCycles earlier, and TMA loads complete without any consumer.
        }
    }
    else if (warp == 1)
    {
        if (lane == 0)
        {
            constexpr uint32_t idesc = idesc_bf16(CM, BN);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int unit = 0;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x)
            {
                for (int kb0 = 0; kb0 < k_blocks && ok; kb0 += span, ++unit)
                {
                    const int acc = unit & 1;
                    const uint32_t acc_phase = (unit >> 1) & 1;
                    if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u))
                    {
                        if (args.error_flag) atomicExch(args.error_flag, kErrConvMmaTimeout);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * C::kAccCols);
                    for (int kb = kb0; kb < kb0 + span && ok; ++kb)
                    {
                        for (int p = 0; p < products; ++p)
                        {
                            if (!mbar_wait(full_bar(stage), phase))
                            {
                                if (args.error_flag) atomicExch(args.error_flag, kErrConvMmaTimeout);
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            const uint64_t b_desc = smem_desc_sw128(tile_b(stage));
#pragma unroll
                            for (int sub = 0; sub < MSUB; ++sub)
                            {
                                const uint64_t a_desc = smem_desc_sw128(tile_a(stage, sub));
#pragma unroll
                                for (int k = 0; k < CK / 16; ++k)
                                    umma_bf16(d_tmem + sub * BN, a_desc + 2u * k, b_desc + 2u * k, idesc,
                                              (kb != kb0 || p != 0 || k != 0) ? 1u : 0u);
                            }
                            umma_commit(empty_bar(stage));
                            if (++stage == C::kStages)
                            {
                                stage = 0;
                                phase ^= 1u;
                            }
                        }
                    }
                    if (ok) umma_commit(tfull_bar(acc));
                }
            }
        }
    }
    else
    {
        constexpr int CW = C::kWarpCols, SLOTS = CW / 16;
        using T = std::conditional_t<PROMOTE, double, float>; // per-tile partials: FP32 in BF16 mode
        const int e = warp - 2, quarter = warp & 3, half = e >> 2;
        // this warp's pixel sub-tile and column range of each tile
        const int sub = MSUB == 2 ? half : 0;
        const int col0 = MSUB == 2 ? 0 : half * CW;
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        float *stage = reinterpret_cast<float *>(base_ptr + C::kEpilogueOffset) + e * C::kStageFloats;
        double2 *group_acc =
            reinterpret_cast<double2 *>(base_ptr + C::kEpilogueOffset + kEpiWarps * C::kStageFloats * 4) + e * 32;
        group_acc[lane] = make_double2(0.0, 0.0);
        __syncwarp();
        int unit = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x)
        {
            const int m_blk = tile / n_tiles, n_blk = tile - m_blk * n_tiles;
            const int seg = m_blk * MSUB + sub;
            const int y = seg / tiles_x, x_first = (seg - y * tiles_x) * CM + quarter * 32;
            // rows of this warp inside the image (0 for a sub-tile past the last row)
            const int limit = y < args.height ? min(32, args.width - x_first) : 0;
            const long long pixel_first = static_cast<long long>(y) * args.width + x_first;
            const uint32_t acc_cols = static_cast<uint32_t>(sub * BN + col0);
            const int col_base = n_blk * BN + col0;
            T s[SLOTS], q[SLOTS];
#pragma unroll
            for (int k = 0; k < SLOTS; ++k) s[k] = q[k] = T(0);
            auto emit = [&](const float(&v)[32], int c) {
                T ps[2] = {T(0), T(0)}, pq[2] = {T(0), T(0)};
                rows_pair<T>(v, stage, col_base + c, limit, pixel_first, lane, args, ps, pq);
                s[c / 16] += ps[0];
                q[c / 16] += pq[0];
                s[c / 16 + 1] += ps[1];
                q[c / 16 + 1] += pq[1];
            };
            if constexpr (!PROMOTE)
            {
                const int acc = unit & 1;
                const uint32_t acc_phase = (unit >> 1) & 1;
                if (!mbar_wait(tfull_bar(acc), acc_phase))
                {
                    if (args.error_flag && lane == 0) atomicExch(args.error_flag, kErrConvEpilogueTimeout);
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < CW; c += 32)
                {
                    float v[32];
                    tmem_load_32(lane_base + acc * C::kAccCols + acc_cols + c, v);
                    emit(v, c);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(tempty_bar(acc));
                ++unit;
            }
            else
            {
                float sum[CW];
#pragma unroll
                for (int j = 0; j < CW; ++j) sum[j] = 0.f;
                for (int kb0 = 0; kb0 < k_blocks; kb0 += span, ++unit)
                {
                    const int acc = unit & 1;
                    const uint32_t acc_phase = (unit >> 1) & 1;
                    if (!mbar_wait(tfull_bar(acc), acc_phase))
                    {
                        if (args.error_flag && lane == 0) atomicExch(args.error_flag, kErrConvEpilogueTimeout);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int c = 0; c < CW; c += 32)
                    {
                        float v[32];
                        tmem_load_32(lane_base + acc * C::kAccCols + acc_cols + c, v);
#pragma unroll
                        for (int j = 0; j < 32; ++j) sum[c + j] += v[j];
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(tempty_bar(acc));
                }
                if (!ok) break;
#pragma unroll
                for (int c = 0; c < CW; c += 32)
                {
                    float v[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = sum[c + j];
                    emit(v, c);
                }
            }
            if (args.stats) flush_stats<T, SLOTS>(s, q, col_base, args.cpg, lane, group_acc);
        }
        // this warp's GroupNorm partials: every slot written (zero for groups it saw no tile of), in the
        // fixed tile order of this CTA, so the sums are deterministic for a given grid
        __syncwarp();
        if (args.stats)
            args.stats[static_cast<size_t>(lane) * gridDim.x * kEpiWarps + blockIdx.x * kEpiWarps + e] = group_acc[lane];
    }
    __syncthreads();
    if (warp == 1)
    {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::kTmemCols);
    }
}

template <int BN, bool PROMOTE, int MSUB> cudaError_t ensure_conv_attributes()
{
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(conv_kernel<BN, PROMOTE, MSUB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    ConvCfg<BN, PROMOTE, MSUB>::kSmemBytes);
    });
    return attr;
}

// NHWC BF16 operand [height][width][channels] as a 3D map with {64, 128, 1} boxes.
bool make_operand_map(CUtensorMap *map, const void *ptr, uint64_t channels, uint64_t width, uint64_t height)
{
    auto fn = tensor_map_encoder();
    if (!fn) return false;
    if ((reinterpret_cast<uintptr_t>(ptr) & 15u) || (channels * 2) % 16) return false;
    const cuuint64_t dims[3] = {channels, width, height};
    const cuuint64_t strides[2] = {channels * 2, channels * width * 2};
    const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(CM), 1};
    const cuuint32_t element_strides[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(ptr), dims, strides, box,
              element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_weight_map(CUtensorMap *map, const void *ptr, uint64_t rows, uint64_t cols, uint32_t box_rows)
{
    auto fn = tensor_map_encoder();
    if (!fn) return false;
    if ((reinterpret_cast<uintptr_t>(ptr) & 15u) || (cols * 2) % 16) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t element_strides[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box,
              element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tile shape of a launch: (BN, MSUB). 32 output columns: 32; FP32-exact mode: 128; BF16 mode: 256 columns,
// or 2 x 128 pixels x 128 columns where the width is not a multiple of 256.
void conv_shape(const ConvLaunch &l, int &bn, int &msub)
{
    msub = 1;
    if (l.cout == 32)
    {
        bn = 32;
        msub = 2;
    }
    else if (l.a_planes == 3) bn = 128;
    else if (l.cout % 256 == 0) bn = 256;
    else
    {
        bn = 128;
        msub = 2;
    }
}

int conv_grid(const ConvLaunch &l, int num_sms)
{
    int bn = 0, msub = 1;
    conv_shape(l, bn, msub);
    const long long segments = static_cast<long long>(l.height) * ((l.width + CM - 1) / CM);
    const long long tiles = (segments + msub - 1) / msub * (l.cout / bn);
    return static_cast<int>(tiles < num_sms ? tiles : num_sms);
}

template <int BN, bool PROMOTE, int MSUB>
int launch_conv_impl(const ConvLaunch &l, ConvArgs args, int num_sms, cudaStream_t stream)
{
    using C = ConvCfg<BN, PROMOTE, MSUB>;
    const cudaError_t attr = ensure_conv_attributes<BN, PROMOTE, MSUB>();
    if (attr != cudaSuccess) return attr;
    CUtensorMap map_a, map_b;
    if (!make_operand_map(&map_a, l.a, static_cast<uint64_t>(l.stride2 ? 4 : 1) * l.a_planes * l.cin, l.width,
                          l.height) ||
        !make_weight_map(&map_b, l.b, static_cast<uint64_t>(l.cout_rows), static_cast<uint64_t>(l.b_row), BN))
        return cudaErrorInvalidValue;
    conv_kernel<BN, PROMOTE, MSUB><<<conv_grid(l, num_sms), kConvThreads, C::kSmemBytes, stream>>>(map_a, map_b, args);
    return cudaGetLastError();
}

// ---- bandwidth kernels ----------------------------------------------------------------------------
int grid_for_count(long long n, int threads)
{
    const long long blocks = (n + threads - 1) / threads;
    return static_cast<int>(blocks < 148LL * 32 ? (blocks > 0 ? blocks : 1) : 148LL * 32);
}

__device__ __forceinline__ void split3f(float x, float &hi, float &mid, float &lo)
{
    hi = __bfloat162float(__float2bfloat16_rn(x));
    const float r1 = x - hi;
    mid = __bfloat162float(__float2bfloat16_rn(r1));
    lo = __bfloat162float(__float2bfloat16_rn(r1 - mid));
}

// 8 consecutive values as one BF16 plane (planes == 1) or three planes `plane_stride` elements apart.
__device__ __forceinline__ void store_planes8(__nv_bfloat16 *dst, long long plane_stride, int planes, const float *v)
{
    if (planes == 1)
    {
        __align__(16) __nv_bfloat162 h[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
        *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(h);
        return;
    }
    __align__(16) __nv_bfloat16 p[3][8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
    {
        float hi, mid, lo;
        split3f(v[j], hi, mid, lo);
        p[0][j] = __float2bfloat16_rn(hi);
        p[1][j] = __float2bfloat16_rn(mid);
        p[2][j] = __float2bfloat16_rn(lo);
    }
#pragma unroll
    for (int q = 0; q < 3; ++q) *reinterpret_cast<uint4 *>(dst + q * plane_stride) = *reinterpret_cast<const uint4 *>(p[q]);
}

__global__ void gn_finalize_kernel(const double2 *stats, int slots, long long count, int cpg,
                                   const float *gamma, const float *beta, float eps, float *scale, float *shift)
{
    __shared__ double part[2][32];
    const int g = blockIdx.x;
    double s = 0.0, q = 0.0;
    for (int i = threadIdx.x; i < slots; i += blockDim.x)
    {
        const double2 v = stats[static_cast<size_t>(g) * slots + i];
        s += v.x;
        q += v.y;
    }
    s = warp_sum(s);
    q = warp_sum(q);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, warps = blockDim.x / 32;
    if (lane == 0)
    {
        part[0][warp] = s;
        part[1][warp] = q;
    }
    __syncthreads();
    if (threadIdx.x < cpg)
    {
        double ts = 0.0, tq = 0.0;
        for (int w = 0; w < warps; ++w)
        {
            ts += part[0][w];
            tq += part[1][w];
        }
        // ErnieGroupNorm: FP64 mean and variance, FP32 scale/bias (src/ernie_groupnorm.cpp:47-61)
        const double mean = ts / static_cast<double>(count);
        double var = tq / static_cast<double>(count) - mean * mean;
        if (var < 0.0) var = 0.0;
        const float inverse = static_cast<float>(1.0 / sqrt(var + static_cast<double>(eps)));
        const int c = g * cpg + threadIdx.x;
        const float sc = __fmul_rn(inverse, gamma ? gamma[c] : 1.f);
        scale[c] = sc;
        shift[c] = __fsub_rn(beta ? beta[c] : 0.f, __fmul_rn(static_cast<float>(mean), sc));
    }
}

// y = x * scale[c] + shift[c] (then Swish x / (1 + exp(-x)) when silu), FP32 NHWC -> BF16 operand planes.
// channels = 2^log2c (the decoder's widths 128, 256, 512); 8 channels per thread and step. BF16 mode
// evaluates the Swish with the fast exponential and division (far below the BF16 rounding that follows);
// FP32-exact mode with expf and an IEEE division. `raw` (nullable) also receives x
// itself as operand planes (the resnet's shortcut-convolution operand, from the same read of x).
__device__ __forceinline__ void gn_apply8(const float4 a, const float4 b, long long e, int c0, int channels,
                                          const float *scale, const float *shift, int silu, __nv_bfloat16 *out,
                                          __nv_bfloat16 *raw, int planes)
{
    const float4 sa = __ldg(reinterpret_cast<const float4 *>(scale + c0)),
                 sb = __ldg(reinterpret_cast<const float4 *>(scale + c0 + 4));
    const float4 ha = __ldg(reinterpret_cast<const float4 *>(shift + c0)),
                 hb = __ldg(reinterpret_cast<const float4 *>(shift + c0 + 4));
    float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    const long long off = planes == 1 ? e : 3 * e - 2 * c0; // pixel p's plane q at p * planes * channels + q * channels
    if (raw) store_planes8(raw + off, channels, planes, v);
    const float sc[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
    const float sh[8] = {ha.x, ha.y, ha.z, ha.w, hb.x, hb.y, hb.z, hb.w};
#pragma unroll
    for (int j = 0; j < 8; ++j)
    {
        float y = __fadd_rn(__fmul_rn(v[j], sc[j]), sh[j]);
        if (silu)
            y = planes == 1 ? __fdividef(y, __fadd_rn(1.f, __expf(-y))) : __fdiv_rn(y, __fadd_rn(1.f, expf(-y)));
        v[j] = y;
    }
    store_planes8(out + off, channels, planes, v);
}

__global__ void gn_apply_kernel(const float *x, long long pixels, int log2c, const float *scale, const float *shift,
                                int silu, __nv_bfloat16 *out, __nv_bfloat16 *raw, int planes)
{
    const int channels = 1 << log2c;
    const long long total = pixels << (log2c - 3);
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
    {
        const long long e = i * 8;
        const float4 *src = reinterpret_cast<const float4 *>(x + e);
        gn_apply8(src[0], src[1], e, static_cast<int>(e & (channels - 1)), channels, scale, shift, silu, out, raw,
                  planes);
    }
}

// Nearest x2 upsampling of FP32 NHWC [h][w][c] into the BF16 operand [2h][2w][planes * c].
__global__ void upsample_kernel(const float *x, int h, int w, int channels, __nv_bfloat16 *out, int planes)
{
    const int per_pixel = channels / 8;
    const long long total = static_cast<long long>(h) * w * per_pixel;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
    {
        const long long p = i / per_pixel;
        const int c0 = static_cast<int>(i - p * per_pixel) * 8;
        const int yy = static_cast<int>(p / w), xx = static_cast<int>(p - static_cast<long long>(yy) * w);
        const float4 *src = reinterpret_cast<const float4 *>(x + p * channels + c0);
        const float4 a = src[0], b = src[1];
        const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int d = 0; d < 4; ++d)
        {
            const long long q = static_cast<long long>(2 * yy + (d >> 1)) * (2 * w) + 2 * xx + (d & 1);
            store_planes8(out + q * planes * channels + c0, channels, planes, v);
        }
    }
}

// ---- encoder passes (encode_vae, src/image_encoder.cpp:28-72) ----
// The encoder's conv_in (3 -> 128, 3x3) as a 1x1 product over im2col columns: RGB bytes normalised in the
// reference's FP32 order (src/image_encoder.cpp:44-51) and gathered per pixel: column t * 3 + c is channel c
// of the neighbour at tap t = ky * 3 + kx (zero outside the image); columns 27..63 are zero.
__global__ void rgb_im2col_kernel(const uint8_t *rgb, int h, int w, __nv_bfloat16 *out, int planes)
{
    const long long pixels = static_cast<long long>(h) * w;
    for (long long p = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; p < pixels;
         p += static_cast<long long>(gridDim.x) * blockDim.x)
    {
        const int y = static_cast<int>(p / w), x = static_cast<int>(p - static_cast<long long>(y) * w);
        __nv_bfloat16 *dst = out + p * planes * 64;
#pragma unroll
        for (int g = 0; g < 8; ++g)
        {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
            {
                const int k = g * 8 + j;
                float value = 0.f;
                if (k < 27)
                {
                    const int t = k / 3, c = k % 3, yy = y + t / 3 - 1, xx = x + t % 3 - 1;
                    if (yy >= 0 && yy < h && xx >= 0 && xx < w)
                        value = __fmul_rn(__fsub_rn(static_cast<float>(rgb[(static_cast<long long>(yy) * w + xx) * 3 + c]),
                                                    127.5f),
                                          1.f / 127.5f);
                }
                v[j] = value;
            }
            store_planes8(dst + g * 8, 64, planes, v);
        }
    }
}

// OIHW [cout][cin][taps] -> [cout][taps * cin] (column t * cin + c).
__global__ void taps_inner_kernel(const float *w, int cout, int cin, int taps, float *out)
{
    const long long total = static_cast<long long>(cout) * cin * taps;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
    {
        const long long row = static_cast<long long>(taps) * cin;
        const long long o = i / row;
        const int r = static_cast<int>(i - o * row), t = r / cin, c = r - t * cin;
        out[i] = w[(o * cin + c) * taps + t];
    }
}

// Space-to-depth operand of a stride-2 convolution: pixel (y, x) of FP32 NHWC x goes to
// [(y / 2) * (w / 2) + x / 2][phase = (y & 1) * 2 + (x & 1)][plane][c] as BF16 plane(s).
__global__ void s2d_operand_kernel(const float *x, int h, int w, int channels, __nv_bfloat16 *out, int planes)
{
    const int per_pixel = channels / 8;
    const long long total = static_cast<long long>(h) * w * per_pixel;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
    {
        const long long p = i / per_pixel;
        const int c0 = static_cast<int>(i - p * per_pixel) * 8;
        const int yy = static_cast<int>(p / w), xx = static_cast<int>(p - static_cast<long long>(yy) * w);
        const float4 *src = reinterpret_cast<const float4 *>(x + p * channels + c0);
        const float4 a = src[0], b = src[1];
        const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        const long long q = static_cast<long long>(yy >> 1) * (w >> 1) + (xx >> 1);
        const int phase = (yy & 1) * 2 + (xx & 1);
        store_planes8(out + (q * 4 + phase) * planes * channels + c0, channels, planes, v);
    }
}

// The encoder's tail (tools/export_vae_encoder.py:74-80): quant_conv in FP32 keeping the posterior's mode
// (outputs 0..31), pixel_unshuffle(2) and the affine-free BatchNorm in eval mode, one thread per pixel of
// the mean. normalized = (packed - running_mean) * (1 / sqrt(running_var + eps)).
__global__ void encoder_output_kernel(const float *hin, int ldh, int h, int w, const float *wq, const float *bq,
                                      const float *rm, const float *rv, float eps, float *mean, float *packed,
                                      float *normalized, int *nonfinite)
{
    __shared__ float ws[32 * 64], bs[32], ms[128], is[128];
    for (int i = threadIdx.x; i < 32 * 64; i += blockDim.x) ws[i] = wq[i];
    if (threadIdx.x < 32) bs[threadIdx.x] = bq[threadIdx.x];
    if (threadIdx.x < 128)
    {
        ms[threadIdx.x] = rm[threadIdx.x];
        is[threadIdx.x] = __frcp_rn(__fsqrt_rn(__fadd_rn(rv[threadIdx.x], eps)));
    }
    __syncthreads();
    const long long pixels = static_cast<long long>(h) * w;
    const int w2 = w / 2;
    const long long plane2 = static_cast<long long>(h / 2) * w2;
    for (long long p = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; p < pixels;
         p += static_cast<long long>(gridDim.x) * blockDim.x)
    {
        const int y = static_cast<int>(p / w), x = static_cast<int>(p - static_cast<long long>(y) * w);
        float in[64];
        const float4 *src = reinterpret_cast<const float4 *>(hin + p * ldh);
#pragma unroll
        for (int k = 0; k < 16; ++k)
        {
            const float4 v = src[k];
            in[4 * k] = v.x;
            in[4 * k + 1] = v.y;
            in[4 * k + 2] = v.z;
            in[4 * k + 3] = v.w;
        }
        const long long q = static_cast<long long>(y >> 1) * w2 + (x >> 1);
        const int phase = (y & 1) * 2 + (x & 1);
        bool finite = true;
#pragma unroll 4
        for (int c = 0; c < 32; ++c)
        {
            float acc = bs[c];
#pragma unroll
            for (int k = 0; k < 64; ++k) acc = fmaf(ws[c * 64 + k], in[k], acc);
            const int pc = c * 4 + phase;
            const float n = __fmul_rn(__fsub_rn(acc, ms[pc]), is[pc]);
            mean[c * pixels + p] = acc;
            packed[pc * plane2 + q] = acc;
            normalized[pc * plane2 + q] = n;
            finite = finite && isfinite(acc) && isfinite(n);
        }
        if (!finite && nonfinite) atomicOr(nonfinite, 1);
    }
}

// post_quant_conv (1x1, 32 -> 32, FP32) on the unpacked latent [32][pixels], written as the conv_in
// operand [pixels][planes * 64] (channels 32..63 zero).
__global__ void vae_input_kernel(const float *unpacked, long long pixels, const float *w, const float *bias,
                                 __nv_bfloat16 *out, int planes)
{
    __shared__ float ws[32 * 32], bs[32];
    for (int i = threadIdx.x; i < 32 * 32; i += blockDim.x) ws[i] = w[i];
    if (threadIdx.x < 32) bs[threadIdx.x] = bias[threadIdx.x];
    __syncthreads();
    for (long long p = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; p < pixels;
         p += static_cast<long long>(gridDim.x) * blockDim.x)
    {
        float u[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) u[c] = unpacked[c * pixels + p];
        float z[8];
        __nv_bfloat16 *dst = out + p * planes * 64;
#pragma unroll 1
        for (int o0 = 0; o0 < 32; o0 += 8)
        {
#pragma unroll
            for (int j = 0; j < 8; ++j)
            {
                float acc = bs[o0 + j];
#pragma unroll
                for (int c = 0; c < 32; ++c) acc = fmaf(ws[(o0 + j) * 32 + c], u[c], acc);
                z[j] = acc;
            }
            store_planes8(dst + o0, 64, planes, z);
        }
        const float zero[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int o0 = 32; o0 < 64; o0 += 8) store_planes8(dst + o0, 64, planes, zero);
    }
}

// Row softmax with the row in registers (n <= 2048 * EPT4 keys, 512 threads): FP32 max and exp, per-thread
// FP32 partial sums reduced in FP64; P = e * (1 / sum) as BF16 planes [rows][planes * ldp], zero from n.
template <int EPT4>
__global__ void __launch_bounds__(512) softmax_rows_reg_kernel(const float *s, int lds, int n, float scale,
                                                               __nv_bfloat16 *p, int ldp, int planes)
{
    __shared__ float red_max[16];
    __shared__ double red_sum[16];
    const long long r = blockIdx.x;
    const float4 *src = reinterpret_cast<const float4 *>(s + r * lds);
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    float4 v[EPT4];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < EPT4; ++k)
    {
        const int i = 4 * (k * 512 + tid);
        float4 t = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        if (i + 3 < n) t = src[k * 512 + tid];
        else if (i < n)
        {
            t.x = s[r * lds + i];
            if (i + 1 < n) t.y = s[r * lds + i + 1];
            if (i + 2 < n) t.z = s[r * lds + i + 2];
        }
        v[k] = t;
        m = fmaxf(m, fmaxf(fmaxf(t.x, t.y), fmaxf(t.z, t.w)));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red_max[warp] = m;
    __syncthreads();
    m = red_max[0];
#pragma unroll
    for (int w = 1; w < 16; ++w) m = fmaxf(m, red_max[w]);
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < EPT4; ++k)
    {
        float4 &t = v[k];
        t.x = expf(__fmul_rn(t.x - m, scale)); // masked keys: exp(-inf) = 0
        t.y = expf(__fmul_rn(t.y - m, scale));
        t.z = expf(__fmul_rn(t.z - m, scale));
        t.w = expf(__fmul_rn(t.w - m, scale));
        sum += (t.x + t.y) + (t.z + t.w);
    }
    double total = warp_sum(static_cast<double>(sum));
    if (lane == 0) red_sum[warp] = total;
    __syncthreads();
    total = 0.0;
#pragma unroll
    for (int w = 0; w < 16; ++w) total += red_sum[w];
    const float inv = static_cast<float>(1.0 / total);
    __nv_bfloat16 *dst = p + r * planes * ldp;
#pragma unroll
    for (int k = 0; k < EPT4; ++k)
    {
        const int i = 4 * (k * 512 + tid);
        if (i >= ldp) break;
        const float e[4] = {v[k].x * inv, v[k].y * inv, v[k].z * inv, v[k].w * inv};
        if (planes == 1)
        {
            __nv_bfloat162 h[2] = {__floats2bfloat162_rn(e[0], e[1]), __floats2bfloat162_rn(e[2], e[3])};
            *reinterpret_cast<uint2 *>(dst + i) = *reinterpret_cast<const uint2 *>(h);
        }
        else
        {
            __align__(8) __nv_bfloat16 q[3][4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
            {
                float hi, mid, lo;
                split3f(e[j], hi, mid, lo);
                q[0][j] = __float2bfloat16_rn(hi);
                q[1][j] = __float2bfloat16_rn(mid);
                q[2][j] = __float2bfloat16_rn(lo);
            }
#pragma unroll
            for (int pl = 0; pl < 3; ++pl)
                *reinterpret_cast<uint2 *>(dst + pl * ldp + i) = *reinterpret_cast<const uint2 *>(q[pl]);
        }
    }
}

// Row softmax of S * scale over the first n columns: FP32 max and exp, FP64 sum; P written as BF16 planes
// [rows][planes * ldp] (columns n..ldp-1 zero). One CTA per row, the row staged in shared memory.
__global__ void softmax_rows_kernel(const float *s, int lds, int n, float scale, __nv_bfloat16 *p, int ldp,
                                    int planes)
{
    extern __shared__ float row[];
    __shared__ float red_max[32];
    __shared__ double red_sum[32];
    const long long r = blockIdx.x;
    const float *src = s + r * lds;
    float m = -INFINITY;
    for (int i = threadIdx.x; i < n; i += blockDim.x)
    {
        const float v = src[i];
        row[i] = v;
        m = fmaxf(m, v);
    }
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, warps = blockDim.x / 32;
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red_max[warp] = m;
    __syncthreads();
    m = red_max[0];
    for (int w = 1; w < warps; ++w) m = fmaxf(m, red_max[w]);
    double sum = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x)
    {
        const float e = expf(__fmul_rn(row[i] - m, scale));
        row[i] = e;
        sum += e;
    }
    sum = warp_sum(sum);
    if (lane == 0) red_sum[warp] = sum;
    __syncthreads();
    double total = 0.0;
    for (int w = 0; w < warps; ++w) total += red_sum[w];
    const double inv = 1.0 / total;
    __nv_bfloat16 *dst = p + r * planes * ldp;
    for (int i0 = threadIdx.x * 8; i0 < ldp; i0 += blockDim.x * 8)
    {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = i0 + j < n ? static_cast<float>(row[i0 + j] * inv) : 0.f;
        store_planes8(dst + i0, ldp, planes, v);
    }
}

// [n][3 * 512] FP32 q|k|v -> Q [n][planes * 512], K [n][planes * 512] and V^T [512][planes * ldv].
__global__ void attention_split_kernel(const float *qkv, int n, __nv_bfloat16 *q, __nv_bfloat16 *k,
                                       __nv_bfloat16 *vt, int ldv, int planes)
{
    constexpr int D = 512;
    // Q and K: 8 channels per thread
    const long long total = static_cast<long long>(n) * (2 * D / 8);
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
    {
        const long long t = i / (2 * D / 8);
        const int c0 = static_cast<int>(i - t * (2 * D / 8)) * 8;
        const float4 *src = reinterpret_cast<const float4 *>(qkv + t * 3 * D + c0);
        const float4 a = src[0], b = src[1];
        const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        if (c0 < D) store_planes8(q + t * planes * D + c0, D, planes, v);
        else store_planes8(k + t * planes * D + (c0 - D), D, planes, v);
    }
}

// V^T through 32 x 32 shared-memory tiles: vt[c][plane * ldv + t] = plane(v[t][c]).
__global__ void transpose_v_kernel(const float *qkv, int n, __nv_bfloat16 *vt, int ldv, int planes)
{
    constexpr int D = 512;
    __shared__ float tile[32][33];
    const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += blockDim.y)
    {
        const int t = t0 + j;
        tile[j][threadIdx.x] = t < n ? qkv[static_cast<long long>(t) * 3 * D + 2 * D + c0 + threadIdx.x] : 0.f;
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += blockDim.y)
    {
        const int t = t0 + threadIdx.x;
        if (t >= n) continue;
        const float x = tile[threadIdx.x][j];
        __nv_bfloat16 *dst = vt + static_cast<long long>(c0 + j) * planes * ldv + t;
        if (planes == 1) dst[0] = __float2bfloat16_rn(x);
        else
        {
            float hi, mid, lo;
            split3f(x, hi, mid, lo);
            dst[0] = __float2bfloat16_rn(hi);
            dst[ldv] = __float2bfloat16_rn(mid);
            dst[2 * ldv] = __float2bfloat16_rn(lo);
        }
    }
}

// OIHW FP32 [cout][cin][taps] -> [cout_rows][3][taps][cin_pad] BF16 planes (hi, mid, lo); rows and channels
// past the tensor are zero. *inexact is set when any weight is not a BF16 value.
__global__ void conv_weight_prep_kernel(const float *w, int cout, int cin, int taps, int cout_rows, int cin_pad,
                                        __nv_bfloat16 *out, int *inexact)
{
    const long long k = static_cast<long long>(taps) * cin_pad;
    const long long total = static_cast<long long>(cout_rows) * k;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
    {
        const long long o = i / k;
        const int rem = static_cast<int>(i - o * k), t = rem / cin_pad, c = rem - t * cin_pad;
        const float x = (o < cout && c < cin) ? w[(o * cin + c) * taps + t] : 0.f;
        float hi, mid, lo;
        split3f(x, hi, mid, lo);
        __nv_bfloat16 *row = out + o * 3 * k;
        row[rem] = __float2bfloat16_rn(hi);
        row[k + rem] = __float2bfloat16_rn(mid);
        row[2 * k + rem] = __float2bfloat16_rn(lo);
        if (mid != 0.f || lo != 0.f) *inexact = 1;
    }
}

// conv_out from its tap-expanded 1x1 product p [pixels][32] (column t * 3 + c = tap t of output channel c):
// out[c][y][x] = bias[c] + sum over the 3x3 taps inside the image of p[(y + dy, x + dx)][t * 3 + c], written as
// the planar FP32 image [3][pixels] and the RGB bytes of rgb_image (src/pipeline.cpp:145-163).
__global__ void conv_out_gather_kernel(const float *p, int h, int w, const float *bias, float *planar, uint8_t *rgb,
                                       int *nonfinite)
{
    const long long pixels = static_cast<long long>(h) * w;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < pixels;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
    {
        const int y = static_cast<int>(i / w), x = static_cast<int>(i - static_cast<long long>(y) * w);
        float acc[3] = {0.f, 0.f, 0.f};
#pragma unroll
        for (int t = 0; t < 9; ++t)
        {
            const int yy = y + t / 3 - 1, xx = x + t % 3 - 1;
            if (yy < 0 || yy >= h || xx < 0 || xx >= w) continue;
            const float *src = p + (static_cast<long long>(yy) * w + xx) * 32 + t * 3;
#pragma unroll
            for (int c = 0; c < 3; ++c) acc[c] += src[c];
        }
        bool finite = true;
#pragma unroll
        for (int c = 0; c < 3; ++c)
        {
            const float v = bias[c] + acc[c];
            planar[c * pixels + i] = v;
            if (!isfinite(v))
            {
                finite = false;
                continue;
            }
            if (rgb)
            {
                const float n = fminf(fmaxf(__fadd_rn(__fmul_rn(v, 0.5f), 0.5f), 0.f), 1.f);
                rgb[i * 3 + c] = static_cast<uint8_t>(rintf(__fmul_rn(n, 255.f)));
            }
        }
        if (!finite && nonfinite) atomicOr(nonfinite, 1);
    }
}

// OIHW [cout][cin][9] -> tap-expanded 1x1 weights [9 * cout][cin] (row t * cout + c = tap t of output c).
__global__ void expand_taps_kernel(const float *w, int cout, int cin, float *out)
{
    const int total = 9 * cout * cin;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x)
    {
        const int row = i / cin, ch = i - row * cin, t = row / cout, c = row - t * cout;
        out[i] = w[(c * cin + ch) * 9 + t];
    }
}

// float(N(0,1) * scale) + offset for (seed, stream, i) (include/ernie_synth.h), optionally rounded to BF16.
__global__ void synth_f32_kernel(uint64_t seed, uint64_t stream_id, float scale, float offset, long long count,
                                 int round_bf16, float *out)
{
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
    {
        const float v = static_cast<float>(ernie_synth_normal(seed, stream_id, static_cast<uint64_t>(i)) *
                                           static_cast<double>(scale)) +
                        offset;
        out[i] = round_bf16 ? ernie_synth_bf16_to_float(ernie_synth_bf16_bits(v)) : v;
    }
}
} // namespace

int prepare_conv_kernels()
{
    cudaError_t e = ensure_conv_attributes<256, false, 1>();
    if (e == cudaSuccess) e = ensure_conv_attributes<128, false, 2>();
    if (e == cudaSuccess) e = ensure_conv_attributes<32, false, 2>();
    if (e == cudaSuccess) e = ensure_conv_attributes<128, true, 1>();
    if (e == cudaSuccess) e = ensure_conv_attributes<32, true, 2>();
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(softmax_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSoftmaxMaxRow * 4);
    return e;
}

int conv_group(int k_blocks)
{
    for (int g = 4; g > 1; --g)
        if (k_blocks % g == 0) return g;
    return 1;
}

int conv_stat_slots(const ConvLaunch &l, int num_sms) { return kEpiWarps * conv_grid(l, num_sms); }

int launch_conv(const ConvLaunch &l, const ConvArgs &epi, int num_sms, cudaStream_t stream)
{
    if (!l.a || !l.b || l.height < 1 || l.width < 1 || l.cin < CK || l.cin % CK || (l.taps != 1 && l.taps != 9) ||
        (l.a_planes != 1 && l.a_planes != 3) || (l.b_planes != 1 && l.b_planes != 3) || num_sms < 1)
        return cudaErrorInvalidValue;
    if (l.b_row < static_cast<long long>(l.b_planes) * l.taps * l.cin || l.cout_rows < l.cout) return cudaErrorInvalidValue;
    if (l.stride2 && l.taps != 9) return cudaErrorInvalidValue;
    const bool promote = l.a_planes == 3;
    if (!promote && l.b_planes != 1) return cudaErrorInvalidValue;
    ConvArgs args = epi;
    args.height = l.height;
    args.width = l.width;
    args.cin = l.cin;
    args.taps = l.taps;
    args.cout = l.cout;
    args.stride2 = l.stride2 ? 1 : 0;
    args.phase_stride = l.a_planes * l.cin;
    args.products = promote ? (l.b_planes == 3 ? 6 : 3) : 1;
    args.group = conv_group(l.taps * l.cin / CK);
    if (args.stats && args.cpg != 4 && args.cpg != 8 && args.cpg != 16) return cudaErrorInvalidValue;
    if ((args.out || args.resid) && (args.ldo < l.cout || args.ldo % 4)) return cudaErrorInvalidValue;
    if (l.cout == 32) return promote ? launch_conv_impl<32, true, 2>(l, args, num_sms, stream)
                                     : launch_conv_impl<32, false, 2>(l, args, num_sms, stream);
    if (l.cout % 128) return cudaErrorInvalidValue;
    if (promote) return launch_conv_impl<128, true, 1>(l, args, num_sms, stream);
    if (l.cout % 256 == 0) return launch_conv_impl<256, false, 1>(l, args, num_sms, stream);
    return launch_conv_impl<128, false, 2>(l, args, num_sms, stream);
}

int launch_gn_finalize(const double2 *stats, int slots, long long count, int cpg, const float *gamma,
                       const float *beta, float eps, float *scale, float *shift, cudaStream_t stream)
{
    if (cpg < 1 || cpg > 256 || slots < 1 || count < 1) return cudaErrorInvalidValue;
    gn_finalize_kernel<<<32, 256, 0, stream>>>(stats, slots, count, cpg, gamma, beta, eps, scale, shift);
    return cudaGetLastError();
}

int launch_gn_apply(const float *x, long long pixels, int channels, const float *scale, const float *shift, int silu,
                    __nv_bfloat16 *out, int planes, cudaStream_t stream, __nv_bfloat16 *raw)
{
    if (channels < 8 || (channels & (channels - 1)) || pixels < 1 || (planes != 1 && planes != 3))
        return cudaErrorInvalidValue;
    int log2c = 0;
    while ((1 << log2c) < channels) ++log2c;
    gn_apply_kernel<<<grid_for_count(pixels * channels / 8, 256), 256, 0, stream>>>(x, pixels, log2c, scale, shift,
                                                                                    silu, out, raw, planes);
    return cudaGetLastError();
}

int launch_upsample(const float *x, int h, int w, int channels, __nv_bfloat16 *out, int planes, cudaStream_t stream)
{
    if (channels % 8 || h < 1 || w < 1) return cudaErrorInvalidValue;
    upsample_kernel<<<grid_for_count(static_cast<long long>(h) * w * channels / 8, 256), 256, 0, stream>>>(
        x, h, w, channels, out, planes);
    return cudaGetLastError();
}

int launch_vae_input(const float *unpacked, long long pixels, const float *w, const float *bias, __nv_bfloat16 *out,
                     int planes, cudaStream_t stream)
{
    if (pixels < 1) return cudaErrorInvalidValue;
    vae_input_kernel<<<grid_for_count(pixels, 128), 128, 0, stream>>>(unpacked, pixels, w, bias, out, planes);
    return cudaGetLastError();
}

int launch_softmax_rows(const float *s, int rows, int lds, int n, float scale, __nv_bfloat16 *p, int ldp, int planes,
                        cudaStream_t stream)
{
    if (n < 1 || n > kSoftmaxMaxRow || ldp % 8 || ldp < n || lds < n || lds % 4) return cudaErrorInvalidValue;
    if (ldp <= 16384)
        softmax_rows_reg_kernel<8><<<rows, 512, 0, stream>>>(s, lds, n, scale, p, ldp, planes);
    else if (ldp <= 32768)
        softmax_rows_reg_kernel<16><<<rows, 512, 0, stream>>>(s, lds, n, scale, p, ldp, planes);
    else
        softmax_rows_kernel<<<rows, 512, static_cast<size_t>(n) * 4, stream>>>(s, lds, n, scale, p, ldp, planes);
    return cudaGetLastError();
}

int launch_attention_split(const float *qkv, int n, __nv_bfloat16 *q, __nv_bfloat16 *k, __nv_bfloat16 *vt, int ldv,
                           int planes, cudaStream_t stream)
{
    if (n < 1 || ldv < n || ldv % 8) return cudaErrorInvalidValue;
    attention_split_kernel<<<grid_for_count(static_cast<long long>(n) * 128, 256), 256, 0, stream>>>(qkv, n, q, k, vt,
                                                                                                    ldv, planes);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    transpose_v_kernel<<<dim3((n + 31) / 32, 512 / 32), dim3(32, 8), 0, stream>>>(qkv, n, vt, ldv, planes);
    return cudaGetLastError();
}

int launch_rgb_im2col(const uint8_t *rgb, int h, int w, __nv_bfloat16 *out, int planes, cudaStream_t stream)
{
    if (!rgb || !out || h < 1 || w < 1 || (planes != 1 && planes != 3)) return cudaErrorInvalidValue;
    rgb_im2col_kernel<<<grid_for_count(static_cast<long long>(h) * w, 128), 128, 0, stream>>>(rgb, h, w, out, planes);
    return cudaGetLastError();
}

int launch_taps_inner(const float *w, int cout, int cin, int taps, float *out, cudaStream_t stream)
{
    if (!w || !out || cout < 1 || cin < 1 || taps < 1) return cudaErrorInvalidValue;
    taps_inner_kernel<<<grid_for_count(static_cast<long long>(cout) * cin * taps, 256), 256, 0, stream>>>(w, cout, cin,
                                                                                                        taps, out);
    return cudaGetLastError();
}

int launch_s2d_operand(const float *x, int h, int w, int channels, __nv_bfloat16 *out, int planes,
                       cudaStream_t stream)
{
    if (!x || !out || h < 2 || w < 2 || (h & 1) || (w & 1) || channels < 8 || channels % 8 ||
        (planes != 1 && planes != 3))
        return cudaErrorInvalidValue;
    s2d_operand_kernel<<<grid_for_count(static_cast<long long>(h) * w * channels / 8, 256), 256, 0, stream>>>(
        x, h, w, channels, out, planes);
    return cudaGetLastError();
}

int launch_encoder_output(const float *hin, int ldh, int h, int w, const float *wq, const float *bq, const float *rm,
                          const float *rv, float eps, float *mean, float *packed, float *normalized, int *nonfinite,
                          cudaStream_t stream)
{
    if (!hin || !wq || !bq || !rm || !rv || !mean || !packed || !normalized || ldh < 64 || ldh % 4 || h < 2 ||
        w < 2 || (h & 1) || (w & 1))
        return cudaErrorInvalidValue;
    encoder_output_kernel<<<grid_for_count(static_cast<long long>(h) * w, 128), 128, 0, stream>>>(
        hin, ldh, h, w, wq, bq, rm, rv, eps, mean, packed, normalized, nonfinite);
    return cudaGetLastError();
}

int launch_conv_weight_prep(const float *w, int cout, int cin, int taps, int cout_rows, int cin_pad,
                            __nv_bfloat16 *out, int *inexact, cudaStream_t stream)
{
    if (cout < 1 || cin < 1 || cout_rows < cout || cin_pad < cin || (taps != 1 && taps != 9))
        return cudaErrorInvalidValue;
    conv_weight_prep_kernel<<<grid_for_count(static_cast<long long>(cout_rows) * taps * cin_pad, 256), 256, 0,
                              stream>>>(w, cout, cin, taps, cout_rows, cin_pad, out, inexact);
    return cudaGetLastError();
}

int launch_conv_out_gather(const float *p, int h, int w, const float *bias, float *planar, uint8_t *rgb, int *nonfinite,
                           cudaStream_t stream)
{
    if (h < 1 || w < 1) return cudaErrorInvalidValue;
    conv_out_gather_kernel<<<grid_for_count(static_cast<long long>(h) * w, 256), 256, 0, stream>>>(p, h, w, bias, planar,
                                                                                                   rgb, nonfinite);
    return cudaGetLastError();
}

int launch_expand_taps(const float *w, int cout, int cin, float *out, cudaStream_t stream)
{
    if (cout < 1 || cin < 1) return cudaErrorInvalidValue;
    expand_taps_kernel<<<grid_for_count(9LL * cout * cin, 256), 256, 0, stream>>>(w, cout, cin, out);
    return cudaGetLastError();
}

int launch_synth_f32(uint64_t seed, uint64_t stream_id, float scale, float offset, long long count, int round_bf16,
                     float *out, cudaStream_t stream)
{
    synth_f32_kernel<<<grid_for_count(count, 256), 256, 0, stream>>>(seed, stream_id, scale, offset, count,
                                                                     round_bf16, out);
    return cudaGetLastError();
}
} // namespace ernie_b200
