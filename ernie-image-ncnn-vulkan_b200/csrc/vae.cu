// The VAE decoder's kernels for sm_100a: a tcgen05 implicit-GEMM convolution and the bandwidth-bound
// GroupNorm / SiLU / upsample / softmax passes around it.
//
// Replaces the ncnn layers of the reference's decoder graph (AutoencoderKLFlux2 post_quant_conv +
// decoder, exported by tools/export_vae.py and run by src/vae.cpp:18-66):
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

namespace ernie_b200
{
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

namespace
{
constexpr int CM = 128, CK = 64, kConvThreads = 192;
enum : int
{
    kErrConvProducerTimeout = 31,
    kErrConvMmaTimeout = 32,
    kErrConvEpilogueTimeout = 33,
};

template <int BN, bool PROMOTE> struct ConvCfg
{
    static_assert(BN == 16 || BN == 128 || BN == 256, "tile widths");
    static_assert(!PROMOTE || BN <= 128, "FP32 promotion keeps a BN-column running sum per thread");
    static constexpr int kStages = BN == 256 ? 4 : BN == 128 ? 6 : 8;
    static constexpr int kABytes = CM * CK * 2;
    static constexpr int kBBytes = BN * CK * 2;
    static constexpr int kStageBytes = kABytes + kBBytes; // a multiple of 1024 for every BN
    static constexpr int kUsedCols = PROMOTE ? 3 * BN : 2 * BN;
    static constexpr int kTmemCols = kUsedCols <= 32    ? 32
                                     : kUsedCols <= 64  ? 64
                                     : kUsedCols <= 128 ? 128
                                     : kUsedCols <= 256 ? 256
                                                        : 512;
    static constexpr int kChunk = BN >= 32 ? 32 : 16;
    static constexpr int kBarrierBytes = 256;
    static constexpr int kSmemBytes = kStages * kStageBytes + kBarrierBytes + 1024;
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

// GroupNorm partials of one chunk: per group of CPG channels, the warp's (sum, sum of squares) over its
// 32 pixels in FP64, stored at stats[group][row_block] (every slot written once: deterministic).
template <int CH, int CPG>
__device__ __forceinline__ void chunk_stats(const float (&v)[CH], bool valid, int col, int row_block,
                                            int row_blocks, int lane, double2 *stats)
{
#pragma unroll
    for (int g = 0; g < CH / CPG; ++g)
    {
        double s = 0.0, q = 0.0;
        if (valid)
        {
#pragma unroll
            for (int j = 0; j < CPG; ++j)
            {
                const double d = v[g * CPG + j];
                s += d;
                q = fma(d, d, q);
            }
        }
        s = warp_sum(s);
        q = warp_sum(q);
        if (lane == 0) stats[static_cast<size_t>(col / CPG + g) * row_blocks + row_block] = make_double2(s, q);
    }
}

template <int CH>
__device__ __forceinline__ void conv_chunk(float (&v)[CH], int col, bool valid, long long pixel, long long pixels,
                                           int row_block, int row_blocks, int lane, const ConvArgs &a)
{
    if (a.bias)
    {
#pragma unroll
        for (int j = 0; j < CH; ++j) v[j] += __ldg(a.bias + col + j);
    }
    if (a.planar)
    {
        // conv_out: planar FP32 [valid_out][pixels] and the RGB bytes of src/pipeline.cpp:145-163
        if (valid)
        {
#pragma unroll
            for (int j = 0; j < CH; ++j)
                if (col + j < a.valid_out)
                {
                    const float x = v[j];
                    a.planar[static_cast<size_t>(col + j) * pixels + pixel] = x;
                    if (!isfinite(x))
                    {
                        if (a.nonfinite) atomicOr(a.nonfinite, 1);
                    }
                    else if (a.rgb)
                    {
                        const float n = fminf(fmaxf(__fadd_rn(__fmul_rn(x, 0.5f), 0.5f), 0.f), 1.f);
                        a.rgb[static_cast<size_t>(pixel) * a.valid_out + col + j] =
                            static_cast<uint8_t>(rintf(__fmul_rn(n, 255.f)));
                    }
                }
        }
        return;
    }
    if (valid && a.resid)
    {
        const float4 *r = reinterpret_cast<const float4 *>(a.resid + pixel * a.ldo + col);
#pragma unroll
        for (int j = 0; j < CH / 4; ++j)
        {
            const float4 t = r[j];
            v[4 * j] += t.x;
            v[4 * j + 1] += t.y;
            v[4 * j + 2] += t.z;
            v[4 * j + 3] += t.w;
        }
    }
    if (valid && a.out)
    {
        float4 *o = reinterpret_cast<float4 *>(a.out + pixel * a.ldo + col);
#pragma unroll
        for (int j = 0; j < CH / 4; ++j) o[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
    if (a.stats)
    {
        switch (a.cpg)
        {
        case 4: chunk_stats<CH, 4>(v, valid, col, row_block, row_blocks, lane, a.stats); break;
        case 8: chunk_stats<CH, 8>(v, valid, col, row_block, row_blocks, lane, a.stats); break;
        default: chunk_stats<CH, 16>(v, valid, col, row_block, row_blocks, lane, a.stats); break;
        }
    }
}

template <int BN, bool PROMOTE>
__global__ void __launch_bounds__(kConvThreads, 1)
    conv_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, ConvArgs args)
{
    using C = ConvCfg<BN, PROMOTE>;
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
    auto tile_a = [&](int s) { return base + s * C::kStageBytes; };
    auto tile_b = [&](int s) { return base + s * C::kStageBytes + C::kABytes; };

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int tiles_x = (args.width + CM - 1) / CM, m_tiles = args.height * tiles_x;
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
            mbar_init(tempty_bar(i), 4);
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
                const int y = m_blk / tiles_x, x0 = (m_blk - y * tiles_x) * CM;
                for (int kb = 0; kb < k_blocks && ok; ++kb)
                {
                    const int tap = kb / cblk, c0 = (kb - tap * cblk) * CK;
                    const int dy = args.taps == 9 ? tap / 3 - 1 : 0, dx = args.taps == 9 ? tap % 3 - 1 : 0;
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
                        tma_load_3d(tile_a(stage), &map_a, full_bar(stage), pa * args.cin + c0, x0 + dx, y + dy);
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
                    const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
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
                            const uint64_t a_desc = smem_desc_sw128(tile_a(stage));
                            const uint64_t b_desc = smem_desc_sw128(tile_b(stage));
#pragma unroll
                            for (int k = 0; k < CK / 16; ++k)
                                umma_bf16(d_tmem, a_desc + 2u * k, b_desc + 2u * k, idesc,
                                          (kb != kb0 || p != 0 || k != 0) ? 1u : 0u);
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
        constexpr int CH = C::kChunk;
        const int quarter = warp & 3;
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        const long long pixels = static_cast<long long>(args.height) * args.width;
        const int row_blocks = m_tiles * 4;
        int unit = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x)
        {
            const int m_blk = tile / n_tiles, n_blk = tile - m_blk * n_tiles;
            const int y = m_blk / tiles_x, x = (m_blk - y * tiles_x) * CM + quarter * 32 + lane;
            const bool valid = x < args.width;
            const long long pixel = static_cast<long long>(y) * args.width + x;
            const int row_block = m_blk * 4 + quarter;
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
#pragma unroll 1
                for (int c = 0; c < BN; c += CH)
                {
                    float v[CH];
                    if constexpr (CH == 32) tmem_load_32(lane_base + acc * BN + c, v);
                    else tmem_load_16(lane_base + acc * BN + c, v);
                    conv_chunk<CH>(v, n_blk * BN + c, valid, pixel, pixels, row_block, row_blocks, lane, args);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(tempty_bar(acc));
                ++unit;
            }
            else
            {
                float sum[BN];
#pragma unroll
                for (int j = 0; j < BN; ++j) sum[j] = 0.f;
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
                    for (int c = 0; c < BN; c += CH)
                    {
                        float v[CH];
                        if constexpr (CH == 32) tmem_load_32(lane_base + acc * BN + c, v);
                        else tmem_load_16(lane_base + acc * BN + c, v);
#pragma unroll
                        for (int j = 0; j < CH; ++j) sum[c + j] += v[j];
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(tempty_bar(acc));
                }
                if (!ok) break;
#pragma unroll
                for (int c = 0; c < BN; c += CH)
                {
                    float v[CH];
#pragma unroll
                    for (int j = 0; j < CH; ++j) v[j] = sum[c + j];
                    conv_chunk<CH>(v, n_blk * BN + c, valid, pixel, pixels, row_block, row_blocks, lane, args);
                }
            }
        }
    }
    __syncthreads();
    if (warp == 1)
    {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::kTmemCols);
    }
}

template <int BN, bool PROMOTE> cudaError_t ensure_conv_attributes()
{
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(conv_kernel<BN, PROMOTE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    ConvCfg<BN, PROMOTE>::kSmemBytes);
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

template <int BN, bool PROMOTE> int launch_conv_impl(const ConvLaunch &l, ConvArgs args, int num_sms, cudaStream_t stream)
{
    const cudaError_t attr = ensure_conv_attributes<BN, PROMOTE>();
    if (attr != cudaSuccess) return attr;
    CUtensorMap map_a, map_b;
    if (!make_operand_map(&map_a, l.a, static_cast<uint64_t>(l.a_planes) * l.cin, l.width, l.height) ||
        !make_weight_map(&map_b, l.b, static_cast<uint64_t>(l.cout_rows), static_cast<uint64_t>(l.b_row), BN))
        return cudaErrorInvalidValue;
    const long long tiles =
        static_cast<long long>(l.height) * ((l.width + CM - 1) / CM) * (l.cout / BN);
    const int grid = tiles < num_sms ? static_cast<int>(tiles) : num_sms;
    conv_kernel<BN, PROMOTE><<<grid, kConvThreads, ConvCfg<BN, PROMOTE>::kSmemBytes, stream>>>(map_a, map_b, args);
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

__global__ void gn_finalize_kernel(const double2 *stats, int row_blocks, long long count, int cpg,
                                   const float *gamma, const float *beta, float eps, float *scale, float *shift)
{
    __shared__ double part[2][32];
    const int g = blockIdx.x;
    double s = 0.0, q = 0.0;
    for (int i = threadIdx.x; i < row_blocks; i += blockDim.x)
    {
        const double2 v = stats[static_cast<size_t>(g) * row_blocks + i];
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
__global__ void gn_apply_kernel(const float *x, long long pixels, int channels, const float *scale,
                                const float *shift, int silu, __nv_bfloat16 *out, int planes)
{
    const int per_pixel = channels / 8;
    const long long total = pixels * per_pixel;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
    {
        const long long p = i / per_pixel;
        const int c0 = static_cast<int>(i - p * per_pixel) * 8;
        const float4 *src = reinterpret_cast<const float4 *>(x + p * channels + c0);
        const float4 a = src[0], b = src[1];
        float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int j = 0; j < 8; ++j)
        {
            float y = __fadd_rn(__fmul_rn(v[j], __ldg(scale + c0 + j)), __ldg(shift + c0 + j));
            if (silu) y = __fdiv_rn(y, __fadd_rn(1.f, expf(-y)));
            v[j] = y;
        }
        store_planes8(out + p * planes * channels + c0, channels, planes, v);
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
    cudaError_t e = ensure_conv_attributes<256, false>();
    if (e == cudaSuccess) e = ensure_conv_attributes<128, false>();
    if (e == cudaSuccess) e = ensure_conv_attributes<16, false>();
    if (e == cudaSuccess) e = ensure_conv_attributes<128, true>();
    if (e == cudaSuccess) e = ensure_conv_attributes<16, true>();
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

int launch_conv(const ConvLaunch &l, const ConvArgs &epi, int num_sms, cudaStream_t stream)
{
    if (!l.a || !l.b || l.height < 1 || l.width < 1 || l.cin < CK || l.cin % CK || (l.taps != 1 && l.taps != 9) ||
        (l.a_planes != 1 && l.a_planes != 3) || (l.b_planes != 1 && l.b_planes != 3) || num_sms < 1)
        return cudaErrorInvalidValue;
    if (l.b_row < static_cast<long long>(l.b_planes) * l.taps * l.cin || l.cout_rows < l.cout) return cudaErrorInvalidValue;
    const bool promote = l.a_planes == 3;
    if (!promote && l.b_planes != 1) return cudaErrorInvalidValue;
    ConvArgs args = epi;
    args.height = l.height;
    args.width = l.width;
    args.cin = l.cin;
    args.taps = l.taps;
    args.cout = l.cout;
    args.products = promote ? (l.b_planes == 3 ? 6 : 3) : 1;
    args.group = conv_group(l.taps * l.cin / CK);
    if (args.stats && args.cpg != 4 && args.cpg != 8 && args.cpg != 16) return cudaErrorInvalidValue;
    if (args.planar && l.cout != 16) return cudaErrorInvalidValue;
    if ((args.out || args.resid) && (args.ldo < l.cout || args.ldo % 4)) return cudaErrorInvalidValue;
    if (l.cout == 16) return promote ? launch_conv_impl<16, true>(l, args, num_sms, stream)
                                     : launch_conv_impl<16, false>(l, args, num_sms, stream);
    if (l.cout % 128) return cudaErrorInvalidValue;
    if (promote) return launch_conv_impl<128, true>(l, args, num_sms, stream);
    if (l.cout % 256 == 0) return launch_conv_impl<256, false>(l, args, num_sms, stream);
    return launch_conv_impl<128, false>(l, args, num_sms, stream);
}

int launch_gn_finalize(const double2 *stats, int row_blocks, long long count, int cpg, const float *gamma,
                       const float *beta, float eps, float *scale, float *shift, cudaStream_t stream)
{
    if (cpg < 1 || cpg > 256 || row_blocks < 1 || count < 1) return cudaErrorInvalidValue;
    gn_finalize_kernel<<<32, 256, 0, stream>>>(stats, row_blocks, count, cpg, gamma, beta, eps, scale, shift);
    return cudaGetLastError();
}

int launch_gn_apply(const float *x, long long pixels, int channels, const float *scale, const float *shift, int silu,
                    __nv_bfloat16 *out, int planes, cudaStream_t stream)
{
    if (channels % 8 || pixels < 1) return cudaErrorInvalidValue;
    gn_apply_kernel<<<grid_for_count(pixels * channels / 8, 256), 256, 0, stream>>>(x, pixels, channels, scale, shift,
                                                                                    silu, out, planes);
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
    if (n < 1 || n > kSoftmaxMaxRow || ldp % 8 || ldp < n || lds < n) return cudaErrorInvalidValue;
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

int launch_conv_weight_prep(const float *w, int cout, int cin, int taps, int cout_rows, int cin_pad,
                            __nv_bfloat16 *out, int *inexact, cudaStream_t stream)
{
    if (cout < 1 || cin < 1 || cout_rows < cout || cin_pad < cin || (taps != 1 && taps != 9))
        return cudaErrorInvalidValue;
    conv_weight_prep_kernel<<<grid_for_count(static_cast<long long>(cout_rows) * taps * cin_pad, 256), 256, 0,
                              stream>>>(w, cout, cin, taps, cout_rows, cin_pad, out, inexact);
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
