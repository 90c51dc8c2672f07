// Persistent, warp-specialised tcgen05 GEMM for sm_100a with the DiT block's fused epilogues.
//
// Replaces the ncnn `Gemm` layers of the reference block graph (block.ncnn.param:19,22,25,61,70,71,74)
// together with the elementwise layers that follow each of them:
//   Qkv        gemm_0/1/2 + reshape/permute + rmsn_9/rmsn_10 (qk-RMSNorm) + the rotary slice/mul/sub/add/concat
//              chain (:29-57), writing head-major Q/K/V for attention;
//   ResidGate  gemm_3 / gemm_6 + mul_15 / mul_21 (gate) + add_16 / add_22 (FP32 residual, ErnieResidualAdd);
//   Geglu      gemm_4 + gemm_5 + ErnieGELU + mul_20 over interleaved [up; gate] weights;
//   F32Bias    head projections (x_embedder conv1x1 + bias, text_proj);
//   FinalEuler output-head linear + bias + transpose to [128,h,w] + euler_step (src/latent_ops.cpp:72-92)
//              + the finite scan (src/latent_ops.cpp:60-70).
//
// Structure (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A [128 x 64] and B [BN x 64] BF16 tiles, 128-byte swizzle, S-stage ring
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer (M=128, N=BN, K=16 per instruction)
//   warps 2..5  epilogue: tcgen05.ld of the FP32 accumulator (one TMEM lane = one output row per
//               thread), fused math, global stores. Two TMEM accumulators let the epilogue of tile
//               i overlap the main loop of tile i+1.
#include "kernels.h"
#include "ptx.cuh"
#include "peer_sync.cuh"
#include <cudaTypedefs.h>
#include <mutex>

namespace ernie_b200
{
namespace
{
constexpr int BM = 128, BK = 64, kThreads = 192;
// Pair GEMMs split the tiles of a last round that would occupy at most half the pairs (a compile-time
// knob so that sweeps can compare against whole tiles).
#ifndef ERNIE_SPLIT_LAST_ROUND
#define ERNIE_SPLIT_LAST_ROUND 1
#endif
constexpr bool kSplitLastRound = ERNIE_SPLIT_LAST_ROUND != 0;

template <int BN, bool PROMOTE> struct Cfg
{
    static_assert(!PROMOTE || BN == 128, "FP32 promotion keeps a 128-column running sum per thread");
    static constexpr int kStages = BN == 256 ? 4 : 6;
    static constexpr int kABytes = BM * BK * 2;
    static constexpr int kBBytes = BN * BK * 2;
    static constexpr int kStageBytes = kABytes + kBBytes;
    // two accumulators (+ a 128-column result buffer when promoting), rounded to a power of two
    static constexpr int kTmemCols = PROMOTE ? 512 : 2 * BN;
    static constexpr int kBarrierBytes = 256;
    // per-epilogue-warp staging tile for coalesced global stores (FP32 [32][36] or BF16 [64][40])
    static constexpr int kStagingBytes = 5120;
    static constexpr int kStagingOffset = kStages * kStageBytes + kBarrierBytes;
    static constexpr int kSmemBytes = kStagingOffset + 4 * kStagingBytes + 1024;
};

__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * erfcf(-0.7071067811865475f * x); }

// The BF16 path's GELU: erfc(|x|/sqrt 2) by Abramowitz & Stegun 7.1.26 (|error| <= 1.5e-7), the form the
// reference's own GPU GELU evaluates (src/ernie_gelu.cpp:13-30); far below the BF16 rounding of h, and
// about half the instructions of erfcf.
__device__ __forceinline__ float gelu_as(float x)
{
    const float z = fabsf(x) * 0.7071067811865475f;
    const float t = __frcp_rn(fmaf(0.3275911f, z, 1.f));
    float poly = fmaf(1.061405429f, t, -1.453152027f);
    poly = fmaf(poly, t, 1.421413741f);
    poly = fmaf(poly, t, -0.284496736f);
    poly = fmaf(poly, t, 0.254829592f);
    const float tail = poly * t * __expf(-z * z);
    return x * (x >= 0.f ? 1.f - 0.5f * tail : 0.5f * tail);
}

__device__ __forceinline__ void split3(float x, __nv_bfloat16 &hi, __nv_bfloat16 &mid, __nv_bfloat16 &lo)
{
    hi = __float2bfloat16_rn(x);
    const float r1 = x - __bfloat162float(hi);
    mid = __float2bfloat16_rn(r1);
    const float r2 = r1 - __bfloat162float(mid);
    lo = __float2bfloat16_rn(r2);
}

// Plane p (0 hi, 1 mid, 2 lo) of x's three-BF16 split (x = hi + mid + lo to 24 significant bits); with
// one plane, plain BF16 rounding.
__device__ __forceinline__ float split_plane(float x, int p)
{
    const float hi = __bfloat162float(__float2bfloat16_rn(x));
    if (p == 0) return hi;
    const float r1 = x - hi, mid = __bfloat162float(__float2bfloat16_rn(r1));
    if (p == 1) return mid;
    return __bfloat162float(__float2bfloat16_rn(r1 - mid));
}

__device__ __forceinline__ void store_f32x4(float *dst, const float *v)
{
    *reinterpret_cast<float4 *>(dst) = make_float4(v[0], v[1], v[2], v[3]);
}

// ---- epilogues ---------------------------------------------------------------------------------
// Each epilogue warp owns 32 rows of the 128-row tile (its TMEM lane quarter); tcgen05.ld gives
// thread `lane` row row0 + lane. Stores that would be strided by a full output row per thread are
// staged through the warp's shared-memory tile and written as whole 64/128-byte row segments.
struct EpiCtx
{
    uint32_t taddr; // TMEM address of the accumulator (this warp's lane quarter, column 0)
    int row0;       // first output row of this warp
    int lane;
    int m;          // valid rows
    int n_blk;
    uint8_t *stage; // this warp's staging tile
};

__device__ __forceinline__ uint4 pack_bf16x8(const float *v)
{
    uint4 r;
    __nv_bfloat162 p0 = __floats2bfloat162_rn(v[0], v[1]), p1 = __floats2bfloat162_rn(v[2], v[3]);
    __nv_bfloat162 p2 = __floats2bfloat162_rn(v[4], v[5]), p3 = __floats2bfloat162_rn(v[6], v[7]);
    r.x = *reinterpret_cast<uint32_t *>(&p0);
    r.y = *reinterpret_cast<uint32_t *>(&p1);
    r.z = *reinterpret_cast<uint32_t *>(&p2);
    r.w = *reinterpret_cast<uint32_t *>(&p3);
    return r;
}

template <int BN> __device__ __forceinline__ void epi_f32_bias(const EpiCtx &e, const GemmEpilogueArgs &a)
{
    const int row = e.row0 + e.lane, col0 = e.n_blk * BN;
    const bool valid = row < e.m;
    float *out = a.out + static_cast<size_t>(row) * a.ldo + col0;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32)
    {
        float v[32];
        tmem_load_32(e.taddr + c, v);
        if (!valid) continue;
        if (a.bias)
        {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] += __ldg(a.bias + col0 + c + j);
        }
#pragma unroll
        for (int j = 0; j < 32; j += 4) store_f32x4(out + c + j, v + j);
    }
}

// ---- the norm folded into the GEMMs (BF16 DiT blocks) ---------------------------------------------
// rinv of `row` from its kFoldParts sums of squares, added in part order.
__device__ __forceinline__ float fold_rinv(const GemmEpilogueArgs &a, int row)
{
    float total = 0.f;
#pragma unroll 8
    for (int p = 0; p < kFoldParts; ++p) total += __ldg(a.fold_sumsq + static_cast<size_t>(p) * a.fold_ld + row);
    return 1.f / sqrtf(total / 4096.f + 1e-6f);
}

// v[j] = rinv * v[j] + bias[col + j] for the 32 accumulator columns starting at col.
__device__ __forceinline__ void fold_apply(float (&v)[32], const float *bias, int col, float rinv)
{
#pragma unroll
    for (int j = 0; j < 32; j += 4)
    {
        const float4 b = __ldg(reinterpret_cast<const float4 *>(bias + col + j));
        v[j] = fmaf(rinv, v[j], b.x);
        v[j + 1] = fmaf(rinv, v[j + 1], b.y);
        v[j + 2] = fmaf(rinv, v[j + 2], b.z);
        v[j + 3] = fmaf(rinv, v[j + 3], b.w);
    }
}

// gemm_3 / gemm_6 + mul_15 / mul_21 + add_16 / add_22: resid += gate * acc, FP32, coalesced rows.
// With fold_out, also the next norm's folded operand and the row sums of squares per 128-column part.
template <int BN> __device__ __forceinline__ void epi_resid_gate(const EpiCtx &e, const GemmEpilogueArgs &a)
{
    float *st = reinterpret_cast<float *>(e.stage); // [32][36]
    const int col0 = e.n_blk * BN, cc = (e.lane & 7) * 4;
    const bool fold = a.fold_out != nullptr;
    float squares[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}; // rows p * 4 + lane / 8 of this part
#pragma unroll 1
    for (int c = 0; c < BN; c += 32)
    {
        float v[32];
        tmem_load_32(e.taddr + c, v);
        float4 *mine = reinterpret_cast<float4 *>(st + e.lane * 36);
#pragma unroll
        for (int j = 0; j < 8; ++j) mine[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        __syncwarp();
        const float4 g = __ldg(reinterpret_cast<const float4 *>(a.gate + col0 + c + cc));
        // all eight residual loads are issued before any store, so their latencies overlap
        float4 r[8];
#pragma unroll
        for (int p = 0; p < 8; ++p)
        {
            const int row = e.row0 + p * 4 + (e.lane >> 3);
            r[p] = row < e.m ? *reinterpret_cast<const float4 *>(a.resid + static_cast<size_t>(row) * a.ldo + col0 + c + cc)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int p = 0; p < 8; ++p)
        {
            const int rr = p * 4 + (e.lane >> 3), row = e.row0 + rr;
            const float4 acc = *reinterpret_cast<const float4 *>(st + rr * 36 + cc);
            r[p].x += g.x * acc.x;
            r[p].y += g.y * acc.y;
            r[p].z += g.z * acc.z;
            r[p].w += g.w * acc.w;
            if (row < e.m)
                *reinterpret_cast<float4 *>(a.resid + static_cast<size_t>(row) * a.ldo + col0 + c + cc) = r[p];
        }
        __syncwarp();
        if (fold)
        {
            const int col = col0 + c + cc;
            const float4 gm = __ldg(reinterpret_cast<const float4 *>(a.fold_gamma + col));
            const float4 sc = __ldg(reinterpret_cast<const float4 *>(a.fold_scale + col));
            const float4 k = make_float4(gm.x * (1.f + sc.x), gm.y * (1.f + sc.y), gm.z * (1.f + sc.z), gm.w * (1.f + sc.w));
#pragma unroll
            for (int p = 0; p < 8; ++p)
            {
                const int row = e.row0 + p * 4 + (e.lane >> 3);
                squares[p] += (r[p].x * r[p].x + r[p].y * r[p].y) + (r[p].z * r[p].z + r[p].w * r[p].w);
                if (row < e.m)
                {
                    __nv_bfloat162 lo = __floats2bfloat162_rn(r[p].x * k.x, r[p].y * k.y);
                    __nv_bfloat162 hi = __floats2bfloat162_rn(r[p].z * k.z, r[p].w * k.w);
                    uint2 packed;
                    packed.x = *reinterpret_cast<uint32_t *>(&lo);
                    packed.y = *reinterpret_cast<uint32_t *>(&hi);
                    *reinterpret_cast<uint2 *>(a.fold_out + static_cast<size_t>(row) * kHidden + col) = packed;
                }
            }
            if ((c + 32) % 128 == 0)
            {
                // the part's 128 columns are done: add the 8 lanes of each row (butterfly), lane 0 of the
                // eight stores the row's sum
                const int part = (col0 + c) / 128;
#pragma unroll
                for (int p = 0; p < 8; ++p)
                {
                    float s = squares[p];
                    s += __shfl_xor_sync(0xffffffffu, s, 1);
                    s += __shfl_xor_sync(0xffffffffu, s, 2);
                    s += __shfl_xor_sync(0xffffffffu, s, 4);
                    const int row = e.row0 + p * 4 + (e.lane >> 3);
                    if ((e.lane & 7) == 0 && row < e.m) a.fold_sumsq[static_cast<size_t>(part) * a.fold_ld + row] = s;
                    squares[p] = 0.f;
                }
            }
        }
    }
}

// The tile spans BN/128 whole 128-wide heads of one of Q, K or V (weights are [Wq; Wk; Wv]).
// Q, K: rmsn_9 / rmsn_10 + the rotary chain, head-major [head][token][128]; V: head-major, or
// transposed [head][dim][token] for the tcgen05 attention (BF16 mode). A head row is read from TMEM
// twice (sum of squares, then the rotation pairs d and d+64 in two 32-pair halves), so at most 64
// values are live per thread and nothing spills to local memory.
template <int BN> __device__ __forceinline__ void epi_qkv(const EpiCtx &e, const GemmEpilogueArgs &a)
{
    const int col0 = e.n_blk * BN;
    const int part = col0 / kHidden; // 0 = Q, 1 = K, 2 = V
    const int head0 = (col0 % kHidden) / kHeadDim;
    const int row = e.row0 + e.lane;
    const bool valid = row < e.m;
    const float4 *cs = reinterpret_cast<const float4 *>(a.cos_t + static_cast<size_t>(valid ? row : 0) * kHeadDim);
    const float4 *sn = reinterpret_cast<const float4 *>(a.sin_t + static_cast<size_t>(valid ? row : 0) * kHeadDim);
    const float4 *gamma = reinterpret_cast<const float4 *>(part == 0 ? a.gamma_q : a.gamma_k);
    const int row_limit = a.row_limit > 0 ? a.row_limit : a.rows_pad;
    __nv_bfloat16 *st = reinterpret_cast<__nv_bfloat16 *>(e.stage);
    // folded norm: the projection of this row is rinv * acc + W shift
    const bool fold = a.fold_bias != nullptr;
    const float rinv = fold && valid ? fold_rinv(a, row) : 1.f;
#pragma unroll 1
    for (int hh = 0; hh < BN / 128; ++hh)
    {
        // destination GPU and its head index (selected with constant indices: no local copy of args)
        const int dest = (head0 + hh) / a.heads_per_dest, head = head0 + hh - dest * a.heads_per_dest;
        void *dst_base = nullptr;
#pragma unroll
        for (int d = 0; d < kMaxDest; ++d)
            if (d == dest) dst_base = part == 0 ? a.q[d] : part == 1 ? a.k[d] : a.v[d];
        const uint32_t tcol = e.taddr + hh * 128;
        const int planes = a.qkv_split3 ? 3 : 1;
        const size_t plane_stride = static_cast<size_t>(a.heads_per_dest) * a.rows_pad * kHeadDim;
        if (part == 2 && a.v_transposed)
        {
            // stage [64 dims][40] then write 64-byte token runs of V^T [head][dim][token], per plane
#pragma unroll 1
            for (int pl = 0; pl < planes * 2; ++pl)
            {
                const int plane = pl >> 1, half = pl & 1;
                __nv_bfloat16 *dst = static_cast<__nv_bfloat16 *>(dst_base) + plane * plane_stride;
#pragma unroll
                for (int c = 0; c < 2; ++c)
                {
                    float chunk[32];
                    tmem_load_32(tcol + half * 64 + c * 32, chunk);
                    if (fold) fold_apply(chunk, a.fold_bias, col0 + hh * 128 + half * 64 + c * 32, rinv);
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        st[(c * 32 + j) * 40 + e.lane] = __float2bfloat16_rn(planes == 3 ? split_plane(chunk[j], plane) : chunk[j]);
                }
                __syncwarp();
#pragma unroll
                for (int p = 0; p < 8; ++p)
                {
                    // 8-row runs: row_limit and row_offset are multiples of 16, so a run is all in or all out
                    const int d = p * 8 + (e.lane >> 2), q4 = e.lane & 3;
                    const uint4 val = *reinterpret_cast<const uint4 *>(st + d * 40 + q4 * 8);
                    if (e.row0 + q4 * 8 < row_limit)
                        *reinterpret_cast<uint4 *>(dst + (static_cast<size_t>(head) * kHeadDim + half * 64 + d) *
                                                             a.rows_pad +
                                                   a.row_offset + e.row0 + q4 * 8) = val;
                }
                __syncwarp();
            }
            continue;
        }
        // x * (mean(x^2) + 1e-6)^(-1/2), summed in dimension order
        float inverse = 1.f;
        if (part < 2)
        {
            float squared = 0.f;
#pragma unroll 1
            for (int c = 0; c < 4; ++c)
            {
                float chunk[32];
                tmem_load_32(tcol + c * 32, chunk);
                if (fold) fold_apply(chunk, a.fold_bias, col0 + hh * 128 + c * 32, rinv);
#pragma unroll
                for (int j = 0; j < 32; ++j) squared += chunk[j] * chunk[j];
            }
            inverse = 1.f / sqrtf(squared * (1.f / 128.f) + 1e-6f);
        }
        const size_t dst_row = static_cast<size_t>(head) * a.rows_pad + a.row_offset;
#pragma unroll 1
        for (int c = 0; c < 2; ++c)
        {
            // lo = dims c*32 + [0,32), hi = dims 64 + c*32 + [0,32): the rotation pairs (d, d+64)
            float lo[32], hi[32];
            tmem_load_32(tcol + c * 32, lo);
            tmem_load_32(tcol + 64 + c * 32, hi);
            if (fold)
            {
                fold_apply(lo, a.fold_bias, col0 + hh * 128 + c * 32, rinv);
                fold_apply(hi, a.fold_bias, col0 + hh * 128 + 64 + c * 32, rinv);
            }
            if (part < 2)
            {
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                {
                    const int d = c * 32 + j;
                    const float4 g1 = __ldg(gamma + d / 4), g2 = __ldg(gamma + 16 + d / 4);
                    const float4 c1 = __ldg(cs + d / 4), s1 = __ldg(sn + d / 4);
                    const float4 c2 = __ldg(cs + 16 + d / 4), s2 = __ldg(sn + 16 + d / 4);
                    const float g1v[4] = {g1.x, g1.y, g1.z, g1.w}, g2v[4] = {g2.x, g2.y, g2.z, g2.w};
                    const float c1v[4] = {c1.x, c1.y, c1.z, c1.w}, s1v[4] = {s1.x, s1.y, s1.z, s1.w};
                    const float c2v[4] = {c2.x, c2.y, c2.z, c2.w}, s2v[4] = {s2.x, s2.y, s2.z, s2.w};
#pragma unroll
                    for (int t = 0; t < 4; ++t)
                    {
                        // ERNIE rotary: halves rotated with the full-width, pair-duplicated angle table
                        const float first = lo[j + t] * inverse * g1v[t], second = hi[j + t] * inverse * g2v[t];
                        lo[j + t] = first * c1v[t] - second * s1v[t];
                        hi[j + t] = second * c2v[t] + first * s2v[t];
                    }
                }
            }
#pragma unroll 1
            for (int plane = 0; plane < planes; ++plane)
            {
                // stage [32 rows][72]: columns 0..31 = lo, 32..63 = hi; then 64-byte row segments
                float pv[32];
#pragma unroll
                for (int half = 0; half < 2; ++half)
                {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                    {
                        const float x = half ? hi[j] : lo[j];
                        pv[j] = planes == 3 ? split_plane(x, plane) : x;
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        *reinterpret_cast<uint4 *>(st + e.lane * 72 + half * 32 + j * 8) = pack_bf16x8(pv + j * 8);
                }
                __syncwarp();
                __nv_bfloat16 *dst = static_cast<__nv_bfloat16 *>(dst_base) + plane * plane_stride;
#pragma unroll
                for (int p = 0; p < 8; ++p)
                {
                    const int rr = p * 4 + (e.lane >> 3), j = e.lane & 7, row_g = e.row0 + rr;
                    const int dim = (j < 4 ? 0 : 64) + c * 32 + (j & 3) * 8;
                    if (row_g < e.m && row_g < row_limit)
                        *reinterpret_cast<uint4 *>(dst + (dst_row + row_g) * kHeadDim + dim) =
                            *reinterpret_cast<const uint4 *>(st + rr * 72 + j * 8);
                }
                __syncwarp();
            }
        }
    }
}

// Interleaved [up; gate] weights in 64-row groups: tile columns g*128 + [0,64) are up-projection
// outputs of features n_blk*BN/2 + g*64 + [0,64), columns g*128 + [64,128) the matching gate outputs.
// gemm_4 + gemm_5 + ErnieGELU + mul_20.
template <int BN> __device__ __forceinline__ void epi_geglu(const EpiCtx &e, const GemmEpilogueArgs &a)
{
    const int row = e.row0 + e.lane;
    const bool valid = row < e.m;
    __nv_bfloat16 *st = reinterpret_cast<__nv_bfloat16 *>(e.stage); // [32][40]
    const bool fold = a.fold_bias != nullptr; // folded norm: rinv * acc + W shift
    const float rinv = fold && valid ? fold_rinv(a, row) : 1.f;
#pragma unroll 1
    for (int g = 0; g < BN / 128; ++g)
    {
#pragma unroll 1
        for (int c = 0; c < 64; c += 32)
        {
            float up[32], gate[32];
            tmem_load_32(e.taddr + g * 128 + c, up);
            tmem_load_32(e.taddr + g * 128 + 64 + c, gate);
            if (fold)
            {
                fold_apply(up, a.fold_bias, e.n_blk * BN + g * 128 + c, rinv);
                fold_apply(gate, a.fold_bias, e.n_blk * BN + g * 128 + 64 + c, rinv);
            }
            const int f = e.n_blk * (BN / 2) + g * 64 + c;
            if (a.silu) // SwiGLU (MistralMLP: silu(gate) * up)
            {
                if (a.h_split3)
                {
#pragma unroll
                    for (int j = 0; j < 32; ++j) up[j] = up[j] * __fdiv_rn(gate[j], 1.f + expf(-gate[j]));
                }
                else
                {
#pragma unroll
                    for (int j = 0; j < 32; ++j) up[j] = up[j] * __fdividef(gate[j], 1.f + __expf(-gate[j]));
                }
            }
            else if (a.h_split3) // FP32-exact mode: erfc as the reference's CPU path computes it
            {
#pragma unroll
                for (int j = 0; j < 32; ++j) up[j] = up[j] * gelu_erf(gate[j]);
            }
            else
            {
#pragma unroll
                for (int j = 0; j < 32; ++j) up[j] = up[j] * gelu_as(gate[j]);
            }
            if (a.h_split3)
            {
                if (!valid) continue;
                __nv_bfloat16 *dst = a.h + static_cast<size_t>(row) * (3 * a.ffn) + f;
#pragma unroll
                for (int j = 0; j < 32; j += 8)
                {
                    __align__(16) __nv_bfloat16 hi[8], mid[8], lo[8];
#pragma unroll
                    for (int t = 0; t < 8; ++t) split3(up[j + t], hi[t], mid[t], lo[t]);
                    *reinterpret_cast<uint4 *>(dst + j) = *reinterpret_cast<const uint4 *>(hi);
                    *reinterpret_cast<uint4 *>(dst + a.ffn + j) = *reinterpret_cast<const uint4 *>(mid);
                    *reinterpret_cast<uint4 *>(dst + 2 * a.ffn + j) = *reinterpret_cast<const uint4 *>(lo);
                }
                continue;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j)
                *reinterpret_cast<uint4 *>(st + e.lane * 40 + j * 8) = pack_bf16x8(up + j * 8);
            __syncwarp();
#pragma unroll
            for (int p = 0; p < 4; ++p)
            {
                const int rr = p * 8 + (e.lane >> 2), q4 = e.lane & 3, row_g = e.row0 + rr;
                if (row_g < e.m)
                    *reinterpret_cast<uint4 *>(a.h + static_cast<size_t>(row_g) * a.ffn + f + q4 * 8) =
                        *reinterpret_cast<const uint4 *>(st + rr * 40 + q4 * 8);
            }
            __syncwarp();
        }
    }
}

// BN = 128 = latent channels. Rows are image tokens; latent and prediction are [128][m]
// (consecutive lanes hold consecutive tokens, so these accesses are already coalesced).
__device__ __forceinline__ void epi_final_euler(const EpiCtx &e, const GemmEpilogueArgs &a)
{
    const int row = e.row0 + e.lane;
    const bool valid = row < e.m;
    bool finite = true;
#pragma unroll 1
    for (int c = 0; c < 128; c += 32)
    {
        float v[32];
        tmem_load_32(e.taddr + c, v);
        if (!valid) continue;
#pragma unroll
        for (int j = 0; j < 32; ++j)
        {
            const int ch = c + j;
            const float prediction = v[j] + __ldg(a.bias + ch);
            const size_t idx = static_cast<size_t>(ch) * (a.ld_latent > 0 ? a.ld_latent : e.m) + row;
            // euler_step: change = delta * v; out = x + change, two roundings (no contraction)
            const float next = __fadd_rn(a.latent[idx], __fmul_rn(a.delta, prediction));
            a.latent[idx] = next;
            if (a.prediction) a.prediction[idx] = prediction;
            finite = finite && isfinite(next);
        }
    }
    if (!finite) atomicOr(a.finite_flag, 1);
}

template <int BN, Epilogue EPI>
__device__ __forceinline__ void run_epilogue(const EpiCtx &e, const GemmEpilogueArgs &args)
{
    if constexpr (EPI == Epilogue::F32Bias) epi_f32_bias<BN>(e, args);
    else if constexpr (EPI == Epilogue::ResidGate) epi_resid_gate<BN>(e, args);
    else if constexpr (EPI == Epilogue::Qkv) epi_qkv<BN>(e, args);
    else if constexpr (EPI == Epilogue::Geglu) epi_geglu<BN>(e, args);
    else epi_final_euler(e, args);
}

// PROMOTE (FP32-exact mode): the tensor core's FP32 accumulation error grows linearly with the
// length of one TMEM accumulation chain (measured on B200: nrmse 4.4e-6 at K=4096, 1.4e-5 at
// K=12288 for exact operands; 6.5e-8 when restarted every 64 elements). With PROMOTE the MMA warp
// restarts the accumulator every `group` k-blocks (two alternating TMEM buffers) and the epilogue
// warps add each partial into FP32 registers, so no chain exceeds group*64 products.
// Output tile t -> (m block, n block). Tiles run through the n blocks of a band of `band` m blocks (m
// fastest inside the band), band after band, so that consecutive rounds of tiles over the SMs reuse
// one band's A rows from L2 while B streams; band >= num_m is the plain m-fastest order.
__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int band, int &m_blk, int &n_blk)
{
    const int per_band = band * num_n;
    const int b = t / per_band, r = t - b * per_band;
    const int first = b * band;
    const int rows = min(band, num_m - first);
    m_blk = first + r % rows;
    n_blk = r / rows;
}

template <int BN, Epilogue EPI, bool PROMOTE>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, int m, int n,
                int k_b, int splits, int group, int band, GemmEpilogueArgs args)
{
    using C = Cfg<BN, PROMOTE>;
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
    const int num_m = (m + BM - 1) / BM, num_n = n / BN, tiles = num_m * num_n;
    const int k_blocks = (k_b * splits) / BK;
    const int span = PROMOTE ? group : k_blocks; // k-blocks per accumulation chain

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
    grid_dependency_wait(); // the previous kernel's writes (A, residual, peer flags) are visible from here
    grid_dependents_launch();

    if (warp == 0)
    {
        if (lane == 0)
        {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            peer_wait_all(args.sync.wait); // sequence parallel: every member's rows of A have landed
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x)
            {
                int m_blk, n_blk;
                tile_coords(tile, num_m, num_n, band, m_blk, n_blk);
                for (int kb = 0; kb < k_blocks; ++kb)
                {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1u))
                    {
                        if (args.error_flag) atomicExch(args.error_flag, kErrGemmProducerTimeout);
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(full_bar(stage), C::kStageBytes);
                    tma_load_2d(tile_a(stage), &map_a, full_bar(stage), kb * BK, m_blk * BM);
                    tma_load_2d(tile_b(stage), &map_b, full_bar(stage), (kb * BK) % k_b, n_blk * BN);
                    if (++stage == C::kStages)
                    {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // On a timeout no drain is needed: the last load was issued before the failed wait
            // began, kWaitLimitCycles earlier, and TMA loads complete without any consumer.
        }
    }
    else if (warp == 1)
    {
        if (lane == 0)
        {
            constexpr uint32_t idesc = idesc_bf16(BM, BN);
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
                        if (args.error_flag) atomicExch(args.error_flag, kErrGemmMmaTimeout);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                    for (int kb = kb0; kb < kb0 + span; ++kb)
                    {
                        if (!mbar_wait(full_bar(stage), phase))
                        {
                            if (args.error_flag) atomicExch(args.error_flag, kErrGemmMmaTimeout);
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint64_t a_desc = smem_desc_sw128(tile_a(stage));
                        const uint64_t b_desc = smem_desc_sw128(tile_b(stage));
#pragma unroll
                        for (int k = 0; k < BK / 16; ++k)
                            umma_bf16(d_tmem, a_desc + 2u * k, b_desc + 2u * k, idesc,
                                      (kb != kb0 || k != 0) ? 1u : 0u);
                        umma_commit(empty_bar(stage));
                        if (++stage == C::kStages)
                        {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                    if (ok) umma_commit(tfull_bar(acc));
                }
            }
        }
    }
    else
    {
        const int quarter = warp & 3;
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        int unit = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x)
        {
            int m_blk, n_blk;
            tile_coords(tile, num_m, num_n, band, m_blk, n_blk);
            const int row0 = m_blk * BM + quarter * 32;
            uint8_t *stage = base_ptr + C::kStagingOffset + quarter * C::kStagingBytes;
            if constexpr (!PROMOTE)
            {
                const int acc = unit & 1;
                const uint32_t acc_phase = (unit >> 1) & 1;
                if (!mbar_wait(tfull_bar(acc), acc_phase))
                {
                    if (args.error_flag && lane == 0) atomicExch(args.error_flag, kErrGemmEpilogueTimeout);
                    break;
                }
                tc_fence_after();
                run_epilogue<BN, EPI>(EpiCtx{lane_base + acc * BN, row0, lane, m, n_blk, stage}, args);
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
                        if (args.error_flag && lane == 0) atomicExch(args.error_flag, kErrGemmEpilogueTimeout);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int c = 0; c < BN; c += 32)
                    {
                        float v[32];
                        tmem_load_32(lane_base + acc * BN + c, v);
#pragma unroll
                        for (int j = 0; j < 32; ++j) sum[c + j] += v[j];
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(tempty_bar(acc));
                }
                if (!ok) break;
                // the FP32 sum goes to the result buffer (columns 2*BN..3*BN) for the shared epilogues
                const uint32_t result = lane_base + 2 * BN;
#pragma unroll
                for (int c = 0; c < BN; c += 32) tmem_store_32(result + c, sum + c);
                tmem_store_wait();
                run_epilogue<BN, EPI>(EpiCtx{result, row0, lane, m, n_blk, stage}, args);
            }
        }
        peer_signal_warp(args.sync.signal); // this warp's stores are done
    }
    __syncthreads();
    if (warp == 1)
    {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::kTmemCols);
    }
}

// ---- CTA-pair GEMM (cta_group::2) ------------------------------------------------------------
// Same warp roles and epilogues as gemm_kernel, on 256 x BN output tiles computed by a cluster of two
// CTAs on neighbouring SMs. CTA r of the pair loads A rows [256*i + 128*r, +128) and B rows
// [BN*j + (BN/2)*r, +BN/2) into its own shared memory; the even CTA's single MMA thread issues
// M=256 tcgen05.mma.cta_group::2 instructions that read both CTAs' tiles and write each CTA's 128
// accumulator rows into that CTA's TMEM. Per 256 x BN x 64 step each SM's shared memory supplies
// 16 KB of A and BN/2 x 128 B of B, half the B traffic of the single-CTA 128 x BN tile, which is
// what bounds the single-CTA kernel. Barrier traffic between the two CTAs:
//   full[s]   (even CTA)  both producers' TMA bytes (expect_tx by the even CTA only)
//   empty[s]  (each CTA)  MMA commit, issued once to each CTA's barrier
//   tfull[i]  (each CTA)  MMA commit after a tile's last k-block, once to each CTA
//   tempty[i] (even CTA)  all 8 epilogue warps of the pair (the odd CTA's arrive remotely)
template <int BN> struct PairCfg
{
    static constexpr int kStages = 6;
    static constexpr int kABytes = BM * BK * 2;
    static constexpr int kBBytes = (BN / 2) * BK * 2;
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kTmemCols = 2 * BN;
    static constexpr int kBarrierBytes = 256;
    static constexpr int kStagingBytes = 5120;
    static constexpr int kStagingOffset = kStages * kStageBytes + kBarrierBytes;
    static constexpr int kSmemBytes = kStagingOffset + 4 * kStagingBytes + 1024;
};

template <int BN, Epilogue EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, int m,
                     int n, int k_b, int band, int split_from, GemmEpilogueArgs args)
{
    using C = PairCfg<BN>;
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

    const uint32_t rank = cluster_ctarank();
    const uint32_t peer = rank ^ 1u;
    const bool leader = rank == 0;
    const int pair = blockIdx.x / 2, pairs = gridDim.x / 2;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int num_m = (m + 2 * BM - 1) / (2 * BM), num_n = n / BN, tiles = num_m * num_n;
    const int k_blocks = k_b / BK;
    // Work units: tiles [0, split_from) whole; each tile of the last, partial round (from split_from on)
    // as two BN/2-column halves, so that round spreads over up to twice as many pairs.
    const bool splitting = BN == 256 && split_from >= 0 && split_from < tiles;
    const int units = splitting ? split_from + 2 * (tiles - split_from) : tiles;
    // unit -> (m block, n block, half: -1 whole tile, 0/1 the left/right BN/2 columns)
    auto unit_coords = [&](int u, int &m_blk, int &n_blk, int &half) {
        half = -1;
        int t = u;
        if (splitting && u >= split_from)
        {
            t = split_from + (u - split_from) / 2;
            half = (u - split_from) & 1;
        }
        tile_coords(t, num_m, num_n, band, m_blk, n_blk);
    };

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
            mbar_init(tempty_bar(i), 8);
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
        tmem_alloc_pair(slot, C::kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync(); // both CTAs' barriers are initialised before any remote arrive or TMA completion
    tc_fence_after();
    const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t *>(base_ptr + (slot - base));
    grid_dependency_wait(); // the previous kernel's writes (A, residual, peer flags) are visible from here
    grid_dependents_launch();

    if (warp == 0)
    {
        if (lane == 0)
        {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            peer_wait_all(args.sync.wait); // sequence parallel: every member's rows of A have landed
            for (int tile = pair; tile < units && ok; tile += pairs)
            {
                int m_blk, n_blk, half;
                unit_coords(tile, m_blk, n_blk, half);
                // a half tile's B rows: BN/4 per CTA at n_blk*BN + half*BN/2 (the box loads BN/2, the MMA
                // reads the first BN/4)
                const int b_row = half < 0 ? n_blk * BN + static_cast<int>(rank) * (BN / 2)
                                           : n_blk * BN + half * (BN / 2) + static_cast<int>(rank) * (BN / 4);
                for (int kb = 0; kb < k_blocks; ++kb)
                {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1u))
                    {
                        if (args.error_flag) atomicExch(args.error_flag, kErrGemmProducerTimeout);
                        ok = false;
                        break;
                    }
                    // the even CTA expects both CTAs' bytes on its full barrier
                    if (leader) mbar_arrive_expect_tx(full_bar(stage), 2 * C::kStageBytes);
                    const uint32_t bar = mapa_shared(full_bar(stage), 0);
                    tma_load_2d_pair(tile_a(stage), &map_a, bar, kb * BK, m_blk * 2 * BM + static_cast<int>(rank) * BM);
                    tma_load_2d_pair(tile_b(stage), &map_b, bar, kb * BK, b_row);
                    if (++stage == C::kStages)
                    {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // tail: wait until the MMA has released every filled stage, so that no commit from the
            // even CTA is still on its way to this CTA's barriers when the CTA exits
            for (int i = 0; i < C::kStages && ok; ++i)
            {
                if (!mbar_wait(empty_bar(stage), phase ^ 1u))
                {
                    if (args.error_flag) atomicExch(args.error_flag, kErrGemmProducerTimeout);
                    ok = false;
                }
                if (++stage == C::kStages)
                {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
    }
    else if (warp == 1)
    {
        if (lane == 0 && leader)
        {
            constexpr uint32_t idesc_whole = idesc_bf16(2 * BM, BN), idesc_half = idesc_bf16(2 * BM, BN / 2);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int unit = 0;
            for (int tile = pair; tile < units && ok; tile += pairs, ++unit)
            {
                int m_blk, n_blk, half;
                unit_coords(tile, m_blk, n_blk, half);
                const uint32_t idesc = half < 0 ? idesc_whole : idesc_half;
                const int acc = unit & 1;
                const uint32_t acc_phase = (unit >> 1) & 1;
                if (!mbar_wait_cluster(tempty_bar(acc), acc_phase ^ 1u))
                {
                    if (args.error_flag) atomicExch(args.error_flag, kErrGemmMmaTimeout);
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = 0; kb < k_blocks; ++kb)
                {
                    if (!mbar_wait(full_bar(stage), phase))
                    {
                        if (args.error_flag) atomicExch(args.error_flag, kErrGemmMmaTimeout);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t a_desc = smem_desc_sw128(tile_a(stage));
                    const uint64_t b_desc = smem_desc_sw128(tile_b(stage));
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                        umma_bf16_pair(d_tmem, a_desc + 2u * k, b_desc + 2u * k, idesc, (kb != 0 || k != 0) ? 1u : 0u);
                    umma_commit_pair(empty_bar(stage));
                    umma_commit_pair(mapa_shared(empty_bar(stage), peer));
                    if (++stage == C::kStages)
                    {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (ok)
                {
                    umma_commit_pair(tfull_bar(acc));
                    umma_commit_pair(mapa_shared(tfull_bar(acc), peer));
                }
            }
        }
    }
    else
    {
        const int quarter = warp & 3;
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        const uint32_t leader_tempty0 = mapa_shared(tempty_bar(0), 0), leader_tempty1 = mapa_shared(tempty_bar(1), 0);
        int unit = 0;
        for (int tile = pair; tile < units; tile += pairs, ++unit)
        {
            int m_blk, n_blk, half;
            unit_coords(tile, m_blk, n_blk, half);
            const int row0 = m_blk * 2 * BM + static_cast<int>(rank) * BM + quarter * 32;
            uint8_t *stage = base_ptr + C::kStagingOffset + quarter * C::kStagingBytes;
            const int acc = unit & 1;
            const uint32_t acc_phase = (unit >> 1) & 1;
            if (!mbar_wait(tfull_bar(acc), acc_phase))
            {
                if (args.error_flag && lane == 0) atomicExch(args.error_flag, kErrGemmEpilogueTimeout);
                break;
            }
            tc_fence_after();
            if constexpr (BN == 256)
            {
                if (half >= 0)
                    run_epilogue<BN / 2, EPI>(EpiCtx{lane_base + acc * BN, row0, lane, m, 2 * n_blk + half, stage}, args);
                else
                    run_epilogue<BN, EPI>(EpiCtx{lane_base + acc * BN, row0, lane, m, n_blk, stage}, args);
            }
            else
                run_epilogue<BN, EPI>(EpiCtx{lane_base + acc * BN, row0, lane, m, n_blk, stage}, args);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc ? leader_tempty1 : leader_tempty0);
        }
        peer_signal_warp(args.sync.signal); // this warp's stores are done
    }
    // no CTA leaves (or frees TMEM) while its partner may still signal its barriers or use its TMEM
    tc_fence_before();
    cluster_sync();
    if (warp == 1)
    {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, C::kTmemCols);
    }
}

// ---- host side ------------------------------------------------------------------------------
// Band of m blocks for tile_coords. While A (m x k_a BF16) fits in L2 next to the streamed B tiles and
// the epilogue's traffic, the m-fastest order keeps it resident and reads B once. A larger A (the down
// projection's 12288-wide rows: 107 MB at 4160 rows, 203 MB at 8256) would be re-read from DRAM in every
// round of tiles; then the m blocks are cut into the fewest equal bands of at most kBandBytes of A, each
// band staying resident while B streams past it once.
#ifndef ERNIE_GEMM_BAND_BYTES
#define ERNIE_GEMM_BAND_BYTES (64ll << 20)
#endif
constexpr long long kBandBytes = ERNIE_GEMM_BAND_BYTES, kResidentA = 96ll << 20;
int tile_band(int num_m, int tile_rows, int k_a)
{
    const long long per_block = static_cast<long long>(tile_rows) * k_a * 2;
    const long long a_bytes = num_m * per_block;
    if (kBandBytes <= 0 || a_bytes <= kResidentA) return num_m;
    const long long bands = (a_bytes + kBandBytes - 1) / kBandBytes;
    return static_cast<int>((num_m + bands - 1) / bands);
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

// Row-major BF16 [rows, cols] operand, 64-column (128-byte) x box_rows boxes, 128-byte swizzle.
bool make_map(CUtensorMap *map, const void *ptr, uint64_t rows, uint64_t cols, uint32_t box_rows)
{
    auto fn = encode_fn();
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

template <int BN, Epilogue EPI, bool PROMOTE> cudaError_t ensure_attributes()
{
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(gemm_kernel<BN, EPI, PROMOTE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    Cfg<BN, PROMOTE>::kSmemBytes);
    });
    return attr;
}

template <int BN, Epilogue EPI> cudaError_t ensure_pair_attributes()
{
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(gemm_pair_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    PairCfg<BN>::kSmemBytes);
    });
    return attr;
}

// Pairs that can be resident at once (one CTA per SM, both SMs of a pair in one GPC).
template <int BN, Epilogue EPI> int resident_pairs(int num_sms)
{
    static std::once_flag once;
    static int pairs = 0;
    std::call_once(once, [num_sms] {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (num_sms / 2));
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = PairCfg<BN>::kSmemBytes;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, gemm_pair_kernel<BN, EPI>, &cfg) == cudaSuccess && clusters > 0)
            pairs = clusters;
        else
            cudaGetLastError();
    });
    return pairs > 0 ? pairs : num_sms / 2;
}

template <int BN, Epilogue EPI>
int launch_pair(const __nv_bfloat16 *a, const __nv_bfloat16 *b, int m, int n, int k_b, const GemmEpilogueArgs &args,
                int num_sms, cudaStream_t stream)
{
    const cudaError_t attr = ensure_pair_attributes<BN, EPI>();
    if (attr != cudaSuccess) return attr;
    CUtensorMap map_a, map_b;
    if (!make_map(&map_a, a, static_cast<uint64_t>(m), static_cast<uint64_t>(k_b), BM) ||
        !make_map(&map_b, b, static_cast<uint64_t>(n), static_cast<uint64_t>(k_b), BN / 2))
        return cudaErrorInvalidValue;
    const int tiles = ((m + 2 * BM - 1) / (2 * BM)) * (n / BN);
    const int max_pairs = resident_pairs<BN, EPI>(num_sms);
    const int pairs = tiles < max_pairs ? tiles : max_pairs;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = PairCfg<BN>::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = 2;
    attrs[0].val.clusterDim.y = 1;
    attrs[0].val.clusterDim.z = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = add_programmatic_attribute(attrs, 1);
    const int band = tile_band((m + 2 * BM - 1) / (2 * BM), 2 * BM, k_b);
    // a last, partial round of at most half the pairs runs as twice as many half-width tiles
    const int rest = tiles % pairs;
    const int split_from = kSplitLastRound && BN == 256 && rest > 0 && 2 * rest <= pairs ? tiles - rest : -1;
    GemmEpilogueArgs launch_args = args;
    launch_args.sync.signal.warps = 2 * pairs * 4; // four epilogue warps per CTA
    return cudaLaunchKernelEx(&cfg, gemm_pair_kernel<BN, EPI>, map_a, map_b, m, n, k_b, band, split_from, launch_args);
}

template <int BN, Epilogue EPI, bool PROMOTE>
int launch_impl(const __nv_bfloat16 *a, const __nv_bfloat16 *b, int m, int n, int k_b, int splits,
                const GemmEpilogueArgs &args, int num_sms, cudaStream_t stream)
{
    using C = Cfg<BN, PROMOTE>;
    const cudaError_t attr = ensure_attributes<BN, EPI, PROMOTE>();
    if (attr != cudaSuccess) return attr;
    CUtensorMap map_a, map_b;
    if (!make_map(&map_a, a, static_cast<uint64_t>(m), static_cast<uint64_t>(k_b) * splits, BM) ||
        !make_map(&map_b, b, static_cast<uint64_t>(n), static_cast<uint64_t>(k_b), BN))
        return cudaErrorInvalidValue;
    const int k_blocks = k_b * splits / BK;
    // promotion every 256 products (fewer if K allows no multiple of 4 k-blocks)
    const int group = k_blocks % 4 == 0 ? 4 : k_blocks % 2 == 0 ? 2 : 1;
    const int tiles = ((m + BM - 1) / BM) * (n / BN);
    const int grid = tiles < num_sms ? tiles : num_sms;
    const int band = tile_band((m + BM - 1) / BM, BM, k_b * splits);
    GemmEpilogueArgs launch_args = args;
    launch_args.sync.signal.warps = grid * 4; // four epilogue warps per CTA
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attrs[1];
    cfg.attrs = attrs;
    cfg.numAttrs = add_programmatic_attribute(attrs, 0);
    return cudaLaunchKernelEx(&cfg, gemm_kernel<BN, EPI, PROMOTE>, map_a, map_b, m, n, k_b, splits, group, band,
                              launch_args);
}

template <int BN, bool PROMOTE>
int dispatch(Epilogue epilogue, const __nv_bfloat16 *a, const __nv_bfloat16 *b, int m, int n, int k_b, int splits,
             const GemmEpilogueArgs &args, int num_sms, cudaStream_t stream)
{
    switch (epilogue)
    {
    case Epilogue::F32Bias: return launch_impl<BN, Epilogue::F32Bias, PROMOTE>(a, b, m, n, k_b, splits, args, num_sms, stream);
    case Epilogue::ResidGate: return launch_impl<BN, Epilogue::ResidGate, PROMOTE>(a, b, m, n, k_b, splits, args, num_sms, stream);
    case Epilogue::Qkv: return launch_impl<BN, Epilogue::Qkv, PROMOTE>(a, b, m, n, k_b, splits, args, num_sms, stream);
    case Epilogue::Geglu: return launch_impl<BN, Epilogue::Geglu, PROMOTE>(a, b, m, n, k_b, splits, args, num_sms, stream);
    case Epilogue::FinalEuler:
        if constexpr (BN == 128) return launch_impl<BN, Epilogue::FinalEuler, PROMOTE>(a, b, m, n, k_b, splits, args, num_sms, stream);
        return cudaErrorInvalidValue;
    }
    return cudaErrorInvalidValue;
}

template <int BN, bool PROMOTE> cudaError_t prepare_all()
{
    cudaError_t e = ensure_attributes<BN, Epilogue::F32Bias, PROMOTE>();
    if (e == cudaSuccess) e = ensure_attributes<BN, Epilogue::ResidGate, PROMOTE>();
    if (e == cudaSuccess) e = ensure_attributes<BN, Epilogue::Qkv, PROMOTE>();
    if (e == cudaSuccess) e = ensure_attributes<BN, Epilogue::Geglu, PROMOTE>();
    if constexpr (BN == 128)
        if (e == cudaSuccess) e = ensure_attributes<BN, Epilogue::FinalEuler, PROMOTE>();
    return e;
}

cudaError_t prepare_pairs()
{
    cudaError_t e = ensure_pair_attributes<256, Epilogue::F32Bias>();
    if (e == cudaSuccess) e = ensure_pair_attributes<256, Epilogue::ResidGate>();
    if (e == cudaSuccess) e = ensure_pair_attributes<256, Epilogue::Qkv>();
    if (e == cudaSuccess) e = ensure_pair_attributes<256, Epilogue::Geglu>();
    // resident pair counts are queried here, outside any stream capture
    int device = 0, sms = 0;
    if (e == cudaSuccess) e = cudaGetDevice(&device);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (e == cudaSuccess)
    {
        resident_pairs<256, Epilogue::F32Bias>(sms);
        resident_pairs<256, Epilogue::ResidGate>(sms);
        resident_pairs<256, Epilogue::Qkv>(sms);
        resident_pairs<256, Epilogue::Geglu>(sms);
    }
    return e;
}

// Measured on B200 (C2 shapes, power-capped clocks): a pair tile takes as long per 128 rows as a
// single-CTA tile for the plain epilogues, and pairs gain only on the long-K, narrow-N projections (out,
// down: 3-5%). They are used when they need no more rounds of tiles over the SMs than single CTAs do;
// otherwise the coarser 256-row quantisation loses (up/gate: 23 rounds instead of 22 at 4160 rows, 3-4%
// slower measured). The QKV GEMM is the exception: its pair rounds run ~13% faster than its single-CTA
// rounds (C2: 0.32-0.35 against 0.36-0.39 ms with 12 pair rounds against 11; C3: 0.48-0.50 against
// 0.50-0.58 ms), so it takes pairs unless they need more than 1/0.87 times the rounds (the 1040-row
// shards of 8-GPU sequence parallelism: 4 pair rounds against 3).
bool use_pairs(int m, int n, int splits, int block_n, bool promote, int num_sms, Epilogue epilogue)
{
    if (promote || splits != 1 || block_n != 256 || num_sms < 2) return false;
    const long long tiles1 = static_cast<long long>((m + BM - 1) / BM) * (n / block_n);
    const long long tiles2 = static_cast<long long>((m + 2 * BM - 1) / (2 * BM)) * (n / block_n);
    const long long rounds1 = (tiles1 + num_sms - 1) / num_sms, rounds2 = (tiles2 + num_sms / 2 - 1) / (num_sms / 2);
    if (epilogue == Epilogue::Qkv) return rounds2 * 87 <= rounds1 * 100;
    return rounds2 <= rounds1;
}
} // namespace

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() { return encode_fn(); }

int prepare_gemm_kernels()
{
    cudaError_t e = prepare_pairs();
    if (e == cudaSuccess) e = prepare_all<256, false>();
    if (e == cudaSuccess) e = prepare_all<128, false>();
    if (e == cudaSuccess) e = prepare_all<128, true>();
    return e;
}

int launch_gemm(const __nv_bfloat16 *a, const __nv_bfloat16 *b, int m, int n, int k_b, int splits, int block_n,
                Epilogue epilogue, const GemmEpilogueArgs &args, int num_sms, cudaStream_t stream, bool promote)
{
    if (m < 1 || n < 1 || k_b < BK || k_b % BK || splits < 1 || splits > 3 || num_sms < 1) return cudaErrorInvalidValue;
    if (block_n != 128 && block_n != 256) return cudaErrorInvalidValue;
    if (promote && block_n != 128) return cudaErrorInvalidValue;
    if (n % block_n) return cudaErrorInvalidValue;
    if (epilogue == Epilogue::FinalEuler && (block_n != 128 || n != 128)) return cudaErrorInvalidValue;
    if (epilogue == Epilogue::Qkv)
    {
        const int limit = args.row_limit > 0 ? args.row_limit : args.rows_pad;
        if (n != 3 * kHidden || args.heads_per_dest < 1 || kHeads % args.heads_per_dest ||
            kHeads / args.heads_per_dest > kMaxDest || args.row_offset < 0 || args.row_offset % 16 || limit % 16 ||
            args.row_offset + limit > args.rows_pad || (args.row_limit == 0 && args.rows_pad < m))
            return cudaErrorInvalidValue;
        for (int d = 0; d < kHeads / args.heads_per_dest; ++d)
            if (!args.q[d] || !args.k[d] || !args.v[d]) return cudaErrorInvalidValue;
    }
    if (epilogue == Epilogue::Geglu && n != 2 * args.ffn) return cudaErrorInvalidValue;
    if (promote) return dispatch<128, true>(epilogue, a, b, m, n, k_b, splits, args, num_sms, stream);
#ifdef ERNIE_PAIRS_FOR // tile-shape sweep: CTA pairs whatever the tile rounds, for epilogues in this bit mask
    const bool pairs_forced = ((ERNIE_PAIRS_FOR >> static_cast<int>(epilogue)) & 1) && block_n == 256 && !promote &&
                              splits == 1;
#else
    const bool pairs_forced = false;
#endif
    if ((pairs_forced || use_pairs(m, n, splits, block_n, promote, num_sms, epilogue)) && epilogue != Epilogue::FinalEuler)
    {
        switch (epilogue)
        {
        case Epilogue::F32Bias: return launch_pair<256, Epilogue::F32Bias>(a, b, m, n, k_b, args, num_sms, stream);
        case Epilogue::ResidGate: return launch_pair<256, Epilogue::ResidGate>(a, b, m, n, k_b, args, num_sms, stream);
        case Epilogue::Qkv: return launch_pair<256, Epilogue::Qkv>(a, b, m, n, k_b, args, num_sms, stream);
        case Epilogue::Geglu: return launch_pair<256, Epilogue::Geglu>(a, b, m, n, k_b, args, num_sms, stream);
        default: return cudaErrorInvalidValue;
        }
    }
    if (block_n == 256) return dispatch<256, false>(epilogue, a, b, m, n, k_b, splits, args, num_sms, stream);
    return dispatch<128, false>(epilogue, a, b, m, n, k_b, splits, args, num_sms, stream);
}
} // namespace ernie_b200
