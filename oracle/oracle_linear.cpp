// CPU restatement, TEST INFRASTRUCTURE ONLY: the dense projection used by every ncnn `Gemm` /
// `InnerProduct` / 1x1 `Convolution` on the reference's hot path.
//
// Reference call sites: block.ncnn.param:19,22,25,61,70,71,74 (Gemm 7=M 8=N 9=K, B transposed, no
// bias: artifacts/2026-09-05/components/direct-block00/block.ncnn.param), head.ncnn.param InnerProduct
// and Convolution layers (artifacts/2026-09-05/components/heads/{input,output}/head.ncnn.param).
// ncnn's CPU Gemm accumulates in FP32; so does this restatement (per output, one FMA chain per block
// of 256 k values, the blocks added in k order). Weights are BF16 values widened exactly to FP32, as
// tools/build_dit_weights.py:110 does before writing the ncnn .bin.
//
// This file is compiled with -ffp-contract=fast (FMA), unlike the rest of the oracle, which
// follows the reference's -ffp-contract=off (src/CMakeLists.txt:11-13) for the Euler update.
#include "ernie_oracle.h"
#include <algorithm>
#include <cstring>
#include <vector>

typedef float v8f __attribute__((vector_size(32)));

static inline v8f load8(const float *p)
{
    v8f v;
    std::memcpy(&v, p, sizeof(v));
    return v;
}

static inline float widen(uint16_t bits)
{
    const uint32_t u = uint32_t(bits) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// C[m][n] = A[m][k] W[n][k]^T (+ bias), cache-blocked: k in blocks of KC, W of each k block packed per
// 16-column panel as [KC][16] floats, rows of A in blocks of MC per thread, a 6 x 16 register tile per
// step (12 FMAs per k on two 8-lane vectors of W and six broadcast A values). Each output adds its k
// blocks in order, every block as one FMA chain per output, so the result does not depend on the thread
// count.
extern "C" void orc_linear(const float *a, const uint16_t *w, const float *bias, int64_t m, int n, int k, float *c)
{
#ifndef ORC_MR
#define ORC_MR 6
#endif
#ifndef ORC_KC
#define ORC_KC 256
#endif
    constexpr int MR = ORC_MR, NR = 16, KC = ORC_KC, MC = 96, GP = 32;
    const int panels = (n + NR - 1) / NR;
    const int64_t row_blocks = (m + MC - 1) / MC;
    std::vector<float> packed(size_t(panels) * NR * KC);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j) c[i * n + j] = 0.f;
    for (int k0 = 0; k0 < k; k0 += KC)
    {
        const int kc = std::min(KC, k - k0);
        // pack this k block of W: panel p holds columns [16p, 16p+16) as [kc][16] (zero past n)
#pragma omp parallel for schedule(static)
        for (int p = 0; p < panels; ++p)
        {
            float *dst = packed.data() + size_t(p) * NR * KC;
            for (int x = 0; x < kc; ++x)
                for (int j = 0; j < NR; ++j)
                {
                    const int col = p * NR + j;
                    dst[size_t(x) * NR + j] = col < n ? widen(w[size_t(col) * k + k0 + x]) : 0.f;
                }
        }
        // tasks: (row block, group of GP panels), so short and wide products still use every core
        const int groups = (panels + GP - 1) / GP;
#pragma omp parallel for schedule(dynamic, 1)
        for (int64_t task = 0; task < row_blocks * groups; ++task)
        {
            const int64_t rb = task / groups;
            const int g = int(task % groups);
            const int64_t i_begin = rb * MC, i_end = std::min<int64_t>(m, i_begin + MC);
            for (int p = g * GP; p < std::min(panels, g * GP + GP); ++p)
            {
                const float *wp = packed.data() + size_t(p) * NR * KC;
                const int ncols = std::min(NR, n - p * NR);
                for (int64_t i0 = i_begin; i0 < i_end; i0 += MR)
                {
                    const int rows = int(std::min<int64_t>(MR, i_end - i0));
                    const float *ar[MR];
                    for (int r = 0; r < MR; ++r) ar[r] = a + (i0 + std::min(r, rows - 1)) * k + k0;
                    v8f acc[MR][2];
                    for (int r = 0; r < MR; ++r) acc[r][0] = acc[r][1] = v8f{0, 0, 0, 0, 0, 0, 0, 0};
                    for (int x = 0; x < kc; ++x)
                    {
                        const v8f w0 = load8(wp + size_t(x) * NR), w1 = load8(wp + size_t(x) * NR + 8);
                        for (int r = 0; r < MR; ++r)
                        {
                            const float s = ar[r][x];
                            const v8f av = v8f{s, s, s, s, s, s, s, s};
                            acc[r][0] += av * w0;
                            acc[r][1] += av * w1;
                        }
                    }
                    for (int r = 0; r < rows; ++r)
                    {
                        float *out = c + (i0 + r) * n + p * NR;
                        for (int j = 0; j < ncols; ++j) out[j] += acc[r][j >> 3][j & 7];
                    }
                }
            }
        }
    }
    if (bias)
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < m; ++i)
            for (int j = 0; j < n; ++j) c[i * n + j] += bias[j];
}
