// CPU restatement, TEST INFRASTRUCTURE ONLY: the dense projection used by every ncnn `Gemm` /
// `InnerProduct` / 1x1 `Convolution` on the reference's hot path.
//
// Reference call sites: block.ncnn.param:19,22,25,61,70,71,74 (Gemm 7=M 8=N 9=K, B transposed, no
// bias: artifacts/2026-09-05/components/direct-block00/block.ncnn.param), head.ncnn.param InnerProduct
// and Convolution layers (artifacts/2026-09-05/components/heads/{input,output}/head.ncnn.param).
// ncnn's CPU Gemm accumulates in FP32; so does this restatement (8-lane partial sums, then a
// pairwise horizontal sum). Weights are BF16 values widened exactly to FP32, as
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

static inline float hsum(v8f v)
{
    const float a = (v[0] + v[4]) + (v[2] + v[6]);
    const float b = (v[1] + v[5]) + (v[3] + v[7]);
    return a + b;
}

static inline float widen(uint16_t bits)
{
    const uint32_t u = uint32_t(bits) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

extern "C" void orc_linear(const float *a, const uint16_t *w, const float *bias, int64_t m, int n, int k, float *c)
{
    constexpr int panel_rows = 16;
    const int kp = (k + 7) & ~7;
    const int panels = (n + panel_rows - 1) / panel_rows;
#pragma omp parallel
    {
        std::vector<float> panel(size_t(panel_rows) * kp, 0.f);
        std::vector<float> rows(2 * size_t(kp), 0.f);
#pragma omp for schedule(dynamic, 1)
        for (int p = 0; p < panels; ++p)
        {
            const int n0 = p * panel_rows;
            const int nb = std::min(panel_rows, n - n0);
            for (int j = 0; j < panel_rows; ++j)
                for (int x = 0; x < kp; ++x)
                    panel[size_t(j) * kp + x] = (j < nb && x < k) ? widen(w[size_t(n0 + j) * k + x]) : 0.f;
            for (int64_t i = 0; i < m; i += 2)
            {
                const bool pair = i + 1 < m;
                const float *a0 = a + i * k;
                const float *a1 = pair ? a + (i + 1) * k : a0;
                if (kp != k)
                {
                    std::fill(rows.begin(), rows.end(), 0.f);
                    std::memcpy(rows.data(), a0, sizeof(float) * k);
                    std::memcpy(rows.data() + kp, a1, sizeof(float) * k);
                    a0 = rows.data();
                    a1 = rows.data() + kp;
                }
                for (int j = 0; j < nb; j += 4)
                {
                    v8f acc[2][4];
                    for (int r = 0; r < 2; ++r)
                        for (int q = 0; q < 4; ++q)
                            acc[r][q] = v8f{0, 0, 0, 0, 0, 0, 0, 0};
                    const float *w0 = panel.data() + size_t(j) * kp;
                    for (int x = 0; x < kp; x += 8)
                    {
                        const v8f x0 = load8(a0 + x), x1 = load8(a1 + x);
                        for (int q = 0; q < 4; ++q)
                        {
                            const v8f wv = load8(w0 + size_t(q) * kp + x);
                            acc[0][q] += x0 * wv;
                            acc[1][q] += x1 * wv;
                        }
                    }
                    for (int q = 0; q < 4 && j + q < nb; ++q)
                    {
                        const float b = bias ? bias[n0 + j + q] : 0.f;
                        c[i * n + n0 + j + q] = hsum(acc[0][q]) + b;
                        if (pair) c[(i + 1) * n + n0 + j + q] = hsum(acc[1][q]) + b;
                    }
                }
            }
        }
    }
}
