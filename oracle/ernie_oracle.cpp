// CPU restatement of the reference's FP32 DiT hot path — TEST INFRASTRUCTURE ONLY (see ernie_oracle.h).
// Compiled with -ffp-contract=off like the reference's library (src/CMakeLists.txt:11-13); the one
// explicit fused multiply-add is the one the reference writes (src/latent_ops.cpp:42).
#include "ernie_oracle.h"
#include "ernie_synth.h"
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace
{
constexpr int kHidden = 4096, kHeads = 32, kHeadDim = 128, kFfn = 12288, kText = 3072, kLatent = 128;
constexpr float kEps = 1e-6f;

float widen(uint16_t bits) { return ernie_synth_bf16_to_float(bits); }
} // namespace

extern "C" {

int orc_num_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int threads)
{
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
}

void orc_synth_bf16(uint64_t seed, uint64_t stream, float scale, float offset, uint16_t *out, int64_t count)
{
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < count; ++i) out[i] = ernie_synth_weight(seed, stream, uint64_t(i), scale, offset);
}

void orc_synth_f32_from_bf16(uint64_t seed, uint64_t stream, float scale, float offset, float *out, int64_t count)
{
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < count; ++i)
        out[i] = widen(ernie_synth_weight(seed, stream, uint64_t(i), scale, offset));
}

void orc_synth_normal_f32(uint64_t seed, uint64_t stream, float scale, float *out, int64_t count)
{
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < count; ++i)
        out[i] = float(ernie_synth_normal(seed, stream, uint64_t(i)) * double(scale));
}

// FlowSchedule::turbo, src/latent_ops.cpp:31-51 (shift 4, PyTorch-style linspace from the nearer end).
int orc_turbo_schedule(int steps, float *sigmas, float *timesteps)
{
    if (steps < 1 || steps > 1000) return -1;
    const float increment = -1.f / float(steps);
    for (int i = 0; i < steps; ++i)
    {
        const float raw = i < (steps + 1) / 2 ? std::fma(increment, float(i), 1.f) : -increment * float(steps - i);
        const float scaled = 4.f * raw;
        const float denominator = 1.f + 3.f * raw;
        sigmas[i] = scaled / denominator;
        timesteps[i] = 1000.f * sigmas[i];
    }
    sigmas[steps] = 0.f;
    return 0;
}

// The literal evenly spaced schedule named by the benchmark configuration (sigma 1 -> 0, no shift),
// evaluated with the same nearer-endpoint linspace as the turbo schedule.
int orc_linear_schedule(int steps, float *sigmas, float *timesteps)
{
    if (steps < 1 || steps > 1000) return -1;
    const float increment = -1.f / float(steps);
    for (int i = 0; i < steps; ++i)
    {
        sigmas[i] = i < (steps + 1) / 2 ? std::fma(increment, float(i), 1.f) : -increment * float(steps - i);
        timesteps[i] = 1000.f * sigmas[i];
    }
    sigmas[steps] = 0.f;
    return 0;
}

// timestep_features, src/denoiser.cpp:22-39 (Timesteps(4096), sin half first).
int orc_timestep_features(float timestep, float *out)
{
    if (!std::isfinite(timestep) || timestep < 0.f || timestep > 1000.f) return -1;
    const float factor = -float(std::log(10000.0));
    for (int i = 0; i < 2048; ++i)
    {
        const float product = factor * float(i);
        const float exponent = product / 2048.f;
        const float phase = timestep * std::exp(exponent);
        out[i] = std::sin(phase);
        out[2048 + i] = std::cos(phase);
    }
    return 0;
}

// rope-inv-freq.f32, tools/prepare_pipeline.py:63: concat over axes (32,48,48) of
// 1 / 256^(arange(0,d,2)/d) in FP32.
void orc_rope_frequencies(float *out)
{
    const int dims[3] = {32, 48, 48};
    int j = 0;
    for (int a = 0; a < 3; ++a)
        for (int i = 0; i < dims[a]; i += 2)
            out[j++] = 1.f / std::pow(256.f, float(i) / float(dims[a]));
}

// make_constants, src/conditioning.cpp:10-44. Token order: image (row-major h x w), then text slots.
int orc_dit_constants(const float *freq, int w, int h, int valid, int text, int token_limit, float *cos_out,
                      float *sin_out, float *mask_out)
{
    if (w < 1 || w > 256 || h < 1 || h > 256 || valid < 1 || text < valid || text > 2048 ||
        w * h + text > token_limit)
        return -1;
    for (int j = 0; j < 64; ++j)
        if (!std::isfinite(freq[j]) || freq[j] <= 0.f) return -1;
    const int image = w * h, length = image + text;
    for (int i = 0; i < length; ++i)
    {
        const int positions[3] = {i < image ? valid : i - image, i < image ? i / w : 0, i < image ? i % w : 0};
        float *c = cos_out + size_t(i) * 128;
        float *s = sin_out + size_t(i) * 128;
        for (int j = 0; j < 64; ++j)
        {
            const int axis = j < 16 ? 0 : j < 40 ? 1 : 2;
            const float phase = float(positions[axis]) * freq[j];
            c[2 * j] = c[2 * j + 1] = std::cos(phase);
            s[2 * j] = s[2 * j + 1] = std::sin(phase);
        }
    }
    for (int k = 0; k < length; ++k) mask_out[k] = k >= image + valid ? -1e30f : 0.f;
    return 0;
}

// ncnn RMSNorm (affine) as wrapped by ErnieNorm in FP32, src/ernie_rmsnorm.cpp:93-97; formula per
// probes/rmsnorm_probe.cpp:85-93: x * (mean(x^2) + eps)^(-1/2) * gamma.
void orc_rmsnorm(const float *x, const float *gamma, int64_t rows, int width, float eps, float *out)
{
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r)
    {
        const float *v = x + r * width;
        double squared = 0;
        for (int i = 0; i < width; ++i) squared += double(v[i]) * v[i];
        const float inverse = float(1.0 / std::sqrt(squared / width + double(eps)));
        float *o = out + r * width;
        for (int i = 0; i < width; ++i) o[i] = v[i] * inverse * gamma[i];
    }
}

// Non-affine LayerNorm(4096, eps 1e-6), head.ncnn.param ln_1 (2=0), probes/rmsnorm_probe.cpp:80-93.
void orc_layernorm(const float *x, int64_t rows, int width, float eps, float *out)
{
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r)
    {
        const float *v = x + r * width;
        double mean = 0;
        for (int i = 0; i < width; ++i) mean += v[i];
        mean /= width;
        double squared = 0;
        for (int i = 0; i < width; ++i) squared += (v[i] - mean) * (v[i] - mean);
        const double inverse = 1.0 / std::sqrt(squared / width + double(eps));
        float *o = out + r * width;
        for (int i = 0; i < width; ++i) o[i] = float((v[i] - mean) * inverse);
    }
}

// ErnieGELU CPU path, src/ernie_gelu.cpp:58: 0.5 x erfc(-x/sqrt2).
void orc_gelu(const float *x, float *out, int64_t count)
{
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < count; ++i) out[i] = 0.5f * x[i] * std::erfc(-0.7071067811865475f * x[i]);
}

// ncnn Swish (nn.SiLU in head.pnnx.param): x / (1 + exp(-x)).
void orc_silu(const float *x, float *out, int64_t count)
{
    for (int64_t i = 0; i < count; ++i) out[i] = x[i] / (1.f + std::exp(-x[i]));
}

// ErnieResidualAdd, src/ernie_residual.cpp:19-92: FP32 a + b.
void orc_residual_add(const float *a, const float *b, float *out, int64_t count)
{
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < count; ++i) out[i] = a[i] + b[i];
}

// ErnieSDPA CPU path (ncnn SDPA with the row mask expanded, src/ernie_attention.cpp:196-221):
// softmax(q k^T / sqrt(width) + mask) v, non-causal. Accumulation in FP64 as the reference's own
// oracle does (tests/test_attention_mask.cpp:75-97, probes/attention_accuracy_probe.cpp:40-56).
// K and V are widened to FP64 once; each dot product and each output row sums 4-lane FP64 vectors.
typedef double v4d __attribute__((vector_size(32)));

static inline v4d load4d(const double *p)
{
    v4d r;
    std::memcpy(&r, p, sizeof(r));
    return r;
}

void orc_sdpa(const float *q, const float *k, const float *v, const float *mask, int heads, int kv_heads,
              int mask_heads, int mask_rows, int nq, int nk, int width, float *out)
{
    const double scale = 1.0 / std::sqrt(double(width));
    const int wp = (width + 3) & ~3; // FP64 rows padded to whole vectors (zeros)
    const int kv_count = kv_heads == 1 ? 1 : heads;
    std::vector<double> kd(size_t(kv_count) * nk * wp, 0.0), vd(size_t(kv_count) * nk * wp, 0.0);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < int64_t(kv_count) * nk; ++r)
        for (int d = 0; d < width; ++d)
        {
            kd[size_t(r) * wp + d] = k[size_t(r) * width + d];
            vd[size_t(r) * wp + d] = v[size_t(r) * width + d];
        }
    // blocks of QB query rows share each pass over K and V (per row the arithmetic is the same)
    constexpr int QB = 16;
    const int qblocks = (nq + QB - 1) / QB;
#pragma omp parallel
    {
        std::vector<double> scores(size_t(QB) * nk), qd(size_t(QB) * wp, 0.0), acc(size_t(QB) * wp);
        double maximum[QB], total[QB];
#pragma omp for schedule(dynamic, 1) collapse(2)
        for (int h = 0; h < heads; ++h)
            for (int b = 0; b < qblocks; ++b)
            {
                const int i0 = b * QB, rows = std::min(QB, nq - i0);
                for (int r = 0; r < rows; ++r)
                {
                    const float *qi = q + (size_t(h) * nq + i0 + r) * width;
                    for (int d = 0; d < width; ++d) qd[size_t(r) * wp + d] = qi[d];
                    maximum[r] = -1e300;
                }
                const int kh = kv_heads == 1 ? 0 : h;
                const double *kh_base = kd.data() + size_t(kh) * nk * wp;
                const double *vh_base = vd.data() + size_t(kh) * nk * wp;
                auto mask_row = [&](int i) -> const float * {
                    return mask ? mask + (size_t(mask_heads == 1 ? 0 : h) * mask_rows + (mask_rows == 1 ? 0 : i)) * nk
                                : nullptr;
                };
                for (int j = 0; j < nk; ++j)
                {
                    const double *kj = kh_base + size_t(j) * wp;
                    for (int r = 0; r < rows; ++r)
                    {
                        const double *qr = qd.data() + size_t(r) * wp;
                        v4d sum = {0, 0, 0, 0};
                        for (int d = 0; d < wp; d += 4) sum += load4d(qr + d) * load4d(kj + d);
                        double s = ((sum[0] + sum[2]) + (sum[1] + sum[3])) * scale;
                        const float *m = mask_row(i0 + r);
                        if (m) s += m[j];
                        scores[size_t(r) * nk + j] = s;
                        maximum[r] = std::max(maximum[r], s);
                    }
                }
                for (int r = 0; r < rows; ++r)
                {
                    double t = 0;
                    double *sr = scores.data() + size_t(r) * nk;
                    for (int j = 0; j < nk; ++j)
                    {
                        sr[j] = std::exp(sr[j] - maximum[r]);
                        t += sr[j];
                    }
                    total[r] = t;
                }
                std::fill(acc.begin(), acc.end(), 0.0);
                for (int j = 0; j < nk; ++j)
                {
                    const double *vj = vh_base + size_t(j) * wp;
                    for (int r = 0; r < rows; ++r)
                    {
                        const double p = scores[size_t(r) * nk + j];
                        if (p == 0.0) continue;
                        double *ar = acc.data() + size_t(r) * wp;
                        const v4d pv = {p, p, p, p};
                        for (int d = 0; d < wp; d += 4)
                        {
                            v4d a4 = load4d(ar + d) + pv * load4d(vj + d);
                            std::memcpy(ar + d, &a4, sizeof(a4));
                        }
                    }
                }
                for (int r = 0; r < rows; ++r)
                {
                    float *o = out + (size_t(h) * nq + i0 + r) * width;
                    for (int d = 0; d < width; ++d) o[d] = float(acc[size_t(r) * wp + d] / total[r]);
                }
            }
    }
}

// euler_step, src/latent_ops.cpp:72-92 (and the contract of check_pair, :22-29).
int orc_euler_step(const float *sample, const float *prediction, float delta, int64_t count, float *out)
{
    if (!std::isfinite(delta) || delta >= 0.f || delta < -1.f) return -1;
    for (int64_t i = 0; i < count; ++i)
    {
        const float change = delta * prediction[i];
        out[i] = sample[i] + change;
    }
    return 0;
}

// finite_latent, src/latent_ops.cpp:60-70.
int orc_finite(const float *x, int64_t count)
{
    for (int64_t i = 0; i < count; ++i)
        if (!std::isfinite(x[i])) return 0;
    return 1;
}

// unpack_for_vae, src/latent_ops.cpp:94-124: BN un-normalise, then channel c -> (c/4, dy, dx).
int orc_unpack_for_vae(const float *packed, const float *mean, const float *variance, int w, int h, float *out)
{
    if (w < 1 || h < 1 || w > 256 || h > 256) return -1;
    float scales[128];
    for (int c = 0; c < 128; ++c)
    {
        if (!std::isfinite(mean[c]) || !std::isfinite(variance[c]) || variance[c] < 0.f) return -1;
        scales[c] = std::sqrt(variance[c] + 1e-5f);
    }
    const int ow = 2 * w;
    for (int c = 0; c < 128; ++c)
    {
        const float *values = packed + size_t(c) * w * h;
        float *target = out + size_t(c / 4) * (2 * h) * ow;
        const int dy = (c % 4) / 2, dx = c % 2;
        for (int y = 0; y < h; ++y)
            for (int x = 0; x < w; ++x)
            {
                const float scaled = values[y * w + x] * scales[c];
                target[(2 * y + dy) * ow + 2 * x + dx] = scaled + mean[c];
            }
    }
    return 0;
}

// One DiT block, in the op order of block.ncnn.param:14-76 / ExportBlock.forward
// (tools/export_dit_block.py:49-68). Input map: modulation rows 0..5 = in1..in6
// (shift_sa, scale_sa, gate_sa, shift_mlp, scale_mlp, gate_mlp), cos = in7, sin = in8, mask = in9.
void orc_block(const float *x, const orc_block_weights *w, const float *mod, const float *cos_t,
               const float *sin_t, const float *mask, int n, float *out)
{
    const float *shift_sa = mod, *scale_sa = mod + kHidden, *gate_sa = mod + 2 * kHidden;
    const float *shift_mlp = mod + 3 * kHidden, *scale_mlp = mod + 4 * kHidden, *gate_mlp = mod + 5 * kHidden;
    const size_t rows = size_t(n);
    std::vector<float> h(rows * kHidden), q(rows * kHidden), k(rows * kHidden), v(rows * kHidden);
    // rmsn_8, add_0 (1 + scale), mul_1, add_2 (+ shift)
    orc_rmsnorm(x, w->gamma_sa, n, kHidden, kEps, h.data());
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < n; ++r)
        for (int i = 0; i < kHidden; ++i)
        {
            float &value = h[size_t(r) * kHidden + i];
            value = value * (1.f + scale_sa[i]) + shift_sa[i];
        }
    // gemm_0/1/2
    orc_linear(h.data(), w->wq, nullptr, n, kHidden, kHidden, q.data());
    orc_linear(h.data(), w->wk, nullptr, n, kHidden, kHidden, k.data());
    orc_linear(h.data(), w->wv, nullptr, n, kHidden, kHidden, v.data());
    // reshape [N,32,128] -> head-major [32][N][128]; rmsn_9/rmsn_10 (width 128) + rotary (:29-57)
    std::vector<float> qh(rows * kHidden), kh(rows * kHidden), vh(rows * kHidden), att(rows * kHidden);
#pragma omp parallel for schedule(static) collapse(2)
    for (int head = 0; head < kHeads; ++head)
        for (int64_t t = 0; t < n; ++t)
        {
            const size_t src = size_t(t) * kHidden + size_t(head) * kHeadDim;
            const size_t dst = (size_t(head) * rows + size_t(t)) * kHeadDim;
            const float *c = cos_t + size_t(t) * kHeadDim;
            const float *s = sin_t + size_t(t) * kHeadDim;
            for (int which = 0; which < 2; ++which)
            {
                const float *gamma = which ? w->gamma_k : w->gamma_q;
                const float *in = (which ? k.data() : q.data()) + src;
                float *o = (which ? kh.data() : qh.data()) + dst;
                double squared = 0;
                for (int d = 0; d < kHeadDim; ++d) squared += double(in[d]) * in[d];
                const float inverse = float(1.0 / std::sqrt(squared / kHeadDim + double(kEps)));
                float normed[kHeadDim];
                for (int d = 0; d < kHeadDim; ++d) normed[d] = in[d] * inverse * gamma[d];
                for (int d = 0; d < 64; ++d)
                {
                    const float first = normed[d], second = normed[d + 64];
                    o[d] = first * c[d] - second * s[d];
                    o[d + 64] = second * c[d + 64] + first * s[d + 64];
                }
            }
            std::memcpy(vh.data() + dst, v.data() + src, sizeof(float) * kHeadDim);
        }
    // sdpa_22 with the 1-row additive mask
    orc_sdpa(qh.data(), kh.data(), vh.data(), mask, kHeads, kHeads, 1, 1, n, n, kHeadDim, att.data());
    // transpose_19 / reshape_15 back to [N,4096]
#pragma omp parallel for schedule(static) collapse(2)
    for (int head = 0; head < kHeads; ++head)
        for (int64_t t = 0; t < n; ++t)
            std::memcpy(h.data() + size_t(t) * kHidden + size_t(head) * kHeadDim,
                        att.data() + (size_t(head) * rows + size_t(t)) * kHeadDim, sizeof(float) * kHeadDim);
    // gemm_3, mul_15 (gate_sa), add_16 (residual, FP32)
    orc_linear(h.data(), w->wo, nullptr, n, kHidden, kHidden, q.data());
    std::vector<float> x1(rows * kHidden);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < n; ++r)
        for (int i = 0; i < kHidden; ++i)
        {
            const size_t idx = size_t(r) * kHidden + i;
            const float gated = gate_sa[i] * q[idx];
            x1[idx] = x[idx] + gated;
        }
    // rmsn_11, add_17, mul_18, add_19
    orc_rmsnorm(x1.data(), w->gamma_mlp, n, kHidden, kEps, h.data());
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < n; ++r)
        for (int i = 0; i < kHidden; ++i)
        {
            float &value = h[size_t(r) * kHidden + i];
            value = value * (1.f + scale_mlp[i]) + shift_mlp[i];
        }
    // gemm_4 (up), gemm_5 (gate), ErnieGELU on gate, mul_20 (up * gelu(gate))
    std::vector<float> up(rows * kFfn), gate(rows * kFfn);
    orc_linear(h.data(), w->wup, nullptr, n, kFfn, kHidden, up.data());
    orc_linear(h.data(), w->wgate, nullptr, n, kFfn, kHidden, gate.data());
    orc_gelu(gate.data(), gate.data(), int64_t(rows) * kFfn);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < int64_t(rows) * kFfn; ++i) up[i] = up[i] * gate[i];
    // gemm_6 (fc2), mul_21 (gate_mlp), add_22 (residual)
    orc_linear(up.data(), w->wfc2, nullptr, n, kHidden, kFfn, q.data());
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < n; ++r)
        for (int i = 0; i < kHidden; ++i)
        {
            const size_t idx = size_t(r) * kHidden + i;
            const float gated = gate_mlp[i] * q[idx];
            out[idx] = x1[idx] + gated;
        }
}

// Input head, head.pnnx.param:4-16 / InputHead.forward (tools/export_dit_heads.py:45-58):
// x = cat(Conv1x1(latent) + b, text_proj(text)); c = L2(SiLU(L1(features)));
// modulation = Linear(SiLU(c)) split into 6 x 4096.
void orc_input_head(const orc_head_weights *w, const float *latent, int width, int height, const float *text,
                    int text_tokens, const float *features, float *x_out, float *c_out, float *mod_out)
{
    const int image = width * height;
    std::vector<float> tokens(size_t(image) * kLatent);
    for (int c = 0; c < kLatent; ++c)
        for (int i = 0; i < image; ++i) tokens[size_t(i) * kLatent + c] = latent[size_t(c) * image + i];
    orc_linear(tokens.data(), w->x_embed_w, w->x_embed_b, image, kHidden, kLatent, x_out);
    orc_linear(text, w->text_proj_w, nullptr, text_tokens, kHidden, kText, x_out + size_t(image) * kHidden);
    std::vector<float> hidden(kHidden), act(kHidden);
    orc_linear(features, w->time1_w, w->time1_b, 1, kHidden, kHidden, hidden.data());
    orc_silu(hidden.data(), act.data(), kHidden);
    orc_linear(act.data(), w->time2_w, w->time2_b, 1, kHidden, kHidden, c_out);
    orc_silu(c_out, act.data(), kHidden);
    orc_linear(act.data(), w->adaln_w, w->adaln_b, 1, 6 * kHidden, kHidden, mod_out);
}

// Output head, head.ncnn.param (output):3-16 / OutputHead.forward (tools/export_dit_heads.py:61-75):
// scale, shift = chunk(Linear(c)) (no SiLU); y = LN(x)(1 + scale) + shift; p = y[:image] Wf^T + bf,
// transposed to [128, h, w].
void orc_output_head(const orc_head_weights *w, const float *x, const float *c, int width, int height,
                     float *prediction)
{
    const int image = width * height;
    std::vector<float> ss(2 * kHidden);
    orc_linear(c, w->final_norm_w, w->final_norm_b, 1, 2 * kHidden, kHidden, ss.data());
    const float *scale = ss.data(), *shift = ss.data() + kHidden;
    std::vector<float> y(size_t(image) * kHidden);
    orc_layernorm(x, image, kHidden, kEps, y.data());
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < image; ++r)
        for (int i = 0; i < kHidden; ++i)
        {
            float &value = y[size_t(r) * kHidden + i];
            value = value * (1.f + scale[i]) + shift[i];
        }
    std::vector<float> p(size_t(image) * kLatent);
    orc_linear(y.data(), w->final_w, w->final_b, image, kLatent, kHidden, p.data());
    for (int i = 0; i < image; ++i)
        for (int ch = 0; ch < kLatent; ++ch) prediction[size_t(ch) * image + i] = p[size_t(i) * kLatent + ch];
}

// run_dit, src/dit.cpp:104-132: input head -> block sequence (src/block_sequence.cpp:56-94) -> output head.
void orc_dit(const orc_head_weights *heads, const orc_block_weights *const *blocks, int num_blocks,
             const float *latent, int width, int height, const float *text, int text_tokens, const float *features,
             const float *cos_t, const float *sin_t, const float *mask, float *prediction)
{
    const int n = width * height + text_tokens;
    std::vector<float> x(size_t(n) * kHidden), y(size_t(n) * kHidden), c(kHidden), mod(6 * kHidden);
    orc_input_head(heads, latent, width, height, text, text_tokens, features, x.data(), c.data(), mod.data());
    for (int b = 0; b < num_blocks; ++b)
    {
        orc_block(x.data(), blocks[b], mod.data(), cos_t, sin_t, mask, n, y.data());
        x.swap(y);
    }
    orc_output_head(heads, x.data(), c.data(), width, height, prediction);
}

// denoise (CPU), src/denoiser.cpp:41-86, including its request checks (:13-20, :46-48).
int orc_denoise(const orc_head_weights *heads, const orc_block_weights *const *blocks, int num_blocks,
                const float *initial, int width, int height, const float *text, int text_tokens,
                const float *cos_t, const float *sin_t, const float *mask, int steps, int start_step, int end_step,
                int schedule, float *latent_out, float *predictions)
{
    if (num_blocks < 1 || num_blocks > 36 || width < 1 || height < 1 || width > 256 || height > 256 ||
        start_step < 0 || start_step > steps || end_step < start_step || end_step > steps)
        return -1;
    std::vector<float> sigmas(size_t(steps) + 1), timesteps(steps);
    if ((schedule == 0 ? orc_turbo_schedule(steps, sigmas.data(), timesteps.data())
                       : orc_linear_schedule(steps, sigmas.data(), timesteps.data())) != 0)
        return -1;
    const int64_t count = int64_t(kLatent) * width * height;
    std::vector<float> sample(initial, initial + count), pred(count), features(kHidden);
    if (!orc_finite(sample.data(), count)) return -1;
    for (int i = start_step; i < end_step; ++i)
    {
        const float delta = sigmas[i + 1] - sigmas[i];
        orc_timestep_features(timesteps[i], features.data());
        orc_dit(heads, blocks, num_blocks, sample.data(), width, height, text, text_tokens, features.data(), cos_t,
                sin_t, mask, pred.data());
        if (orc_euler_step(sample.data(), pred.data(), delta, count, sample.data()) != 0) return -1;
        if (predictions) std::memcpy(predictions + size_t(i - start_step) * count, pred.data(), sizeof(float) * count);
        if (!orc_finite(sample.data(), count)) return i + 1;
    }
    std::memcpy(latent_out, sample.data(), sizeof(float) * count);
    return 0;
}

} // extern "C"
