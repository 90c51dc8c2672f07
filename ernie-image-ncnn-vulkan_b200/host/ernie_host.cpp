// C++ host surface (include/ernie_b200/ernie.h) over the C ABI. Host orchestration only.
#include "ernie_b200/ernie.h"
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <limits>
#include <new>
#include <numeric>
#include <random>
#include <utility>

namespace ernie
{
namespace
{
using Clock = std::chrono::steady_clock;
double seconds_since(Clock::time_point t) { return std::chrono::duration<double>(Clock::now() - t).count(); }

void require(bool ok, const char *message)
{
    if (!ok) throw std::invalid_argument(message);
}

void check_latent(const Tensor &t)
{
    require(!t.empty() && t.dims == 3 && t.c == 128 && t.w >= 1 && t.h >= 1 && t.w <= 256 && t.h <= 256,
            "Expected pack1 FP32 [128,H,W] latent with 1 <= H,W <= 256");
}

void check_latent(const DeviceTensor &t)
{
    require(!t.empty() && t.dims == 3 && t.c == 128 && t.w >= 1 && t.h >= 1 && t.w <= 256 && t.h <= 256 &&
                t.bytes() >= size_t(128) * t.w * t.h * 4,
            "Expected pack1 FP32 [128,H,W] latent with 1 <= H,W <= 256");
}
} // namespace

void check_cuda(int result, const char *action)
{
    if (result == ERNIE_CUDA_OK) return;
    const std::string message = std::string(action) + ": " + ernie_cuda_last_error();
    if (result == ERNIE_CUDA_OUT_OF_MEMORY) throw GpuAllocationError(message);
    throw std::runtime_error(message);
}

// ---- DeviceTensor -------------------------------------------------------------------------------
DeviceTensor::DeviceTensor(GpuContext &ctx, size_t bytes, int w_, int h_, int c_, int dims_)
    : w(w_), h(h_), c(c_), dims(dims_), ctx_(&ctx), bytes_(bytes)
{
    check_cuda(ernie_cuda_malloc(ctx.handle(), bytes, &ptr_), "allocate device tensor");
}

DeviceTensor::DeviceTensor(DeviceTensor &&o) noexcept
    : w(o.w), h(o.h), c(o.c), dims(o.dims), ctx_(o.ctx_), ptr_(o.ptr_), bytes_(o.bytes_)
{
    o.ptr_ = nullptr;
    o.bytes_ = 0;
}

DeviceTensor &DeviceTensor::operator=(DeviceTensor &&o) noexcept
{
    if (this != &o)
    {
        if (ptr_) ernie_cuda_free(ctx_->handle(), ptr_);
        w = o.w, h = o.h, c = o.c, dims = o.dims, ctx_ = o.ctx_, ptr_ = o.ptr_, bytes_ = o.bytes_;
        o.ptr_ = nullptr;
        o.bytes_ = 0;
    }
    return *this;
}

DeviceTensor::~DeviceTensor()
{
    if (ptr_ && ctx_ && ctx_->available()) ernie_cuda_free(ctx_->handle(), ptr_);
}

DeviceTensor DeviceTensor::upload(GpuContext &ctx, const Tensor &host)
{
    DeviceTensor t(ctx, host.total() * 4, host.w, host.h, host.c, host.dims);
    check_cuda(ernie_cuda_upload(ctx.handle(), t.ptr_, host.ptr(), host.total() * 4), "upload tensor");
    return t;
}

Tensor DeviceTensor::download() const
{
    Tensor out;
    out.w = w, out.h = h, out.c = c, out.dims = dims;
    out.data.resize(size_t(w) * h * c);
    if (out.data.size() * 4 > bytes_) throw std::logic_error("Device tensor smaller than its shape");
    check_cuda(ernie_cuda_download(ctx_->handle(), out.ptr(), ptr_, out.data.size() * 4), "download tensor");
    return out;
}

// ---- GpuContext ---------------------------------------------------------------------------------
GpuContext::GpuContext(bool enabled, int requested_index, bool require_device)
{
    if (!enabled)
    {
        initialization_error_ = "GPU disabled";
        if (require_device) throw std::runtime_error("A CUDA device is required");
        return;
    }
    int count = 0;
    if (ernie_cuda_device_count(&count) != ERNIE_CUDA_OK || count < 1)
    {
        initialization_error_ = std::string("No CUDA device: ") + ernie_cuda_last_error();
        if (require_device) throw std::runtime_error(initialization_error_);
        return;
    }
    const int index = requested_index < 0 ? 0 : requested_index;
    if (index >= count)
    {
        initialization_error_ = "CUDA device index out of range";
        if (require_device) throw std::invalid_argument(initialization_error_);
        return;
    }
    const int rc = ernie_cuda_context_create(index, &handle_);
    if (rc != ERNIE_CUDA_OK)
    {
        initialization_error_ = ernie_cuda_last_error();
        handle_ = nullptr;
        if (require_device) check_cuda(rc, "create CUDA context");
        return;
    }
    device_ = index;
}

GpuContext::~GpuContext()
{
    if (handle_) ernie_cuda_context_destroy(handle_);
}

ernie_cuda_context *GpuContext::handle() const
{
    if (!handle_) throw std::logic_error("GPU context is not available");
    return handle_;
}

void GpuContext::synchronize() const { check_cuda(ernie_cuda_context_synchronize(handle()), "synchronize"); }

// ---- latent ops ---------------------------------------------------------------------------------
static FlowSchedule make_schedule(int steps, int kind)
{
    require(steps >= 1 && steps <= 1000, "Steps must be in [1,1000]");
    FlowSchedule s;
    s.sigmas.resize(size_t(steps) + 1);
    s.timesteps.resize(steps);
    check_cuda(ernie_cuda_schedule(steps, kind, s.sigmas.data(), s.timesteps.data()), "schedule");
    return s;
}
FlowSchedule FlowSchedule::turbo(int steps) { return make_schedule(steps, ERNIE_SCHEDULE_TURBO); }
FlowSchedule FlowSchedule::linear(int steps) { return make_schedule(steps, ERNIE_SCHEDULE_LINEAR); }

float FlowSchedule::delta(size_t step) const
{
    if (step >= timesteps.size() || sigmas.size() != timesteps.size() + 1)
        throw std::out_of_range("Euler schedule exhausted or malformed");
    return sigmas[step + 1] - sigmas[step];
}

void euler_step(GpuContext &ctx, const DeviceTensor &sample, const DeviceTensor &prediction, float delta,
                DeviceTensor &next)
{
    check_latent(sample);
    check_latent(prediction);
    require(sample.w == prediction.w && sample.h == prediction.h && std::isfinite(delta) && delta < 0.f && delta >= -1.f,
            "Incompatible Euler shapes or delta outside [-1,0)");
    if (next.empty() || next.bytes() < sample.bytes())
        next = DeviceTensor(ctx, sample.bytes(), sample.w, sample.h, sample.c, 3);
    check_cuda(ernie_cuda_euler_step(ctx.handle(), sample.f32(), prediction.f32(), delta, sample.w, sample.h, next.f32()),
               "Euler step");
}

bool finite_latent(GpuContext &ctx, const DeviceTensor &value)
{
    check_latent(value);
    int finite = 0;
    check_cuda(ernie_cuda_finite_latent(ctx.handle(), value.f32(), value.w, value.h, &finite), "finite check");
    return finite != 0;
}

DeviceTensor unpack_for_vae(GpuContext &ctx, const DeviceTensor &packed, const Tensor &mean, const Tensor &variance)
{
    check_latent(packed);
    require(mean.total() == 128 && variance.total() == 128, "Expected pack1 FP32 [128] BN statistics");
    for (size_t c = 0; c < 128; ++c)
        require(std::isfinite(mean[c]) && std::isfinite(variance[c]) && variance[c] >= 0.f, "Invalid BN statistics");
    const DeviceTensor m = DeviceTensor::upload(ctx, mean), v = DeviceTensor::upload(ctx, variance);
    DeviceTensor out(ctx, size_t(32) * 4 * packed.w * packed.h * 4, 2 * packed.w, 2 * packed.h, 32, 3);
    check_cuda(ernie_cuda_unpack_for_vae(ctx.handle(), packed.f32(), m.f32(), v.f32(), packed.w, packed.h, out.f32()),
               "unpack for VAE");
    ctx.synchronize();
    return out;
}

// ---- conditioning and features --------------------------------------------------------------------
std::vector<Tensor> dit_constants(const std::vector<float> &frequencies, int width, int height, int valid_text,
                                  int text_bucket, int token_limit)
{
    require(frequencies.empty() || frequencies.size() == 64, "Invalid DiT position dimensions or frequency file");
    require(width >= 1 && height >= 1 && text_bucket >= 1 && width * height + text_bucket <= 10240,
            "Invalid DiT position dimensions or frequency file");
    const int n = width * height + text_bucket;
    Tensor cos(128, n), sin(128, n), mask(n, 1);
    const int rc = ernie_cuda_dit_constants(frequencies.empty() ? nullptr : frequencies.data(), width, height,
                                            valid_text, text_bucket, token_limit, cos.ptr(), sin.ptr(), mask.ptr());
    if (rc != ERNIE_CUDA_OK) throw std::invalid_argument(ernie_cuda_last_error());
    return {cos, sin, mask};
}

Tensor pad_text(const Tensor &embeddings, int bucket)
{
    require(!embeddings.empty() && embeddings.dims == 2 && embeddings.w == 3072 && embeddings.h >= 1 &&
                embeddings.h <= bucket && bucket <= 2048,
            "Invalid text embeddings or padding bucket");
    Tensor out(3072, bucket);
    std::copy(embeddings.data.begin(), embeddings.data.end(), out.data.begin());
    return out;
}

Tensor timestep_features(float timestep)
{
    Tensor out(4096);
    const int rc = ernie_cuda_timestep_features(timestep, out.ptr());
    if (rc != ERNIE_CUDA_OK) throw std::invalid_argument(ernie_cuda_last_error());
    return out;
}

// ---- layers ----------------------------------------------------------------------------------------
void set_attention_query_rows(GpuContext &ctx, int rows)
{
    require(rows == 128 || rows == 64 || rows == 32 || rows == 16, "Attention query rows must be 128, 64, 32 or 16");
    check_cuda(ernie_cuda_set_attention_query_rows(ctx.handle(), rows), "set attention query rows");
}

int attention_query_rows(GpuContext &ctx)
{
    int rows = 0;
    check_cuda(ernie_cuda_attention_query_rows(ctx.handle(), &rows), "attention query rows");
    return rows;
}

DeviceTensor sdpa(GpuContext &ctx, const DeviceTensor &q, const DeviceTensor &k, const DeviceTensor &v,
                  const DeviceTensor *mask)
{
    // ncnn layout: q (w=width, h=nq, c=heads), k/v (w=width, h=nk, c=kv_heads), mask (w=nk, h=rows, c=mask_heads)
    require(q.w == k.w && k.w == v.w && k.h == v.h && k.c == v.c && q.w >= 1 && q.w <= 128, "SDPA shapes differ");
    const int mask_heads = mask ? mask->c : 1, mask_rows = mask ? mask->h : 1;
    if (mask) require(mask->w == k.h, "SDPA mask width must equal the key count");
    DeviceTensor out(ctx, q.bytes(), q.w, q.h, q.c, 3);
    check_cuda(ernie_cuda_sdpa(ctx.handle(), q.f32(), k.f32(), v.f32(), mask ? mask->f32() : nullptr, q.c, k.c, mask_heads,
                               mask_rows, q.h, k.h, q.w, out.f32()),
               "SDPA");
    return out;
}

DeviceTensor rms_norm(GpuContext &ctx, const DeviceTensor &x, const Tensor &gamma, float eps)
{
    require(x.w == 128 || x.w == 3072 || x.w == 4096, "RMSNorm width must be 128, 3072 or 4096");
    require(int(gamma.total()) == x.w, "RMSNorm affine weights must match the width");
    const DeviceTensor g = DeviceTensor::upload(ctx, gamma);
    DeviceTensor out(ctx, x.bytes(), x.w, x.h, x.c, x.dims);
    check_cuda(ernie_cuda_rmsnorm(ctx.handle(), x.f32(), g.f32(), int64_t(x.h) * x.c, x.w, eps, out.f32()), "RMSNorm");
    ctx.synchronize();
    return out;
}

DeviceTensor layer_norm(GpuContext &ctx, const DeviceTensor &x, float eps)
{
    require(x.w == 4096, "LayerNorm width must be 4096");
    DeviceTensor out(ctx, x.bytes(), x.w, x.h, x.c, x.dims);
    check_cuda(ernie_cuda_layernorm(ctx.handle(), x.f32(), int64_t(x.h) * x.c, x.w, eps, out.f32()), "LayerNorm");
    return out;
}

void gelu_inplace(GpuContext &ctx, DeviceTensor &x)
{
    const int64_t count = int64_t(x.w) * x.h * x.c;
    check_cuda(ernie_cuda_gelu(ctx.handle(), x.f32(), count), "ErnieGELU");
}

DeviceTensor residual_add(GpuContext &ctx, const DeviceTensor &a, const DeviceTensor &b)
{
    require(a.w == b.w && a.h == b.h && a.c == b.c, "Residual shapes differ");
    DeviceTensor out(ctx, a.bytes(), a.w, a.h, a.c, a.dims);
    check_cuda(ernie_cuda_residual_add(ctx.handle(), a.f32(), b.f32(), out.f32(), int64_t(a.w) * a.h * a.c),
               "ErnieResidualAdd");
    return out;
}

// ---- weights ------------------------------------------------------------------------------------------
DitModel::DitModel(GpuContext &ctx, int num_blocks) : ctx_(ctx), num_blocks_(num_blocks)
{
    require(num_blocks >= 1 && num_blocks <= 36, "Require 1..36 blocks");
    check_cuda(ernie_cuda_model_create(ctx.handle(), num_blocks, &handle_), "allocate DiT weights");
}

DitModel::~DitModel()
{
    if (handle_) ernie_cuda_model_destroy(handle_);
}

void DitModel::upload_block(int block, const BlockWeights &w)
{
    const size_t sq = size_t(4096) * 4096, ffn = size_t(12288) * 4096;
    require(w.wq.size() == sq && w.wk.size() == sq && w.wv.size() == sq && w.wo.size() == sq && w.wup.size() == ffn &&
                w.wgate.size() == ffn && w.wfc2.size() == ffn && w.gamma_sa.size() == 4096 &&
                w.gamma_mlp.size() == 4096 && w.gamma_q.size() == 128 && w.gamma_k.size() == 128,
            "Block weights must provide all 11 tensors with the ERNIE shapes");
    const ernie_cuda_block_weights c{w.wq.data(),       w.wk.data(),        w.wv.data(),      w.wo.data(),
                                     w.wup.data(),      w.wgate.data(),     w.wfc2.data(),    w.gamma_sa.data(),
                                     w.gamma_mlp.data(), w.gamma_q.data(), w.gamma_k.data()};
    check_cuda(ernie_cuda_model_upload_block(handle_, block, &c), "upload block weights");
}

void DitModel::upload_heads(const HeadWeights &w)
{
    const ernie_cuda_head_weights c{w.x_embed_w.data(), w.x_embed_b.data(), w.text_proj_w.data(), w.time1_w.data(),
                                    w.time1_b.data(),   w.time2_w.data(),   w.time2_b.data(),     w.adaln_w.data(),
                                    w.adaln_b.data(),   w.final_norm_w.data(), w.final_norm_b.data(), w.final_w.data(),
                                    w.final_b.data()};
    check_cuda(ernie_cuda_model_upload_heads(handle_, &c), "upload head weights");
}

void DitModel::synthesize(uint64_t seed) { check_cuda(ernie_cuda_model_synthesize(handle_, seed), "synthesize weights"); }

uint64_t DitModel::bytes() const
{
    uint64_t b = 0;
    check_cuda(ernie_cuda_model_bytes(handle_, &b), "model bytes");
    return b;
}

// ---- sessions, block sequence, DiT, denoise --------------------------------------------------------------
DenoiseSession::DenoiseSession(DitModel &model, int width, int height, int text_tokens, int valid_text,
                               Precision precision)
    : model_(model), width_(width), height_(height), tokens_(width * height + text_tokens)
{
    const ernie_cuda_shape shape{width, height, text_tokens, valid_text};
    const int rc = ernie_cuda_session_create(model.handle(), &shape,
                                             precision == Precision::FP32 ? ERNIE_PRECISION_FP32 : ERNIE_PRECISION_BF16,
                                             &handle_);
    if (rc == ERNIE_CUDA_ERROR) throw std::invalid_argument(ernie_cuda_last_error());
    check_cuda(rc, "create denoise session");
}

DenoiseSession::~DenoiseSession()
{
    if (handle_) ernie_cuda_session_destroy(handle_);
}

void DenoiseSession::set_constants(const std::vector<Tensor> &k)
{
    require(k.size() == 4, "Require four constants: text, cosine, sine and mask");
    const size_t n = size_t(tokens_);
    require(k[1].total() == n * 128 && k[2].total() == n * 128 && k[3].total() == n, "Constants do not match the shape");
    require(k[0].empty() || k[0].total() == size_t(tokens_ - width_ * height_) * 3072, "Text must be [slots][3072]");
    check_cuda(ernie_cuda_session_set_conditioning(handle_, k[0].empty() ? nullptr : k[0].ptr(), k[1].ptr(), k[2].ptr(),
                                                   k[3].ptr()),
               "set constants");
}

void run_block_sequence(DenoiseSession &s, DeviceTensor &x, const DeviceTensor &modulation, int first, int count,
                        BlockSequenceStats &stats)
{
    require(count >= 1 && first >= 0 && first + count <= s.model().num_blocks() && count <= 36,
            "Require 1..36 blocks");
    require(x.w == 4096 && x.h == s.tokens() && x.bytes() >= size_t(s.tokens()) * 4096 * 4, "x must be [N][4096] FP32");
    require(modulation.bytes() >= size_t(6) * 4096 * 4, "Require six shared modulation vectors");
    stats = {};
    const auto start = Clock::now();
    check_cuda(ernie_cuda_session_blocks(s.handle(), first, count, x.f32(), modulation.f32()), "run block sequence");
    s.model().context().synchronize();
    stats.compute_seconds.push_back(seconds_since(start));
    stats.compute_submissions = 1;
}

DeviceTensor run_dit(DenoiseSession &s, const DeviceTensor &latent, float timestep, DitStats &stats)
{
    check_latent(latent);
    require(latent.w == s.width() && latent.h == s.height(), "Latent does not match the session shape");
    stats = {};
    DeviceTensor prediction(s.model().context(), latent.bytes(), latent.w, latent.h, 128, 3);
    const auto start = Clock::now();
    check_cuda(ernie_cuda_session_dit(s.handle(), latent.f32(), timestep, prediction.f32()), "run DiT");
    stats.blocks.compute_seconds.push_back(seconds_since(start));
    return prediction;
}

Tensor denoise(DenoiseSession &s, const Tensor &initial, int steps, std::vector<DenoiseStepStats> &stats,
               const StepObserver &observer, int start_step, int schedule_kind)
{
    check_latent(initial);
    require(initial.w == s.width() && initial.h == s.height(), "Latent does not match the session shape");
    require(start_step >= 0 && start_step <= steps, "Denoising start step must be in [0,steps]");
    const FlowSchedule schedule = schedule_kind == ERNIE_SCHEDULE_LINEAR ? FlowSchedule::linear(steps)
                                                                           : FlowSchedule::turbo(steps);
    stats.clear();
    Tensor sample = initial;
    for (float v : sample.data) require(std::isfinite(v), "Initial latent is not finite");
    if (!observer)
    {
        // the whole range in one CUDA graph; per-step stats carry the range's average time
        const auto start = Clock::now();
        int failed = 0;
        const int rc = ernie_cuda_session_denoise(s.handle(), initial.ptr(), sample.ptr(), steps, start_step, steps,
                                                  schedule_kind, nullptr, &failed);
        const double each = (steps - start_step) ? seconds_since(start) / (steps - start_step) : 0.0;
        const int done = rc == ERNIE_CUDA_OK ? steps : (failed ? failed : start_step);
        for (int i = start_step; i < steps && i < std::max(done, start_step + 1); ++i)
        {
            DenoiseStepStats st;
            st.timestep = schedule.timesteps[i];
            st.delta = schedule.delta(i);
            st.elapsed_seconds = each;
            st.complete = rc == ERNIE_CUDA_OK || i + 1 < done;
            stats.push_back(st);
        }
        if (failed) throw std::runtime_error("Non-finite latent after denoise step " + std::to_string(failed));
        check_cuda(rc, "denoise");
        return sample;
    }
    Tensor prediction(s.width(), s.height(), 128);
    for (int i = start_step; i < steps; ++i)
    {
        DenoiseStepStats st;
        st.timestep = schedule.timesteps[i];
        st.delta = schedule.delta(i);
        const auto start = Clock::now();
        int failed = 0;
        const int rc = ernie_cuda_session_denoise(s.handle(), sample.ptr(), sample.ptr(), steps, i, i + 1, schedule_kind,
                                                  prediction.ptr(), &failed);
        st.elapsed_seconds = seconds_since(start);
        if (rc != ERNIE_CUDA_OK)
        {
            stats.push_back(st);
            if (failed) throw std::runtime_error("Non-finite latent after denoise step " + std::to_string(failed));
            check_cuda(rc, "denoise step");
        }
        st.complete = true;
        stats.push_back(st);
        observer(size_t(i), prediction, sample);
    }
    return sample;
}

// ---- recovery (src/vulkan_denoise.cpp:40-202 semantics) ------------------------------------------------
Tensor denoise_with_recovery(DenoiseBackend &backend, const Tensor &initial, int steps, int start_step,
                             const CudaDenoiseSettings &settings, CudaDenoiseStats &total,
                             const CudaDenoiseObservers &observer)
{
    check_latent(initial);
    require(settings.retries <= 3 && start_step >= 0 && start_step <= steps, "Invalid recovery session");
    for (float v : initial.data) require(std::isfinite(v), "Invalid recovery session");
    const FlowSchedule schedule = settings.schedule == ERNIE_SCHEDULE_LINEAR ? FlowSchedule::linear(steps)
                                                                               : FlowSchedule::turbo(steps);
    total = {};
    Tensor checkpoint = initial;
    int resume = start_step;
    for (unsigned attempt = 0; resume < steps; ++attempt)
    {
        total.query_rows = 128 >> attempt;
        std::string failure;
        bool observer_failed = false;
        try
        {
            backend.begin_attempt(attempt, checkpoint, total.query_rows);
            try
            {
                for (int i = resume; i < steps; ++i)
                {
                    if (settings.before_step) settings.before_step(attempt, i);
                    DenoiseStepStats st;
                    st.timestep = schedule.timesteps[i];
                    st.delta = schedule.delta(i);
                    const auto start = Clock::now();
                    Tensor prediction = backend.run_step(i, st.timestep, st.delta);
                    Tensor saved = backend.latent();
                    for (float v : saved.data)
                        if (!std::isfinite(v)) throw std::runtime_error("Non-finite latent after denoise step " + std::to_string(i + 1));
                    // commit only after the whole checkpoint transfer succeeded
                    checkpoint = std::move(saved);
                    resume = i + 1;
                    st.elapsed_seconds = seconds_since(start);
                    st.complete = true;
                    if (observer.step)
                    {
                        try
                        {
                            observer.step(size_t(i), prediction, checkpoint, st);
                        }
                        catch (...)
                        {
                            observer_failed = true;
                            throw;
                        }
                    }
                }
            }
            catch (...)
            {
                backend.end_attempt();
                throw;
            }
            backend.end_attempt();
        }
        catch (const GpuAllocationError &error)
        {
            if (observer_failed) throw;
            failure = error.what();
        }
        catch (const std::bad_alloc &)
        {
            if (observer_failed) throw;
            failure = "Memory allocation failed";
        }
        if (failure.empty()) break;
        if (attempt >= settings.retries)
            throw GpuAllocationError("Denoise allocation recovery exhausted after " + std::to_string(attempt) +
                                     " retries at step " + std::to_string(resume + 1) + ": " + failure);
        ++total.retries;
        if (observer.retry) observer.retry(total.retries, resume, 128 >> (attempt + 1), failure);
    }
    return checkpoint;
}

CudaDenoiseBackend::CudaDenoiseBackend(DitModel &model, int width, int height, int text_tokens, int valid_text,
                                       Precision precision, std::vector<Tensor> constants)
    : model_(model), width_(width), height_(height), text_(text_tokens), valid_(valid_text), precision_(precision),
      constants_(std::move(constants))
{
}

void CudaDenoiseBackend::begin_attempt(unsigned, const Tensor &checkpoint, int query_rows)
{
    // each attempt owns its activations; a retry rebuilds them from the host checkpoint
    session_ = std::make_unique<DenoiseSession>(model_, width_, height_, text_, valid_, precision_);
    session_->set_constants(constants_);
    set_attention_query_rows(model_.context(), query_rows);
    float *latent = nullptr;
    check_cuda(ernie_cuda_session_latent(session_->handle(), &latent), "session latent");
    check_cuda(ernie_cuda_upload(model_.context().handle(), latent, checkpoint.ptr(), checkpoint.total() * 4),
               "upload checkpoint");
}

Tensor CudaDenoiseBackend::run_step(int step, float, float)
{
    Tensor latent_now = latent();
    Tensor prediction(width_, height_, 128);
    int failed = 0;
    const int rc = ernie_cuda_session_denoise(session_->handle(), latent_now.ptr(), latent_now.ptr(), steps, step,
                                              step + 1, ERNIE_SCHEDULE_TURBO, prediction.ptr(), &failed);
    if (failed) throw std::runtime_error("Non-finite latent after denoise step " + std::to_string(failed));
    check_cuda(rc, "denoise step");
    return prediction;
}

Tensor CudaDenoiseBackend::latent()
{
    Tensor out(width_, height_, 128);
    float *latent = nullptr;
    check_cuda(ernie_cuda_session_latent(session_->handle(), &latent), "session latent");
    check_cuda(ernie_cuda_download(model_.context().handle(), out.ptr(), latent, out.total() * 4), "download latent");
    return out;
}

void CudaDenoiseBackend::end_attempt() { session_.reset(); }

// ---- pipeline DiT stage -----------------------------------------------------------------------
Tensor read_tensor(const std::string &path, int w, int h, int c)
{
    require(w >= 1 && h >= 1 && c >= 1, "Invalid tensor shape");
    std::error_code ec;
    const auto bytes = std::filesystem::file_size(path, ec);
    if (ec || bytes != size_t(w) * h * c * 4) throw std::runtime_error("Wrong tensor size: " + path);
    Tensor out = c > 1 ? Tensor(w, h, c) : h > 1 ? Tensor(w, h) : Tensor(w);
    std::ifstream file(path, std::ios::binary);
    if (!file.read(reinterpret_cast<char *>(out.ptr()), std::streamsize(out.total() * 4)))
        throw std::runtime_error("Tensor read failed");
    for (float v : out.data)
        if (!std::isfinite(v)) throw std::runtime_error("Tensor contains non-finite values: " + path);
    return out;
}

void write_tensor(const std::string &path, const Tensor &value)
{
    if (std::filesystem::exists(path)) throw std::runtime_error("Trace file exists");
    if (value.empty()) throw std::runtime_error("Trace tensor must be FP32");
    std::ofstream out(path, std::ios::binary);
    out.write(reinterpret_cast<const char *>(value.ptr()), std::streamsize(value.total() * 4));
    if (!out) throw std::runtime_error("Trace write failed");
}

std::string numbered(const std::string &stem, int index)
{
    return stem + (index < 10 ? "0" : "") + std::to_string(index);
}

Tensor initial_noise(int width, int height, uint32_t seed)
{
    require(width >= 1 && height >= 1 && width <= 256 && height <= 256, "Invalid latent shape");
    Tensor noise(width, height, 128);
    std::mt19937 engine(seed);
    std::normal_distribution<float> normal(0.f, 1.f);
    for (float &v : noise.data) v = normal(engine); // channel-major: channel c holds values [c*w*h, (c+1)*w*h)
    return noise;
}

namespace
{
bool finite_latent_tensor(const Tensor &t)
{
    return !t.empty() && t.dims == 3 && t.c == 128 &&
           std::all_of(t.data.begin(), t.data.end(), [](float v) { return std::isfinite(v); });
}

// An img2img request starts inside a flow schedule of 1..1000 steps whose sigmas run from exactly one
// down to exactly zero, finite, strictly decreasing and inside [0, 1].
void check_img2img_schedule(const FlowSchedule &schedule)
{
    const std::vector<float> &sigma = schedule.sigmas;
    const size_t steps = schedule.timesteps.size();
    require(steps >= 1 && steps <= 1000 && sigma.size() == steps + 1 && sigma.front() == 1.f && sigma.back() == 0.f,
            "Invalid img2img flow schedule");
    for (size_t i = 0; i < steps; ++i)
    {
        const bool ok = std::isfinite(sigma[i]) && std::isfinite(schedule.timesteps[i]) && sigma[i] > sigma[i + 1] &&
                        sigma[i] >= 0.f && sigma[i] <= 1.f;
        require(ok, "Img2img flow schedule must descend from one to zero");
    }
}

// Steps an img2img request runs: steps * strength rounded half up in FP32, at least one and at most all.
int img2img_denoise_steps(int steps, float strength)
{
    const int rounded = int(std::floor(float(steps) * strength + .5f));
    return std::clamp(rounded, 1, steps);
}

// sigma * noise + (1 - sigma) * image with each product and the sum rounded to FP32 on its own (this
// file is compiled without floating-point contraction).
Tensor noised_image(const Tensor &image, const Tensor &noise, float sigma)
{
    Tensor out(image.w, image.h, 128);
    const float kept = 1.f - sigma;
    std::transform(noise.data.begin(), noise.data.end(), image.data.begin(), out.data.begin(), [&](float n, float x) {
        const float noise_part = sigma * n;
        const float image_part = kept * x;
        return noise_part + image_part;
    });
    if (!finite_latent_tensor(out)) throw std::runtime_error("Non-finite img2img initial latent");
    return out;
}
} // namespace

Img2ImgStart make_img2img_start(const Tensor &encoded, const Tensor &saved_noise, const FlowSchedule &schedule,
                                float strength, int threads)
{
    require(std::isfinite(strength) && strength >= 0.f && strength <= 1.f && threads >= 1 && threads <= 256,
            "Img2img requires strength in [0,1] and threads in [1,256]");
    check_img2img_schedule(schedule);
    require(finite_latent_tensor(encoded), "Encoded img2img latent must be finite");
    const int steps = int(schedule.timesteps.size());
    Img2ImgStart start;
    if (strength == 0.f)
    {
        start.start_step = steps; // nothing to denoise: the encoded image itself
        start.latent = encoded;
        return start;
    }
    require(finite_latent_tensor(saved_noise) && saved_noise.w == encoded.w && saved_noise.h == encoded.h,
            "Img2img noise must be finite and match the encoded shape");
    start.denoise_steps = img2img_denoise_steps(steps, strength);
    start.start_step = steps - start.denoise_steps;
    start.sigma = schedule.sigmas[size_t(start.start_step)];
    start.latent = start.sigma == 1.f ? saved_noise : noised_image(encoded, saved_noise, start.sigma);
    return start;
}

DitStageResult run_dit_stage(DitModel &model, const Tensor &text, int text_bucket, const std::vector<float> &frequencies,
                             const DitStageRequest &r, const std::function<void(const DitStageProgress &)> &notify)
{
    require(r.width % 16 == 0 && r.height % 16 == 0 && r.width >= 16 && r.height >= 16 && r.width <= 4096 &&
                r.height <= 4096,
            "Width and height must be multiples of 16 in [16,4096]");
    require(r.steps >= 1 && r.steps <= 1000, "Steps must be in [1,1000]");
    require(text.dims == 2 && text.w == 3072 && text.h >= 1 && text.h <= text_bucket, "Text must be [T][3072], T <= bucket");
    require(r.oom_retries <= 3, "oom_retries must be in [0,3]");
    const int w = r.width / 16, h = r.height / 16, valid = text.h;
    const auto rotary = dit_constants(frequencies, w, h, valid, text_bucket);
    std::vector<Tensor> constants{pad_text(text, text_bucket), rotary[0], rotary[1], rotary[2]};
    const Tensor noise = r.latent.empty() ? initial_noise(w, h, r.seed) : read_tensor(r.latent, w, h, 128);
    DitStageResult result;
    Tensor initial = noise;
    if (!r.encoded.empty())
    {
        // img2img (src/pipeline.cpp:533-538): the start latent and step from the encoded image
        require(r.encoded.w == w && r.encoded.h == h, "Encoded image latent does not match the request size");
        Img2ImgStart start = make_img2img_start(r.encoded, noise, FlowSchedule::turbo(r.steps), r.strength);
        initial = std::move(start.latent);
        result.start_step = start.start_step;
    }
    // progress counts the executed steps (src/pipeline.cpp:180-186): step i is number i - start + 1
    auto step_done = [&](int i, double seconds) {
        if (notify) notify({"denoise", i - result.start_step + 1, r.steps - result.start_step, seconds});
    };
    auto recover = [&](const Tensor &from, int start) {
        CudaDenoiseBackend backend(model, w, h, text_bucket, valid, r.precision, constants);
        backend.steps = r.steps;
        CudaDenoiseSettings settings;
        settings.retries = r.oom_retries;
        CudaDenoiseObservers observers;
        observers.step = [&](size_t i, const Tensor &prediction, const Tensor &latent, const DenoiseStepStats &st) {
            if (!r.trace.empty())
            {
                write_tensor((std::filesystem::path(r.trace) / ("prediction-" + std::to_string(i) + ".f32")).string(),
                             prediction);
                write_tensor((std::filesystem::path(r.trace) / ("step-" + std::to_string(i) + ".f32")).string(), latent);
            }
            result.steps.push_back(st);
            step_done(int(i), st.elapsed_seconds);
        };
        observers.retry = [&](unsigned retry, int, int, const std::string &) {
            if (notify) notify({"memory-recovery", int(retry), int(r.oom_retries), 0});
        };
        return denoise_with_recovery(backend, from, r.steps, start, settings, result.recovery, observers);
    };
    if (result.start_step >= r.steps)
    {
        result.latent = initial; // strength 0: the reconstruction latent, no step runs
        return result;
    }
    if (!r.trace.empty())
    {
        require(std::filesystem::is_directory(r.trace), "Trace folder does not exist");
        result.latent = recover(initial, result.start_step);
        return result;
    }
    try
    {
        DenoiseSession session(model, w, h, text_bucket, valid, r.precision);
        session.set_constants(constants);
        result.latent = denoise(session, initial, r.steps, result.steps, {}, result.start_step);
        for (size_t i = 0; i < result.steps.size(); ++i)
            step_done(result.start_step + int(i), result.steps[i].elapsed_seconds);
    }
    catch (const GpuAllocationError &)
    {
        result.steps.clear();
        result.latent = recover(initial, result.start_step);
    }
    return result;
}

// ---- the VAE stage --------------------------------------------------------------------------------
RgbImage rgb_image(const Tensor &decoded)
{
    if (decoded.empty() || decoded.dims != 3 || decoded.c != 3) throw std::runtime_error("VAE output must be pack1 RGB FP32");
    // [-1, 1] -> [0, 1] clamped -> bytes by round-to-nearest-even of value * 255, as FP32 arithmetic
    auto to_byte = [](float v) {
        if (!std::isfinite(v)) throw std::runtime_error("VAE produced non-finite pixels");
        const float unit = std::clamp(v / 2.f + .5f, 0.f, 1.f);
        return static_cast<uint8_t>(std::nearbyint(unit * 255.f));
    };
    const size_t plane = size_t(decoded.w) * size_t(decoded.h);
    RgbImage image{decoded.w, decoded.h, std::vector<uint8_t>(plane * 3)};
    uint8_t *out = image.pixels.data();
    for (size_t p = 0; p < plane; ++p)
        for (size_t c = 0; c < 3; ++c) *out++ = to_byte(decoded.data[c * plane + p]); // interleaved RGB
    return image;
}

VaeDecoder::VaeDecoder(GpuContext &ctx) : ctx_(ctx)
{
    require(ctx.available(), "VAE decoder needs a CUDA device");
    check_cuda(ernie_cuda_vae_create(ctx.handle(), &handle_), "create VAE decoder");
}

VaeDecoder::~VaeDecoder()
{
    if (handle_) ernie_cuda_vae_destroy(handle_);
}

std::vector<std::pair<std::string, std::vector<int>>> VaeDecoder::tensors()
{
    int count = 0;
    check_cuda(ernie_cuda_vae_tensor_count(&count), "VAE tensor count");
    std::vector<std::pair<std::string, std::vector<int>>> out;
    for (int i = 0; i < count; ++i)
    {
        char name[128];
        int dims[4] = {0, 0, 0, 0}, ndim = 0;
        check_cuda(ernie_cuda_vae_tensor_info(i, name, sizeof(name), dims, &ndim), "VAE tensor info");
        out.emplace_back(name, std::vector<int>(dims, dims + ndim));
    }
    return out;
}

void VaeDecoder::upload(const std::string &name, const Tensor &value)
{
    const int rc = ernie_cuda_vae_upload(handle_, name.c_str(), value.ptr(), value.total());
    if (rc == ERNIE_CUDA_ERROR) throw std::invalid_argument(ernie_cuda_last_error());
    check_cuda(rc, "upload VAE tensor");
}

void VaeDecoder::synthesize(uint64_t seed, bool bf16_weights)
{
    check_cuda(ernie_cuda_vae_synthesize(handle_, seed, bf16_weights ? 1 : 0), "synthesize VAE weights");
}

namespace
{
int precision_code(Precision p) { return p == Precision::FP32 ? ERNIE_PRECISION_FP32 : ERNIE_PRECISION_BF16; }

void check_unpacked(int c, int w, int h, int dims)
{
    require(dims == 3 && c == 32 && w >= 1 && h >= 1 && w <= 256 && h <= 256 && w * h <= 57344,
            "Expected pack1 FP32 [32,H,W] unpacked latent with 1 <= H,W <= 256 and H*W <= 57344");
}
} // namespace

Tensor VaeDecoder::decode(const Tensor &unpacked, Precision precision, VaeStats *stats)
{
    check_unpacked(unpacked.c, unpacked.w, unpacked.h, unpacked.dims);
    if (stats) stats->details.clear();
    const auto begin = Clock::now();
    Tensor decoded(8 * unpacked.w, 8 * unpacked.h, 3);
    const int rc = ernie_cuda_vae_decode(handle_, unpacked.ptr(), unpacked.w, unpacked.h, precision_code(precision),
                                         decoded.ptr(), nullptr, nullptr);
    if (stats)
        stats->details.push_back({"extract_compute_composite", rc == ERNIE_CUDA_OK ? "complete" : "failed",
                                  seconds_since(begin)});
    check_cuda(rc, "Decode VAE");
    return decoded;
}

DeviceTensor VaeDecoder::decode(const DeviceTensor &unpacked, Precision precision, RgbImage *image)
{
    check_unpacked(unpacked.c, unpacked.w, unpacked.h, unpacked.dims);
    const int w = 8 * unpacked.w, h = 8 * unpacked.h;
    DeviceTensor decoded(ctx_, size_t(3) * w * h * 4, w, h, 3, 3);
    DeviceTensor bytes;
    if (image) bytes = DeviceTensor(ctx_, size_t(3) * w * h, w, h, 3, 3);
    int nonfinite = 0;
    check_cuda(ernie_cuda_vae_decode_device(handle_, unpacked.f32(), unpacked.w, unpacked.h, precision_code(precision),
                                            decoded.f32(), image ? static_cast<uint8_t *>(bytes.data()) : nullptr,
                                            &nonfinite),
               "Decode VAE");
    if (image)
    {
        if (nonfinite) throw std::runtime_error("VAE produced non-finite pixels");
        image->width = w;
        image->height = h;
        image->pixels.resize(size_t(3) * w * h);
        check_cuda(ernie_cuda_download(ctx_.handle(), image->pixels.data(), bytes.data(), image->pixels.size()),
                   "download RGB bytes");
    }
    return decoded;
}

VaeStageResult run_vae_stage(VaeDecoder &vae, const Tensor &latent, const Tensor &mean, const Tensor &variance,
                             Precision precision, const std::string &trace)
{
    check_latent(latent);
    GpuContext &ctx = vae.context();
    const auto begin = Clock::now();
    VaeStageResult result;
    const DeviceTensor packed = DeviceTensor::upload(ctx, latent);
    const DeviceTensor unpacked = unpack_for_vae(ctx, packed, mean, variance);
    const DeviceTensor decoded = vae.decode(unpacked, precision, &result.image);
    if (decoded.w != latent.w * 16 || decoded.h != latent.h * 16)
        throw std::runtime_error("Decoded resolution differs from model");
    result.decoded = decoded.download();
    result.unpacked = unpacked.download();
    if (!trace.empty())
    {
        const std::filesystem::path folder(trace);
        write_tensor((folder / "final.f32").string(), latent);
        write_tensor((folder / "unpacked.f32").string(), result.unpacked);
        write_tensor((folder / "decoded.f32").string(), result.decoded);
    }
    result.seconds = seconds_since(begin);
    return result;
}

// ---- the VAE encoder ---------------------------------------------------------------------------------
VaeEncoder::VaeEncoder(GpuContext &ctx) : ctx_(ctx)
{
    require(ctx.available(), "VAE encoder needs a CUDA device");
    check_cuda(ernie_cuda_vae_encoder_create(ctx.handle(), &handle_), "create VAE encoder");
}

VaeEncoder::~VaeEncoder()
{
    if (handle_) ernie_cuda_vae_encoder_destroy(handle_);
}

std::vector<std::pair<std::string, std::vector<int>>> VaeEncoder::tensors()
{
    int count = 0;
    check_cuda(ernie_cuda_vae_encoder_tensor_count(&count), "VAE encoder tensor count");
    std::vector<std::pair<std::string, std::vector<int>>> out;
    for (int i = 0; i < count; ++i)
    {
        char name[128];
        int dims[4] = {0, 0, 0, 0}, ndim = 0;
        check_cuda(ernie_cuda_vae_encoder_tensor_info(i, name, sizeof(name), dims, &ndim), "VAE encoder tensor info");
        out.emplace_back(name, std::vector<int>(dims, dims + ndim));
    }
    return out;
}

void VaeEncoder::upload(const std::string &name, const Tensor &value)
{
    const int rc = ernie_cuda_vae_encoder_upload(handle_, name.c_str(), value.ptr(), value.total());
    if (rc == ERNIE_CUDA_ERROR) throw std::invalid_argument(ernie_cuda_last_error());
    check_cuda(rc, "upload VAE encoder tensor");
}

void VaeEncoder::synthesize(uint64_t seed, bool bf16_weights)
{
    check_cuda(ernie_cuda_vae_encoder_synthesize(handle_, seed, bf16_weights ? 1 : 0), "synthesize VAE encoder");
}

VaeEncoding encode_vae(VaeEncoder &encoder, const RgbImage &rgb, Precision precision)
{
    const bool shape_ok = rgb.width >= 16 && rgb.height >= 16 && rgb.width % 16 == 0 && rgb.height % 16 == 0 &&
                          rgb.width <= 2048 && rgb.height <= 2048;
    if (!shape_ok || rgb.pixels.size() != size_t(rgb.width) * size_t(rgb.height) * 3)
        throw std::invalid_argument("RGB shape has no VAE encoder program");
    VaeEncoding out;
    out.mean = Tensor(rgb.width / 8, rgb.height / 8, 32);
    out.packed = Tensor(rgb.width / 16, rgb.height / 16, 128);
    out.normalized = Tensor(rgb.width / 16, rgb.height / 16, 128);
    int nonfinite = 0;
    check_cuda(ernie_cuda_vae_encode(encoder.handle(), rgb.pixels.data(), rgb.width, rgb.height,
                                     precision_code(precision), out.mean.ptr(), out.packed.ptr(),
                                     out.normalized.ptr(), &nonfinite),
               "Encode VAE");
    if (nonfinite)
    {
        const std::pair<const char *, const Tensor *> outputs[3] = {
            {"mean", &out.mean}, {"packed", &out.packed}, {"normalized", &out.normalized}};
        for (const auto &o : outputs)
            for (float v : o.second->data)
                if (!std::isfinite(v)) throw std::runtime_error(std::string("Non-finite VAE encoder ") + o.first);
        throw std::runtime_error("Non-finite VAE encoder output");
    }
    return out;
}

// ---- the prompt encoder -----------------------------------------------------------------------------
namespace
{
std::vector<const char *> c_paths(const std::vector<std::string> &files)
{
    require(!files.empty(), "No safetensors files");
    std::vector<const char *> out;
    for (const auto &f : files) out.push_back(f.c_str());
    return out;
}

void check_request(int rc, const char *action)
{
    if (rc == ERNIE_CUDA_ERROR) throw std::invalid_argument(std::string(action) + ": " + ernie_cuda_last_error());
    check_cuda(rc, action);
}
} // namespace

Tensor text_embeddings(const std::string &path, const std::vector<uint32_t> &ids, int bucket)
{
    require(bucket >= 1 && bucket <= 2048, "Text bucket must be in [1,2048]");
    require(!ids.empty() && ids.size() <= size_t(bucket), "Invalid token IDs or BF16 embedding table size");
    Tensor out(3072, bucket);
    check_request(ernie_cuda_text_embeddings(path.c_str(), ids.data(), static_cast<int>(ids.size()), bucket, out.ptr()),
                  "text embeddings");
    return out;
}

std::vector<Tensor> text_constants(const std::vector<float> &inverse_frequencies, int bucket)
{
    require(inverse_frequencies.size() == 64, "Invalid YaRN frequency table size");
    require(bucket >= 1 && bucket <= 2048, "Text bucket must be in [1,2048]");
    Tensor cos(128, bucket), sin(128, bucket), mask(bucket, bucket);
    check_request(ernie_cuda_text_constants(inverse_frequencies.data(), bucket, cos.ptr(), sin.ptr(), mask.ptr()),
                  "text constants");
    return {cos, sin, mask};
}

std::vector<Tensor> text_constants(const std::string &inverse_frequency_path, int bucket)
{
    std::ifstream file(inverse_frequency_path, std::ios::binary);
    file.seekg(0, std::ios::end);
    require(file && file.tellg() == std::streampos(64 * 4), "Invalid YaRN frequency table size");
    std::vector<float> f(64);
    file.seekg(0);
    if (!file.read(reinterpret_cast<char *>(f.data()), 64 * 4)) throw std::runtime_error("Cannot read YaRN frequencies");
    return text_constants(f, bucket);
}

TextModel::TextModel(GpuContext &ctx, int num_layers) : ctx_(ctx), num_layers_(num_layers)
{
    require(ctx.available(), "Text encoder needs a CUDA device");
    check_request(ernie_cuda_text_model_create(ctx.handle(), num_layers, &handle_), "create text encoder");
}

TextModel::~TextModel()
{
    if (handle_) ernie_cuda_text_model_destroy(handle_);
}

void TextModel::synthesize(uint64_t seed)
{
    check_cuda(ernie_cuda_text_model_synthesize(handle_, seed), "synthesize text encoder");
}

void TextModel::load_safetensors(const std::vector<std::string> &files)
{
    const auto paths = c_paths(files);
    check_request(ernie_cuda_text_model_load_safetensors(handle_, num_layers_, paths.data(), static_cast<int>(paths.size())),
                  "load text encoder checkpoint");
}

Tensor run_text_blocks(TextModel &model, const Tensor &input, const std::vector<Tensor> &constants, Precision precision,
                       BlockSequenceStats &stats, int layers)
{
    require(constants.size() == 3, "Text path requires 1..25 blocks and cos/sin/causal mask");
    const int bucket = input.h;
    require(input.dims == 2 && input.w == 3072 && bucket >= 1 && bucket <= 2048, "Expected a [bucket][3072] FP32 prompt");
    require(constants[0].w == 128 && constants[0].h == bucket && constants[1].w == 128 && constants[1].h == bucket,
            "Text constants have wrong layout");
    const Tensor &mask = constants[2];
    require(mask.w == bucket && mask.h == bucket, "Text constants have wrong layout");
    for (int t = 0; t < bucket; ++t)
        for (int k = 0; k < bucket; ++k)
        {
            const float m = mask[size_t(t) * bucket + k];
            require(k > t ? m <= -1e30f : m == 0.f, "Only the causal text mask is supported");
        }
    stats = {};
    stats.peak_loaded_nets = 1;
    const auto begin = Clock::now();
    Tensor out(3072, bucket);
    check_request(ernie_cuda_text_run_blocks(model.handle(), input.ptr(), bucket, constants[0].ptr(), constants[1].ptr(),
                                             precision_code(precision), layers > 0 ? layers : model.num_layers(), out.ptr()),
                  "text blocks");
    stats.compute_seconds.push_back(seconds_since(begin));
    stats.compute_submissions = 1;
    return out;
}

void load_safetensors(DitModel &model, const std::vector<std::string> &files, bool heads)
{
    const auto paths = c_paths(files);
    check_request(ernie_cuda_model_load_safetensors(model.handle(), model.num_blocks(), paths.data(),
                                                    static_cast<int>(paths.size()), heads ? 1 : 0),
                  "load DiT checkpoint");
}

void load_safetensors(VaeDecoder &vae, const std::vector<std::string> &files)
{
    const auto paths = c_paths(files);
    check_request(ernie_cuda_vae_load_safetensors(vae.handle(), paths.data(), static_cast<int>(paths.size())),
                  "load VAE checkpoint");
}

void load_safetensors(VaeEncoder &encoder, const std::vector<std::string> &files)
{
    const auto paths = c_paths(files);
    check_request(
        ernie_cuda_vae_encoder_load_safetensors(encoder.handle(), paths.data(), static_cast<int>(paths.size())),
        "load VAE encoder checkpoint");
}

GeneratedImage generate_from_ids(GenerationModels &m, const std::vector<uint32_t> &ids, int text_bucket,
                                 const DitStageRequest &request,
                                 const std::function<void(const DitStageProgress &)> &notify)
{
    const auto start = Clock::now();
    require(m.dit_text_tokens >= int(ids.size()), "Prompt longer than the DiT text slots");
    GeneratedImage out;
    const Tensor embedded = text_embeddings(m.embeddings, ids, text_bucket);
    BlockSequenceStats stats;
    const Tensor encoded =
        run_text_blocks(m.text, embedded, text_constants(m.text_frequencies, text_bucket), request.precision, stats);
    out.text = Tensor(3072, int(ids.size()));
    std::copy(encoded.data.begin(), encoded.data.begin() + long(ids.size()) * 3072, out.text.data.begin());
    out.text_seconds = seconds_since(start);
    if (notify) notify({"text", int(ids.size()), text_bucket, out.text_seconds});
    if (!request.trace.empty()) write_tensor((std::filesystem::path(request.trace) / "text.f32").string(), out.text);
    const auto dit_start = Clock::now();
    DitStageResult dit = run_dit_stage(m.dit, out.text, m.dit_text_tokens, m.dit_frequencies, request, notify);
    out.dit_seconds = seconds_since(dit_start);
    out.start_step = dit.start_step;
    out.latent = std::move(dit.latent);
    VaeStageResult vae = run_vae_stage(m.vae, out.latent, m.bn_mean, m.bn_variance, request.precision, request.trace);
    out.vae_seconds = vae.seconds;
    out.decoded = std::move(vae.decoded);
    out.image = std::move(vae.image);
    out.elapsed_seconds = seconds_since(start);
    return out;
}
GeneratedImage generate_img2img_from_ids(GenerationModels &m, const std::vector<uint32_t> &ids, int text_bucket,
                                         const RgbImage &input, const DitStageRequest &request,
                                         const std::function<void(const DitStageProgress &)> &notify)
{
    const auto start = Clock::now();
    if (!m.encoder) throw std::invalid_argument("Selected model package has no img2img encoder");
    if (!std::isfinite(request.strength) || request.strength < 0.f || request.strength > 1.f)
        throw std::invalid_argument("img2img strength must be in [0,1]");
    if (input.width != request.width || input.height != request.height)
        throw std::invalid_argument("Invalid img2img resize identity");
    const VaeEncoding encoding = encode_vae(*m.encoder, input, request.precision);
    const double encoder_seconds = seconds_since(start);
    if (!request.trace.empty())
    {
        const std::filesystem::path folder(request.trace);
        const auto rgb_path = folder / "input.rgb";
        if (std::filesystem::exists(rgb_path)) throw std::runtime_error("Trace file exists");
        std::ofstream rgb(rgb_path, std::ios::binary);
        if (!rgb.write(reinterpret_cast<const char *>(input.pixels.data()), std::streamsize(input.pixels.size())))
            throw std::runtime_error("Cannot write img2img input trace");
        const auto text_path = folder / "img2img.txt";
        if (std::filesystem::exists(text_path)) throw std::runtime_error("Trace file exists");
        std::ofstream text(text_path);
        text << "source_width=" << input.width << "\nsource_height=" << input.height << "\nwidth=" << input.width
             << "\nheight=" << input.height << "\nstrength=" << std::to_string(request.strength) << "\n";
        if (!text) throw std::runtime_error("Cannot write img2img input trace");
        write_tensor((folder / "encoder-mean.f32").string(), encoding.mean);
        write_tensor((folder / "encoder-packed.f32").string(), encoding.packed);
        write_tensor((folder / "encoder-normalized.f32").string(), encoding.normalized);
    }
    if (request.strength == 0.f)
    {
        // strength 0: the encoded image decoded straight back (src/pipeline.cpp:419-436)
        GeneratedImage out;
        VaeStageResult vae =
            run_vae_stage(m.vae, encoding.normalized, m.bn_mean, m.bn_variance, request.precision, request.trace);
        out.latent = encoding.normalized;
        out.start_step = request.steps; // no step runs
        out.decoded = std::move(vae.decoded);
        out.image = std::move(vae.image);
        out.vae_seconds = encoder_seconds + vae.seconds;
        out.elapsed_seconds = seconds_since(start);
        return out;
    }
    DitStageRequest r = request;
    r.encoded = encoding.normalized;
    GeneratedImage out = generate_from_ids(m, ids, text_bucket, r, notify);
    out.elapsed_seconds = seconds_since(start);
    return out;
}
// ---- the optional prompt enhancer --------------------------------------------------------------------
namespace
{
void pe_options_check(const PeOptions &o)
{
    if (o.max_tokens < 1 || o.max_tokens > 2048 || !std::isfinite(o.temperature) || o.temperature <= 0 ||
        !std::isfinite(o.top_p) || o.top_p <= 0 || o.top_p > 1)
        throw std::invalid_argument("PE requires max tokens 1..2048, positive temperature and top-p in (0,1]");
}
} // namespace

void TextModel::load_pe_safetensors(const std::vector<std::string> &files)
{
    const auto paths = c_paths(files);
    check_request(ernie_cuda_pe_model_load_safetensors(handle_, num_layers_, paths.data(), static_cast<int>(paths.size())),
                  "load PE checkpoint");
}

void TextModel::synthesize_head(uint64_t seed)
{
    check_cuda(ernie_cuda_text_model_synthesize_head(handle_, seed), "synthesize PE head");
}

uint32_t sample_pe_token(const std::vector<float> &logits, const PeOptions &options, std::mt19937 &random)
{
    pe_options_check(options);
    if (logits.empty()) throw std::invalid_argument("PE logits must be an FP32 vector");
    if (!std::all_of(logits.begin(), logits.end(), [](float v) { return std::isfinite(v); }))
        throw std::runtime_error("Non-finite PE logits");
    const auto top = std::max_element(logits.begin(), logits.end()); // the first of equal maxima
    if (options.greedy) return uint32_t(top - logits.begin());
    // Tokens by descending logit, equal logits in ascending token order.
    std::vector<uint32_t> ranked(logits.size());
    std::iota(ranked.begin(), ranked.end(), 0u);
    std::sort(ranked.begin(), ranked.end(), [&](uint32_t a, uint32_t b) {
        return logits[a] != logits[b] ? logits[a] > logits[b] : a < b;
    });
    // Relative probabilities exp((logit - max) / temperature) in double, summed in ranked order.
    std::vector<double> weight(ranked.size());
    double total = 0;
    for (size_t i = 0; i < ranked.size(); ++i)
        total += weight[i] = std::exp((double(logits[ranked[i]]) - double(*top)) / double(options.temperature));
    // Nucleus: the shortest ranked prefix holding top_p of the total weight, never empty.
    const double nucleus = double(options.top_p) * total;
    size_t kept = 0;
    double mass = 0;
    while (kept < weight.size())
    {
        mass += weight[kept++];
        if (mass >= nucleus) break;
    }
    std::discrete_distribution<size_t> draw(weight.begin(), weight.begin() + std::ptrdiff_t(kept));
    return ranked[draw(random)];
}

PeSession::PeSession(TextModel &model, int capacity, Precision precision) : ctx_(model.context())
{
    if (capacity < 1 || capacity > 4096) throw std::invalid_argument("PE requires 1..26 blocks and capacity 1..4096");
    check_request(ernie_cuda_pe_session_create(model.handle(), capacity, precision_code(precision), &handle_),
                  "create PE session");
}

PeSession::~PeSession()
{
    if (handle_) ernie_cuda_pe_session_destroy(handle_);
}

void PeSession::reset() { check_cuda(ernie_cuda_pe_session_reset(handle_), "reset PE session"); }

int PeSession::position() const
{
    int p = 0;
    check_cuda(ernie_cuda_pe_session_position(handle_, &p), "PE position");
    return p;
}

Tensor PeSession::append(const Tensor &embedded, const Tensor &cos, const Tensor &sin, bool single)
{
    const int rows = embedded.h;
    if (embedded.dims != 2 || embedded.w != 3072 || cos.dims != 2 || sin.dims != 2 || cos.w != 128 || sin.w != 128 ||
        cos.h != rows || sin.h != rows)
        throw std::invalid_argument("PE requires pack1 FP32 matrices with matching token rows");
    if (rows < 1 || rows > (single ? 1 : 32)) throw std::invalid_argument("PE token count or session capacity exceeded");
    Tensor hidden(3072, rows);
    check_request(ernie_cuda_pe_session_append(handle_, embedded.ptr(), cos.ptr(), sin.ptr(), rows, hidden.ptr()),
                  "PE step");
    return hidden;
}

Tensor PeSession::step(const Tensor &embedded, const Tensor &cos, const Tensor &sin)
{
    return append(embedded, cos, sin, true);
}

Tensor PeSession::append_chunk(const Tensor &embedded, const Tensor &cos, const Tensor &sin)
{
    return append(embedded, cos, sin, false);
}

std::vector<float> PeSession::logits(const float *hidden_row)
{
    std::vector<float> out(131072);
    check_request(ernie_cuda_pe_logits(handle_, hidden_row, out.data()), "PE logits");
    return out;
}

PeResult enhance_prompt_from_ids(TextModel &model, const std::string &embeddings, const std::vector<float> &frequencies,
                                 const std::vector<uint32_t> &input_ids, const PeOptions &options, Precision precision,
                                 int prefill_chunk, const PeProgress &progress, const PeLogits &observe)
{
    pe_options_check(options);
    if (prefill_chunk < 1 || prefill_chunk > 32) throw std::invalid_argument("PE prefill chunk must be in [1,32]");
    if (input_ids.empty() || input_ids.size() > 2048) throw std::invalid_argument("PE chat input exceeds 2048 tokens");
    if (frequencies.size() != 64) throw std::runtime_error("Invalid PE YaRN table");
    for (float f : frequencies)
        if (!std::isfinite(f) || f <= 0) throw std::runtime_error("Invalid PE frequency");
    PeResult result;
    result.input_ids = input_ids;
    PeSession session(model, int(input_ids.size()) + options.max_tokens, precision);
    // rotary rows of `count` tokens from the session's position: phase = float(position) * f in FP32
    auto rotary = [&](int count, Tensor &cos, Tensor &sin) {
        cos = Tensor(128, count);
        sin = Tensor(128, count);
        for (int r = 0; r < count; ++r)
            for (int i = 0; i < 64; ++i)
            {
                const float phase = float(session.position() + r) * frequencies[size_t(i)];
                cos[size_t(r) * 128 + size_t(i)] = cos[size_t(r) * 128 + size_t(i) + 64] = std::cos(phase);
                sin[size_t(r) * 128 + size_t(i)] = sin[size_t(r) * 128 + size_t(i) + 64] = std::sin(phase);
            }
    };
    auto advance = [&](const std::vector<uint32_t> &ids) {
        const Tensor embedded = text_embeddings(embeddings, ids, int(ids.size()));
        Tensor cos, sin;
        rotary(int(ids.size()), cos, sin);
        return ids.size() == 1 ? session.step(embedded, cos, sin) : session.append_chunk(embedded, cos, sin);
    };
    Tensor hidden;
    for (size_t first = 0; first < input_ids.size();)
    {
        const size_t count = std::min(size_t(prefill_chunk), input_ids.size() - first);
        hidden = advance(std::vector<uint32_t>(input_ids.begin() + long(first), input_ids.begin() + long(first + count)));
        first += count;
        if (progress && (prefill_chunk > 1 || first % 8 == 0 || first == input_ids.size()))
            progress("prefill", int(first), int(input_ids.size()));
    }
    std::mt19937 random(options.seed);
    for (int i = 0; i < options.max_tokens; ++i)
    {
        const std::vector<float> logits = session.logits(hidden.ptr() + size_t(hidden.h - 1) * 3072);
        if (observe) observe(i, logits);
        const uint32_t token = sample_pe_token(logits, options, random);
        result.generated_ids.push_back(token);
        if (progress && ((i + 1) % 8 == 0 || token == 2 || i + 1 == options.max_tokens))
            progress("decode", i + 1, options.max_tokens);
        if (token == 2)
        {
            result.eos = true;
            break;
        }
        if (i + 1 < options.max_tokens) hidden = advance({token});
    }
    return result;
}
} // namespace ernie
