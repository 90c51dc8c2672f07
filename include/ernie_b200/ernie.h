// C++ host surface of the B200 DiT denoiser, mirroring mingshi2333/ernie-image-ncnn-vulkan's denoiser,
// DiT, block-sequence, latent-op, conditioning, layer, weight-placement/-session, GPU-context and
// recovery interfaces (each declaration names the reference header it mirrors). ncnn::Mat / VkMat
// arguments become ernie::Tensor (host FP32) and ernie::DeviceTensor (CUDA memory). Everything here
// calls the C ABI of include/ernie_cuda.h; failures throw the reference's exception types
// (GpuAllocationError for allocation failures, std::invalid_argument for contract violations,
// std::runtime_error otherwise).
#pragma once
#include "ernie_cuda.h"
#include <cstdint>
#include <functional>
#include <map>
#include <memory>
#include <optional>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

namespace ernie
{
// ---- errors (src/vulkan_memory.h:11-17, check_ncnn_memory src/vulkan_memory.cpp:21-30) --------
class GpuAllocationError : public std::runtime_error
{
  public:
    using std::runtime_error::runtime_error;
};
// 0 -> return, -100 -> GpuAllocationError, anything else -> std::runtime_error("<action>: <message>").
void check_cuda(int result, const char *action);

// ---- tensors ------------------------------------------------------------------------------------
// Host FP32 tensor with ncnn's (w, h, c) naming: dims 1 = [w], 2 = [h][w], 3 = [c][h][w].
struct Tensor
{
    int w = 0, h = 1, c = 1, dims = 0;
    std::vector<float> data;
    Tensor() = default;
    explicit Tensor(int w_) : w(w_), dims(1), data(size_t(w_)) {}
    Tensor(int w_, int h_) : w(w_), h(h_), dims(2), data(size_t(w_) * h_) {}
    Tensor(int w_, int h_, int c_) : w(w_), h(h_), c(c_), dims(3), data(size_t(w_) * h_ * c_) {}
    bool empty() const { return data.empty(); }
    size_t total() const { return data.size(); }
    float *ptr() { return data.data(); }
    const float *ptr() const { return data.data(); }
    float &operator[](size_t i) { return data[i]; }
    float operator[](size_t i) const { return data[i]; }
};

class GpuContext;

// Device allocation owned by the caller (freed on destruction), shape in ncnn naming.
class DeviceTensor
{
  public:
    DeviceTensor() = default;
    DeviceTensor(GpuContext &ctx, size_t bytes, int w, int h = 1, int c = 1, int dims = 1);
    DeviceTensor(DeviceTensor &&) noexcept;
    DeviceTensor &operator=(DeviceTensor &&) noexcept;
    DeviceTensor(const DeviceTensor &) = delete;
    DeviceTensor &operator=(const DeviceTensor &) = delete;
    ~DeviceTensor();
    static DeviceTensor upload(GpuContext &ctx, const Tensor &host);
    Tensor download() const; // FP32 tensors only
    void *data() const { return ptr_; }
    float *f32() const { return static_cast<float *>(ptr_); }
    size_t bytes() const { return bytes_; }
    bool empty() const { return ptr_ == nullptr; }
    int w = 0, h = 1, c = 1, dims = 0;

  private:
    GpuContext *ctx_ = nullptr;
    void *ptr_ = nullptr;
    size_t bytes_ = 0;
};

// ---- GPU context (src/gpu_context.h:12-27) -------------------------------------------------------
// One CUDA device + stream. With enabled=false or no device (and require_device=false), available()
// is false and initialization_error() says why; nothing falls back to the CPU.
class GpuContext
{
  public:
    explicit GpuContext(bool enabled, int requested_index = -1, bool require_device = true);
    ~GpuContext();
    GpuContext(const GpuContext &) = delete;
    GpuContext &operator=(const GpuContext &) = delete;
    bool available() const noexcept { return handle_ != nullptr; }
    const std::string &initialization_error() const noexcept { return initialization_error_; }
    ernie_cuda_context *handle() const;
    int device() const noexcept { return device_; }
    void synchronize() const;

  private:
    ernie_cuda_context *handle_ = nullptr;
    int device_ = -1;
    std::string initialization_error_;
};

// ---- latent ops (src/latent_ops.h:15-57) ---------------------------------------------------------
struct FlowSchedule
{
    std::vector<float> sigmas;    // steps + 1, last 0
    std::vector<float> timesteps; // 1000 * sigma
    static FlowSchedule turbo(int steps = 8);
    static FlowSchedule linear(int steps = 8);
    float delta(size_t step) const; // sigma[step+1] - sigma[step]; std::out_of_range past the end
};
// Device latents [128][h][w]. Shapes and delta are validated as in src/latent_ops.cpp:11-29.
void euler_step(GpuContext &, const DeviceTensor &sample, const DeviceTensor &prediction, float delta,
                DeviceTensor &next);
bool finite_latent(GpuContext &, const DeviceTensor &value);
DeviceTensor unpack_for_vae(GpuContext &, const DeviceTensor &packed, const Tensor &mean, const Tensor &variance);

// ---- conditioning (src/conditioning.h:12-15) and features (src/denoiser.h:12) --------------------
// Returns {cosine [N][128], sine [N][128], mask [N]}; frequency table (64 values) or empty for the
// official table. token_limit 6144 (static graphs) or 10240 (runtime).
std::vector<Tensor> dit_constants(const std::vector<float> &frequencies, int width, int height, int valid_text,
                                  int text_bucket, int token_limit = 10240);
Tensor pad_text(const Tensor &embeddings /*[T][3072]*/, int bucket);
Tensor timestep_features(float timestep);

// ---- ERNIE layer contracts (register_layers, src/ernie_gelu.cpp:108-116) --------------------------
void set_attention_query_rows(GpuContext &, int rows); // 128, 64, 32 or 16, else std::invalid_argument
int attention_query_rows(GpuContext &);
// ErnieSDPA: q [heads][nq][w], k/v [kv_heads][nk][w], optional mask [mask_heads][rows][nk] (rows 1 or nq).
DeviceTensor sdpa(GpuContext &, const DeviceTensor &q, const DeviceTensor &k, const DeviceTensor &v,
                  const DeviceTensor *mask);
DeviceTensor rms_norm(GpuContext &, const DeviceTensor &x, const Tensor &gamma, float eps = 1e-6f); // w 128/3072/4096
DeviceTensor layer_norm(GpuContext &, const DeviceTensor &x, float eps = 1e-6f);                     // w 4096
void gelu_inplace(GpuContext &, DeviceTensor &x);                                                   // total % 4
DeviceTensor residual_add(GpuContext &, const DeviceTensor &a, const DeviceTensor &b);

// ---- weights --------------------------------------------------------------------------------------
// Host copy of one block's BF16 weights (tools/build_dit_weights.py:19-31 bindings).
struct BlockWeights
{
    std::vector<uint16_t> wq, wk, wv, wo, wup, wgate, wfc2;
    std::vector<float> gamma_sa, gamma_mlp, gamma_q, gamma_k;
};
struct HeadWeights
{
    std::vector<uint16_t> x_embed_w, text_proj_w, time1_w, time2_w, adaln_w, final_norm_w, final_w;
    std::vector<float> x_embed_b, time1_b, time2_b, adaln_b, final_norm_b, final_b;
};
// Device-resident DiT weights (all blocks stay in HBM: 15.7 GB for 36 blocks in BF16).
class DitModel
{
  public:
    DitModel(GpuContext &ctx, int num_blocks);
    ~DitModel();
    DitModel(const DitModel &) = delete;
    DitModel &operator=(const DitModel &) = delete;
    void upload_block(int block, const BlockWeights &);
    void upload_heads(const HeadWeights &);
    void synthesize(uint64_t seed); // seeded random init (include/ernie_synth.h)
    int num_blocks() const noexcept { return num_blocks_; }
    uint64_t bytes() const;
    ernie_cuda_model *handle() const noexcept { return handle_; }
    GpuContext &context() const noexcept { return ctx_; }

  private:
    GpuContext &ctx_;
    ernie_cuda_model *handle_ = nullptr;
    int num_blocks_ = 0;
};

// WeightPlacement (src/weight_placement.h:20-51): the decision logic of the reference, with the
// CUDA device budget (cudaMemGetInfo) as the reader.
enum class WeightMemory { Auto, Device, Host };
WeightMemory parse_weight_memory(const std::string &value);
struct DeviceMemoryBudget
{
    std::uint64_t budget_bytes = 0, usage_bytes = 0;
};
struct WeightPlacementDecision
{
    bool host = false;
    const char *reason = "unavailable";
    std::optional<std::uint64_t> available_bytes;
    std::uint64_t weight_bytes = 0, reserve_bytes = 0;
};
WeightPlacementDecision choose_weight_placement(WeightMemory mode, bool shape_prefers_host, std::uint64_t weight_bytes,
                                                std::uint64_t reserve_bytes, std::optional<DeviceMemoryBudget> memory);
class WeightPlacement
{
  public:
    using BudgetReader = std::function<std::optional<DeviceMemoryBudget>()>;
    using Observer = std::function<void(const std::string &component, const WeightPlacementDecision &)>;
    WeightPlacement(WeightMemory mode, std::uint64_t reserve_bytes, BudgetReader reader = {}, Observer observer = {});
    // weight_bytes = the component's payload estimate (the reference uses 2x the file size)
    bool use_host(const std::string &component, std::uint64_t weight_bytes, bool shape_prefers_host,
                  bool cache_prefers_host = false, const char *host_reason = "cache");
    std::uint64_t host_requests() const { return host_requests_; }
    std::uint64_t device_requests() const { return device_requests_; }
    std::uint64_t unavailable_queries() const { return unavailable_queries_; }

  private:
    WeightMemory mode_;
    std::uint64_t reserve_bytes_, host_requests_ = 0, device_requests_ = 0, unavailable_queries_ = 0;
    BudgetReader reader_;
    Observer observer_;
};
WeightPlacement::BudgetReader cuda_memory_budget_reader(GpuContext &);

// WeightSession (src/weight_session.h:29-73): request-local cache of prepared per-block payloads with
// one lease at a time. Admitted entries stay while the rest stream (LRU would miss every block of a
// repeated 36-block scan). The payload type is opaque here.
struct WeightBudget
{
    std::uint64_t host_bytes = 0;
    std::uint64_t reserve_bytes = 3ull * 1024 * 1024 * 1024;
};
struct WeightSessionStats
{
    std::uint64_t hits = 0, loads = 0, admissions = 0, evictions = 0;
    std::uint64_t live_bytes = 0, peak_bytes = 0, cached_nets = 0, peak_nets = 0;
    std::uint64_t unavailable_queries = 0;
};
class WeightSession
{
    struct State;

  public:
    using Payload = std::shared_ptr<void>;
    using AvailableReader = std::function<std::optional<std::uint64_t>()>;
    using Inspector = std::function<std::optional<std::uint64_t>(const Payload &)>;
    using Loader = std::function<Payload(bool prefer_cache)>;
    class Lease
    {
      public:
        Lease() = default;
        Lease(const Lease &) = delete;
        Lease &operator=(const Lease &) = delete;
        Lease(Lease &&) noexcept;
        Lease &operator=(Lease &&) noexcept;
        ~Lease();
        const Payload &payload() const;
        bool cached() const { return charge_ != 0; }
        void complete(); // only after all work using the payload has completed
      private:
        friend class WeightSession;
        Lease(std::shared_ptr<State>, std::size_t, Payload, std::uint64_t);
        void release(bool completed);
        std::shared_ptr<State> state_;
        std::size_t block_ = 0;
        Payload payload_;
        std::uint64_t charge_ = 0;
    };
    WeightSession(WeightBudget, AvailableReader, Inspector);
    ~WeightSession();
    WeightSession(const WeightSession &) = delete;
    WeightSession &operator=(const WeightSession &) = delete;
    Lease acquire(std::size_t block, const std::string &identity, const void *request_identity,
                  std::uint64_t estimated_bytes, const Loader &);
    void cancel();
    WeightSessionStats stats() const;
    bool contains(std::size_t block) const;

  private:
    std::shared_ptr<State> state_;
};

// ---- block sequence / DiT / denoise ---------------------------------------------------------------
enum class Precision { BF16, FP32 };
struct BlockSequenceStats // src/block_sequence.h:20-32
{
    std::vector<double> load_seconds, compute_seconds;
    int peak_loaded_nets = 0, compute_submissions = 0;
};
struct DitStats // src/dit.h:6-14
{
    BlockSequenceStats blocks;
    double input_head_seconds = 0, output_head_seconds = 0;
};
using CudaStageObserver = std::function<void(const std::string &, const DeviceTensor &)>;

// A request: shape, precision and the four constants (text, cos, sin, mask) on the device.
class DenoiseSession
{
  public:
    DenoiseSession(DitModel &model, int width, int height, int text_tokens, int valid_text, Precision precision);
    ~DenoiseSession();
    DenoiseSession(const DenoiseSession &) = delete;
    DenoiseSession &operator=(const DenoiseSession &) = delete;
    // constants: text [T][3072] (may be empty), cos [N][128], sin [N][128], mask [N]
    void set_constants(const std::vector<Tensor> &constants);
    int tokens() const noexcept { return tokens_; }
    int width() const noexcept { return width_; }
    int height() const noexcept { return height_; }
    ernie_cuda_session *handle() const noexcept { return handle_; }
    DitModel &model() const noexcept { return model_; }

  private:
    DitModel &model_;
    ernie_cuda_session *handle_ = nullptr;
    int width_, height_, tokens_;
};

// run_block_sequence (src/block_sequence.h:38-60): blocks [first, first+count) on x [N][4096] (device,
// in place) with the shared modulation [6][4096] (device). 1..36 blocks.
void run_block_sequence(DenoiseSession &, DeviceTensor &x, const DeviceTensor &modulation, int first, int count,
                        BlockSequenceStats &stats);
// run_dit (src/dit.h:17-40): one prediction [128][h][w] for latent [128][h][w] at `timestep`.
DeviceTensor run_dit(DenoiseSession &, const DeviceTensor &latent, float timestep, DitStats &stats);

struct DenoiseStepStats // src/denoiser.h:18-24
{
    float timestep = 0, delta = 0;
    DitStats dit;
    double elapsed_seconds = 0;
    bool complete = false;
};
using StepObserver = std::function<void(size_t, const Tensor &prediction, const Tensor &latent)>;
// denoise (src/denoiser.h:30-44): steps [start_step, steps) of the turbo schedule; the observer
// (optional) sees each step's prediction and latent (forcing one step per launch). Throws
// std::invalid_argument on contract errors and std::runtime_error("Non-finite latent after denoise
// step k"); stats holds the executed steps, a failed one with complete = false.
Tensor denoise(DenoiseSession &, const Tensor &initial, int steps, std::vector<DenoiseStepStats> &stats,
               const StepObserver &observer = {}, int start_step = 0, int schedule = ERNIE_SCHEDULE_TURBO);

// ---- recovery (src/vulkan_denoise.h:8-47) ---------------------------------------------------------
// One attempt runs steps on some backend; on GpuAllocationError (or std::bad_alloc) the wrapper
// retries from the last host checkpoint with the same absolute schedule, at most `retries` times,
// halving the recorded attention query rows (128 >> attempt). Any other failure propagates.
class DenoiseBackend
{
  public:
    virtual ~DenoiseBackend() = default;
    // Prepare an attempt from the checkpoint (may throw GpuAllocationError).
    virtual void begin_attempt(unsigned attempt, const Tensor &checkpoint, int query_rows) = 0;
    // Run absolute step i of the schedule; returns the prediction, updates the backend's latent.
    virtual Tensor run_step(int step, float timestep, float delta) = 0;
    virtual Tensor latent() = 0;     // download the current latent (the checkpoint source)
    virtual void end_attempt() = 0;  // release the attempt's resources (also after a failure)
};
struct CudaDenoiseSettings
{
    unsigned retries = 3;
    int schedule = ERNIE_SCHEDULE_TURBO;
    std::function<void(unsigned attempt, int step)> before_step; // test seam, invoked before each step
};
struct CudaDenoiseStats
{
    unsigned retries = 0;
    int query_rows = 128;
};
struct CudaDenoiseObservers
{
    std::function<void(size_t, const Tensor &prediction, const Tensor &latent, const DenoiseStepStats &)> step;
    std::function<void(unsigned attempt, int step, int rows, const std::string &)> retry;
};
Tensor denoise_with_recovery(DenoiseBackend &, const Tensor &initial, int steps, int start_step,
                             const CudaDenoiseSettings &, CudaDenoiseStats &, const CudaDenoiseObservers & = {});
// The B200 backend: a DenoiseSession per attempt on one model.
class CudaDenoiseBackend : public DenoiseBackend
{
  public:
    CudaDenoiseBackend(DitModel &model, int width, int height, int text_tokens, int valid_text, Precision,
                       std::vector<Tensor> constants);
    void begin_attempt(unsigned attempt, const Tensor &checkpoint, int query_rows) override;
    Tensor run_step(int step, float timestep, float delta) override;
    Tensor latent() override;
    void end_attempt() override;
    int steps = 8; // schedule length the steps belong to

  private:
    DitModel &model_;
    int width_, height_, text_, valid_;
    Precision precision_;
    std::vector<Tensor> constants_;
    std::unique_ptr<DenoiseSession> session_;
};

// ---- the pipeline's DiT stage (src/pipeline.cpp:164-300 and :513-531, src/tensor_io.h:8-10) -------
// Raw little-endian FP32 files, channel after channel. read_tensor checks the byte size and that every
// value is finite; write_tensor refuses to overwrite ("Trace file exists").
Tensor read_tensor(const std::string &path, int w, int h = 1, int c = 1);
void write_tensor(const std::string &path, const Tensor &value);
std::string numbered(const std::string &stem, int index); // "block-07"
// Initial noise of a request without a latent file: std::mt19937(seed) feeding
// std::normal_distribution<float>(0, 1), channel after channel, as src/pipeline.cpp:520-531 draws it.
Tensor initial_noise(int width, int height, uint32_t seed);
// img2img start (src/img2img.h:7-19): the latent and step to begin denoising an encoded image from.
// `encoded` is the patchified, BN-normalised mean posterior [128][h][w]; strength 0 returns it unchanged
// (start_step = schedule length) without using the noise; otherwise denoise_steps = clamp(round-half-up
// (steps * strength), 1, steps), start_step = steps - denoise_steps and the latent is
// sigma * noise + (1 - sigma) * encoded at sigma = sigmas[start_step] (the noise itself when sigma is 1).
// std::invalid_argument for strength outside [0,1], threads outside [1,256], a malformed schedule, or a
// non-finite / mismatched encoded latent or noise.
struct Img2ImgStart
{
    Tensor latent; // independent storage, never aliases the inputs
    int start_step = 0;
    int denoise_steps = 0;
    float sigma = 0.f;
};
Img2ImgStart make_img2img_start(const Tensor &encoded, const Tensor &saved_noise, const FlowSchedule &schedule,
                                float strength, int threads = 4);

struct DitStageRequest // the GenerationRequest fields the DiT stage reads (include/ernie/pipeline.h)
{
    int width = 1024, height = 1024; // pixels, multiples of 16 (the packed latent is width/16 x height/16)
    int steps = 8;
    uint32_t seed = 0;
    std::string latent;              // optional initial latent file [128][height/16][width/16]
    std::string trace;               // optional existing folder: prediction-i.f32 and step-i.f32 per step
    Precision precision = Precision::BF16;
    unsigned oom_retries = 3;
    Tensor encoded;                  // img2img: the encoded image latent [128][h][w] (empty: text to image)
    float strength = 1.f;            // img2img strength
};
struct DitStageProgress // the "denoise" / "memory-recovery" notifications of src/pipeline.cpp:180-186, 259
{
    std::string stage;
    int step = 0, total = 0;
    double seconds = 0;
};
struct DitStageResult
{
    Tensor latent;                        // [128][h][w] after the last step
    std::vector<DenoiseStepStats> steps;  // executed steps
    CudaDenoiseStats recovery;
    int start_step = 0;                   // first executed step (img2img)
};
// text: the encoder's [T][3072] rows for the T prompt tokens, padded to `text_bucket` slots; frequencies:
// the 64 RoPE inverse frequencies (empty = the built-in table). Without a trace the whole schedule runs
// as one CUDA graph, and an allocation failure falls back to denoise_with_recovery from the initial
// latent; with a trace every step goes through denoise_with_recovery and its tensors are written.
DitStageResult run_dit_stage(DitModel &model, const Tensor &text, int text_bucket, const std::vector<float> &frequencies,
                             const DitStageRequest &request,
                             const std::function<void(const DitStageProgress &)> &notify = {});

// ---- the pipeline's VAE stage (src/vae.h:8-22, src/pipeline.cpp:145-163 and :554-575) -------------
struct RgbImage // interleaved RGB bytes, row after row (include/ernie/pipeline.h)
{
    int width = 0, height = 0;
    std::vector<uint8_t> pixels;
};
// rgb_image (src/pipeline.cpp:145-163): decoded [3][H][W] FP32 -> bytes nearbyint(clamp(x / 2 + 0.5, 0, 1) *
// 255) in FP32; std::runtime_error for a tensor that is not [3][H][W] or holds a non-finite value.
RgbImage rgb_image(const Tensor &decoded);
struct VaeStats // src/vae.h:9-13
{
    struct Detail
    {
        std::string boundary, status;
        double seconds = 0;
    };
    std::vector<Detail> details;
};
// decode_vae on the B200: the AutoencoderKLFlux2 post_quant_conv + decoder the reference exports
// (tools/export_vae.py), weights resident on the device and addressed by their diffusers names (FP32).
class VaeDecoder
{
  public:
    explicit VaeDecoder(GpuContext &ctx);
    ~VaeDecoder();
    VaeDecoder(const VaeDecoder &) = delete;
    VaeDecoder &operator=(const VaeDecoder &) = delete;
    // every tensor the decoder holds: diffusers name and shape, in execution order
    static std::vector<std::pair<std::string, std::vector<int>>> tensors();
    void upload(const std::string &name, const Tensor &value);
    void synthesize(uint64_t seed, bool bf16_weights = false); // include/ernie_synth.h, VAE section
    // unpacked [32][h][w] -> decoded [3][8h][8w]; stats gets the "extract_compute_composite" boundary
    Tensor decode(const Tensor &unpacked, Precision precision = Precision::BF16, VaeStats *stats = nullptr);
    // device tensors; `image` (nullable) receives the RGB bytes, and then a non-finite value throws as
    // rgb_image does
    DeviceTensor decode(const DeviceTensor &unpacked, Precision precision, RgbImage *image = nullptr);
    GpuContext &context() const { return ctx_; }
    ernie_cuda_vae *handle() const noexcept { return handle_; }

  private:
    GpuContext &ctx_;
    ernie_cuda_vae *handle_ = nullptr;
};
struct VaeStageResult
{
    Tensor unpacked; // [32][2h][2w]
    Tensor decoded;  // [3][16h][16w]
    RgbImage image;
    double seconds = 0;
};
// The stage after the denoise loop (src/pipeline.cpp:554-575): unpack_for_vae with the package's BN
// statistics, decode_vae and rgb_image. With a trace folder it writes final.f32, unpacked.f32 and
// decoded.f32 (refusing to overwrite, as write_tensor does).
VaeStageResult run_vae_stage(VaeDecoder &vae, const Tensor &latent, const Tensor &mean, const Tensor &variance,
                             Precision precision = Precision::BF16, const std::string &trace = {});

// ---- the VAE encoder (src/image_encoder.h:9-20): img2img's image latent ----------------------------
struct VaeEncoding // src/image_encoder.h:9-14
{
    Tensor mean;       // [32][H/8][W/8]: quant_conv(encoder(x))[:32], the posterior's mode
    Tensor packed;     // [128][H/16][W/16]: pixel_unshuffle(mean, 2)
    Tensor normalized; // [128][H/16][W/16]: BatchNorm(packed), make_img2img_start's `encoded`
};
// The AutoencoderKLFlux2 encoder + quant_conv + bn the reference exports (tools/export_vae_encoder.py),
// weights resident on the device and addressed by their diffusers names (FP32).
class VaeEncoder
{
  public:
    explicit VaeEncoder(GpuContext &ctx);
    ~VaeEncoder();
    VaeEncoder(const VaeEncoder &) = delete;
    VaeEncoder &operator=(const VaeEncoder &) = delete;
    static std::vector<std::pair<std::string, std::vector<int>>> tensors();
    void upload(const std::string &name, const Tensor &value);
    void synthesize(uint64_t seed, bool bf16_weights = false);
    GpuContext &context() const { return ctx_; }
    ernie_cuda_vae_encoder *handle() const noexcept { return handle_; }

  private:
    GpuContext &ctx_;
    ernie_cuda_vae_encoder *handle_ = nullptr;
};
// encode_vae (src/image_encoder.cpp:28-72) on the B200. std::invalid_argument for pixels that are not
// width * height * 3 bytes or sides that are not multiples of 16 in [16, 2048] (the reference admits only
// its reviewed 32x32, 64x32, 512x384 and 1024x1024); std::runtime_error "Non-finite VAE encoder ..." for a
// non-finite output, as validate_output throws. FP32-exact mode is the parity mode of the reference's CPU
// FP32 contract; BF16 mode uses BF16 convolution operands.
VaeEncoding encode_vae(VaeEncoder &encoder, const RgbImage &rgb, Precision precision = Precision::FP32);

// ---- the prompt encoder (src/text_encoder.h:8-26) ------------------------------------------------
// text_embeddings: the rows of ids from the [131072][3072] BF16 table (the reference's raw
// "text/embeddings.bf16" file, or a checkpoint .safetensors with language_model.model.embed_tokens.weight)
// as [bucket][3072] FP32, rows past the prompt zero. std::invalid_argument for a bucket outside [1,2048],
// no ids, more ids than the bucket, an id outside the vocabulary or a table of the wrong size.
Tensor text_embeddings(const std::string &path, const std::vector<uint32_t> &ids, int bucket);
// text_constants: {cos, sin, causal mask} for a bucket from the 64 YaRN inverse frequencies (the values, or
// the reference's 256-byte "text/rope-inv-freq.f32" file).
std::vector<Tensor> text_constants(const std::vector<float> &inverse_frequencies, int bucket);
std::vector<Tensor> text_constants(const std::string &inverse_frequency_path, int bucket);
// The Mistral decoder layers of the prompt encoder, resident on the device.
class TextModel
{
  public:
    TextModel(GpuContext &ctx, int num_layers = 25);
    ~TextModel();
    TextModel(const TextModel &) = delete;
    TextModel &operator=(const TextModel &) = delete;
    void synthesize(uint64_t seed);
    // language_model.model.layers.{0..num_layers-1}.* from the official (possibly sharded) safetensors
    void load_safetensors(const std::vector<std::string> &files);
    // the prompt enhancer's checkpoint: model.layers.{l}.*, model.norm and lm_head (or tied embeddings)
    void load_pe_safetensors(const std::vector<std::string> &files);
    void synthesize_head(uint64_t seed); // include/ernie_synth.h, ERNIE_SYNTH_TEXT_HEAD_LAYER
    int num_layers() const noexcept { return num_layers_; }
    ernie_cuda_text_model *handle() const noexcept { return handle_; }
    GpuContext &context() const noexcept { return ctx_; }

  private:
    GpuContext &ctx_;
    ernie_cuda_text_model *handle_ = nullptr;
    int num_layers_ = 0;
};
// run_text_blocks (src/text_encoder.h:16-18): `layers` (default all) layers over the embedded prompt with
// the constants {cos, sin, mask} of text_constants (the mask must be its causal mask). stats gets one
// compute time for the whole sequence of layers (the layers stay resident: no per-block load).
Tensor run_text_blocks(TextModel &model, const Tensor &input, const std::vector<Tensor> &constants,
                       Precision precision, BlockSequenceStats &stats, int layers = 0);

// ---- the optional prompt enhancer (src/prompt_enhancer.h:10-28, src/pe_session.h:9-42) ------------
struct PeOptions // include/ernie/pipeline.h
{
    int max_tokens = 2048;
    float temperature = .6f, top_p = .95f;
    uint32_t seed = 42;
    bool greedy = false;
};
// sample_pe_token (src/prompt_enhancer.cpp:33-66): std::invalid_argument for options outside max tokens
// 1..2048, a positive finite temperature and top-p in (0, 1], or an empty logits vector; std::runtime_error
// for non-finite logits. Greedy: the first maximum. Otherwise the tokens by descending logit (stable),
// weights exp((logit - max) / temperature) in double, the shortest prefix reaching top_p of the total,
// drawn with std::discrete_distribution from `random`.
uint32_t sample_pe_token(const std::vector<float> &logits, const PeOptions &options, std::mt19937 &random);
// PeSession on the B200: the layers of `model` (the PE checkpoint's, with its LM head) and a K/V cache of
// `capacity` tokens (1..4096).
class PeSession
{
  public:
    PeSession(TextModel &model, int capacity, Precision precision = Precision::FP32);
    ~PeSession();
    PeSession(const PeSession &) = delete;
    PeSession &operator=(const PeSession &) = delete;
    // one token (step) or 1..32 tokens (append_chunk): embedded [rows][3072], cos / sin [rows][128] ->
    // hidden [rows][3072]; std::invalid_argument past the capacity or for non-finite inputs
    Tensor step(const Tensor &embedded, const Tensor &cos, const Tensor &sin);
    Tensor append_chunk(const Tensor &embedded, const Tensor &cos, const Tensor &sin);
    void reset();
    int position() const;
    // the LM head on one hidden row [3072] -> logits [131072]
    std::vector<float> logits(const float *hidden_row);

  private:
    Tensor append(const Tensor &embedded, const Tensor &cos, const Tensor &sin, bool single);
    GpuContext &ctx_;
    ernie_cuda_pe_session *handle_ = nullptr;
};
struct PeResult // src/prompt_enhancer.h:12-18 (the text is the tokenizer's: out of scope here)
{
    std::vector<uint32_t> input_ids, generated_ids;
    bool eos = false;
};
using PeProgress = std::function<void(const char *, int, int)>;
using PeLogits = std::function<void(int, const std::vector<float> &)>;
// enhance_prompt (src/prompt_enhancer.cpp:68-197) after the tokenizer: the chat prompt's token ids through
// the session (prefill one token at a time, or in chunks of prefill_chunk <= 32), then up to
// options.max_tokens sampled tokens, stopping after the end-of-sequence token 2. embeddings: the PE's BF16
// table (raw or a checkpoint with model.embed_tokens.weight); frequencies: its 64 YaRN inverse
// frequencies (rope-inv-freq.f32). Progress "prefill" / "decode" as the reference reports them.
PeResult enhance_prompt_from_ids(TextModel &model, const std::string &embeddings, const std::vector<float> &frequencies,
                                 const std::vector<uint32_t> &input_ids, const PeOptions &options,
                                 Precision precision = Precision::FP32, int prefill_chunk = 1,
                                 const PeProgress &progress = {}, const PeLogits &observe = {});

// ---- generate from token ids (src/pipeline.cpp:489-575, everything after the tokenizer) -------------
struct GenerationModels // the device-resident stages and the package's small tables
{
    TextModel &text;                      // layers 0..24 of the prompt encoder
    DitModel &dit;
    VaeDecoder &vae;
    std::string embeddings;               // text/embeddings.bf16, or a checkpoint with embed_tokens
    std::vector<float> text_frequencies;  // text/rope-inv-freq.f32 (64 YaRN inverse frequencies)
    std::vector<float> dit_frequencies;   // dit/rope-inv-freq.f32 (empty: the built-in table)
    Tensor bn_mean, bn_variance;          // vae/bn-mean.f32, vae/bn-variance.f32 ([128])
    int dit_text_tokens = 0;              // model.cfg dit_text_tokens
    VaeEncoder *encoder = nullptr;        // img2img only (vae/encoder.*)
};
struct GeneratedImage
{
    RgbImage image;
    Tensor text;    // the prompt rows of the encoder's output [T][3072] (trace text.f32)
    Tensor latent;  // [128][h][w] after the last step
    Tensor decoded; // [3][16h][16w]
    int start_step = 0;
    double text_seconds = 0, dit_seconds = 0, vae_seconds = 0, elapsed_seconds = 0;
};
// The token ids of a prompt through the prompt encoder (at `text_bucket` slots), the DiT stage and the VAE
// stage, with the reference's traces (text.f32, the DiT stage's files, final/unpacked/decoded.f32) when
// request.trace names a folder, and the "text" / "denoise" progress notifications.
GeneratedImage generate_from_ids(GenerationModels &models, const std::vector<uint32_t> &ids, int text_bucket,
                                 const DitStageRequest &request,
                                 const std::function<void(const DitStageProgress &)> &notify = {});
// img2img (src/pipeline.cpp:341-345, :392-437, :536-540): the input image (request.width x request.height)
// through models.encoder; strength 0 decodes the encoded latent straight back (no prompt, no DiT), otherwise
// the encoded latent is request.encoded for the DiT stage's start step. Traces as the reference writes them:
// input.rgb, img2img.txt, encoder-mean/packed/normalized.f32. std::invalid_argument without an encoder, for a
// strength outside [0, 1] or an image whose size differs from the request's.
GeneratedImage generate_img2img_from_ids(GenerationModels &models, const std::vector<uint32_t> &ids,
                                         int text_bucket, const RgbImage &input, const DitStageRequest &request,
                                         const std::function<void(const DitStageProgress &)> &notify = {});

// ---- official checkpoints (safetensors) ------------------------------------------------------------
void load_safetensors(DitModel &model, const std::vector<std::string> &files, bool heads = true);
void load_safetensors(VaeDecoder &vae, const std::vector<std::string> &files);
void load_safetensors(VaeEncoder &encoder, const std::vector<std::string> &files);
} // namespace ernie
