/* C ABI of the B200-native ERNIE-Image-Turbo DiT denoiser hot path (libernie_b200.so).
 *
 * Drop-in boundary for mingshi2333/ernie-image-ncnn-vulkan's ncnn/Vulkan denoiser path. Plain
 * pointers and sizes only. Return codes follow ncnn's convention as the reference maps it in
 * check_ncnn_memory (src/vulkan_memory.cpp:21-30): 0 = success, -100 = (device) allocation failure
 * (the C++ wrapper throws GpuAllocationError), -1 = any other failure (std::runtime_error or
 * std::invalid_argument). ernie_cuda_last_error() returns the calling thread's last message.
 *
 * Memory: "dev" pointers are CUDA device memory owned by the caller (allocate with
 * ernie_cuda_malloc or any CUDA allocator on the context's device); they must outlive the work
 * enqueued on the context's stream, as the reference requires of its VkMat arguments
 * (src/dit.h:26-29, src/latent_ops.h:32-35). "host" pointers are ordinary host memory and are
 * consumed or filled before the call returns. Tensors are dense row-major FP32 unless noted;
 * weights are BF16 bit patterns (uint16_t).
 *
 * Threading: a context owns one CUDA stream on one device. Calls on one context are serialised by
 * the caller, as ernie::generate calls are (include/ernie/pipeline.h:145). Use one context (and one
 * host thread) per GPU for data-parallel work.
 */
#ifndef ERNIE_CUDA_H
#define ERNIE_CUDA_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

#define ERNIE_CUDA_OK 0
#define ERNIE_CUDA_ERROR (-1)
#define ERNIE_CUDA_OUT_OF_MEMORY (-100)

/* Arithmetic modes. BF16: BF16 GEMM/attention operands, FP32 accumulation, FP32 residual stream,
   norms, softmax and latent (the reference's use_bf16_storage path). FP32: FP32-exact mode
   (activations split into three BF16 planes against exact-BF16 weights; FP32 attention with FP64
   softmax sums), gated like the reference's FP32 path. */
#define ERNIE_PRECISION_BF16 0
#define ERNIE_PRECISION_FP32 1
#define ERNIE_SCHEDULE_TURBO 0  /* FlowSchedule::turbo, src/latent_ops.cpp:31-51 */
#define ERNIE_SCHEDULE_LINEAR 1 /* evenly spaced sigmas 1 -> 0 (benchmark configuration) */

/* Block tensor ids for ernie_cuda_model_read_tensor (test hook). */
#define ERNIE_TENSOR_WQKV 0  /* [12288,4096] = [Wq; Wk; Wv] */
#define ERNIE_TENSOR_WO 1    /* [4096,4096] */
#define ERNIE_TENSOR_WUPGATE 2 /* [24576,4096], 64-row groups interleaved: up g, gate g, ... */
#define ERNIE_TENSOR_WFC2 3  /* [4096,12288] */

typedef struct ernie_cuda_context ernie_cuda_context;
typedef struct ernie_cuda_model ernie_cuda_model;
typedef struct ernie_cuda_session ernie_cuda_session;
typedef struct ernie_cuda_text_model ernie_cuda_text_model; /* prompt encoder layers (Text encoder section) */
typedef struct ernie_cuda_vae ernie_cuda_vae;               /* VAE decoder (VAE decoder section) */
typedef struct ernie_cuda_vae_encoder ernie_cuda_vae_encoder; /* VAE encoder (VAE encoder section) */
typedef struct ernie_cuda_pe_session ernie_cuda_pe_session;   /* prompt enhancer (Prompt enhancer section) */

/* Host weights of one block, as tools/build_dit_weights.py:19-31 binds them to the block graph. */
typedef struct
{
    const uint16_t *wq, *wk, *wv, *wo; /* [4096,4096] BF16, [out,in] */
    const uint16_t *wup, *wgate;       /* [12288,4096] */
    const uint16_t *wfc2;              /* [4096,12288] */
    const float *gamma_sa, *gamma_mlp; /* [4096] adaLN_sa_ln / adaLN_mlp_ln */
    const float *gamma_q, *gamma_k;    /* [128] norm_q / norm_k */
} ernie_cuda_block_weights;

/* Host weights of the input and output heads (tools/export_dit_heads.py:19 HEADS). */
typedef struct
{
    const uint16_t *x_embed_w;    /* [4096,128] x_embedder.proj (1x1 conv) */
    const float *x_embed_b;       /* [4096] */
    const uint16_t *text_proj_w;  /* [4096,3072] */
    const uint16_t *time1_w;      /* [4096,4096] time_embedding.linear_1 */
    const float *time1_b;
    const uint16_t *time2_w;      /* [4096,4096] time_embedding.linear_2 */
    const float *time2_b;
    const uint16_t *adaln_w;      /* [24576,4096] adaLN_modulation.1 */
    const float *adaln_b;
    const uint16_t *final_norm_w; /* [8192,4096] final_norm.linear */
    const float *final_norm_b;
    const uint16_t *final_w;      /* [128,4096] final_linear */
    const float *final_b;
} ernie_cuda_head_weights;

/* Packed latent geometry and text slots of one request (src/shape_plan.h:10-29, model.cfg keys). */
typedef struct
{
    int width, height; /* packed latent grid, 1..256 */
    int text_tokens;   /* DiT text slots (bucket), 1..2048 */
    int valid_text;    /* valid text tokens T, 1..text_tokens */
} ernie_cuda_shape;

const char *ernie_cuda_last_error(void);
int ernie_cuda_device_count(int *count);

/* ---- GPU context: replaces GpuContext (src/gpu_context.h:12-27) -------------------------- */
int ernie_cuda_context_create(int device, ernie_cuda_context **out);
int ernie_cuda_context_destroy(ernie_cuda_context *ctx);
/* Wait for the stream; reports a device-side protocol timeout (bounded waits) as -1. */
int ernie_cuda_context_synchronize(ernie_cuda_context *ctx);
/* Device budget reader (replaces the Vulkan budget reader, src/weight_placement.cpp:75-97). */
int ernie_cuda_context_memory(ernie_cuda_context *ctx, uint64_t *free_bytes, uint64_t *total_bytes);
int ernie_cuda_context_sm_count(ernie_cuda_context *ctx, int *sms);
int ernie_cuda_malloc(ernie_cuda_context *ctx, size_t bytes, void **dev);
int ernie_cuda_free(ernie_cuda_context *ctx, void *dev);
int ernie_cuda_upload(ernie_cuda_context *ctx, void *dev, const void *host, size_t bytes);
int ernie_cuda_download(ernie_cuda_context *ctx, void *host, const void *dev, size_t bytes);
int ernie_cuda_memset(ernie_cuda_context *ctx, void *dev, int value, size_t bytes);
/* Device time between two points on the context stream, for benchmarks (milliseconds). */
int ernie_cuda_event_record(ernie_cuda_context *ctx, int slot);
int ernie_cuda_event_elapsed(ernie_cuda_context *ctx, int start_slot, int end_slot, float *ms);

/* ---- Resident weights: replace the per-block Net load/stream of run_block_sequence
        (src/block_sequence.cpp:119-278), WeightPlacement (src/weight_placement.h:34-51) and
        WeightSession (src/weight_session.h:29-73). All 36 blocks fit in HBM (15.7 GB BF16). --- */
int ernie_cuda_model_create(ernie_cuda_context *ctx, int num_blocks, ernie_cuda_model **out);
int ernie_cuda_model_destroy(ernie_cuda_model *model);
int ernie_cuda_model_upload_block(ernie_cuda_model *model, int block, const ernie_cuda_block_weights *host);
int ernie_cuda_model_upload_heads(ernie_cuda_model *model, const ernie_cuda_head_weights *host);
/* Seeded random-init weights generated on the device (include/ernie_synth.h protocol). */
int ernie_cuda_model_synthesize(ernie_cuda_model *model, uint64_t seed);
int ernie_cuda_model_read_tensor(ernie_cuda_model *model, int block, int tensor, void *host, size_t bytes);
int ernie_cuda_model_bytes(ernie_cuda_model *model, uint64_t *bytes);

/* ---- ERNIE layer contracts (src/ernie_gelu.cpp:108-116 register_layers), dev pointers ---- */
/* ErnieSDPA (src/ernie_attention.cpp:158-233): out = softmax(q k^T / sqrt(width) + mask) v.
   q [heads][nq][width], k/v [kv_heads][nk][width] with kv_heads 1 or heads, mask NULL or
   [mask_heads][mask_rows][nk] additive with mask_heads 1 or heads and mask_rows 1 or nq,
   width 1..128. FP32 in/out, FP64 softmax accumulation. */
int ernie_cuda_sdpa(ernie_cuda_context *ctx, const float *q, const float *k, const float *v, const float *mask,
                    int heads, int kv_heads, int mask_heads, int mask_rows, int nq, int nk, int width, float *out);
/* BF16 flash path of the same operator (tcgen05/TMEM kernel) on head-major BF16 q/k
   [heads][rows_pad][128] and transposed v [heads][128][rows_pad] (rows_pad a multiple of 128, padded
   rows zero), keys >= kv_len excluded, optional additive row mask [nq]. Output token-major BF16
   [nq][heads*128]. */
int ernie_cuda_sdpa_bf16(ernie_cuda_context *ctx, const uint16_t *q, const uint16_t *k, const uint16_t *vt,
                         const float *mask, int heads, int nq, int rows_pad, int kv_len, uint16_t *out);
/* set_attention_query_rows (src/ernie_attention.cpp:245-255): 128, 64, 32 or 16, else -1.
   The flash kernels need no query chunking; the value is recorded for the recovery contract. */
int ernie_cuda_set_attention_query_rows(ernie_cuda_context *ctx, int rows);
int ernie_cuda_attention_query_rows(ernie_cuda_context *ctx, int *rows);
/* ErnieNorm RMSNorm (src/ernie_rmsnorm.cpp:21-135): width 128, 3072 or 4096, affine. */
int ernie_cuda_rmsnorm(ernie_cuda_context *ctx, const float *x, const float *gamma, int64_t rows, int width,
                       float eps, float *out);
/* ErnieNorm LayerNorm: width 4096, non-affine. */
int ernie_cuda_layernorm(ernie_cuda_context *ctx, const float *x, int64_t rows, int width, float eps, float *out);
/* ErnieGELU (src/ernie_gelu.cpp:35-103): in place, count % 4 == 0 else -1. */
int ernie_cuda_gelu(ernie_cuda_context *ctx, float *data, int64_t count);
/* ErnieResidualAdd (src/ernie_residual.cpp:19-92): FP32 out = a + b. */
int ernie_cuda_residual_add(ernie_cuda_context *ctx, const float *a, const float *b, float *out, int64_t count);
/* tcgen05 GEMM: c[M,N] = a[M,K] (BF16) * w[N,K]^T (BF16) + bias (nullable), FP32 out.
   K and N multiples of 64 and 128. */
int ernie_cuda_linear_bf16(ernie_cuda_context *ctx, const uint16_t *a, const uint16_t *w, const float *bias,
                           float *c, int m, int n, int k);

/* ---- Latent ops (src/latent_ops.h:15-57), dev pointers, latent [128][h][w] ------------------ */
int ernie_cuda_euler_step(ernie_cuda_context *ctx, const float *sample, const float *prediction, float delta,
                          int width, int height, float *out);
int ernie_cuda_finite_latent(ernie_cuda_context *ctx, const float *latent, int width, int height, int *finite);
int ernie_cuda_unpack_for_vae(ernie_cuda_context *ctx, const float *packed, const float *mean,
                              const float *variance, int width, int height, float *out);
/* Host helpers of the same path: FlowSchedule::turbo / linear (sigmas [steps+1], timesteps
   [steps]), timestep_features (src/denoiser.cpp:22-39), dit_constants (src/conditioning.cpp:10-44)
   from the 64-value frequency table (NULL = the official table of tools/prepare_pipeline.py:63). */
int ernie_cuda_schedule(int steps, int schedule, float *sigmas, float *timesteps);
int ernie_cuda_timestep_features(float timestep, float *out4096);
int ernie_cuda_dit_constants(const float *freq64, int width, int height, int valid_text, int text_tokens,
                             int token_limit, float *cos_out, float *sin_out, float *mask_out);

/* ---- Request session: one shape, one precision; activations sized once ------------------- */
int ernie_cuda_session_create(ernie_cuda_model *model, const ernie_cuda_shape *shape, int precision,
                              ernie_cuda_session **out);
int ernie_cuda_session_destroy(ernie_cuda_session *session);
/* Conditioning constants of the request (the four `constants` of denoise, src/denoiser.h:26-27):
   text [text_tokens][3072] (padded, pad_text src/conditioning.cpp:56-67; NULL skips text_proj),
   cos/sin [N][128], mask [N] with N = width*height + text_tokens. Host pointers. text_proj runs
   once here, not once per step. */
int ernie_cuda_session_set_conditioning(ernie_cuda_session *session, const float *text, const float *cos_table,
                                        const float *sin_table, const float *mask);
int ernie_cuda_session_tokens(ernie_cuda_session *session, int *tokens);
/* run_block_sequence (src/block_sequence.h:38-60): blocks [first, first+count) on x (dev,
   [N][4096] FP32, updated in place) with shared modulation (dev [6][4096]: shift_sa, scale_sa,
   gate_sa, shift_mlp, scale_mlp, gate_mlp). */
int ernie_cuda_session_blocks(ernie_cuda_session *session, int first, int count, float *x, const float *modulation);
/* run_dit (src/dit.h:17-40): one prediction [128][h][w] for latent [128][h][w] at `timestep`
   (dev pointers). */
int ernie_cuda_session_dit(ernie_cuda_session *session, const float *latent, float timestep, float *prediction);
/* denoise (src/denoiser.h:30-44) on the session's device latent: steps [start_step, end_step)
   of an S-step schedule, captured as a CUDA graph when use_graph != 0. The latent lives at
   ernie_cuda_session_latent(). *failed_step receives the first step k (1-based) after which the
   latent was non-finite, else 0 (and the call returns -1 in that case). */
int ernie_cuda_session_latent(ernie_cuda_session *session, float **latent_dev);
int ernie_cuda_session_denoise_device(ernie_cuda_session *session, int steps, int start_step, int end_step,
                                      int schedule, int use_graph, int *failed_step);
/* Same loop end to end with host buffers: initial -> final (host [128][h][w]); predictions
   (nullable, host [end-start][128][h][w]) receives every step's DiT output. */
int ernie_cuda_session_denoise(ernie_cuda_session *session, const float *initial, float *final_latent, int steps,
                               int start_step, int end_step, int schedule, float *predictions, int *failed_step);

/* Initial noise of a request without a latent file (src/pipeline.cpp:520-531): std::mt19937(seed) feeding
   std::normal_distribution<float>(0, 1), channel after channel, into out [128][height][width]. Host-only. */
int ernie_cuda_initial_noise(unsigned seed, int width, int height, float *out);

/* ---- Text encoder (the prompt encoder before the denoise loop) ------------------------------------
   run_text_blocks (src/text_encoder.h:16-18, src/text_encoder.cpp:106-166) on one B200: the Mistral decoder
   layers the reference exports per block (tools/export_text_block.py:51-61: hidden 3072, 32 query and 8
   K/V heads of 128, SwiGLU 9216, RMSNorm eps 1e-5, no biases), all layers resident on the device (the
   pipeline runs layers 0..24). Input: the embedded prompt [bucket][3072] FP32 (text_embeddings; rows past
   the prompt zero), cos/sin [bucket][128] of ernie_cuda_text_constants; the attention mask is the causal
   mask text_constants builds. Output: the hidden state [bucket][3072] after `layers` layers (1..num_layers).
   precision: BF16 (BF16 GEMM operands, FP32 accumulation, residual, norms and attention) or FP32
   (three-plane FP32-exact GEMMs against the exact-BF16 weights; FP32 attention with FP64 sums). */
/* One layer's weights as the official checkpoint stores them (language_model.model.layers.N.*). */
typedef struct
{
    const uint16_t *wq;             /* [4096,3072] BF16 self_attn.q_proj */
    const uint16_t *wk, *wv;        /* [1024,3072] self_attn.k_proj / v_proj */
    const uint16_t *wo;             /* [3072,4096] self_attn.o_proj */
    const uint16_t *wgate, *wup;    /* [9216,3072] mlp.gate_proj / up_proj */
    const uint16_t *wdown;          /* [3072,9216] mlp.down_proj */
    const float *gamma_attn;        /* [3072] input_layernorm */
    const float *gamma_mlp;         /* [3072] post_attention_layernorm */
} ernie_cuda_text_layer_weights;
int ernie_cuda_text_model_create(ernie_cuda_context *ctx, int num_layers, ernie_cuda_text_model **out);
int ernie_cuda_text_model_destroy(ernie_cuda_text_model *model);
int ernie_cuda_text_model_bytes(ernie_cuda_text_model *model, uint64_t *bytes);
int ernie_cuda_text_model_upload_layer(ernie_cuda_text_model *model, int layer, const ernie_cuda_text_layer_weights *host);
/* Seeded random-init weights (include/ernie_synth.h, text encoder streams). */
int ernie_cuda_text_model_synthesize(ernie_cuda_text_model *model, uint64_t seed);
/* text_constants (src/text_encoder.cpp:76-104), host: inv_freq[64] (the YaRN inverse frequencies) ->
   cos/sin [bucket][128] (both halves of a row repeat the 64 angles t * f_j) and, if mask is not null, the
   causal mask [bucket][bucket] (0 on and below the diagonal, -FLT_MAX above). */
int ernie_cuda_text_constants(const float *inv_freq, int bucket, float *cos_out, float *sin_out, float *mask);
/* Host buffers, synchronous. */
int ernie_cuda_text_run_blocks(ernie_cuda_text_model *model, const float *input, int bucket, const float *cos_t,
                               const float *sin_t, int precision, int layers, float *out);
/* Device buffers on the context's stream (synchronous: the kernels' status is checked). */
int ernie_cuda_text_run_blocks_device(ernie_cuda_text_model *model, const float *input, int bucket,
                                      const float *cos_t, const float *sin_t, int precision, int layers, float *out);

/* Prompt-token embeddings (text_embeddings, src/text_encoder.cpp:48-75): rows ids[0..count) of the
   [131072][3072] table into out [bucket][3072] FP32 (rows past count zero). `path` is the reference's raw
   BF16 table ("text/embeddings.bf16") or a checkpoint .safetensors holding
   language_model.model.embed_tokens.weight. Only the requested rows are read. */
int ernie_cuda_text_embeddings(const char *path, const uint32_t *ids, int count, int bucket, float *out);

/* ---- Official checkpoints (safetensors, BF16) ------------------------------------------------------
   Read the official tensors straight into the resident models, in place of the reference's packaging
   tools (tools/build_dit_weights.py, tools/build_text_weights.py, tools/export_vae.py). A checkpoint may be
   sharded over several files; each tensor is taken from the file that holds it. GEMM weights must be BF16
   (loaded losslessly); norm weights and biases may be BF16, F16 or F32. Shapes are checked (a 1x1
   convolution's trailing unit dimensions match a linear weight), non-finite values rejected.
     DiT:  layers.{b}.{self_attention.to_q/to_k/to_v/to_out.0, mlp.up_proj/gate_proj/linear_fc2}.weight,
           layers.{b}.{adaLN_sa_ln, adaLN_mlp_ln, self_attention.norm_q, self_attention.norm_k}.weight
           for b < num_blocks (tools/build_dit_weights.py:19-31); with_heads: x_embedder.proj, text_proj,
           time_embedding.linear_1/linear_2, adaLN_modulation.1, final_norm.linear, final_linear
           (tools/export_dit_heads.py:19).
     Text: language_model.model.layers.{l}.{self_attn.q/k/v/o_proj, mlp.gate/up/down_proj,
           input_layernorm, post_attention_layernorm}.weight for l < num_layers.
     VAE:  every name of ernie_cuda_vae_tensor_info (post_quant_conv.*, decoder.*).
     VAE encoder: every name of ernie_cuda_vae_encoder_tensor_info (encoder.*, quant_conv.*,
           bn.running_mean, bn.running_var). */
int ernie_cuda_model_load_safetensors(ernie_cuda_model *model, int num_blocks, const char *const *files, int count,
                                      int with_heads);
int ernie_cuda_text_model_load_safetensors(ernie_cuda_text_model *model, int num_layers, const char *const *files,
                                           int count);
int ernie_cuda_vae_load_safetensors(ernie_cuda_vae *vae, const char *const *files, int count);
int ernie_cuda_vae_encoder_load_safetensors(ernie_cuda_vae_encoder *encoder, const char *const *files, int count);
/* The prompt enhancer's checkpoint: model.layers.{l}.* for l < num_layers (the same tensor names as the
   text layers after "language_model."), model.norm.weight and lm_head.weight (or, tied,
   model.embed_tokens.weight) into a text model and its LM head. */
int ernie_cuda_pe_model_load_safetensors(ernie_cuda_text_model *model, int num_layers, const char *const *files,
                                         int count);
/* The header of one file: the number of tensors, and tensor `index` (in name order): name, dtype
   ("BF16", "F16", "F32", ...; 8 bytes), shape (up to 8 dims). */
int ernie_cuda_safetensors_count(const char *path, int *count);
int ernie_cuda_safetensors_entry(const char *path, int index, char *name, size_t name_bytes, char *dtype,
                                 int64_t *dims, int *ndim);

/* ---- VAE decoder (the stage after the denoise loop) -----------------------------------------------
   decode_vae (src/vae.h:16-22, src/vae.cpp:18-64) of the pinned AutoencoderKLFlux2 post_quant_conv +
   decoder, and rgb_image (src/pipeline.cpp:145-163), on one B200. Weights are addressed by their
   diffusers parameter names and shapes (ernie_cuda_vae_tensor_info lists all of them, e.g.
   "decoder.up_blocks.2.resnets.0.conv_shortcut.weight" [256,512,1,1]), uploaded as FP32. The input is
   the unpacked latent [32][height][width] (ernie_cuda_unpack_for_vae's output); the output is the
   decoded image [3][8*height][8*width] FP32 and, optionally, its RGB bytes [8*height][8*width][3]
   (clamp(x/2 + 0.5, 0, 1) * 255 rounded to nearest even). *nonfinite (nullable) is set to 1 when a
   decoded value is not finite: the reference's rgb_image throws there; those pixels' bytes are
   unspecified. 1 <= width, height <= 256 with width * height <= 57344 (the mid-block attention row).
   precision: ERNIE_PRECISION_BF16 (BF16 convolution operands, FP32 accumulation and residuals) or
   ERNIE_PRECISION_FP32 (three-plane FP32-exact operands; the reference's FP32 CPU path is the gate). */
int ernie_cuda_vae_create(ernie_cuda_context *ctx, ernie_cuda_vae **out);
int ernie_cuda_vae_destroy(ernie_cuda_vae *vae);
int ernie_cuda_vae_tensor_count(int *count);
/* name (NUL-terminated, name_bytes >= 64 suffices) and shape (up to 4 dims) of tensor `index`. */
int ernie_cuda_vae_tensor_info(int index, char *name, size_t name_bytes, int *dims, int *ndim);
int ernie_cuda_vae_upload(ernie_cuda_vae *vae, const char *name, const float *host, size_t count);
/* Seeded random-init weights (include/ernie_synth.h, VAE section); bf16_weights rounds the convolution
   and projection weights to BF16 values. */
int ernie_cuda_vae_synthesize(ernie_cuda_vae *vae, uint64_t seed, int bf16_weights);
int ernie_cuda_vae_bytes(ernie_cuda_vae *vae, uint64_t *weights, uint64_t *workspace);
/* Kernel launches of one decode of this shape (builds the shape's workspace and graph). */
int ernie_cuda_vae_launches(ernie_cuda_vae *vae, int width, int height, int precision, int *launches);
/* Eager run of the decode with CUDA events around every launch (measurement hook): per kernel class the
   mean milliseconds over `iters` runs and the algorithmic work of one run, ms[6] and work[6] indexed
   0 convolutions (FLOPs), 1 attention score/value GEMMs (FLOPs), 2 softmax (bytes), 3 GroupNorm (bytes),
   4 upsample (bytes), 5 other bandwidth passes (bytes). */
int ernie_cuda_vae_profile(ernie_cuda_vae *vae, int width, int height, int precision, int iters, double *ms,
                           double *work);
/* Host buffers, synchronous. */
int ernie_cuda_vae_decode(ernie_cuda_vae *vae, const float *unpacked, int width, int height, int precision,
                          float *decoded, uint8_t *rgb, int *nonfinite);
/* Device buffers on the context's stream; synchronous only when nonfinite is non-null. */
int ernie_cuda_vae_decode_device(ernie_cuda_vae *vae, const float *unpacked, int width, int height, int precision,
                                 float *decoded, uint8_t *rgb, int *nonfinite);

/* ---- VAE encoder (img2img's image latent) -------------------------------------------------------
   encode_vae (src/image_encoder.h:9-20, src/image_encoder.cpp:28-72) of the pinned AutoencoderKLFlux2
   encoder + quant_conv + bn as tools/export_vae_encoder.py:74-80 wraps it, on one B200. Input: RGB bytes
   [height][width][3], normalised as (v - 127.5f) * (1 / 127.5f). Outputs (the reference's VaeEncoding,
   FP32 planar): mean [32][height/8][width/8] (quant_conv(encoder(x))[:32], the posterior's mode), packed
   = pixel_unshuffle(mean, 2) [128][height/16][width/16], normalized = (packed - bn.running_mean) /
   sqrt(bn.running_var + 1e-4) [128][height/16][width/16] (make_img2img_start's `encoded`). *nonfinite
   (nullable) is set to 1 when an output is not finite (the reference throws there). Sides are multiples
   of 16 up to 2048 (the reference admits its reviewed 32x32, 64x32, 512x384 and 1024x1024). Weights by
   diffusers name (ernie_cuda_vae_encoder_tensor_info), uploaded as FP32. precision as for the decoder;
   the reference's encoder is CPU FP32 only, so FP32-exact mode is its parity mode. */
int ernie_cuda_vae_encoder_create(ernie_cuda_context *ctx, ernie_cuda_vae_encoder **out);
int ernie_cuda_vae_encoder_destroy(ernie_cuda_vae_encoder *encoder);
int ernie_cuda_vae_encoder_tensor_count(int *count);
int ernie_cuda_vae_encoder_tensor_info(int index, char *name, size_t name_bytes, int *dims, int *ndim);
int ernie_cuda_vae_encoder_upload(ernie_cuda_vae_encoder *encoder, const char *name, const float *host, size_t count);
/* Seeded random-init weights (include/ernie_synth.h, VAE section; bn.running_var = 1 + 0.1 N(0,1)). */
int ernie_cuda_vae_encoder_synthesize(ernie_cuda_vae_encoder *encoder, uint64_t seed, int bf16_weights);
int ernie_cuda_vae_encoder_bytes(ernie_cuda_vae_encoder *encoder, uint64_t *weights, uint64_t *workspace);
int ernie_cuda_vae_encoder_launches(ernie_cuda_vae_encoder *encoder, int width, int height, int precision,
                                    int *launches);
/* As ernie_cuda_vae_profile; class 4 is the stride-2 convolutions' operand pass. */
int ernie_cuda_vae_encoder_profile(ernie_cuda_vae_encoder *encoder, int width, int height, int precision, int iters,
                                   double *ms, double *work);
/* Host buffers, synchronous. */
int ernie_cuda_vae_encode(ernie_cuda_vae_encoder *encoder, const uint8_t *rgb, int width, int height, int precision,
                          float *mean, float *packed, float *normalized, int *nonfinite);
/* Device buffers on the context's stream; synchronous only when nonfinite is non-null. */
int ernie_cuda_vae_encode_device(ernie_cuda_vae_encoder *encoder, const uint8_t *rgb, int width, int height,
                                 int precision, float *mean, float *packed, float *normalized, int *nonfinite);

/* ---- Prompt enhancer (optional: the LM that rewrites the prompt before the text encoder) -------------
   PeSession (src/pe_session.h:9-42) and the head of enhance_prompt (src/prompt_enhancer.cpp:68-197) on one
   B200: the Mistral decoder layers of a text model (the PE checkpoint's 26 layers) with a per-layer K/V
   cache, and the LM head of head.ncnn.param (tools/build_pe_model.py:100-105: RMSNorm eps 1e-5, then the
   131072 x 3072 projection). The tokenizer and sampling stay on the host (the C++ surface has
   sample_pe_token and enhance_prompt_from_ids). precision: ERNIE_PRECISION_FP32 (FP32-exact; the
   reference's PE is CPU FP32) or ERNIE_PRECISION_BF16. */
/* LM head weights of a text model: final RMSNorm weight [3072] FP32 and lm_head [131072][3072] BF16. */
int ernie_cuda_text_model_upload_head(ernie_cuda_text_model *model, const float *norm, const uint16_t *lm_head);
/* Seeded random-init head (include/ernie_synth.h, ERNIE_SYNTH_TEXT_HEAD_LAYER). */
int ernie_cuda_text_model_synthesize_head(ernie_cuda_text_model *model, uint64_t seed);
/* A session of `capacity` tokens (1..4096) over all the model's layers. */
int ernie_cuda_pe_session_create(ernie_cuda_text_model *model, int capacity, int precision,
                                 ernie_cuda_pe_session **out);
int ernie_cuda_pe_session_destroy(ernie_cuda_pe_session *session);
int ernie_cuda_pe_session_reset(ernie_cuda_pe_session *session);
int ernie_cuda_pe_session_position(ernie_cuda_pe_session *session, int *position);
/* append_chunk / step: `rows` (1..32) new tokens at the session's position, embedded [rows][3072] and
   their rotary rows cos / sin [rows][128] (host FP32) -> the last layer's hidden states [rows][3072]
   (host). Rejects more rows than the capacity left and non-finite inputs; a call that fails on the device
   leaves the session unusable until reset (as PeSession does). */
int ernie_cuda_pe_session_append(ernie_cuda_pe_session *session, const float *embedded, const float *cos,
                                 const float *sin, int rows, float *hidden);
/* logits [131072] (host FP32) of one hidden row [3072] through the model's LM head. */
int ernie_cuda_pe_logits(ernie_cuda_pe_session *session, const float *hidden, float *logits);

/* ---- Ulysses sequence parallelism (one process per GPU, 2, 4 or 8 members, BF16) ---------------
   Tokens are split into contiguous shards of S = ceil(N / world) rows (rounded up to 16); every member
   holds the full weights. Per block, the QKV GEMM's epilogue stores each head of this GPU's rows straight
   into the memory of the member that attends with it (32/world heads each, over the whole sequence),
   and the attention kernel stores each output row back into the memory of the member owning that token
   (NVLink peer stores into buffers shared through CUDA IPC), with a bounded device-side barrier after
   each. Each member keeps its own token slice of the latent across steps; denoise takes and returns
   whole latents. Setup: create on every member, exchange the 64-byte handles through any host channel,
   connect with all handles in rank order. All members must then make the same calls in the same order;
   destroying a connected session is such a call too (the members leave together). */
#define ERNIE_CUDA_SP_HANDLE_BYTES 64
int ernie_cuda_session_create_sp(ernie_cuda_model *model, const ernie_cuda_shape *shape, int precision, int rank,
                                 int world, ernie_cuda_session **out);
int ernie_cuda_sp_handle(ernie_cuda_session *session, void *handle);
int ernie_cuda_sp_connect(ernie_cuda_session *session, const void *handles);
/* Layout of rank `rank`: shard rows S, gathered rows (world*S rounded up to 128), this rank's image rows,
   real rows, and the first text slot it owns. Host-only. */
int ernie_cuda_sp_layout(int tokens, int image_tokens, int world, int rank, int *shard, int *full_rows,
                         int *image_rows, int *real_rows, int *text_begin);

/* Non-finite check that allocates no device memory. It has no counterpart in the reference.
   Applications that reserve their device memory at start-up and forbid device allocation afterwards
   use it instead of ernie_cuda_finite_latent, which allocates a status word per call. Scratch is a
   fixed 512-byte device array (128 per-channel status words) that every GPU loading the library holds
   until exit; latents outside 128 x [1..256] x [1..256] are rejected (-1). Each call looks up that
   array's device address on the context's device; the first call on a device may load the library's
   device code there, so make it at start-up. Every call shares the array and clears it first; calls
   that overlap on the GPU race on it. The call waits for the context's stream. */
int ernie_cuda_finite_latent_noalloc(ernie_cuda_context *ctx, const float *latent, int width, int height,
                                     int *finite);

/* Benchmark hooks: average device time in ms of `iters` back-to-back launches of one kernel of the
   block on the session's buffers, cycling through the model's blocks so that weights stream from HBM
   as in a step (kernel 0 norm+modulate, 1 QKV GEMM, 2 attention, 3 out-proj GEMM, 4 MLP
   norm+modulate, 5 up/gate GEMM, 6 down GEMM, 7 a whole block, 8 a whole denoise step after one has
   run, 9 the same step without its blocks; 10..16 = part 0..6 timed inside consecutive whole blocks,
   at most 7 of them; 17 a whole block enqueued part by part, which in a sequence-parallel session
   synchronises through the two barrier kernels instead of the kernels' completion flags); and the
   number of kernels one denoise step launches. */
int ernie_cuda_session_profile(ernie_cuda_session *session, int kernel, int iters, float *ms);
int ernie_cuda_session_launches_per_step(ernie_cuda_session *session, int *launches);

#ifdef __cplusplus
}
#endif
#endif
