/* CPU restatement of the reference's FP32 DiT hot path — TEST INFRASTRUCTURE ONLY.
 *
 * This library is the parity checker and the timed CPU baseline. Only tests/, the smoke check
 * in __graft_entry__.py and bench.py's CPU-baseline leg may load it; the CUDA product never
 * links, calls or falls back to it.
 *
 * It restates, function by function, the arithmetic of mingshi2333/ernie-image-ncnn-vulkan's
 * `--device cpu` path (ncnn CPU layers driven by the pnnx-exported graphs). The reference itself
 * cannot be built here: its `third_party/ncnn` submodule is empty (pin 3b7bdba7, sources.lock.json)
 * and its PyTorch spec imports `diffusers`, which is not installed. Each function names the
 * reference file:line it follows. Parity of this restatement is pinned at operator level by the
 * reference's own known-answer tests (tests/test_attention_mask.cpp, probes/attention_accuracy_probe.cpp,
 * probes/gelu_probe.cpp, probes/rmsnorm_probe.cpp, tests/test_residual_contract.cpp,
 * tests/test_latent_contract.cpp, tests/test_bf16_gemm.cpp, tests/test_memory_execution.cpp:324-329);
 * block- and step-level real-weight parity is unpinned because the reference ships no tensors.
 */
#ifndef ERNIE_ORACLE_H
#define ERNIE_ORACLE_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

typedef struct
{
    const uint16_t *wq, *wk, *wv, *wo; /* [4096,4096] BF16 bits, [out,in] */
    const uint16_t *wup, *wgate;       /* [12288,4096] */
    const uint16_t *wfc2;              /* [4096,12288] */
    const float *gamma_sa, *gamma_mlp; /* [4096] */
    const float *gamma_q, *gamma_k;    /* [128] */
} orc_block_weights;

typedef struct
{
    const uint16_t *x_embed_w;    /* [4096,128] (1x1 conv) */
    const float *x_embed_b;       /* [4096] */
    const uint16_t *text_proj_w;  /* [4096,3072], no bias */
    const uint16_t *time1_w;      /* [4096,4096] */
    const float *time1_b;         /* [4096] */
    const uint16_t *time2_w;      /* [4096,4096] */
    const float *time2_b;         /* [4096] */
    const uint16_t *adaln_w;      /* [24576,4096] */
    const float *adaln_b;         /* [24576] */
    const uint16_t *final_norm_w; /* [8192,4096] */
    const float *final_norm_b;    /* [8192] */
    const uint16_t *final_w;      /* [128,4096] */
    const float *final_b;         /* [128] */
} orc_head_weights;

int orc_num_threads(void);
void orc_set_num_threads(int threads);

/* Synthetic weights and inputs (ernie_synth.h protocol), filled into caller buffers. */
void orc_synth_bf16(uint64_t seed, uint64_t stream, float scale, float offset, uint16_t *out, int64_t count);
void orc_synth_f32_from_bf16(uint64_t seed, uint64_t stream, float scale, float offset, float *out, int64_t count);
void orc_synth_normal_f32(uint64_t seed, uint64_t stream, float scale, float *out, int64_t count);

/* Schedules, features and constants. Return 0, or -1 for an invalid request. */
int orc_turbo_schedule(int steps, float *sigmas, float *timesteps);
int orc_linear_schedule(int steps, float *sigmas, float *timesteps);
int orc_timestep_features(float timestep, float *out4096);
void orc_rope_frequencies(float *out64);
int orc_dit_constants(const float *freq64, int width, int height, int valid, int text, int token_limit,
                      float *cos_out, float *sin_out, float *mask_out);

/* Operators. */
void orc_rmsnorm(const float *x, const float *gamma, int64_t rows, int width, float eps, float *out);
void orc_layernorm(const float *x, int64_t rows, int width, float eps, float *out);
void orc_gelu(const float *x, float *out, int64_t count);
void orc_silu(const float *x, float *out, int64_t count);
void orc_residual_add(const float *a, const float *b, float *out, int64_t count);
/* q [heads][nq][width], k,v [kv_heads][nk][width], mask [mask_heads][mask_rows][nk] (mask_rows 1 or nq),
   out [heads][nq][width]; kv_heads and mask_heads are 1 or heads. FP64 softmax and accumulation. */
void orc_sdpa(const float *q, const float *k, const float *v, const float *mask, int heads, int kv_heads,
              int mask_heads, int mask_rows, int nq, int nk, int width, float *out);
/* C[M,N] = A[M,K] * W[N,K]^T (+ bias[N]); W is BF16 bits. */
void orc_linear(const float *a, const uint16_t *w, const float *bias, int64_t m, int n, int k, float *c);
int orc_euler_step(const float *sample, const float *prediction, float delta, int64_t count, float *out);
int orc_finite(const float *x, int64_t count);
int orc_unpack_for_vae(const float *packed, const float *mean, const float *variance, int width, int height,
                       float *out);

/* Model stages. */
void orc_block(const float *x, const orc_block_weights *w, const float *modulation /*[6][4096]*/,
               const float *cos_table, const float *sin_table, const float *mask, int tokens, float *out);
void orc_input_head(const orc_head_weights *w, const float *latent /*[128][h][w]*/, int width, int height,
                    const float *text /*[text][3072]*/, int text_tokens, const float *features /*[4096]*/,
                    float *x_out /*[N][4096]*/, float *c_out /*[4096]*/, float *modulation_out /*[6][4096]*/);
void orc_output_head(const orc_head_weights *w, const float *x /*[N][4096]*/, const float *c, int width,
                     int height, float *prediction /*[128][h][w]*/);
/* One DiT prediction over `blocks` blocks (blocks[i] points at block i's weights). */
void orc_dit(const orc_head_weights *heads, const orc_block_weights *const *blocks, int num_blocks,
             const float *latent, int width, int height, const float *text, int text_tokens,
             const float *features, const float *cos_table, const float *sin_table, const float *mask,
             float *prediction);
/* Euler loop (src/denoiser.cpp:41-86). schedule: 0 = turbo, 1 = linear. predictions may be NULL,
   else [steps][128*h*w]. Returns 0, -1 for invalid requests, or k>0 if the latent became
   non-finite after step k. */
int orc_denoise(const orc_head_weights *heads, const orc_block_weights *const *blocks, int num_blocks,
                const float *initial, int width, int height, const float *text, int text_tokens,
                const float *cos_table, const float *sin_table, const float *mask, int steps, int start_step,
                int end_step, int schedule, float *latent_out, float *predictions);

#ifdef __cplusplus
}
#endif
#endif
