// C ABI of the prompt encoder (include/ernie_cuda.h, "Text encoder"): the Mistral decoder layers the
// reference runs one ncnn block at a time (run_text_blocks, src/text_encoder.cpp:106-166; the block graph
// is tools/export_text_block.py:51-61 TextBlock.forward) with every layer's weights resident on the device,
// and the constants of text_constants (src/text_encoder.cpp:76-104). Host orchestration only.
//
// Per layer (hidden 3072, 32 query heads and 8 K/V heads of 128, SwiGLU 9216, RMSNorm eps 1e-5):
//   norm_modulate (RMSNorm, input_layernorm) -> tcgen05 GEMM [q; k; v] (F32 out) -> rotary ->
//   causal grouped-query attention (BF16 mode: the tcgen05 flash kernel of the DiT with its causal and
//   grouped-K/V options; FP32-exact mode: FP32 attention with FP64 sums) -> GEMM o_proj, residual added
//   in its epilogue (gate 1) ->
//   RMSNorm (post_attention_layernorm) -> GEMM [up; gate] with the SwiGLU epilogue -> GEMM down_proj +
//   residual.
#include "capi_internal.h"
#include "ernie_synth.h"
#include "kernels.h"
#include <cmath>
#include <limits>
#include <memory>
#include <vector>

using namespace ernie_b200;
using namespace ernie_b200::capi;

namespace
{
constexpr int kTH = 3072, kTQ = 4096, kTKV = 1024, kTQkv = kTQ + 2 * kTKV, kTFfn = 9216, kTMaxLayers = 26;
constexpr int kTMaxBucket = 2048;
constexpr float kTEps = 1e-5f;

struct TextLayer
{
    __nv_bfloat16 *wqkv = nullptr; // [6144][3072]: q_proj, k_proj, v_proj rows
    __nv_bfloat16 *wo = nullptr;   // [3072][4096]
    __nv_bfloat16 *wug = nullptr;  // [18432][3072]: up_proj / gate_proj interleaved in 64-row groups
    __nv_bfloat16 *wdown = nullptr; // [3072][9216]
    float *gamma_attn = nullptr, *gamma_mlp = nullptr; // [3072]
};

struct TextWork
{
    int tokens = 0, precision = -1, planes = 1;
    int rows_pad = 0;
    float *x = nullptr, *qkv = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *cos_t = nullptr, *sin_t = nullptr;
    __nv_bfloat16 *a = nullptr, *h = nullptr;
    __nv_bfloat16 *qb = nullptr, *kb = nullptr, *vtb = nullptr; // BF16 mode: the tcgen05 attention's operands
    void *alloc = nullptr;
};
} // namespace

struct ernie_cuda_text_model
{
    ernie_cuda_context *ctx = nullptr;
    int num_layers = 0;
    std::vector<TextLayer> layers;
    float *ones = nullptr; // the residual epilogue's gate
    void *alloc = nullptr;
    uint64_t bytes = 0;
    TextWork work;
    // the prompt enhancer's LM head (allocated on first upload): final RMSNorm weight and lm_head
    float *head_norm = nullptr;
    __nv_bfloat16 *lm_head = nullptr; // [131072][3072]
    void *head_alloc = nullptr;
    bool head_loaded = false;
};

namespace
{
void free_work(TextWork &w)
{
    if (w.alloc) cudaFree(w.alloc);
    w = TextWork{};
}

int ensure_work(ernie_cuda_text_model *m, int tokens, int precision)
{
    TextWork &w = m->work;
    if (w.alloc && w.tokens == tokens && w.precision == precision) return ERNIE_CUDA_OK;
    free_work(w);
    w.tokens = tokens;
    w.precision = precision;
    w.planes = precision == ERNIE_PRECISION_FP32 ? 3 : 1;
    const size_t t = static_cast<size_t>(tokens);
    w.rows_pad = (tokens + 127) / 128 * 128;
    const size_t rp = static_cast<size_t>(w.rows_pad);
    Arena arena;
    arena.add(&w.qb, rp * kTQ);
    arena.add(&w.kb, rp * kTKV);
    arena.add(&w.vtb, rp * kTKV);
    arena.add(&w.x, t * kTH);
    arena.add(&w.qkv, t * kTQkv);
    arena.add(&w.q, t * kTQ);
    arena.add(&w.k, t * kTKV);
    arena.add(&w.v, t * kTKV);
    arena.add(&w.cos_t, t * 128);
    arena.add(&w.sin_t, t * 128);
    arena.add(&w.a, t * w.planes * kTQ);
    arena.add(&w.h, t * w.planes * kTFfn);
    const cudaError_t e = arena.allocate();
    if (e != cudaSuccess)
    {
        w = TextWork{};
        return from_cuda(e, "Allocate text encoder workspace");
    }
    w.alloc = arena.base;
    // the attention operands' padding rows / columns stay zero (keys past the prompt are masked, and V^T's
    // padding columns meet zero probabilities)
    const cudaError_t z = cudaMemset(w.qb, 0, rp * (kTQ + 2 * kTKV) * 2);
    if (z != cudaSuccess) return from_cuda(z, "Clear text encoder workspace");
    return ERNIE_CUDA_OK;
}

// Tile width of a BF16 GEMM: a short prompt's GEMMs (at most two 128-row tiles) stream their weights, and
// 128-wide tiles put twice as many SMs on the stream; longer prompts keep 256-wide (or paired) tiles, which
// read less B per FLOP (measured: 128-wide o_proj/down tiles were slower at 2048 tokens).
int text_block_n(int m, int, int)
{
    return m <= 256 ? 128 : 256;
}

// run_text_blocks on the model's device workspace: w.x [tokens][3072] in, updated in place.
int enqueue_layers(ernie_cuda_text_model *m, int count)
{
    TextWork &w = m->work;
    cudaStream_t s = m->ctx->stream;
    const int sms = m->ctx->num_sms, T = w.tokens;
    const bool fp32 = w.precision == ERNIE_PRECISION_FP32;
    const int splits = fp32 ? 3 : 1;
    const int bn_qkv = fp32 ? 128 : text_block_n(T, kTQkv, sms), bn_h = fp32 ? 128 : text_block_n(T, kTH, sms);
    const int bn_glu = fp32 ? 128 : text_block_n(T, 2 * kTFfn, sms);
    for (int l = 0; l < count; ++l)
    {
        const TextLayer &L = m->layers[static_cast<size_t>(l)];
        GemmEpilogueArgs f32;
        f32.out = w.qkv;
        f32.ldo = kTQkv;
        f32.error_flag = m->ctx->error_flag;
        ERNIE_LAUNCH(launch_norm_modulate(w.x, T, kTH, L.gamma_attn, nullptr, nullptr, kTEps, 0, w.a, fp32 ? 1 : 0, s),
                     "text input_layernorm");
        ERNIE_LAUNCH(launch_gemm(w.a, L.wqkv, T, kTQkv, kTH, splits, bn_qkv, Epilogue::F32Bias, f32, sms, s, fp32),
                     "text qkv projection");
        if (!fp32)
        {
            // BF16 mode: the tcgen05 flash attention, causal over 8 grouped K/V heads
            ERNIE_LAUNCH(launch_text_rope_bf16(w.qkv, w.cos_t, w.sin_t, T, w.rows_pad, w.qb, w.kb, w.vtb, s),
                         "text rotary");
            FlashOutput fo;
            fo.dst[0] = w.a;
            fo.rows_per_dest = T;
            fo.ld = kTQ;
            ERNIE_LAUNCH(launch_flash_tc(w.qb, w.kb, w.vtb, nullptr, T, w.rows_pad, T, 32, fo, m->ctx->error_flag, s,
                                         1, 8),
                         "text attention");
        }
        else
        {
        ERNIE_LAUNCH(launch_text_rope(w.qkv, w.cos_t, w.sin_t, T, w.q, w.k, w.v, s), "text rotary");
        AttentionF32Args at{};
        at.q = w.q;
        at.k = w.k;
        at.v = w.v;
        at.heads = 32;
        at.kv_heads = 8;
        at.mask_heads = 1;
        at.mask_rows = 1;
        at.nq = at.nk = at.kv_len = T;
        at.width = 128;
        at.q_head_stride = static_cast<long long>(T) * 128;
        at.kv_head_stride = static_cast<long long>(T) * 128;
        at.causal = 1;
        at.out_mode = 1;
        at.out_split3 = w.a;
        ERNIE_LAUNCH(launch_attention_f32(at, s), "text attention");
        }
        GemmEpilogueArgs res;
        res.resid = w.x;
        res.ldo = kTH; // the residual's row stride
        res.gate = m->ones;
        res.error_flag = m->ctx->error_flag;
        ERNIE_LAUNCH(launch_gemm(w.a, L.wo, T, kTH, kTQ, splits, bn_h, Epilogue::ResidGate, res, sms, s, fp32),
                     "text o_proj");
        ERNIE_LAUNCH(launch_norm_modulate(w.x, T, kTH, L.gamma_mlp, nullptr, nullptr, kTEps, 0, w.a, fp32 ? 1 : 0, s),
                     "text post_attention_layernorm");
        GemmEpilogueArgs glu;
        glu.h = w.h;
        glu.h_split3 = fp32 ? 1 : 0;
        glu.ffn = kTFfn;
        glu.silu = 1;
        glu.error_flag = m->ctx->error_flag;
        ERNIE_LAUNCH(launch_gemm(w.a, L.wug, T, 2 * kTFfn, kTH, splits, bn_glu, Epilogue::Geglu, glu, sms, s, fp32),
                     "text gate/up projection");
        ERNIE_LAUNCH(launch_gemm(w.h, L.wdown, T, kTH, kTFfn, splits, bn_h, Epilogue::ResidGate, res, sms, s, fp32),
                     "text down_proj");
    }
    return ERNIE_CUDA_OK;
}

int check_status(ernie_cuda_text_model *m)
{
    int flag = 0;
    ERNIE_CUDA(cudaMemcpyAsync(&flag, m->ctx->error_flag, sizeof(int), cudaMemcpyDeviceToHost, m->ctx->stream),
               "read status");
    ERNIE_CUDA(cudaStreamSynchronize(m->ctx->stream), "text encoder");
    if (flag) return fail(ERNIE_CUDA_ERROR, "Text encoder kernel protocol timeout (status " + std::to_string(flag) + ")");
    return ERNIE_CUDA_OK;
}
} // namespace

extern "C" int ernie_cuda_text_model_create(ernie_cuda_context *ctx, int num_layers, ernie_cuda_text_model **out)
{
    if (!ctx || !out) return fail(ERNIE_CUDA_ERROR, "null argument");
    *out = nullptr;
    if (num_layers < 1 || num_layers > kTMaxLayers) return fail(ERNIE_CUDA_ERROR, "Text encoder requires 1..26 layers");
    DeviceGuard guard(ctx->device);
    auto m = std::make_unique<ernie_cuda_text_model>();
    m->ctx = ctx;
    m->num_layers = num_layers;
    m->layers.resize(static_cast<size_t>(num_layers));
    Arena arena;
    for (auto &L : m->layers)
    {
        arena.add(&L.wqkv, static_cast<size_t>(kTQkv) * kTH);
        arena.add(&L.wo, static_cast<size_t>(kTH) * kTQ);
        arena.add(&L.wug, static_cast<size_t>(2 * kTFfn) * kTH);
        arena.add(&L.wdown, static_cast<size_t>(kTH) * kTFfn);
        arena.add(&L.gamma_attn, kTH);
        arena.add(&L.gamma_mlp, kTH);
    }
    arena.add(&m->ones, kTH);
    m->bytes = arena.bytes();
    const cudaError_t e = arena.allocate();
    if (e != cudaSuccess) return from_cuda(e, "Allocate text encoder weights");
    m->alloc = arena.base;
    std::vector<float> ones(kTH, 1.f);
    const cudaError_t c = cudaMemcpy(m->ones, ones.data(), kTH * 4, cudaMemcpyHostToDevice);
    if (c != cudaSuccess)
    {
        cudaFree(m->alloc);
        return from_cuda(c, "Upload text encoder constants");
    }
    *out = m.release();
    return ERNIE_CUDA_OK;
}

extern "C" int ernie_cuda_text_model_destroy(ernie_cuda_text_model *m)
{
    if (!m) return ERNIE_CUDA_OK;
    DeviceGuard guard(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    free_work(m->work);
    if (m->alloc) cudaFree(m->alloc);
    if (m->head_alloc) cudaFree(m->head_alloc);
    delete m;
    return ERNIE_CUDA_OK;
}

extern "C" int ernie_cuda_text_model_bytes(ernie_cuda_text_model *m, uint64_t *bytes)
{
    if (!m || !bytes) return fail(ERNIE_CUDA_ERROR, "null argument");
    *bytes = m->bytes;
    return ERNIE_CUDA_OK;
}

extern "C" int ernie_cuda_text_model_upload_layer(ernie_cuda_text_model *m, int layer,
                                                  const ernie_cuda_text_layer_weights *w)
{
    if (!m || !w || layer < 0 || layer >= m->num_layers) return fail(ERNIE_CUDA_ERROR, "Invalid text layer upload");
    if (!w->wq || !w->wk || !w->wv || !w->wo || !w->wgate || !w->wup || !w->wdown || !w->gamma_attn || !w->gamma_mlp)
        return fail(ERNIE_CUDA_ERROR, "Text layer weights must provide all 9 tensors");
    DeviceGuard guard(m->ctx->device);
    const TextLayer &L = m->layers[static_cast<size_t>(layer)];
    auto copy = [](void *dst, const void *src, size_t bytes) { return cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice); };
    ERNIE_CUDA(copy(L.wqkv, w->wq, size_t(kTQ) * kTH * 2), "upload q_proj");
    ERNIE_CUDA(copy(L.wqkv + size_t(kTQ) * kTH, w->wk, size_t(kTKV) * kTH * 2), "upload k_proj");
    ERNIE_CUDA(copy(L.wqkv + size_t(kTQ + kTKV) * kTH, w->wv, size_t(kTKV) * kTH * 2), "upload v_proj");
    ERNIE_CUDA(copy(L.wo, w->wo, size_t(kTH) * kTQ * 2), "upload o_proj");
    const size_t group = size_t(64) * kTH; // [up; gate] interleaved in 64-row groups (the gated epilogue's layout)
    for (int g = 0; g < kTFfn / 64; ++g)
    {
        ERNIE_CUDA(copy(L.wug + size_t(2 * g) * group, w->wup + size_t(g) * group, group * 2), "upload up_proj");
        ERNIE_CUDA(copy(L.wug + size_t(2 * g + 1) * group, w->wgate + size_t(g) * group, group * 2), "upload gate_proj");
    }
    ERNIE_CUDA(copy(L.wdown, w->wdown, size_t(kTH) * kTFfn * 2), "upload down_proj");
    ERNIE_CUDA(copy(L.gamma_attn, w->gamma_attn, kTH * 4), "upload input_layernorm");
    ERNIE_CUDA(copy(L.gamma_mlp, w->gamma_mlp, kTH * 4), "upload post_attention_layernorm");
    return ERNIE_CUDA_OK;
}

extern "C" int ernie_cuda_text_model_synthesize(ernie_cuda_text_model *m, uint64_t seed)
{
    if (!m) return fail(ERNIE_CUDA_ERROR, "null model");
    DeviceGuard guard(m->ctx->device);
    cudaStream_t s = m->ctx->stream;
    const float std = ERNIE_SYNTH_WEIGHT_STD;
    for (int l = 0; l < m->num_layers; ++l)
    {
        const TextLayer &L = m->layers[static_cast<size_t>(l)];
        auto sid = [l](int t) { return static_cast<uint64_t>(ERNIE_SYNTH_TEXT_STREAM(l, t)); };
        ERNIE_LAUNCH(launch_synth_bf16(seed, sid(ERNIE_SYNTH_TEXT_WQ), std, 0.f, kTQ, kTH, kTQ, 0, 0, L.wqkv, s), "synth");
        ERNIE_LAUNCH(launch_synth_bf16(seed, sid(ERNIE_SYNTH_TEXT_WK), std, 0.f, kTKV, kTH, kTKV, 0, kTQ, L.wqkv, s),
                     "synth");
        ERNIE_LAUNCH(launch_synth_bf16(seed, sid(ERNIE_SYNTH_TEXT_WV), std, 0.f, kTKV, kTH, kTKV, 0, kTQ + kTKV, L.wqkv,
                                       s),
                     "synth");
        ERNIE_LAUNCH(launch_synth_bf16(seed, sid(ERNIE_SYNTH_TEXT_WO), std, 0.f, kTH, kTQ, kTH, 0, 0, L.wo, s), "synth");
        ERNIE_LAUNCH(launch_synth_bf16(seed, sid(ERNIE_SYNTH_TEXT_WUP), std, 0.f, kTFfn, kTH, 64, 128, 0, L.wug, s),
                     "synth");
        ERNIE_LAUNCH(launch_synth_bf16(seed, sid(ERNIE_SYNTH_TEXT_WGATE), std, 0.f, kTFfn, kTH, 64, 128, 64, L.wug, s),
                     "synth");
        ERNIE_LAUNCH(launch_synth_bf16(seed, sid(ERNIE_SYNTH_TEXT_WDOWN), std, 0.f, kTH, kTFfn, kTH, 0, 0, L.wdown, s),
                     "synth");
        ERNIE_LAUNCH(launch_synth_f32_bf16(seed, sid(ERNIE_SYNTH_TEXT_GAMMA_ATTN), std, 1.f, kTH, L.gamma_attn, s),
                     "synth");
        ERNIE_LAUNCH(launch_synth_f32_bf16(seed, sid(ERNIE_SYNTH_TEXT_GAMMA_MLP), std, 1.f, kTH, L.gamma_mlp, s),
                     "synth");
    }
    return from_cuda(cudaStreamSynchronize(s), "synthesize text weights");
}

extern "C" int ernie_cuda_text_constants(const float *inv_freq, int bucket, float *cos_out, float *sin_out,
                                         float *mask)
{
    if (!inv_freq || !cos_out || !sin_out) return fail(ERNIE_CUDA_ERROR, "null argument");
    if (bucket < 1 || bucket > kTMaxBucket) return fail(ERNIE_CUDA_ERROR, "Text bucket must be in [1,2048]");
    for (int j = 0; j < 64; ++j)
        if (!std::isfinite(inv_freq[j]) || inv_freq[j] <= 0.f) return fail(ERNIE_CUDA_ERROR, "Invalid YaRN frequency");
    for (int t = 0; t < bucket; ++t)
    {
        float *c = cos_out + static_cast<size_t>(t) * 128, *s = sin_out + static_cast<size_t>(t) * 128;
        for (int j = 0; j < 64; ++j)
        {
            const float phase = float(t) * inv_freq[j]; // host code: -ffp-contract=off
            c[j] = c[j + 64] = std::cos(phase);
            s[j] = s[j + 64] = std::sin(phase);
        }
        if (mask)
            for (int k = 0; k < bucket; ++k)
                mask[static_cast<size_t>(t) * bucket + k] = k > t ? -std::numeric_limits<float>::max() : 0.f;
    }
    return ERNIE_CUDA_OK;
}

namespace
{
int run_text(ernie_cuda_text_model *m, const float *input, int bucket, const float *cos_t, const float *sin_t,
             int precision, int layers, float *out, cudaMemcpyKind in_kind, cudaMemcpyKind out_kind)
{
    if (!m || !input || !cos_t || !sin_t || !out) return fail(ERNIE_CUDA_ERROR, "null argument");
    if (bucket < 1 || bucket > kTMaxBucket) return fail(ERNIE_CUDA_ERROR, "Text bucket must be in [1,2048]");
    if (layers < 1 || layers > m->num_layers) return fail(ERNIE_CUDA_ERROR, "Text path requires 1..num_layers blocks");
    if (precision != ERNIE_PRECISION_BF16 && precision != ERNIE_PRECISION_FP32)
        return fail(ERNIE_CUDA_ERROR, "Unknown precision");
    DeviceGuard guard(m->ctx->device);
    ERNIE_TRY(ensure_work(m, bucket, precision));
    TextWork &w = m->work;
    cudaStream_t s = m->ctx->stream;
    const size_t t = static_cast<size_t>(bucket);
    ERNIE_CUDA(cudaMemcpyAsync(w.x, input, t * kTH * 4, in_kind, s), "text input");
    ERNIE_CUDA(cudaMemcpyAsync(w.cos_t, cos_t, t * 128 * 4, in_kind, s), "text cos");
    ERNIE_CUDA(cudaMemcpyAsync(w.sin_t, sin_t, t * 128 * 4, in_kind, s), "text sin");
    ERNIE_TRY(enqueue_layers(m, layers));
    ERNIE_CUDA(cudaMemcpyAsync(out, w.x, t * kTH * 4, out_kind, s), "text output");
    return check_status(m);
}
} // namespace

extern "C" int ernie_cuda_text_run_blocks(ernie_cuda_text_model *m, const float *input, int bucket, const float *cos_t,
                                          const float *sin_t, int precision, int layers, float *out)
{
    return run_text(m, input, bucket, cos_t, sin_t, precision, layers, out, cudaMemcpyHostToDevice,
                    cudaMemcpyDeviceToHost);
}

extern "C" int ernie_cuda_text_run_blocks_device(ernie_cuda_text_model *m, const float *input, int bucket,
                                                 const float *cos_t, const float *sin_t, int precision, int layers,
                                                 float *out)
{
    return run_text(m, input, bucket, cos_t, sin_t, precision, layers, out, cudaMemcpyDeviceToDevice,
                    cudaMemcpyDeviceToDevice);
}

// ---- prompt enhancer (PeSession, src/pe_session.cpp; enhance_prompt, src/prompt_enhancer.cpp) -------
// The PE is the same Mistral decoder layer (the PE block graph, src/pe_graph.cpp, is the text block plus
// past_k / past_v inputs) over the 26 layers of its own checkpoint, with an LM head of RMSNorm + a
// 131072 x 3072 projection tied to the embeddings (head.ncnn.param, tools/build_pe_model.py:100-105).
// Per chunk of 1..32 new tokens at the session's position: the layer as above, the rotated K / V rows
// appended to the layer's FP32 cache, and the FP32 attention of the chunk's queries over every cached key
// up to each query's own position (FP64 sums). Decode steps (up to 4 rows) and the LM head stream their
// weights through warp-per-row products (launch_gemv), captured once per session as a CUDA graph that reads
// the position from device memory; prefill chunks use the tensor-core GEMM. Every chunk's attention runs
// one CTA per (head, query row) with the cached keys split over its warps.
namespace
{
constexpr int kPeMaxRows = 32, kPeMaxCapacity = 4096, kPeVocab = 131072;

int ensure_head(ernie_cuda_text_model *m)
{
    if (m->head_alloc) return ERNIE_CUDA_OK;
    Arena arena;
    arena.add(&m->head_norm, kTH);
    arena.add(&m->lm_head, static_cast<size_t>(kPeVocab) * kTH);
    const cudaError_t e = arena.allocate();
    if (e != cudaSuccess) return from_cuda(e, "Allocate PE head");
    m->head_alloc = arena.base;
    return ERNIE_CUDA_OK;
}
} // namespace

struct ernie_cuda_pe_session
{
    ernie_cuda_text_model *model = nullptr;
    int capacity = 0, precision = 0, planes = 1, position = 0;
    bool valid = true;
    float *kcache = nullptr, *vcache = nullptr; // [layers][8][capacity][128]
    float *x = nullptr, *qkv = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *cos_t = nullptr, *sin_t = nullptr;
    __nv_bfloat16 *a = nullptr, *h = nullptr;
    float *hrow = nullptr, *logits = nullptr;
    __nv_bfloat16 *ha = nullptr;
    int *d_position = nullptr;                 // the device mirror of `position`
    cudaGraphExec_t step_graph[5] = {};        // captured decode steps of 1..4 rows
    void *alloc = nullptr;
};

namespace
{
// One chunk of `rows` tokens through every layer, appending to the caches at s->position.
int pe_enqueue(ernie_cuda_pe_session *ps, int rows)
{
    ernie_cuda_text_model *m = ps->model;
    cudaStream_t s = m->ctx->stream;
    const int sms = m->ctx->num_sms, T = rows, pos = ps->position;
    const bool fp32 = ps->precision == ERNIE_PRECISION_FP32;
    const int splits = fp32 ? 3 : 1;
    const int bn = fp32 ? 128 : text_block_n(T, kTH, sms);
    const size_t layer_cache = static_cast<size_t>(8) * ps->capacity * 128;
    // decode steps (a few rows) stream the weights through warp-per-row products; prefill chunks use the
    // tensor cores
    const bool gemv = T <= 4;
    auto product = [&](const __nv_bfloat16 *a, const __nv_bfloat16 *w, int n_rows, int k, GemvEpilogue epi,
                       float *out, int ldo) {
        GemvArgs g;
        g.a = a;
        g.rows = T;
        g.k = k;
        g.planes = ps->planes;
        g.w = w;
        g.n_rows = n_rows;
        g.out = out;
        g.ldo = ldo;
        g.h = ps->h;
        g.ffn = kTFfn;
        g.h_split3 = fp32 ? 1 : 0;
        return launch_gemv(g, epi, s);
    };
    for (int l = 0; l < m->num_layers; ++l)
    {
        const TextLayer &L = m->layers[static_cast<size_t>(l)];
        float *kc = ps->kcache + static_cast<size_t>(l) * layer_cache;
        float *vc = ps->vcache + static_cast<size_t>(l) * layer_cache;
        GemmEpilogueArgs f32;
        f32.out = ps->qkv;
        f32.ldo = kTQkv;
        f32.error_flag = m->ctx->error_flag;
        ERNIE_LAUNCH(launch_norm_modulate(ps->x, T, kTH, L.gamma_attn, nullptr, nullptr, kTEps, 0, ps->a, fp32 ? 1 : 0, s),
                     "PE input_layernorm");
        ERNIE_LAUNCH(gemv ? product(ps->a, L.wqkv, kTQkv, kTH, GemvEpilogue::F32Out, ps->qkv, kTQkv)
                          : launch_gemm(ps->a, L.wqkv, T, kTQkv, kTH, splits, bn, Epilogue::F32Bias, f32, sms, s, fp32),
                     "PE qkv projection");
        ERNIE_LAUNCH(launch_text_rope(ps->qkv, ps->cos_t, ps->sin_t, T, ps->q, ps->k, ps->v, s), "PE rotary");
        // the chunk's K / V rows of each of the 8 heads into the caches at rows pos..pos+T-1 (the position read
        // on the device, so that a captured decode step does not depend on it)
        ERNIE_LAUNCH(launch_pe_cache_append(ps->k, ps->v, T, kc, vc, ps->capacity, ps->d_position, s), "PE K/V cache");
        AttentionF32Args at{};
        at.q = ps->q;
        at.k = kc;
        at.v = vc;
        at.heads = 32;
        at.kv_heads = 8;
        at.mask_heads = 1;
        at.mask_rows = 1;
        at.nq = T;
        at.nk = at.kv_len = pos + T;
        at.width = 128;
        at.q_head_stride = static_cast<long long>(T) * 128;
        at.kv_head_stride = static_cast<long long>(ps->capacity) * 128;
        at.causal = 1;
        at.causal_offset = pos;
        // every chunk (at most 32 rows) on the key-split kernel: one CTA per (head, row) keeps all SMs busy
        at.decode = 1;
        at.position = ps->d_position;
        at.nk = ps->capacity; // the bound; the kernel reads kv_len from the position
        at.out_mode = fp32 ? 1 : 2; // the o_proj operand: three BF16 planes or BF16, token-major
        at.out_split3 = ps->a;
        ERNIE_LAUNCH(launch_attention_f32(at, s), "PE attention");
        GemmEpilogueArgs res;
        res.resid = ps->x;
        res.ldo = kTH;
        res.gate = m->ones;
        res.error_flag = m->ctx->error_flag;
        ERNIE_LAUNCH(gemv ? product(ps->a, L.wo, kTH, kTQ, GemvEpilogue::Resid, ps->x, kTH)
                          : launch_gemm(ps->a, L.wo, T, kTH, kTQ, splits, bn, Epilogue::ResidGate, res, sms, s, fp32),
                     "PE o_proj");
        ERNIE_LAUNCH(launch_norm_modulate(ps->x, T, kTH, L.gamma_mlp, nullptr, nullptr, kTEps, 0, ps->a, fp32 ? 1 : 0, s),
                     "PE post_attention_layernorm");
        GemmEpilogueArgs glu;
        glu.h = ps->h;
        glu.h_split3 = fp32 ? 1 : 0;
        glu.ffn = kTFfn;
        glu.silu = 1;
        glu.error_flag = m->ctx->error_flag;
        ERNIE_LAUNCH(gemv ? product(ps->a, L.wug, 2 * kTFfn, kTH, GemvEpilogue::SwiGLU, nullptr, 0)
                          : launch_gemm(ps->a, L.wug, T, 2 * kTFfn, kTH, splits,
                                        fp32 ? 128 : text_block_n(T, 2 * kTFfn, sms), Epilogue::Geglu, glu, sms, s,
                                        fp32),
                     "PE gate/up projection");
        ERNIE_LAUNCH(gemv ? product(ps->h, L.wdown, kTH, kTFfn, GemvEpilogue::Resid, ps->x, kTH)
                          : launch_gemm(ps->h, L.wdown, T, kTH, kTFfn, splits, bn, Epilogue::ResidGate, res, sms, s, fp32),
                     "PE down_proj");
    }
    ERNIE_LAUNCH(launch_pe_advance(ps->d_position, T, s), "PE position");
    return ERNIE_CUDA_OK;
}

// A decode step of `rows` rows, captured once per session and replayed (its inputs and the position are
// read from the session's device buffers).
int pe_step_graph(ernie_cuda_pe_session *ps, int rows)
{
    if (ps->step_graph[rows]) return ERNIE_CUDA_OK;
    cudaStream_t s = ps->model->ctx->stream;
    cudaGraph_t graph = nullptr;
    ERNIE_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "Begin PE capture");
    const int rc = pe_enqueue(ps, rows);
    const cudaError_t e = cudaStreamEndCapture(s, &graph);
    if (rc != ERNIE_CUDA_OK || e != cudaSuccess)
    {
        if (graph) cudaGraphDestroy(graph);
        return rc != ERNIE_CUDA_OK ? rc : from_cuda(e, "End PE capture");
    }
    const cudaError_t i = cudaGraphInstantiate(&ps->step_graph[rows], graph, 0);
    cudaGraphDestroy(graph);
    if (i != cudaSuccess)
    {
        ps->step_graph[rows] = nullptr;
        return from_cuda(i, "Instantiate PE step");
    }
    return ERNIE_CUDA_OK;
}

bool all_finite(const float *p, size_t n)
{
    for (size_t i = 0; i < n; ++i)
        if (!std::isfinite(p[i])) return false;
    return true;
}
} // namespace

extern "C" int ernie_cuda_text_model_upload_head(ernie_cuda_text_model *m, const float *norm, const uint16_t *lm_head)
{
    if (!m || !norm || !lm_head) return fail(ERNIE_CUDA_ERROR, "null argument");
    if (!all_finite(norm, kTH)) return fail(ERNIE_CUDA_ERROR, "PE head norm is not finite");
    DeviceGuard guard(m->ctx->device);
    ERNIE_TRY(ensure_head(m));
    ERNIE_CUDA(cudaMemcpy(m->head_norm, norm, kTH * 4, cudaMemcpyHostToDevice), "upload PE head norm");
    ERNIE_CUDA(cudaMemcpy(m->lm_head, lm_head, static_cast<size_t>(kPeVocab) * kTH * 2, cudaMemcpyHostToDevice),
               "upload PE lm_head");
    m->head_loaded = true;
    return ERNIE_CUDA_OK;
}

extern "C" int ernie_cuda_text_model_synthesize_head(ernie_cuda_text_model *m, uint64_t seed)
{
    if (!m) return fail(ERNIE_CUDA_ERROR, "null model");
    DeviceGuard guard(m->ctx->device);
    ERNIE_TRY(ensure_head(m));
    cudaStream_t s = m->ctx->stream;
    const float std = ERNIE_SYNTH_WEIGHT_STD;
    const uint64_t w = ERNIE_SYNTH_TEXT_STREAM(ERNIE_SYNTH_TEXT_HEAD_LAYER, 0);
    const uint64_t n = ERNIE_SYNTH_TEXT_STREAM(ERNIE_SYNTH_TEXT_HEAD_LAYER, 1);
    ERNIE_LAUNCH(launch_synth_bf16(seed, w, std, 0.f, kPeVocab, kTH, kPeVocab, 0, 0, m->lm_head, s), "synth");
    ERNIE_LAUNCH(launch_synth_f32_bf16(seed, n, std, 1.f, kTH, m->head_norm, s), "synth");
    ERNIE_CUDA(cudaStreamSynchronize(s), "synthesize PE head");
    m->head_loaded = true;
    return ERNIE_CUDA_OK;
}

extern "C" int ernie_cuda_pe_session_create(ernie_cuda_text_model *m, int capacity, int precision,
                                            ernie_cuda_pe_session **out)
{
    if (!m || !out) return fail(ERNIE_CUDA_ERROR, "null argument");
    *out = nullptr;
    if (capacity < 1 || capacity > kPeMaxCapacity)
        return fail(ERNIE_CUDA_ERROR, "PE requires 1..26 blocks and capacity 1..4096");
    if (precision != ERNIE_PRECISION_BF16 && precision != ERNIE_PRECISION_FP32)
        return fail(ERNIE_CUDA_ERROR, "Unknown precision");
    DeviceGuard guard(m->ctx->device);
    auto ps = std::make_unique<ernie_cuda_pe_session>();
    ps->model = m;
    ps->capacity = capacity;
    ps->precision = precision;
    ps->planes = precision == ERNIE_PRECISION_FP32 ? 3 : 1;
    const size_t cache = static_cast<size_t>(m->num_layers) * 8 * capacity * 128, r = kPeMaxRows;
    Arena arena;
    arena.add(&ps->kcache, cache);
    arena.add(&ps->vcache, cache);
    arena.add(&ps->x, r * kTH);
    arena.add(&ps->qkv, r * kTQkv);
    arena.add(&ps->q, r * kTQ);
    arena.add(&ps->k, r * kTKV);
    arena.add(&ps->v, r * kTKV);
    arena.add(&ps->cos_t, r * 128);
    arena.add(&ps->sin_t, r * 128);
    arena.add(&ps->a, r * ps->planes * kTQ);
    arena.add(&ps->h, r * ps->planes * kTFfn);
    arena.add(&ps->hrow, kTH);
    arena.add(&ps->ha, static_cast<size_t>(ps->planes) * kTH);
    arena.add(&ps->logits, kPeVocab);
    arena.add(&ps->d_position, 1);
    const cudaError_t e = arena.allocate();
    if (e != cudaSuccess) return from_cuda(e, "Allocate PE session");
    ps->alloc = arena.base;
    cudaError_t z = cudaMemset(ps->d_position, 0, sizeof(int));
    if (z == cudaSuccess) z = static_cast<cudaError_t>(prepare_gemv_kernels());
    if (z != cudaSuccess)
    {
        cudaFree(ps->alloc);
        return from_cuda(z, "Prepare PE session");
    }
    *out = ps.release();
    return ERNIE_CUDA_OK;
}

extern "C" int ernie_cuda_pe_session_destroy(ernie_cuda_pe_session *ps)
{
    if (!ps) return ERNIE_CUDA_OK;
    DeviceGuard guard(ps->model->ctx->device);
    cudaStreamSynchronize(ps->model->ctx->stream);
    for (cudaGraphExec_t g : ps->step_graph)
        if (g) cudaGraphExecDestroy(g);
    if (ps->alloc) cudaFree(ps->alloc);
    delete ps;
    return ERNIE_CUDA_OK;
}

extern "C" int ernie_cuda_pe_session_reset(ernie_cuda_pe_session *ps)
{
    if (!ps) return fail(ERNIE_CUDA_ERROR, "null argument");
    DeviceGuard guard(ps->model->ctx->device);
    ERNIE_CUDA(cudaMemsetAsync(ps->d_position, 0, sizeof(int), ps->model->ctx->stream), "reset PE position");
    ERNIE_CUDA(cudaStreamSynchronize(ps->model->ctx->stream), "reset PE position");
    ps->position = 0;
    ps->valid = true;
    return ERNIE_CUDA_OK;
}

extern "C" int ernie_cuda_pe_session_position(ernie_cuda_pe_session *ps, int *position)
{
    if (!ps || !position) return fail(ERNIE_CUDA_ERROR, "null argument");
    *position = ps->position;
    return ERNIE_CUDA_OK;
}

extern "C" int ernie_cuda_pe_session_append(ernie_cuda_pe_session *ps, const float *embedded, const float *cos,
                                            const float *sin, int rows, float *hidden)
{
    if (!ps || !embedded || !cos || !sin || !hidden) return fail(ERNIE_CUDA_ERROR, "null argument");
    if (!ps->valid) return fail(ERNIE_CUDA_ERROR, "PE session failed; reset before reuse");
    if (rows < 1 || rows > kPeMaxRows || rows > ps->capacity - ps->position)
        return fail(ERNIE_CUDA_ERROR, "PE token count or session capacity exceeded");
    const size_t r = static_cast<size_t>(rows);
    if (!all_finite(embedded, r * kTH) || !all_finite(cos, r * 128) || !all_finite(sin, r * 128))
        return fail(ERNIE_CUDA_ERROR, "PE tensor contains non-finite values");
    ernie_cuda_text_model *m = ps->model;
    DeviceGuard guard(m->ctx->device);
    cudaStream_t s = m->ctx->stream;
    ps->valid = false; // until this chunk has completed
    ERNIE_CUDA(cudaMemcpyAsync(ps->x, embedded, r * kTH * 4, cudaMemcpyHostToDevice, s), "PE input");
    ERNIE_CUDA(cudaMemcpyAsync(ps->cos_t, cos, r * 128 * 4, cudaMemcpyHostToDevice, s), "PE cos");
    ERNIE_CUDA(cudaMemcpyAsync(ps->sin_t, sin, r * 128 * 4, cudaMemcpyHostToDevice, s), "PE sin");
    if (rows <= 4)
    {
        ERNIE_TRY(pe_step_graph(ps, rows));
        ERNIE_CUDA(cudaGraphLaunch(ps->step_graph[rows], s), "PE step");
    }
    else
        ERNIE_TRY(pe_enqueue(ps, rows));
    ERNIE_CUDA(cudaMemcpyAsync(hidden, ps->x, r * kTH * 4, cudaMemcpyDeviceToHost, s), "PE hidden");
    ERNIE_TRY(check_status(m));
    ps->position += rows;
    ps->valid = true;
    return ERNIE_CUDA_OK;
}

extern "C" int ernie_cuda_pe_logits(ernie_cuda_pe_session *ps, const float *hidden, float *logits)
{
    if (!ps || !hidden || !logits) return fail(ERNIE_CUDA_ERROR, "null argument");
    ernie_cuda_text_model *m = ps->model;
    if (!m->head_loaded) return fail(ERNIE_CUDA_ERROR, "PE head not uploaded");
    if (!all_finite(hidden, kTH)) return fail(ERNIE_CUDA_ERROR, "PE tensor contains non-finite values");
    DeviceGuard guard(m->ctx->device);
    cudaStream_t s = m->ctx->stream;
    const bool fp32 = ps->precision == ERNIE_PRECISION_FP32;
    ERNIE_CUDA(cudaMemcpyAsync(ps->hrow, hidden, kTH * 4, cudaMemcpyHostToDevice, s), "PE head input");
    ERNIE_LAUNCH(launch_norm_modulate(ps->hrow, 1, kTH, m->head_norm, nullptr, nullptr, kTEps, 0, ps->ha, fp32 ? 1 : 0, s),
                 "PE head norm");
    GemvArgs g;
    g.a = ps->ha;
    g.rows = 1;
    g.k = kTH;
    g.planes = ps->planes;
    g.w = m->lm_head;
    g.n_rows = kPeVocab;
    g.out = ps->logits;
    g.ldo = kPeVocab;
    ERNIE_LAUNCH(launch_gemv(g, GemvEpilogue::F32Out, s), "PE lm_head");
    ERNIE_CUDA(cudaMemcpyAsync(logits, ps->logits, static_cast<size_t>(kPeVocab) * 4, cudaMemcpyDeviceToHost, s),
               "PE logits");
    return check_status(m);
}
