// C ABI of the VAE decoder and encoder (include/ernie_cuda.h, "VAE decoder", "VAE encoder"): resident
// weights addressed by their diffusers parameter names, a per-shape workspace, and the layer program replayed
// as one CUDA graph. Host orchestration only; the arithmetic is in vae.cu's kernels.
//
// The program follows the reference's exported decoder graph (AutoencoderKLFlux2 post_quant_conv +
// decoder as vae/head.ncnn.param lists it, run by decode_vae, src/vae.cpp:18-64): post_quant_conv 1x1
// 32->32, conv_in 3x3 32->512, mid block (resnet, single-head self-attention over all pixels, resnet),
// four up blocks of three resnets (512, 512, 256, 128 channels; 1x1 shortcut where the width changes)
// with nearest x2 upsampling + conv after the first three, GroupNorm(32, eps 1e-6) + Swish, conv_out
// 3x3 128->3. The RGB bytes follow rgb_image (src/pipeline.cpp:145-163).
//
// The encoder program follows encode_vae (src/image_encoder.cpp:28-72) over the wrapper its export traces
// (tools/export_vae_encoder.py:74-80): RGB bytes normalised as (v - 127.5f) * (1 / 127.5f), conv_in 3x3
// 3->128, four down blocks of two resnets (128, 256, 512, 512 channels) with a 3x3 stride-2 convolution
// (input padded by one zero row and column at the bottom and right) after the first three, the decoder's
// mid block, GroupNorm(32, eps 1e-6) + Swish, conv_out 3x3 512->64, quant_conv 1x1 keeping channels 0..31
// (the posterior's mode: mean), pixel_unshuffle(2) (packed) and BatchNorm(128, eps 1e-4, no affine, eval)
// (normalized).
#include "capi_internal.h"
#include "ernie_synth.h"
#include "kernels.h"
#include <algorithm>
#include <cmath>
#include <map>
#include <memory>
#include <string>
#include <tuple>
#include <vector>

using namespace ernie_b200;
using namespace ernie_b200::capi;

namespace
{
constexpr float kGroupNormEps = 1e-6f, kEncoderBnEps = 1e-4f;
constexpr int kGroups = 32, kMaxLatentSide = 256, kMaxImageSide = 2048;

struct ConvW
{
    int cin = 0, cout = 0, taps = 1, cin_pad = 0, cout_rows = 0;
    // conv_out: stored as the 1x1 convolution to its 9 taps x 3 outputs (rows t * 3 + c, padded to 32),
    // whose product a gather kernel sums over the 3x3 neighbourhood
    bool tap_expanded = false;
    // the encoder's conv_in: a 1x1 product over the 27 im2col columns of its RGB input (padded to 64)
    bool im2col = false;
    // Downsample2D: 3x3 stride 2 over the space-to-depth operand (ConvLaunch::stride2)
    bool stride2 = false;
    __nv_bfloat16 *w = nullptr; // [cout_rows][3 * dev_taps() * cin_pad]: hi, mid, lo planes
    float *bias = nullptr;      // [cout_rows]
    int inexact = 0;            // some weight is not a BF16 value (FP32-exact mode multiplies 3 planes)
    int dev_taps() const { return tap_expanded || im2col ? 1 : taps; }
};
struct NormW
{
    int c = 0;
    float *gamma = nullptr, *beta = nullptr;
};
struct ResnetW
{
    int cin = 0, cout = 0;
    NormW norm1, norm2;
    ConvW conv1, conv2, shortcut;
    bool has_shortcut = false;
};
struct AttnW
{
    NormW norm;
    ConvW qkv, out; // qkv rows: to_q, to_k, to_v
};

enum class Role
{
    ConvWeight,
    ConvBias,
    Vector, // GroupNorm gamma/beta, post_quant_conv weight and bias: FP32 copied as is
};

struct Param
{
    std::string name;
    std::vector<int> shape;
    Role role = Role::Vector;
    ConvW *conv = nullptr;
    int row_offset = 0;
    float **slot = nullptr; // Role::Vector tensors other than GroupNorm gamma/beta: the layout's pointer
    float *dst = nullptr;
    float scale = 0.f, offset = 0.f; // synthetic initialisation (include/ernie_synth.h)
    bool loaded = false;
    size_t count() const
    {
        size_t n = 1;
        for (int d : shape) n *= static_cast<size_t>(d);
        return n;
    }
};

// Builders of diffusers parameter tables (names, shapes, resident destinations).
struct LayoutBase
{
    std::vector<Param> params;
    std::vector<ConvW *> convs;
    std::vector<NormW *> norms;

    LayoutBase() = default;
    LayoutBase(const LayoutBase &) = delete; // params and convs point into the object
    LayoutBase &operator=(const LayoutBase &) = delete;

    void conv(const std::string &name, ConvW &c, int cin, int cout, int taps)
    {
        c.cin = cin;
        c.cout = cout;
        c.taps = taps;
        c.cin_pad = (cin + 63) / 64 * 64;
        c.cout_rows = cout < 16 ? 16 : cout;
        convs.push_back(&c);
        const int k = taps == 9 ? 3 : 1;
        add(name + ".weight", {cout, cin, k, k}, Role::ConvWeight, &c, 0, 1.f / std::sqrt(float(cin * taps)), 0.f);
        add(name + ".bias", {cout}, Role::ConvBias, &c, 0, 0.02f, 0.f);
    }
    void norm(const std::string &name, NormW &n, int c)
    {
        n.c = c;
        norms.push_back(&n);
        add(name + ".weight", {c}, Role::Vector, nullptr, 0, 0.1f, 1.f);
        add(name + ".bias", {c}, Role::Vector, nullptr, 0, 0.1f, 0.f);
    }
    void resnet(const std::string &name, ResnetW &r, int cin, int cout)
    {
        r.cin = cin;
        r.cout = cout;
        norm(name + ".norm1", r.norm1, cin);
        conv(name + ".conv1", r.conv1, cin, cout, 9);
        norm(name + ".norm2", r.norm2, cout);
        conv(name + ".conv2", r.conv2, cout, cout, 9);
        if (cin != cout)
        {
            r.has_shortcut = true;
            conv(name + ".conv_shortcut", r.shortcut, cin, cout, 1);
        }
    }
    // The mid block's single-head attention (prefix ends in "attentions.0."): GroupNorm, to_q/k/v as one
    // 1536-row 1x1 product, to_out.0.
    void attention(const std::string &prefix, AttnW &attn)
    {
        norm(prefix + "group_norm", attn.norm, 512);
        attn.qkv.cin = 512;
        attn.qkv.cout = 1536;
        attn.qkv.taps = 1;
        attn.qkv.cin_pad = 512;
        attn.qkv.cout_rows = 1536;
        convs.push_back(&attn.qkv);
        const float lin = 1.f / std::sqrt(512.f);
        const char *proj[3] = {"to_q", "to_k", "to_v"};
        for (int i = 0; i < 3; ++i)
        {
            const std::string base = prefix + proj[i];
            add(base + ".weight", {512, 512}, Role::ConvWeight, &attn.qkv, 512 * i, lin, 0.f);
            add(base + ".bias", {512}, Role::ConvBias, &attn.qkv, 512 * i, 0.02f, 0.f);
        }
        attn.out.cin = 512;
        attn.out.cout = 512;
        attn.out.taps = 1;
        attn.out.cin_pad = 512;
        attn.out.cout_rows = 512;
        convs.push_back(&attn.out);
        add(prefix + "to_out.0.weight", {512, 512}, Role::ConvWeight, &attn.out, 0, lin, 0.f);
        add(prefix + "to_out.0.bias", {512}, Role::ConvBias, &attn.out, 0, 0.02f, 0.f);
    }
    void add(const std::string &name, std::vector<int> shape, Role role, ConvW *c, int row_offset, float scale,
             float offset, float **slot = nullptr)
    {
        Param p;
        p.name = name;
        p.shape = std::move(shape);
        p.role = role;
        p.conv = c;
        p.row_offset = row_offset;
        p.scale = scale;
        p.offset = offset;
        p.slot = slot;
        params.push_back(std::move(p));
    }
};

// Diffusers parameter names and shapes of the decoder, in the order the reference graph runs them.
struct Layout : LayoutBase
{
    float *pq_w = nullptr, *pq_b = nullptr;
    ConvW conv_in;
    ResnetW mid[2];
    AttnW attn;
    ResnetW up[4][3];
    ConvW upsample[3];
    NormW norm_out;
    ConvW conv_out;

    static constexpr int kUpOut[4] = {512, 512, 256, 128};

    Layout()
    {
        add("post_quant_conv.weight", {32, 32, 1, 1}, Role::Vector, nullptr, 0, 1.f / std::sqrt(32.f), 0.f, &pq_w);
        add("post_quant_conv.bias", {32}, Role::Vector, nullptr, 0, 0.02f, 0.f, &pq_b);
        conv("decoder.conv_in", conv_in, 32, 512, 9);
        resnet("decoder.mid_block.resnets.0", mid[0], 512, 512);
        attention("decoder.mid_block.attentions.0.", attn);
        resnet("decoder.mid_block.resnets.1", mid[1], 512, 512);
        int c = 512;
        for (int i = 0; i < 4; ++i)
        {
            for (int j = 0; j < 3; ++j)
            {
                resnet("decoder.up_blocks." + std::to_string(i) + ".resnets." + std::to_string(j), up[i][j], c,
                       kUpOut[i]);
                c = kUpOut[i];
            }
            if (i < 3) conv("decoder.up_blocks." + std::to_string(i) + ".upsamplers.0.conv", upsample[i], c, c, 9);
        }
        norm("decoder.conv_norm_out", norm_out, 128);
        conv("decoder.conv_out", conv_out, 128, 3, 9);
        conv_out.tap_expanded = true;
        conv_out.cout_rows = 32;
    }
};

// Diffusers parameter names and shapes of the encoder (+ quant_conv, bn), in execution order.
struct EncoderLayout : LayoutBase
{
    ConvW conv_in;
    ResnetW down[4][2];
    ConvW downsample[3];
    ResnetW mid[2];
    AttnW attn;
    NormW norm_out;
    ConvW conv_out;
    float *quant_w = nullptr, *quant_b = nullptr, *bn_mean = nullptr, *bn_var = nullptr;

    static constexpr int kDownOut[4] = {128, 256, 512, 512};

    EncoderLayout()
    {
        conv("encoder.conv_in", conv_in, 3, 128, 9);
        conv_in.im2col = true;
        int c = 128;
        for (int i = 0; i < 4; ++i)
        {
            for (int j = 0; j < 2; ++j)
            {
                resnet("encoder.down_blocks." + std::to_string(i) + ".resnets." + std::to_string(j), down[i][j], c,
                       kDownOut[i]);
                c = kDownOut[i];
            }
            if (i < 3)
            {
                conv("encoder.down_blocks." + std::to_string(i) + ".downsamplers.0.conv", downsample[i], c, c, 9);
                downsample[i].stride2 = true;
            }
        }
        resnet("encoder.mid_block.resnets.0", mid[0], 512, 512);
        attention("encoder.mid_block.attentions.0.", attn);
        resnet("encoder.mid_block.resnets.1", mid[1], 512, 512);
        norm("encoder.conv_norm_out", norm_out, 512);
        conv("encoder.conv_out", conv_out, 512, 64, 9);
        conv_out.cout_rows = 128; // the 128-channel tile; rows 64..127 stay zero
        add("quant_conv.weight", {64, 64, 1, 1}, Role::Vector, nullptr, 0, 1.f / std::sqrt(64.f), 0.f, &quant_w);
        add("quant_conv.bias", {64}, Role::Vector, nullptr, 0, 0.02f, 0.f, &quant_b);
        add("bn.running_mean", {128}, Role::Vector, nullptr, 0, 0.02f, 0.f, &bn_mean);
        add("bn.running_var", {128}, Role::Vector, nullptr, 0, 0.1f, 1.f, &bn_var);
    }
};

// Buffers of one decode (encode) shape and precision: the decoder's levels L0..L3 at 1x, 2x, 4x, 8x the
// latent side, the encoder's at 1x, 1/2, 1/4, 1/8 the image side.
struct Plan
{
    int h0 = 0, w0 = 0, precision = 0, planes = 1;
    int n = 0, npad = 0; // attention tokens (h0 * w0) and their padding to 256
    float *input = nullptr, *x = nullptr, *h1 = nullptr, *sc = nullptr, *qkv = nullptr, *s = nullptr, *o = nullptr;
    float *scale = nullptr, *shift = nullptr, *decoded = nullptr;
    __nv_bfloat16 *a = nullptr, *a2 = nullptr, *q = nullptr, *k = nullptr, *vt = nullptr, *p = nullptr;
    double2 *stats_x = nullptr, *stats_h = nullptr;
    uint8_t *rgb = nullptr;
    uint8_t *rgb_in = nullptr;                                      // encoder input
    float *mean = nullptr, *packed = nullptr, *normalized = nullptr; // encoder outputs
    int *nonfinite = nullptr;
    void *alloc = nullptr;
    cudaGraphExec_t graph = nullptr;
    int launches = 0;
    size_t bytes = 0;
};

size_t pixels_of(int h, int w) { return static_cast<size_t>(h) * static_cast<size_t>(w); }

// Resident weights of one layout, their staging buffers and the current shape's plan.
template <class L> struct VaeModel
{
    ernie_cuda_context *ctx = nullptr;
    L layout;
    void *alloc = nullptr;
    float *staging = nullptr, *staging2 = nullptr;
    int *d_inexact = nullptr;
    uint64_t bytes = 0;
    std::unique_ptr<Plan> plan;
};
} // namespace

struct ernie_cuda_vae : VaeModel<Layout>
{
};
struct ernie_cuda_vae_encoder : VaeModel<EncoderLayout>
{
};

namespace
{
void free_plan(Plan *p)
{
    if (!p) return;
    if (p->graph) cudaGraphExecDestroy(p->graph);
    if (p->alloc) cudaFree(p->alloc);
}

// Mid-block attention (p.n tokens) and GroupNorm buffers, common to both programs.
void add_common(Arena &arena, Plan &p, int num_sms)
{
    p.npad = (p.n + 255) / 256 * 256;
    const int slots_max = 8 * num_sms; // GroupNorm partial slots per group (8 per conv CTA)
    arena.add(&p.qkv, static_cast<size_t>(p.n) * 1536);
    arena.add(&p.q, static_cast<size_t>(p.planes) * 512 * p.npad);
    arena.add(&p.k, static_cast<size_t>(p.planes) * 512 * p.npad);
    arena.add(&p.vt, static_cast<size_t>(p.planes) * 512 * p.npad);
    arena.add(&p.s, static_cast<size_t>(p.n) * p.npad);
    arena.add(&p.p, static_cast<size_t>(p.planes) * p.n * p.npad);
    arena.add(&p.o, static_cast<size_t>(p.n) * 512);
    arena.add(&p.stats_x, static_cast<size_t>(kGroups) * slots_max);
    arena.add(&p.stats_h, static_cast<size_t>(kGroups) * slots_max);
    arena.add(&p.scale, 512);
    arena.add(&p.shift, 512);
    arena.add(&p.nonfinite, 1);
}

int allocate_plan(ernie_cuda_context *ctx, Arena &arena, std::unique_ptr<Plan> &plan, std::unique_ptr<Plan> &out)
{
    Plan &p = *plan;
    p.bytes = arena.bytes();
    const cudaError_t e = arena.allocate();
    if (e != cudaSuccess) return from_cuda(e, "Allocate VAE workspace");
    p.alloc = arena.base;
    // K's rows and V^T's columns past the last token stay zero: their scores and products vanish
    cudaError_t z = cudaMemsetAsync(p.k, 0, static_cast<size_t>(p.planes) * 512 * p.npad * 2, ctx->stream);
    if (z == cudaSuccess) z = cudaMemsetAsync(p.vt, 0, static_cast<size_t>(p.planes) * 512 * p.npad * 2, ctx->stream);
    if (z == cudaSuccess) z = cudaStreamSynchronize(ctx->stream);
    if (z != cudaSuccess)
    {
        free_plan(plan.get());
        return from_cuda(z, "Clear VAE workspace");
    }
    out = std::move(plan);
    return ERNIE_CUDA_OK;
}

// Decoder: h0 x w0 is the unpacked latent.
int plan_create(ernie_cuda_vae *v, int h0, int w0, int precision, std::unique_ptr<Plan> &out)
{
    auto plan = std::make_unique<Plan>();
    Plan &p = *plan;
    p.h0 = h0;
    p.w0 = w0;
    p.precision = precision;
    p.planes = precision == ERNIE_PRECISION_FP32 ? 3 : 1;
    p.n = h0 * w0;
    const size_t px0 = pixels_of(h0, w0), top = 64 * px0;
    Arena arena;
    arena.add(&p.input, 32 * px0);
    arena.add(&p.x, 16384 * px0);
    arena.add(&p.h1, 8192 * px0);
    arena.add(&p.sc, 8192 * px0);
    arena.add(&p.a, static_cast<size_t>(p.planes) * 16384 * px0);
    arena.add(&p.a2, static_cast<size_t>(p.planes) * 16384 * px0); // shortcut-convolution operand
    arena.add(&p.decoded, 3 * top);
    arena.add(&p.rgb, 3 * top);
    add_common(arena, p, v->ctx->num_sms);
    return allocate_plan(v->ctx, arena, plan, out);
}

// Encoder: h0 x w0 is the image (multiples of 16). Largest tensors: 128 channels at full size (level 0),
// 256 x 1/4 for the level-1 shortcut, the level-0 stride-2 operand (4 phases x 128 channels x 1/4).
int plan_create(ernie_cuda_vae_encoder *v, int h0, int w0, int precision, std::unique_ptr<Plan> &out)
{
    auto plan = std::make_unique<Plan>();
    Plan &p = *plan;
    p.h0 = h0;
    p.w0 = w0;
    p.precision = precision;
    p.planes = precision == ERNIE_PRECISION_FP32 ? 3 : 1;
    p.n = (h0 / 8) * (w0 / 8);
    const size_t px = pixels_of(h0, w0);
    Arena arena;
    arena.add(&p.rgb_in, 3 * px);
    arena.add(&p.x, 128 * px);
    arena.add(&p.h1, 128 * px);
    arena.add(&p.sc, 64 * px);
    arena.add(&p.a, static_cast<size_t>(p.planes) * 128 * px);
    arena.add(&p.a2, static_cast<size_t>(p.planes) * 32 * px);
    arena.add(&p.mean, 32 * px / 64);
    arena.add(&p.packed, 128 * px / 256);
    arena.add(&p.normalized, 128 * px / 256);
    add_common(arena, p, v->ctx->num_sms);
    return allocate_plan(v->ctx, arena, plan, out);
}

// ---- the decoder program -----------------------------------------------------------------------------
// Kernel classes of the profile (ernie_cuda_vae_profile): algorithmic FLOPs for the tensor-core classes,
// algorithmic HBM bytes for the others.
enum ProfileClass : int
{
    kProfConv = 0,      // decoder convolutions and the attention's 1x1 projections (FLOPs)
    kProfAttnGemm = 1,  // attention scores q k^T and probabilities x v (FLOPs)
    kProfSoftmax = 2,   // bytes
    kProfNorm = 3,      // GroupNorm statistics + apply (+ Swish) (bytes)
    kProfUpsample = 4,  // bytes (decoder: nearest x2 upsampling; encoder: the stride-2 operand)
    kProfOther = 5,     // post_quant_conv input, attention split, operand conversions (bytes)
    kProfClasses = 6
};

// Events around every launch of an eager run, summed per class after the run.
struct Profiler
{
    std::vector<cudaEvent_t> events;
    std::vector<int> classes;
    std::vector<double> work;
    size_t used = 0;
    int begin(cudaStream_t stream)
    {
        if (events.size() < 2 * (used + 1))
        {
            cudaEvent_t a = nullptr, b = nullptr;
            ERNIE_CUDA(cudaEventCreate(&a), "profile event");
            ERNIE_CUDA(cudaEventCreate(&b), "profile event");
            events.push_back(a);
            events.push_back(b);
        }
        ERNIE_CUDA(cudaEventRecord(events[2 * used], stream), "profile event");
        return ERNIE_CUDA_OK;
    }
    int end(cudaStream_t stream, int cls, double w)
    {
        ERNIE_CUDA(cudaEventRecord(events[2 * used + 1], stream), "profile event");
        if (classes.size() <= used)
        {
            classes.push_back(cls);
            work.push_back(w);
        }
        ++used;
        return ERNIE_CUDA_OK;
    }
    ~Profiler()
    {
        for (cudaEvent_t e : events) cudaEventDestroy(e);
    }
};

struct Program
{
    ernie_cuda_context *ctx;
    Plan &p;
    cudaStream_t stream;
    int sms;
    Profiler *prof = nullptr;
    int slots_x = 0, slots_h = 0; // GroupNorm partial slots written by the last producer of x / h1
    bool fp32() const { return p.planes == 3; }

    // One operation of `kernels` launches, of profile class `cls` and algorithmic work `work`.
    template <class F> int op(int cls, double work, int kernels, const char *what, F &&launch)
    {
        if (prof) ERNIE_TRY(prof->begin(stream));
        ERNIE_LAUNCH(launch(), what);
        p.launches += kernels;
        if (prof) ERNIE_TRY(prof->end(stream, cls, work));
        return ERNIE_CUDA_OK;
    }
    double bytes_bf16(double elements) const { return 2.0 * p.planes * elements; }

    int conv(const ConvW &c, const __nv_bfloat16 *a, int h, int w, const ConvArgs &epi)
    {
        ConvLaunch l;
        l.a = a;
        l.a_planes = p.planes;
        l.b = c.w;
        l.b_planes = fp32() && c.inexact ? 3 : 1;
        l.b_row = 3LL * c.dev_taps() * c.cin_pad;
        l.cout_rows = c.cout_rows;
        l.height = h;
        l.width = w;
        l.cin = c.cin_pad;
        l.taps = c.dev_taps();
        l.cout = c.cout_rows;
        l.stride2 = c.stride2 ? 1 : 0;
        ConvArgs args = epi;
        args.bias = c.tap_expanded ? nullptr : c.bias; // conv_out's bias is added by the gather
        args.error_flag = ctx->error_flag;
        const double flops = 2.0 * pixels_of(h, w) * c.cout * c.cin * c.taps;
        if (args.stats) (args.stats == p.stats_x ? slots_x : slots_h) = conv_stat_slots(l, sms);
        return op(kProfConv, flops, 1, "VAE convolution", [&] { return launch_conv(l, args, sms, stream); });
    }
    // GroupNorm(32) of x (statistics from its producer) + optional Swish -> operand `a`
    // (raw: also x itself as operand planes, from the same read)
    int group_norm(const NormW &n, const float *x, const double2 *stats, int h, int w, bool silu,
                   __nv_bfloat16 *raw = nullptr)
    {
        const int cpg = n.c / kGroups;
        const long long pixels = static_cast<long long>(pixels_of(h, w));
        const double elements = static_cast<double>(pixels) * n.c;
        return op(kProfNorm, 4.0 * elements + bytes_bf16(elements) * (raw ? 2 : 1), 2, "GroupNorm", [&] {
            const int e = launch_gn_finalize(stats, stats == p.stats_x ? slots_x : slots_h, pixels * cpg, cpg, n.gamma,
                                             n.beta, kGroupNormEps, p.scale, p.shift, stream);
            return e != 0 ? e
                          : launch_gn_apply(x, pixels, n.c, p.scale, p.shift, silu ? 1 : 0, p.a, p.planes, stream, raw);
        });
    }
    ConvArgs writes_x(int cout, const float *resid)
    {
        ConvArgs e;
        e.out = p.x;
        e.ldo = cout;
        e.resid = resid;
        e.stats = p.stats_x;
        e.cpg = cout / kGroups;
        return e;
    }
    int to_operand(const float *src, long long rows, int cols)
    {
        const double elements = static_cast<double>(rows) * cols;
        return op(kProfOther, 4.0 * elements + bytes_bf16(elements), 1, "operand",
                  [&] { return launch_to_operand(src, rows, cols, p.a, fp32() ? 1 : 0, stream); });
    }
    // ResnetBlock2D: x <- shortcut(x) + conv2(swish(norm2(conv1(swish(norm1(x))))))
    int resnet(const ResnetW &r, int h, int w)
    {
        const float *resid = p.x;
        ERNIE_TRY(group_norm(r.norm1, p.x, p.stats_x, h, w, true, r.has_shortcut ? p.a2 : nullptr));
        if (r.has_shortcut)
        {
            ConvArgs e;
            e.out = p.sc;
            e.ldo = r.cout;
            ERNIE_TRY(conv(r.shortcut, p.a2, h, w, e));
            resid = p.sc;
        }
        ConvArgs e1;
        e1.out = p.h1;
        e1.ldo = r.cout;
        e1.stats = p.stats_h;
        e1.cpg = r.cout / kGroups;
        ERNIE_TRY(conv(r.conv1, p.a, h, w, e1));
        ERNIE_TRY(group_norm(r.norm2, p.h1, p.stats_h, h, w, true));
        return conv(r.conv2, p.a, h, w, writes_x(r.cout, resid));
    }
    // Attention block over all h*w pixels (one head of 512): x <- x + out(softmax(q k^T / sqrt 512) v)
    int attention(const AttnW &at, int h, int w)
    {
        const int n = p.n, npad = p.npad;
        ERNIE_TRY(group_norm(at.norm, p.x, p.stats_x, h, w, false));
        ConvArgs eq;
        eq.out = p.qkv;
        eq.ldo = 1536;
        ERNIE_TRY(conv(at.qkv, p.a, h, w, eq));
        ERNIE_TRY(op(kProfOther, 4.0 * n * 1536 + bytes_bf16(1536.0 * n), 2, "attention split",
                     [&] { return launch_attention_split(p.qkv, n, p.q, p.k, p.vt, npad, p.planes, stream); }));
        ConvLaunch ls;
        ls.a = p.q;
        ls.a_planes = p.planes;
        ls.b = p.k;
        ls.b_planes = p.planes;
        ls.b_row = static_cast<long long>(p.planes) * 512;
        ls.cout_rows = npad;
        ls.height = 1;
        ls.width = n;
        ls.cin = 512;
        ls.taps = 1;
        ls.cout = npad;
        ConvArgs es;
        es.out = p.s;
        es.ldo = npad;
        es.error_flag = ctx->error_flag;
        const double gemm = 2.0 * n * n * 512;
        ERNIE_TRY(op(kProfAttnGemm, gemm, 1, "attention scores", [&] { return launch_conv(ls, es, sms, stream); }));
        ERNIE_TRY(op(kProfSoftmax, 4.0 * n * n + bytes_bf16(static_cast<double>(n) * npad), 1, "attention softmax", [&] {
            return launch_softmax_rows(p.s, n, npad, n, 1.f / std::sqrt(512.f), p.p, npad, p.planes, stream);
        }));
        ConvLaunch lo;
        lo.a = p.p;
        lo.a_planes = p.planes;
        lo.b = p.vt;
        lo.b_planes = p.planes;
        lo.b_row = static_cast<long long>(p.planes) * npad;
        lo.cout_rows = 512;
        lo.height = 1;
        lo.width = n;
        lo.cin = npad;
        lo.taps = 1;
        lo.cout = 512;
        ConvArgs eo;
        eo.out = p.o;
        eo.ldo = 512;
        eo.error_flag = ctx->error_flag;
        ERNIE_TRY(op(kProfAttnGemm, gemm, 1, "attention values", [&] { return launch_conv(lo, eo, sms, stream); }));
        ERNIE_TRY(to_operand(p.o, n, 512));
        return conv(at.out, p.a, h, w, writes_x(512, p.x));
    }
    int run(const Layout &L)
    {
        int h = p.h0, w = p.w0;
        const double px = static_cast<double>(pixels_of(h, w));
        ERNIE_TRY(op(kProfOther, 4.0 * 32 * px + bytes_bf16(64.0 * px), 1, "post_quant_conv", [&] {
            return launch_vae_input(p.input, static_cast<long long>(px), L.pq_w, L.pq_b, p.a, p.planes, stream);
        }));
        ERNIE_TRY(conv(L.conv_in, p.a, h, w, writes_x(512, nullptr)));
        ERNIE_TRY(resnet(L.mid[0], h, w));
        ERNIE_TRY(attention(L.attn, h, w));
        ERNIE_TRY(resnet(L.mid[1], h, w));
        for (int i = 0; i < 4; ++i)
        {
            for (int j = 0; j < 3; ++j) ERNIE_TRY(resnet(L.up[i][j], h, w));
            if (i == 3) break;
            const int c = L.up[i][2].cout;
            const double elements = static_cast<double>(pixels_of(h, w)) * c;
            ERNIE_TRY(op(kProfUpsample, 4.0 * elements + bytes_bf16(4.0 * elements), 1, "upsample",
                         [&] { return launch_upsample(p.x, h, w, c, p.a, p.planes, stream); }));
            h *= 2;
            w *= 2;
            ERNIE_TRY(conv(L.upsample[i], p.a, h, w, writes_x(c, nullptr)));
        }
        ERNIE_TRY(group_norm(L.norm_out, p.x, p.stats_x, h, w, true));
        // conv_out: the 1x1 product to 9 taps x 3 outputs (into h1, free here), then the 3x3 tap sum
        ConvArgs e;
        e.out = p.h1;
        e.ldo = 32;
        ERNIE_TRY(conv(L.conv_out, p.a, h, w, e));
        const double px_top = static_cast<double>(pixels_of(h, w));
        return op(kProfOther, px_top * (32 * 4 + 3 * 4 + 3), 1, "conv_out gather", [&] {
            return launch_conv_out_gather(p.h1, h, w, L.conv_out.bias, p.decoded, p.rgb, p.nonfinite, stream);
        });
    }
    int run(const EncoderLayout &L)
    {
        int h = p.h0, w = p.w0;
        const double px = static_cast<double>(pixels_of(h, w));
        ERNIE_TRY(op(kProfOther, 3.0 * px + bytes_bf16(64.0 * px), 1, "encoder input",
                     [&] { return launch_rgb_im2col(p.rgb_in, h, w, p.a, p.planes, stream); }));
        ERNIE_TRY(conv(L.conv_in, p.a, h, w, writes_x(128, nullptr)));
        for (int i = 0; i < 4; ++i)
        {
            for (int j = 0; j < 2; ++j) ERNIE_TRY(resnet(L.down[i][j], h, w));
            if (i == 3) break;
            const int c = L.down[i][1].cout;
            const double elements = static_cast<double>(pixels_of(h, w)) * c;
            ERNIE_TRY(op(kProfUpsample, 4.0 * elements + bytes_bf16(elements), 1, "downsample operand",
                         [&] { return launch_s2d_operand(p.x, h, w, c, p.a, p.planes, stream); }));
            h /= 2;
            w /= 2;
            ERNIE_TRY(conv(L.downsample[i], p.a, h, w, writes_x(c, nullptr)));
        }
        ERNIE_TRY(resnet(L.mid[0], h, w));
        ERNIE_TRY(attention(L.attn, h, w));
        ERNIE_TRY(resnet(L.mid[1], h, w));
        ERNIE_TRY(group_norm(L.norm_out, p.x, p.stats_x, h, w, true));
        ConvArgs e;
        e.out = p.h1;
        e.ldo = L.conv_out.cout_rows;
        ERNIE_TRY(conv(L.conv_out, p.a, h, w, e));
        const double px_mean = static_cast<double>(pixels_of(h, w));
        return op(kProfOther, px_mean * (64 * 4 + 3 * 32 * 4), 1, "quant_conv + unshuffle + batch norm", [&] {
            return launch_encoder_output(p.h1, L.conv_out.cout_rows, h, w, L.quant_w, L.quant_b, L.bn_mean, L.bn_var,
                                         kEncoderBnEps, p.mean, p.packed, p.normalized, p.nonfinite, stream);
        });
    }
};

bool vae_shape_ok(int width, int height)
{
    return width >= 1 && height >= 1 && width <= kMaxLatentSide && height <= kMaxLatentSide &&
           width * height <= kSoftmaxMaxRow;
}

// The encoder's images: sides multiples of 16 (an even mean for pixel_unshuffle), at most 2048, and a mid
// block of at most kSoftmaxMaxRow tokens.
bool encoder_shape_ok(int width, int height)
{
    return width >= 16 && height >= 16 && width % 16 == 0 && height % 16 == 0 && width <= kMaxImageSide &&
           height <= kMaxImageSide && (width / 8) * (height / 8) <= kSoftmaxMaxRow;
}

template <class V> int find_param(V *v, const char *name)
{
    for (size_t i = 0; i < v->layout.params.size(); ++i)
        if (v->layout.params[i].name == name) return static_cast<int>(i);
    return -1;
}

// Moves staged FP32 values (device) of parameter i to their resident form.
template <class V> int place(V *v, Param &prm)
{
    cudaStream_t stream = v->ctx->stream;
    if (prm.role == Role::Vector)
    {
        ERNIE_CUDA(cudaMemcpyAsync(prm.dst, v->staging, prm.count() * 4, cudaMemcpyDeviceToDevice, stream), "place");
    }
    else if (prm.role == Role::ConvBias)
    {
        ERNIE_CUDA(cudaMemcpyAsync(prm.conv->bias + prm.row_offset, v->staging, prm.count() * 4,
                                   cudaMemcpyDeviceToDevice, stream),
                   "place bias");
    }
    else
    {
        ConvW &c = *prm.conv;
        const int cout = prm.shape[0];
        const int rows = prm.row_offset == 0 && cout == c.cout ? c.cout_rows : cout;
        ERNIE_CUDA(cudaMemsetAsync(v->d_inexact, 0, sizeof(int), stream), "clear flag");
        if (c.tap_expanded)
        {
            ERNIE_LAUNCH(launch_expand_taps(v->staging, c.cout, c.cin, v->staging2, stream), "expand taps");
            ERNIE_LAUNCH(launch_conv_weight_prep(v->staging2, 9 * c.cout, c.cin, 1, c.cout_rows, c.cin_pad, c.w,
                                                 v->d_inexact, stream),
                         "prepare weights");
        }
        else if (c.im2col)
        {
            ERNIE_LAUNCH(launch_taps_inner(v->staging, c.cout, c.cin, c.taps, v->staging2, stream), "im2col weights");
            ERNIE_LAUNCH(launch_conv_weight_prep(v->staging2, c.cout, c.taps * c.cin, 1, c.cout_rows, c.cin_pad, c.w,
                                                 v->d_inexact, stream),
                         "prepare weights");
        }
        else
            ERNIE_LAUNCH(launch_conv_weight_prep(v->staging, cout, c.cin, c.taps, rows, c.cin_pad,
                                                 c.w + static_cast<size_t>(prm.row_offset) * 3 * c.taps * c.cin_pad,
                                                 v->d_inexact, stream),
                         "prepare weights");
        int inexact = 0;
        ERNIE_CUDA(cudaMemcpyAsync(&inexact, v->d_inexact, sizeof(int), cudaMemcpyDeviceToHost, stream), "read flag");
        ERNIE_CUDA(cudaStreamSynchronize(stream), "prepare weights");
        c.inexact |= inexact;
    }
    prm.loaded = true;
    return ERNIE_CUDA_OK;
}

template <class V> void drop_plan(V *v)
{
    if (v->plan)
    {
        free_plan(v->plan.get());
        v->plan.reset();
    }
}

template <class V> int ensure_plan(V *v, int width, int height, int precision)
{
    if (v->plan && v->plan->w0 == width && v->plan->h0 == height && v->plan->precision == precision)
        return ERNIE_CUDA_OK;
    drop_plan(v);
    std::unique_ptr<Plan> plan;
    ERNIE_TRY(plan_create(v, height, width, precision, plan));
    // capture the whole program once; every later call of this shape replays it
    Program prog{v->ctx, *plan, v->ctx->stream, v->ctx->num_sms};
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamBeginCapture(v->ctx->stream, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess)
    {
        free_plan(plan.get());
        return from_cuda(e, "Begin VAE capture");
    }
    const int rc = prog.run(v->layout);
    e = cudaStreamEndCapture(v->ctx->stream, &graph);
    if (rc != ERNIE_CUDA_OK || e != cudaSuccess)
    {
        if (graph) cudaGraphDestroy(graph);
        free_plan(plan.get());
        return rc != ERNIE_CUDA_OK ? rc : from_cuda(e, "End VAE capture");
    }
    e = cudaGraphInstantiate(&plan->graph, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess)
    {
        free_plan(plan.get());
        return from_cuda(e, "Instantiate VAE graph");
    }
    v->plan = std::move(plan);
    return ERNIE_CUDA_OK;
}

template <class V> int check_loaded(V *v)
{
    for (const auto &prm : v->layout.params)
        if (!prm.loaded) return fail(ERNIE_CUDA_ERROR, "VAE tensor not uploaded: " + prm.name);
    return ERNIE_CUDA_OK;
}

template <class V> int run_graph(V *v, int width, int height, int precision)
{
    ERNIE_TRY(check_loaded(v));
    ERNIE_TRY(ensure_plan(v, width, height, precision));
    Plan &p = *v->plan;
    ERNIE_CUDA(cudaMemsetAsync(p.nonfinite, 0, sizeof(int), v->ctx->stream), "clear flag");
    ERNIE_CUDA(cudaGraphLaunch(p.graph, v->ctx->stream), "VAE graph");
    return ERNIE_CUDA_OK;
}

template <class V> int read_status(V *v, int *nonfinite)
{
    int flags[2] = {0, 0};
    ERNIE_CUDA(cudaMemcpyAsync(&flags[0], v->plan->nonfinite, sizeof(int), cudaMemcpyDeviceToHost, v->ctx->stream),
               "read flag");
    ERNIE_CUDA(cudaMemcpyAsync(&flags[1], v->ctx->error_flag, sizeof(int), cudaMemcpyDeviceToHost, v->ctx->stream),
               "read status");
    ERNIE_CUDA(cudaStreamSynchronize(v->ctx->stream), "VAE graph");
    if (flags[1]) return fail(ERNIE_CUDA_ERROR, "VAE kernel protocol timeout (status " + std::to_string(flags[1]) + ")");
    if (nonfinite) *nonfinite = flags[0];
    return ERNIE_CUDA_OK;
}

template <class V> int model_create(ernie_cuda_context *ctx, V **out)
{
    if (!ctx || !out) return fail(ERNIE_CUDA_ERROR, "null argument");
    *out = nullptr;
    DeviceGuard guard(ctx->device);
    auto v = std::make_unique<V>();
    v->ctx = ctx;
    auto &L = v->layout;
    Arena arena;
    size_t staging = 0;
    for (auto &prm : L.params) staging = std::max(staging, prm.count());
    arena.add(&v->staging, staging);
    arena.add(&v->staging2, staging); // re-ordered copy (tap-expanded or im2col weights)
    arena.add(&v->d_inexact, 1);
    for (auto &prm : L.params)
        if (prm.slot) arena.add(prm.slot, prm.count());
    for (ConvW *c : L.convs)
    {
        arena.add(&c->w, static_cast<size_t>(c->cout_rows) * 3 * c->dev_taps() * c->cin_pad);
        arena.add(&c->bias, static_cast<size_t>(c->cout_rows));
    }
    for (NormW *n : L.norms)
    {
        arena.add(&n->gamma, static_cast<size_t>(n->c));
        arena.add(&n->beta, static_cast<size_t>(n->c));
    }
    v->bytes = arena.bytes();
    ERNIE_CUDA(arena.allocate(), "Allocate VAE weights");
    v->alloc = arena.base;
    // zero padding rows/channels and the padded biases
    cudaError_t e = cudaMemsetAsync(v->alloc, 0, arena.bytes(), ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess)
    {
        cudaFree(v->alloc);
        return from_cuda(e, "Clear VAE weights");
    }
    // destinations of the FP32 vectors: the layout's own pointers, else GroupNorm gamma/beta in table order
    size_t norm_index = 0;
    for (auto &prm : L.params)
    {
        if (prm.role != Role::Vector) continue;
        if (prm.slot) prm.dst = *prm.slot;
        else
        {
            NormW *n = L.norms[norm_index / 2];
            prm.dst = norm_index % 2 == 0 ? n->gamma : n->beta;
            ++norm_index;
        }
    }
    *out = v.release();
    return ERNIE_CUDA_OK;
}

template <class V> int model_destroy(V *v)
{
    if (!v) return ERNIE_CUDA_OK;
    DeviceGuard guard(v->ctx->device);
    cudaStreamSynchronize(v->ctx->stream);
    drop_plan(v);
    if (v->alloc) cudaFree(v->alloc);
    delete v;
    return ERNIE_CUDA_OK;
}

template <class L> int table_count(int *count)
{
    if (!count) return fail(ERNIE_CUDA_ERROR, "null argument");
    static const L table;
    *count = static_cast<int>(table.params.size());
    return ERNIE_CUDA_OK;
}

template <class L> int table_info(int index, char *name, size_t name_bytes, int *dims, int *ndim)
{
    static const L table;
    if (index < 0 || index >= static_cast<int>(table.params.size()) || !name || !dims || !ndim)
        return fail(ERNIE_CUDA_ERROR, "Invalid VAE tensor index or null argument");
    const Param &prm = table.params[static_cast<size_t>(index)];
    if (prm.name.size() + 1 > name_bytes) return fail(ERNIE_CUDA_ERROR, "Name buffer too small");
    std::copy(prm.name.begin(), prm.name.end(), name);
    name[prm.name.size()] = '\0';
    *ndim = static_cast<int>(prm.shape.size());
    for (size_t d = 0; d < prm.shape.size(); ++d) dims[d] = prm.shape[d];
    return ERNIE_CUDA_OK;
}

template <class V> int model_upload(V *v, const char *name, const float *host, size_t count)
{
    if (!v || !name || !host) return fail(ERNIE_CUDA_ERROR, "null argument");
    const int i = find_param(v, name);
    if (i < 0) return fail(ERNIE_CUDA_ERROR, std::string("Unknown VAE tensor: ") + name);
    Param &prm = v->layout.params[static_cast<size_t>(i)];
    if (count != prm.count()) return fail(ERNIE_CUDA_ERROR, "VAE tensor size differs: " + prm.name);
    for (size_t j = 0; j < count; ++j)
        if (!std::isfinite(host[j])) return fail(ERNIE_CUDA_ERROR, "VAE tensor is not finite: " + prm.name);
    if (prm.name == "bn.running_var")
        for (size_t j = 0; j < count; ++j)
            if (!(host[j] >= 0.f)) return fail(ERNIE_CUDA_ERROR, "VAE tensor is negative: " + prm.name);
    DeviceGuard guard(v->ctx->device);
    ERNIE_CUDA(cudaMemcpyAsync(v->staging, host, count * 4, cudaMemcpyHostToDevice, v->ctx->stream), "upload");
    ERNIE_TRY(place(v, prm));
    ERNIE_CUDA(cudaStreamSynchronize(v->ctx->stream), "upload");
    drop_plan(v); // FP32-exact plane counts may change
    return ERNIE_CUDA_OK;
}

template <class V> int model_synthesize(V *v, uint64_t seed, int bf16_weights)
{
    if (!v) return fail(ERNIE_CUDA_ERROR, "null argument");
    DeviceGuard guard(v->ctx->device);
    for (auto &prm : v->layout.params)
    {
        const bool round = bf16_weights && prm.role == Role::ConvWeight;
        ERNIE_LAUNCH(launch_synth_f32(seed, ernie_synth_name_stream(prm.name.c_str()), prm.scale, prm.offset,
                                      static_cast<long long>(prm.count()), round ? 1 : 0, v->staging, v->ctx->stream),
                     "synthesize");
        ERNIE_TRY(place(v, prm));
    }
    ERNIE_CUDA(cudaStreamSynchronize(v->ctx->stream), "synthesize");
    drop_plan(v);
    return ERNIE_CUDA_OK;
}

template <class V> int model_bytes(V *v, uint64_t *weights, uint64_t *workspace)
{
    if (!v) return fail(ERNIE_CUDA_ERROR, "null argument");
    if (weights) *weights = v->bytes;
    if (workspace) *workspace = v->plan ? v->plan->bytes : 0;
    return ERNIE_CUDA_OK;
}

bool precision_ok(int precision) { return precision == ERNIE_PRECISION_BF16 || precision == ERNIE_PRECISION_FP32; }

template <class V> int model_launches(V *v, int width, int height, int precision, int *launches)
{
    DeviceGuard guard(v->ctx->device);
    ERNIE_TRY(check_loaded(v));
    ERNIE_TRY(ensure_plan(v, width, height, precision));
    *launches = v->plan->launches;
    return ERNIE_CUDA_OK;
}

template <class V> int model_profile(V *v, int width, int height, int precision, int iters, double *ms, double *work)
{
    DeviceGuard guard(v->ctx->device);
    ERNIE_TRY(check_loaded(v));
    ERNIE_TRY(ensure_plan(v, width, height, precision));
    Plan &p = *v->plan;
    Profiler prof;
    for (int c = 0; c < kProfClasses; ++c) ms[c] = work[c] = 0.0;
    for (int it = 0; it < iters; ++it)
    {
        const int launches = p.launches;
        prof.used = 0;
        Program prog{v->ctx, p, v->ctx->stream, v->ctx->num_sms, &prof};
        const int rc = prog.run(v->layout);
        p.launches = launches;
        ERNIE_TRY(rc);
        ERNIE_CUDA(cudaStreamSynchronize(v->ctx->stream), "VAE profile");
        for (size_t i = 0; i < prof.used; ++i)
        {
            float t = 0.f;
            ERNIE_CUDA(cudaEventElapsedTime(&t, prof.events[2 * i], prof.events[2 * i + 1]), "profile event");
            ms[prof.classes[i]] += t / iters;
            if (it == 0) work[prof.classes[i]] += prof.work[i];
        }
    }
    return ERNIE_CUDA_OK;
}

// One encode with the RGB bytes and the three outputs at `kind` (host or device) addresses.
int encode_impl(ernie_cuda_vae_encoder *v, const uint8_t *rgb, int width, int height, int precision, float *mean,
                float *packed, float *normalized, int *nonfinite, cudaMemcpyKind in, cudaMemcpyKind out)
{
    if (!v || !rgb || !mean || !packed || !normalized) return fail(ERNIE_CUDA_ERROR, "null argument");
    if (!encoder_shape_ok(width, height))
        return fail(ERNIE_CUDA_ERROR, "Unsupported VAE encoder image shape (sides multiples of 16, at most 2048)");
    if (!precision_ok(precision)) return fail(ERNIE_CUDA_ERROR, "Unknown precision");
    DeviceGuard guard(v->ctx->device);
    ERNIE_TRY(check_loaded(v));
    ERNIE_TRY(ensure_plan(v, width, height, precision));
    Plan &p = *v->plan;
    const size_t px = pixels_of(height, width);
    cudaStream_t stream = v->ctx->stream;
    ERNIE_CUDA(cudaMemcpyAsync(p.rgb_in, rgb, 3 * px, in, stream), "encoder input");
    ERNIE_TRY(run_graph(v, width, height, precision));
    ERNIE_CUDA(cudaMemcpyAsync(mean, p.mean, 32 * px / 64 * 4, out, stream), "encoder mean");
    ERNIE_CUDA(cudaMemcpyAsync(packed, p.packed, 128 * px / 256 * 4, out, stream), "encoder packed");
    ERNIE_CUDA(cudaMemcpyAsync(normalized, p.normalized, 128 * px / 256 * 4, out, stream), "encoder normalized");
    if (!nonfinite && out == cudaMemcpyDeviceToDevice) return ERNIE_CUDA_OK; // stays asynchronous
    int flag = 0;
    ERNIE_TRY(read_status(v, &flag));
    if (nonfinite) *nonfinite = flag;
    return ERNIE_CUDA_OK;
}
} // namespace

// ---- VAE decoder ---------------------------------------------------------------------------------------
extern "C" int ernie_cuda_vae_create(ernie_cuda_context *ctx, ernie_cuda_vae **out) { return model_create(ctx, out); }

extern "C" int ernie_cuda_vae_destroy(ernie_cuda_vae *v) { return model_destroy(v); }

extern "C" int ernie_cuda_vae_tensor_count(int *count) { return table_count<Layout>(count); }

extern "C" int ernie_cuda_vae_tensor_info(int index, char *name, size_t name_bytes, int *dims, int *ndim)
{
    return table_info<Layout>(index, name, name_bytes, dims, ndim);
}

extern "C" int ernie_cuda_vae_upload(ernie_cuda_vae *v, const char *name, const float *host, size_t count)
{
    return model_upload(v, name, host, count);
}

extern "C" int ernie_cuda_vae_synthesize(ernie_cuda_vae *v, uint64_t seed, int bf16_weights)
{
    return model_synthesize(v, seed, bf16_weights);
}

extern "C" int ernie_cuda_vae_bytes(ernie_cuda_vae *v, uint64_t *weights, uint64_t *workspace)
{
    return model_bytes(v, weights, workspace);
}

extern "C" int ernie_cuda_vae_launches(ernie_cuda_vae *v, int width, int height, int precision, int *launches)
{
    if (!v || !launches) return fail(ERNIE_CUDA_ERROR, "null argument");
    if (!vae_shape_ok(width, height)) return fail(ERNIE_CUDA_ERROR, "Unsupported VAE latent shape");
    if (!precision_ok(precision)) return fail(ERNIE_CUDA_ERROR, "Unknown precision");
    return model_launches(v, width, height, precision, launches);
}

extern "C" int ernie_cuda_vae_decode_device(ernie_cuda_vae *v, const float *unpacked, int width, int height,
                                            int precision, float *decoded, uint8_t *rgb, int *nonfinite)
{
    if (!v || !unpacked || !decoded) return fail(ERNIE_CUDA_ERROR, "null argument");
    if (!vae_shape_ok(width, height)) return fail(ERNIE_CUDA_ERROR, "Unsupported VAE latent shape");
    if (!precision_ok(precision)) return fail(ERNIE_CUDA_ERROR, "Unknown precision");
    DeviceGuard guard(v->ctx->device);
    ERNIE_TRY(check_loaded(v));
    ERNIE_TRY(ensure_plan(v, width, height, precision));
    Plan &p = *v->plan;
    const size_t in = 32 * pixels_of(height, width), out = 3 * 64 * pixels_of(height, width);
    ERNIE_CUDA(cudaMemcpyAsync(p.input, unpacked, in * 4, cudaMemcpyDeviceToDevice, v->ctx->stream), "VAE input");
    ERNIE_TRY(run_graph(v, width, height, precision));
    ERNIE_CUDA(cudaMemcpyAsync(decoded, p.decoded, out * 4, cudaMemcpyDeviceToDevice, v->ctx->stream), "VAE output");
    if (rgb) ERNIE_CUDA(cudaMemcpyAsync(rgb, p.rgb, out, cudaMemcpyDeviceToDevice, v->ctx->stream), "RGB output");
    if (!nonfinite) return ERNIE_CUDA_OK; // stays asynchronous
    return read_status(v, nonfinite);
}

extern "C" int ernie_cuda_vae_decode(ernie_cuda_vae *v, const float *unpacked, int width, int height, int precision,
                                     float *decoded, uint8_t *rgb, int *nonfinite)
{
    if (!v || !unpacked || !decoded) return fail(ERNIE_CUDA_ERROR, "null argument");
    if (!vae_shape_ok(width, height)) return fail(ERNIE_CUDA_ERROR, "Unsupported VAE latent shape");
    if (!precision_ok(precision)) return fail(ERNIE_CUDA_ERROR, "Unknown precision");
    DeviceGuard guard(v->ctx->device);
    ERNIE_TRY(check_loaded(v));
    ERNIE_TRY(ensure_plan(v, width, height, precision));
    Plan &p = *v->plan;
    const size_t in = 32 * pixels_of(height, width), out = 3 * 64 * pixels_of(height, width);
    ERNIE_CUDA(cudaMemcpyAsync(p.input, unpacked, in * 4, cudaMemcpyHostToDevice, v->ctx->stream), "VAE input");
    ERNIE_TRY(run_graph(v, width, height, precision));
    ERNIE_CUDA(cudaMemcpyAsync(decoded, p.decoded, out * 4, cudaMemcpyDeviceToHost, v->ctx->stream), "VAE output");
    if (rgb) ERNIE_CUDA(cudaMemcpyAsync(rgb, p.rgb, out, cudaMemcpyDeviceToHost, v->ctx->stream), "RGB output");
    int flag = 0;
    ERNIE_TRY(read_status(v, &flag));
    if (nonfinite) *nonfinite = flag;
    return ERNIE_CUDA_OK;
}

extern "C" int ernie_cuda_vae_profile(ernie_cuda_vae *v, int width, int height, int precision, int iters, double *ms,
                                      double *work)
{
    if (!v || !ms || !work || iters < 1) return fail(ERNIE_CUDA_ERROR, "null argument or iters < 1");
    if (!vae_shape_ok(width, height)) return fail(ERNIE_CUDA_ERROR, "Unsupported VAE latent shape");
    if (!precision_ok(precision)) return fail(ERNIE_CUDA_ERROR, "Unknown precision");
    return model_profile(v, width, height, precision, iters, ms, work);
}

// ---- VAE encoder ---------------------------------------------------------------------------------------
extern "C" int ernie_cuda_vae_encoder_create(ernie_cuda_context *ctx, ernie_cuda_vae_encoder **out)
{
    return model_create(ctx, out);
}

extern "C" int ernie_cuda_vae_encoder_destroy(ernie_cuda_vae_encoder *v) { return model_destroy(v); }

extern "C" int ernie_cuda_vae_encoder_tensor_count(int *count) { return table_count<EncoderLayout>(count); }

extern "C" int ernie_cuda_vae_encoder_tensor_info(int index, char *name, size_t name_bytes, int *dims, int *ndim)
{
    return table_info<EncoderLayout>(index, name, name_bytes, dims, ndim);
}

extern "C" int ernie_cuda_vae_encoder_upload(ernie_cuda_vae_encoder *v, const char *name, const float *host,
                                             size_t count)
{
    return model_upload(v, name, host, count);
}

extern "C" int ernie_cuda_vae_encoder_synthesize(ernie_cuda_vae_encoder *v, uint64_t seed, int bf16_weights)
{
    return model_synthesize(v, seed, bf16_weights);
}

extern "C" int ernie_cuda_vae_encoder_bytes(ernie_cuda_vae_encoder *v, uint64_t *weights, uint64_t *workspace)
{
    return model_bytes(v, weights, workspace);
}

extern "C" int ernie_cuda_vae_encoder_launches(ernie_cuda_vae_encoder *v, int width, int height, int precision,
                                               int *launches)
{
    if (!v || !launches) return fail(ERNIE_CUDA_ERROR, "null argument");
    if (!encoder_shape_ok(width, height)) return fail(ERNIE_CUDA_ERROR, "Unsupported VAE encoder image shape");
    if (!precision_ok(precision)) return fail(ERNIE_CUDA_ERROR, "Unknown precision");
    return model_launches(v, width, height, precision, launches);
}

extern "C" int ernie_cuda_vae_encoder_profile(ernie_cuda_vae_encoder *v, int width, int height, int precision,
                                              int iters, double *ms, double *work)
{
    if (!v || !ms || !work || iters < 1) return fail(ERNIE_CUDA_ERROR, "null argument or iters < 1");
    if (!encoder_shape_ok(width, height)) return fail(ERNIE_CUDA_ERROR, "Unsupported VAE encoder image shape");
    if (!precision_ok(precision)) return fail(ERNIE_CUDA_ERROR, "Unknown precision");
    return model_profile(v, width, height, precision, iters, ms, work);
}

extern "C" int ernie_cuda_vae_encode(ernie_cuda_vae_encoder *v, const uint8_t *rgb, int width, int height,
                                     int precision, float *mean, float *packed, float *normalized, int *nonfinite)
{
    return encode_impl(v, rgb, width, height, precision, mean, packed, normalized, nonfinite, cudaMemcpyHostToDevice,
                       cudaMemcpyDeviceToHost);
}

extern "C" int ernie_cuda_vae_encode_device(ernie_cuda_vae_encoder *v, const uint8_t *rgb, int width, int height,
                                            int precision, float *mean, float *packed, float *normalized,
                                            int *nonfinite)
{
    return encode_impl(v, rgb, width, height, precision, mean, packed, normalized, nonfinite,
                       cudaMemcpyDeviceToDevice, cudaMemcpyDeviceToDevice);
}
