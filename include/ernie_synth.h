/* Seeded, counter-based synthetic data for the ERNIE DiT hot path.
 *
 * The reference's official weights (23 GB BF16 safetensors) and its golden tensors are not
 * available, so every parity case and benchmark runs on seeded random-init weights and inputs.
 * Element i of stream s under seed k is a pure function of (k, s, i): the CPU oracle, the host
 * weight uploader and the device-side weight generator all produce identical bytes without
 * sharing any state.
 *
 *   weights   N(0, 0.02) rounded to BF16 (official weights are stored as BF16 and loaded
 *             losslessly; reference tools/build_dit_weights.py:96-115)
 *   norm γ    1 + N(0, 0.02) rounded to BF16
 *   inputs    N(0, 1) in FP32 (latent noise, text features, hidden states)
 *
 * Normal deviates use the Box-Muller transform (cosine branch) on two 53-bit uniforms taken
 * from a SplitMix64 hash of the counter. Host and device evaluate the same double-precision
 * formula; libm and CUDA's double log/cos may differ in the last ulp, which cannot change a
 * BF16-rounded weight except with probability ~2^-44 per element (tests compare bytes).
 *
 * Header-only, C and CUDA compatible.
 */
#ifndef ERNIE_SYNTH_H
#define ERNIE_SYNTH_H
#include <stdint.h>
#include <math.h>

#if defined(__CUDACC__)
#define ERNIE_SYNTH_FN static inline __host__ __device__
#else
#define ERNIE_SYNTH_FN static inline
#endif

ERNIE_SYNTH_FN uint64_t ernie_synth_mix(uint64_t x)
{
    x += 0x9E3779B97F4A7C15ULL;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
    return x ^ (x >> 31);
}

/* Standard normal deviate for (seed, stream, index). */
ERNIE_SYNTH_FN double ernie_synth_normal(uint64_t seed, uint64_t stream, uint64_t index)
{
    const uint64_t key = ernie_synth_mix(seed ^ ernie_synth_mix(stream * 0xD1B54A32D192ED03ULL));
    const uint64_t h1 = ernie_synth_mix(key + 2 * index);
    const uint64_t h2 = ernie_synth_mix(key + 2 * index + 1);
    const double u1 = ((double)(h1 >> 11) + 1.0) * (1.0 / 9007199254740992.0); /* (0,1] */
    const double u2 = (double)(h2 >> 11) * (1.0 / 9007199254740992.0);         /* [0,1) */
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586476925 * u2);
}

/* Round-to-nearest-even FP32 -> BF16 bits (finite inputs). */
ERNIE_SYNTH_FN uint16_t ernie_synth_bf16_bits(float value)
{
    union { float f; uint32_t u; } bits;
    bits.f = value;
    const uint32_t rounded = bits.u + 0x7FFFu + ((bits.u >> 16) & 1u);
    return (uint16_t)(rounded >> 16);
}

ERNIE_SYNTH_FN float ernie_synth_bf16_to_float(uint16_t value)
{
    union { float f; uint32_t u; } bits;
    bits.u = (uint32_t)value << 16;
    return bits.f;
}

/* Weight element: BF16(scale * N(0,1) + offset). */
ERNIE_SYNTH_FN uint16_t ernie_synth_weight(uint64_t seed, uint64_t stream, uint64_t index, float scale,
                                           float offset)
{
    const float value = (float)(ernie_synth_normal(seed, stream, index) * (double)scale) + offset;
    return ernie_synth_bf16_bits(value);
}

/* Stream identifiers. Block tensors use ERNIE_SYNTH_BLOCK_STREAM(block, tensor). */
enum ernie_synth_tensor
{
    ERNIE_SYNTH_WQ = 0,
    ERNIE_SYNTH_WK = 1,
    ERNIE_SYNTH_WV = 2,
    ERNIE_SYNTH_WO = 3,
    ERNIE_SYNTH_WUP = 4,
    ERNIE_SYNTH_WGATE = 5,
    ERNIE_SYNTH_WFC2 = 6,
    ERNIE_SYNTH_GAMMA_SA = 7,
    ERNIE_SYNTH_GAMMA_MLP = 8,
    ERNIE_SYNTH_GAMMA_Q = 9,
    ERNIE_SYNTH_GAMMA_K = 10,
    /* heads (stream = tensor id, block-independent) */
    ERNIE_SYNTH_X_EMBED_W = 32,
    ERNIE_SYNTH_X_EMBED_B = 33,
    ERNIE_SYNTH_TEXT_PROJ_W = 34,
    ERNIE_SYNTH_TIME1_W = 35,
    ERNIE_SYNTH_TIME1_B = 36,
    ERNIE_SYNTH_TIME2_W = 37,
    ERNIE_SYNTH_TIME2_B = 38,
    ERNIE_SYNTH_ADALN_W = 39,
    ERNIE_SYNTH_ADALN_B = 40,
    ERNIE_SYNTH_FINAL_NORM_W = 41,
    ERNIE_SYNTH_FINAL_NORM_B = 42,
    ERNIE_SYNTH_FINAL_W = 43,
    ERNIE_SYNTH_FINAL_B = 44,
    /* inputs */
    ERNIE_SYNTH_LATENT = 48,
    ERNIE_SYNTH_TEXT = 49,
    ERNIE_SYNTH_HIDDEN = 50,
    ERNIE_SYNTH_TEMB = 51
};
#define ERNIE_SYNTH_BLOCK_STREAM(block, tensor) ((uint64_t)((block) + 1) * 64u + (uint64_t)(tensor))
#define ERNIE_SYNTH_WEIGHT_STD 0.02f

/* Text encoder layers (Mistral decoder layers of the prompt encoder): BF16 weights N(0, 0.02) and RMSNorm
 * weights 1 + N(0, 0.02) as for the DiT blocks, streams ERNIE_SYNTH_TEXT_STREAM(layer, tensor). */
enum ernie_synth_text_tensor
{
    ERNIE_SYNTH_TEXT_WQ = 0,
    ERNIE_SYNTH_TEXT_WK = 1,
    ERNIE_SYNTH_TEXT_WV = 2,
    ERNIE_SYNTH_TEXT_WO = 3,
    ERNIE_SYNTH_TEXT_WGATE = 4,
    ERNIE_SYNTH_TEXT_WUP = 5,
    ERNIE_SYNTH_TEXT_WDOWN = 6,
    ERNIE_SYNTH_TEXT_GAMMA_ATTN = 7,
    ERNIE_SYNTH_TEXT_GAMMA_MLP = 8
};
#define ERNIE_SYNTH_TEXT_STREAM(layer, tensor) (0x54455854ULL * 4096u + (uint64_t)((layer) + 1) * 64u + (uint64_t)(tensor))
/* The prompt enhancer's LM head on a text model: lm_head [131072][3072] N(0, 0.02) BF16 and the final
 * RMSNorm weight 1 + N(0, 0.02), streams ERNIE_SYNTH_TEXT_STREAM(ERNIE_SYNTH_TEXT_HEAD_LAYER, 0 / 1). */
#define ERNIE_SYNTH_TEXT_HEAD_LAYER 1023

/* VAE decoder tensors are addressed by their diffusers parameter name (e.g. "decoder.conv_in.weight"):
 * stream = FNV-1a 64 of the name. Values are FP32, float(N(0,1) * scale) + offset, with
 *   convolution / linear weights   scale 1/sqrt(fan_in), offset 0
 *   GroupNorm weights (gamma)      scale 0.1, offset 1
 *   GroupNorm biases (beta)        scale 0.1, offset 0
 *   other biases                   scale 0.02, offset 0
 * optionally rounded to BF16 (weights stored as BF16). */
ERNIE_SYNTH_FN uint64_t ernie_synth_name_stream(const char *name)
{
    uint64_t h = 0xCBF29CE484222325ULL;
    for (; *name; ++name)
    {
        h ^= (uint64_t)(unsigned char)*name;
        h *= 0x100000001B3ULL;
    }
    return h;
}

#endif
