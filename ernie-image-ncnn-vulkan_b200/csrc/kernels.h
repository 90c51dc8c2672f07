// Internal launch interface of the sm_100a kernels (host side). Plain pointers and sizes; all
// buffers are device memory owned by the caller and must outlive the enqueued work.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace ernie_b200
{
constexpr int kHidden = 4096, kHeads = 32, kHeadDim = 128, kFfn = 12288, kTextDim = 3072, kLatent = 128;

enum class Epilogue : int
{
    F32Bias = 0,    // out[r, c] = acc + bias[c] (bias may be null), FP32, row stride ldo
    Qkv = 1,        // per-head qk-RMSNorm + 3-axis RoPE on Q,K; write Q,K,V head-major
    ResidGate = 2,  // resid[r, c] += gate[c] * acc (FP32, in place)
    Geglu = 3,      // h[r, f] = up * gelu_erf(gate) from [up; gate] weights interleaved in 64-row groups
    FinalEuler = 4, // pred = acc + bias; latent[c][r] = latent + delta * pred (no FMA); finite flag
};

// Programmatic dependent launch of the DiT block's kernels (GEMMs, tcgen05 attention, the two-row
// norm): each is launched with the programmatic-serialization attribute, so its CTAs may run their
// set-up (barrier init, TMEM allocation, tensor-map prefetch) while the previous kernel drains, and
// each waits for that kernel (griddepcontrol.wait) before its first global-memory access.
// Off by default: with the early trigger the C2 step measured 68.1-68.8 ms against 66.8-67.1 with plain
// stream order (C1 18.6 against 18.2), in a same-box A/B.
#ifndef ERNIE_PDL
#define ERNIE_PDL 0
#endif
constexpr bool kProgrammaticLaunch = ERNIE_PDL != 0;

// Appends the programmatic-serialization attribute to `attrs` (when enabled); returns the new count.
inline unsigned add_programmatic_attribute(cudaLaunchAttribute *attrs, unsigned count)
{
    if (!kProgrammaticLaunch) return count;
    attrs[count].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[count].val.programmaticStreamSerializationAllowed = 1;
    return count + 1;
}

// Destinations of the fused sequence-parallel stores (one per GPU of the group).
constexpr int kMaxDest = 8;

// Completion flags of a sequence-parallel group, carried by the kernels themselves (used instead of the
// two barrier kernels when a whole block is enqueued). A producing kernel (the QKV GEMM, whose epilogue
// stores heads into their owners; the attention, whose epilogue stores rows into their owners) counts
// its finishing warps; the last one publishes the next epoch into slot `rank` of every member (release,
// system scope). A consuming kernel's loading threads wait (acquire, bounded by timeout_ns) until every
// slot of this GPU's array reaches this GPU's own epoch of that producer, before their first bulk load.
struct PeerSignal
{
    unsigned *counter = nullptr;         // this GPU: warps of the current launch that have finished
    int warps = 0;                       // warps that arrive per launch (set by the launcher)
    unsigned *epoch = nullptr;           // this GPU: launches of the producer signalled so far
    unsigned *peer_slot[kMaxDest] = {};  // member p's arrival slot for this GPU
    int members = 0;
};
struct PeerWait
{
    const unsigned *slots = nullptr; // this GPU's [members] arrival slots
    const unsigned *epoch = nullptr; // this GPU's epoch of the producer (its own launch has signalled)
    int members = 0;
    long long timeout_ns = 0;
    int *error_flag = nullptr;
};
struct PeerSync
{
    PeerWait wait;     // before the first load (slots null: no wait)
    PeerSignal signal; // after the last store (counter null: no signal)
};

struct GemmEpilogueArgs
{
    // F32Bias
    float *out = nullptr;
    int ldo = 0;
    const float *bias = nullptr;
    // ResidGate
    float *resid = nullptr;
    const float *gate = nullptr;
    // Qkv: head h of output row r goes to destination d = h / heads_per_dest (a GPU of a sequence-parallel
    // group, through peer memory; destination 0 alone on one GPU) as head h % heads_per_dest, row
    // row_offset + r, of [heads][rows_pad][128] arrays (BF16 or FP32); BF16 V^T is [heads][128][rows_pad].
    // Rows at or past row_limit (0: rows_pad) are not written.
    void *q[kMaxDest] = {}, *k[kMaxDest] = {}, *v[kMaxDest] = {};
    int heads_per_dest = 32;
    int row_offset = 0, row_limit = 0;
    int rows_pad = 0;
    int qkv_split3 = 0;   // FP32-exact mode: each of Q, K, V^T as three BF16 planes (hi, mid, lo), plane
                          // p at element offset p * heads_per_dest * rows_pad * 128
    int v_transposed = 0; // V written as [heads][128][rows_pad] (per plane) for the tcgen05 attention
    const float *gamma_q = nullptr, *gamma_k = nullptr; // [128]
    const float *cos_t = nullptr, *sin_t = nullptr;     // [rows][128]
    // Geglu: BF16 [rows][ffn] or, when split3, hi/mid/lo BF16 planes at column offsets 0, ffn, 2*ffn
    __nv_bfloat16 *h = nullptr;
    int h_split3 = 0;
    int ffn = 0;
    int silu = 0; // Geglu with SiLU instead of GELU: h = up * silu(gate) (the text encoder's SwiGLU MLP)
    // FinalEuler
    float *latent = nullptr;     // [128][ld_latent] (ld_latent 0: rows)
    int ld_latent = 0;
    float *prediction = nullptr; // optional [128][rows]
    float delta = 0.f;
    int *finite_flag = nullptr; // set to 1 if any updated latent value is not finite
    // RMSNorm + modulate folded into the GEMMs around it (BF16 DiT blocks), with x' the FP32 residual row
    // and g = gamma * (1 + scale): norm(x') g + shift = rinv (x' g) + shift, rinv = (sum x'^2 / 4096 + 1e-6)^(-1/2).
    // Producer (ResidGate with fold_out): also writes bf16(x' g) to fold_out (row stride kHidden) and the
    // sum of x'^2 over each 128-column part p of the row to fold_sumsq[p * fold_ld + row].
    // Consumer (Qkv, Geglu with fold_bias): A holds bf16(x' g); each accumulator becomes
    // rinv * acc + fold_bias[col] (fold_bias = W shift), rinv from the row's kFoldParts sums.
    __nv_bfloat16 *fold_out = nullptr;
    const float *fold_gamma = nullptr, *fold_scale = nullptr;
    float *fold_sumsq = nullptr;
    int fold_ld = 0;
    const float *fold_bias = nullptr;
    // all
    int *error_flag = nullptr;
    PeerSync sync; // sequence parallel: wait before the first A/B load, signal after the last store
};
constexpr int kFoldParts = kHidden / 128; // 128-column parts of a folded row's sum of squares

// C[M, N] = A[M, K_a] * B[N, K_b]^T with BF16 operands and FP32 accumulation on tcgen05.
// K_a = splits * K_b: in FP32-exact mode A holds `splits` BF16 planes (hi, mid, lo) side by side
// and every plane multiplies the same exact-BF16 weights. `promote` (block_n 128 only) restarts
// the tensor-core accumulator every 256 products and sums the partials in FP32 registers.
// Geglu weights are [up; gate] interleaved in 64-row groups. Returns a cudaError_t.
int launch_gemm(const __nv_bfloat16 *a, const __nv_bfloat16 *b, int m, int n, int k_b, int splits, int block_n,
                Epilogue epilogue, const GemmEpilogueArgs &args, int num_sms, cudaStream_t stream,
                bool promote = false);

// Row statistics + modulation: y = norm(x) * (1 + scale) + shift, written as BF16 or as 3 BF16 planes.
// centered = 0: RMSNorm with gamma; centered = 1: non-affine LayerNorm. scale/shift may be null.
int launch_norm_modulate(const float *x, int rows, int width, const float *gamma, const float *scale,
                         const float *shift, float eps, int centered, __nv_bfloat16 *out, int split3,
                         cudaStream_t stream);
// Channel-major latent [128][tokens] -> token-major BF16 A operand [tokens][128] (or 3 planes).
int launch_latent_to_tokens(const float *latent, int tokens, __nv_bfloat16 *out, int split3, cudaStream_t stream,
                            int ld = 0);
// FP32 [rows][cols] -> BF16 [rows][cols] (or 3 BF16 planes [rows][3*cols]).
int launch_to_operand(const float *src, long long rows, int cols, __nv_bfloat16 *out, int split3, cudaStream_t stream);
// y[n] = W[n, :] . act(x) + bias[n]; act = SiLU when silu_input.
int launch_gemv(const __nv_bfloat16 *w, const float *x, const float *bias, float *y, int n, int k, int silu_input,
                cudaStream_t stream);

// tcgen05 flash attention (BF16 operands, FP32 softmax/accumulation in TMEM and registers):
// q, k head-major [heads][rows_pad][128], vt transposed [heads][128][rows_pad]; keys >= kv_len
// excluded, optional additive row mask [rows]. Output token-major BF16 [rows][heads*128].
int launch_flash_tc(const __nv_bfloat16 *q, const __nv_bfloat16 *k, const __nv_bfloat16 *vt, const float *mask,
                    int rows, int rows_pad, int kv_len, int heads, __nv_bfloat16 *out, int *error_flag,
                    cudaStream_t stream);
// Output rows scattered over destinations: row r goes to dst[r / rows_per_dest], row r % rows_per_dest,
// columns col_offset + head*128 of a [rows][ld] BF16 array (sequence parallel: each token row to the
// GPU that owns it, through peer memory).
struct FlashOutput
{
    __nv_bfloat16 *dst[kMaxDest] = {};
    int rows_per_dest = 0, ld = 0, col_offset = 0;
};
// causal: key j > query i excluded; kv_heads (0: heads) K/V heads, query head h reading K/V head
// h / (heads / kv_heads), k [kv_heads][rows_pad][128], vt [kv_heads][128][rows_pad].
int launch_flash_tc(const __nv_bfloat16 *q, const __nv_bfloat16 *k, const __nv_bfloat16 *vt, const float *mask,
                    int rows, int rows_pad, int kv_len, int heads, const FlashOutput &out, int *error_flag,
                    cudaStream_t stream, int causal = 0, int kv_heads = 0, const PeerSync *sync = nullptr);
// Barrier of a sequence-parallel group over peer memory: this GPU's arrival is stored (release, system
// scope) into slot `rank` of every member's slots; then it waits (acquire, bounded by `timeout_ns`) until
// every member's arrival in its own slots reaches the same epoch. Epochs count up on the device, so the
// barrier can sit inside a CUDA graph. On timeout it sets error_flag and returns.
struct PeerBarrier
{
    unsigned *slots = nullptr;              // this GPU's [world] arrival slots
    unsigned *peer_slots[kMaxDest] = {};    // every member's slots (this GPU's own included)
    unsigned *epoch = nullptr;              // this GPU's barrier counter
    int rank = 0, world = 1;
    long long timeout_ns = 0;
    int *error_flag = nullptr;
};
int launch_peer_barrier(const PeerBarrier &barrier, cudaStream_t stream);
// The signal alone, for a member whose producing kernel has no rows to run.
int launch_peer_signal(const PeerSignal &signal, cudaStream_t stream);
// Stores `bytes` (a multiple of 4) of src into every destination (peer memory included).
struct PeerPut
{
    void *dst[kMaxDest] = {};
    int members = 0;
};
int launch_peer_put(const void *src, size_t bytes, const PeerPut &put, cudaStream_t stream);
int prepare_flash_kernels();
// FP32-exact attention on the tensor cores: q3, k3 = three BF16 planes [3][heads][rows_pad][128], vt3 =
// [3][heads][128][rows_pad]; out_split3 = token-major [rows][3 * heads * 128] planes (hi, mid, lo).
int launch_flash_f32(const __nv_bfloat16 *q3, const __nv_bfloat16 *k3, const __nv_bfloat16 *vt3, const float *mask,
                     int rows, int rows_pad, int kv_len, int heads, __nv_bfloat16 *out_split3, int *error_flag,
                     cudaStream_t stream);
int prepare_flash_f32_kernels();

// FP32 attention with FP64 softmax accumulation. q [heads][q_stride rows][width] (head stride
// q_head_stride elements), k/v [kv_heads][...] with kv_heads dividing heads (query head h reads K/V head
// h / (heads / kv_heads)); mask [mask_heads][mask_rows][nk] additive (nullable); causal: key j > query i
// excluded (key tiles past the diagonal skipped). out_mode 0: FP32 [heads][nq][width]; 1: split-3 BF16
// token-major [nq][3*heads*width]; 2: BF16 token-major [nq][heads*width] (in out_split3).
struct AttentionF32Args
{
    const float *q, *k, *v, *mask;
    int heads, kv_heads, mask_heads, mask_rows, nq, nk, kv_len, width;
    long long q_head_stride, kv_head_stride;
    int out_mode;
    float *out_f32;
    __nv_bfloat16 *out_split3;
    int causal;            // key j visible to query i iff j <= i + causal_offset
    int causal_offset = 0; // position of query 0 (a KV-cached chunk appended after causal_offset keys)
    int decode = 0;        // 1..32 query rows of width 128: one CTA per (head, row), keys split over its warps
    // decode only, nullable: the device-resident position of query 0, in place of causal_offset (and
    // kv_len = *position + nq), so that a captured step is position-independent
    const int *position = nullptr;
};
int launch_attention_f32(const AttentionF32Args &args, cudaStream_t stream);

int launch_euler(const float *sample, const float *prediction, float delta, long long count, float *out,
                 cudaStream_t stream);
int launch_finite(const float *x, long long count, int *flag, cudaStream_t stream);
int launch_unpack_for_vae(const float *packed, const float *mean, const float *variance, int w, int h, float *out,
                          cudaStream_t stream);
int launch_gelu(float *data, long long count, cudaStream_t stream);
int launch_residual_add(const float *a, const float *b, float *out, long long count, cudaStream_t stream);
int launch_rmsnorm(const float *x, const float *gamma, long long rows, int width, float eps, int centered,
                   float *out, cudaStream_t stream);

// ---- VAE decoder (vae.cu) --------------------------------------------------------------------------
// Implicit-GEMM convolution on tcgen05 (stride 1, same padding): out[pixel][c] over an NHWC BF16 operand.
struct ConvArgs
{
    // geometry and schedule (set by launch_conv)
    int height = 0, width = 0, cin = 0, taps = 0, cout = 0, products = 1, group = 1;
    int stride2 = 0, phase_stride = 0; // stride-2 taps over a space-to-depth operand (ConvLaunch::stride2)
    // out[pixel][c] = acc + bias[c] + resid[pixel][c], FP32 NHWC with row stride ldo (resid may equal out)
    float *out = nullptr;
    int ldo = 0;
    const float *bias = nullptr;
    const float *resid = nullptr;
    // GroupNorm partials of the written values: stats[group][slot] = (sum, sum of squares) in FP64 over
    // groups of cpg channels (4, 8 or 16); one slot per epilogue warp (conv_stat_slots of them)
    double2 *stats = nullptr;
    int cpg = 0;
    int *error_flag = nullptr;
};
struct ConvLaunch
{
    const __nv_bfloat16 *a = nullptr; // operand [height][width][a_planes * cin] (planes side by side per pixel)
    int a_planes = 1;                 // 3: FP32-exact mode (hi, mid, lo)
    const __nv_bfloat16 *b = nullptr; // weights [cout_rows][b_row]: plane p, tap t, channel c at p*taps*cin + t*cin + c
    int b_planes = 1;                 // weight planes multiplied in FP32-exact mode (1: exact-BF16 weights)
    long long b_row = 0;
    int cout_rows = 0;
    int height = 0, width = 0, cin = 0, taps = 1, cout = 0; // cin a multiple of 64; cout 32 or a multiple of 128
    // 3x3 stride-2 convolution whose input is padded by one zero row and column at the bottom and right
    // (Downsample2D): `a` is the space-to-depth operand [height][width][4][a_planes][cin] of the
    // [2 height][2 width] input (launch_s2d_operand) and height/width are the output's; tap (ky, kx) reads
    // phase (ky & 1, kx & 1) at (y + ky / 2, x + kx / 2), and the zero padding is TMA's fill past the edge.
    int stride2 = 0;
};
// GroupNorm partial slots per group that launch_conv writes for this launch (8 per CTA of its grid).
int conv_stat_slots(const ConvLaunch &launch, int num_sms);
constexpr int kSoftmaxMaxRow = 57344; // keys per attention row (the row is staged in shared memory)
int launch_conv(const ConvLaunch &launch, const ConvArgs &epilogue, int num_sms, cudaStream_t stream);
// ---- VAE encoder passes ----
// conv_in as a 1x1 product: RGB bytes [h][w][3] -> (v - 127.5f) * (1 / 127.5f), gathered into the 3x3
// neighbourhood's 27 values per pixel (column t * 3 + c for tap t = ky * 3 + kx, zero outside the image)
// as the operand [h * w][planes * 64] (columns 27..63 zero).
int launch_rgb_im2col(const uint8_t *rgb, int h, int w, __nv_bfloat16 *out, int planes, cudaStream_t stream);
// OIHW FP32 [cout][cin][taps] -> [cout][taps * cin] (column t * cin + c): im2col column order.
int launch_taps_inner(const float *w, int cout, int cin, int taps, float *out, cudaStream_t stream);
// FP32 NHWC [h][w][channels] (h, w even) -> the stride-2 convolution's operand [h/2][w/2][4][planes][channels]
// (phase (y & 1) * 2 + (x & 1)).
int launch_s2d_operand(const float *x, int h, int w, int channels, __nv_bfloat16 *out, int planes,
                       cudaStream_t stream);
// quant_conv (1x1 over the 64 conv_out channels of `hin` [h][w][ldh], FP32) keeping outputs 0..31 (the
// posterior's mode): mean [32][h][w]; packed = pixel_unshuffle(mean, 2) [128][h/2][w/2] (channel
// c * 4 + (y & 1) * 2 + (x & 1)); normalized[c] = (packed[c] - rm[c]) / sqrt(rv[c] + eps). Any non-finite
// output sets *nonfinite.
int launch_encoder_output(const float *hin, int ldh, int h, int w, const float *wq, const float *bq, const float *rm,
                          const float *rv, float eps, float *mean, float *packed, float *normalized, int *nonfinite,
                          cudaStream_t stream);
// scale[c] = gamma[c] / sqrt(var_g + eps), shift[c] = beta[c] - mean_g * scale[c] from `slots` partials of
// each of 32 groups.
int launch_gn_finalize(const double2 *stats, int slots, long long count, int cpg, const float *gamma,
                       const float *beta, float eps, float *scale, float *shift, cudaStream_t stream);
// x * scale + shift (+ Swish), FP32 NHWC [pixels][channels] -> BF16 operand [pixels][planes * channels];
// raw (nullable) receives x itself in the same operand layout.
int launch_gn_apply(const float *x, long long pixels, int channels, const float *scale, const float *shift, int silu,
                    __nv_bfloat16 *out, int planes, cudaStream_t stream, __nv_bfloat16 *raw = nullptr);
// Nearest x2 of FP32 NHWC [h][w][channels] -> BF16 operand [2h][2w][planes * channels].
int launch_upsample(const float *x, int h, int w, int channels, __nv_bfloat16 *out, int planes, cudaStream_t stream);
// post_quant_conv (w [32][32], bias [32], FP32) of the unpacked latent [32][pixels] -> operand [pixels][planes * 64].
int launch_vae_input(const float *unpacked, long long pixels, const float *w, const float *bias, __nv_bfloat16 *out,
                     int planes, cudaStream_t stream);
// softmax(S[r, :n] * scale) -> BF16 planes [rows][planes * ldp] (columns n.. zero).
int launch_softmax_rows(const float *s, int rows, int lds, int n, float scale, __nv_bfloat16 *p, int ldp, int planes,
                        cudaStream_t stream);
// [n][1536] FP32 q|k|v -> Q, K [n][planes * 512] and V^T [512][planes * ldv] BF16 planes.
int launch_attention_split(const float *qkv, int n, __nv_bfloat16 *q, __nv_bfloat16 *k, __nv_bfloat16 *vt, int ldv,
                           int planes, cudaStream_t stream);
// conv_out (3 outputs) from its tap-expanded 1x1 product p [pixels][32]: bias + 3x3 tap sum, written as the
// planar image [3][h*w] and RGB bytes [h*w][3] (clamp(x/2 + 0.5, 0, 1) * 255, nearest even; rgb nullable),
// non-finite flag.
int launch_conv_out_gather(const float *p, int h, int w, const float *bias, float *planar, uint8_t *rgb, int *nonfinite,
                           cudaStream_t stream);
// OIHW [cout][cin][9] FP32 -> tap-expanded [9 * cout][cin] (row t * cout + c).
int launch_expand_taps(const float *w, int cout, int cin, float *out, cudaStream_t stream);
// OIHW FP32 [cout][cin][taps] -> conv weights [cout_rows][3 * taps * cin_pad] (three BF16 planes).
int launch_conv_weight_prep(const float *w, int cout, int cin, int taps, int cout_rows, int cin_pad,
                            __nv_bfloat16 *out, int *inexact, cudaStream_t stream);
int launch_synth_f32(uint64_t seed, uint64_t stream_id, float scale, float offset, long long count, int round_bf16,
                     float *out, cudaStream_t stream);
int prepare_conv_kernels();

// ---- text encoder (text.cu) -------------------------------------------------------------------------
// qkv FP32 [tokens][6144] -> rotated head-major q [32][tokens][128], k [8][tokens][128] and v [8][tokens][128].
int launch_text_rope(const float *qkv, const float *cos_t, const float *sin_t, int tokens, float *q, float *k, float *v,
                     cudaStream_t stream);
// Weight-streaming product for the prompt enhancer's decode steps (1..4 rows): y[r][n] = sum_k x[r][k] W[n][k]
// over BF16 weights [n_rows][k] and an A operand in the tensor-core layout ([rows][planes * k] BF16; planes 3:
// x = hi + mid + lo in FP32). F32Out: out[r][n] = y (row stride ldo). Resid: out[r][n] += y. SwiGLU over
// interleaved [up; gate] 64-row groups (n_rows = 2 * ffn): h[r][i] = up_i * silu(gate_i), written as the
// next product's operand (BF16, or three planes with h_split3), with the GEMM epilogue's arithmetic.
enum class GemvEpilogue : int
{
    F32Out = 0,
    Resid = 1,
    SwiGLU = 2,
};
struct GemvArgs
{
    const __nv_bfloat16 *a = nullptr;
    int rows = 0, k = 0, planes = 1;
    const __nv_bfloat16 *w = nullptr;
    int n_rows = 0;
    float *out = nullptr;
    int ldo = 0;
    __nv_bfloat16 *h = nullptr;
    int ffn = 0, h_split3 = 0;
};
int launch_gemv(const GemvArgs &args, GemvEpilogue epilogue, cudaStream_t stream);
int prepare_gemv_kernels(); // shared-memory attribute, before any stream capture
// The chunk's K / V rows (head-major [8][rows][128]) into the caches [8][capacity][128] at rows
// *position.., then (advance) *position += rows.
int launch_pe_cache_append(const float *k, const float *v, int rows, float *k_cache, float *v_cache, int capacity,
                           const int *position, cudaStream_t stream);
int launch_pe_advance(int *position, int rows, cudaStream_t stream);
// The same as the BF16 operands of the tcgen05 attention: q [32][rows_pad][128], k [8][rows_pad][128],
// v^T [8][128][rows_pad].
int launch_text_rope_bf16(const float *qkv, const float *cos_t, const float *sin_t, int tokens, int rows_pad,
                          __nv_bfloat16 *q, __nv_bfloat16 *k, __nv_bfloat16 *vt, cudaStream_t stream);

// Synthetic weights on device (ernie_synth.h protocol). rows x cols BF16 written at `out` with a
// destination row index map: dst_row = (row / group) * group_stride + group_offset + row % group.
int launch_synth_bf16(uint64_t seed, uint64_t stream_id, float scale, float offset, long long rows, int cols,
                      int group, long long group_stride, long long group_offset, __nv_bfloat16 *out,
                      cudaStream_t stream);
// Sets the shared-memory attributes of every kernel once (call before any stream capture).
int prepare_gemm_kernels();
int prepare_attention_kernels();
int launch_synth_f32_bf16(uint64_t seed, uint64_t stream_id, float scale, float offset, long long count, float *out,
                          cudaStream_t stream);
} // namespace ernie_b200
