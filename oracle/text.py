"""CPU restatement of the prompt encoder's layers — TEST INFRASTRUCTURE ONLY.

Only tests/ and bench.py's CPU-baseline leg use this module, as the checker; the CUDA product never
imports it.

What it restates: run_text_blocks (src/text_encoder.cpp:106-166) runs, per layer, the graph the reference
exports from the pinned transformers MistralDecoderLayer (tools/export_text_block.py:51-61, TextBlock):

    n = rms_norm(x, input_layernorm, 1e-5)
    q, k, v = q_proj(n) [32 heads], k_proj(n), v_proj(n) [8 heads], head width 128
    q, k = rotary(q), rotary(k)        (ExportBlock.rotary, tools/export_dit_block.py:39-47: half-split)
    a = softmax(q k^T / sqrt(128) + causal mask) v    (query head h uses K/V head h // 4)
    x = x + o_proj(a)
    x = x + down_proj(silu(gate_proj(m)) * up_proj(m)),  m = rms_norm(x, post_attention_layernorm, 1e-5)

with the constants of text_constants (src/text_encoder.cpp:76-104): cos/sin of t * f_j repeated over both
halves of the 128-wide row and the causal mask (-FLT_MAX above the diagonal). float64 throughout; the
weights are the exact BF16 values. Synthetic weights follow include/ernie_synth.h's text streams.

The prompt enhancer (src/prompt_enhancer.cpp, src/pe_session.cpp) runs the same layer over its own
checkpoint with a K/V cache: by causality, appending tokens chunk by chunk must give each token the hidden
state of the full causal run, which is what the tests compare against. Its head (head.ncnn.param,
tools/build_pe_model.py:100-105) is rms_norm(h, model.norm) @ lm_head^T.

Parity of values is unpinned: the reference's text fixtures hash in*.f32 / out0.f32 files that are not in
its tree, and the official weights are not available.
"""
import numpy as np

from oracle import WEIGHT_STD, bf16_to_f32, synth_bf16, synth_f32_from_bf16

HIDDEN, Q, KV, HEADS, KV_HEADS, HEAD_DIM, FFN, EPS = 3072, 4096, 1024, 32, 8, 128, 9216, 1e-5
WQ, WK, WV, WO, WGATE, WUP, WDOWN, GAMMA_ATTN, GAMMA_MLP = range(9)
SHAPES = {WQ: (Q, HIDDEN), WK: (KV, HIDDEN), WV: (KV, HIDDEN), WO: (HIDDEN, Q), WGATE: (FFN, HIDDEN),
          WUP: (FFN, HIDDEN), WDOWN: (HIDDEN, FFN)}
NAMES = {WQ: "wq", WK: "wk", WV: "wv", WO: "wo", WGATE: "wgate", WUP: "wup", WDOWN: "wdown",
         GAMMA_ATTN: "gamma_attn", GAMMA_MLP: "gamma_mlp"}


def text_stream(layer, tensor):
    """ERNIE_SYNTH_TEXT_STREAM(layer, tensor)."""
    return 0x54455854 * 4096 + (layer + 1) * 64 + tensor


class TextLayerWeights:
    """Seeded random-init weights of one prompt-encoder layer (BF16 bits; RMSNorm weights as FP32)."""

    def __init__(self, seed, layer):
        self.bits = {t: synth_bf16(seed, text_stream(layer, t), int(np.prod(s))).reshape(s) for t, s in SHAPES.items()}
        self.gammas = {t: synth_f32_from_bf16(seed, text_stream(layer, t), HIDDEN, WEIGHT_STD, 1.0)
                       for t in (GAMMA_ATTN, GAMMA_MLP)}

    def upload_dict(self):
        """The tensors as ernie_cuda.TextModel.upload_layer takes them."""
        d = {NAMES[t]: b for t, b in self.bits.items()}
        d.update({NAMES[t]: g for t, g in self.gammas.items()})
        return d

    def f32(self, t):
        if not hasattr(self, "_f32"):
            self._f32 = {}
        if t not in self._f32:
            self._f32[t] = bf16_to_f32(self.bits[t])
        return self._f32[t]


def text_constants(inv_freq, bucket):
    """cos, sin [bucket][128] as float32 (t * f_j in FP32, both halves repeated)."""
    f = np.asarray(inv_freq, np.float32)
    phase = np.arange(bucket, dtype=np.float32)[:, None] * f[None, :]
    c, s = np.cos(phase.astype(np.float64)), np.sin(phase.astype(np.float64))
    return (np.concatenate([c, c], 1).astype(np.float32), np.concatenate([s, s], 1).astype(np.float32))


def rms_norm(x, gamma):
    return x / np.sqrt((x * x).mean(axis=1, keepdims=True) + EPS) * np.asarray(gamma, np.float64)


def rotary(x, cos, sin):
    """x [T][heads][128]; the half-split rotation with full-width cos/sin rows."""
    c, s = np.asarray(cos, np.float64)[:, None, :], np.asarray(sin, np.float64)[:, None, :]
    first, second = x[..., :64], x[..., 64:]
    return np.concatenate([first * c[..., :64] - second * s[..., :64], second * c[..., 64:] + first * s[..., 64:]], -1)


def layer(w, x, cos, sin):
    """One decoder layer on x [T][3072] (float64)."""
    t = x.shape[0]
    n = rms_norm(x, w.gammas[GAMMA_ATTN])
    q = (n @ w.f32(WQ).T.astype(np.float64)).reshape(t, HEADS, HEAD_DIM)
    k = (n @ w.f32(WK).T.astype(np.float64)).reshape(t, KV_HEADS, HEAD_DIM)
    v = (n @ w.f32(WV).T.astype(np.float64)).reshape(t, KV_HEADS, HEAD_DIM)
    q, k = rotary(q, cos, sin), rotary(k, cos, sin)
    causal = np.triu(np.full((t, t), -np.inf), 1)
    a = np.empty((t, HEADS, HEAD_DIM))
    for h in range(HEADS):
        kv = h // (HEADS // KV_HEADS)
        s = q[:, h] @ k[:, kv].T / np.sqrt(float(HEAD_DIM)) + causal
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        a[:, h] = (p / p.sum(axis=1, keepdims=True)) @ v[:, kv]
    x = x + a.reshape(t, Q) @ w.f32(WO).T.astype(np.float64)
    m = rms_norm(x, w.gammas[GAMMA_MLP])
    g = m @ w.f32(WGATE).T.astype(np.float64)
    u = m @ w.f32(WUP).T.astype(np.float64)
    return x + ((g / (1.0 + np.exp(-g))) * u) @ w.f32(WDOWN).T.astype(np.float64)


def run_blocks(layers, x, cos, sin):
    """run_text_blocks over the given layer weights, in order."""
    x = np.asarray(x, np.float64)
    for w in layers:
        x = layer(w, x, cos, sin)
    return x


HEAD_LAYER = 1023  # ERNIE_SYNTH_TEXT_HEAD_LAYER


def head_weights(seed, rows):
    """The synthetic PE head: final RMSNorm weight [3072] and the first `rows` rows of lm_head (float32)."""
    gamma = synth_f32_from_bf16(seed, text_stream(HEAD_LAYER, 1), HIDDEN, WEIGHT_STD, 1.0)
    w = bf16_to_f32(synth_bf16(seed, text_stream(HEAD_LAYER, 0), rows * HIDDEN).reshape(rows, HIDDEN))
    return gamma, w


def head_logits(gamma, w, hidden):
    """Logits of one hidden row against the given lm_head rows (float64)."""
    h = np.asarray(hidden, np.float64).reshape(1, HIDDEN)
    return (rms_norm(h, gamma) @ np.asarray(w, np.float64).T)[0]
