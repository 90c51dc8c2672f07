"""ctypes binding of the CPU restatement (oracle/liboracle.so) — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this module, and
only as the checker or the timed CPU baseline. The CUDA product never imports it.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

HIDDEN, HEADS, HEAD_DIM, FFN, TEXT_DIM, LATENT = 4096, 32, 128, 12288, 3072, 128
WEIGHT_STD = 0.02

# Stream ids, mirroring include/ernie_synth.h.
WQ, WK, WV, WO, WUP, WGATE, WFC2, GAMMA_SA, GAMMA_MLP, GAMMA_Q, GAMMA_K = range(11)
(X_EMBED_W, X_EMBED_B, TEXT_PROJ_W, TIME1_W, TIME1_B, TIME2_W, TIME2_B, ADALN_W, ADALN_B,
 FINAL_NORM_W, FINAL_NORM_B, FINAL_W, FINAL_B) = range(32, 45)
LATENT_STREAM, TEXT_STREAM, HIDDEN_STREAM, TEMB_STREAM = 48, 49, 50, 51


def block_stream(block, tensor):
    return (block + 1) * 64 + tensor


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = ctypes.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


P = ctypes.c_void_p
I64 = ctypes.c_int64
U64 = ctypes.c_uint64
F = ctypes.c_float
I = ctypes.c_int


class BlockWeightsC(ctypes.Structure):
    _fields_ = [(name, P) for name in
                ("wq", "wk", "wv", "wo", "wup", "wgate", "wfc2", "gamma_sa", "gamma_mlp", "gamma_q", "gamma_k")]


class HeadWeightsC(ctypes.Structure):
    _fields_ = [(name, P) for name in
                ("x_embed_w", "x_embed_b", "text_proj_w", "time1_w", "time1_b", "time2_w", "time2_b",
                 "adaln_w", "adaln_b", "final_norm_w", "final_norm_b", "final_w", "final_b")]


def _declare(l):
    sig = {
        "orc_num_threads": (I, []),
        "orc_set_num_threads": (None, [I]),
        "orc_synth_bf16": (None, [U64, U64, F, F, P, I64]),
        "orc_synth_f32_from_bf16": (None, [U64, U64, F, F, P, I64]),
        "orc_synth_normal_f32": (None, [U64, U64, F, P, I64]),
        "orc_turbo_schedule": (I, [I, P, P]),
        "orc_linear_schedule": (I, [I, P, P]),
        "orc_timestep_features": (I, [F, P]),
        "orc_rope_frequencies": (None, [P]),
        "orc_dit_constants": (I, [P, I, I, I, I, I, P, P, P]),
        "orc_rmsnorm": (None, [P, P, I64, I, F, P]),
        "orc_layernorm": (None, [P, I64, I, F, P]),
        "orc_gelu": (None, [P, P, I64]),
        "orc_silu": (None, [P, P, I64]),
        "orc_residual_add": (None, [P, P, P, I64]),
        "orc_sdpa": (None, [P, P, P, P, I, I, I, I, I, I, I, P]),
        "orc_linear": (None, [P, P, P, I64, I, I, P]),
        "orc_euler_step": (I, [P, P, F, I64, P]),
        "orc_finite": (I, [P, I64]),
        "orc_unpack_for_vae": (I, [P, P, P, I, I, P]),
        "orc_block": (None, [P, ctypes.POINTER(BlockWeightsC), P, P, P, P, I, P]),
        "orc_input_head": (None, [ctypes.POINTER(HeadWeightsC), P, I, I, P, I, P, P, P, P]),
        "orc_output_head": (None, [ctypes.POINTER(HeadWeightsC), P, P, I, I, P]),
        "orc_dit": (None, [ctypes.POINTER(HeadWeightsC), P, I, P, I, I, P, I, P, P, P, P, P]),
        "orc_denoise": (I, [ctypes.POINTER(HeadWeightsC), P, I, P, I, I, P, I, P, P, P, I, I, I, I, P, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(l, name)
        fn.restype = res
        fn.argtypes = args


def ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ---------------------------------------------------------------- synthetic data
def synth_bf16(seed, stream, count, scale=WEIGHT_STD, offset=0.0):
    out = np.empty(count, dtype=np.uint16)
    lib().orc_synth_bf16(seed, stream, scale, offset, ptr(out), count)
    return out


def synth_f32_from_bf16(seed, stream, count, scale=WEIGHT_STD, offset=0.0):
    out = np.empty(count, dtype=np.float32)
    lib().orc_synth_f32_from_bf16(seed, stream, scale, offset, ptr(out), count)
    return out


def synth_normal(seed, stream, count, scale=1.0):
    out = np.empty(count, dtype=np.float32)
    lib().orc_synth_normal_f32(seed, stream, scale, ptr(out), count)
    return out


def bf16_to_f32(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


class BlockWeights:
    """Seeded random-init weights of one DiT block (BF16 bits; norm gammas widened to FP32)."""

    SHAPES = {WQ: (HIDDEN, HIDDEN), WK: (HIDDEN, HIDDEN), WV: (HIDDEN, HIDDEN), WO: (HIDDEN, HIDDEN),
              WUP: (FFN, HIDDEN), WGATE: (FFN, HIDDEN), WFC2: (HIDDEN, FFN)}

    def __init__(self, seed, block):
        self.seed, self.block = seed, block
        self.mats = {t: synth_bf16(seed, block_stream(block, t), int(np.prod(s))).reshape(s)
                     for t, s in self.SHAPES.items()}
        self.gammas = {t: synth_f32_from_bf16(seed, block_stream(block, t), n, WEIGHT_STD, 1.0)
                       for t, n in ((GAMMA_SA, HIDDEN), (GAMMA_MLP, HIDDEN), (GAMMA_Q, HEAD_DIM),
                                    (GAMMA_K, HEAD_DIM))}
        self.c = BlockWeightsC(*(ptr(self.mats[t]) for t in (WQ, WK, WV, WO, WUP, WGATE, WFC2)),
                               *(ptr(self.gammas[t]) for t in (GAMMA_SA, GAMMA_MLP, GAMMA_Q, GAMMA_K)))


class HeadWeights:
    """Seeded random-init input/output head weights (biases are BF16 values held in FP32)."""

    MATS = {X_EMBED_W: (HIDDEN, LATENT), TEXT_PROJ_W: (HIDDEN, TEXT_DIM), TIME1_W: (HIDDEN, HIDDEN),
            TIME2_W: (HIDDEN, HIDDEN), ADALN_W: (6 * HIDDEN, HIDDEN), FINAL_NORM_W: (2 * HIDDEN, HIDDEN),
            FINAL_W: (LATENT, HIDDEN)}
    BIASES = {X_EMBED_B: HIDDEN, TIME1_B: HIDDEN, TIME2_B: HIDDEN, ADALN_B: 6 * HIDDEN,
              FINAL_NORM_B: 2 * HIDDEN, FINAL_B: LATENT}

    def __init__(self, seed):
        self.seed = seed
        self.mats = {t: synth_bf16(seed, t, int(np.prod(s))).reshape(s) for t, s in self.MATS.items()}
        self.biases = {t: synth_f32_from_bf16(seed, t, n) for t, n in self.BIASES.items()}
        m, b = self.mats, self.biases
        self.c = HeadWeightsC(ptr(m[X_EMBED_W]), ptr(b[X_EMBED_B]), ptr(m[TEXT_PROJ_W]), ptr(m[TIME1_W]),
                              ptr(b[TIME1_B]), ptr(m[TIME2_W]), ptr(b[TIME2_B]), ptr(m[ADALN_W]),
                              ptr(b[ADALN_B]), ptr(m[FINAL_NORM_W]), ptr(b[FINAL_NORM_B]), ptr(m[FINAL_W]),
                              ptr(b[FINAL_B]))


def block_modulation(seed, block_input_seed_stream=TEMB_STREAM):
    """Shared adaLN vectors as the reference's block fixture builds them
    (tools/export_dit_block.py:88-90): N(0,1)*0.15, with +0.5 on gate_sa and gate_mlp."""
    mod = synth_normal(seed, block_input_seed_stream, 6 * HIDDEN, 0.15).reshape(6, HIDDEN)
    mod[2] += 0.5
    mod[5] += 0.5
    return mod


# ---------------------------------------------------------------- schedules and constants
def schedule(steps, kind="turbo"):
    sig = np.empty(steps + 1, np.float32)
    ts = np.empty(steps, np.float32)
    fn = lib().orc_turbo_schedule if kind == "turbo" else lib().orc_linear_schedule
    if fn(steps, ptr(sig), ptr(ts)) != 0:
        raise ValueError("Steps must be in [1,1000]")
    return sig, ts


def timestep_features(t):
    out = np.empty(HIDDEN, np.float32)
    if lib().orc_timestep_features(t, ptr(out)) != 0:
        raise ValueError("Timestep must be finite and in [0,1000]")
    return out


def rope_frequencies():
    out = np.empty(64, np.float32)
    lib().orc_rope_frequencies(ptr(out))
    return out


def dit_constants(width, height, valid, text, token_limit=10240, freq=None):
    freq = rope_frequencies() if freq is None else f32(freq)
    n = width * height + text
    cos, sin, mask = np.empty((n, 128), np.float32), np.empty((n, 128), np.float32), np.empty(n, np.float32)
    if lib().orc_dit_constants(ptr(freq), width, height, valid, text, token_limit, ptr(cos), ptr(sin), ptr(mask)):
        raise ValueError("Invalid DiT position dimensions or frequency file")
    return cos, sin, mask


# ---------------------------------------------------------------- operators
def rmsnorm(x, gamma, eps=1e-6):
    x = f32(x)
    out = np.empty_like(x)
    w = x.shape[-1]
    lib().orc_rmsnorm(ptr(x), ptr(f32(gamma)), x.size // w, w, eps, ptr(out))
    return out


def layernorm(x, eps=1e-6):
    x = f32(x)
    out = np.empty_like(x)
    w = x.shape[-1]
    lib().orc_layernorm(ptr(x), x.size // w, w, eps, ptr(out))
    return out


def gelu(x):
    x = f32(x)
    out = np.empty_like(x)
    lib().orc_gelu(ptr(x), ptr(out), x.size)
    return out


def residual_add(a, b):
    a, b = f32(a), f32(b)
    out = np.empty_like(a)
    lib().orc_residual_add(ptr(a), ptr(b), ptr(out), a.size)
    return out


def sdpa(q, k, v, mask=None):
    """q [H,nq,W], k/v [Hk,nk,W], mask [Hm,rows,nk] or [rows,nk] or [nk]."""
    q, k, v = f32(q), f32(k), f32(v)
    heads, nq, width = q.shape
    kv_heads, nk, _ = k.shape
    mh, mr = 1, 1
    if mask is not None:
        mask = f32(mask)
        if mask.ndim == 3:
            mh, mr = mask.shape[0], mask.shape[1]
        elif mask.ndim == 2:
            mr = mask.shape[0]
    out = np.empty_like(q)
    lib().orc_sdpa(ptr(q), ptr(k), ptr(v), ptr(mask), heads, kv_heads, mh, mr, nq, nk, width, ptr(out))
    return out


def linear(a, w_bits, bias=None):
    a = f32(a)
    w_bits = np.ascontiguousarray(w_bits, dtype=np.uint16)
    n, k = w_bits.shape
    m = a.size // k
    out = np.empty((m, n), np.float32)
    lib().orc_linear(ptr(a), ptr(w_bits), ptr(None if bias is None else f32(bias)), m, n, k, ptr(out))
    return out


def euler_step(sample, prediction, delta):
    sample, prediction = f32(sample), f32(prediction)
    out = np.empty_like(sample)
    if lib().orc_euler_step(ptr(sample), ptr(prediction), delta, sample.size, ptr(out)):
        raise ValueError("Incompatible Euler shapes or delta outside [-1,0)")
    return out


def finite(x):
    x = f32(x)
    return bool(lib().orc_finite(ptr(x), x.size))


def unpack_for_vae(packed, mean, variance):
    packed = f32(packed)
    _, h, w = packed.shape
    out = np.empty((32, 2 * h, 2 * w), np.float32)
    if lib().orc_unpack_for_vae(ptr(packed), ptr(f32(mean)), ptr(f32(variance)), w, h, ptr(out)):
        raise ValueError("Invalid BN statistics")
    return out


# ---------------------------------------------------------------- model stages
def block(x, weights, modulation, cos, sin, mask):
    x = f32(x)
    out = np.empty_like(x)
    lib().orc_block(ptr(x), ctypes.byref(weights.c), ptr(f32(modulation)), ptr(f32(cos)), ptr(f32(sin)),
                    ptr(f32(mask)), x.shape[0], ptr(out))
    return out


def input_head(heads, latent, text, features):
    latent, text = f32(latent), f32(text)
    _, h, w = latent.shape
    n = w * h + text.shape[0]
    x = np.empty((n, HIDDEN), np.float32)
    c = np.empty(HIDDEN, np.float32)
    mod = np.empty((6, HIDDEN), np.float32)
    lib().orc_input_head(ctypes.byref(heads.c), ptr(latent), w, h, ptr(text), text.shape[0], ptr(f32(features)),
                         ptr(x), ptr(c), ptr(mod))
    return x, c, mod


def output_head(heads, x, c, width, height):
    out = np.empty((LATENT, height, width), np.float32)
    lib().orc_output_head(ctypes.byref(heads.c), ptr(f32(x)), ptr(f32(c)), width, height, ptr(out))
    return out


def _block_array(blocks):
    arr = (ctypes.POINTER(BlockWeightsC) * len(blocks))(*[ctypes.pointer(b.c) for b in blocks])
    return arr


def dit(heads, blocks, latent, text, features, cos, sin, mask):
    latent = f32(latent)
    _, h, w = latent.shape
    out = np.empty_like(latent)
    arr = _block_array(blocks)
    lib().orc_dit(ctypes.byref(heads.c), ctypes.cast(arr, P), len(blocks), ptr(latent), w, h, ptr(f32(text)),
                  text.shape[0], ptr(f32(features)), ptr(f32(cos)), ptr(f32(sin)), ptr(f32(mask)), ptr(out))
    return out


def denoise(heads, blocks, initial, text, cos, sin, mask, steps, start_step=0, end_step=None, kind="turbo",
            keep_predictions=False):
    initial = f32(initial)
    _, h, w = initial.shape
    end_step = steps if end_step is None else end_step
    out = np.empty_like(initial)
    preds = np.empty((end_step - start_step,) + initial.shape, np.float32) if keep_predictions else None
    arr = _block_array(blocks)
    rc = lib().orc_denoise(ctypes.byref(heads.c), ctypes.cast(arr, P), len(blocks), ptr(initial), w, h,
                           ptr(f32(text)), text.shape[0], ptr(f32(cos)), ptr(f32(sin)), ptr(f32(mask)), steps,
                           start_step, end_step, 0 if kind == "turbo" else 1, ptr(out), ptr(preds))
    if rc < 0:
        raise ValueError("Invalid denoise request")
    if rc > 0:
        raise RuntimeError(f"Non-finite latent after denoise step {rc}")
    return (out, preds) if keep_predictions else out
