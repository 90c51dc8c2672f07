"""CPU restatement of the VAE decoder and encoder stages — TEST INFRASTRUCTURE ONLY.

Only tests/ and bench.py's CPU-baseline leg use this module, as the checker; the CUDA product never
imports it.

What it restates:
* decode_vae (src/vae.cpp:18-64) runs the reference's exported graph of the pinned diffusers
  AutoencoderKLFlux2 (diffusers 0.41.0.dev0 at commit 7643c482, not vendored in the reference tree):
  decoder(post_quant_conv(x)) (tools/export_vae.py:33-39), whose layer list is
  artifacts/2026-09-05/pipeline/models/vae-128x128-specialized-v1/head.ncnn.param (committed in
  execution order as tests/golden/vae_decoder_graph.json). The published architecture of that decoder:
  conv_in 3x3; mid block = resnet, single-head attention over all pixels (GroupNorm, q/k/v/out linear
  projections, softmax(q k^T / sqrt(512)) v, residual), resnet; four up blocks of three resnets with
  nearest x2 upsampling + 3x3 conv after the first three; GroupNorm + Swish; conv_out 3x3.
  ResnetBlock2D: shortcut(x) + conv2(swish(norm2(conv1(swish(norm1(x)))))), shortcut a 1x1 conv where
  the width changes.
* GroupNorm as the reference's CPU layer computes it (src/ernie_groupnorm.cpp:33-64): per group, the
  mean and the centred variance in FP64, then x * (gamma / sqrt(var + eps)) + beta.
* Swish as ncnn evaluates it: x / (1 + exp(-x)).
* rgb_image (src/pipeline.cpp:145-163): byte = nearbyint(clamp(x / 2 + 0.5, 0, 1) * 255) in FP32,
  non-finite values rejected.
* encode_vae (src/image_encoder.cpp:28-72): RGB bytes -> (v - 127.5f) * (1 / 127.5f) in FP32
  (image_encoder.cpp:44-51, tools/export_vae_encoder.py:30-34), then the traced wrapper of
  tools/export_vae_encoder.py:74-80 over the same pinned AutoencoderKLFlux2: mean =
  quant_conv(encoder(x))[:32] (the posterior's mode), packed = pixel_unshuffle(mean, 2), normalized =
  BatchNorm2d(128, eps 1e-4, affine=False, eval) of packed. The published encoder: conv_in 3x3 3->128;
  four down blocks of two resnets (128, 256, 512, 512 channels) with a 3x3 stride-2 convolution after
  the first three, its input padded by one zero row and column at the bottom and right; the same mid
  block as the decoder; GroupNorm + Swish; conv_out 3x3 512->64.

The arithmetic is float64 throughout (the reference's CPU path is FP32); the reference's gates absorb
the difference. Parity of values is unpinned: the reference ships no decoder output fixture (the
fixture's in0/out0 tensors are not in its tree); the decoder graph's topology is pinned by the golden
JSON. The encoder has neither an exported graph nor output tensors in the reference tree: its topology
follows the export script's wrapper and the published architecture, and its values are unpinned too.

Synthetic weights follow include/ernie_synth.h's VAE rule (stream = FNV-1a 64 of the diffusers name).
"""
import numpy as np

from oracle import synth_normal

GROUPS, EPS, WIDTH = 32, 1e-6, 512
UP_OUT = (512, 512, 256, 128)
DOWN_OUT = (128, 256, 512, 512)
BN_EPS = 1e-4  # the encoder's BatchNorm (tools/export_vae_encoder.py:58,93)


class _Table:
    """Builder of [(diffusers name, shape)] lists."""

    def __init__(self):
        self.t = []

    def conv(self, name, cin, cout, k):
        self.t.extend([(name + ".weight", (cout, cin, k, k)), (name + ".bias", (cout,))])

    def norm(self, name, c):
        self.t.extend([(name + ".weight", (c,)), (name + ".bias", (c,))])

    def resnet(self, name, cin, cout):
        self.norm(name + ".norm1", cin)
        self.conv(name + ".conv1", cin, cout, 3)
        self.norm(name + ".norm2", cout)
        self.conv(name + ".conv2", cout, cout, 3)
        if cin != cout:
            self.conv(name + ".conv_shortcut", cin, cout, 1)

    def mid_block(self, prefix):
        self.resnet(prefix + "mid_block.resnets.0", 512, 512)
        a = prefix + "mid_block.attentions.0."
        self.norm(a + "group_norm", 512)
        for p in ("to_q", "to_k", "to_v", "to_out.0"):
            self.t.extend([(a + p + ".weight", (512, 512)), (a + p + ".bias", (512,))])
        self.resnet(prefix + "mid_block.resnets.1", 512, 512)


def encoder_table():
    """[(diffusers name, shape)] of the encoder + quant_conv + bn in execution order."""
    b = _Table()
    b.conv("encoder.conv_in", 3, 128, 3)
    c = 128
    for i, cout in enumerate(DOWN_OUT):
        for j in range(2):
            b.resnet(f"encoder.down_blocks.{i}.resnets.{j}", c, cout)
            c = cout
        if i < 3:
            b.conv(f"encoder.down_blocks.{i}.downsamplers.0.conv", c, c, 3)
    b.mid_block("encoder.")
    b.norm("encoder.conv_norm_out", 512)
    b.conv("encoder.conv_out", 512, 64, 3)
    b.conv("quant_conv", 64, 64, 1)
    b.t.extend([("bn.running_mean", (128,)), ("bn.running_var", (128,))])
    return b.t


def tensor_table():
    """[(diffusers name, shape)] of the decoder in execution order."""
    t = [("post_quant_conv.weight", (32, 32, 1, 1)), ("post_quant_conv.bias", (32,))]

    def conv(name, cin, cout, k):
        t.extend([(name + ".weight", (cout, cin, k, k)), (name + ".bias", (cout,))])

    def norm(name, c):
        t.extend([(name + ".weight", (c,)), (name + ".bias", (c,))])

    def resnet(name, cin, cout):
        norm(name + ".norm1", cin)
        conv(name + ".conv1", cin, cout, 3)
        norm(name + ".norm2", cout)
        conv(name + ".conv2", cout, cout, 3)
        if cin != cout:
            conv(name + ".conv_shortcut", cin, cout, 1)

    conv("decoder.conv_in", 32, 512, 3)
    resnet("decoder.mid_block.resnets.0", 512, 512)
    a = "decoder.mid_block.attentions.0."
    norm(a + "group_norm", 512)
    for p in ("to_q", "to_k", "to_v", "to_out.0"):
        t.extend([(a + p + ".weight", (512, 512)), (a + p + ".bias", (512,))])
    resnet("decoder.mid_block.resnets.1", 512, 512)
    c = 512
    for i, cout in enumerate(UP_OUT):
        for j in range(3):
            resnet(f"decoder.up_blocks.{i}.resnets.{j}", c, cout)
            c = cout
        if i < 3:
            conv(f"decoder.up_blocks.{i}.upsamplers.0.conv", c, c, 3)
    norm("decoder.conv_norm_out", 128)
    conv("decoder.conv_out", 128, 3, 3)
    return t


def name_stream(name):
    """FNV-1a 64 of the name (ernie_synth_name_stream)."""
    h = 0xCBF29CE484222325
    for b in name.encode():
        h = ((h ^ b) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def synth_rule(name, shape):
    """(scale, offset, is a convolution/projection weight) of include/ernie_synth.h's VAE rule."""
    if len(shape) >= 2:
        fan_in = int(np.prod(shape[1:]))
        fp32_layer = name.startswith(("post_quant_conv", "quant_conv"))  # computed in FP32, never rounded
        return np.float32(1.0) / np.sqrt(np.float32(fan_in)), np.float32(0.0), not fp32_layer
    if name == "bn.running_var":
        return np.float32(0.1), np.float32(1.0), False
    if "norm" in name:
        return np.float32(0.1), np.float32(1.0 if name.endswith(".weight") else 0.0), False
    return np.float32(0.02), np.float32(0.0), False


def bf16_round(x):
    bits = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
    return rounded.astype(np.uint32).view(np.float32)


def synth_weights(seed, bf16_weights=False, table=None):
    """{name: float32 array} as ernie_cuda_vae_synthesize (ernie_cuda_vae_encoder_synthesize with
    table=encoder_table()) makes them."""
    out = {}
    for name, shape in (table if table is not None else tensor_table()):
        scale, offset, is_weight = synth_rule(name, shape)
        v = synth_normal(seed, name_stream(name), int(np.prod(shape)), float(scale)) + offset
        if bf16_weights and is_weight:
            v = bf16_round(v)
        out[name] = v.reshape(shape)
    return out


# ---- layers (float64) --------------------------------------------------------------------------------
def conv2d(x, w, b):
    """Stride-1 convolution with same padding: x [C][H][W], w [O][C][k][k]."""
    c, h, wd = x.shape
    o, _, k, _ = w.shape
    w = np.asarray(w, np.float64)
    if k == 1:
        y = w.reshape(o, c) @ x.reshape(c, h * wd)
    else:
        xp = np.pad(x, ((0, 0), (1, 1), (1, 1)))
        cols = np.empty((c, 9, h, wd))
        for ky in range(3):
            for kx in range(3):
                cols[:, ky * 3 + kx] = xp[:, ky:ky + h, kx:kx + wd]
        y = w.reshape(o, c * 9) @ cols.reshape(c * 9, h * wd)
    return (y + np.asarray(b, np.float64)[:, None]).reshape(o, h, wd)


def group_norm(x, gamma, beta, groups=GROUPS, eps=EPS):
    c = x.shape[0]
    g = x.reshape(groups, -1)
    mean = g.mean(axis=1, keepdims=True)
    var = ((g - mean) ** 2).mean(axis=1, keepdims=True)
    y = ((g - mean) / np.sqrt(var + eps)).reshape(x.shape)
    return y * np.asarray(gamma, np.float64).reshape(c, 1, 1) + np.asarray(beta, np.float64).reshape(c, 1, 1)


def swish(x):
    return x / (1.0 + np.exp(-x))


def resnet(w, name, x):
    h = conv2d(swish(group_norm(x, w[name + ".norm1.weight"], w[name + ".norm1.bias"])),
               w[name + ".conv1.weight"], w[name + ".conv1.bias"])
    h = conv2d(swish(group_norm(h, w[name + ".norm2.weight"], w[name + ".norm2.bias"])),
               w[name + ".conv2.weight"], w[name + ".conv2.bias"])
    if name + ".conv_shortcut.weight" in w:
        x = conv2d(x, w[name + ".conv_shortcut.weight"], w[name + ".conv_shortcut.bias"])
    return x + h


def attention(w, x, a="decoder.mid_block.attentions.0."):
    c, h, wd = x.shape
    t = group_norm(x, w[a + "group_norm.weight"], w[a + "group_norm.bias"]).reshape(c, h * wd).T

    def linear(p, v):
        return v @ np.asarray(w[a + p + ".weight"], np.float64).T + np.asarray(w[a + p + ".bias"], np.float64)

    q, k, v = linear("to_q", t), linear("to_k", t), linear("to_v", t)
    s = (q @ k.T) / np.sqrt(float(c))
    s -= s.max(axis=1, keepdims=True)
    e = np.exp(s)
    o = (e / e.sum(axis=1, keepdims=True)) @ v
    return x + linear("to_out.0", o).T.reshape(c, h, wd)


def decode(w, unpacked):
    """decoder(post_quant_conv(unpacked)): [32][h][w] -> [3][8h][8w] (float64)."""
    x = conv2d(np.asarray(unpacked, np.float64), w["post_quant_conv.weight"], w["post_quant_conv.bias"])
    x = conv2d(x, w["decoder.conv_in.weight"], w["decoder.conv_in.bias"])
    x = resnet(w, "decoder.mid_block.resnets.0", x)
    x = attention(w, x)
    x = resnet(w, "decoder.mid_block.resnets.1", x)
    for i in range(4):
        for j in range(3):
            x = resnet(w, f"decoder.up_blocks.{i}.resnets.{j}", x)
        if i < 3:
            x = np.repeat(np.repeat(x, 2, axis=1), 2, axis=2)
            x = conv2d(x, w[f"decoder.up_blocks.{i}.upsamplers.0.conv.weight"],
                       w[f"decoder.up_blocks.{i}.upsamplers.0.conv.bias"])
    x = swish(group_norm(x, w["decoder.conv_norm_out.weight"], w["decoder.conv_norm_out.bias"]))
    return conv2d(x, w["decoder.conv_out.weight"], w["decoder.conv_out.bias"])


def rgb_image(decoded):
    """rgb_image (src/pipeline.cpp:145-163): FP32 [3][H][W] -> bytes [H][W][3]; raises on non-finite."""
    d = np.asarray(decoded, np.float32)
    if not np.isfinite(d).all():
        raise ValueError("VAE produced non-finite pixels")
    n = np.clip(d / np.float32(2.0) + np.float32(0.5), np.float32(0.0), np.float32(1.0))
    return np.rint(n * np.float32(255.0)).astype(np.uint8).transpose(1, 2, 0).copy()


# ---- encoder -------------------------------------------------------------------------------------------
def normalize_rgb(rgb):
    """RGB bytes [H][W][3] -> FP32 [3][H][W] as (v - 127.5f) * (1 / 127.5f) (src/image_encoder.cpp:44-51)."""
    v = np.asarray(rgb, np.uint8).astype(np.float32)
    return ((v - np.float32(127.5)) * np.float32(1.0 / 127.5)).transpose(2, 0, 1).copy()


def downsample(x, w, b):
    """Downsample2D(padding=0): zero row/column appended at the bottom/right, then a 3x3 stride-2 conv."""
    c, h, wd = x.shape
    o = w.shape[0]
    xp = np.pad(x, ((0, 0), (0, 1), (0, 1)))
    oh, ow = h // 2, wd // 2
    cols = np.empty((c, 9, oh, ow))
    for ky in range(3):
        for kx in range(3):
            cols[:, ky * 3 + kx] = xp[:, ky:ky + 2 * oh:2, kx:kx + 2 * ow:2]
    y = np.asarray(w, np.float64).reshape(o, c * 9) @ cols.reshape(c * 9, oh * ow)
    return (y + np.asarray(b, np.float64)[:, None]).reshape(o, oh, ow)


def pixel_unshuffle(x, r=2):
    """out[c * r * r + i * r + j][y][x] = in[c][y * r + i][x * r + j] (torch pixel_unshuffle)."""
    c, h, wd = x.shape
    return x.reshape(c, h // r, r, wd // r, r).transpose(0, 2, 4, 1, 3).reshape(c * r * r, h // r, wd // r)


def encode(w, rgb):
    """(mean [32][H/8][W/8], packed [128][H/16][W/16], normalized [128][H/16][W/16]) in float64."""
    x = conv2d(normalize_rgb(rgb).astype(np.float64), w["encoder.conv_in.weight"], w["encoder.conv_in.bias"])
    for i in range(4):
        for j in range(2):
            x = resnet(w, f"encoder.down_blocks.{i}.resnets.{j}", x)
        if i < 3:
            x = downsample(x, w[f"encoder.down_blocks.{i}.downsamplers.0.conv.weight"],
                           w[f"encoder.down_blocks.{i}.downsamplers.0.conv.bias"])
    x = resnet(w, "encoder.mid_block.resnets.0", x)
    x = attention(w, x, "encoder.mid_block.attentions.0.")
    x = resnet(w, "encoder.mid_block.resnets.1", x)
    x = swish(group_norm(x, w["encoder.conv_norm_out.weight"], w["encoder.conv_norm_out.bias"]))
    x = conv2d(x, w["encoder.conv_out.weight"], w["encoder.conv_out.bias"])
    mean = conv2d(x, w["quant_conv.weight"], w["quant_conv.bias"])[:32]
    packed = pixel_unshuffle(mean)
    rm = np.asarray(w["bn.running_mean"], np.float64)[:, None, None]
    rv = np.asarray(w["bn.running_var"], np.float64)[:, None, None]
    return mean, packed, (packed - rm) / np.sqrt(rv + BN_EPS)


def rgb_fixture(width, height):
    """Deterministic RGB test pattern of the reference's encoder fixtures (tools/export_vae_encoder.py:25-28)."""
    y, x, c = np.indices((height, width, 3), dtype=np.int32)
    return ((13 * x + 29 * y + 71 * c + (x * y) % 19) % 256).astype(np.uint8)
