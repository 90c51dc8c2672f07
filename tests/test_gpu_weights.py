"""Official checkpoint loading on a B200: safetensors files under the official tensor names, written from the
seeded weights, load into the models bit for bit as the device-side synthesis makes them (compared through
each model's output: a DiT prediction, the prompt encoder's hidden state, a VAE decode)."""
import numpy as np
import pytest

import ernie_cuda as ec
import oracle as o
import text as ot
import vae as ov
from conftest import write_safetensors

pytestmark = pytest.mark.gpu
SEED = 5
BLOCK_NAMES = {o.WQ: "self_attention.to_q.weight", o.WK: "self_attention.to_k.weight",
               o.WV: "self_attention.to_v.weight", o.WO: "self_attention.to_out.0.weight",
               o.WUP: "mlp.up_proj.weight", o.WGATE: "mlp.gate_proj.weight", o.WFC2: "mlp.linear_fc2.weight"}
GAMMA_NAMES = {o.GAMMA_SA: "adaLN_sa_ln.weight", o.GAMMA_MLP: "adaLN_mlp_ln.weight",
               o.GAMMA_Q: "self_attention.norm_q.weight", o.GAMMA_K: "self_attention.norm_k.weight"}
HEAD_MATS = {o.X_EMBED_W: "x_embedder.proj.weight", o.TEXT_PROJ_W: "text_proj.weight",
             o.TIME1_W: "time_embedding.linear_1.weight", o.TIME2_W: "time_embedding.linear_2.weight",
             o.ADALN_W: "adaLN_modulation.1.weight", o.FINAL_NORM_W: "final_norm.linear.weight",
             o.FINAL_W: "final_linear.weight"}
HEAD_BIASES = {o.X_EMBED_B: "x_embedder.proj.bias", o.TIME1_B: "time_embedding.linear_1.bias",
               o.TIME2_B: "time_embedding.linear_2.bias", o.ADALN_B: "adaLN_modulation.1.bias",
               o.FINAL_NORM_B: "final_norm.linear.bias", o.FINAL_B: "final_linear.bias"}
TEXT_NAMES = {ot.WQ: "self_attn.q_proj.weight", ot.WK: "self_attn.k_proj.weight", ot.WV: "self_attn.v_proj.weight",
              ot.WO: "self_attn.o_proj.weight", ot.WGATE: "mlp.gate_proj.weight", ot.WUP: "mlp.up_proj.weight",
              ot.WDOWN: "mlp.down_proj.weight"}


def bits(x):
    """BF16 bits of FP32 values that are BF16 values."""
    return (np.ascontiguousarray(x, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def test_dit_checkpoint_in_two_shards(ctx, tmp_path):
    blocks = {}
    for b in range(2):
        w = o.BlockWeights(SEED, b)
        for t, n in BLOCK_NAMES.items():
            blocks[f"layers.{b}.{n}"] = ("BF16", w.mats[t])
        for t, n in GAMMA_NAMES.items():
            blocks[f"layers.{b}.{n}"] = ("BF16", bits(w.gammas[t]))
    h = o.HeadWeights(SEED)
    heads = {n: ("BF16", h.mats[t]) for t, n in HEAD_MATS.items()}
    heads["x_embedder.proj.weight"] = ("BF16", h.mats[o.X_EMBED_W].reshape(4096, 128, 1, 1))  # the 1x1 conv
    heads.update({n: ("BF16", bits(h.biases[t])) for t, n in HEAD_BIASES.items()})
    shard1, shard2 = str(tmp_path / "dit-1.safetensors"), str(tmp_path / "dit-2.safetensors")
    write_safetensors(shard1, blocks)
    write_safetensors(shard2, heads)
    synth, loaded = ec.Model(ctx, 2), ec.Model(ctx, 2)
    try:
        synth.synthesize(SEED)
        loaded.load_safetensors([shard1, shard2])
        w, hh, text, valid = 4, 4, 8, 6
        rng = np.random.default_rng(0)
        latent = rng.standard_normal((128, hh, w)).astype(np.float32)
        txt = rng.standard_normal((text, 3072)).astype(np.float32)
        cos, sin, mask = ec.dit_constants(w, hh, valid, text)
        out = []
        for m in (synth, loaded):
            s = ec.Session(m, w, hh, text, valid, ec.BF16)
            try:
                s.set_conditioning(txt, cos, sin, mask)
                out.append(s.dit(latent, 500.0))
            finally:
                s.close()
        assert np.isfinite(out[0]).all() and np.array_equal(out[0], out[1])
        three = ec.Model(ctx, 3)
        try:
            with pytest.raises(ec.CudaError, match="Missing tensor"):
                three.load_safetensors([shard1, shard2])  # no block 2 in the files
        finally:
            three.close()
    finally:
        synth.close()
        loaded.close()


def test_text_checkpoint(ctx, tmp_path):
    tensors = {}
    for layer in range(2):
        w = ot.TextLayerWeights(SEED, layer)
        p = f"language_model.model.layers.{layer}."
        tensors.update({p + n: ("BF16", w.bits[t]) for t, n in TEXT_NAMES.items()})
        tensors[p + "input_layernorm.weight"] = ("BF16", bits(w.gammas[ot.GAMMA_ATTN]))
        tensors[p + "post_attention_layernorm.weight"] = ("BF16", bits(w.gammas[ot.GAMMA_MLP]))
    path = str(tmp_path / "text.safetensors")
    write_safetensors(path, tensors)
    synth, loaded = ec.TextModel(ctx, 2), ec.TextModel(ctx, 2)
    try:
        synth.synthesize(SEED)
        loaded.load_safetensors(path)
        x = (np.random.default_rng(1).standard_normal((20, 3072)) * 0.2).astype(np.float32)
        cos, sin, _ = ec.text_constants((1.0 / 1000000.0 ** (np.arange(64) / 64)).astype(np.float32), 20)
        a, b = synth.run_blocks(x, cos, sin), loaded.run_blocks(x, cos, sin)
        assert np.isfinite(a).all() and np.array_equal(a, b)
    finally:
        synth.close()
        loaded.close()


@pytest.mark.parametrize("bf16", [False, True], ids=["f32", "bf16"])
def test_vae_checkpoint(ctx, tmp_path, bf16):
    weights = ov.synth_weights(SEED, bf16_weights=bf16)
    tensors = {}
    for name, shape in ov.tensor_table():
        _, _, is_weight = ov.synth_rule(name, shape)
        tensors[name] = ("BF16", bits(weights[name])) if bf16 and is_weight else ("F32", weights[name])
    path = str(tmp_path / "vae.safetensors")
    write_safetensors(path, tensors)
    synth, loaded = ec.Vae(ctx), ec.Vae(ctx)
    try:
        synth.synthesize(SEED, bf16_weights=bf16)
        loaded.load_safetensors(path)
        u = np.random.default_rng(2).standard_normal((32, 6, 10)).astype(np.float32)
        for precision in (ec.BF16, ec.FP32):
            a, _, _ = synth.decode(u, precision)
            b, _, _ = loaded.decode(u, precision)
            assert np.isfinite(a).all() and np.array_equal(a, b)
    finally:
        synth.close()
        loaded.close()


def test_vae_encoder_checkpoint(ctx, tmp_path):
    """The official VAE file holds encoder.*, quant_conv.* and bn.* beside the decoder's tensors (here BF16
    convolution weights, FP32 vectors, and a decoder tensor the encoder skips)."""
    weights = ov.synth_weights(SEED, bf16_weights=True, table=ov.encoder_table())
    tensors = {}
    for name, shape in ov.encoder_table():
        _, _, is_weight = ov.synth_rule(name, shape)
        tensors[name] = ("BF16", bits(weights[name])) if is_weight else ("F32", weights[name])
    tensors["decoder.conv_in.bias"] = ("F32", np.zeros(512, np.float32))
    path = str(tmp_path / "vae.safetensors")
    write_safetensors(path, tensors)
    synth, loaded = ec.VaeEncoder(ctx), ec.VaeEncoder(ctx)
    try:
        synth.synthesize(SEED, bf16_weights=True)
        loaded.load_safetensors(path)
        rgb = np.random.default_rng(3).integers(0, 256, (32, 48, 3), dtype=np.uint8)
        for precision in (ec.BF16, ec.FP32):
            a, b = synth.encode(rgb, precision), loaded.encode(rgb, precision)
            for x, y in zip(a[:3], b[:3]):
                assert np.isfinite(x).all() and np.array_equal(x, y)
    finally:
        synth.close()
        loaded.close()
