"""VAE encoder stage on the CPU: the reference's normalisation known answers, the oracle's layers against
direct restatements, and the library's tensor table against the oracle's (encode_vae,
src/image_encoder.cpp:28-72, over the wrapper of tools/export_vae_encoder.py:74-80)."""
import numpy as np
import pytest

import ernie_cuda as ec
import vae as ov


def test_normalization_known_answers():
    """tests/test_img2img_encoder.py:16-23: 0 -> -1, 255 -> 1, 127 -> (127 - 127.5f) * (1 / 127.5f) in FP32."""
    x = ov.normalize_rgb(np.array([[[0, 127, 255]]], np.uint8))
    assert x.shape == (3, 1, 1) and x.dtype == np.float32
    assert x[0, 0, 0] == np.float32(-1) and x[2, 0, 0] == np.float32(1)
    expected = np.float32(np.float32(127) - np.float32(127.5)) * np.float32(1 / 127.5)
    assert x[1, 0, 0].view(np.uint32) == expected.view(np.uint32)


def test_rgb_fixture_pattern():
    rgb = ov.rgb_fixture(32, 16)
    assert rgb.shape == (16, 32, 3) and rgb.dtype == np.uint8
    assert np.array_equal(rgb, ov.rgb_fixture(32, 16))
    y, x, c = 5, 7, 2
    assert rgb[y, x, c] == (13 * x + 29 * y + 71 * c + (x * y) % 19) % 256


def test_pixel_unshuffle_against_loops():
    x = np.random.default_rng(1).standard_normal((3, 6, 8))
    u = ov.pixel_unshuffle(x)
    assert u.shape == (12, 3, 4)
    for c in range(3):
        for i in range(2):
            for j in range(2):
                for yy in range(3):
                    for xx in range(4):
                        assert u[c * 4 + i * 2 + j, yy, xx] == x[c, 2 * yy + i, 2 * xx + j]


def test_downsample_against_direct_sum():
    """3x3 stride 2 with one zero row/column appended at the bottom/right (Downsample2D, padding=0)."""
    rng = np.random.default_rng(2)
    x = rng.standard_normal((3, 6, 8))
    w = rng.standard_normal((4, 3, 3, 3))
    b = rng.standard_normal(4)
    got = ov.downsample(x, w, b)
    assert got.shape == (4, 3, 4)
    for o in range(4):
        for oy in range(3):
            for ox in range(4):
                acc = b[o]
                for c in range(3):
                    for ky in range(3):
                        for kx in range(3):
                            yy, xx = 2 * oy + ky, 2 * ox + kx
                            if yy < 6 and xx < 8:
                                acc += w[o, c, ky, kx] * x[c, yy, xx]
                assert abs(got[o, oy, ox] - acc) < 1e-12


def test_library_and_oracle_tables_agree():
    assert ec.vae_encoder_tensors() == ov.encoder_table()


def test_encoder_table_structure():
    """conv_in 3->128; down blocks 128, 256, 512, 512 with 1x1 shortcuts where the width changes and three
    same-width 3x3 downsamplers; the decoder's mid block (same shapes); conv_out 512->64 (mean and log-variance);
    quant_conv 64x64; the 128-channel BatchNorm of the packed latent."""
    table = dict(ov.encoder_table())
    assert table["encoder.conv_in.weight"] == (128, 3, 3, 3)
    assert [table[f"encoder.down_blocks.{i}.downsamplers.0.conv.weight"] for i in range(3)] == [
        (128, 128, 3, 3), (256, 256, 3, 3), (512, 512, 3, 3)]
    assert "encoder.down_blocks.3.downsamplers.0.conv.weight" not in table
    shortcuts = sorted(n for n in table if "conv_shortcut.weight" in n)
    assert shortcuts == ["encoder.down_blocks.1.resnets.0.conv_shortcut.weight",
                         "encoder.down_blocks.2.resnets.0.conv_shortcut.weight"]
    decoder = dict(ov.tensor_table())
    mid_enc = {n[len("encoder."):]: s for n, s in table.items() if n.startswith("encoder.mid_block.")}
    mid_dec = {n[len("decoder."):]: s for n, s in decoder.items() if n.startswith("decoder.mid_block.")}
    assert mid_enc == mid_dec
    assert table["encoder.conv_out.weight"] == (64, 512, 3, 3)
    assert table["quant_conv.weight"] == (64, 64, 1, 1)
    assert table["bn.running_mean"] == table["bn.running_var"] == (128,)


def test_encode_shapes_and_batch_norm():
    w = ov.synth_weights(7, table=ov.encoder_table())
    assert (w["bn.running_var"] > 0).all()
    mean, packed, normalized = ov.encode(w, ov.rgb_fixture(32, 48))
    assert mean.shape == (32, 6, 4) and packed.shape == (128, 3, 2) and normalized.shape == (128, 3, 2)
    assert np.array_equal(packed, ov.pixel_unshuffle(mean))
    rm, rv = (w[n].astype(np.float64)[:, None, None] for n in ("bn.running_mean", "bn.running_var"))
    expect = (packed - rm) / np.sqrt(rv + 1e-4)
    assert np.allclose(normalized, expect, rtol=0, atol=1e-12)


def test_bf16_weight_rounding_spares_the_fp32_layers():
    w = ov.synth_weights(7, bf16_weights=True, table=ov.encoder_table())
    assert np.array_equal(w["encoder.conv_in.weight"], ov.bf16_round(w["encoder.conv_in.weight"]))
    assert not np.array_equal(w["quant_conv.weight"], ov.bf16_round(w["quant_conv.weight"]))
