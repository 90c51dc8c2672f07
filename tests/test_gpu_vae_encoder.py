"""VAE encoder on a B200 (encode_vae, src/image_encoder.cpp:28-72) against the CPU oracle (oracle/vae.py
encode) on seeded synthetic weights.

Gates (atol, rtol, nrmse) are the reference's encoder fixture gate (tools/export_vae_encoder.py:97: fp32
{2e-4, 2e-4, 2e-5}) for FP32-exact mode on all three outputs (mean, packed, normalized), the component
FP16 gate (tools/export_dit_heads.py:88-90) for BF16 mode, and the BF16 gate between the two modes at
sizes the oracle cannot reach in seconds.
"""
import numpy as np
import pytest

import ernie_cuda as ec
import vae as ov
from conftest import gate

pytestmark = pytest.mark.gpu
SEED = 13
ENC_FP32 = (2e-4, 2e-4, 2e-5)
ENC_FP16 = (0.03, 0.03, 0.02)
ENC_BF16 = (0.2, 0.2, 0.1)


@pytest.fixture(scope="module")
def weights():
    return ov.synth_weights(SEED, table=ov.encoder_table())


@pytest.fixture(scope="module")
def encoder(ctx):
    e = ec.VaeEncoder(ctx)
    e.synthesize(SEED)
    yield e
    e.close()


def image(width, height, seed=None):
    if seed is None:
        return ov.rgb_fixture(width, height)
    return np.random.default_rng(seed).integers(0, 256, (height, width, 3), dtype=np.uint8)


def check_outputs(ref, got, gates, label):
    for name, r, g in zip(("mean", "packed", "normalized"), ref, got):
        assert r.shape == g.shape, (name, r.shape, g.shape)
        ok, metrics = gate(r, g, *gates)
        print(label, name, metrics)
        assert ok, (name, metrics)


# the reference's reviewed small shapes (32x32, 64x32) and a ragged one
@pytest.mark.parametrize("shape", [(32, 32), (64, 32), (48, 80)])
@pytest.mark.parametrize("precision", [ec.FP32, ec.BF16], ids=["fp32", "bf16"])
def test_encode_against_oracle(encoder, weights, shape, precision):
    rgb = image(*shape, seed=None if shape != (48, 80) else 3)
    ref = ov.encode(weights, rgb)
    mean, packed, normalized, bad = encoder.encode(rgb, precision)
    assert bad == 0
    check_outputs(ref, (mean, packed, normalized), ENC_FP32 if precision == ec.FP32 else ENC_FP16,
                  f"VAE encode {shape} {'fp32' if precision == ec.FP32 else 'bf16'}")
    assert np.array_equal(packed, ov.pixel_unshuffle(mean)), "packed must be mean's pixel_unshuffle bit for bit"


def test_bf16_weights_take_the_three_product_path(ctx):
    w = ov.synth_weights(SEED + 1, bf16_weights=True, table=ov.encoder_table())
    e = ec.VaeEncoder(ctx)
    try:
        e.synthesize(SEED + 1, bf16_weights=True)
        rgb = image(32, 48, seed=5)
        got = e.encode(rgb, ec.FP32)[:3]
    finally:
        e.close()
    check_outputs(ov.encode(w, rgb), got, ENC_FP32, "VAE encode, BF16 weights, FP32-exact")


def test_uploaded_weights_equal_synthesized(ctx, encoder, weights):
    e = ec.VaeEncoder(ctx)
    try:
        for name, array in weights.items():
            e.upload(name, array)
        rgb = image(32, 32, seed=6)
        for precision in (ec.FP32, ec.BF16):
            a, b = e.encode(rgb, precision), encoder.encode(rgb, precision)
            for x, y in zip(a[:3], b[:3]):
                assert np.array_equal(x, y)
    finally:
        e.close()


def test_repeat_and_shape_switch_are_bit_exact(encoder):
    a, b = image(64, 32, seed=7), image(32, 96, seed=8)
    first = encoder.encode(a, ec.BF16)
    other = encoder.encode(b, ec.BF16)
    again = encoder.encode(a, ec.BF16)
    assert other[0].shape == (32, 12, 4)
    for x, y in zip(first[:3], again[:3]):
        assert np.array_equal(x, y)


def test_device_entry_matches_host_entry(ctx, encoder):
    rgb = image(48, 32, seed=9)
    host = encoder.encode(rgb, ec.BF16)
    src = ctx.to_device(rgb)
    outs = [ctx.buffer(x.nbytes) for x in host[:3]]
    try:
        encoder.encode_device(src, 48, 32, *outs, precision=ec.BF16)
        ctx.synchronize()
        for buf, x in zip(outs, host[:3]):
            assert np.array_equal(buf.download(x.shape), x)
    finally:
        src.free()
        for b in outs:
            b.free()


def test_nonfinite_output_is_flagged(ctx):
    e = ec.VaeEncoder(ctx)
    try:
        e.synthesize(SEED)
        e.upload("encoder.conv_out.bias", np.full(64, 1e38, np.float32))
        e.upload("quant_conv.weight", np.ones((64, 64, 1, 1), np.float32))
        _, _, normalized, bad = e.encode(image(32, 32), ec.BF16)
        assert bad == 1 and not np.isfinite(normalized).all()
    finally:
        e.close()


def test_rejects_invalid_requests(ctx, encoder):
    for w, h in [(40, 32), (32, 0), (4096, 32), (8, 8)]:
        with pytest.raises(ec.CudaError):
            encoder.encode(np.zeros((max(h, 1), w, 3), np.uint8) if h else np.zeros((0, w, 3), np.uint8))
    with pytest.raises(ec.CudaError):
        encoder.upload("encoder.conv_in.weight", np.zeros(7, np.float32))
    with pytest.raises(ec.CudaError):
        encoder.upload("decoder.conv_in.weight", np.zeros((512, 32, 3, 3), np.float32))
    with pytest.raises(ec.CudaError, match="negative"):
        encoder.upload("bn.running_var", -np.ones(128, np.float32))
    fresh = ec.VaeEncoder(ctx)
    try:
        fresh.upload("encoder.conv_in.bias", np.zeros(128, np.float32))
        with pytest.raises(ec.CudaError, match="not uploaded"):
            fresh.encode(image(32, 32))
    finally:
        fresh.close()


@pytest.mark.parametrize("shape", [(512, 384), (1024, 1024)], ids=["512x384", "1024x1024"])
def test_reviewed_large_shapes_bf16_against_fp32_mode(encoder, shape):
    """The reference's reviewed large shapes (tools/specialize_vae_encoder_1024.py; 1024x1024 has 16384
    mid-block tokens), where the oracle would take minutes: BF16 mode against FP32-exact mode within the BF16
    gate, both finite and repeatable."""
    rgb = image(*shape)
    exact = encoder.encode(rgb, ec.FP32)
    fast = encoder.encode(rgb, ec.BF16)
    again = encoder.encode(rgb, ec.BF16)
    assert exact[3] == 0 and fast[3] == 0
    for x, y in zip(fast[:3], again[:3]):
        assert np.array_equal(x, y)
    check_outputs(exact[:3], fast[:3], ENC_BF16, f"VAE encode {shape[0]}x{shape[1]}, BF16 vs FP32-exact")
