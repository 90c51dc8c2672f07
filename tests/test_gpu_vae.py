"""VAE decoder on a B200 (decode_vae + rgb_image, src/vae.cpp:18-64, src/pipeline.cpp:145-163) against the
CPU oracle (oracle/vae.py) on seeded synthetic weights.

Gates (atol, rtol, nrmse) are the reference's VAE gates: the component fixture's "fp32", "fp16" and "bf16"
gates (tools/export_dit_heads.py:88-90, written into the VAE fixture by tools/export_vae.py) and the
decoder cross-check's FP32 gate (tools/diagnose_vae_cross.py:22). FP32-exact mode is held to the FP32
gate; BF16 mode (BF16 convolution operands, FP32 accumulation, FP32 residuals and norms) to the tighter
FP16 gate.
"""
import numpy as np
import pytest

import ernie_cuda as ec
import vae as ov
from conftest import gate

pytestmark = pytest.mark.gpu
SEED = 7
VAE_FP32 = (2e-4, 2e-4, 2e-5)
VAE_FP16 = (0.03, 0.03, 0.02)
VAE_BF16 = (0.2, 0.2, 0.1)


@pytest.fixture(scope="module")
def weights():
    return ov.synth_weights(SEED)


@pytest.fixture(scope="module")
def vae(ctx):
    v = ec.Vae(ctx)
    v.synthesize(SEED)
    yield v
    v.close()


def latent(h, w, seed=1):
    return np.random.default_rng(seed).standard_normal((32, h, w)).astype(np.float32)


@pytest.mark.parametrize("shape", [(8, 8), (12, 20)])
@pytest.mark.parametrize("precision", [ec.FP32, ec.BF16], ids=["fp32", "bf16"])
def test_decode_against_oracle(vae, weights, shape, precision):
    u = latent(*shape)
    ref = ov.decode(weights, u)
    got, rgb, bad = vae.decode(u, precision, rgb=True)
    assert got.shape == (3, 8 * shape[0], 8 * shape[1]) and bad == 0
    ok, metrics = gate(ref, got, *(VAE_FP32 if precision == ec.FP32 else VAE_FP16))
    print("VAE decode", shape, "fp32" if precision == ec.FP32 else "bf16", metrics)
    assert ok, metrics
    assert np.array_equal(rgb, ov.rgb_image(got)), "RGB bytes must follow rgb_image exactly"


def test_bf16_weights_take_the_three_product_path(ctx):
    """Exact-BF16 weights: FP32-exact mode multiplies the three operand planes by one weight plane."""
    w = ov.synth_weights(SEED + 1, bf16_weights=True)
    v = ec.Vae(ctx)
    try:
        v.synthesize(SEED + 1, bf16_weights=True)
        u = latent(8, 12, seed=2)
        got, _, _ = v.decode(u, ec.FP32)
    finally:
        v.close()
    ok, metrics = gate(ov.decode(w, u), got, *VAE_FP32)
    print("VAE decode, BF16 weights, FP32-exact", metrics)
    assert ok, metrics


def test_uploaded_weights_equal_synthesized(ctx, vae, weights):
    """The upload path (diffusers names, FP32) and device-side synthesis hold the same weights."""
    v = ec.Vae(ctx)
    try:
        for name, array in weights.items():
            v.upload(name, array)
        u = latent(8, 8, seed=3)
        for precision in (ec.FP32, ec.BF16):
            a, _, _ = v.decode(u, precision)
            b, _, _ = vae.decode(u, precision)
            assert np.array_equal(a, b)
    finally:
        v.close()


def test_repeat_and_shape_switch_are_bit_exact(vae):
    u1, u2 = latent(8, 8, seed=4), latent(4, 12, seed=5)
    first, _, _ = vae.decode(u1, ec.BF16)
    other, _, _ = vae.decode(u2, ec.BF16)
    again, _, _ = vae.decode(u1, ec.BF16)
    assert other.shape == (3, 32, 96)
    assert np.array_equal(first, again)


def test_device_entry_matches_host_entry(ctx, vae):
    u = latent(8, 16, seed=6)
    host, _, _ = vae.decode(u, ec.BF16)
    src = ctx.to_device(u)
    dst = ctx.buffer(host.nbytes)
    try:
        vae.decode_device(src, 16, 8, dst, ec.BF16)
        ctx.synchronize()
        assert np.array_equal(dst.download(host.shape), host)
    finally:
        src.free()
        dst.free()


def test_nonfinite_input_is_flagged(vae):
    u = latent(4, 4, seed=7)
    u[3, 1, 2] = np.nan
    out, _, bad = vae.decode(u, ec.BF16, rgb=True)
    assert bad == 1 and not np.isfinite(out).all()


def test_rejects_invalid_requests(ctx, vae):
    with pytest.raises(ec.CudaError):
        vae.decode(np.zeros((32, 0, 4), np.float32))
    with pytest.raises(ec.CudaError):
        vae.decode(np.zeros((32, 4, 300), np.float32))
    with pytest.raises(ec.CudaError):
        vae.upload("decoder.conv_in.weight", np.zeros(7, np.float32))
    with pytest.raises(ec.CudaError):
        vae.upload("decoder.no_such.weight", np.zeros(1, np.float32))
    bad = np.zeros((512,), np.float32)
    bad[3] = np.inf
    with pytest.raises(ec.CudaError):
        vae.upload("decoder.mid_block.resnets.0.norm1.weight", bad)
    fresh = ec.Vae(ctx)
    try:
        fresh.upload("decoder.conv_in.bias", np.zeros(512, np.float32))
        with pytest.raises(ec.CudaError, match="not uploaded"):
            fresh.decode(latent(4, 4))
    finally:
        fresh.close()


def test_full_size_bf16_against_fp32_mode(vae):
    """1024 x 1024 output (128 x 128 unpacked latent), where the oracle would take minutes: BF16 mode against
    the FP32-exact mode within the reference's BF16 gate, both finite and repeatable."""
    u = latent(128, 128, seed=8)
    exact, rgb, bad = vae.decode(u, ec.FP32, rgb=True)
    assert bad == 0 and np.isfinite(exact).all()
    fast, _, _ = vae.decode(u, ec.BF16)
    again, _, _ = vae.decode(u, ec.BF16)
    assert np.array_equal(fast, again)
    ok, metrics = gate(exact, fast, *VAE_BF16)
    print("VAE 1024x1024, BF16 vs FP32-exact", metrics)
    assert ok, metrics
    assert np.array_equal(rgb, ov.rgb_image(exact))


def test_fixed_1376x768_shape(vae):
    """The reference's fixed decoder shape (tools/vae_shape_contract.py:2: latent 96 x 172, image 1376 x 768):
    ragged 128-pixel segments on every level, 16512 attention tokens (padded to 16640) on the 32K-key softmax
    path. BF16 against FP32-exact within the BF16 gate; both finite."""
    u = latent(96, 172, seed=9)
    exact, _, bad = vae.decode(u, ec.FP32)
    fast, rgb, bad2 = vae.decode(u, ec.BF16, rgb=True)
    assert bad == 0 and bad2 == 0 and exact.shape == (3, 768, 1376)
    ok, metrics = gate(exact, fast, *VAE_BF16)
    print("VAE 1376x768, BF16 vs FP32-exact", metrics)
    assert ok, metrics
    assert np.array_equal(rgb, ov.rgb_image(fast))
