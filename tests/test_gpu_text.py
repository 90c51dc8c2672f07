"""Prompt encoder on a B200 (run_text_blocks, src/text_encoder.cpp:106-166) against the CPU oracle
(oracle/text.py) on seeded synthetic weights.

Gates (atol, rtol, nrmse): the reference's text-block fixture gates (tools/export_text_block.py:89-91:
fp32 {2e-4, 2e-4, 2e-5}, fp16 {0.03, 0.03, 0.02}) for one and two layers, and the per-tensor pipeline
gates (tools/validate_pipeline.py:218-222) for the full 25-layer stack.
"""
import numpy as np
import pytest

import ernie_cuda as ec
import text as ot
from conftest import GATES, gate

pytestmark = pytest.mark.gpu
SEED = 3
FREQ = (1.0 / 1000000.0 ** (np.arange(64) / 64)).astype(np.float32)
TEXT_FP32 = (2e-4, 2e-4, 2e-5)
TEXT_FP16 = (0.03, 0.03, 0.02)


@pytest.fixture(scope="module")
def host_layers():
    return [ot.TextLayerWeights(SEED, 0), ot.TextLayerWeights(SEED, 1)]


@pytest.fixture(scope="module")
def model(ctx, host_layers):
    """25 layers: 0 and 1 synthesized on the device, 2..24 uploaded, alternating the two host weight sets."""
    m = ec.TextModel(ctx, 25)
    m.synthesize(SEED)
    for layer in range(2, 25):
        m.upload_layer(layer, host_layers[layer % 2].upload_dict())
    yield m
    m.close()


def prompt(tokens, seed=0):
    return (np.random.default_rng(seed).standard_normal((tokens, 3072)) * 0.2).astype(np.float32)


@pytest.mark.parametrize("layers", [1, 2])
@pytest.mark.parametrize("precision", [ec.FP32, ec.BF16], ids=["fp32", "bf16"])
def test_layers_against_oracle(model, host_layers, layers, precision):
    x = prompt(40)
    cos, sin, _ = ec.text_constants(FREQ, 40)
    ref = ot.run_blocks(host_layers[:layers], x, cos, sin)
    got = model.run_blocks(x, cos, sin, precision, layers)
    ok, metrics = gate(ref, got, *(TEXT_FP32 if precision == ec.FP32 else TEXT_FP16))
    print("text layers", layers, "fp32" if precision == ec.FP32 else "bf16", metrics)
    assert ok, metrics


@pytest.mark.parametrize("precision", [ec.FP32, ec.BF16], ids=["fp32", "bf16"])
def test_25_layers_against_oracle(model, host_layers, precision):
    x = prompt(24, seed=1)
    cos, sin, _ = ec.text_constants(FREQ, 24)
    ref = ot.run_blocks([host_layers[i % 2] for i in range(25)], x, cos, sin)
    got = model.run_blocks(x, cos, sin, precision)
    ok, metrics = gate(ref, got, *GATES["pipeline_fp32" if precision == ec.FP32 else "pipeline_bf16"])
    print("text 25 layers", "fp32" if precision == ec.FP32 else "bf16", metrics)
    assert ok, metrics


def test_padding_cannot_reach_earlier_tokens(model):
    """The causal mask: rows past the prompt (the bucket's padding) leave the prompt rows bit-identical."""
    x = prompt(64, seed=2)
    cos, sin, _ = ec.text_constants(FREQ, 64)
    y = model.run_blocks(x, cos, sin, ec.BF16, 3)
    x2 = x.copy()
    x2[37:] = 0.0
    y2 = model.run_blocks(x2, cos, sin, ec.BF16, 3)
    assert np.array_equal(y[:37], y2[:37]) and not np.array_equal(y[37:], y2[37:])


def test_synthesized_equal_uploaded(ctx, model, host_layers):
    m = ec.TextModel(ctx, 2)
    try:
        for layer in range(2):
            m.upload_layer(layer, host_layers[layer].upload_dict())
        x = prompt(16, seed=3)
        cos, sin, _ = ec.text_constants(FREQ, 16)
        assert np.array_equal(m.run_blocks(x, cos, sin, ec.BF16), model.run_blocks(x, cos, sin, ec.BF16, 2))
    finally:
        m.close()


def test_device_entry_and_long_bucket(ctx, model):
    """A 300-token bucket (the attention's 64-row query tiles and 32-key tiles both ragged) through the device
    entry; BF16 mode within the pipeline gate of the FP32-exact mode; repeat bit-exact."""
    x = prompt(300, seed=4)
    cos, sin, _ = ec.text_constants(FREQ, 300)
    exact = model.run_blocks(x, cos, sin, ec.FP32, 4)
    host = model.run_blocks(x, cos, sin, ec.BF16, 4)
    bufs = [ctx.to_device(a) for a in (x, cos, sin)]
    out = ctx.buffer(x.nbytes)
    try:
        model.run_blocks_device(bufs[0], 300, bufs[1], bufs[2], out, ec.BF16, 4)
        dev = out.download(x.shape)
    finally:
        for b in bufs + [out]:
            b.free()
    assert np.array_equal(dev, host)
    ok, metrics = gate(exact, host, *GATES["pipeline_bf16"])
    print("text 300 tokens, 4 layers, BF16 vs FP32-exact", metrics)
    assert ok, metrics


def test_rejects_invalid_requests(ctx, model, host_layers):
    cos, sin, _ = ec.text_constants(FREQ, 8)
    with pytest.raises(ec.CudaError):
        model.run_blocks(prompt(8), cos, sin, ec.BF16, 26)
    with pytest.raises(ec.CudaError):
        ec.TextModel(ctx, 27)
    with pytest.raises(ec.CudaError):
        model.upload_layer(25, host_layers[0].upload_dict())
