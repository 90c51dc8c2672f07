"""Block, DiT and denoise parity of the B200 path against the CPU oracle on seeded inputs (B200 only).

Gates are the reference's own (tools/export_dit_block.py:163-165, tools/export_dit_heads.py:88-90,
tools/validate_pipeline.py:218-222); BF16 uses the relative-L2 tolerances stated with them.
"""
import numpy as np
import pytest

import ernie_cuda as ec
import oracle as o
from conftest import GATES, gate

pytestmark = pytest.mark.gpu
SEED = 11
NUM_BLOCKS = 2


@pytest.fixture(scope="module")
def model(ctx):
    m = ec.Model(ctx, NUM_BLOCKS)
    m.synthesize(SEED)
    yield m
    m.close()


@pytest.fixture(scope="module")
def host_blocks():
    return [o.BlockWeights(SEED, b) for b in range(NUM_BLOCKS)]


@pytest.fixture(scope="module")
def host_heads():
    return o.HeadWeights(SEED)


def block_case(w, h, text, valid, scale=1.0):
    cos, sin, mask = o.dit_constants(w, h, valid, text)
    n = w * h + text
    x = o.synth_normal(SEED, o.HIDDEN_STREAM, n * 4096, scale).reshape(n, 4096)
    mod = o.block_modulation(SEED)
    return x, mod, cos, sin, mask


@pytest.mark.parametrize("precision", [ec.FP32, ec.BF16])
# square grids, a ragged one (5 x 3, 7 text slots of which 5 valid), the smallest request (one image
# token, one text slot) and the scaled-activation case of tools/export_dit_heads.py:172-173
@pytest.mark.parametrize("w,h,text,valid,scale", [(4, 4, 8, 6, 1.0), (16, 16, 32, 24, 1.0), (32, 32, 32, 24, 1.0),
                                                  (5, 3, 7, 5, 1.0), (1, 1, 1, 1, 1.0), (4, 4, 8, 6, 512.0)])
def test_block_parity(model, host_blocks, precision, w, h, text, valid, scale):
    x, mod, cos, sin, mask = block_case(w, h, text, valid, scale)
    ref = o.block(x, host_blocks[0], mod, cos, sin, mask)
    s = ec.Session(model, w, h, text, valid, precision)
    try:
        s.set_conditioning(None, cos, sin, mask)
        got = s.blocks(x, mod, first=0, count=1)
        again = s.blocks(x, mod, first=0, count=1)
    finally:
        s.close()
    assert np.array_equal(got, again), "repeat execution must be bit-exact (probes/block_runner.cpp:197-203)"
    ok, metrics = gate(ref, got, *GATES["block_fp32" if precision == ec.FP32 else "block_bf16"])
    assert ok, metrics


@pytest.mark.parametrize("precision", [ec.FP32, ec.BF16])
def test_block_sequence_parity(model, host_blocks, precision):
    x, mod, cos, sin, mask = block_case(8, 6, 16, 10)
    ref = x
    for b in host_blocks:
        ref = o.block(ref, b, mod, cos, sin, mask)
    s = ec.Session(model, 8, 6, 16, 10, precision)
    try:
        s.set_conditioning(None, cos, sin, mask)
        got = s.blocks(x, mod)
    finally:
        s.close()
    ok, metrics = gate(ref, got, *GATES["block_fp32" if precision == ec.FP32 else "block_bf16"])
    assert ok, metrics


def dit_case(w, h, text, valid):
    latent = o.synth_normal(SEED, o.LATENT_STREAM, 128 * h * w).reshape(128, h, w)
    txt = o.synth_normal(SEED, o.TEXT_STREAM, text * 3072).reshape(text, 3072)
    txt[valid:] = 0.0  # pad_text zero-fills the slots past the valid tokens (src/conditioning.cpp:56-67)
    cos, sin, mask = o.dit_constants(w, h, valid, text)
    return latent, txt, cos, sin, mask


@pytest.mark.parametrize("precision", [ec.FP32, ec.BF16])
def test_dit_prediction_parity(model, host_blocks, host_heads, precision):
    w, h, text, valid = 8, 8, 16, 12
    latent, txt, cos, sin, mask = dit_case(w, h, text, valid)
    t = 923.0769
    ref = o.dit(host_heads, host_blocks, latent, txt, o.timestep_features(t), cos, sin, mask)
    s = ec.Session(model, w, h, text, valid, precision)
    try:
        s.set_conditioning(txt, cos, sin, mask)
        got = s.dit(latent, t)
    finally:
        s.close()
    ok, metrics = gate(ref, got, *GATES["head_fp32" if precision == ec.FP32 else "head_bf16"])
    assert ok, metrics


@pytest.mark.parametrize("precision", [ec.FP32, ec.BF16])
@pytest.mark.parametrize("kind", [ec.TURBO, ec.LINEAR])
def test_denoise_parity(model, host_blocks, host_heads, precision, kind):
    w, h, text, valid = 8, 8, 16, 12
    latent, txt, cos, sin, mask = dit_case(w, h, text, valid)
    steps = 8
    ref, ref_preds = o.denoise(host_heads, host_blocks, latent, txt, cos, sin, mask, steps, 0, 3,
                               "turbo" if kind == ec.TURBO else "linear", keep_predictions=True)
    s = ec.Session(model, w, h, text, valid, precision)
    try:
        s.set_conditioning(txt, cos, sin, mask)
        got, preds = s.denoise(latent, steps, 0, 3, kind, keep_predictions=True)
        # resume from a checkpoint: steps [0,1) then [1,3) must equal [0,3) bit-exactly
        part = s.denoise(latent, steps, 0, 1, kind)
        resumed = s.denoise(part, steps, 1, 3, kind)
    finally:
        s.close()
    assert np.array_equal(resumed, got)
    name = "pipeline_fp32" if precision == ec.FP32 else "pipeline_bf16"
    ok, metrics = gate(ref, got, *GATES[name])
    assert ok, metrics
    for i in range(3):
        ok, metrics = gate(ref_preds[i], preds[i], *GATES[name])
        assert ok, (i, metrics)


def test_denoise_reports_nonfinite(model):
    w, h, text, valid = 4, 4, 8, 6
    latent, txt, cos, sin, mask = dit_case(w, h, text, valid)
    s = ec.Session(model, w, h, text, valid, ec.BF16)
    try:
        s.set_conditioning(txt * np.float32(1e38), cos, sin, mask)
        with pytest.raises(ec.CudaError, match="Non-finite latent after denoise step 1"):
            s.denoise(latent, 8, 0, 2)
        bad = latent.copy()
        bad[0, 0, 0] = np.nan
        with pytest.raises(ec.CudaError, match="Initial latent is not finite"):
            s.denoise(bad, 8, 0, 1)
    finally:
        s.close()


def test_graphs_survive_new_conditioning(model):
    """A session keeps its step graphs when the next request has the same valid-key count and mask
    kind; the graphs read the new text rows, tables and mask from the refilled buffers."""
    w, h, text, valid = 8, 8, 16, 12
    latent, txt, cos, sin, mask = dit_case(w, h, text, valid)
    other = (txt * 0.5 + 0.25).astype(np.float32)
    other[valid:] = 0.0
    s = ec.Session(model, w, h, text, valid, ec.BF16)
    fresh = ec.Session(model, w, h, text, valid, ec.BF16)
    try:
        s.set_conditioning(txt, cos, sin, mask)
        first = s.denoise(latent, 8, 0, 2)
        s.set_conditioning(other, cos, sin, mask)  # same shape: cached graphs stay
        reused = s.denoise(latent, 8, 0, 2)
        fresh.set_conditioning(other, cos, sin, mask)
        ref = fresh.denoise(latent, 8, 0, 2)
    finally:
        s.close()
        fresh.close()
    assert not np.array_equal(first, reused)
    assert np.array_equal(reused, ref)
