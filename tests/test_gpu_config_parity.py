"""One DiT block at the token counts the benchmark configurations run, against the CPU oracle (B200 only).

The small-shape block tests pin the op order, modulation and RoPE layout; these pin the same block at the
shapes the headline numbers are quoted on, where the attention runs over thousands of keys and the RoPE
grid and text mask take their real forms:

* C2: 64x64 packed latent + 64 text slots, all valid (4160 tokens).
* C3: 86x48 packed latent (a non-square 3-axis RoPE grid, src/conditioning.cpp:10-44) + the 2048-slot
  text bucket (src/shape_plan.h:12) with 1080 valid tokens, so the last 968 keys carry the -1e30 mask of
  src/conditioning.cpp:41-42 (6176 tokens, 5208 valid keys).
* C4: 128x64 packed latent + 64 text slots (8256 tokens).

Both precisions are gated with the reference's block gates (tools/export_dit_block.py:163-165, pass rule
tools/validate_dit_block.py:113-120). The oracle's output is computed once per shape (7-20 s on the host).
"""
import numpy as np
import pytest

import ernie_cuda as ec
import oracle as o
from conftest import GATES, gate

pytestmark = pytest.mark.gpu
SEED = 11

# name: (w, h, text slots, valid text)
CONFIGS = {"c2": (64, 64, 64, 64), "c3": (86, 48, 2048, 1080), "c4": (128, 64, 64, 64)}


@pytest.fixture(scope="module")
def model(ctx):
    m = ec.Model(ctx, 1)
    m.synthesize(SEED)
    yield m
    m.close()


@pytest.fixture(scope="module")
def weights():
    return o.BlockWeights(SEED, 0)


_cases = {}


def config_case(name, weights):
    """Inputs and the oracle's block output for one configuration (cached for the module)."""
    if name not in _cases:
        w, h, text, valid = CONFIGS[name]
        cos, sin, mask = o.dit_constants(w, h, valid, text)
        n = w * h + text
        x = o.synth_normal(SEED, o.HIDDEN_STREAM, n * 4096).reshape(n, 4096)
        mod = o.block_modulation(SEED)
        ref = o.block(x, weights, mod, cos, sin, mask)
        _cases[name] = (x, mod, cos, sin, mask, ref)
    return _cases[name]


def test_c3_mask_and_grid_shape(weights):
    """The C3 case really has a non-square grid and 968 masked keys at the end of the text bucket."""
    w, h, text, valid = CONFIGS["c3"]
    _, _, cos, _, mask, _ = config_case("c3", weights)
    assert w != h and cos.shape == (w * h + text, 128)
    masked = np.flatnonzero(mask != 0)
    assert masked.size == 968 and masked[0] == w * h + valid and masked[-1] == w * h + text - 1
    assert np.all(mask[masked] == np.float32(-1e30))


@pytest.mark.parametrize("precision", [ec.FP32, ec.BF16], ids=["fp32", "bf16"])
@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_block_at_config_shape(model, weights, name, precision):
    w, h, text, valid = CONFIGS[name]
    x, mod, cos, sin, mask, ref = config_case(name, weights)
    s = ec.Session(model, w, h, text, valid, precision)
    try:
        s.set_conditioning(None, cos, sin, mask)
        got = s.blocks(x, mod, first=0, count=1)
    finally:
        s.close()
    ok, metrics = gate(ref, got, *GATES["block_fp32" if precision == ec.FP32 else "block_bf16"])
    # the rows of the masked text slots are outputs too (the reference computes every row)
    image = w * h
    _, image_metrics = gate(ref[:image], got[:image], *GATES["block_bf16"])
    print(f"block {name} {'fp32' if precision == ec.FP32 else 'bf16'} tokens={w * h + text} "
          f"nrmse={metrics['nrmse']:.3e} max_abs={metrics['max_abs_error']:.3e} "
          f"ref_max={metrics['reference_max_abs']:.3e} image_rows_nrmse={image_metrics['nrmse']:.3e}")
    assert ok, metrics
