"""Prompt encoder on the CPU: text_constants against its restatement, the oracle layer against a direct
restatement of the attention, and the library's entry points without a GPU."""
import numpy as np
import pytest

import ernie_cuda as ec
import text as ot

FREQ = (1.0 / 1000000.0 ** (np.arange(64) / 64)).astype(np.float32)


@pytest.mark.parametrize("bucket", [1, 7, 64])
def test_text_constants_match_restatement(bucket):
    cos, sin, mask = ec.text_constants(FREQ, bucket, mask=True)
    rc, rs = ot.text_constants(FREQ, bucket)
    # cosf/sinf of the FP32 phase against cos/sin in float64 rounded once: at most one FP32 ulp apart
    assert np.abs(cos - rc).max() <= 1.2e-7 and np.abs(sin - rs).max() <= 1.2e-7
    assert np.array_equal(cos[:, :64], cos[:, 64:]) and np.array_equal(sin[:, :64], sin[:, 64:])
    expected = np.where(np.triu(np.ones((bucket, bucket), bool), 1), -np.finfo(np.float32).max, 0).astype(np.float32)
    assert np.array_equal(mask, expected)


def test_text_constants_reject_bad_input():
    with pytest.raises(ec.CudaError):
        ec.text_constants(FREQ, 0)
    with pytest.raises(ec.CudaError):
        ec.text_constants(FREQ, 2049)
    bad = FREQ.copy()
    bad[5] = 0.0
    with pytest.raises(ec.CudaError):
        ec.text_constants(bad, 4)


def test_oracle_attention_is_causal_gqa():
    """The oracle layer: a change in token j leaves every earlier token's output unchanged."""
    w = ot.TextLayerWeights(2, 0)
    cos, sin = ot.text_constants(FREQ, 6)
    x = np.random.default_rng(0).standard_normal((6, 3072)) * 0.2
    y = ot.layer(w, x, cos, sin)
    x2 = x.copy()
    x2[4] += 1.0
    y2 = ot.layer(w, x2, cos, sin)
    assert np.array_equal(y[:4], y2[:4]) and not np.allclose(y[4:], y2[4:])


def test_rotary_matches_definition():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((3, 2, 128))
    cos, sin = ot.text_constants(FREQ, 3)
    r = ot.rotary(x, cos, sin)
    for t in range(3):
        for j in range(64):
            a, b = x[t, :, j], x[t, :, j + 64]
            np.testing.assert_allclose(r[t, :, j], a * cos[t, j] - b * sin[t, j], rtol=1e-12)
            np.testing.assert_allclose(r[t, :, j + 64], b * cos[t, j + 64] + a * sin[t, j + 64], rtol=1e-12)
