"""The prompt enhancer's KV-cached decoder on a B200 (PeSession, src/pe_session.cpp; the head of
enhance_prompt, src/prompt_enhancer.cpp:172-181) against the CPU oracle (oracle/text.py).

By causality, hidden states produced chunk by chunk over the K/V cache must equal the full causal run of
the same layers (the reference's own chunk-plan test, tests/test_pe_prefill.cpp, uses the plans below).
Gates: the text block fixture's fp32 {2e-4, 2e-4, 2e-5} and fp16 {0.03, 0.03, 0.02}
(tools/export_text_block.py:89-91).
"""
import numpy as np
import pytest

import ernie_cuda as ec
import text as ot
from conftest import gate

pytestmark = pytest.mark.gpu
SEED = 11
FREQ = (1.0 / 1000000.0 ** (np.arange(64) / 64)).astype(np.float32)
PE_FP32 = (2e-4, 2e-4, 2e-5)
PE_FP16 = (0.03, 0.03, 0.02)
# the last plan runs 2- to 4-row chunks through the decode products
PLANS = [[17], [8, 8, 1], [5, 1, 11], [1] * 17, [4, 3, 2, 4, 1, 3]]


@pytest.fixture(scope="module")
def model(ctx):
    m = ec.TextModel(ctx, 2)
    m.synthesize(SEED)
    m.synthesize_head(SEED)
    yield m
    m.close()


@pytest.fixture(scope="module")
def layers():
    return [ot.TextLayerWeights(SEED, 0), ot.TextLayerWeights(SEED, 1)]


def prompt(tokens, seed=0):
    return (np.random.default_rng(seed).standard_normal((tokens, 3072)) * 0.2).astype(np.float32)


def run_plan(session, x, cos, sin, plan):
    out, first = [], 0
    for count in plan:
        out.append(session.append(x[first:first + count], cos[first:first + count], sin[first:first + count]))
        first += count
        assert session.position() == first
    return np.concatenate(out)


@pytest.mark.parametrize("plan", PLANS, ids=["17", "8-8-1", "5-1-11", "ones", "4-3-2-4-1-3"])
@pytest.mark.parametrize("precision", [ec.FP32, ec.BF16], ids=["fp32", "bf16"])
def test_cached_decode_equals_full_causal_run(model, layers, plan, precision):
    x = prompt(17)
    cos, sin, _ = ec.text_constants(FREQ, 17)
    ref = ot.run_blocks(layers, x, cos, sin)
    a, b = ec.PeSession(model, 17, precision), ec.PeSession(model, 17, precision)
    try:
        got = run_plan(a, x, cos, sin, plan)
        again = run_plan(b, x, cos, sin, plan)
    finally:
        a.close()
        b.close()
    assert np.array_equal(got, again), "an independent session with the same plan differs"
    ok, metrics = gate(ref, got, *(PE_FP32 if precision == ec.FP32 else PE_FP16))
    print("PE plan", plan[:3], "fp32" if precision == ec.FP32 else "bf16", metrics)
    assert ok, metrics


@pytest.mark.parametrize("precision", [ec.FP32, ec.BF16], ids=["fp32", "bf16"])
def test_logits_against_oracle(model, layers, precision):
    """The LM head on the last hidden row: the first 2048 vocabulary rows against the oracle, all finite."""
    x = prompt(5, seed=1)
    cos, sin, _ = ec.text_constants(FREQ, 5)
    s = ec.PeSession(model, 8, precision)
    try:
        hidden = s.append(x, cos, sin)
        logits = s.logits(hidden[-1])
    finally:
        s.close()
    assert logits.shape == (ec.PE_VOCAB,) and np.isfinite(logits).all()
    gamma, w = ot.head_weights(SEED, 2048)
    ref = ot.head_logits(gamma, w, ot.run_blocks(layers, x, cos, sin)[-1])
    ok, metrics = gate(ref, logits[:2048], *(PE_FP32 if precision == ec.FP32 else PE_FP16))
    print("PE logits", "fp32" if precision == ec.FP32 else "bf16", metrics)
    assert ok, metrics


def test_long_context_positions(model, layers):
    """A 300-token prefill in chunks of 32 then single steps: every row against the full causal run."""
    n = 300
    x = prompt(n, seed=2)
    cos, sin, _ = ec.text_constants(FREQ, n)
    plan = [32] * 9 + [1] * (n - 288)
    s = ec.PeSession(model, n, ec.FP32)
    try:
        got = run_plan(s, x, cos, sin, plan)
    finally:
        s.close()
    ok, metrics = gate(ot.run_blocks(layers, x, cos, sin), got, *PE_FP32)
    print("PE 300 tokens", metrics)
    assert ok, metrics


def test_session_contracts(ctx, model):
    x = prompt(4, seed=3)
    cos, sin, _ = ec.text_constants(FREQ, 4)
    s = ec.PeSession(model, 3, ec.BF16)
    try:
        with pytest.raises(ec.CudaError, match="capacity"):
            s.append(x, cos, sin)  # 4 rows into a capacity of 3
        s.append(x[:3], cos[:3], sin[:3])
        with pytest.raises(ec.CudaError, match="capacity"):
            s.append(x[:1], cos[:1], sin[:1])
        s.reset()
        assert s.position() == 0
        bad = x[:1].copy()
        bad[0, 5] = np.nan
        with pytest.raises(ec.CudaError, match="non-finite"):
            s.append(bad, cos[:1], sin[:1])
        assert s.position() == 0
    finally:
        s.close()
    big = ec.PeSession(model, 40, ec.BF16)
    try:
        x33 = prompt(33, seed=4)
        c33, s33, _ = ec.text_constants(FREQ, 33)
        with pytest.raises(ec.CudaError):
            big.append(x33, c33, s33)  # at most 32 rows per chunk
    finally:
        big.close()
    for capacity in (0, 4097):
        with pytest.raises(ec.CudaError):
            ec.PeSession(model, capacity)
    plain = ec.TextModel(ctx, 1)
    try:
        plain.synthesize(SEED)
        s = ec.PeSession(plain, 4)
        try:
            h = s.append(x[:1], cos[:1], sin[:1])
            with pytest.raises(ec.CudaError, match="head"):
                s.logits(h[0])
        finally:
            s.close()
    finally:
        plain.close()
