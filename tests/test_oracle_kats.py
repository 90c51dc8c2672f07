"""Pin the CPU restatement (oracle/) to the reference's own known-answer tests (CPU only)."""
import os

import numpy as np
import pytest

import oracle as o

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_kats.npz"))

import importlib.util

_spec = importlib.util.spec_from_file_location("make_golden", os.path.join(os.path.dirname(__file__), "golden",
                                                                           "make_golden.py"))
mg = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(mg)


def golden_values(name, full):
    flat = np.asarray(full).ravel()
    if name + "_idx" in GOLDEN:
        flat = flat[GOLDEN[name + "_idx"]]
    return flat.astype(np.float64), GOLDEN[name]


@pytest.mark.parametrize("queries,keys,width", [(3, 17, 128), (257, 65, 128), (3, 17, 124)])
@pytest.mark.parametrize("mask_heads", [1, 2])
@pytest.mark.parametrize("shift", [0, 3])
def test_attention_mask_kat(queries, keys, width, mask_heads, shift):
    # tests/test_attention_mask.cpp: FP64 reference |d| < 3e-6; dense and row masks agree exactly.
    q, k, v = mg.attention_mask_inputs(queries, keys, width)
    row = mg.attention_mask_row(keys, shift, mask_heads)
    out_row = o.sdpa(q, k, v, row if mask_heads == 2 else row[0])
    dense = np.repeat(row, queries, axis=1)
    out_dense = o.sdpa(q, k, v, dense if mask_heads == 2 else dense[0])
    assert np.array_equal(out_row, out_dense)
    got, ref = golden_values(f"attn_q{queries}_k{keys}_w{width}_mh{mask_heads}_s{shift}", out_row)
    assert np.abs(got - ref).max() < 3e-6


def test_attention_accuracy_probe():
    # probes/attention_accuracy_probe.cpp:87-92: max 3e-6, constant column 5e-7, NRMSE 5e-7.
    q, k, v, mask, _ = mg.accuracy_probe_inputs()
    out = o.sdpa(q, k, v, mask)
    ref = GOLDEN["attn_probe"].reshape(out.shape)
    err = out.astype(np.float64) - ref
    assert np.abs(err).max() <= 3e-6
    assert np.abs(out[:, :, 0].astype(np.float64) - 1.0).max() <= 5e-7
    assert np.sqrt((err ** 2).sum() / (ref ** 2).sum()) <= 5e-7


@pytest.mark.parametrize("shape", [0, 1])
def test_gelu_kat(shape):
    # probes/gelu_probe.cpp:70-77: FP32 limit 2e-6 against 0.5 x erfc(-x/sqrt2).
    x = mg.gelu_inputs(shape)
    got, ref = golden_values(f"gelu_{shape}", o.gelu(x))
    assert np.abs(got - ref).max() <= 2e-6


@pytest.mark.parametrize("width", [128, 3072, 4096])
@pytest.mark.parametrize("scale", [1.0, 512.0])
def test_rmsnorm_kat(width, scale):
    # probes/rmsnorm_probe.cpp:72-99: FP32 limit 2e-6.
    values, weight = mg.norm_inputs(width, scale)
    got, ref = golden_values(f"rms_w{width}_s{int(scale)}", o.rmsnorm(values, weight))
    assert np.abs(got - ref).max() <= 2e-6


@pytest.mark.parametrize("scale", [1.0, 1024.0])
def test_layernorm_kat(scale):
    values, _ = mg.norm_inputs(4096, scale)
    got, ref = golden_values(f"ln_w4096_s{int(scale)}", o.layernorm(values))
    assert np.abs(got - ref).max() <= 2e-6


def test_residual_contract():
    # tests/test_residual_contract.cpp:57-64: values beyond FP16 range add exactly in FP32.
    y = np.arange(4)[:, None]
    i = np.arange(4096)[None, :]
    a = (np.where(i % 2 == 1, -1.0, 1.0) * (70000.0 + y * 128.0)).astype(np.float32)
    b = ((i % 8) * 128.0).astype(np.float32)
    b = np.broadcast_to(b, a.shape).copy()
    s = o.residual_add(a, b)
    assert np.array_equal(s, a + b)
    normed = o.rmsnorm(s, np.ones(4096, np.float32))
    ref = s.astype(np.float64) / np.sqrt((s.astype(np.float64) ** 2).mean(axis=1, keepdims=True) + 1e-6)
    assert np.abs(normed - ref).max() <= 1e-3


@pytest.mark.parametrize("m,n,k,bias", [(32, 48, 64, False), (1, 48, 32, True), (32, 128, 64, False),
                                        (130, 256, 128, True), (300, 512, 4096, False)])
def test_bf16_gemm_exact(m, n, k, bias):
    # tests/test_bf16_gemm.cpp:46-58: operands are exact multiples of 1/8, every sum is exact.
    a, w, b = mg.gemm_inputs(m, n, k)
    bits = (w.view(np.uint32) >> 16).astype(np.uint16)
    assert np.array_equal(o.bf16_to_f32(bits), w)
    got = o.linear(a, bits, b if bias else None)
    _, ref = golden_values(f"gemm_m{m}_n{n}_k{k}_b{int(bias)}", got)
    got_s, _ = golden_values(f"gemm_m{m}_n{n}_k{k}_b{int(bias)}", got)
    assert np.array_equal(got_s, ref)


def test_latent_contract():
    # tests/test_latent_contract.cpp:19-46
    with pytest.raises(ValueError):
        o.schedule(0)
    with pytest.raises(ValueError):
        o.schedule(1001)
    sig, ts = o.schedule(8)
    assert sig[0] == 1.0 and sig[-1] == 0.0
    assert np.all(np.diff(sig) < 0)
    assert np.array_equal(sig.astype(np.float64), GOLDEN["turbo8_sigmas"])
    assert np.array_equal(ts, (np.float32(1000.0) * sig[:-1]).astype(np.float32))
    x = np.ones((128, 5, 3), np.float32)
    p = np.ones((128, 5, 3), np.float32)
    assert o.finite(x)
    x[42].flat[7] = np.inf
    assert not o.finite(x)
    x[42].flat[7] = np.nan
    assert not o.finite(x)
    x[42].flat[7] = 1.0
    for bad in (0.0, np.nan, -1.5):
        with pytest.raises(ValueError):
            o.euler_step(x, p, bad)
    out = o.euler_step(x, p, -1.0)
    assert np.all(out == 0.0)
    mean, var = np.zeros(128, np.float32), np.ones(128, np.float32)
    var[42] = -1.0
    with pytest.raises(ValueError):
        o.unpack_for_vae(x, mean, var)


def test_recovery_tiny_denoiser_euler():
    # tests/test_memory_execution.cpp:324-329: v = 0.125 x through the schedule, independent within 3e-7.
    sig, _ = o.schedule(4)
    x = np.linspace(-2, 2, 128 * 6, dtype=np.float32).reshape(128, 2, 3)
    expected = x[:, 0, 0].astype(np.float32).copy()
    cur = x
    for i in range(4):
        delta = np.float32(sig[i + 1] - sig[i])
        cur = o.euler_step(cur, (cur * np.float32(0.125)).astype(np.float32), delta)
        expected = (expected + delta * (expected * np.float32(0.125))).astype(np.float32)
    assert np.abs(cur[:, 0, 0] - expected).max() <= 3e-7


def test_timestep_features_and_constants():
    f = o.timestep_features(500.0)
    assert f.shape == (4096,)
    # sin half first (flip_sin_to_cos=false): feature 0 is sin(t), feature 2048 is cos(t)
    assert abs(f[0] - np.sin(np.float32(500.0))) < 1e-6 and abs(f[2048] - np.cos(np.float32(500.0))) < 1e-6
    with pytest.raises(ValueError):
        o.timestep_features(1000.5)
    freq = o.rope_frequencies()
    assert freq.shape == (64,) and freq[0] == 1.0 and freq[16] == 1.0 and freq[40] == 1.0
    cos, sin, mask = o.dit_constants(4, 3, 5, 8)
    n = 12 + 8
    assert cos.shape == (n, 128) and mask.shape == (n,)
    assert np.all(mask[:12 + 5] == 0) and np.all(mask[12 + 5:] == np.float32(-1e30))
    # image token 5 sits at (T=5, y=1, x=1); pair-duplicated angle table
    close = lambda a, b: abs(float(a) - float(b)) < 1e-6
    assert cos[5, 0] == cos[5, 1] and close(cos[5, 0], np.cos(5.0 * freq[0]))
    assert close(sin[5, 32], np.sin(1.0 * freq[16]))
    assert close(sin[5, 80], np.sin(1.0 * freq[40]))
    # text slot j: positions (j, 0, 0)
    assert close(cos[12 + 3, 0], np.cos(3.0 * freq[0])) and cos[12 + 3, 40] == 1.0
    with pytest.raises(ValueError):
        o.dit_constants(4, 3, 9, 8)


def test_block_rotary_matches_restated_equations():
    # Cross-check the oracle block against an independent numpy restatement of ExportBlock.forward
    # (tools/export_dit_block.py:38-68) on a tiny random block (2 image rows + text, 1 block).
    seed = 3
    w = o.BlockWeights(seed, 0)
    cos, sin, mask = o.dit_constants(3, 2, 3, 4)
    n = cos.shape[0]
    x = o.synth_normal(seed, o.HIDDEN_STREAM, n * 4096).reshape(n, 4096)
    mod = o.block_modulation(seed)
    got = o.block(x, w, mod, cos, sin, mask)

    def rms(v, g):
        v = v.astype(np.float64)
        return v / np.sqrt((v ** 2).mean(-1, keepdims=True) + 1e-6) * g

    f = lambda t: o.bf16_to_f32(w.mats[t]).astype(np.float64)
    h = rms(x, w.gammas[o.GAMMA_SA]) * (1 + mod[1]) + mod[0]
    q = (h @ f(o.WQ).T).reshape(n, 32, 128).transpose(1, 0, 2)
    k = (h @ f(o.WK).T).reshape(n, 32, 128).transpose(1, 0, 2)
    v = (h @ f(o.WV).T).reshape(n, 32, 128).transpose(1, 0, 2)

    def rot(t):
        a, b = t[..., :64], t[..., 64:]
        return np.concatenate((a * cos[:, :64] - b * sin[:, :64], b * cos[:, 64:] + a * sin[:, 64:]), -1)

    q = rot(rms(q, w.gammas[o.GAMMA_Q]))
    k = rot(rms(k, w.gammas[o.GAMMA_K]))
    s = q @ k.transpose(0, 2, 1) / np.sqrt(128.0) + mask.astype(np.float64)
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    att = (p / p.sum(-1, keepdims=True)) @ v
    att = att.transpose(1, 0, 2).reshape(n, 4096)
    x1 = x + mod[2] * (att @ f(o.WO).T)
    m = rms(x1, w.gammas[o.GAMMA_MLP]) * (1 + mod[4]) + mod[3]
    up = m @ f(o.WUP).T
    gate = m @ f(o.WGATE).T
    from math import erfc, sqrt
    gelu = 0.5 * gate * np.vectorize(lambda t: erfc(-t / sqrt(2.0)))(gate)
    ref = x1 + mod[5] * ((up * gelu) @ f(o.WFC2).T)
    err = got - ref
    assert np.sqrt((err ** 2).sum() / (ref ** 2).sum()) < 2e-6
