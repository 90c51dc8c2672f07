"""CUDA kernels through the C ABI against the reference KATs and the CPU oracle (B200 only)."""
import os

import numpy as np
import pytest

import ernie_cuda as ec
import oracle as o
from test_oracle_kats import GOLDEN, golden_values, mg

pytestmark = pytest.mark.gpu


def bf16_bits(x):
    """Round-to-nearest-even FP32 -> BF16 bits."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


@pytest.mark.parametrize("m,n,k,bias", [(32, 128, 64, False), (130, 256, 128, True), (300, 512, 4096, False)])
def test_linear_exact_kat(ctx, m, n, k, bias):
    # tests/test_bf16_gemm.cpp operands: exact BF16 multiples of 1/8, so the tcgen05 result is exact.
    a, w, b = mg.gemm_inputs(m, n, k)
    got = ctx.linear_bf16(bf16_bits(a), bf16_bits(w), b if bias else None)
    flat, ref = golden_values(f"gemm_m{m}_n{n}_k{k}_b{int(bias)}", got)
    assert np.array_equal(flat, ref)


# on 148 SMs these run on CTA pairs (256-row tiles, chosen when they need no more tile rounds than
# single CTAs): (100, 256), (4160, 1024), (256, 512), (1000, 256), (3000, 768), (4096, 4096); the
# others on single CTAs
@pytest.mark.parametrize("m,n,k", [(1, 128, 64), (100, 256, 4096), (1056, 4096, 4096), (4160, 1024, 12288),
                                   (256, 512, 128), (1000, 256, 128), (3000, 768, 640), (4096, 4096, 64)])
def test_linear_random(ctx, m, n, k):
    rng = np.random.default_rng(m + n + k)
    a = bf16_bits(rng.standard_normal((m, k), dtype=np.float32))
    w = bf16_bits(rng.standard_normal((n, k), dtype=np.float32) * 0.02)
    bias = rng.standard_normal(n).astype(np.float32)
    got = ctx.linear_bf16(a, w, bias)
    ref = o.bf16_to_f32(a).astype(np.float64) @ o.bf16_to_f32(w).astype(np.float64).T + bias
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err < 3e-5, err  # FP32 accumulation over K up to 12288


def test_device_weights_match_host_generator(ctx):
    model = ec.Model(ctx, 2)
    try:
        model.synthesize(7)
        host = o.BlockWeights(7, 1)
        wqkv = model.read_tensor(1, ec.TENSOR_WQKV, 3 * 4096 * 4096).reshape(3 * 4096, 4096)
        assert np.array_equal(wqkv[:4096], host.mats[o.WQ])
        assert np.array_equal(wqkv[4096:8192], host.mats[o.WK])
        assert np.array_equal(wqkv[8192:], host.mats[o.WV])
        ug = model.read_tensor(1, ec.TENSOR_WUPGATE, 2 * 12288 * 4096).reshape(192, 2, 64, 4096)
        assert np.array_equal(ug[:, 0].reshape(12288, 4096), host.mats[o.WUP])
        assert np.array_equal(ug[:, 1].reshape(12288, 4096), host.mats[o.WGATE])
        fc2 = model.read_tensor(1, ec.TENSOR_WFC2, 4096 * 12288).reshape(4096, 12288)
        assert np.array_equal(fc2, host.mats[o.WFC2])
    finally:
        model.close()


@pytest.mark.parametrize("queries,keys,width", [(3, 17, 128), (257, 65, 128), (3, 17, 124)])
@pytest.mark.parametrize("mask_heads", [1, 2])
@pytest.mark.parametrize("shift", [0, 3])
def test_sdpa_mask_kat(ctx, queries, keys, width, mask_heads, shift):
    # tests/test_attention_mask.cpp: FP64 reference within 3e-6; row mask == dense mask bit-exactly.
    q, k, v = mg.attention_mask_inputs(queries, keys, width)
    row = mg.attention_mask_row(keys, shift, mask_heads)
    out_row = ctx.sdpa(q, k, v, row if mask_heads == 2 else row[0])
    dense = np.repeat(row, queries, axis=1)
    out_dense = ctx.sdpa(q, k, v, dense if mask_heads == 2 else dense[0])
    assert np.array_equal(out_row, out_dense)
    got, ref = golden_values(f"attn_q{queries}_k{keys}_w{width}_mh{mask_heads}_s{shift}", out_row)
    assert np.abs(got - ref).max() < 3e-6


def test_sdpa_accuracy_probe(ctx):
    # probes/attention_accuracy_probe.cpp: 4160 keys, max 3e-6, constant column 5e-7, NRMSE 5e-7.
    q, k, v, mask, _ = mg.accuracy_probe_inputs()
    out = ctx.sdpa(q, k, v, mask)
    ref = GOLDEN["attn_probe"].reshape(out.shape)
    err = out.astype(np.float64) - ref
    assert np.abs(err).max() <= 3e-6
    assert np.abs(out[:, :, 0].astype(np.float64) - 1.0).max() <= 5e-7
    assert np.sqrt((err ** 2).sum() / (ref ** 2).sum()) <= 5e-7


@pytest.mark.parametrize("n,valid,masked", [(288, 280, False), (1056, 1048, False), (4160, 4160, False),
                                            (200, 130, True), (100, 100, False), (6176, 5208, False)])
def test_sdpa_bf16_flash(ctx, n, valid, masked):
    rng = np.random.default_rng(n)
    heads, pad = 4, (n + 127) // 128 * 128
    q = np.zeros((heads, pad, 128), np.float32)
    k = np.zeros_like(q)
    v = np.zeros_like(q)
    q[:, :n] = rng.standard_normal((heads, n, 128)) * 1.5
    k[:, :n] = rng.standard_normal((heads, n, 128)) * 1.5
    v[:, :n] = rng.standard_normal((heads, n, 128))
    qb, kb, vb = bf16_bits(q), bf16_bits(k), bf16_bits(v)
    vt = np.ascontiguousarray(vb.transpose(0, 2, 1))  # the tcgen05 kernel takes V^T [heads][128][rows_pad]
    bq, bk, bv = ctx.to_device(qb), ctx.to_device(kb), ctx.to_device(vt)
    out = ctx.buffer(n * heads * 128 * 2)
    mask = None
    if masked:  # additive row mask inside the valid range (a general ErnieSDPA row mask)
        mask = np.where(np.arange(n) % 7 == 3, np.float32(-1e30), np.float32(0.0)).astype(np.float32)
        mask[:valid] += rng.uniform(-2.0, 0.0, valid).astype(np.float32) * (np.arange(valid) % 7 != 3)
    bm = ctx.to_device(mask) if masked else None
    ec.check(ec.lib().ernie_cuda_sdpa_bf16(ctx.handle, bq.c, bk.c, bv.c, bm.c if bm else None, heads, n, pad, valid,
                                           out.c))
    ctx.synchronize()
    got = o.bf16_to_f32(out.download((n, heads * 128), np.uint16)).reshape(n, heads, 128).transpose(1, 0, 2)
    ref = o.sdpa(o.bf16_to_f32(qb)[:, :n], o.bf16_to_f32(kb)[:, :valid], o.bf16_to_f32(vb)[:, :valid],
                 None if mask is None else mask[:valid])
    err = got.astype(np.float64) - ref
    assert np.sqrt((err ** 2).sum() / (ref.astype(np.float64) ** 2).sum()) < 1e-2
    for b in (bq, bk, bv, out, bm):
        if b:
            b.free()


@pytest.mark.parametrize("shape", [0, 1])
def test_gelu_kat(ctx, shape):
    x = mg.gelu_inputs(shape)
    got, ref = golden_values(f"gelu_{shape}", ctx.gelu(x))
    assert np.abs(got - ref).max() <= 2e-6
    with pytest.raises(ec.CudaError):
        ctx.gelu(np.zeros(6, np.float32))


@pytest.mark.parametrize("width", [128, 3072, 4096])
@pytest.mark.parametrize("scale", [1.0, 512.0])
def test_rmsnorm_kat(ctx, width, scale):
    values, weight = mg.norm_inputs(width, scale)
    got, ref = golden_values(f"rms_w{width}_s{int(scale)}", ctx.rmsnorm(values, weight))
    assert np.abs(got - ref).max() <= 2e-6


@pytest.mark.parametrize("scale", [1.0, 1024.0])
def test_layernorm_kat(ctx, scale):
    values, _ = mg.norm_inputs(4096, scale)
    got, ref = golden_values(f"ln_w4096_s{int(scale)}", ctx.layernorm(values))
    assert np.abs(got - ref).max() <= 2e-6
    with pytest.raises(ec.CudaError):
        ctx.rmsnorm(np.ones((2, 64), np.float32), np.ones(64, np.float32))


def test_residual_and_latent_ops(ctx):
    y = np.arange(4)[:, None]
    i = np.arange(4096)[None, :]
    a = (np.where(i % 2 == 1, -1.0, 1.0) * (70000.0 + y * 128.0)).astype(np.float32)
    b = np.broadcast_to(((i % 8) * 128.0).astype(np.float32), a.shape).copy()
    assert np.array_equal(ctx.residual_add(a, b), a + b)
    rng = np.random.default_rng(0)
    x = rng.standard_normal((128, 48, 86)).astype(np.float32)
    v = rng.standard_normal((128, 48, 86)).astype(np.float32)
    for delta in (-0.0344828, -0.3636364):
        assert np.array_equal(ctx.euler_step(x, v, np.float32(delta)), o.euler_step(x, v, np.float32(delta)))
    with pytest.raises(ec.CudaError):
        ctx.euler_step(x, v, 0.0)
    assert ctx.finite_latent(x)
    bad = x.copy()
    bad[42, 3, 7] = np.inf
    assert not ctx.finite_latent(bad)
    bad[42, 3, 7] = np.nan
    assert not ctx.finite_latent(bad)
    mean = rng.standard_normal(128).astype(np.float32)
    var = rng.uniform(0.1, 3.0, 128).astype(np.float32)
    assert np.array_equal(ctx.unpack_for_vae(x, mean, var), o.unpack_for_vae(x, mean, var))
    var[5] = -1.0
    with pytest.raises(ec.CudaError):
        ctx.unpack_for_vae(x, mean, var)
