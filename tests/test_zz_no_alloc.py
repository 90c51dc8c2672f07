"""The allocation-free non-finite check (ernie_cuda_finite_latent_noalloc) against the allocating one.

Applications that reserve their device memory at start-up and forbid device allocation afterwards
use the no-alloc entry point. It must agree with ernie_cuda_finite_latent on consecutive calls,
because every call reuses the same static device array. This file sorts last so that a failure here
leaves every other test already run. It passes both alone and after the others.
"""
import ctypes

import numpy as np
import pytest

import ernie_cuda as ec

pytestmark = pytest.mark.gpu


def finite_both(ctx, latent):
    _, h, w = latent.shape
    buf = ctx.to_device(np.ascontiguousarray(latent, np.float32))
    try:
        static_flag, alloc_flag = ctypes.c_int(-1), ctypes.c_int(-1)
        ec.check(ec.lib().ernie_cuda_finite_latent_noalloc(ctx.handle, buf.c, w, h, ctypes.byref(static_flag)))
        ec.check(ec.lib().ernie_cuda_finite_latent(ctx.handle, buf.c, w, h, ctypes.byref(alloc_flag)))
        return static_flag.value, alloc_flag.value
    finally:
        buf.free()


def test_noalloc_matches_allocating_check_on_consecutive_calls(ctx):
    rng = np.random.default_rng(7)
    clean = rng.standard_normal((128, 48, 86)).astype(np.float32)
    bad = clean.copy()
    bad[127, 47, 85] = np.nan
    bad[3, 0, 0] = np.inf
    # clean, then non-finite, then clean again: the shared status array must not carry over
    assert finite_both(ctx, clean) == (1, 1)
    assert finite_both(ctx, bad) == (0, 0)
    assert finite_both(ctx, clean) == (1, 1)
    one_bad = clean[:, :16, :16].copy()
    one_bad[64, 15, 15] = -np.inf
    assert finite_both(ctx, one_bad) == (0, 0)
    assert finite_both(ctx, np.zeros((128, 256, 256), np.float32)) == (1, 1)


def test_noalloc_rejects_sizes_beyond_its_scratch(ctx):
    buf = ctx.buffer(128 * 4)
    try:
        flag = ctypes.c_int(-1)
        with pytest.raises(ec.CudaError, match="1 <= H,W <= 256"):
            ec.check(ec.lib().ernie_cuda_finite_latent_noalloc(ctx.handle, buf.c, 257, 1, ctypes.byref(flag)))
        with pytest.raises(ec.CudaError):
            ec.check(ec.lib().ernie_cuda_finite_latent_noalloc(ctx.handle, buf.c, 0, 4, ctypes.byref(flag)))
    finally:
        buf.free()
