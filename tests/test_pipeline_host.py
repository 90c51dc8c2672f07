"""The pipeline's initial noise (src/pipeline.cpp:520-531: std::mt19937(seed) feeding
std::normal_distribution<float>(0, 1) channel after channel) on the host, no GPU.

The library draws it with the C++ standard library, as the reference does. The check here restates the
engine (numpy's legacy MT19937 shares init_genrand seeding) and the Marsaglia polar method the GNU
library uses for normal_distribution<float> (canonical floats from one 32-bit draw each, pairs (x, y)
accepted when 0 < x^2 + y^2 <= 1, y * m returned first and x * m on the next call) in float32, with a
tolerance of 4 ulp (numpy's float32 logarithm against the C library's: at most 3 ulp apart on 32k values).
"""
import numpy as np
import pytest

import ernie_cuda as ec


def mt19937_draws(seed, n):
    return np.random.RandomState(seed).randint(0, 2**32, size=n, dtype=np.uint32)


def polar_normals(seed, count):
    raw = mt19937_draws(seed, 4 * count + 64)
    pos = 0
    out = np.empty(count, np.float32)
    saved = None
    f32 = np.float32
    for i in range(count):
        if saved is not None:
            out[i], saved = saved, None
            continue
        while True:
            u = f32(f32(raw[pos]) / f32(4294967296.0))
            v = f32(f32(raw[pos + 1]) / f32(4294967296.0))
            pos += 2
            if u >= 1:
                u = np.nextafter(f32(1), f32(0))
            if v >= 1:
                v = np.nextafter(f32(1), f32(0))
            x = f32(f32(2) * u - f32(1))
            y = f32(f32(2) * v - f32(1))
            r2 = f32(f32(x * x) + f32(y * y))
            if 0 < r2 <= 1:
                break
        mult = f32(np.sqrt(f32(f32(-2) * np.log(r2)) / r2))
        saved = f32(x * mult)
        out[i] = f32(y * mult)
    return out


def test_mt19937_known_answer():
    # the C++ standard's check: the 10000th output of a default-constructed mt19937 (seed 5489)
    assert mt19937_draws(5489, 10000)[-1] == 4123659995


@pytest.mark.parametrize("seed,w,h", [(0, 4, 3), (42, 8, 8), (123456789, 5, 7)])
def test_initial_noise_matches_restatement(seed, w, h):
    got = ec.initial_noise(seed, w, h)
    ref = polar_normals(seed, 128 * w * h).reshape(128, h, w)
    np.testing.assert_allclose(got, ref, rtol=4e-6, atol=1e-7)


def test_initial_noise_is_standard_normal_and_deterministic():
    a = ec.initial_noise(7, 64, 64)
    assert np.array_equal(a, ec.initial_noise(7, 64, 64))
    assert not np.array_equal(a, ec.initial_noise(8, 64, 64))
    assert abs(a.mean()) < 0.01 and abs(a.std() - 1) < 0.01


def test_initial_noise_rejects_bad_shapes():
    out = np.empty(128, np.float32)
    assert ec.lib().ernie_cuda_initial_noise(0, 0, 1, ec.ptr(out)) != 0
    assert ec.lib().ernie_cuda_initial_noise(0, 257, 1, ec.ptr(out)) != 0
