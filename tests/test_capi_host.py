"""The C-ABI library loads, exports every declared entry point, and its host-side pieces of the path
(schedule, time features, RoPE/mask constants, argument validation) match the oracle (CPU only)."""
import numpy as np
import pytest

import ernie_cuda as ec
import oracle as o


def test_library_exports_every_declared_symbol():
    lib = ec.lib()
    declared = ec.declared_functions()
    assert len(declared) >= 40
    missing = [name for name in declared if not hasattr(lib, name)]
    assert not missing, missing
    assert set(declared) == set(ec.SIGNATURES), set(declared) ^ set(ec.SIGNATURES)


def test_library_exports_nothing_undeclared():
    """The shared library's dynamic symbol table and include/ernie_cuda.h name the same C entry points:
    no `ernie_cuda_*` function is exported without a declaration (read with `nm -D`)."""
    import shutil
    import subprocess
    if shutil.which("nm") is None:
        pytest.skip("binutils nm is not installed")
    table = subprocess.run(["nm", "-D", "--defined-only", ec.LIB_PATH], capture_output=True, text=True, check=True)
    exported = {cols[2] for cols in (line.split() for line in table.stdout.splitlines())
                if len(cols) == 3 and cols[1] == "T" and cols[2].startswith("ernie_cuda_")}
    declared = set(ec.declared_functions())
    assert exported == declared, {"undeclared exports": sorted(exported - declared),
                                  "declared but not exported": sorted(declared - exported)}


@pytest.mark.parametrize("kind,name", [(ec.TURBO, "turbo"), (ec.LINEAR, "linear")])
def test_schedule_matches_oracle(kind, name):
    for steps in list(range(1, 40)) + [100, 999, 1000]:
        sig, ts = ec.schedule(steps, kind)
        osig, ots = o.schedule(steps, name)
        assert np.array_equal(sig, osig) and np.array_equal(ts, ots)
    for bad in (0, 1001):
        with pytest.raises(ec.CudaError):
            ec.schedule(bad, kind)


def test_timestep_features_match_oracle():
    _, ts = o.schedule(8)
    for t in list(ts) + [0.0, 1000.0, 123.456, 999.99]:
        assert np.array_equal(ec.timestep_features(np.float32(t)), o.timestep_features(np.float32(t)))
    for bad in (-0.5, 1000.01, float("nan"), float("inf")):
        with pytest.raises(ec.CudaError):
            ec.timestep_features(bad)


@pytest.mark.parametrize("w,h,valid,text", [(32, 32, 24, 32), (64, 64, 64, 64), (86, 48, 1080, 2048),
                                            (128, 64, 64, 64), (1, 1, 1, 1), (4, 4, 6, 8)])
def test_dit_constants_match_oracle(w, h, valid, text):
    cos, sin, mask = ec.dit_constants(w, h, valid, text)
    ocos, osin, omask = o.dit_constants(w, h, valid, text)
    assert np.array_equal(cos, ocos) and np.array_equal(sin, osin) and np.array_equal(mask, omask)


def test_dit_constants_validation():
    for args in ((0, 4, 1, 1), (257, 4, 1, 1), (4, 4, 0, 8), (4, 4, 9, 8), (4, 4, 1, 2049), (120, 90, 8, 8)):
        with pytest.raises(ec.CudaError):
            ec.dit_constants(*args)
    # the static graph limit (6144) applies when requested, as in src/conditioning.cpp:45-48
    with pytest.raises(ec.CudaError):
        ec.dit_constants(65, 64, 64, 2048, token_limit=6144)
    ec.dit_constants(65, 64, 64, 2048, token_limit=10240)


def test_official_frequency_table():
    freq = o.rope_frequencies()
    a, _, _ = ec.dit_constants(3, 2, 1, 1, freq=freq)
    b, _, _ = ec.dit_constants(3, 2, 1, 1)
    assert np.array_equal(a, b)
    bad = freq.copy()
    bad[3] = -1.0
    with pytest.raises(ec.CudaError):
        ec.dit_constants(3, 2, 1, 1, freq=bad)


def test_error_codes_without_device():
    # With no visible B200 the context call fails loudly; nothing falls back to the CPU.
    try:
        visible = ec.device_count()
    except ec.CudaError:
        visible = 0  # no driver in this container: cudaGetDeviceCount itself reports the failure
    if visible > 0:
        pytest.skip("a CUDA device is visible")
    with pytest.raises(ec.CudaError):
        ec.Context(0)
