import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PACKAGE = os.path.join(ROOT, "ernie-image-ncnn-vulkan_b200")
for path in (PACKAGE, os.path.join(ROOT, "oracle")):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA library through its C ABI)")


def write_safetensors(path, tensors, metadata=None):
    """Writes {name: (dtype, array)} as a safetensors file (dtype "BF16" takes uint16 bits, "F32" float32,
    "F16" float16); tensors are laid out in name order."""
    import json
    import struct
    header, blobs, offset = {}, [], 0
    for name in sorted(tensors):
        dtype, array = tensors[name]
        raw = np.ascontiguousarray(array).tobytes()
        header[name] = {"dtype": dtype, "shape": list(np.shape(array)), "data_offsets": [offset, offset + len(raw)]}
        blobs.append(raw)
        offset += len(raw)
    if metadata:
        header["__metadata__"] = metadata
    text = json.dumps(header).encode()
    text += b" " * (-len(text) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(text)))
        f.write(text)
        for raw in blobs:
            f.write(raw)


def gate(reference, actual, atol, rtol, nrmse):
    """Reference gate (tools/validate_dit_block.py:113-120): max|d| <= atol + rtol*max|ref| and
    ||d||_2 / ||ref||_2 <= nrmse. Returns (passed, metrics)."""
    ref = np.asarray(reference, np.float64).ravel()
    got = np.asarray(actual, np.float64).ravel()
    delta = got - ref
    max_abs = float(np.abs(delta).max()) if delta.size else 0.0
    ref_max = float(np.abs(ref).max()) if ref.size else 0.0
    rel = float(np.sqrt((delta ** 2).sum() / max((ref ** 2).sum(), 1e-30)))
    ok = bool(np.isfinite(got).all()) and max_abs <= atol + rtol * ref_max and rel <= nrmse
    return ok, {"max_abs_error": max_abs, "reference_max_abs": ref_max, "nrmse": rel}


GATES = {
    # tools/export_dit_block.py:163-165 (block), tools/export_dit_heads.py:88-90 (heads)
    "block_fp32": (2e-4, 2e-4, 2e-5),
    "block_bf16": (0.15, 0.08, 0.03),
    "head_fp32": (2e-4, 2e-4, 2e-5),
    "head_bf16": (0.2, 0.2, 0.1),
    # tools/validate_pipeline.py:218-222 per-tensor pipeline gates (nrmse, global rtol, atol) mapped to
    # (atol, rtol, nrmse)
    "pipeline_fp32": (2e-4, 0.01, 0.003),
    "pipeline_bf16": (0.03, 0.25, 0.15),
}


@pytest.fixture(scope="session")
def ctx():
    import ernie_cuda
    c = ernie_cuda.Context(0)
    yield c
    c.close()
