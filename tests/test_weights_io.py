"""Official checkpoint files on the CPU: the safetensors reader (header, shapes, dtypes, malformed files)
and text_embeddings (src/text_encoder.cpp:48-75) over the raw BF16 table and over a checkpoint."""
import json
import os
import struct

import numpy as np
import pytest

import ernie_cuda as ec
from conftest import write_safetensors


def test_header_is_read(tmp_path):
    path = str(tmp_path / "a.safetensors")
    write_safetensors(path, {"b.weight": ("BF16", np.arange(6, dtype=np.uint16).reshape(2, 3)),
                             "a.bias": ("F32", np.ones(4, np.float32)),
                             "c": ("F16", np.zeros((1, 1, 2), np.float16))}, metadata={"format": "pt"})
    assert ec.safetensors_entries(path) == [("a.bias", "F32", (4,)), ("b.weight", "BF16", (2, 3)),
                                            ("c", "F16", (1, 1, 2))]


def _raw(path, header, data=b""):
    text = json.dumps(header).encode() if isinstance(header, dict) else header
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(text)) + text + data)


@pytest.mark.parametrize("case", ["truncated", "bad_json", "past_end", "byte_count", "duplicate", "negative"])
def test_malformed_files_are_rejected(tmp_path, case):
    path = str(tmp_path / "bad.safetensors")
    if case == "truncated":
        with open(path, "wb") as f:
            f.write(struct.pack("<Q", 100) + b"{}")
    elif case == "bad_json":
        _raw(path, b'{"x": {"dtype": "F32", "shape": [1], "data_offsets": [0, 4]', b"\0" * 4)
    elif case == "past_end":
        _raw(path, {"x": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}, b"\0" * 8)
    elif case == "byte_count":
        _raw(path, {"x": {"dtype": "F32", "shape": [3], "data_offsets": [0, 16]}}, b"\0" * 16)
    elif case == "duplicate":
        _raw(path, b'{"x": {"dtype": "F32", "shape": [1], "data_offsets": [0, 4]}, '
                   b'"x": {"dtype": "F32", "shape": [1], "data_offsets": [0, 4]}}', b"\0" * 4)
    else:
        _raw(path, {"x": {"dtype": "F32", "shape": [-1], "data_offsets": [0, 4]}}, b"\0" * 4)
    with pytest.raises(ec.CudaError):
        ec.safetensors_entries(path)


def _bf16_bits(x):
    bits = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return (((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16)).astype(np.uint16)


def test_text_embeddings_from_raw_table_and_checkpoint(tmp_path):
    vocab, width = 131072, 3072
    rng = np.random.default_rng(0)
    ids = np.array([5, 131071, 0, 77], np.uint32)
    rows = _bf16_bits(rng.standard_normal((len(ids), width)))
    # the reference's raw table, sparse except the rows read
    raw = str(tmp_path / "embeddings.bf16")
    with open(raw, "wb") as f:
        f.truncate(vocab * width * 2)
        for i, r in zip(ids, rows):
            f.seek(int(i) * width * 2)
            f.write(r.tobytes())
    got = ec.text_embeddings(raw, ids, 8)
    expect = np.zeros((8, width), np.float32)
    expect[:4] = (rows.astype(np.uint32) << 16).view(np.float32)
    assert np.array_equal(got, expect)
    # the checkpoint tensor (header + sparse data)
    ckpt = str(tmp_path / "text.safetensors")
    name = "language_model.model.embed_tokens.weight"
    text = json.dumps({name: {"dtype": "BF16", "shape": [vocab, width], "data_offsets": [0, vocab * width * 2]}})
    text = text.encode() + b" " * (-len(text) % 8)
    with open(ckpt, "wb") as f:
        f.write(struct.pack("<Q", len(text)) + text)
        base = f.tell()
        f.truncate(base + vocab * width * 2)
        for i, r in zip(ids, rows):
            f.seek(base + int(i) * width * 2)
            f.write(r.tobytes())
    assert np.array_equal(ec.text_embeddings(ckpt, ids, 8), expect)
    with pytest.raises(ec.CudaError):
        ec.text_embeddings(raw, np.array([131072], np.uint32), 4)
    with pytest.raises(ec.CudaError):
        ec.text_embeddings(raw, ids, 3)  # more ids than the bucket
    short = str(tmp_path / "short.bf16")
    with open(short, "wb") as f:
        f.truncate(1024)
    with pytest.raises(ec.CudaError):
        ec.text_embeddings(short, ids, 8)
