"""Generate tests/golden/reference_kats.npz: known-answer vectors of the reference's own tests.

The reference (mingshi2333/ernie-image-ncnn-vulkan) ships no tensors and cannot be built here, so the
golden vectors are its known-answer tests: the closed-form inputs written in its test and probe
sources, with expected outputs from the same independent FP64 formulas those tests use as oracles.
Each block names the reference file it restates. Run from the repository root:

    python tests/golden/make_golden.py

Large expected tensors are stored at 4096 seeded sample positions (indices saved beside them).
"""
import math
import os

import numpy as np

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_kats.npz")
SAMPLES = 4096


def sample(name, full, store):
    flat = np.asarray(full).ravel()
    if flat.size <= 8192:
        store[name] = flat.astype(np.float64)
        return
    idx = np.sort(np.random.default_rng(20260905).choice(flat.size, SAMPLES, replace=False))
    store[name + "_idx"] = idx.astype(np.int64)
    store[name] = flat[idx].astype(np.float64)


# tests/test_attention_mask.cpp:18-31 (inputs) and :47-58 (masks), :72-97 (FP64 oracle).
def attention_mask_inputs(queries, keys, width, heads=2):
    i = np.arange(queries)[:, None]
    d = np.arange(width)[None, :]
    q = np.stack([((i * 3 + d * 7 + h) % 17 - 8) / 32.0 for h in range(heads)]).astype(np.float32)
    j = np.arange(keys)[:, None]
    k = (((j * 7 + d) % 19 - 9) / 32.0).astype(np.float32)[None]
    v = (((j * 3 + d * 5) % 23 - 11) / 16.0).astype(np.float32)[None]
    return q, k, v


def attention_mask_row(keys, shift, mask_heads):
    rows = []
    for h in range(mask_heads):
        visible = keys - 4 - shift - h
        rows.append(np.where(np.arange(keys) < visible, 0.0, -1e30).astype(np.float32))
    return np.stack(rows)[:, None, :]  # [mask_heads, 1, keys]


def fp64_attention(q, k, v, visible_per_head):
    heads, nq, width = q.shape
    out = np.empty((heads, nq, width))
    for h in range(heads):
        kv = 0 if k.shape[0] == 1 else h
        vis = visible_per_head[h]
        s = q[h].astype(np.float64) @ k[kv, :vis].astype(np.float64).T / math.sqrt(width)
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        out[h] = (p @ v[kv, :vis].astype(np.float64)) / p.sum(axis=1, keepdims=True)
    return out


# probes/attention_accuracy_probe.cpp:24-56
def accuracy_probe_inputs():
    width, queries, keys, heads, visible = 128, 5, 4160, 2, 4128
    i = np.arange(queries)[:, None]
    d = np.arange(width)[None, :]
    q = np.stack([np.where(i == 0, 0.0, (((d * 17 + i * 13 + h) % 41) - 20) / 40.0) for h in range(heads)])
    j = np.arange(keys)[:, None]
    k = np.stack([(((j * 7 + d * 19 + h * 11) % 101) - 50) / 64.0 for h in range(heads)])
    v = np.stack([np.where(d == 0, 1.0, (((j * 47 + d * 13 + h * 31) % 257) - 128) / 128.0) for h in range(heads)])
    mask = np.where(np.arange(keys) < visible, 0.0, -1e30)[None, :].repeat(queries, 0)
    return q.astype(np.float32), k.astype(np.float32), v.astype(np.float32), mask.astype(np.float32), visible


# probes/gelu_probe.cpp:52-73
def gelu_inputs(shape_index):
    if shape_index == 0:
        c, h, w = 1, 16, 4096
    else:
        c, h, w = 3, 257, 128
    count = c * h * w
    return (-12.0 + 24.0 * np.arange(count) / (count - 1)).astype(np.float32)


def gelu_fp64(x):
    x = x.astype(np.float64)
    return 0.5 * x * np.array([math.erfc(-t / math.sqrt(2.0)) for t in x])


# probes/rmsnorm_probe.cpp:54-96
def norm_inputs(width, scale):
    weight = (0.5 + (np.arange(width) % 8) * 0.0625).astype(np.float32)
    if width == 128:
        c, h = 8, 5
    else:
        c, h = 1, 8
    cc = np.arange(c)[:, None, None]
    row = np.arange(h)[None, :, None]
    x = np.arange(width)[None, None, :]
    values = (scale * (0.5 + ((x + row + cc) % 8) * 0.125)).astype(np.float32).reshape(c * h, width)
    return values, weight


def norm_fp64(values, weight, centered):
    v = values.astype(np.float64)
    mean = v.mean(axis=1, keepdims=True) if centered else 0.0
    delta = v - mean
    inverse = 1.0 / np.sqrt((delta ** 2).sum(axis=1, keepdims=True) / v.shape[1] + 1e-6)
    return delta * inverse * (1.0 if centered else weight.astype(np.float64))


# tests/test_bf16_gemm.cpp:30-44
def gemm_inputs(m, n, k):
    row = np.arange(m)[:, None]
    inner = np.arange(k)[None, :]
    a = (((row * 13 + inner * 7) % 17 - 3) * np.where(row % 3 == 0, -0.125, 0.125)).astype(np.float32)
    inner2 = np.arange(k)[:, None]
    col = np.arange(n)[None, :]
    w_kn = (((inner2 * 5 + col * 11) % 9 - 2) * 0.125).astype(np.float32)  # weight_value(inner, column)
    bias = ((np.arange(n) % 5 - 2) * 0.125).astype(np.float32)
    return a, np.ascontiguousarray(w_kn.T), bias


def main():
    store = {}
    for queries, keys, width in ((3, 17, 128), (257, 65, 128), (3, 17, 124)):
        for mask_heads in (1, 2):
            for shift in (0, 3):
                q, k, v = attention_mask_inputs(queries, keys, width)
                visible = [keys - 4 - shift - (0 if mask_heads == 1 else h) for h in range(2)]
                name = f"attn_q{queries}_k{keys}_w{width}_mh{mask_heads}_s{shift}"
                sample(name, fp64_attention(q, k, v, visible), store)
    q, k, v, mask, visible = accuracy_probe_inputs()
    store["attn_probe"] = fp64_attention(q, k, v, [visible, visible]).ravel()
    for s in (0, 1):
        x = gelu_inputs(s)
        sample(f"gelu_{s}", gelu_fp64(x), store)
    for width in (128, 3072, 4096):
        for scale in (1.0, 512.0):
            values, weight = norm_inputs(width, scale)
            sample(f"rms_w{width}_s{int(scale)}", norm_fp64(values, weight, False), store)
    for scale in (1.0, 1024.0):
        values, weight = norm_inputs(4096, scale)
        sample(f"ln_w4096_s{int(scale)}", norm_fp64(values, weight, True), store)
    # tests/test_bf16_gemm.cpp:203-204 shapes (projection without bias, single row with column bias) and
    # larger shapes that fit the tensor-core tile; all products and sums are exact in FP32.
    for (m, n, k, with_bias) in ((32, 48, 64, False), (1, 48, 32, True), (32, 128, 64, False), (130, 256, 128, True),
                                 (300, 512, 4096, False)):
        a, w, bias = gemm_inputs(m, n, k)
        exact = a.astype(np.float64) @ w.astype(np.float64).T + (bias if with_bias else 0.0)
        sample(f"gemm_m{m}_n{n}_k{k}_b{int(with_bias)}", exact, store)
    # src/latent_ops.cpp:31-51 turbo schedule for 8 steps, FP32 arithmetic emulated exactly.
    steps = 8
    inc = np.float32(-1.0) / np.float32(steps)
    sig = []
    for i in range(steps):
        if i < (steps + 1) // 2:
            raw = np.float32(float(inc) * i + 1.0)  # fma: one rounding of the exact product-sum
        else:
            raw = np.float32(-inc * np.float32(steps - i))
        sig.append(np.float32(np.float32(4.0) * raw) / np.float32(np.float32(1.0) + np.float32(3.0) * raw))
    sig.append(np.float32(0.0))
    store["turbo8_sigmas"] = np.array(sig, np.float64)
    np.savez_compressed(OUT, **store)
    print(OUT, sum(v.nbytes for v in store.values()), "bytes", len(store), "arrays")


if __name__ == "__main__":
    main()
