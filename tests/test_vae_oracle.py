"""VAE decoder stage on the CPU: topology against the reference's exported graph, the oracle's layers
against direct restatements, the RGB conversion's known answers, and the library's tensor table."""
import json
import os

import numpy as np
import pytest

import ernie_cuda as ec
import vae as ov

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "vae_decoder_graph.json")


@pytest.fixture(scope="module")
def graph():
    with open(GOLDEN) as f:
        return json.load(f)["layers"]


def conv_layers(table):
    """(num_output, kernel, weight count) of every convolution, in the table's order, with the attention's
    four projections folded into one entry like the graph's MultiHeadAttention."""
    out = []
    for name, shape in table:
        if not name.endswith(".weight") or len(shape) < 2:
            continue
        if ".attentions." in name:
            if name.endswith("to_q.weight"):
                out.append(("attention", 512, int(np.prod(shape))))
            continue
        out.append((shape[0], shape[2], int(np.prod(shape))))
    return out


def graph_convs(graph):
    out = []
    for layer in graph:
        if layer["type"] == "Convolution":
            out.append((layer["num_output"], layer["kernel"], layer["weight_data_size"]))
        elif layer["type"] == "MultiHeadAttention":
            out.append(("attention", layer["embed_dim"], layer["weight_data_size"]))
    return out


@pytest.mark.parametrize("source", ["oracle", "library"])
def test_convolutions_match_the_reference_graph(graph, source):
    table = ov.tensor_table() if source == "oracle" else ec.vae_tensors()
    assert conv_layers(table) == graph_convs(graph)


@pytest.mark.parametrize("source", ["oracle", "library"])
def test_group_norms_match_the_reference_graph(graph, source):
    table = ov.tensor_table() if source == "oracle" else ec.vae_tensors()
    norms = [shape[0] for name, shape in table if "norm" in name and name.endswith(".weight")]
    ref = [layer["channels"] for layer in graph if layer["type"] == "GroupNorm"]
    assert norms == ref
    assert {layer["groups"] for layer in graph if layer["type"] == "GroupNorm"} == {ov.GROUPS}
    assert {layer["eps"] for layer in graph if layer["type"] == "GroupNorm"} == {ov.EPS}


def test_graph_structure(graph):
    """Three nearest x2 upsamplings, one single-head attention, a Swish after every GroupNorm but the
    attention's, and a residual add per resnet and the attention (15)."""
    interp = [layer for layer in graph if layer["type"] == "Interp"]
    assert len(interp) == 3 and all(layer["height_scale"] == 2.0 and layer["resize_type"] == 1 for layer in interp)
    mha = [layer for layer in graph if layer["type"] == "MultiHeadAttention"]
    assert len(mha) == 1 and mha[0]["num_heads"] == 1
    assert sum(layer["type"] == "Swish" for layer in graph) == sum(layer["type"] == "GroupNorm" for layer in graph) - 1
    assert sum(layer["type"] == "BinaryOp" for layer in graph) == 15


def test_library_and_oracle_tables_agree():
    assert ec.vae_tensors() == ov.tensor_table()


def test_conv2d_against_direct_sum():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((5, 6, 7))
    w = rng.standard_normal((4, 5, 3, 3))
    b = rng.standard_normal(4)
    xp = np.pad(x, ((0, 0), (1, 1), (1, 1)))
    ref = np.empty((4, 6, 7))
    for o in range(4):
        for y in range(6):
            for xx in range(7):
                ref[o, y, xx] = b[o] + np.sum(w[o] * xp[:, y:y + 3, xx:xx + 3])
    np.testing.assert_allclose(ov.conv2d(x, w, b), ref, rtol=1e-12, atol=1e-12)


def test_group_norm_two_pass():
    """ErnieGroupNorm's FP64 two-pass statistics (src/ernie_groupnorm.cpp:47-61) on a group whose mean
    dwarfs its spread, and the affine map per channel."""
    rng = np.random.default_rng(4)
    x = 1e4 + rng.standard_normal((64, 3, 5))
    gamma, beta = rng.standard_normal(64), rng.standard_normal(64)
    y = ov.group_norm(x, gamma, beta)
    g = x.reshape(32, -1)
    for k in range(32):
        vals = g[k]
        mean = sum(vals) / len(vals)
        var = sum((v - mean) ** 2 for v in vals) / len(vals)
        for c in (2 * k, 2 * k + 1):
            np.testing.assert_allclose(y[c], (x[c] - mean) / np.sqrt(var + 1e-6) * gamma[c] + beta[c], rtol=1e-9,
                                       atol=1e-9)


def test_rgb_known_answers():
    """rgb_image's rounding (src/pipeline.cpp:158-159): clamp(x/2 + 0.5) * 255, nearest even."""
    values = np.array([-3.0, -1.0, -0.5, 0.0, 1 / 255.0, 0.5, 1.0, 7.0, 0.0039215683], np.float32)
    decoded = np.tile(values.reshape(1, 1, -1), (3, 1, 1))
    rgb = ov.rgb_image(decoded)
    expected = [0, 0, 64, 128, 128, 191, 255, 255, 128]
    assert rgb[0, :, 0].tolist() == expected
    with pytest.raises(ValueError):
        ov.rgb_image(np.full((3, 1, 1), np.nan, np.float32))


def test_synthetic_weights_are_seeded():
    a = ov.synth_weights(5)
    b = ov.synth_weights(5, bf16_weights=True)
    w = a["decoder.conv_in.weight"]
    assert w.dtype == np.float32 and abs(float(w.std()) * np.sqrt(32 * 9) - 1.0) < 0.02
    assert abs(float(a["decoder.conv_norm_out.weight"].mean()) - 1.0) < 0.05
    assert np.array_equal(ov.bf16_round(b["decoder.conv_in.weight"]), b["decoder.conv_in.weight"])
    assert np.array_equal(a["post_quant_conv.weight"], b["post_quant_conv.weight"])
    assert not np.array_equal(a["decoder.conv_in.weight"], b["decoder.conv_in.weight"])


def test_oracle_decode_shapes_and_range():
    w = ov.synth_weights(7)
    u = np.random.default_rng(1).standard_normal((32, 3, 5)).astype(np.float32)
    out = ov.decode(w, u)
    assert out.shape == (3, 24, 40) and np.isfinite(out).all() and 0.05 < float(out.std()) < 50.0
