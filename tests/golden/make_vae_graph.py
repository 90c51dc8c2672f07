"""Generates tests/golden/vae_decoder_graph.json from the reference's exported VAE decoder graph.

The reference exports the pinned AutoencoderKLFlux2 post_quant_conv + decoder to ncnn
(tools/export_vae.py) and specialises its two spatial reshapes per shape (tools/vae_shape_contract.py);
artifacts/2026-09-05/pipeline/models/vae-128x128-specialized-v1/head.ncnn.param is that graph for a
128 x 128 latent. This script keeps, in execution order, every compute layer with the parameters that
fix the architecture (convolution widths, kernel sizes and weight counts; GroupNorm groups, channels and
eps; the attention's width, heads and weight count; interpolation scale). Run it where the reference
tree is present; the JSON it writes is committed so the tests need no reference checkout.

    python tests/golden/make_vae_graph.py <reference root>
"""
import json
import os
import sys

GRAPH = "artifacts/2026-09-05/pipeline/models/vae-128x128-specialized-v1/head.ncnn.param"
KEEP = {
    "Convolution": {"0": "num_output", "1": "kernel", "4": "pad", "5": "bias_term", "6": "weight_data_size"},
    "GroupNorm": {"0": "groups", "1": "channels", "2": "eps", "3": "affine"},
    "MultiHeadAttention": {"0": "embed_dim", "1": "num_heads", "2": "weight_data_size"},
    "Interp": {"0": "resize_type", "1": "height_scale", "2": "width_scale"},
    "Swish": {},
    "BinaryOp": {"0": "op_type"},
}


def parse(text):
    lines = text.splitlines()
    if lines[0].strip() != "7767517":
        raise ValueError("not an ncnn param file")
    layers = []
    for line in lines[2:]:
        fields = line.split()
        if not fields or fields[0] not in KEEP:
            continue
        kind, name = fields[0], fields[1]
        n_in, n_out = int(fields[2]), int(fields[3])
        params = dict(f.split("=", 1) for f in fields[4 + n_in + n_out:])
        kept = {}
        for key, label in KEEP[kind].items():
            if key in params:
                value = params[key]
                kept[label] = float(value) if ("." in value or "e" in value) else int(value)
        layers.append({"type": kind, "name": name, **kept})
    return layers


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ERNIE_REFERENCE_ROOT", "")
    path = os.path.join(root, GRAPH)
    with open(path) as f:
        layers = parse(f.read())
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "vae_decoder_graph.json")
    with open(out, "w") as f:
        json.dump({"source": GRAPH, "layers": layers}, f, indent=1)
        f.write("\n")
    print(f"{len(layers)} layers -> {out}")


if __name__ == "__main__":
    main()
