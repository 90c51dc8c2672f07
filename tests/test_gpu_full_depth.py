"""Full-depth denoise on a B200: all 36 blocks and all 8 turbo steps.

* Against the CPU oracle, with the reference's per-tensor pipeline gates (tools/validate_pipeline.py:218-222),
  on a small token count so the oracle finishes in seconds. The 36 device blocks alternate two weight sets
  (blocks 0 and 1 of the seeded model) so the oracle needs only two sets in host memory.
* At the C1 geometry (32x32 latent + 32 text slots, 24 valid; 1056 tokens), where the oracle would take
  tens of minutes: BF16 mode against the FP32-exact mode within the BF16 pipeline gate, and each mode
  repeated bit-exactly.
"""
import numpy as np
import pytest

import ernie_cuda as ec
import oracle as o
from conftest import GATES, gate

pytestmark = pytest.mark.gpu
SEED = 11
MAT_NAMES = {"wq": o.WQ, "wk": o.WK, "wv": o.WV, "wo": o.WO, "wup": o.WUP, "wgate": o.WGATE, "wfc2": o.WFC2}
GAMMA_NAMES = {"gamma_sa": o.GAMMA_SA, "gamma_mlp": o.GAMMA_MLP, "gamma_q": o.GAMMA_Q, "gamma_k": o.GAMMA_K}


@pytest.fixture(scope="module")
def deep():
    ctx = ec.Context(0)
    model = ec.Model(ctx, 36)
    model.synthesize(SEED)  # heads and blocks 0, 1 as the host generator makes them
    host = [o.BlockWeights(SEED, 0), o.BlockWeights(SEED, 1)]
    for b in range(2, 36):
        w = host[b % 2]
        model.upload_block(b, {n: w.mats[t] for n, t in MAT_NAMES.items()},
                           {n: w.gammas[t] for n, t in GAMMA_NAMES.items()})
    yield ctx, model, [host[b % 2] for b in range(36)], o.HeadWeights(SEED)
    model.close()
    ctx.close()


def case(w, h, text, valid):
    latent = o.synth_normal(SEED, o.LATENT_STREAM, 128 * h * w).reshape(128, h, w)
    txt = o.synth_normal(SEED, o.TEXT_STREAM, text * 3072).reshape(text, 3072)
    txt[valid:] = 0.0
    cos, sin, mask = o.dit_constants(w, h, valid, text)
    return latent, txt, cos, sin, mask


SMALL = (4, 4, 8, 6)  # w, h, text slots, valid text: 24 tokens


@pytest.fixture(scope="module")
def oracle_final(deep):
    """The oracle's 8-step, 36-block result at the small shape (computed once, ~15-30 s on the host)."""
    _, _, host_blocks, host_heads = deep
    latent, txt, cos, sin, mask = case(*SMALL)
    return o.denoise(host_heads, host_blocks, latent, txt, cos, sin, mask, 8)


@pytest.mark.parametrize("precision", [ec.FP32, ec.BF16])
def test_36_blocks_8_steps_against_oracle(deep, oracle_final, precision):
    ctx, model, _, _ = deep
    w, h, text, valid = SMALL
    latent, txt, cos, sin, mask = case(w, h, text, valid)
    ref = oracle_final
    s = ec.Session(model, w, h, text, valid, precision)
    try:
        s.set_conditioning(txt, cos, sin, mask)
        got = s.denoise(latent, 8)
    finally:
        s.close()
    ok, metrics = gate(ref, got, *GATES["pipeline_fp32" if precision == ec.FP32 else "pipeline_bf16"])
    print("36 blocks x 8 steps vs oracle", "fp32" if precision == ec.FP32 else "bf16", metrics)
    assert ok, metrics


C1 = (32, 32, 32, 32)  # 32x32 packed latent (512x512) + 32 text tokens, 1056 tokens


@pytest.fixture(scope="module")
def oracle_c1_step(deep):
    """The oracle's first turbo step at the full C1 geometry through all 36 blocks (about a minute on the
    host): the prediction of step 0 and the latent after it."""
    _, _, host_blocks, host_heads = deep
    latent, txt, cos, sin, mask = case(*C1)
    return o.denoise(host_heads, host_blocks, latent, txt, cos, sin, mask, 8, 0, 1, keep_predictions=True)


@pytest.mark.parametrize("precision", [ec.FP32, ec.BF16], ids=["fp32", "bf16"])
def test_c1_full_step_against_oracle(deep, oracle_c1_step, precision):
    """One whole denoise step at C1 (input head, 36 blocks, output head, Euler) against the oracle with the
    per-tensor pipeline gates of tools/validate_pipeline.py:218-222 on the prediction and the latent."""
    ctx, model, _, _ = deep
    w, h, text, valid = C1
    latent, txt, cos, sin, mask = case(w, h, text, valid)
    ref_latent, ref_preds = oracle_c1_step
    s = ec.Session(model, w, h, text, valid, precision)
    try:
        s.set_conditioning(txt, cos, sin, mask)
        got, preds = s.denoise(latent, 8, 0, 1, keep_predictions=True)
    finally:
        s.close()
    name = "pipeline_fp32" if precision == ec.FP32 else "pipeline_bf16"
    ok_pred, pred_metrics = gate(ref_preds[0], preds[0], *GATES[name])
    ok_latent, latent_metrics = gate(ref_latent, got, *GATES[name])
    mode = "fp32" if precision == ec.FP32 else "bf16"
    print(f"C1 step 0, 36 blocks vs oracle {mode}: prediction nrmse={pred_metrics['nrmse']:.3e} "
          f"max_abs={pred_metrics['max_abs_error']:.3e}; latent nrmse={latent_metrics['nrmse']:.3e} "
          f"max_abs={latent_metrics['max_abs_error']:.3e}")
    assert ok_pred, pred_metrics
    assert ok_latent, latent_metrics


def test_c1_geometry_bf16_against_fp32_mode(deep):
    ctx, model, _, _ = deep
    w, h, text, valid = 32, 32, 32, 24
    latent, txt, cos, sin, mask = case(w, h, text, valid)
    out = {}
    for precision in (ec.FP32, ec.BF16):
        s = ec.Session(model, w, h, text, valid, precision)
        try:
            s.set_conditioning(txt, cos, sin, mask)
            first = s.denoise(latent, 8)
            again = s.denoise(latent, 8)
        finally:
            s.close()
        assert np.isfinite(first).all() and np.array_equal(first, again), "repeat execution must be bit-exact"
        out[precision] = first
    ok, metrics = gate(out[ec.FP32], out[ec.BF16], *GATES["pipeline_bf16"])
    print("C1 geometry, 36 blocks x 8 steps, BF16 vs FP32-exact", metrics)
    assert ok, metrics


def test_c2_geometry_bf16_against_fp32_mode(deep):
    """The headline configuration's geometry (64x64 packed latent + 64 text slots, 4160 tokens), all 36
    blocks and 8 steps: BF16 mode against the FP32-exact mode (which passes the oracle's FP32 gates at this
    block shape) within the BF16 pipeline gate, each mode repeating bit-exactly."""
    ctx, model, _, _ = deep
    w, h, text, valid = 64, 64, 64, 64
    latent, txt, cos, sin, mask = case(w, h, text, valid)
    out = {}
    for precision in (ec.FP32, ec.BF16):
        s = ec.Session(model, w, h, text, valid, precision)
        try:
            s.set_conditioning(txt, cos, sin, mask)
            first = s.denoise(latent, 8)
            again = s.denoise(latent, 8)
        finally:
            s.close()
        assert np.isfinite(first).all() and np.array_equal(first, again), "repeat execution must be bit-exact"
        out[precision] = first
    ok, metrics = gate(out[ec.FP32], out[ec.BF16], *GATES["pipeline_bf16"])
    print("C2 geometry, 36 blocks x 8 steps, BF16 vs FP32-exact", metrics)
    assert ok, metrics


def test_c1_step_folded_norm_against_unfolded(deep, oracle_c1_step, monkeypatch):
    """ERNIE_FOLD_NORM=1 folds each BF16 block's two RMSNorm + modulate passes into the GEMMs around them
    (the residual GEMMs write bf16(x g) and each row's sums of squares, the next GEMM applies rinv and
    W shift); the default keeps the norm kernels. One C1 step through 36 blocks in both forms against the oracle:
    the folded form within the pipeline gate and no further from the oracle than the norm-kernel form
    allows for one BF16 rounding of its own."""
    ctx, model, _, _ = deep
    w, h, text, valid = C1
    latent, txt, cos, sin, mask = case(w, h, text, valid)
    ref_latent, ref_preds = oracle_c1_step
    out = {}
    for fold in ("1", "0"):
        monkeypatch.setenv("ERNIE_FOLD_NORM", fold)
        s = ec.Session(model, w, h, text, valid, ec.BF16)
        try:
            s.set_conditioning(txt, cos, sin, mask)
            got, preds = s.denoise(latent, 8, 0, 1, keep_predictions=True)
            again, _ = s.denoise(latent, 8, 0, 1, keep_predictions=True)
        finally:
            s.close()
        assert np.array_equal(got, again), "repeat execution must be bit-exact"
        out[fold] = gate(ref_preds[0], preds[0], *GATES["pipeline_bf16"])
    (ok_f, m_f), (ok_u, m_u) = out["1"], out["0"]
    print(f"C1 step 0 prediction vs oracle: folded nrmse={m_f['nrmse']:.3e} max_abs={m_f['max_abs_error']:.3e}; "
          f"norm kernels nrmse={m_u['nrmse']:.3e} max_abs={m_u['max_abs_error']:.3e}")
    assert ok_f and ok_u, (m_f, m_u)
    assert m_f["nrmse"] <= 1.25 * m_u["nrmse"], (m_f, m_u)


@pytest.mark.parametrize("shape", [(32, 32, 32, 24), (86, 48, 2048, 1080)], ids=["c1_padded", "c3"])
@pytest.mark.parametrize("precision", [ec.FP32, ec.BF16], ids=["fp32", "bf16"])
def test_denoise_skips_rows_past_the_last_visible_key(deep, monkeypatch, shape, precision):
    """The denoise computes the image rows and the text rows up to the last visible key only: later text
    slots are masked keys whose own rows no image row reads (C3: 968 of 6176 rows). ERNIE_ALL_ROWS=1
    computes every row; the latents must be identical bit for bit, and a block-level call in between (which
    computes and stores every row) must not change the next denoise."""
    ctx, model, host_blocks, _ = deep
    w, h, text, valid = shape
    latent, txt, cos, sin, mask = case(w, h, text, valid)
    steps = (0, 2) if w * h <= 1024 else (0, 1)
    out = {}
    for all_rows in ("1", "0"):
        monkeypatch.setenv("ERNIE_ALL_ROWS", all_rows)
        s = ec.Session(model, w, h, text, valid, precision)
        try:
            s.set_conditioning(txt, cos, sin, mask)
            out[all_rows] = s.denoise(latent, 8, *steps)
            if all_rows == "0":
                n = w * h + text
                x = o.synth_normal(SEED, o.HIDDEN_STREAM, n * 4096).reshape(n, 4096)
                s.blocks(x, o.block_modulation(SEED), first=0, count=1)
                again = s.denoise(latent, 8, *steps)
                assert np.array_equal(out["0"], again), "a block-level call changed the next denoise"
        finally:
            s.close()
    assert np.isfinite(out["0"]).all()
    assert np.array_equal(out["0"], out["1"]), np.abs(out["0"] - out["1"]).max()
