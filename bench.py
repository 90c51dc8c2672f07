"""Benchmark of the B200 DiT denoiser hot path (one JSON line on rank 0).

Workload (the metric's 1024x1024 case): 36-block ERNIE DiT, 4096 image tokens
(64x64 packed latent) + 64 text tokens, BF16 mode, turbo 8-step schedule, one seed per GPU
(data-parallel, no collective in the data path; weak scaling). A bench "step" is one full denoise
step (input head, 36 blocks, output head, Euler update) on every rank's seed; images/s counts 8 steps
per image. Weights are seeded random-init (no checkpoint is available), inputs seeded N(0,1).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "ernie-image-ncnn-vulkan_b200"))
import dp  # noqa: E402  (data-parallel helpers of the package)

METRIC = "DiT denoise ms/step and images/s (8-step 1024²) at 1/2/4/8 B200; % BF16 peak"
# BASELINE.json configs as (packed width, packed height, DiT text slots, valid text tokens, precision).
# c2 is the metric's workload and the default; the others run single-GPU for their own bench lines.
CONFIGS = {
    "c1": (32, 32, 32, 32, "bf16", "C1 512x512: 32x32 packed latent (1024 image tokens) + 32 text tokens"),
    "c1-fp32": (32, 32, 32, 32, "fp32", "C1 512x512 in FP32-exact mode"),
    "c2": (64, 64, 64, 64, "bf16", "C2 1024x1024: 64x64 packed latent (4096 image tokens) + 64 text tokens"),
    "c3": (86, 48, 2048, 1080, "bf16",
           "C3 1376x768: 86x48 packed latent (4128 image tokens) + 2048-slot text bucket, 968 padded keys"),
    "c4": (128, 64, 64, 64, "bf16", "C4 2048x1024: 128x64 packed latent (8192 image tokens) + 64 text tokens"),
}
WIDTH, HEIGHT, TEXT, VALID = CONFIGS["c2"][:4]
STEPS_PER_IMAGE = 8
NUM_BLOCKS = 36
PARAMS_PER_BLOCK = 218_103_808  # 7 GEMMs: 4*4096^2 + 3*4096*12288
# DRAM bytes of one C2 up/gate GEMM launch from an ncu capture of the same launch shape (239.6 MB read +
# 93.1 MB written); the algorithmic bytes are A 34 MB + W 201 MB + h 102 MB = 337 MB.
UPGATE_TRAFFIC_C2 = 332.7e6


def step_flops(tokens, valid_keys, blocks=NUM_BLOCKS):
    """Algorithmic FLOPs of one denoise step: 2*N*params (GEMMs) + 4*N*N_valid*4096 (QK^T and PV)."""
    return blocks * (2.0 * tokens * PARAMS_PER_BLOCK + 4.0 * tokens * valid_keys * 4096)


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        p = json.load(open(path))
        return p["bf16_tflops"], p.get("bf16_tflops_sustained", p["bf16_tflops"]), p["hbm_gbs"], "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = [l.split(",") for l in open(self.file.name).read().strip().splitlines() if l.strip()]
        os.unlink(self.file.name)
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].strip().replace(".", "").isdigit()]
        note = None
        if not sm:
            # a timed region shorter than the sampling interval: one sample right after it
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=10)
                rows = [l.split(",") for l in out.stdout.strip().splitlines() if l.strip()]
            except (OSError, subprocess.TimeoutExpired):
                rows = []
            sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].strip().replace(".", "").isdigit()]
            if not sm:
                return None
            note = "timed region shorter than the 200 ms sampling interval: one sample taken right after it"
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows if len(r) >= 9 for i in range(4) if r[5 + i].strip() == "Active"})
        info = {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "samples": len(sm) if not note else 0,
                "reasons": reasons}
        if note:
            info["note"] = note
        return info


def dist_setup(gpus):
    rank, local, world = dp.world_from_env()
    if world != gpus and world > 1:
        raise SystemExit(f"--gpus {gpus} but WORLD_SIZE {world}")
    pg = None
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
        pg = dist
    return rank, local, world, pg


def barrier(pg):
    dp.barrier(pg)


def max_over_ranks(pg, value):
    return dp.max_over_ranks(pg, value, device="cuda")


def cpu_baseline_block(threads=None):
    """One oracle (CPU restatement) DiT block at the workload's token count, timed on the host cores."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as o
    if threads:
        o.lib().orc_set_num_threads(threads)
    seed = 0
    w = o.BlockWeights(seed, 0)
    cos, sin, mask = o.dit_constants(WIDTH, HEIGHT, VALID, TEXT)
    n = WIDTH * HEIGHT + TEXT
    x = o.synth_normal(seed, o.HIDDEN_STREAM, n * 4096).reshape(n, 4096)
    mod = o.block_modulation(seed)
    t0 = time.perf_counter()
    o.block(x, w, mod, cos, sin, mask)
    dt = time.perf_counter() - t0
    return dt, o.lib().orc_num_threads()


# The reference's own published CPU timing of the same block: ncnn CPU FP32 on 4 threads of a Ryzen 7 7745HX,
# 4.484 / 4.434 / 4.403 s for one 4160-token block (artifacts/2026-09-05/dit-block/README.md:53 of the
# reference). It cannot be reproduced here (empty ncnn submodule); it is printed beside the port's timing so
# that the GPU/CPU ratio can also be read against the real ncnn CPU path (about 3x faster per core).
REFERENCE_CPU_BLOCK_S = 4.434
REFERENCE_CPU_THREADS = 4


def reference_published_cpu():
    image_s = REFERENCE_CPU_BLOCK_S * NUM_BLOCKS * STEPS_PER_IMAGE
    return {"value": 1.0 / image_s, "unit": "images/s", "cores": REFERENCE_CPU_THREADS,
            "block_s": REFERENCE_CPU_BLOCK_S,
            "source": "reference artifacts/2026-09-05/dit-block/README.md:53: ncnn CPU FP32, 4 threads, Ryzen 7 "
                      "7745HX, one 4160-token block (median of 3); x36 blocks x8 steps; published, not re-run",
            "applies_to": "c2 (4160 tokens)"}


def run_reference(args):
    """--impl reference: the CPU restatement of the reference's CPU path on this host's cores (the
    reference itself cannot be built: empty ncnn submodule, no Rust toolchain, no Vulkan)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    times = []
    cores = 1
    for i in range(args.warmup + args.steps):
        dt, cores = cpu_baseline_block()
        if i >= args.warmup:
            times.append(dt)
    block_s = statistics.median(times)
    step_s = block_s * NUM_BLOCKS
    image_s = step_s * STEPS_PER_IMAGE
    value = 1.0 / image_s
    # ms_per_step is the measured time of one timed step of this run (one block: the bounded sample), so
    # steps x ms_per_step matches the run's own clock; the 36-block DiT step it extrapolates to is in config
    line = {"metric": METRIC, "impl": "reference", "value": value, "unit": "images/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": block_s * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{args.workload}, 36 blocks, 8 steps, 1 seed",
                       "sample": "each timed step is 1 DiT block (ms_per_step); value extrapolates the median "
                                 "block x36 blocks x8 steps",
                       "extrapolated_ms_per_dit_step": step_s * 1e3},
            "cpu_baseline": {"value": value, "unit": "images/s", "cores": cores, "kind": "port",
                             "sample": f"one DiT block ({WIDTH * HEIGHT + TEXT} tokens) of the oracle per step; "
                                       "x36 x8 extrapolated",
                             "reference_published": reference_published_cpu() if args.config == "c2" else None},
            "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


DATASHEET_BF16_TFLOPS = 2250.0  # B200 dense BF16, NVIDIA's datasheet figure (context beside the measured peak)
KERNELS = {"norm_modulate": 0, "qkv_gemm": 1, "attention": 2, "out_gemm": 3, "upgate_gemm": 5, "down_gemm": 6}

# ---- the stage after the denoise loop: VAE decode (--stage vae) -----------------------------------------
VAE_METRIC = "VAE decode images/s (1024² output from the 128x128x32 unpacked latent); % BF16 peak"
VAE_LATENT = (128, 128)  # unpacked latent [32][h][w] of a 1024x1024 image (the C2 request's decode)
VAE_SAMPLE = (16, 16)    # CPU sample: a 128x128 output, 1/64 of the pixels


def vae_cpu_sample():
    """The oracle's decode (float64 numpy, all host cores) of one VAE_SAMPLE latent: (seconds, threads)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import vae as ov
    threads = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_info
        threads = max((i.get("num_threads", 1) for i in threadpool_info()), default=threads)
    except ImportError:
        pass
    w = ov.synth_weights(4321)
    u = np.random.default_rng(0).standard_normal((32,) + VAE_SAMPLE).astype(np.float32)
    ov.decode(w, u)  # warm
    t0 = time.perf_counter()
    ov.decode(w, u)
    return time.perf_counter() - t0, threads


def vae_cpu_line_fields(seconds, threads):
    scale = (VAE_LATENT[0] * VAE_LATENT[1]) / (VAE_SAMPLE[0] * VAE_SAMPLE[1])
    image_s = seconds * scale
    return 1.0 / image_s, {"value": 1.0 / image_s, "unit": "images/s", "cores": threads, "kind": "port",
                           "sample": f"oracle decode of a {VAE_SAMPLE[0]}x{VAE_SAMPLE[1]} latent "
                                     f"({8 * VAE_SAMPLE[0]}x{8 * VAE_SAMPLE[1]} output, {seconds:.2f} s), "
                                     f"scaled x{scale:.0f} by pixel count (the attention's quadratic term, "
                                     "5% of the 1024² FLOPs, is not scaled up)"}


# ---- the stage before the denoise loop: prompt encoder (--stage text) -------------------------------------
TEXT_METRIC = "prompt encoder ms/prompt (25 Mistral decoder layers, hidden 3072) at the request's text bucket"
TEXT_LAYER_FLOPS = 2 * (3072 * 6144 + 4096 * 3072 + 3072 * 18432 + 9216 * 3072)  # GEMM FLOPs per token per layer
TEXT_LAYER_BYTES = 2 * (6144 * 3072 + 3072 * 4096 + 18432 * 3072 + 3072 * 9216)  # BF16 weight bytes per layer


def text_flops(bucket, layers=25):
    """GEMMs (2 * tokens * params) + causal attention (2 * 2 * 32 heads * 128 * tokens * (tokens + 1) / 2)."""
    return layers * (bucket * TEXT_LAYER_FLOPS + 2.0 * 2 * 32 * 128 * bucket * (bucket + 1) / 2)


def text_cpu_sample(bucket):
    """The oracle's layer (float64 numpy) at a bounded token count, timed on the host cores: (s per layer, tokens)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import text as ot
    tokens = min(bucket, 64)
    w = ot.TextLayerWeights(4321, 0)
    f = (1.0 / 1000000.0 ** (np.arange(64) / 64)).astype(np.float32)
    cos, sin = ot.text_constants(f, tokens)
    x = np.random.default_rng(0).standard_normal((tokens, 3072)) * 0.2
    ot.layer(w, x, cos, sin)  # warm (weight widening cached)
    t0 = time.perf_counter()
    ot.layer(w, x, cos, sin)
    return time.perf_counter() - t0, tokens


def run_text_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    times, tokens = [], 1
    for i in range(args.warmup + args.steps):
        dt, tokens = text_cpu_sample(TEXT)
        if i >= args.warmup:
            times.append(dt)
    ms = 1000.0 * statistics.median(times) * 25 * (TEXT / tokens)
    cpu = {"value": ms, "unit": "ms/prompt", "cores": os.cpu_count() or 1, "kind": "port",
           "sample": f"one oracle layer at {tokens} tokens, x25 layers" +
                     (f", x{TEXT / tokens:.0f} by token count" if TEXT > tokens else "")}
    line = {"metric": TEXT_METRIC, "impl": "reference", "value": ms, "unit": "ms/prompt", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * statistics.median(times),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": f"prompt encode, {TEXT}-token bucket, 25 layers",
                       "sample": cpu["sample"] + " (ms_per_step: one timed sample)"},
            "cpu_baseline": cpu,
            "e2e": {"value": ms, "unit": "ms/prompt", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_text(args):
    """One prompt encode per GPU per step (25 layers at the config's text bucket)."""
    import ernie_cuda as ec
    rank, local, world, pg = dist_setup(args.gpus)
    ctx = ec.Context(local)
    model = ec.TextModel(ctx, 25)
    model.synthesize(4321)
    precision = ec.BF16 if args.precision == "bf16" else ec.FP32
    bucket = TEXT
    f = (1.0 / 1000000.0 ** (np.arange(64) / 64)).astype(np.float32)
    cos, sin, _ = ec.text_constants(f, bucket)
    x = (np.random.default_rng(dp.request_seed(3000, rank)).standard_normal((bucket, 3072)) * 0.2).astype(np.float32)
    bx, bc, bs, bo = ctx.to_device(x), ctx.to_device(cos), ctx.to_device(sin), ctx.buffer(x.nbytes)
    for _ in range(args.warmup):
        model.run_blocks_device(bx, bucket, bc, bs, bo, precision)
    clocks = ClockSampler(local)
    barrier(pg)
    ctx.synchronize()
    clocks.start()
    ctx.record(0)
    for _ in range(args.steps):
        model.run_blocks_device(bx, bucket, bc, bs, bo, precision)
    ctx.record(1)
    ctx.synchronize()
    clock_info = clocks.stop()
    barrier(pg)
    ms = max_over_ranks(pg, ctx.elapsed(0, 1)) / args.steps
    flops = text_flops(bucket)
    bf16_peak, _, hbm_peak, peak_kind = peaks()
    weight_gbs = 25 * TEXT_LAYER_BYTES / (ms * 1e-3) / 1e9
    tflops = flops / (ms * 1e-3) / 1e12
    bound = "hbm" if bucket <= 256 else "tensor"
    roofline = ({"bound": "hbm", "kernel": "whole encode (weight streaming)", "achieved": weight_gbs, "peak": hbm_peak,
                 "unit": "GB/s", "frac": weight_gbs / hbm_peak, "peak_kind": peak_kind, "traffic": None}
                if bound == "hbm" else
                {"bound": "tensor", "kernel": "whole encode", "achieved": tflops, "peak": bf16_peak, "unit": "TFLOP/s",
                 "frac": tflops / bf16_peak, "peak_kind": peak_kind, "traffic": None})
    e2e = None
    if not args.no_e2e:
        model.run_blocks(x, cos, sin, precision)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            out = model.run_blocks(x, cos, sin, precision)
        dt = max_over_ranks(pg, (time.perf_counter() - t0) / args.steps)
        assert np.isfinite(out).all()
        e2e = {"value": 1000.0 * dt, "unit": "ms/prompt", "h2d_bytes_per_step": x.nbytes + cos.nbytes + sin.nbytes,
               "d2h_bytes_per_step": out.nbytes,
               "call": "ernie_cuda_text_run_blocks (host embedded prompt and constants in, host hidden state out)"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        layer_s, tokens = text_cpu_sample(bucket)
        est = layer_s * 25 * (bucket / tokens)
        cpu = {"value": 1000.0 * est, "unit": "ms/prompt", "cores": os.cpu_count() or 1, "kind": "port",
               "sample": f"one oracle layer at {tokens} tokens ({layer_s:.2f} s), x25 layers"
                         + (f", x{bucket / tokens:.0f} by token count" if bucket > tokens else "")}
    if rank == 0:
        line = {"metric": TEXT_METRIC, "value": ms, "unit": "ms/prompt", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": False, "scaling": "weak",
                "vs_baseline": None, "dtype": args.precision, "data": "synthetic",
                "config": {"workload": f"prompt encode, {bucket}-token bucket, 25 layers, one prompt per GPU",
                           "tokens": bucket, "tflops": tflops, "weight_stream_gbs": weight_gbs,
                           "l2": "inputs larger than L2 (5.65 GB of weights per encode)"},
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": 8 * 25 * args.steps,
                "clocks": clock_info}
        print(json.dumps(line), flush=True)
    for b in (bx, bc, bs, bo):
        b.free()
    model.close()
    ctx.close()
    if pg is not None:
        pg.destroy_process_group()


def run_vae_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    times = []
    threads = 1
    for i in range(args.warmup + args.steps):
        dt, threads = vae_cpu_sample()
        if i >= args.warmup:
            times.append(dt)
    value, cpu = vae_cpu_line_fields(statistics.median(times), threads)
    line = {"metric": VAE_METRIC, "impl": "reference", "value": value, "unit": "images/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * statistics.median(times),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": "VAE decode of one 1024x1024 image",
                       "sample": cpu["sample"] + " (ms_per_step: one timed sample)"},
            "cpu_baseline": cpu,
            "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_vae(args):
    """One VAE decode per GPU per step (independent images, no collective)."""
    import ernie_cuda as ec
    rank, local, world, pg = dist_setup(args.gpus)
    ctx = ec.Context(local)
    vae = ec.Vae(ctx)
    vae.synthesize(4321)
    precision = ec.BF16 if args.precision == "bf16" else ec.FP32
    h, w = tuple(int(v) for v in args.vae_latent.split(",")) if args.vae_latent else VAE_LATENT
    u = np.random.default_rng(dp.request_seed(2000, rank)).standard_normal((32, h, w)).astype(np.float32)
    out_elems = 3 * 64 * h * w
    src, dst, rgb = ctx.to_device(u), ctx.buffer(out_elems * 4), ctx.buffer(out_elems)
    launches = vae.launches(w, h, precision)
    for _ in range(args.warmup):
        vae.decode_device(src, w, h, dst, precision, rgb)
    clocks = ClockSampler(local)
    barrier(pg)
    ctx.synchronize()
    clocks.start()
    ctx.record(0)
    for _ in range(args.steps):
        vae.decode_device(src, w, h, dst, precision, rgb)
    ctx.record(1)
    ctx.synchronize()
    clock_info = clocks.stop()
    barrier(pg)
    ms = max_over_ranks(pg, ctx.elapsed(0, 1)) / args.steps
    images_per_s = world * 1000.0 / ms

    prof = vae.profile(w, h, precision, iters=3)
    bf16_peak, _, hbm_peak, peak_kind = peaks()
    classes = {}
    for name, (t, work) in prof.items():
        tensor = name in ("conv", "attention_gemm")
        rate = work / (t * 1e-3) / (1e12 if tensor else 1e9) if t > 0 else 0.0
        classes[name] = {"ms": t, "work": work, "work_unit": "FLOP" if tensor else "byte",
                         "achieved": rate, "unit": "TFLOP/s" if tensor else "GB/s",
                         "frac": rate / (bf16_peak if tensor else hbm_peak)}
    total_flops = prof["conv"][1] + prof["attention_gemm"][1]
    conv = classes["conv"]

    e2e = None
    if not args.no_e2e:
        vae.decode(u, precision, rgb=True)
        barrier(pg)
        reps = max(1, args.steps)
        t0 = time.perf_counter()
        for _ in range(reps):
            decoded, pixels, bad = vae.decode(u, precision, rgb=True)
        dt = max_over_ranks(pg, (time.perf_counter() - t0) / reps)
        assert bad == 0 and np.isfinite(decoded).all()
        e2e = {"value": world / dt, "unit": "images/s", "h2d_bytes_per_step": u.nbytes,
               "d2h_bytes_per_step": decoded.nbytes + pixels.nbytes,
               "call": "ernie_cuda_vae_decode (host unpacked latent in, host decoded FP32 + RGB bytes out)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        _, cpu = vae_cpu_line_fields(*vae_cpu_sample())

    if rank == 0:
        line = {"metric": VAE_METRIC, "value": images_per_s, "unit": "images/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": args.precision, "data": "synthetic",
                "config": {"workload": "VAE decode (post_quant_conv + AutoencoderKLFlux2 decoder + RGB bytes) of "
                                       f"one {8 * w}x{8 * h} image per GPU per step, seeded synthetic weights",
                           "global_batch": world, "parallelism": f"dp{world}",
                           "l2": "inputs larger than L2 (activations of 0.5-1 GB per layer at the top levels)",
                           "decode_tflops": total_flops / (ms * 1e-3) / 1e12, "kernel_classes": classes},
                "roofline": {"bound": "tensor", "kernel": "conv_kernel (all decoder convolutions)",
                             "achieved": conv["achieved"], "peak": bf16_peak, "unit": "TFLOP/s",
                             "frac": conv["achieved"] / bf16_peak, "peak_kind": peak_kind, "traffic": None},
                "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches * args.steps, "clocks": clock_info}
        print(json.dumps(line), flush=True)
    vae.close()
    ctx.close()
    if pg is not None:
        pg.destroy_process_group()


# ---- img2img's image latent: VAE encode (--stage vae-encode) -------------------------------------------
VAE_ENC_METRIC = "VAE encode images/s (1024² RGB -> mean, packed and normalized latents); % BF16 peak"
VAE_ENC_IMAGE = (1024, 1024)  # (height, width): the reference's reviewed large encoder shape
VAE_ENC_SAMPLE = (128, 128)   # CPU sample: 1/64 of the pixels


def vae_encode_cpu_sample():
    """The oracle's encode (float64 numpy, all host cores) of one VAE_ENC_SAMPLE image: (seconds, threads)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import vae as ov
    threads = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_info
        threads = max((i.get("num_threads", 1) for i in threadpool_info()), default=threads)
    except ImportError:
        pass
    w = ov.synth_weights(4321, table=ov.encoder_table())
    rgb = ov.rgb_fixture(VAE_ENC_SAMPLE[1], VAE_ENC_SAMPLE[0])
    ov.encode(w, rgb)  # warm
    t0 = time.perf_counter()
    ov.encode(w, rgb)
    return time.perf_counter() - t0, threads


def vae_encode_cpu_fields(seconds, threads):
    scale = (VAE_ENC_IMAGE[0] * VAE_ENC_IMAGE[1]) / (VAE_ENC_SAMPLE[0] * VAE_ENC_SAMPLE[1])
    image_s = seconds * scale
    return 1.0 / image_s, {"value": 1.0 / image_s, "unit": "images/s", "cores": threads, "kind": "port",
                           "sample": f"oracle encode of a {VAE_ENC_SAMPLE[1]}x{VAE_ENC_SAMPLE[0]} image "
                                     f"({seconds:.2f} s), scaled x{scale:.0f} by pixel count (the attention's "
                                     "quadratic term, 11% of the 1024² FLOPs, is not scaled up)"}


def run_vae_encode_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    times, threads = [], 1
    for i in range(args.warmup + args.steps):
        dt, threads = vae_encode_cpu_sample()
        if i >= args.warmup:
            times.append(dt)
    value, cpu = vae_encode_cpu_fields(statistics.median(times), threads)
    line = {"metric": VAE_ENC_METRIC, "impl": "reference", "value": value, "unit": "images/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * statistics.median(times),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": "VAE encode of one 1024x1024 image",
                       "sample": cpu["sample"] + " (ms_per_step: one timed sample)"},
            "cpu_baseline": cpu,
            "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_vae_encode(args):
    """One VAE encode per GPU per step (independent images, no collective)."""
    import ernie_cuda as ec
    rank, local, world, pg = dist_setup(args.gpus)
    ctx = ec.Context(local)
    enc = ec.VaeEncoder(ctx)
    enc.synthesize(4321)
    precision = ec.BF16 if args.precision == "bf16" else ec.FP32
    h, w = VAE_ENC_IMAGE
    rgb = np.random.default_rng(dp.request_seed(4000, rank)).integers(0, 256, (h, w, 3), dtype=np.uint8)
    src = ctx.to_device(rgb)
    outs = [ctx.buffer(32 * h * w // 64 * 4), ctx.buffer(128 * h * w // 256 * 4), ctx.buffer(128 * h * w // 256 * 4)]
    launches = enc.launches(w, h, precision)
    for _ in range(args.warmup):
        enc.encode_device(src, w, h, *outs, precision=precision)
    clocks = ClockSampler(local)
    barrier(pg)
    ctx.synchronize()
    clocks.start()
    ctx.record(0)
    for _ in range(args.steps):
        enc.encode_device(src, w, h, *outs, precision=precision)
    ctx.record(1)
    ctx.synchronize()
    clock_info = clocks.stop()
    barrier(pg)
    ms = max_over_ranks(pg, ctx.elapsed(0, 1)) / args.steps

    prof = enc.profile(w, h, precision, iters=3)
    bf16_peak, _, hbm_peak, peak_kind = peaks()
    classes = {}
    for name, (t, work) in prof.items():
        tensor = name in ("conv", "attention_gemm")
        rate = work / (t * 1e-3) / (1e12 if tensor else 1e9) if t > 0 else 0.0
        classes[name] = {"ms": t, "work": work, "work_unit": "FLOP" if tensor else "byte",
                         "achieved": rate, "unit": "TFLOP/s" if tensor else "GB/s",
                         "frac": rate / (bf16_peak if tensor else hbm_peak)}
    total_flops = prof["conv"][1] + prof["attention_gemm"][1]
    conv = classes["conv"]

    e2e = None
    if not args.no_e2e:
        enc.encode(rgb, precision)
        barrier(pg)
        reps = max(1, args.steps)
        t0 = time.perf_counter()
        for _ in range(reps):
            mean, packed, normalized, bad = enc.encode(rgb, precision)
        dt = max_over_ranks(pg, (time.perf_counter() - t0) / reps)
        assert bad == 0 and np.isfinite(normalized).all()
        e2e = {"value": world / dt, "unit": "images/s", "h2d_bytes_per_step": rgb.nbytes,
               "d2h_bytes_per_step": mean.nbytes + packed.nbytes + normalized.nbytes,
               "call": "ernie_cuda_vae_encode (host RGB bytes in, host mean/packed/normalized FP32 out)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        _, cpu = vae_encode_cpu_fields(*vae_encode_cpu_sample())

    if rank == 0:
        line = {"metric": VAE_ENC_METRIC, "value": world * 1000.0 / ms, "unit": "images/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": args.precision, "data": "synthetic",
                "config": {"workload": "VAE encode (AutoencoderKLFlux2 encoder + quant_conv + pixel_unshuffle + "
                                       f"BatchNorm) of one {w}x{h} RGB image per GPU per step, seeded synthetic "
                                       "weights", "global_batch": world, "parallelism": f"dp{world}",
                           "l2": "inputs larger than L2 (activations of 0.5 GB per layer at the top level)",
                           "encode_tflops": total_flops / (ms * 1e-3) / 1e12, "kernel_classes": classes},
                "roofline": {"bound": "tensor", "kernel": "conv_kernel (all encoder convolutions)",
                             "achieved": conv["achieved"], "peak": bf16_peak, "unit": "TFLOP/s",
                             "frac": conv["achieved"] / bf16_peak, "peak_kind": peak_kind, "traffic": None},
                "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches * args.steps, "clocks": clock_info}
        print(json.dumps(line), flush=True)
    src.free()
    for b in outs:
        b.free()
    enc.close()
    ctx.close()
    if pg is not None:
        pg.destroy_process_group()


# ---- the optional prompt enhancer (--stage pe) ---------------------------------------------------------
PE_METRIC = "prompt enhancer decode ms/token (26 Mistral layers + 131072-way LM head, K/V cache after a 512-token prompt)"
PE_LAYERS, PE_PROMPT = 26, 512
# BF16 weights streamed per decoded token: 26 layers x (q/k/v/o + gate/up/down) + the LM head
PE_BYTES_PER_TOKEN = PE_LAYERS * TEXT_LAYER_BYTES + 2 * 131072 * 3072


def pe_cpu_sample():
    """One decode token of the oracle (float64 numpy, all host cores): one layer on one token x 26 plus the LM
    head measured on 16384 of its 131072 rows x 8. Returns (seconds per token, sample description)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import text as ot
    w = ot.TextLayerWeights(4321, 0)
    f = (1.0 / 1000000.0 ** (np.arange(64) / 64)).astype(np.float32)
    cos, sin = ot.text_constants(f, 1)
    x = np.random.default_rng(0).standard_normal((1, 3072)) * 0.2
    ot.layer(w, x, cos, sin)  # warm (weight widening cached)
    t0 = time.perf_counter()
    ot.layer(w, x, cos, sin)
    layer_s = time.perf_counter() - t0
    gamma, head = ot.head_weights(4321, 16384)
    head64 = head.astype(np.float64)
    t0 = time.perf_counter()
    ot.head_logits(gamma, head64, x[0])
    head_s = (time.perf_counter() - t0) * 8
    return PE_LAYERS * layer_s + head_s, (f"one oracle layer on one token ({layer_s:.3f} s) x26 + the LM head on "
                                          f"16384 rows ({head_s / 8:.3f} s) x8; attention over the cache omitted")


def run_pe_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    times, sample = [], ""
    for i in range(args.warmup + args.steps):
        dt, sample = pe_cpu_sample()
        if i >= args.warmup:
            times.append(dt)
    ms = 1000.0 * statistics.median(times)
    cpu = {"value": ms, "unit": "ms/token", "cores": os.cpu_count() or 1, "kind": "port", "sample": sample}
    line = {"metric": PE_METRIC, "impl": "reference", "value": ms, "unit": "ms/token", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": "prompt enhancer decode, one token", "sample": sample}, "cpu_baseline": cpu,
            "e2e": {"value": ms, "unit": "ms/token", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_pe(args):
    """One decoded token per GPU per step: PeSession append of one row + the LM head, after a 512-token prefill."""
    import ernie_cuda as ec
    rank, local, world, pg = dist_setup(args.gpus)
    ctx = ec.Context(local)
    model = ec.TextModel(ctx, PE_LAYERS)
    model.synthesize(4321)
    model.synthesize_head(4321)
    precision = ec.BF16 if args.precision == "bf16" else ec.FP32
    total = PE_PROMPT + args.warmup + args.steps
    f = (1.0 / 1000000.0 ** (np.arange(64) / 64)).astype(np.float32)
    cos, sin, _ = ec.text_constants(f, min(total, 2048))
    x = (np.random.default_rng(dp.request_seed(5000, rank)).standard_normal((total, 3072)) * 0.2).astype(np.float32)
    session = ec.PeSession(model, total, precision)
    t0 = time.perf_counter()
    for c in range(0, PE_PROMPT, 32):
        hidden = session.append(x[c:c + 32], cos[c:c + 32], sin[c:c + 32])
    prefill_s = time.perf_counter() - t0
    pos = PE_PROMPT
    for _ in range(args.warmup):
        hidden = session.append(x[pos:pos + 1], cos[pos:pos + 1], sin[pos:pos + 1])
        logits = session.logits(hidden[0])
        pos += 1
    clocks = ClockSampler(local)
    barrier(pg)
    ctx.synchronize()
    clocks.start()
    ctx.record(0)
    w0 = time.perf_counter()
    for _ in range(args.steps):
        hidden = session.append(x[pos:pos + 1], cos[pos:pos + 1], sin[pos:pos + 1])
        logits = session.logits(hidden[0])
        pos += 1
    ctx.record(1)
    ctx.synchronize()
    wall = time.perf_counter() - w0
    clock_info = clocks.stop()
    barrier(pg)
    ms = max_over_ranks(pg, ctx.elapsed(0, 1)) / args.steps
    e2e_ms = 1000.0 * max_over_ranks(pg, wall) / args.steps
    assert np.isfinite(logits).all()
    _, _, hbm_peak, peak_kind = peaks()
    gbs = PE_BYTES_PER_TOKEN / (ms * 1e-3) / 1e9
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        s_tok, sample = pe_cpu_sample()
        cpu = {"value": 1000.0 * s_tok, "unit": "ms/token", "cores": os.cpu_count() or 1, "kind": "port",
               "sample": sample}
    if rank == 0:
        line = {"metric": PE_METRIC, "value": ms, "unit": "ms/token", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": False, "scaling": "weak",
                "vs_baseline": None, "dtype": args.precision, "data": "synthetic",
                "config": {"workload": f"prompt enhancer, {PE_LAYERS} layers, {PE_PROMPT}-token prompt prefilled in "
                                       "32-token chunks, then one token per step (append + LM head), one session "
                                       "per GPU", "prefill_tokens_per_s": PE_PROMPT / prefill_s,
                           "weight_bytes_per_token": PE_BYTES_PER_TOKEN,
                           "l2": "inputs larger than L2 (6.9 GB of weights per token)"},
                "roofline": {"bound": "hbm", "kernel": "whole decode step (weight streaming)", "achieved": gbs,
                             "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak, "peak_kind": peak_kind,
                             "traffic": None},
                "cpu_baseline": cpu,
                "e2e": {"value": e2e_ms, "unit": "ms/token", "h2d_bytes_per_step": 3072 * 4 + 2 * 128 * 4,
                        "d2h_bytes_per_step": 3072 * 4 + 131072 * 4,
                        "call": "ernie_cuda_pe_session_append (one host row) + ernie_cuda_pe_logits (host logits)"},
                # per token: 9 kernels per layer (norm, qkv, rotary, cache append, attention, o_proj, norm,
                # gate/up, down), the position advance, and the head (norm + product)
                "gpu_launches": args.steps * (9 * PE_LAYERS + 3), "clocks": clock_info}
        print(json.dumps(line), flush=True)
    session.close()
    model.close()
    ctx.close()
    if pg is not None:
        pg.destroy_process_group()


def nccl_version(torch):
    v = torch.cuda.nccl.version()
    return ".".join(map(str, v)) if isinstance(v, (tuple, list)) else str(v)


def run_exchange(args):
    """Reference for the sequence-parallel exchange: the same bytes moved by NCCL all-to-alls instead of the
    library's epilogue peer stores. Per DiT block, one all_to_all_single of this rank's Q, K and V rows of
    every member's heads (3 x S x 4096 BF16 values out) and one of the attention rows back (S x 4096); 36
    blocks per step; no compute, so the time is what a plain NCCL exchange adds to each step if nothing
    hides it. Device-timed with CUDA events on the launching stream, max over ranks."""
    import torch
    import ernie_cuda as ec
    rank, local, world, pg = dist_setup(args.gpus)
    if world < 2:
        if rank == 0:
            print(json.dumps({"metric": "SP exchange ms/step (NCCL all-to-all reference)",
                              "unavailable": "needs 2 or more ranks under torchrun"}), flush=True)
        return
    tokens, image = WIDTH * HEIGHT + TEXT, WIDTH * HEIGHT
    shard = ec.sp_layout(tokens, image, world, rank)[0]
    dev = torch.device("cuda", local)
    qkv_in = torch.randn(3 * shard * 4096, device=dev).to(torch.bfloat16)
    qkv_out = torch.empty_like(qkv_in)
    o_in = torch.randn(shard * 4096, device=dev).to(torch.bfloat16)
    o_out = torch.empty_like(o_in)
    blocks = args.blocks

    def step():
        for _ in range(blocks):
            pg.all_to_all_single(qkv_out, qkv_in)
            pg.all_to_all_single(o_out, o_in)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    barrier(pg)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        step()
    end.record()
    torch.cuda.synchronize(dev)
    barrier(pg)
    ms_step = max_over_ranks(pg, start.elapsed_time(end) / args.steps)
    if rank == 0:
        sent = (4 * shard * 4096 * 2) * (world - 1) // world  # bytes that leave this GPU per block
        ms_block = ms_step / blocks
        print(json.dumps({
            "metric": "SP exchange ms/step (NCCL all-to-all reference)", "impl": "nccl-reference",
            "value": ms_step, "unit": "ms/step", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": False, "data": "synthetic",
            "config": {"workload": f"{args.workload}: the exchange volumes of one Ulysses step, {blocks} blocks x 2 "
                                   "all_to_all_single (Q/K/V rows out, attention rows back), BF16",
                       "shard_rows": shard, "ms_per_block": ms_block, "bytes_out_per_rank_per_block": sent,
                       "gb_per_s_out_per_rank": sent / (ms_block * 1e-3) / 1e9,
                       "nccl": nccl_version(torch)}}), flush=True)
    pg.destroy_process_group()


def pipeline_stages(ctx, args, ms_per_step, reps=3):
    """Device time of the whole image on this GPU: prompt encode (25 layers at the config's text bucket),
    8 denoise steps (the metric's ms_per_step x 8) and the VAE decode (unpacked latent 2h x 2w), BF16."""
    import ernie_cuda as ec
    out = {"denoise_ms": 8 * ms_per_step}
    text = ec.TextModel(ctx, 25)
    vae = ec.Vae(ctx)
    bufs = []
    try:
        text.synthesize(4321)
        vae.synthesize(4321)
        f = (1.0 / 1000000.0 ** (np.arange(64) / 64)).astype(np.float32)
        cos, sin, _ = ec.text_constants(f, TEXT)
        x = (np.random.default_rng(7).standard_normal((TEXT, 3072)) * 0.2).astype(np.float32)
        bx, bc, bs, bo = ctx.to_device(x), ctx.to_device(cos), ctx.to_device(sin), ctx.buffer(x.nbytes)
        u = np.random.default_rng(8).standard_normal((32, 2 * HEIGHT, 2 * WIDTH)).astype(np.float32)
        bu, bd = ctx.to_device(u), ctx.buffer(3 * 64 * u[0].size * 4)
        bufs = [bx, bc, bs, bo, bu, bd]
        for _ in range(2):
            text.run_blocks_device(bx, TEXT, bc, bs, bo, ec.BF16)
            vae.decode_device(bu, 2 * WIDTH, 2 * HEIGHT, bd, ec.BF16)
        ctx.synchronize()
        ctx.record(0)
        for _ in range(reps):
            text.run_blocks_device(bx, TEXT, bc, bs, bo, ec.BF16)
        ctx.record(1)
        for _ in range(reps):
            vae.decode_device(bu, 2 * WIDTH, 2 * HEIGHT, bd, ec.BF16)
        ctx.record(2)
        ctx.synchronize()
        out["text_encode_ms"] = ctx.elapsed(0, 1) / reps
        out["vae_decode_ms"] = ctx.elapsed(1, 2) / reps
        out["image_ms"] = out["text_encode_ms"] + out["denoise_ms"] + out["vae_decode_ms"]
        out["images_per_s_per_gpu"] = 1000.0 / out["image_ms"]
        out["note"] = ("text encoder + 8 DiT steps + VAE decode of one image on one GPU, BF16, device time; the "
                       "tokenizer is out of scope")
    finally:
        for b in bufs:
            b.free()
        text.close()
        vae.close()
    return out


def run_kernel_only(args):
    """Set up the C2 session (with --blocks resident blocks) and launch one block kernel `iters` times.
    Used under ncu on a small case: a 2-block model keeps the device footprint near 1.6 GB while every
    operand of the C2 kernels is still larger than L2."""
    import ernie_cuda as ec
    ctx = ec.Context(0)
    model = ec.Model(ctx, args.blocks)
    model.synthesize(1234)
    session = ec.Session(model, WIDTH, HEIGHT, TEXT, VALID, ec.BF16 if args.precision == "bf16" else ec.FP32)
    rng = np.random.default_rng(0)
    cos, sin, mask = ec.dit_constants(WIDTH, HEIGHT, VALID, TEXT)
    session.set_conditioning(rng.standard_normal((TEXT, 3072), dtype=np.float32), cos, sin, mask)
    session.denoise(rng.standard_normal((128, HEIGHT, WIDTH), dtype=np.float32), STEPS_PER_IMAGE, 0, 1)
    # the buffers now hold one real step's activations; each block kernel ran `blocks` times above
    ms = session.profile(KERNELS[args.kernel_only], args.iters)
    print(json.dumps({"kernel": args.kernel_only, "ms_per_launch": ms, "launches": args.iters + 1}), flush=True)
    session.close()
    model.close()
    ctx.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--precision", choices=["bf16", "fp32"], default=None)
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c2")
    ap.add_argument("--parallel", choices=["dp", "sp"], default=None,
                    help="dp: one seed per GPU (default); sp: one request split over the GPUs by Ulysses "
                         "sequence parallelism (default for --config c4)")
    ap.add_argument("--blocks", type=int, default=NUM_BLOCKS, help=argparse.SUPPRESS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-stages", action="store_true", help="skip the prompt-encode and VAE stage timings")
    ap.add_argument("--kernel-only", choices=sorted(KERNELS), default=None,
                    help="profiling aid: only run `iters` launches of one block kernel at the C2 shape")
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--stage", choices=["dit", "vae", "text", "vae-encode", "pe", "exchange"], default="dit",
                    help="dit: the denoise loop (the metric); vae: the VAE decode after it; text: the prompt "
                         "encoder before it (at the config's text bucket); vae-encode: img2img's image encoder "
                         "(1024x1024); pe: the optional prompt enhancer's decode; exchange: NCCL all-to-alls of the "
                         "sequence-parallel exchange volumes (the reference for the fused peer stores)")
    ap.add_argument("--vae-latent", default=None,
                    help="profiling aid: H,W of the unpacked latent of --stage vae (default 128,128: 1024x1024)")
    args = ap.parse_args()
    global WIDTH, HEIGHT, TEXT, VALID
    WIDTH, HEIGHT, TEXT, VALID, config_precision, args.workload = CONFIGS[args.config]
    args.precision = args.precision or config_precision
    if args.kernel_only:
        return run_kernel_only(args)
    if args.warmup < 3:
        args.warmup = 3
    if args.stage == "vae":
        return run_vae_reference(args) if args.impl == "reference" else run_vae(args)
    if args.stage == "text":
        return run_text_reference(args) if args.impl == "reference" else run_text(args)
    if args.stage == "vae-encode":
        return run_vae_encode_reference(args) if args.impl == "reference" else run_vae_encode(args)
    if args.stage == "pe":
        return run_pe_reference(args) if args.impl == "reference" else run_pe(args)
    if args.stage == "exchange":
        return run_exchange(args)
    if args.impl == "reference":
        return run_reference(args)

    import ernie_cuda as ec
    rank, local, world, pg = dist_setup(args.gpus)
    parallel = args.parallel or ("sp" if args.config == "c4" else "dp")
    sp = parallel == "sp" and world > 1
    ctx = ec.Context(local)
    model = ec.Model(ctx, args.blocks)
    model.synthesize(1234)
    precision = ec.BF16 if args.precision == "bf16" else ec.FP32
    tokens = WIDTH * HEIGHT + TEXT
    n_valid = WIDTH * HEIGHT + VALID
    if sp:
        # one request over all ranks; the members' memory handles travel through the process group
        def exchange(handle):
            handles = [None] * world
            pg.all_gather_object(handles, handle)
            return handles
        session = ec.Session(model, WIDTH, HEIGHT, TEXT, VALID, precision, sp=(rank, world, exchange))
        shard, _, img_rows, local_rows, _ = ec.sp_layout(tokens, WIDTH * HEIGHT, world, rank)
        seed = dp.request_seed(1000, 0)
    else:
        session = ec.Session(model, WIDTH, HEIGHT, TEXT, VALID, precision)
        # data parallel: one independent request (seed) per GPU, no collective in the data path
        seed = dp.request_seed(1000, dp.shard_requests(world, rank, world)[0])
        local_rows = tokens
    rng = np.random.default_rng(seed)
    latent = rng.standard_normal((128, HEIGHT, WIDTH), dtype=np.float32)
    text = rng.standard_normal((TEXT, 3072), dtype=np.float32)
    cos, sin, mask = ec.dit_constants(WIDTH, HEIGHT, VALID, TEXT)
    session.set_conditioning(text, cos, sin, mask)
    # one GPU computes the image rows and the text rows up to the last visible key (later text slots are
    # masked keys no image row reads); the FLOPs below are those of the rows computed
    rows_computed = tokens if sp or os.environ.get("ERNIE_ALL_ROWS") == "1" else n_valid
    flops = step_flops(rows_computed, n_valid, args.blocks) / (world if sp else 1)  # per GPU
    launches_per_step = session.launches_per_step()

    # warm-up: graph capture of every step index, then W steps
    lat_ptr = session.latent_ptr()
    if sp:  # this rank's token slice [128][S] of the latent
        device_latent = np.zeros((128, shard), np.float32)
        device_latent[:, :img_rows] = latent.reshape(128, -1)[:, rank * shard: rank * shard + img_rows]
    else:
        device_latent = latent
    ec.check(ec.lib().ernie_cuda_upload(ctx.handle, lat_ptr, ec.ptr(device_latent), device_latent.nbytes))
    for i in range(args.warmup):
        session.denoise_device(STEPS_PER_IMAGE, i % STEPS_PER_IMAGE, i % STEPS_PER_IMAGE + 1)
    for i in range(STEPS_PER_IMAGE):
        session.denoise_device(STEPS_PER_IMAGE, i, i + 1)

    # timed region: K steps, device-timed with CUDA events on the library's stream
    ec.check(ec.lib().ernie_cuda_upload(ctx.handle, lat_ptr, ec.ptr(device_latent), device_latent.nbytes))
    clocks = ClockSampler(local)
    barrier(pg)
    ctx.synchronize()
    clocks.start()
    ctx.record(0)
    for i in range(args.steps):
        session.denoise_device(STEPS_PER_IMAGE, i % STEPS_PER_IMAGE, i % STEPS_PER_IMAGE + 1)
    ctx.record(1)
    ctx.synchronize()
    clock_info = clocks.stop()
    barrier(pg)
    ms = ctx.elapsed(0, 1)
    ms_max = max_over_ranks(pg, ms)
    ms_per_step = ms_max / args.steps
    images_per_s = (1 if sp else world) * 1000.0 / (ms_per_step * STEPS_PER_IMAGE)

    # dominant kernel, timed live: the up/gate GEMM (largest of the 7 per block)
    prof = {}
    for kernel, name in ((1, "qkv_gemm"), (2, "attention"), (3, "out_gemm"), (5, "upgate_gemm"), (6, "down_gemm"),
                         (0, "norm_modulate"), (7, "block")):
        prof[name] = session.profile(kernel, 10 if kernel < 7 else 36)
    # the same parts timed inside consecutive whole blocks (what the step sees: neighbours' L2 state,
    # clocks under the block's mixed load); the per-kernel numbers above are back-to-back repeats
    in_block = {name: session.profile(10 + kernel, 7) for kernel, name in
                ((0, "norm_modulate"), (1, "qkv_gemm"), (2, "attention"), (3, "out_gemm"), (4, "norm_mlp"),
                 (5, "upgate_gemm"), (6, "down_gemm"))}
    if sp:  # the same block with the two barrier kernels instead of the kernels' completion flags
        prof["block_barriers"] = session.profile(17, 36)
    prof["step_eager"] = session.profile(8, 2)  # one step enqueued without a graph
    prof["heads"] = session.profile(9, 10)  # input head, GEMVs, output head + Euler of one step
    bf16_peak, bf16_sustained, hbm_peak, peak_kind = peaks()
    # per-launch algorithmic FLOPs on this GPU: GEMMs over its token rows; attention over every query
    # row for its share of the heads (SP: 32/P heads, the all-to-alls inside the timed launch)
    T = local_rows
    kernel_flops = {"qkv_gemm": 2.0 * T * 4096 * 12288,
                    "attention": 4.0 * tokens * n_valid * 4096 / (world if sp else 1),
                    "out_gemm": 2.0 * T * 4096 * 4096, "upgate_gemm": 2.0 * T * 4096 * 24576,
                    "down_gemm": 2.0 * T * 12288 * 4096}
    dominant = "upgate_gemm"
    achieved = kernel_flops[dominant] / (prof[dominant] * 1e-3) / 1e12
    step_tflops = flops / (ms_per_step * 1e-3) / 1e12

    # end to end through the public API: host latent in, 8-step denoise, host latent out
    # end to end through the public API, per image: the request's conditioning (text rows, RoPE
    # tables, mask: host -> device, text_proj) and the 8-step denoise from a host latent to a host latent
    e2e = None
    if not args.no_e2e:
        session.set_conditioning(text, cos, sin, mask)
        out = session.denoise(latent, STEPS_PER_IMAGE)  # warm (graph for the full range)
        barrier(pg)
        t0 = time.perf_counter()
        reps = max(1, args.steps // STEPS_PER_IMAGE)
        for _ in range(reps):
            session.set_conditioning(text, cos, sin, mask)
            out = session.denoise(latent, STEPS_PER_IMAGE)
        dt = (time.perf_counter() - t0) / reps
        dt = max_over_ranks(pg, dt)
        assert np.isfinite(out).all()
        h2d = latent.nbytes + text.nbytes + cos.nbytes + sin.nbytes + mask.nbytes
        e2e = {"value": (1 if sp else world) / dt, "unit": "images/s", "h2d_bytes_per_step": h2d // STEPS_PER_IMAGE,
               "d2h_bytes_per_step": latent.nbytes // STEPS_PER_IMAGE,
               "call": "ernie_cuda_session_set_conditioning + ernie_cuda_session_denoise (8 steps, host buffers) "
                       "per image; bytes per step = per-image bytes / 8"}

    # the other stages of the same image (not part of the metric): prompt encode before the loop and VAE
    # decode after it, device-timed on this GPU
    stages = None
    if not args.no_stages and not sp:
        stages = pipeline_stages(ctx, args, ms_per_step)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        block_s, cores = cpu_baseline_block()
        image_s = block_s * args.blocks * STEPS_PER_IMAGE
        cpu = {"value": 1.0 / image_s, "unit": "images/s", "cores": cores, "kind": "port",
               "sample": f"one DiT block at {tokens} tokens on the CPU restatement ({block_s:.2f} s), "
                         f"extrapolated x{args.blocks} blocks x{STEPS_PER_IMAGE} steps",
               "reference_published": reference_published_cpu() if args.config == "c2" else None}

    if rank == 0:
        line = {"metric": METRIC, "value": images_per_s, "unit": "images/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
                "scaling": "strong" if sp else "weak", "vs_baseline": None, "dtype": args.precision,
                "data": "synthetic",
                "config": {"workload": f"{args.workload}, {args.blocks} blocks, turbo 8-step schedule, " +
                                       ("one request split over the GPUs" if sp else "one seed per GPU"),
                           "global_batch": 1 if sp else world, "seq_len": tokens,
                           "parallelism": f"sp{world}" if sp else f"dp{world}", "rows_per_gpu": T,
                           "rows_computed": rows_computed,
                           "l2": "inputs larger than L2 (15.7 GB of weights streamed per step)",
                           "step_tflops": step_tflops, "step_frac_of_bf16_peak": step_tflops / bf16_peak,
                           "step_frac_of_datasheet_bf16": step_tflops / DATASHEET_BF16_TFLOPS,
                           "norms": "folded into the GEMMs after block 1 (the residual epilogues write bf16(x g) and "
                                    "row sums of squares, the QKV / up-gate epilogues apply rinv and W shift)"
                                    if args.precision == "bf16" and os.environ.get("ERNIE_FOLD_NORM", "0") == "1"
                                    else "two norm kernels per block",
                           "kernel_ms": prof, "kernel_ms_in_block": in_block, "pipeline_stages": stages},
                "roofline": {"bound": "tensor", "kernel": dominant, "achieved": achieved, "peak": bf16_peak,
                             "unit": "TFLOP/s", "frac": achieved / bf16_peak, "peak_kind": peak_kind,
                             "traffic": UPGATE_TRAFFIC_C2 if args.config == "c2" else None,
                             "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one C2 up/gate "
                                               "launch (profiles/gemm_kernels_c2.md); algorithmic 337 MB"},
                "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches_per_step * args.steps,
                "clocks": clock_info}
        print(json.dumps(line), flush=True)
    session.close()
    model.close()
    ctx.close()
    if pg is not None:
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
