"""bench.py's output contract, checked on the CPU through its reference arm (the CPU restatement timed on the
host cores): one JSON line with the keys and types the benchmark driver reads, at least 3 warm-up steps,
and ranks other than 0 of a multi-process launch (environment variables alone, and a real 2-rank torchrun
launch) exiting 0 without doing the work or printing a line."""
import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ARGS = ["--impl", "reference", "--stage", "vae-encode", "--steps", "1", "--warmup", "1"]
TOP_LEVEL = {"metric": str, "value": float, "unit": str, "n_gpus": int, "steps": int, "warmup": int,
             "ms_per_step": float, "higher_is_better": bool, "scaling": str, "dtype": str, "data": str,
             "config": dict, "impl": str, "cpu_baseline": dict, "e2e": dict}


def run(args, env=None):
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                          timeout=900, cwd=ROOT, env=env)


def json_lines(stdout):
    return [json.loads(line) for line in stdout.splitlines() if line.startswith("{")]


def test_reference_arm_prints_one_complete_line():
    start = time.perf_counter()
    r = run(ARGS)
    wall_s = time.perf_counter() - start
    assert r.returncode == 0, r.stderr[-2000:]
    lines = json_lines(r.stdout)
    assert len(lines) == 1
    d = lines[0]
    for key, kind in TOP_LEVEL.items():
        assert key in d, key
        assert isinstance(d[key], kind) or (kind is float and isinstance(d[key], int)), (key, d[key])
    assert "vs_baseline" in d
    assert d["impl"] == "reference" and d["steps"] == 1 and d["warmup"] == 3  # raised to the minimum of 3
    assert d["value"] > 0 and d["scaling"] in ("weak", "strong")
    cpu = d["cpu_baseline"]
    assert cpu["kind"] in ("port", "reference") and cpu["cores"] >= 1 and cpu["value"] == d["value"]
    assert cpu["unit"] == d["unit"] and isinstance(cpu["sample"], str) and cpu["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert isinstance(d["config"].get("workload"), str)
    # ms_per_step is the measured time of one timed step, so the timed steps fit in the run's own clock
    assert d["steps"] * d["ms_per_step"] / 1000.0 <= wall_s, (d["ms_per_step"], wall_s)


def test_other_ranks_exit_without_work():
    env = dict(os.environ, RANK="1", LOCAL_RANK="1", WORLD_SIZE="2")
    r = run(ARGS, env)
    assert r.returncode == 0, r.stderr[-2000:]
    assert json_lines(r.stdout) == []


def test_reference_arm_under_torchrun_prints_one_line():
    """Launched as the driver launches N > 1 (torchrun, one process per rank): rank 0 alone prints."""
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(port), os.path.join(ROOT, "bench.py"), "--gpus", "2", *ARGS]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = json_lines(r.stdout)
    assert len(lines) == 1 and lines[0]["impl"] == "reference" and lines[0]["n_gpus"] == 2, r.stdout[-2000:]
