"""Build recipe of libernie_b200.so: every CUDA source compiled for sm_100a with nvcc, linked into
one in-tree shared library (so the built file travels with the source tree to the GPU box).

    python ernie-image-ncnn-vulkan_b200/build.py [--force]

ERNIE_NVCC_FLAGS adds nvcc options, e.g. the kernels' compile-time launch-shape knobs for an A/B build:
    ERNIE_NVCC_FLAGS="-DERNIE_FLASH_SHORT_LAST=0" python ernie-image-ncnn-vulkan_b200/build.py --force
"""
import concurrent.futures
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
HOST = os.path.join(HERE, "host")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libernie_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
INCLUDES = ["-I" + os.path.join(ROOT, "include"), "-I" + CSRC]
NVCC_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
                     "-Xcompiler", "-fPIC,-ffp-contract=off"] + INCLUDES + os.environ.get("ERNIE_NVCC_FLAGS", "").split()
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-ffp-contract=off"] + INCLUDES + ["-I/usr/local/cuda/include"]


def sources():
    cu = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))
    cpp = sorted(os.path.join(HOST, f) for f in os.listdir(HOST) if f.endswith(".cpp")) if os.path.isdir(HOST) else []
    return cu, cpp


def headers():
    out = []
    for d in (CSRC, HOST, os.path.join(ROOT, "include"), os.path.join(ROOT, "include", "ernie_b200")):
        if os.path.isdir(d):
            out += [os.path.join(d, f) for f in os.listdir(d) if f.endswith((".h", ".cuh", ".hpp"))]
    return out


def _stale(src, obj, deps):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return os.path.getmtime(src) > t or any(os.path.getmtime(h) > t for h in deps)


def _compile(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("compile failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r.stderr


def build(force=False, verbose=False):
    os.makedirs(OBJ, exist_ok=True)
    cu, cpp = sources()
    deps = headers()
    jobs, objs = [], []
    for src in cu:
        obj = os.path.join(OBJ, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or _stale(src, obj, deps):
            jobs.append([NVCC] + NVCC_FLAGS + ["-c", src, "-o", obj])
    for src in cpp:
        obj = os.path.join(OBJ, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or _stale(src, obj, deps):
            jobs.append(["g++"] + CXX_FLAGS + ["-c", src, "-o", obj])
    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as pool:
        for log in pool.map(_compile, jobs):
            if verbose and log:
                print(log)
    if jobs or not os.path.exists(LIB):
        link = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart_static", "-lrt", "-ldl", "-lpthread"]
        _compile(link)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
