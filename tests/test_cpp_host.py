"""Build and run the C++ host-surface tests (tests/cpp/) against libernie_b200.so."""
import os
import subprocess

import pytest

import ernie_cuda as ec

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.dirname(ec.LIB_PATH)


def build(name, tmp_path):
    exe = str(tmp_path / name)
    cmd = ["g++", "-std=c++17", "-O1", "-I" + os.path.join(ROOT, "include"), os.path.join(ROOT, "tests", "cpp", name + ".cpp"),
           "-L" + LIBDIR, "-lernie_b200", "-Wl,-rpath," + LIBDIR, "-o", exe]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_host_contracts(tmp_path):
    exe = build("test_host_logic", tmp_path)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr + r.stdout
    assert "host contracts passed" in r.stdout


@pytest.mark.gpu
def test_host_surface_on_gpu(tmp_path):
    exe = build("test_host_gpu", tmp_path)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr + r.stdout
    assert "host GPU contracts passed" in r.stdout
