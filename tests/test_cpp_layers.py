"""The C++ layer mirror (seedvr2-ncnn-valkan_b200/host/s2_layers.hpp) through its
runner, tests/cpp/layer_runner.cpp: the reference runners' block and VAE cases
built with load_param / load_model / forward on the B200, against the
reference's own CPU layer code (oracle/_ref), plus the reference's -1 return
codes for bad parameters and blobs.

CPU: the header and runner compile (g++, C++17, -Wall -Werror).
GPU: the runner links against the library and passes every case.
"""
from __future__ import annotations

import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "seedvr2-ncnn-valkan_b200", "lib")
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libs2ref.so")
SRC = os.path.join(ROOT, "tests", "cpp", "layer_runner.cpp")
FLAGS = ["-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror", "-I" + os.path.join(ROOT, "include"),
         "-I" + os.path.join(ROOT, "seedvr2-ncnn-valkan_b200", "host")]


def gxx():
    exe = shutil.which("g++")
    if exe is None:
        pytest.skip("g++ not available")
    return exe


def test_header_and_runner_compile():
    r = subprocess.run([gxx(), *FLAGS, "-fsyntax-only", SRC], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr


@pytest.mark.gpu
def test_layer_runner_on_gpu(tmp_path):
    assert os.path.exists(os.path.join(LIBDIR, "libs2b200.so")), "build the library first"
    assert os.path.exists(REF_SO), "the reference build (oracle/_ref) is missing"
    exe = str(tmp_path / "layer_runner")
    r = subprocess.run([gxx(), *FLAGS, SRC, "-L" + LIBDIR, "-ls2b200", "-Wl,-rpath," + LIBDIR, "-ldl", "-o", exe],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([exe, REF_SO], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("[")]
    assert len(lines) == 11 and all(ln.endswith("PASS") for ln in lines), r.stdout
