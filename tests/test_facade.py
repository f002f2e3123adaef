"""The C++ facade include/qkv.hpp (qwfn::state / engine snapshot methods over the C ABI): a C++
program, tests/facade_check.cpp, is compiled against the headers and libqkv.so and run on a
host-only engine here, and on cuda:0 under -m gpu."""
from __future__ import annotations

import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


@pytest.fixture(scope="module")
def facade_bin(qkvlib, tmp_path_factory):
    out = str(tmp_path_factory.mktemp("facade") / "facade_check")
    libdir = os.path.dirname(qkvlib.LIB_PATH)
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror",
           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(CUDA, "include"),
           os.path.join(ROOT, "tests", "facade_check.cpp"), "-o", out,
           "-L", libdir, "-lqkv", f"-Wl,-rpath,{libdir}",
           "-L", os.path.join(CUDA, "lib64"), "-lcudart", f"-Wl,-rpath,{os.path.join(CUDA, 'lib64')}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return out


def run(binary: str, device: int) -> str:
    r = subprocess.run([binary, str(device)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


def test_facade_host_only(facade_bin):
    assert "facade ok (device -1)" in run(facade_bin, -1)


@pytest.mark.gpu
def test_facade_on_device(facade_bin, cuda):
    assert "facade ok (device 0)" in run(facade_bin, 0)
