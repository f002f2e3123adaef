"""The ggml-node adapter include/qkv_ggml.hpp: a C++ program, tests/ggml_shim_check.cpp, builds the
operands the reference's graph builds for its attention nodes (src/qwfn_graph.cpp:454-471,
653-705) and routes them through the adapter.  Host-only here: every malformed view is refused.
Under -m gpu: a prefill and a fused decode step through the adapter against the C oracle."""
from __future__ import annotations

import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


@pytest.fixture(scope="module")
def shim_bin(qkvlib, oracle, tmp_path_factory):
    out = str(tmp_path_factory.mktemp("shim") / "ggml_shim_check")
    libdir = os.path.dirname(qkvlib.LIB_PATH)
    odir = os.path.join(ROOT, "oracle", "_build")
    cmd = ["g++", "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror",
           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(CUDA, "include"),
           os.path.join(ROOT, "tests", "ggml_shim_check.cpp"), "-o", out,
           "-L", libdir, "-lqkv", f"-Wl,-rpath,{libdir}", "-L", odir, "-loracle", f"-Wl,-rpath,{odir}",
           "-L", os.path.join(CUDA, "lib64"), "-lcudart", f"-Wl,-rpath,{os.path.join(CUDA, 'lib64')}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return out


def run(binary: str, device: int) -> str:
    r = subprocess.run([binary, str(device)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


def test_adapter_rejects_malformed_views(shim_bin):
    assert "ggml shim ok (device -1)" in run(shim_bin, -1)


@pytest.mark.gpu
def test_adapter_prefill_and_decode_on_device(shim_bin, cuda):
    out = run(shim_bin, 0)
    assert "ggml shim ok (device 0)" in out, out
