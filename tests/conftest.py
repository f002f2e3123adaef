"""Shared fixtures.  `-m gpu` tests need a CUDA device and the sm_100a build of libqkv.so;
everything else runs on the CPU (oracle, host logic, ABI surface, gloo multi-rank paths)."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built libqkv.so")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def qkvlib():
    import qwfn_hybrid_b200 as Q
    if not os.path.exists(Q.LIB_PATH):
        from qwfn_hybrid_b200 import build
        build.build()
    Q.lib()
    return Q


@pytest.fixture(scope="session")
def cuda(qkvlib):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("a -m gpu test ran without a CUDA device")
    torch.cuda.init()
    return torch.device("cuda:0")


def rng(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)
