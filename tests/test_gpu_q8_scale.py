"""GPU: the q8_0 block-scale arithmetic of the quantisers (kernels A, C, D and the projection
epilogue) -- d = amax / 127 and id = 1 / d as an FMA correction step and one Newton-Raphson step --
equals the device's IEEE division and reciprocal for every non-negative float, so the quantised
bytes are those of ggml's quantize_row_q8_0 (src/qwfn_graph.cpp's q8_0 caches) bit for bit."""
from __future__ import annotations

import ctypes

import pytest

pytestmark = pytest.mark.gpu


def test_scale_equals_ieee_division_and_reciprocal_everywhere(cuda, qkvlib):
    div, rcp = ctypes.c_uint64(7), ctypes.c_uint64(7)
    assert qkvlib.lib().qkv_debug_check_q8_scale(ctypes.byref(div), ctypes.byref(rcp)) == 0
    assert (div.value, rcp.value) == (0, 0)
