"""Generates tests/golden/q8_0_gguf.npz: q8_0 golden vectors produced by gguf-py 0.19.0.

gguf-py (the llama.cpp project's Python package) states that its Q8_0.quantize_blocks is
bit-exact with ggml's reference quantize_row_q8_0 (gguf/quants.py:378-393).  It is the only
piece of the reference's arithmetic that can be executed in this container (ggml itself is
not present), so it pins the oracle's and the GPU append kernel's block bytes.

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import os

import numpy as np
from gguf.constants import GGMLQuantizationType
from gguf.quants import quantize


def edge_blocks() -> np.ndarray:
    """Hand-made 32-element blocks that stress the rounding rules."""
    rows = []
    rows.append(np.zeros(32, np.float32))                                  # d == 0
    one = np.zeros(32, np.float32); one[7] = 3.25; rows.append(one)        # a single max
    neg = np.zeros(32, np.float32); neg[31] = -1e-3; rows.append(neg)      # a single negative max
    # d == 1 exactly: x*id == x, so every k+0.5 is a rounding tie (away from zero vs even)
    ties = np.array([127.0] + [k + 0.5 for k in range(-15, 16)], np.float32)
    rows.append(ties)
    # d == 0.5: ties at k/2 + 0.25
    ties2 = np.array([63.5] + [k / 2 + 0.25 for k in range(-15, 16)], np.float32)
    rows.append(ties2)
    # d = 1 + 2^-11 is halfway between two fp16 values: fp16(d) must round to even (1.0)
    half = np.full(32, 0.25, np.float32); half[0] = np.float32(127.0 * (1 + 2.0 ** -11)); rows.append(half)
    # mixed magnitudes in one block, large and tiny scales
    rows.append(np.linspace(-1000, 1000, 32, dtype=np.float32))
    rows.append(np.linspace(-1e-6, 3e-6, 32, dtype=np.float32))
    rows.append(np.array([(-1) ** k * (k + 1) * 1.7 for k in range(32)], np.float32))
    return np.stack(rows)


def main() -> None:
    rng = np.random.default_rng(0)
    rand_rows = rng.standard_normal((48, 512), dtype=np.float32)
    scaled = (rng.standard_normal((16, 512), dtype=np.float32) * np.float32(37.0))
    edges = edge_blocks()
    edge_rows = np.concatenate([edges.reshape(-1), np.zeros((-edges.size) % 512, np.float32)]).reshape(-1, 512)
    x = np.concatenate([rand_rows, scaled, edge_rows], axis=0).astype(np.float32)
    q = quantize(x, GGMLQuantizationType.Q8_0)
    assert q.dtype == np.uint8 and q.shape == (x.shape[0], 512 // 32 * 34)
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "q8_0_gguf.npz")
    np.savez_compressed(out, x=x, q8_0=q, gguf_version=np.array("0.19.0"))
    print(f"wrote {out}: {x.shape[0]} rows of 512 -> {q.shape}")


if __name__ == "__main__":
    main()
