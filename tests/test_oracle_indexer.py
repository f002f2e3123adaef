"""The indexer oracle (orc_idx_*) on the CPU: its fixed-order fp32 arithmetic restated
independently in numpy float32 (bit-exact), its meaning checked against float64 (rms-norm, rope,
relu-sum), and the selection rule of the reference's decode path (src/qwfn_engine.cpp:1072-1105,
src/qwfn_graph.cpp:556-579): forced incomplete tail block, best whole blocks with ties to the
lower index, everything when there are no more than k_blocks blocks."""
from __future__ import annotations

import numpy as np
import pytest

f32 = np.float32


def bfly(part: np.ndarray) -> np.float32:
    v = part.astype(f32).copy()
    for o in (16, 8, 4, 2, 1):
        v = (v + v[np.arange(32) ^ o]).astype(f32)
    return v[0]


def np_pool(keys16: np.ndarray, n_blocks: int, w: np.ndarray, eps: float, rope_dim: int, cs: np.ndarray):
    k = keys16[:4 * n_blocks].view(np.float16).astype(f32).reshape(n_blocks, 4, 128)
    out = np.empty((n_blocks, 128), dtype=np.uint16)
    h = rope_dim // 2
    for b in range(n_blocks):
        x = k[b, 0].copy()
        for m in range(1, 4):
            x = (x + k[b, m]).astype(f32)
        x = (x * f32(0.25)).astype(f32)
        sq = (x * x).astype(f32).reshape(32, 4)
        part = sq[:, 0].copy()
        for j in range(1, 4):
            part = (part + sq[:, j]).astype(f32)
        s = bfly(part)
        scale = f32(1.0) / np.sqrt(f32(s * f32(1 / 128)) + f32(eps), dtype=f32)
        y = ((x * f32(scale)).astype(f32) * w).astype(f32)
        o = y.copy()
        if h:
            c, sn = cs[b, :h, 0], cs[b, :h, 1]
            o[:h] = ((y[:h] * c).astype(f32) - (y[h:2 * h] * sn).astype(f32)).astype(f32)
            o[h:2 * h] = ((y[:h] * sn).astype(f32) + (y[h:2 * h] * c).astype(f32)).astype(f32)
        out[b] = o.astype(np.float16).view(np.uint16)
    return out


def np_score(q: np.ndarray, pooled_b: np.ndarray) -> np.float32:
    qh = q.astype(np.float16).astype(f32)
    k = pooled_b.view(np.float16).astype(f32)
    tot = 0.0
    for h in range(q.shape[0]):
        p = (qh[h] * k).astype(f32)
        part = []
        for j in range(4):
            a = f32(0.0)
            for e in range(32 * j, 32 * j + 32):
                a = f32(a + p[e])
            part.append(a)
        d = f32(f32(part[0] + part[1]) + f32(part[2] + part[3]))
        tot = tot + float(max(d, f32(0.0)))
    return f32(tot)


@pytest.fixture(scope="module")
def keys():
    r = np.random.default_rng(90)
    raw = (r.standard_normal((64 * 4, 128)) * 3).astype(np.float32)
    return raw.astype(np.float16).view(np.uint16)


@pytest.mark.parametrize("rope_dim", [64, 0, 128])
def test_pool_bit_exact_vs_numpy(oracle, keys, rope_dim):
    r = np.random.default_rng(91)
    w = (1 + 0.1 * r.standard_normal(128)).astype(np.float32)
    got = oracle.idx_pool(keys, 64, w, 1e-6, rope_dim, 1e7)
    cs = oracle.idx_rope_table(64, rope_dim, 1e7)
    want = np_pool(keys, 64, w, 1e-6, rope_dim, cs)
    np.testing.assert_array_equal(got, want)


def test_pool_meaning_in_float64(oracle, keys):
    """mean -> rms-norm -> weight -> NEOX-paired rotation by theta_i = 4b * base^(-2i/64)."""
    r = np.random.default_rng(92)
    w = (1 + 0.1 * r.standard_normal(128)).astype(np.float32)
    got = oracle.idx_pool(keys, 64, w, 1e-6, 64, 1e7).view(np.float16).astype(np.float64)
    k = keys.view(np.float16).astype(np.float64).reshape(64, 4, 128)
    x = k.mean(axis=1)
    y = x / np.sqrt((x * x).mean(axis=1, keepdims=True) + 1e-6) * w
    p = 4 * np.arange(64)[:, None]
    th = p * (1e7 ** (-2 * np.arange(32) / 64))[None, :]
    want = y.copy()
    want[:, :32] = y[:, :32] * np.cos(th) - y[:, 32:64] * np.sin(th)
    want[:, 32:64] = y[:, :32] * np.sin(th) + y[:, 32:64] * np.cos(th)
    # fp16 storage + the fp32 angle recurrence (large p * tiny frequencies lose a few ulps)
    np.testing.assert_allclose(got, want, rtol=2e-3, atol=5e-3)


def test_rope_table_matches_ggml_recurrence(oracle):
    cs = oracle.idx_rope_table(300, 64, 1e7)
    ts = np.float32(np.power(np.float32(1e7), np.float32(-2.0 / 64)))
    th = np.float32(4 * 299)
    for i in range(32):
        assert cs[299, i, 0] == np.float32(np.cos(np.float64(th))) or abs(cs[299, i, 0] - np.cos(th)) < 1e-6
        th = np.float32(th * ts)


def test_score_bit_exact_and_meaning(oracle, keys):
    r = np.random.default_rng(93)
    pooled = oracle.idx_pool(keys, 64, np.ones(128, np.float32), 1e-6, 64, 1e7)
    q = r.standard_normal((4, 128)).astype(np.float32)
    _, scores = oracle.idx_select(q, pooled, 64 * 4 - 1, 10)
    for b in range(64):
        assert scores[b] == np_score(q, pooled[b])
    ref = np.maximum(q.astype(np.float16).astype(np.float64) @ pooled.view(np.float16).astype(np.float64).T, 0).sum(0)
    np.testing.assert_allclose(scores, ref, rtol=1e-5, atol=1e-5)


def test_select_rules(oracle, keys):
    pooled = oracle.idx_pool(keys, 64, np.ones(128, np.float32), 1e-6, 64, 1e7)
    r = np.random.default_rng(94)
    q = r.standard_normal((4, 128)).astype(np.float32)
    # few blocks: everything up to the block holding pos
    kept, _ = oracle.idx_select(q, pooled, 37, 10)
    np.testing.assert_array_equal(kept, np.arange(10))
    kept, _ = oracle.idx_select(q, pooled, 41, 10)          # blocks 0..10 = 11 > 10: select
    assert len(kept) == 10 and kept[-1] == 10               # 41 = 4*10+1: tail block 10 incomplete, forced
    kept, scores = oracle.idx_select(q, pooled, 43, 10)     # 43 = 4*10+3: block 10 whole, nothing forced
    assert len(kept) == 10
    order = sorted(range(11), key=lambda b: (-scores[b], b))[:10]
    np.testing.assert_array_equal(kept, np.sort(order))
    kept, scores = oracle.idx_select(q, pooled, 255, 16)    # 64 whole blocks, keep 16
    order = sorted(range(64), key=lambda b: (-scores[b], b))[:16]
    np.testing.assert_array_equal(kept, np.sort(order))


def test_select_ties_to_lower_index(oracle):
    # identical pooled keys: every whole block scores the same, the lowest indices win
    one = np.full((40, 128), np.float16(0.5)).view(np.uint16)
    q = np.ones((4, 128), np.float32)
    kept, scores = oracle.idx_select(q, one, 4 * 39 + 1, 8)  # tail block 39 incomplete
    assert np.all(scores == scores[0])
    np.testing.assert_array_equal(kept, [0, 1, 2, 3, 4, 5, 6, 39])
    q = -q                                                   # all relu'd to zero: still ties
    kept, scores = oracle.idx_select(q, one, 4 * 39 + 3, 8)
    assert np.all(scores == 0)
    np.testing.assert_array_equal(kept, np.arange(8))
