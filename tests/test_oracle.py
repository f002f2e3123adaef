"""The CPU oracle against the reference's golden vectors and against independent restatements."""
from __future__ import annotations

import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "q8_0_gguf.npz")


def test_q8_0_matches_gguf_golden(oracle):
    d = np.load(GOLDEN)
    got = oracle.quantize_rows(d["x"])
    assert np.array_equal(got, d["q8_0"]), f"{int((got != d['q8_0']).sum())} bytes differ from gguf-py"


def test_q8_0_matches_gguf_live(oracle):
    gq = pytest.importorskip("gguf.quants")
    from gguf.constants import GGMLQuantizationType
    r = np.random.default_rng(11)
    x = np.concatenate([r.standard_normal((200, 512), dtype=np.float32),
                        (r.standard_normal((50, 512), dtype=np.float32) * 1e-3),
                        np.round(r.standard_normal((50, 512)) * 8).astype(np.float32) / 2])
    assert np.array_equal(oracle.quantize_rows(x), gq.quantize(x, GGMLQuantizationType.Q8_0))


def test_q8_0_ties_round_half_away(oracle):
    x = np.zeros((1, 32), np.float32)
    x[0, 0] = 127.0               # d == 1 exactly, so x*id == x
    x[0, 1:5] = [0.5, 1.5, -0.5, -2.5]
    q = oracle.quantize_rows(x)[0]
    assert list(q[2:7].view(np.int8)) == [127, 1, 2, -1, -3]
    assert int(q[0]) | (int(q[1]) << 8) == 0x3C00   # fp16(1.0)


def test_dequantize_roundtrip(oracle):
    d = np.load(GOLDEN)
    gq = pytest.importorskip("gguf.quants")
    from gguf.constants import GGMLQuantizationType
    assert np.array_equal(oracle.dequantize_rows(d["q8_0"]), gq.dequantize(d["q8_0"], GGMLQuantizationType.Q8_0))


def test_fp16_conversion_matches_numpy(oracle):
    r = np.random.default_rng(3)
    vals = np.concatenate([r.standard_normal(2000).astype(np.float32) * 10.0 ** r.integers(-9, 6, 2000),
                           np.array([0.0, -0.0, 65504.0, 65519.0, 65520.0, 1e-8, 5.96e-8, 2.98e-8, 2.99e-8,
                                     6.1035e-5, 1 + 2 ** -11, 1 + 3 * 2 ** -11, np.inf, -np.inf], np.float32)])
    for v in vals:
        h = oracle.fp32_to_fp16_bits(float(v))
        assert h == int(np.float32(v).astype(np.float16).view(np.uint16)), v
        assert oracle.fp16_bits_to_fp32(h) == float(np.uint16(h).view(np.float16))


def _attn_f64(oracle, Q, K, V, q_pos, n_head_kv, scale):
    """Independent float64 restatement: quantised Q, dequantised K/V, exact softmax."""
    T, H, hd = Q.shape
    G = H // n_head_kv
    Kd = oracle.dequantize_rows(K).reshape(K.shape[0], n_head_kv, hd).astype(np.float64)
    Vd = oracle.dequantize_rows(V).reshape(V.shape[0], n_head_kv, hd).astype(np.float64)
    Qd = oracle.dequantize_rows(oracle.quantize_rows(Q)).astype(np.float64)
    out = np.zeros((T, H, hd))
    for t in range(T):
        n = q_pos[t] + 1
        for h in range(H):
            s = Kd[:n, h // G] @ Qd[t, h] * scale
            p = np.exp(s - s.max())
            out[t, h] = (p @ Vd[:n, h // G]) / p.sum()
    return out


@pytest.mark.parametrize("n_kv,T", [(1, 1), (5, 2), (97, 3), (1000, 4)])
def test_attention_oracle_vs_float64(oracle, n_kv, T):
    r = np.random.default_rng(n_kv)
    H, Hkv, hd = 16, 2, 256
    Kf = r.standard_normal((n_kv, Hkv * hd), dtype=np.float32)
    Vf = r.standard_normal((n_kv, Hkv * hd), dtype=np.float32)
    K, V = oracle.quantize_rows(Kf), oracle.quantize_rows(Vf)
    Q = r.standard_normal((T, H, hd), dtype=np.float32)
    q_pos = np.arange(n_kv - T, n_kv, dtype=np.int32)
    got = oracle.attn(Q, K, V, q_pos, Hkv, 1 / 16)
    ref = _attn_f64(oracle, Q, K, V, q_pos, Hkv, 1 / 16)
    np.testing.assert_allclose(got, ref, atol=2e-5, rtol=1e-4)


def test_attention_oracle_cell_list_and_mask(oracle):
    r = np.random.default_rng(5)
    Kf = r.standard_normal((300, 512), dtype=np.float32)
    K, V = oracle.quantize_rows(Kf), oracle.quantize_rows(r.standard_normal((300, 512), dtype=np.float32))
    Q = r.standard_normal((2, 16, 256), dtype=np.float32)
    cells = np.array([3, 7, 100, 250, 299], np.int32)
    a = oracle.attn(Q, K, V, [298, 299], 2, 0.0625, cells=cells)
    # same cells gathered into a dense cache: rows visible by position, 299 hidden from token 0
    a2 = oracle.attn(Q, K[cells], V[cells], [3, 4], 2, 0.0625)
    np.testing.assert_array_equal(a, a2)
    # a query with no visible cell returns zeros (S == 0)
    z = oracle.attn(Q[:1], K, V, [-1], 2, 0.0625)
    assert not z.any()


def test_selection_oracle_properties(oracle):
    r = np.random.default_rng(9)
    nb, top = 40, 8
    K = oracle.quantize_rows(r.standard_normal((nb * 64, 512), dtype=np.float32))
    summ = oracle.block_summary(K, 2, 256, 64, nb)
    Q = r.standard_normal((3, 16, 256), dtype=np.float32)
    idx, scores = oracle.select_blocks(Q, 2, summ, nb, top)
    for h in range(2):
        sel = list(idx[h])
        assert sel[:3] == [0, nb - 2, nb - 1]               # forced blocks, by index
        rest = [b for b in range(nb) if b not in (0, nb - 2, nb - 1)]
        order = sorted(rest, key=lambda b: (-scores[h, b], b))
        assert sel[3:] == order[:top - 3]
    # block summary = fp16 mean of the dequantised keys
    deq = oracle.dequantize_rows(K).reshape(nb, 64, 2, 256).mean(axis=1)
    np.testing.assert_allclose(summ.view(np.float16).astype(np.float32), deq.transpose(1, 0, 2), rtol=2e-3, atol=1e-3)


def test_selection_small_context_keeps_all(oracle):
    Q = np.ones((1, 16, 256), np.float32)
    summ = np.zeros((2, 5, 256), np.uint16)
    idx, _ = oracle.select_blocks(Q, 2, summ, 5, 8)
    assert list(idx[0]) == [0, 1, 2, 3, 4, -1, -1, -1]
