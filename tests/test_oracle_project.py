"""The projection oracle (orc_project) on the CPU against a float64 restatement of the reference's
decode projections (graph_builder::qsa_dec_qkv, src/qwfn_graph.cpp:582-608): Q and K rms-normed per
head with their norm weights and roped on the first rope_dim dims (NEOX pairs, text positions), V
plain; query rows taken from attn_q.weight's per-head query/gate interleave."""
from __future__ import annotations

import numpy as np


def bf16_bits(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)     # round to nearest even


def bf16_vals(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def ref_project(x, Wq, Wk, Wv, n_head, n_head_kv, qn, kn, eps, rope_dim, base, pos):
    T = x.shape[0]
    x = x.astype(np.float64)
    half = rope_dim // 2

    def norm_rope(y, w, t):
        y = y / np.sqrt((y * y).mean() + eps) * w
        th = (pos + t) * base ** (-2.0 * np.arange(half) / rope_dim)
        o = y.copy()
        o[:half] = y[:half] * np.cos(th) - y[half:2 * half] * np.sin(th)
        o[half:2 * half] = y[:half] * np.sin(th) + y[half:2 * half] * np.cos(th)
        return o

    wq, wk, wv = bf16_vals(Wq), bf16_vals(Wk), bf16_vals(Wv)
    Q = np.zeros((T, n_head, 256))
    K = np.zeros((T, n_head_kv * 256))
    V = np.zeros_like(K)
    for t in range(T):
        for h in range(n_head):
            Q[t, h] = norm_rope(wq[h * 512:h * 512 + 256] @ x[t], qn, t)
        for h in range(n_head_kv):
            K[t, h * 256:(h + 1) * 256] = norm_rope(wk[h * 256:(h + 1) * 256] @ x[t], kn, t)
            V[t, h * 256:(h + 1) * 256] = wv[h * 256:(h + 1) * 256] @ x[t]
    return Q, K, V


def test_project_oracle_matches_float64(oracle):
    r = np.random.default_rng(31)
    n_embd, n_head, n_head_kv, T, pos = 512, 2, 1, 3, 1000
    x = r.standard_normal((T, n_embd), dtype=np.float32)
    Wq = bf16_bits(r.standard_normal((2 * n_head * 256, n_embd)) / np.sqrt(n_embd))
    Wk = bf16_bits(r.standard_normal((n_head_kv * 256, n_embd)) / np.sqrt(n_embd))
    Wv = bf16_bits(r.standard_normal((n_head_kv * 256, n_embd)) / np.sqrt(n_embd))
    qn = (1 + 0.1 * r.standard_normal(256)).astype(np.float32)
    kn = (1 + 0.1 * r.standard_normal(256)).astype(np.float32)
    Q, K, V = oracle.project(x, Wq, Wk, Wv, n_head, n_head_kv, qn, kn, 1e-6, 64, 1e7, pos)
    Qr, Kr, Vr = ref_project(x, Wq, Wk, Wv, n_head, n_head_kv, qn, kn, 1e-6, 64, 1e7, pos)
    np.testing.assert_allclose(Q, Qr, rtol=1e-4, atol=2e-4)
    np.testing.assert_allclose(K, Kr, rtol=1e-4, atol=2e-4)
    np.testing.assert_allclose(V, Vr, rtol=1e-4, atol=2e-4)
    # the gate rows (odd 256-row groups of Wq) play no part
    Wq2 = Wq.copy()
    Wq2[256:512] = 0
    Q2, _, _ = oracle.project(x, Wq2, Wk, Wv, n_head, n_head_kv, qn, kn, 1e-6, 64, 1e7, pos)
    np.testing.assert_array_equal(Q2, Q)
