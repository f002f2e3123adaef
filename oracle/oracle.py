"""ctypes front of the CPU oracle (oracle/qkv_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU
baseline arm as the checker.  The product (qwfn_hybrid_b200, libqkv.so) never imports it.

Layouts are ggml's: a q8_0 row of n elements is n/32 blocks of {fp16 d, int8 qs[32]} (34 bytes);
a KV cache row holds n_head_kv heads back to back (src/qwfn_graph.cpp:458-464 views).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

QK = 32
BLOCK_BYTES = 34


def build() -> str:
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        i64, i32, f32 = ctypes.c_int64, ctypes.c_int, ctypes.c_float
        L.orc_fp32_to_fp16.argtypes = [f32]
        L.orc_fp32_to_fp16.restype = ctypes.c_uint16
        L.orc_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        L.orc_fp16_to_fp32.restype = f32
        L.orc_quantize_rows_q8_0.argtypes = [P, P, i64, i64, i32]
        L.orc_dequantize_row_q8_0.argtypes = [P, P, i64]
        L.orc_attn_q8_0.argtypes = [P, i64, i32, i32, i32, P, P, P, i64, P, f32, P, i32]
        L.orc_attn_q8_0_sparse.argtypes = [P, i64, i32, i32, i32, P, P, P, P, P, f32, P, i32]
        L.orc_block_summary.argtypes = [P, i32, i32, i32, i64, P, i32]
        L.orc_select_blocks.argtypes = [P, i64, i32, i32, i32, P, i64, i32, P, P]
        L.orc_blocks_to_cells.argtypes = [P, i32, i32, i64, P]
        L.orc_blocks_to_cells.restype = i64
        L.orc_max_threads.restype = i32
        L.orc_idx_rope_table.argtypes = [i64, i32, f32, P]
        L.orc_idx_pool.argtypes = [P, i64, P, f32, i32, P, P]
        L.orc_idx_score.argtypes = [P, i32, P]
        L.orc_idx_score.restype = f32
        L.orc_idx_select.argtypes = [P, i32, P, i64, i32, P, P]
        L.orc_idx_select.restype = i64
        L.orc_project.argtypes = [P, i32, i32, P, P, P, i32, i32, P, P, f32, i32, f32, i32, P, P, P]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def max_threads() -> int:
    return int(lib().orc_max_threads())


def fp32_to_fp16_bits(x: float) -> int:
    return int(lib().orc_fp32_to_fp16(ctypes.c_float(x)))


def fp16_bits_to_fp32(h: int) -> float:
    return float(lib().orc_fp16_to_fp32(h))


def quantize_rows(x: np.ndarray, threads: int = 0) -> np.ndarray:
    """float32 [..., k] -> uint8 [..., k/32*34] (ggml q8_0 rows)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    k = x.shape[-1]
    assert k % QK == 0
    rows = x.reshape(-1, k)
    out = np.empty((rows.shape[0], k // QK * BLOCK_BYTES), dtype=np.uint8)
    lib().orc_quantize_rows_q8_0(_p(rows), _p(out), rows.shape[0], k, threads or max_threads())
    return out.reshape(x.shape[:-1] + (k // QK * BLOCK_BYTES,))


def dequantize_rows(y: np.ndarray) -> np.ndarray:
    y = np.ascontiguousarray(y, dtype=np.uint8)
    nbytes = y.shape[-1]
    assert nbytes % BLOCK_BYTES == 0
    k = nbytes // BLOCK_BYTES * QK
    rows = y.reshape(-1, nbytes)
    out = np.empty((rows.shape[0], k), dtype=np.float32)
    for r in range(rows.shape[0]):
        lib().orc_dequantize_row_q8_0(_p(rows[r]), _p(out[r]), k)
    return out.reshape(y.shape[:-1] + (k,))


def attn(Q: np.ndarray, K: np.ndarray, V: np.ndarray, q_pos, n_head_kv: int, scale: float,
         cells: np.ndarray | None = None, n_cells: int | None = None, threads: int = 0) -> np.ndarray:
    """Q float32 [T, n_head, hd]; K/V uint8 [n_kv, n_head_kv*hd/32*34]; returns [T, n_head, hd]."""
    Q = np.ascontiguousarray(Q, dtype=np.float32)
    T, n_head, hd = Q.shape
    K = np.ascontiguousarray(K, dtype=np.uint8)
    V = np.ascontiguousarray(V, dtype=np.uint8)
    qp = np.ascontiguousarray(np.asarray(q_pos, dtype=np.int32).reshape(T))
    out = np.empty_like(Q)
    if cells is not None:
        cells = np.ascontiguousarray(cells, dtype=np.int32)
        n = cells.shape[0]
        cp = _p(cells)
    else:
        n = K.shape[0] if n_cells is None else n_cells
        cp = None
    lib().orc_attn_q8_0(_p(Q), T, n_head, n_head_kv, hd, _p(K), _p(V), cp, n, _p(qp),
                        ctypes.c_float(scale), _p(out), threads or max_threads())
    return out


def attn_sparse(Q: np.ndarray, K: np.ndarray, V: np.ndarray, q_pos, n_head_kv: int, scale: float,
                cells_per_head: list, threads: int = 0) -> np.ndarray:
    Q = np.ascontiguousarray(Q, dtype=np.float32)
    T, n_head, hd = Q.shape
    qp = np.ascontiguousarray(np.asarray(q_pos, dtype=np.int32).reshape(T))
    arrs = [np.ascontiguousarray(c, dtype=np.int32) for c in cells_per_head]
    ptrs = (ctypes.c_void_p * n_head_kv)(*[a.ctypes.data for a in arrs])
    ns = np.array([a.shape[0] for a in arrs], dtype=np.int64)
    out = np.empty_like(Q)
    lib().orc_attn_q8_0_sparse(_p(Q), T, n_head, n_head_kv, hd, _p(np.ascontiguousarray(K)),
                               _p(np.ascontiguousarray(V)), ctypes.cast(ptrs, ctypes.c_void_p), _p(ns),
                               _p(qp), ctypes.c_float(scale), _p(out), threads or max_threads())
    return out


def block_summary(K: np.ndarray, n_head_kv: int, head_dim: int, block_tokens: int, n_blocks: int,
                  threads: int = 0) -> np.ndarray:
    """fp16 bits uint16 [n_head_kv, n_blocks, head_dim]."""
    K = np.ascontiguousarray(K, dtype=np.uint8)
    out = np.empty((n_head_kv, n_blocks, head_dim), dtype=np.uint16)
    lib().orc_block_summary(_p(K), n_head_kv, head_dim, block_tokens, n_blocks, _p(out), threads or max_threads())
    return out


def select_blocks(Q: np.ndarray, n_head_kv: int, summary: np.ndarray, n_blocks: int, top_k: int):
    """Returns (idx int32 [n_head_kv, top_k], scores float32 [n_head_kv, n_blocks])."""
    Q = np.ascontiguousarray(Q, dtype=np.float32)
    T, n_head, hd = Q.shape
    summary = np.ascontiguousarray(summary, dtype=np.uint16)
    idx = np.empty((n_head_kv, top_k), dtype=np.int32)
    scores = np.empty((n_head_kv, n_blocks), dtype=np.float32)
    lib().orc_select_blocks(_p(Q), T, n_head, n_head_kv, hd, _p(summary), n_blocks, top_k, _p(idx), _p(scores))
    return idx, scores


def blocks_to_cells(blocks: np.ndarray, block_tokens: int, n_kv: int) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.int32)
    out = np.empty(blocks.shape[0] * block_tokens, dtype=np.int32)
    n = lib().orc_blocks_to_cells(_p(blocks), blocks.shape[0], block_tokens, n_kv, _p(out))
    return out[:n]


# ---- QSA lightning indexer (decode path) ------------------------------------------------------
IDX_KEY, IDX_R = 128, 4


def idx_rope_table(n_blocks: int, rope_dim: int, freq_base: float) -> np.ndarray:
    """float32 [n_blocks, rope_dim/2, 2] {cos, sin} at block positions 4b."""
    out = np.zeros((n_blocks, max(rope_dim // 2, 1), 2), dtype=np.float32)
    lib().orc_idx_rope_table(n_blocks, rope_dim, ctypes.c_float(freq_base), _p(out))
    return out


def idx_pool(keys16: np.ndarray, n_blocks: int, norm_w: np.ndarray, eps: float, rope_dim: int,
             freq_base: float) -> np.ndarray:
    """Raw fp16 key bits uint16 [>= 4*n_blocks, 128] -> pooled fp16 bits uint16 [n_blocks, 128]."""
    keys16 = np.ascontiguousarray(keys16[:IDX_R * n_blocks], dtype=np.uint16)
    cs = idx_rope_table(n_blocks, rope_dim, freq_base)
    w = np.ascontiguousarray(norm_w, dtype=np.float32)
    out = np.empty((n_blocks, IDX_KEY), dtype=np.uint16)
    lib().orc_idx_pool(_p(keys16), n_blocks, _p(w), ctypes.c_float(eps), rope_dim, _p(cs), _p(out))
    return out


def idx_select(q: np.ndarray, pooled: np.ndarray, pos: int, k_blocks: int):
    """q float32 [n_head, 128]; pooled uint16 [>= (pos+1)//4, 128].  Returns (kept block ids
    ascending, scores of the whole blocks)."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    pooled = np.ascontiguousarray(pooled, dtype=np.uint16)
    whole = (pos + 1) // IDX_R
    scores = np.zeros(max(whole, 1), dtype=np.float32)
    blocks = np.empty(k_blocks, dtype=np.int32)
    n = lib().orc_idx_select(_p(q), q.shape[0], _p(pooled), pos, k_blocks, _p(scores), _p(blocks))
    return blocks[:n].copy(), scores[:whole]


# ---- fused projections (decode) ------------------------------------------------------------------
def project(x: np.ndarray, Wq, Wk: np.ndarray, Wv: np.ndarray, n_head: int, n_head_kv: int, q_norm, k_norm,
            eps: float, rope_dim: int, freq_base: float, pos: int):
    """x float32 [T, n_embd]; W* bf16 bits uint16 [rows, n_embd] (Wq may be None).  Returns
    (Q [T, n_head, 256] or None, K [T, n_head_kv*256], V [T, n_head_kv*256]) float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    T, n_embd = x.shape
    Q = np.zeros((T, n_head, 256), np.float32) if Wq is not None else None
    K = np.zeros((T, n_head_kv * 256), np.float32)
    V = np.zeros_like(K)
    wq = np.ascontiguousarray(Wq, dtype=np.uint16) if Wq is not None else None
    qn = np.ascontiguousarray(q_norm, dtype=np.float32) if q_norm is not None else None
    kn = np.ascontiguousarray(k_norm, dtype=np.float32)
    wk = np.ascontiguousarray(Wk, dtype=np.uint16)
    wv = np.ascontiguousarray(Wv, dtype=np.uint16)
    lib().orc_project(_p(x), T, n_embd, _p(wq) if wq is not None else None, _p(wk), _p(wv), n_head, n_head_kv,
                      _p(qn) if qn is not None else None, _p(kn), ctypes.c_float(eps), rope_dim,
                      ctypes.c_float(freq_base), pos, _p(Q) if Q is not None else None, _p(K), _p(V))
    return Q, K, V

