"""GPU: the indexer's prefill side (qsa_top_k + qsa_mask in graph_builder::sparse_attn,
src/qwfn_graph.cpp:313-415, with engine::fill_chunk_qsa's bias, src/qwfn_engine.cpp:1276-1320).

Per query row at position q: whole blocks before it are scored, the incomplete block holding q is
forced in, the best blocks up to k_blocks = 513 are kept (all of them when there are no more), and
the row attends causally to the kept cells only.  Checked against the oracle: kept blocks bit-exact
(oracle.idx_select on the device's pooled keys), attention over the kept cells (oracle.attn with a
cell list) within the attention tolerance.
"""
from __future__ import annotations

import numpy as np
import pytest

from helpers import append_rows, assert_close, normal, to_dev
from test_gpu_indexer import N_HEAD_IDX, idx_engine, read_idx

pytestmark = pytest.mark.gpu
SCALE = 1 / 16


def bf16(x: np.ndarray):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16)
    return t.view(torch.int16).cuda(), t.float().numpy()


def run_chunks(eng, oracle, n, chunk, seed):
    """Append n positions chunk by chunk (K/V rows, indexer keys) and run the sparse prefill of
    every chunk; returns host copies of everything the checks need."""
    import torch
    Kf, Vf = normal(seed, (n, 512)), normal(seed + 1, (n, 512))
    kr = normal(seed + 2, (n, 128), 2.0)
    q_idx = normal(seed + 3, (n, N_HEAD_IDX, 128))
    qbits, qvals = bf16(normal(seed + 4, (n, 16, 256)))
    out = torch.full((n, 16, 256), float("nan"), device="cuda")
    blocks = torch.full((n, eng.k_blocks), -7, dtype=torch.int32, device="cuda")
    n_out = torch.zeros(n, dtype=torch.int32, device="cuda")
    qd = to_dev(q_idx)
    for a in range(0, n, chunk):
        b = min(n, a + chunk)
        append_rows(eng, 0, 0, a, Kf[a:b], Vf[a:b])
        eng.idx_append(0, 0, a, to_dev(kr[a:b]))
        eng.attn_prefill_qsa(0, 0, a, qd[a:b], qbits[a:b], b - a, SCALE, out[a:b], blocks[a:b], n_out[a:b])
    torch.cuda.synchronize()
    assert eng.device_status() == 0
    _, pooled = read_idx(eng, 0, 0, 0, n // 4)
    return (oracle.quantize_rows(Kf), oracle.quantize_rows(Vf), q_idx, qvals, out.cpu().numpy(),
            blocks.cpu().numpy(), n_out.cpu().numpy(), pooled)


def check_rows(oracle, rows, K, V, q_idx, qvals, got, blocks, n_out, pooled, attn_rows):
    for q in rows:
        kept, _ = oracle.idx_select(q_idx[q], pooled, q, 513)
        assert n_out[q] == len(kept), q
        np.testing.assert_array_equal(blocks[q, :len(kept)], kept, err_msg=f"row {q}")
    for q in attn_rows:
        kept, _ = oracle.idx_select(q_idx[q], pooled, q, 513)
        cells = (4 * kept[:, None] + np.arange(4)[None, :]).reshape(-1)
        cells = cells[cells <= q].astype(np.int32)
        ref = oracle.attn(qvals[q][None], K, V, [q], 2, SCALE, cells=cells)
        assert_close(got[q][None], ref, f"row {q}")


def test_sparse_prefill_16k_prompt(cuda, qkvlib, oracle):
    """A 16384-token prompt in 32 chunks of 512: every row of the last chunk and of chunk 4
    (positions 2048..2559, where the selection starts) bit-exact; 64 rows of each attended."""
    eng, _ = idx_engine(qkvlib, n_ctx=16384, n_slots=1)
    eng.seq_alloc(0)
    n, C = 16384, 512
    K, V, q_idx, qvals, got, blocks, n_out, pooled = run_chunks(eng, oracle, n, C, 700)
    r = np.random.default_rng(7)
    for c in (4, 31):
        rows = np.arange(c * C, (c + 1) * C)
        attn_rows = np.sort(np.r_[rows[:2], rows[-2:], r.choice(rows, 60, replace=False)])
        check_rows(oracle, rows, K, V, q_idx, qvals, got, blocks, n_out, pooled, attn_rows)
    assert np.all(n_out[2052:] == 513) and np.all(n_out[:2048] == np.arange(2048) // 4 + 1)


def test_sparse_prefill_ragged_chunks(cuda, qkvlib, oracle):
    """Chunks that do not start or end on a block (130 rows), rows in incomplete blocks, every row
    checked in full."""
    eng, _ = idx_engine(qkvlib, n_ctx=4096, n_slots=1)
    eng.seq_alloc(0)
    n = 3000
    K, V, q_idx, qvals, got, blocks, n_out, pooled = run_chunks(eng, oracle, n, 130, 710)
    rows = np.arange(1950, n)
    check_rows(oracle, rows, K, V, q_idx, qvals, got, blocks, n_out, pooled, rows[::7])


def test_sparse_prefill_keeps_everything_below_the_budget(cuda, qkvlib, oracle):
    """Below 513 blocks every block is kept: the sparse prefill is the dense causal prefill."""
    import torch
    eng, _ = idx_engine(qkvlib, n_ctx=4096, n_slots=1)
    eng.seq_alloc(0)
    n = 1500
    Kf, Vf = normal(720, (n, 512)), normal(721, (n, 512))
    append_rows(eng, 0, 0, 0, Kf, Vf)
    eng.idx_append(0, 0, 0, to_dev(normal(722, (n, 128))))
    qbits, _ = bf16(normal(723, (n, 16, 256)))
    q_idx = to_dev(normal(724, (n, N_HEAD_IDX, 128)))
    dense, sparse = (torch.empty((n, 16, 256), device="cuda") for _ in range(2))
    eng.attn_prefill(0, 0, 0, qbits, n, SCALE, dense)
    eng.attn_prefill_qsa(0, 0, 0, q_idx, qbits, n, SCALE, sparse)
    torch.cuda.synchronize()
    assert eng.device_status() == 0
    np.testing.assert_array_equal(sparse.cpu().numpy(), dense.cpu().numpy())
