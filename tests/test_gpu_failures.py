"""Failure detection on the GPU, in forms that fault nothing and hang nothing.

* A selection id past the sequence is rejected by the decode kernel before any address is formed:
  the tile is skipped and the device status reports ST_BAD_INDEX (2).
* Every wait of the decode kernels is bounded.  A test-only switch (qkv_debug_decode_wait) makes
  the next launch withhold one tile copy while still waiting for its bytes, with a 1 ms limit: the
  call returns, the status reports ST_TIMEOUT (4), and the next launch on the same context is
  correct.  One long sequence (two tile stages per CTA, the long-pair merge kernel) and 40 short
  ones (one stage, the row merge kernel) are covered.
"""
from __future__ import annotations

import time

import numpy as np
import pytest

from helpers import HD, append_rows, assert_close, engine, normal, to_dev

pytestmark = pytest.mark.gpu
ST_BAD_INDEX, ST_TIMEOUT = 2, 4


def _fill(eng, oracle, lens, seed):
    kv = []
    for i, n in enumerate(lens):
        eng.seq_alloc(i)
        Kf, Vf = normal(seed + i, (n, 512)), normal(seed + 500 + i, (n, 512))
        append_rows(eng, 0, i, 0, Kf, Vf)
        kv.append((oracle.quantize_rows(Kf), oracle.quantize_rows(Vf)))
    return kv


def test_selection_past_the_context_sets_bad_index(cuda, qkvlib, oracle):
    import torch
    n, T = 1000, 3                      # 16 blocks of 64
    with engine(qkvlib, n_slots=1) as eng:
        (K, V), = _fill(eng, oracle, [n], 10)
        Q = normal(11, (1, T, 16, HD))
        q, out = to_dev(Q), torch.empty((1, T, 16, HD), device="cuda")
        bad = to_dev(np.array([[[0, 5, 40], [1, 15, 16]]], dtype=np.int32))   # 40 and 16 are past block 15
        eng.attn_decode(0, [0], [n - T], q, T, 1 / 16, out, sel=bad, n_sel=3)
        torch.cuda.synchronize()
        assert eng.device_status() & ST_BAD_INDEX
        assert eng.device_status() == 0   # read and cleared
        good = to_dev(np.array([[[0, 5, 15], [1, 14, 15]]], dtype=np.int32))
        eng.attn_decode(0, [0], [n - T], q, T, 1 / 16, out, sel=good, n_sel=3)
        torch.cuda.synchronize()
        assert eng.device_status() == 0
        cells = [oracle.blocks_to_cells(np.array(b, np.int32), 64, n) for b in ([0, 5, 15], [1, 14, 15])]
        ref = oracle.attn_sparse(Q[0], K, V, np.arange(n - T, n), 2, 1 / 16, cells)
        assert_close(out.cpu().numpy()[0], ref, "after the bad index")


@pytest.mark.parametrize("lens", [[16000], [3000] * 40], ids=["one-long-sequence", "forty-sequences"])
def test_withheld_tile_copy_times_out_and_the_context_recovers(cuda, qkvlib, oracle, lens):
    import torch
    T = 3
    with engine(qkvlib, n_slots=len(lens), n_ctx=16384) as eng:
        kv = _fill(eng, oracle, lens, 20)
        Q = normal(21, (len(lens), T, 16, HD))
        q, out = to_dev(Q), torch.empty((len(lens), T, 16, HD), device="cuda")
        pos = [n - T for n in lens]
        eng.debug_decode_wait(1_000_000, withhold_unit=0)    # 1 ms; unit 0 never gets its first tile
        t0 = time.perf_counter()
        eng.attn_decode(0, list(range(len(lens))), pos, q, T, 1 / 16, out)
        torch.cuda.synchronize()
        assert time.perf_counter() - t0 < 5.0
        assert eng.device_status() & ST_TIMEOUT
        eng.debug_decode_wait(0)                               # default limit, nothing withheld
        eng.attn_decode(0, list(range(len(lens))), pos, q, T, 1 / 16, out)
        torch.cuda.synchronize()
        assert eng.device_status() == 0
        got = out.cpu().numpy()
        for i, n in enumerate(lens[:3]):
            ref = oracle.attn(Q[i], kv[i][0], kv[i][1], np.arange(n - T, n), 2, 1 / 16)
            assert_close(got[i], ref, f"seq {i} after the timed-out launch")
