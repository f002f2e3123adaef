"""The MTP head's K/V cache (graph_builder::mtp_head_kv, src/qwfn_graph.cpp:883-922; written by
engine::prefill_mtp_kv and mtp_step, src/qwfn_engine.cpp:1818-1838).

The reference keeps the head's one attention block (the nextn block, the last layer of the MTP
model) in a second qwfn::state that follows the trunk's positions.  Here it is one more attention
layer of the same engine -- layer index n_attn (12 for the model) -- so it shares the slot, the
page table, snapshots and restores with the trunk.  Its row for position p is written once token
p + 1 is known, so the head's rows trail the trunk's by one; the rows of rejected drafts are
simply written again later (qkv_append at a position below n_past overwrites).
"""
from __future__ import annotations

import numpy as np
import pytest

from helpers import HD, append_rows, assert_close, decode, engine, normal, read_rows, to_dev

pytestmark = pytest.mark.gpu
TRUNK, HEAD = 0, 1   # an engine of one trunk attention layer and the head's layer


def test_head_rows_trail_the_trunk_and_are_rewritten(cuda, qkvlib, oracle):
    n = 700
    with engine(qkvlib, n_layer=2, n_slots=1) as eng:
        eng.seq_alloc(0)
        append_rows(eng, TRUNK, 0, 0, normal(800, (n, 512)), normal(801, (n, 512)))
        Kh, Vh = normal(802, (n - 1, 512)), normal(803, (n - 1, 512))
        append_rows(eng, HEAD, 0, 0, Kh, Vh)                 # rows 0 .. n-2: one behind the trunk
        assert eng.n_past(0) == n
        Q = normal(804, (1, 16, HD))
        got = decode(eng, HEAD, [0], [n - 2], Q, 1)          # the head attends up to its last row
        K, V = read_rows(eng, HEAD, 0, 0, n - 1)
        assert np.array_equal(K, oracle.quantize_rows(Kh)) and np.array_equal(V, oracle.quantize_rows(Vh))
        assert_close(got.reshape(1, 16, HD), oracle.attn(Q, K, V, [n - 2], 2, 1 / 16), "head decode")
        # two drafts rejected: the head's rows n-3, n-2 are written again with the accepted tokens'
        Kn, Vn = normal(805, (2, 512)), normal(806, (2, 512))
        append_rows(eng, HEAD, 0, n - 3, Kn, Vn)
        K2, V2 = read_rows(eng, HEAD, 0, 0, n - 1)
        assert np.array_equal(K2[:n - 3], K[:n - 3]) and np.array_equal(V2[:n - 3], V[:n - 3])
        assert np.array_equal(K2[n - 3:], oracle.quantize_rows(Kn)) and np.array_equal(V2[n - 3:], oracle.quantize_rows(Vn))
        got2 = decode(eng, HEAD, [0], [n - 2], Q, 1)
        assert_close(got2.reshape(1, 16, HD), oracle.attn(Q, K2, V2, [n - 2], 2, 1 / 16), "head decode after rewrite")
        # the trunk's rows are untouched by the head's writes
        Kt, _ = read_rows(eng, TRUNK, 0, 0, n)
        assert np.array_equal(Kt, oracle.quantize_rows(normal(800, (n, 512))))


def test_head_layer_rides_in_snapshots(cuda, qkvlib, oracle):
    """A shared-prefix snapshot carries the head's rows with the trunk's (same pages)."""
    n = 520
    with engine(qkvlib, n_layer=2, n_slots=2) as eng:
        eng.seq_alloc(0)
        append_rows(eng, TRUNK, 0, 0, normal(810, (n, 512)), normal(811, (n, 512)))
        append_rows(eng, HEAD, 0, 0, normal(812, (n - 1, 512)), normal(813, (n - 1, 512)))
        snap = eng.snapshot_save(0)
        eng.seq_alloc(1)
        eng.snapshot_load(snap, 1)
        for layer, rows in ((TRUNK, n), (HEAD, n - 1)):
            a = read_rows(eng, layer, 0, 0, rows)
            b = read_rows(eng, layer, 1, 0, rows)
            assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
        assert eng.pages(1) == eng.pages(0)
        snap.release()
