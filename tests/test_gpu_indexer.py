"""GPU: the QSA lightning indexer (decode path) against the CPU oracle -- raw fp16 keys and pooled
block keys bit-exact (qsa_pool_blocks, src/qwfn_graph.cpp:280-299), kept blocks and scores
bit-exact (qsa_dec_cells + the decode bias, src/qwfn_graph.cpp:556-579,
src/qwfn_engine.cpp:1072-1105), and the sparse attention over the kept cells within the
attention tolerance (src/qwfn_graph.cpp:653-705)."""
from __future__ import annotations

import numpy as np
import pytest

from helpers import append_rows, assert_close, engine, normal, read_rows, to_dev

pytestmark = pytest.mark.gpu

N_HEAD_IDX, TOP_K, ROPE_DIM, BASE, EPS = 4, 2048, 64, 1e7, 1e-6


def idx_engine(qkvlib, n_layer=1, n_ctx=16384, n_slots=2, rope_dim=ROPE_DIM, **kw):
    eng = engine(qkvlib, n_layer=n_layer, n_ctx=n_ctx, n_slots=n_slots, **kw)
    w = (1 + 0.2 * np.random.default_rng(5).standard_normal((n_layer, 128))).astype(np.float32)
    kb = eng.indexer_enable(N_HEAD_IDX, TOP_K, rope_dim, BASE, EPS, k_norm=w)
    assert kb == 513
    return eng, w


def fill(eng, layer, slot, n, seed, chunks=None):
    """K/V rows and indexer keys for positions 0..n-1; returns (K, V, raw keys) float32."""
    Kf = normal(seed, (n, 512))
    Vf = normal(seed + 1, (n, 512))
    kr = normal(seed + 2, (n, 128), 2.0)
    bounds = chunks or [(0, n)]
    for a, b in bounds:
        append_rows(eng, layer, slot, a, Kf[a:b], Vf[a:b])
        eng.idx_append(layer, slot, a, to_dev(kr[a:b]))
    return Kf, Vf, kr


def read_idx(eng, layer, slot, n, n_blk):
    import torch
    keys = torch.empty((max(n, 1), 128), dtype=torch.int16, device="cuda")
    pooled = torch.empty((max(n_blk, 1), 128), dtype=torch.int16, device="cuda")
    eng.idx_read(layer, slot, 0, n, keys, 0, n_blk, pooled)
    torch.cuda.synchronize()
    return keys.cpu().numpy().view(np.uint16)[:n], pooled.cpu().numpy().view(np.uint16)[:n_blk]


def test_keys_and_pooled_bit_exact(cuda, qkvlib, oracle):
    eng, w = idx_engine(qkvlib)
    eng.seq_alloc(0)
    n = 1003
    _, _, kr = fill(eng, 0, 0, n, 300, chunks=[(0, 1), (1, 4), (4, 257), (257, 258), (258, 600), (600, 1003)])
    keys, pooled = read_idx(eng, 0, 0, n, n // 4)
    np.testing.assert_array_equal(keys, kr.astype(np.float16).view(np.uint16))
    want = oracle.idx_pool(keys, n // 4, w[0], EPS, ROPE_DIM, BASE)
    np.testing.assert_array_equal(pooled, want)
    assert eng.device_status() == 0


def _select(eng, slots, pos0, q, T):
    import torch
    nv = len(slots) * T
    blocks = torch.full((nv, eng.k_blocks), -7, dtype=torch.int32, device="cuda")
    n_out = torch.zeros(nv, dtype=torch.int32, device="cuda")
    scores = torch.zeros((nv, eng.cfg.n_ctx // 4), dtype=torch.float32, device="cuda")
    eng.idx_select(0, slots, pos0, to_dev(q), T, blocks, n_out, scores)
    torch.cuda.synchronize()
    return blocks.cpu().numpy(), n_out.cpu().numpy(), scores.cpu().numpy()


def test_select_bit_exact(cuda, qkvlib, oracle):
    eng, w = idx_engine(qkvlib)
    eng.seq_alloc(0)
    eng.seq_alloc(1)
    n0, n1 = 5000, 1000            # 1250 blocks (selection) and 250 blocks (everything kept)
    fill(eng, 0, 0, n0, 310)
    fill(eng, 0, 1, n1, 320)
    T = 3
    q = normal(330, (2, T, N_HEAD_IDX, 128))
    pos0 = [n0 - T, n1 - T]
    blocks, n_out, scores = _select(eng, [0, 1], pos0, q, T)
    for i, (slot, n) in enumerate(((0, n0), (1, n1))):
        _, pooled = read_idx(eng, 0, slot, 0, n // 4)
        for t in range(T):
            pos = pos0[i] + t
            kept, sc = oracle.idx_select(q[i, t], pooled, pos, 513)
            v = i * T + t
            assert n_out[v] == len(kept), (i, t)
            np.testing.assert_array_equal(blocks[v, :len(kept)], kept)
            assert np.all(blocks[v, len(kept):] == -1)
            if len(kept) == 513:     # scores are computed when there is a selection to make
                np.testing.assert_array_equal(scores[v, :len(sc)], sc)
    # 4997 = 4*1249+1 and 4998: tail block 1249 forced; 4999: block 1249 whole
    assert blocks[0, 512] == 1249 and blocks[1, 512] == 1249
    assert eng.device_status() == 0


def test_select_ties_to_lower_index(cuda, qkvlib, oracle):
    """Equal pooled keys (equal raw keys in every block, no rope): all scores tie, lower indices win."""
    eng, w = idx_engine(qkvlib, rope_dim=0)
    eng.seq_alloc(0)
    n = 8192
    Kf, Vf = normal(340, (n, 512)), normal(341, (n, 512))
    append_rows(eng, 0, 0, 0, Kf, Vf)
    kr = np.tile(normal(342, (4, 128)), (n // 4, 1))
    eng.idx_append(0, 0, 0, to_dev(kr))
    q = normal(343, (1, 2, N_HEAD_IDX, 128))
    blocks, n_out, _ = _select(eng, [0], [4095], q, 2)      # 4095: whole block 1023; 4096: tail 1024
    _, pooled = read_idx(eng, 0, 0, 0, n // 4)
    assert np.all(pooled == pooled[0])
    for t in range(2):
        kept, sc = oracle.idx_select(q[0, t], pooled, 4095 + t, 513)
        np.testing.assert_array_equal(blocks[t, :n_out[t]], kept)
    np.testing.assert_array_equal(blocks[0], np.arange(513))
    np.testing.assert_array_equal(blocks[1], np.r_[np.arange(512), 1024])


def test_attn_decode_qsa_matches_oracle(cuda, qkvlib, oracle):
    import torch
    eng, w = idx_engine(qkvlib)
    eng.seq_alloc(0)
    eng.seq_alloc(1)
    n0, n1 = 6001, 900
    fill(eng, 0, 0, n0, 350)
    fill(eng, 0, 1, n1, 360)
    T = 3
    q_idx = normal(370, (2, T, N_HEAD_IDX, 128))
    Q = normal(371, (2, T, 16, 256))
    pos0 = [n0 - T, n1 - T]
    out = torch.full((2, T, 16, 256), float("nan"), dtype=torch.float32, device="cuda")
    eng.attn_decode_qsa(0, [0, 1], pos0, to_dev(q_idx), to_dev(Q), T, 1 / 16, out)
    torch.cuda.synchronize()
    assert eng.device_status() == 0
    got = out.cpu().numpy()
    for i, (slot, n) in enumerate(((0, n0), (1, n1))):
        kq, vq = read_rows(eng, 0, slot, 0, n)
        _, pooled = read_idx(eng, 0, slot, 0, n // 4)
        for t in range(T):
            pos = pos0[i] + t
            kept, _ = oracle.idx_select(q_idx[i, t], pooled, pos, 513)
            cells = (4 * kept[:, None] + np.arange(4)[None, :]).reshape(-1)
            cells = cells[cells <= pos].astype(np.int32)
            ref = oracle.attn(Q[i, t:t + 1], kq, vq, [pos], 2, 1 / 16, cells=cells)
            assert_close(got[i, t:t + 1], ref, f"seq {i} token {t}")


def test_copy_on_write_keeps_snapshot_keys(cuda, qkvlib, oracle):
    import torch
    eng, w = idx_engine(qkvlib, n_layer=2)
    eng.seq_alloc(0)
    eng.seq_alloc(1)
    n = 700
    fill(eng, 1, 0, n, 380)
    fill(eng, 0, 0, n, 390)
    keys0, pooled0 = read_idx(eng, 1, 0, n, n // 4)
    snap = eng.snapshot_save(0)
    eng.snapshot_load(snap, 1, n_keep=n - 6)              # partial last page, shared
    kr = normal(400, (10, 128), 2.0)
    Kf, Vf = normal(401, (10, 512)), normal(402, (10, 512))
    append_rows(eng, 1, 1, n - 6, Kf, Vf)                   # copy-on-write of the shared page
    eng.idx_append(1, 1, n - 6, to_dev(kr))
    torch.cuda.synchronize()
    k0b, p0b = read_idx(eng, 1, 0, n, n // 4)
    np.testing.assert_array_equal(k0b, keys0)               # the snapshot's slot is untouched
    np.testing.assert_array_equal(p0b, pooled0)
    k1, p1 = read_idx(eng, 1, 1, n + 4, (n + 4) // 4)
    np.testing.assert_array_equal(k1[:n - 6], keys0[:n - 6])
    np.testing.assert_array_equal(k1[n - 6:], kr.astype(np.float16).view(np.uint16))
    np.testing.assert_array_equal(p1, oracle.idx_pool(k1, (n + 4) // 4, w[1], EPS, ROPE_DIM, BASE))
    snap.release()
    assert eng.device_status() == 0


def test_host_blob_order_and_indexer_rows(cuda, qkvlib, oracle):
    """snapshot_parts order (src/qwfn_engine.cpp:987-998): layer by layer in the model's order, an
    attention layer's K rows, V rows and indexer rows, a recurrent layer's state and conv; import
    re-pools the indexer's whole blocks."""
    import torch
    from test_gpu_snapshot import rec_state, set_rec_state
    rec = dict(rec_n_layer=6, rec_head_dim=16, rec_n_head=2, conv_channels=32, conv_hist=3)
    eng, w = idx_engine(qkvlib, n_layer=2, n_ctx=4096, attn_interval=4, **rec)
    eng.seq_alloc(0)
    eng.seq_alloc(1)
    n = 530
    kr = [fill(eng, l, 0, n, 500 + 10 * l)[2] for l in range(2)]
    state = set_rec_state(eng, 0, seed=9)
    snap = eng.snapshot_save(0)
    blob = bytes(eng.snapshot_to_host(snap))
    rows = n * 2 * 272
    off = 0
    for il in range(8):
        if (il + 1) % 4 == 0:
            a = il // 4
            kq, vq = read_rows(eng, a, 0, 0, n)
            assert blob[off:off + rows] == kq.tobytes(); off += rows
            assert blob[off:off + rows] == vq.tobytes(); off += rows
            assert blob[off:off + n * 256] == kr[a].astype(np.float16).tobytes(); off += n * 256
        else:
            r = il - (il + 1) // 4
            for kind in (0, 1):
                part = state[2 * r + kind].tobytes()
                assert blob[off:off + len(part)] == part, (il, kind); off += len(part)
    assert off == len(blob) == snap.info()[1]
    snap2 = eng.snapshot_from_host(blob, n)
    eng.snapshot_load(snap2, 1)
    torch.cuda.synchronize()
    for a in range(2):
        k1, p1 = read_idx(eng, a, 1, n, n // 4)
        k0, p0 = read_idx(eng, a, 0, n, n // 4)
        np.testing.assert_array_equal(k1, k0)
        np.testing.assert_array_equal(p1, p0)
        np.testing.assert_array_equal(p1, oracle.idx_pool(k1, n // 4, w[a], EPS, ROPE_DIM, BASE))
    for x, y in zip(rec_state(eng, 1), state):
        np.testing.assert_array_equal(x, y)
    snap.release()
    snap2.release()
    assert eng.device_status() == 0


@pytest.mark.parametrize("T", [1, 4])
def test_select_and_attend_many_sequences(cuda, qkvlib, oracle, T):
    """23 sequences x T tokens: launches split into whole sequences (21 or 16 per decode launch),
    contexts from T tokens to past 513 blocks."""
    import torch
    n_seq = 23
    eng, w = idx_engine(qkvlib, n_ctx=2600, n_slots=n_seq)
    lens = [T, T + 1, T + 2] + [int(x) for x in np.linspace(40, 2590, n_seq - 3)]
    for s, n in enumerate(lens):
        eng.seq_alloc(s)
        fill(eng, 0, s, n, 600 + 7 * s)
    q_idx = normal(700, (n_seq, T, N_HEAD_IDX, 128))
    Q = normal(701, (n_seq, T, 16, 256))
    pos0 = [n - T for n in lens]
    blocks, n_out, _ = _select(eng, list(range(n_seq)), pos0, q_idx, T)
    out = torch.full((n_seq, T, 16, 256), float("nan"), dtype=torch.float32, device="cuda")
    eng.attn_decode_qsa(0, list(range(n_seq)), pos0, to_dev(q_idx), to_dev(Q), T, 1 / 16, out)
    torch.cuda.synchronize()
    assert eng.device_status() == 0
    got = out.cpu().numpy()
    for s, n in enumerate(lens):
        kq, vq = read_rows(eng, 0, s, 0, n)
        _, pooled = read_idx(eng, 0, s, 0, n // 4)
        for t in range(T):
            pos = pos0[s] + t
            kept, _ = oracle.idx_select(q_idx[s, t], pooled, pos, 513)
            v = s * T + t
            np.testing.assert_array_equal(blocks[v, :n_out[v]], kept)
            cells = (4 * kept[:, None] + np.arange(4)[None, :]).reshape(-1)
            cells = cells[cells <= pos].astype(np.int32)
            ref = oracle.attn(Q[s, t:t + 1], kq, vq, [pos], 2, 1 / 16, cells=cells)
            assert_close(got[s, t:t + 1], ref, f"seq {s} (len {n}) token {t}")


def test_rollback_and_reappend_repools(cuda, qkvlib, oracle):
    """Rewinding n_past and appending new keys over old positions pools the touched blocks again."""
    import torch
    eng, w = idx_engine(qkvlib, n_ctx=1030, n_rollback=3)   # n_ctx not a multiple of 4 (last block partial)
    eng.seq_alloc(0)
    fill(eng, 0, 0, 1030, 800)
    eng.rollback_arm(0, 3)
    eng.rollback_n(0, 3)                           # n_past 1027
    kr = normal(801, (3, 128), 2.0)
    append_rows(eng, 0, 0, 1027, normal(802, (3, 512)), normal(803, (3, 512)))
    eng.idx_append(0, 0, 1027, to_dev(kr))
    torch.cuda.synchronize()
    keys, pooled = read_idx(eng, 0, 0, 1030, 1030 // 4)
    np.testing.assert_array_equal(keys[1027:], kr.astype(np.float16).view(np.uint16))
    np.testing.assert_array_equal(pooled, oracle.idx_pool(keys, 1030 // 4, w[0], EPS, ROPE_DIM, BASE))
    assert eng.device_status() == 0


def test_indexer_errors(cuda, qkvlib):
    import ctypes
    import torch
    eng = engine(qkvlib, n_ctx=1024, n_slots=1)
    eng.seq_alloc(0)
    k = torch.zeros(4, 128, device="cuda")
    with pytest.raises(qkvlib.QkvError) as e:      # not enabled
        eng.idx_append(0, 0, 0, k)
    assert e.value.status == qkvlib.ERR_STATE
    L = qkvlib.lib()
    assert L.qkv_indexer_enable(eng.handle, None, None) == qkvlib.ERR_INVALID
    for bad in ((4, 128, 8, 2048, 64), (4, 64, 4, 2048, 64), (9, 128, 4, 2048, 64), (4, 128, 4, 2048, 62)):
        c = qkvlib.QkvIndexerConfig(*bad, 1e7, 1e-6)       # ratio, key length, heads, rope dims
        assert L.qkv_indexer_enable(eng.handle, ctypes.byref(c), None) == qkvlib.ERR_INVALID, bad
    eng.indexer_enable(4, 2048, 64, 1e7, 1e-6)
    with pytest.raises(qkvlib.QkvError) as e:      # beyond n_past
        eng.idx_append(0, 0, 5, k)
    assert e.value.status == qkvlib.ERR_INVALID
    with pytest.raises(qkvlib.QkvError) as e:      # keys not 16-byte aligned
        eng.idx_append(0, 0, 0, k.view(-1)[1:129].view(1, 128), n_rows=1)
    assert e.value.status == qkvlib.ERR_INVALID
    blocks = torch.empty(513, dtype=torch.int32, device="cuda")
    n_out = torch.empty(1, dtype=torch.int32, device="cuda")
    with pytest.raises(qkvlib.QkvError) as e:      # positions not appended yet
        eng.idx_select(0, [0], [0], torch.zeros(1, 1, 4, 128, device="cuda"), 1, blocks, n_out)
    assert e.value.status == qkvlib.ERR_INVALID
    with pytest.raises(qkvlib.QkvError) as e:      # enabled twice
        eng.indexer_enable(4, 2048, 64, 1e7, 1e-6)
    assert e.value.status == qkvlib.ERR_STATE
