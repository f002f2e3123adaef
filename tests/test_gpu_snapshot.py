"""GPU: kernel E and the block manager -- shared-prefix snapshots (page sharing, copy-on-write),
host blobs in the reference's snapshot_parts order, recurrent-state copies, rollback."""
from __future__ import annotations

import numpy as np
import pytest

from helpers import HD, ROW, append_rows, decode, engine, normal, read_rows, to_dev

pytestmark = pytest.mark.gpu

REC = dict(rec_n_layer=3, rec_head_dim=16, rec_n_head=4, conv_channels=64, conv_hist=3)


class _DevMem:
    """A raw device range as a zero-copy float32 tensor (CUDA array interface)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes // 4,), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}


def dev_view(ptr: int, nbytes: int):
    import torch
    return torch.as_tensor(_DevMem(ptr, nbytes), device="cuda")


def rec_state(eng, slot, which=0):
    import torch
    out = []
    torch.cuda.synchronize()
    for l in range(eng.cfg.rec_n_layer):
        for kind in (0, 1):
            p, n = eng.state_ptr(slot, l, kind, which)
            out.append(dev_view(p, n).cpu().numpy())
    return out


def set_rec_state(eng, slot, seed, which=0):
    import torch
    vals = []
    for l in range(eng.cfg.rec_n_layer):
        for kind in (0, 1):
            p, n = eng.state_ptr(slot, l, kind, which)
            a = normal(seed * 100 + l * 2 + kind, (n // 4,))
            dev_view(p, n).copy_(torch.from_numpy(a))
            vals.append(a)
    torch.cuda.synchronize()
    return vals


def test_snapshot_share_restore_and_copy_on_write(cuda, qkvlib, oracle):
    eng = engine(qkvlib, n_layer=2, n_slots=4, **REC)
    eng.seq_alloc(0)
    n = 700
    Kf = [normal(10 + l, (n, 512)) for l in range(2)]
    Vf = [normal(20 + l, (n, 512)) for l in range(2)]
    for l in range(2):
        append_rows(eng, l, 0, 0, Kf[l], Vf[l])
    saved_state = set_rec_state(eng, 0, seed=1)
    snap = eng.snapshot_save(0)
    assert snap.n_past == n
    eng.seq_alloc(1)
    eng.seq_alloc(2)
    eng.snapshot_load(snap, 1)
    eng.snapshot_load(snap, 2, n_keep=300)
    assert eng.pages(1) == eng.pages(0) and eng.pages(2) == eng.pages(0)[:2]
    # divergent tails: each slot writes its own rows into what were shared pages
    tail1 = [normal(30 + l, (10, 512)) for l in range(2)]
    tail2 = [normal(40 + l, (50, 512)) for l in range(2)]
    own0 = [normal(50 + l, (1, 512)) for l in range(2)]
    for l in range(2):
        append_rows(eng, l, 1, n, tail1[l], tail1[l])
        append_rows(eng, l, 2, 300, tail2[l], tail2[l])
        append_rows(eng, l, 0, n, own0[l], own0[l])
    for l in range(2):
        Kq, Vq = oracle.quantize_rows(Kf[l]), oracle.quantize_rows(Vf[l])
        K0, V0 = read_rows(eng, l, 0, 0, n + 1)
        assert np.array_equal(K0[:n], Kq) and np.array_equal(V0[:n], Vq)
        assert np.array_equal(K0[n:], oracle.quantize_rows(own0[l]))
        K1, _ = read_rows(eng, l, 1, 0, n + 10)
        assert np.array_equal(K1[:n], Kq) and np.array_equal(K1[n:], oracle.quantize_rows(tail1[l]))
        K2, V2 = read_rows(eng, l, 2, 0, 350)
        assert np.array_equal(K2[:300], Kq[:300]) and np.array_equal(V2[:300], Vq[:300])
        assert np.array_equal(K2[300:], oracle.quantize_rows(tail2[l]))
    for a, b in zip(rec_state(eng, 1), saved_state):
        assert np.array_equal(a, b)
    snap.release()


def test_decode_after_restore_is_identical(cuda, qkvlib, oracle):
    eng = engine(qkvlib, n_slots=3)
    eng.seq_alloc(0)
    n = 3333
    append_rows(eng, 0, 0, 0, normal(1, (n, 512)), normal(2, (n, 512)))
    Q = normal(3, (1, 16, HD))
    a = decode(eng, 0, [0], [n - 1], Q, 1)
    snap = eng.snapshot_save(0)
    eng.seq_alloc(2)
    eng.snapshot_load(snap, 2)
    b = decode(eng, 0, [2], [n - 1], Q, 1)
    assert np.array_equal(a, b)
    snap.release()


def test_snapshot_host_blob_roundtrip(cuda, qkvlib, oracle):
    eng = engine(qkvlib, n_layer=2, n_slots=3, **REC)
    eng.seq_alloc(0)
    n = 333
    Kf = [normal(60 + l, (n, 512)) for l in range(2)]
    Vf = [normal(70 + l, (n, 512)) for l in range(2)]
    for l in range(2):
        append_rows(eng, l, 0, 0, Kf[l], Vf[l])
    state = set_rec_state(eng, 0, seed=7)
    snap = eng.snapshot_save(0)
    blob = eng.snapshot_to_host(snap)
    # layout: per attention layer K rows then V rows (ggml q8_0), then per recurrent layer rs, conv
    off = 0
    for l in range(2):
        for X in (Kf[l], Vf[l]):
            nb = n * 2 * ROW
            assert bytes(blob[off:off + nb]) == oracle.quantize_rows(X).tobytes()
            off += nb
    for a in state:
        assert bytes(blob[off:off + a.nbytes]) == a.tobytes()
        off += a.nbytes
    assert off == len(blob)
    snap2 = eng.snapshot_from_host(blob, n)
    eng.seq_alloc(2)
    eng.snapshot_load(snap2, 2)
    for l in range(2):
        K, V = read_rows(eng, l, 2, 0, n)
        assert np.array_equal(K, oracle.quantize_rows(Kf[l])) and np.array_equal(V, oracle.quantize_rows(Vf[l]))
    for a, b in zip(rec_state(eng, 2), state):
        assert np.array_equal(a, b)
    with pytest.raises(qkvlib.QkvError) as e:
        eng.snapshot_from_host(blob[:-4], n)
    assert e.value.status == qkvlib.ERR_MISMATCH
    snap.release()
    snap2.release()


def test_restore_many_and_rollback(cuda, qkvlib, oracle):
    eng = engine(qkvlib, n_slots=10, n_rollback=2, **REC)
    eng.seq_alloc(0)
    append_rows(eng, 0, 0, 0, normal(1, (512, 512)), normal(2, (512, 512)))
    state = set_rec_state(eng, 0, seed=3)
    snap = eng.snapshot_save(0)
    slots = list(range(1, 10))
    for s in slots:
        eng.seq_alloc(s)
    keep = [512 - 7 * s for s in slots]
    eng.snapshot_load_many(snap, slots, keep)
    for s, k in zip(slots, keep):
        assert eng.n_past(s) == k
        for a, b in zip(rec_state(eng, s), state):
            assert np.array_equal(a, b)
    # rollback: the state two tokens back is what rollback snapshot 1 holds
    back2 = set_rec_state(eng, 4, seed=9, which=2)
    eng.rollback_arm(4, 2)
    n4 = eng.n_past(4)
    eng.rollback_n(4, 2)
    assert eng.n_past(4) == n4 - 2
    for a, b in zip(rec_state(eng, 4), back2):
        assert np.array_equal(a, b)
    # reset zeroes the recurrent state
    eng.reset(5)
    assert all(not a.any() for a in rec_state(eng, 5))
    snap.release()
