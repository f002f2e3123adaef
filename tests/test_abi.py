"""The C-ABI library on the CPU: it loads, exports every symbol include/qkv.h declares, and its
host logic (page pool, refcounts, copy-on-write bookkeeping, snapshots, rollback, errors, LPT
sharding) behaves on a host-only engine (device < 0, no kernels)."""
from __future__ import annotations

import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols() -> set[str]:
    src = open(os.path.join(ROOT, "include", "qkv.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return set(re.findall(r"\b(qkv_[a-z0-9_]+)\s*\(", src))


def test_every_declared_symbol_is_exported(qkvlib):
    names = declared_symbols()
    assert len(names) >= 30
    L = qkvlib.lib()
    missing = [n for n in sorted(names) if not hasattr(L, n)]
    assert not missing, missing
    assert names == set(qkvlib.EXPORTS), names ^ set(qkvlib.EXPORTS)


def host_engine(qkvlib, **kw):
    args = dict(n_layer=2, n_head=16, n_head_kv=2, n_ctx=4096, n_slots=4, n_pages=12, device=-1)
    args.update(kw)
    return qkvlib.Engine(**args)


def test_create_rejects_bad_shapes(qkvlib):
    with pytest.raises(qkvlib.QkvError) as e:
        host_engine(qkvlib, head_dim=128)
    assert e.value.status == qkvlib.ERR_INVALID
    with pytest.raises(qkvlib.QkvError):
        host_engine(qkvlib, n_head=15)


def test_pages_allocate_on_append_and_free(qkvlib):
    eng = host_engine(qkvlib)
    eng.seq_alloc(0)
    assert eng.pages_free() == 12
    with pytest.raises(qkvlib.QkvError) as e:   # host-only: pages reserved, no rows written
        eng.append(0, 0, 0, 1, 1, n_rows=600)
    assert e.value.status == qkvlib.ERR_UNSUPPORTED
    assert eng.n_past(0) == 600 and len(eng.pages(0)) == 3 and eng.pages_free() == 9
    eng.seq_free(0)
    assert eng.pages_free() == 12


def test_append_position_rules(qkvlib):
    eng = host_engine(qkvlib)
    eng.seq_alloc(1)
    with pytest.raises(qkvlib.QkvError) as e:
        eng.append(0, 1, 5, 1, 1, n_rows=1)        # pos beyond n_past
    assert e.value.status == qkvlib.ERR_INVALID
    with pytest.raises(qkvlib.QkvError) as e:
        eng.append(2, 1, 0, 1, 1, n_rows=1)        # bad layer
    assert e.value.status == qkvlib.ERR_INVALID
    with pytest.raises(qkvlib.QkvError) as e:
        eng.append(0, 2, 0, 1, 1, n_rows=1)        # slot not allocated
    assert e.value.status == qkvlib.ERR_STATE
    with pytest.raises(qkvlib.QkvError) as e:
        eng.append(0, 1, 0, 1, 1, n_rows=5000)     # beyond n_ctx
    assert e.value.status == qkvlib.ERR_STATE


def test_pool_exhaustion_is_all_or_nothing(qkvlib):
    eng = host_engine(qkvlib, n_pages=4)
    eng.seq_alloc(0)
    eng.seq_alloc(1)
    with pytest.raises(qkvlib.QkvError):
        eng.append(0, 0, 0, 1, 1, n_rows=768)      # 3 pages
    with pytest.raises(qkvlib.QkvError) as e:
        eng.append(0, 1, 0, 1, 1, n_rows=512)      # needs 2, 1 free
    assert e.value.status == qkvlib.ERR_NO_MEMORY
    assert eng.pages(1) == [] and eng.pages_free() == 1 and eng.n_past(1) == 0


def test_snapshot_shares_pages_and_copy_on_write(qkvlib):
    eng = host_engine(qkvlib)
    eng.seq_alloc(0)
    with pytest.raises(qkvlib.QkvError):
        eng.append(0, 0, 0, 1, 1, n_rows=300)      # pages 2 (one partial)
    pages = eng.pages(0)
    snap = eng.snapshot_save(0)
    assert snap.n_past == 300
    assert [eng.refcount(p) for p in pages] == [2, 2]
    free_before = eng.pages_free()
    # restore into two other slots keeping different prefixes
    eng.seq_alloc(1)
    eng.seq_alloc(2)
    eng.snapshot_load(snap, 1)
    eng.snapshot_load(snap, 2, n_keep=200)
    assert eng.pages(1) == pages and eng.pages(2) == pages[:1]
    assert eng.refcount(pages[0]) == 4 and eng.refcount(pages[1]) == 3
    assert eng.pages_free() == free_before           # nothing copied yet
    # slot 2 writes into the shared first page: it gets a private copy
    with pytest.raises(qkvlib.QkvError):
        eng.append(0, 2, 200, 1, 1, n_rows=10)
    p2 = eng.pages(2)
    assert p2[0] not in pages and eng.refcount(pages[0]) == 3 and eng.pages_free() == free_before - 1
    # the source slot appending into its partial page also copies (the snapshot keeps the original)
    with pytest.raises(qkvlib.QkvError):
        eng.append(0, 0, 300, 1, 1, n_rows=1)
    assert eng.pages(0)[1] != pages[1] and eng.refcount(pages[1]) == 2
    snap.release()
    eng.seq_free(1)
    assert eng.refcount(pages[1]) == 0 and eng.refcount(pages[0]) == 1   # slot 0 still holds it


def test_restore_own_snapshot_and_bad_keep(qkvlib):
    eng = host_engine(qkvlib)
    eng.seq_alloc(0)
    with pytest.raises(qkvlib.QkvError):
        eng.append(0, 0, 0, 1, 1, n_rows=257)
    snap = eng.snapshot_save(0)
    eng.snapshot_load(snap, 0)                        # restoring a slot's own snapshot is safe
    assert eng.n_past(0) == 257 and all(eng.refcount(p) == 2 for p in eng.pages(0))
    with pytest.raises(qkvlib.QkvError) as e:
        eng.snapshot_load(snap, 0, n_keep=258)
    assert e.value.status == qkvlib.ERR_INVALID
    eng.snapshot_load_many(snap, [0], [10])
    assert eng.n_past(0) == 10 and len(eng.pages(0)) == 1


def test_rollback_requires_armed_depth(qkvlib):
    eng = host_engine(qkvlib, n_rollback=3, rec_n_layer=2, rec_head_dim=8, rec_n_head=2, conv_channels=16)
    eng.seq_alloc(0)
    with pytest.raises(qkvlib.QkvError):
        eng.append(0, 0, 0, 1, 1, n_rows=20)
    with pytest.raises(qkvlib.QkvError) as e:
        eng.rollback_n(0, 1)
    assert e.value.status == qkvlib.ERR_STATE
    eng.rollback_arm(0, 3)
    with pytest.raises(qkvlib.QkvError):
        eng.rollback_n(0, 4)
    eng.rollback_n(0, 2)
    assert eng.n_past(0) == 18
    with pytest.raises(qkvlib.QkvError):               # depth cleared by the rollback
        eng.rollback_n(0, 1)
    with pytest.raises(qkvlib.QkvError):
        eng.rollback_arm(0, 4)


def test_reset_releases_pages(qkvlib):
    eng = host_engine(qkvlib)
    eng.seq_alloc(3)
    with pytest.raises(qkvlib.QkvError):
        eng.append(1, 3, 0, 1, 1, n_rows=1000)
    eng.reset(3)
    assert eng.n_past(3) == 0 and eng.pages(3) == [] and eng.pages_free() == 12


def test_summary_and_bytes(qkvlib):
    eng = host_engine(qkvlib)
    assert "host only" in eng.summary() and eng.bytes() == 0


def test_shard_lpt(qkvlib):
    costs = [5, 9, 1, 7, 3, 3, 8]
    owner = qkvlib.shard_lpt(costs, 3)
    loads = [sum(c for c, o in zip(costs, owner) if o == r) for r in range(3)]
    assert sorted(loads) == [12, 12, 12]
    assert qkvlib.shard_lpt([4, 4], 1) == [0, 0]
    with pytest.raises(qkvlib.QkvError):
        qkvlib.shard_lpt([1], 0)


def test_reserve_covers_only_future_positions(qkvlib):
    eng = host_engine(qkvlib, n_pages=8)
    eng.seq_alloc(0)
    with pytest.raises(qkvlib.QkvError):
        eng.append(0, 0, 0, 1, 1, n_rows=512)     # two full pages
    snap = eng.snapshot_save(0)
    eng.reserve(0, 700)                            # shared full pages stay shared, one new page
    assert [eng.refcount(p) for p in eng.pages(0)] == [2, 2, 1] and eng.n_past(0) == 512
    eng.reserve(0, 100)                            # nothing to do below n_past
    assert len(eng.pages(0)) == 3
    snap.release()
