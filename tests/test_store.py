"""The device saved-sequence store (qkv_store_*): the reference server's saved_seq list, its
restore_or_reset and shared_prefix_split (tools/qwfn_server.cpp:764-800, 1380-1430), on a
host-only engine here (pages, refcounts and byte accounting; no kernels) and on cuda:0 under -m gpu
(the reference's snaptest: save, run something unrelated, restore, get the same rows and
attention as a straight run -- tools/qwfn_snaptest.cpp)."""
from __future__ import annotations

import numpy as np
import pytest

PAGE_BYTES_2H = 278528     # one page, two KV heads, K and V


def host_engine(qkvlib, **kw):
    args = dict(n_layer=2, n_head=16, n_head_kv=2, n_ctx=8192, n_slots=2, n_pages=64, device=-1)
    args.update(kw)
    return qkvlib.Engine(**args)


def fill(eng, slot, n, qkvlib):
    """Host-only engines reserve the pages of an append and report that no rows were written."""
    eng.reset(slot)
    for layer in range(eng.cfg.n_layer):
        with pytest.raises(qkvlib.QkvError):
            eng.append(layer, slot, 0, 1, 1, n_rows=n)
    assert eng.n_past(slot) == n


def held(n_tok, n_layer=2, rec=0):
    return -(-n_tok // 256) * PAGE_BYTES_2H * n_layer + rec


def test_save_keeps_lru_order_and_limits(qkvlib):
    eng = host_engine(qkvlib)
    eng.seq_alloc(0)
    st = qkvlib.Store(eng, cap_bytes=held(2048) * 3, max_entries=4)
    toks = {}
    for i, n in enumerate((600, 700, 800)):
        fill(eng, 0, n, qkvlib)
        toks[i] = list(range(i * 10_000, i * 10_000 + n))
        assert st.save(0, toks[i])
    assert [e[0] for e in st.entries()] == [600, 700, 800]
    assert st.info() == (3, held(600) + held(700) + held(800))
    # equal tokens replace (and become most recent)
    fill(eng, 0, 600, qkvlib)
    assert st.save(0, toks[0])
    assert [e[0] for e in st.entries()] == [700, 800, 600]
    # more than max_entries: least recently used leaves
    for n in (900, 1000):
        fill(eng, 0, n, qkvlib)
        assert st.save(0, list(range(50_000 + n, 50_000 + 2 * n)))
    assert [e[0] for e in st.entries()] == [800, 600, 900, 1000]
    # a snapshot above the cap is not kept, and is not an error
    fill(eng, 0, 6600, qkvlib)
    assert not st.save(0, list(range(6600)))
    assert st.info()[0] == 4
    # byte cap: a big entry pushes old ones out until the total fits
    fill(eng, 0, 4000, qkvlib)
    assert st.save(0, list(range(7, 4007)))
    n_e, b = st.info()
    assert b <= held(2048) * 3 and [e[0] for e in st.entries()][-1] == 4000
    assert b == sum(e[1] for e in st.entries())
    st.close()


def test_save_requires_tokens_for_every_position(qkvlib):
    eng = host_engine(qkvlib)
    eng.seq_alloc(0)
    st = qkvlib.Store(eng, cap_bytes=1 << 30)
    fill(eng, 0, 300, qkvlib)
    with pytest.raises(qkvlib.QkvError) as e:
        st.save(0, list(range(299)))
    assert e.value.status == qkvlib.ERR_INVALID and "300" in str(e.value)
    with pytest.raises(qkvlib.QkvError):
        st.save(1, [])                         # slot 1 not allocated
    assert st.info() == (0, 0)


def test_restore_or_reset_picks_longest_strict_prefix(qkvlib):
    eng = host_engine(qkvlib)
    eng.seq_alloc(0)
    st = qkvlib.Store(eng, cap_bytes=1 << 30)
    base = list(range(1000, 4000))
    for n in (2100, 2600, 3000):
        fill(eng, 0, n, qkvlib)
        st.save(0, base[:n])
    # extends 2100 and 2600 (not 3000: the prompt must be strictly longer than the entry)
    prompt = base[:2600] + [7, 8, 9]
    assert st.restore_or_reset(0, prompt) == 2600
    assert eng.n_past(0) == 2600
    assert [e[0] for e in st.entries()] == [2100, 3000, 2600]        # restored one is most recent
    # shared pages: the slot and the entry reference the same pages
    pages = eng.pages(0)
    assert all(eng.refcount(p) >= 2 for p in pages)
    assert st.restore_or_reset(0, base[:3000]) == 2600               # 3000 itself is not a strict prefix
    # nothing matches: the slot is reset
    assert st.restore_or_reset(0, [5] * 4000) == 0
    assert eng.n_past(0) == 0 and eng.pages(0) == []
    st.close()
    # the store's page references are gone with it
    assert all(eng.refcount(p) == 0 for p in pages)


def test_prefix_split_rules(qkvlib):
    eng = host_engine(qkvlib)
    eng.seq_alloc(0)
    st = qkvlib.Store(eng, cap_bytes=1 << 30)
    sysprompt = list(range(3000))
    fill(eng, 0, 2500, qkvlib)
    st.save(0, sysprompt[:2400] + list(range(90_000, 90_100)))       # shares 2400 tokens
    prompt = sysprompt + [1, 2, 3]
    assert st.prefix_split(prompt, n_consumed=0) == 2400
    assert st.prefix_split(prompt, n_consumed=2399) == 0             # L >= consumed + 2 fails
    assert st.prefix_split(prompt, n_consumed=2048) == 0             # engine already holds >= 2048
    assert st.prefix_split(prompt[:2416], n_consumed=0) == 0         # L + 16 < prompt length fails
    assert st.prefix_split(prompt[:2417], n_consumed=0) == 2400
    assert st.prefix_split(prompt, n_consumed=0, min_prefix=2401) == 0
    # once the prefix itself is saved, no second split
    fill(eng, 0, 2400, qkvlib)
    st.save(0, sysprompt[:2400])
    assert st.prefix_split(prompt, n_consumed=0) == 0


def test_evict_releases_pages(qkvlib):
    eng = host_engine(qkvlib, n_pages=12)
    eng.seq_alloc(0)
    st = qkvlib.Store(eng, cap_bytes=1 << 30)
    fill(eng, 0, 1500, qkvlib)                 # 6 pages
    st.save(0, list(range(1500)))
    eng.reset(0)
    assert eng.pages_free() == 6                # the entry keeps its pages
    fill(eng, 0, 1536, qkvlib)
    with pytest.raises(qkvlib.QkvError) as e:   # the pool is full
        eng.append(0, 0, 1536, 1, 1, n_rows=1)
    assert e.value.status == qkvlib.ERR_NO_MEMORY
    st.evict(1)
    assert st.info() == (0, 0) and eng.pages_free() == 6
    with pytest.raises(qkvlib.QkvError) as e:   # host-only: the page is reserved now
        eng.append(0, 0, 1536, 1, 1, n_rows=1)
    assert e.value.status == qkvlib.ERR_UNSUPPORTED


@pytest.mark.gpu
def test_store_snaptest_on_device(cuda, qkvlib, oracle):
    """Save a conversation, run an unrelated one in the same slot, restore: rows, recurrent state
    and decode attention equal a straight run."""
    import torch
    from helpers import append_rows, decode, engine, normal, read_rows
    from test_gpu_snapshot import REC, rec_state, set_rec_state

    eng = engine(qkvlib, n_layer=2, n_slots=2, **REC)
    eng.seq_alloc(0)
    st = qkvlib.Store(eng, cap_bytes=8 << 30)
    n = 2300
    Kf = [normal(40 + l, (n, 512)) for l in range(2)]
    Vf = [normal(50 + l, (n, 512)) for l in range(2)]
    for l in range(2):
        append_rows(eng, l, 0, 0, Kf[l], Vf[l])
    want_state = set_rec_state(eng, 0, seed=7)
    Q = normal(60, (1, 3, 16, 256))
    straight = decode(eng, 1, [0], [n - 3], Q, 3)
    want_rows = read_rows(eng, 1, 0, 0, n)
    toks = list(range(100, 100 + n))
    assert st.save(0, toks)

    # an unrelated conversation in the same slot
    assert st.restore_or_reset(0, [9] * 50) == 0
    for l in range(2):
        append_rows(eng, l, 0, 0, normal(70 + l, (900, 512)), normal(80 + l, (900, 512)))
    set_rec_state(eng, 0, seed=8)

    assert st.restore_or_reset(0, toks + [1, 2]) == n
    torch.cuda.synchronize()
    assert eng.n_past(0) == n
    for a, b in zip(rec_state(eng, 0), want_state):
        np.testing.assert_array_equal(a, b)
    got_rows = read_rows(eng, 1, 0, 0, n)
    for a, b in zip(got_rows, want_rows):
        np.testing.assert_array_equal(a, b)
    again = decode(eng, 1, [0], [n - 3], Q, 3)
    np.testing.assert_array_equal(again, straight)
    assert eng.device_status() == 0
    st.close()
