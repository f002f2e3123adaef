"""GPU parity: kernel A (append), the ggml-layout transforms, kernel C (decode / verify) and
kernel B (summaries, selection, sparse decode) against the CPU oracle.  Bit-exact for q8_0
bytes, block summaries and selection indices; attention within atol 2e-3 + rtol 1e-3."""
from __future__ import annotations

import os

import numpy as np
import pytest

from helpers import ATOL, HD, ROW, append_rows, assert_close, decode, engine, normal, read_rows, to_dev

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "q8_0_gguf.npz")


def test_append_bit_exact_vs_gguf_golden(cuda, qkvlib, oracle):
    g = np.load(GOLDEN)
    x, q = g["x"], g["q8_0"]             # rows of 512 = 2 heads x 256
    eng = engine(qkvlib)
    eng.seq_alloc(0)
    append_rows(eng, 0, 0, 0, x, x[::-1].copy())
    K, V = read_rows(eng, 0, 0, 0, x.shape[0])
    assert np.array_equal(K, q), f"{int((K != q).sum())} K bytes differ from gguf-py"
    assert np.array_equal(V, q[::-1]), "V bytes differ from gguf-py"


@pytest.mark.parametrize("n,chunk", [(700, 4096), (70, 1), (300, 7)])
def test_append_bit_exact_vs_oracle(cuda, qkvlib, oracle, n, chunk):
    Kf, Vf = normal(n, (n, 512)), normal(n + 1, (n, 512), 3.0)
    eng = engine(qkvlib, n_layer=2)
    eng.seq_alloc(1)
    append_rows(eng, 1, 1, 0, Kf, Vf, chunk=chunk)
    K, V = read_rows(eng, 1, 1, 0, n)
    assert np.array_equal(K, oracle.quantize_rows(Kf))
    assert np.array_equal(V, oracle.quantize_rows(Vf))
    assert eng.n_past(1) == n and len(eng.pages(1)) == (n + 255) // 256


def test_gather_and_write_rows(cuda, qkvlib, oracle):
    import torch
    n = 600
    Kf, Vf = normal(1, (n, 512)), normal(2, (n, 512))
    eng = engine(qkvlib)
    eng.seq_alloc(0)
    append_rows(eng, 0, 0, 0, Kf, Vf)
    cells = np.random.default_rng(0).integers(0, n, 333).astype(np.int32)
    Kg = torch.empty((333, 2 * ROW), dtype=torch.uint8, device="cuda")
    Vg = torch.empty_like(Kg)
    eng.gather_rows(0, 0, to_dev(cells), Kg, Vg)
    torch.cuda.synchronize()
    Kq, Vq = oracle.quantize_rows(Kf), oracle.quantize_rows(Vf)
    assert np.array_equal(Kg.cpu().numpy(), Kq[cells]) and np.array_equal(Vg.cpu().numpy(), Vq[cells])
    # ggml rows written into another slot read back unchanged
    eng.seq_alloc(2)
    eng.write_rows(0, 2, 0, n, to_dev(Kq), to_dev(Vq))
    K2, V2 = read_rows(eng, 0, 2, 0, n)
    assert np.array_equal(K2, Kq) and np.array_equal(V2, Vq)


def fill_seq(eng, oracle, layer, slot, n, seed, scale=1.0):
    Kf, Vf = normal(seed, (n, 512), scale), normal(seed + 1000, (n, 512))
    append_rows(eng, layer, slot, 0, Kf, Vf)
    return oracle.quantize_rows(Kf), oracle.quantize_rows(Vf)


@pytest.mark.parametrize("n_kv,T", [(1, 1), (63, 1), (64, 2), (65, 3), (200, 4), (4097, 1), (5000, 3)])
def test_decode_dense_vs_oracle(cuda, qkvlib, oracle, n_kv, T):
    eng = engine(qkvlib)
    eng.seq_alloc(0)
    K, V = fill_seq(eng, oracle, 0, 0, n_kv, seed=n_kv)
    Q = normal(7 + T, (T, 16, HD))
    got = decode(eng, 0, [0], [n_kv - T], Q, T)
    ref = oracle.attn(Q, K, V, np.arange(n_kv - T, n_kv), 2, 1 / 16)
    assert_close(got.reshape(ref.shape), ref, f"n_kv={n_kv} T={T}")


def test_decode_ragged_batch_vs_oracle(cuda, qkvlib, oracle):
    lens = [3000, 17, 1025, 64, 2222]
    T = 3
    eng = engine(qkvlib, n_slots=6)
    kv = {}
    for i, n in enumerate(lens):
        eng.seq_alloc(i + 1)
        kv[i] = fill_seq(eng, oracle, 0, i + 1, n, seed=100 + i)
    Q = normal(5, (len(lens), T, 16, HD))
    got = decode(eng, 0, [i + 1 for i in range(len(lens))], [n - T for n in lens], Q, T)
    for i, n in enumerate(lens):
        ref = oracle.attn(Q[i], kv[i][0], kv[i][1], np.arange(n - T, n), 2, 1 / 16)
        assert_close(got[i], ref, f"seq {i} (n_kv {n})")


def test_decode_model_shape_gqa12(cuda, qkvlib, oracle):
    """The reference model's own head shape: 24 query heads over 2 KV heads."""
    eng = engine(qkvlib, n_head=24)
    eng.seq_alloc(0)
    n, T = 777, 2
    K, V = fill_seq(eng, oracle, 0, 0, n, seed=3)
    Q = normal(4, (T, 24, HD))
    got = decode(eng, 0, [0], [n - T], Q, T)
    ref = oracle.attn(Q, K, V, np.arange(n - T, n), 2, 1 / 16)
    assert_close(got.reshape(ref.shape), ref, "gqa12")


def test_decode_rejects_unwritten_positions(cuda, qkvlib):
    eng = engine(qkvlib)
    eng.seq_alloc(0)
    append_rows(eng, 0, 0, 0, normal(0, (10, 512)), normal(1, (10, 512)))
    with pytest.raises(qkvlib.QkvError) as e:
        decode(eng, 0, [0], [9], normal(2, (2, 16, HD)), 2)
    assert e.value.status == qkvlib.ERR_INVALID


def sparse_case(cuda, qkvlib, oracle, n_kv, T, top_k, seed, block_offset_std=np.sqrt(2.0)):
    r = np.random.default_rng(seed)
    nb = (n_kv + 63) // 64
    off = (r.standard_normal((nb, 2, 1)) * block_offset_std).astype(np.float32)
    Kf = normal(seed + 1, (nb * 64, 2, HD)) + off.repeat(64, axis=0)
    Kf = Kf[:n_kv].reshape(n_kv, 512)
    Vf = normal(seed + 2, (n_kv, 512))
    eng = engine(qkvlib, n_ctx=max(8192, n_kv + 64), select_block=64)
    eng.seq_alloc(0)
    append_rows(eng, 0, 0, 0, Kf, Vf)
    Kq, Vq = oracle.quantize_rows(Kf), oracle.quantize_rows(Vf)
    Q = normal(seed + 3, (T, 16, HD))
    import torch
    idx = torch.empty((1, 2, top_k), dtype=torch.int32, device="cuda")
    scores = torch.full((1, 2, eng.cfg.n_ctx // 64), float("nan"), dtype=torch.float32, device="cuda")
    eng.select_blocks(0, [0], [n_kv - T], to_dev(Q[None]), T, top_k, idx, scores)
    torch.cuda.synchronize()
    summ = oracle.block_summary(Kq, 2, HD, 64, max(nb - 2, 0))
    summ_full = np.zeros((2, nb, HD), np.uint16)
    summ_full[:, :max(nb - 2, 0)] = summ
    ref_idx, ref_scores = oracle.select_blocks(Q, 2, summ_full, nb, top_k)
    got_idx = idx.cpu().numpy()[0]
    got_scores = scores.cpu().numpy()[0][:, :nb]
    assert np.array_equal(got_scores.view(np.uint32), ref_scores.view(np.uint32)), "block scores not bit-exact"
    assert np.array_equal(got_idx, ref_idx), "selection indices not bit-exact"
    got = decode(eng, 0, [0], [n_kv - T], Q, T, sel=idx, n_sel=top_k)
    cells = [oracle.blocks_to_cells(ref_idx[h][ref_idx[h] >= 0], 64, n_kv) for h in range(2)]
    ref = oracle.attn_sparse(Q, Kq, Vq, np.arange(n_kv - T, n_kv), 2, 1 / 16, cells)
    assert_close(got.reshape(ref.shape), ref, "sparse decode")
    return got_idx


def test_sparse_select_and_decode_small(cuda, qkvlib, oracle):
    sparse_case(cuda, qkvlib, oracle, n_kv=64 * 50 + 17, T=3, top_k=8, seed=1)


def test_sparse_select_fewer_blocks_than_topk(cuda, qkvlib, oracle):
    idx = sparse_case(cuda, qkvlib, oracle, n_kv=300, T=2, top_k=8, seed=2)
    assert list(idx[0]) == [0, 1, 2, 3, 4, -1, -1, -1]


def test_sparse_select_wide_batch(cuda, qkvlib, oracle):
    """40 sequences x 2 KV heads of 64 blocks: the selection grids take their coarser split
    (32 candidates per score CTA, 8 rank CTAs per head) instead of a single sequence's finest
    one; every sequence's scores and indices bit-exact."""
    import torch
    n_seq, n_kv, T, top_k = 40, 64 * 64, 3, 8
    nb = n_kv // 64
    eng = engine(qkvlib, n_ctx=n_kv + 64, n_slots=n_seq, select_block=64)
    Qs, refs = [], []
    for s in range(n_seq):
        r = np.random.default_rng(100 + s)
        off = (r.standard_normal((nb, 2, 1)) * np.sqrt(2.0)).astype(np.float32)
        Kf = (normal(200 + s, (nb * 64, 2, HD)) + off.repeat(64, axis=0)).reshape(n_kv, 512)
        Vf = normal(300 + s, (n_kv, 512))
        eng.seq_alloc(s)
        append_rows(eng, 0, s, 0, Kf, Vf)
        Q = normal(400 + s, (T, 16, HD))
        Qs.append(Q)
        summ_full = np.zeros((2, nb, HD), np.uint16)
        summ_full[:, :nb - 2] = oracle.block_summary(oracle.quantize_rows(Kf), 2, HD, 64, nb - 2)
        refs.append(oracle.select_blocks(Q, 2, summ_full, nb, top_k))
    idx = torch.empty((n_seq, 2, top_k), dtype=torch.int32, device="cuda")
    scores = torch.full((n_seq, 2, eng.cfg.n_ctx // 64), float("nan"), dtype=torch.float32, device="cuda")
    eng.select_blocks(0, list(range(n_seq)), [n_kv - T] * n_seq, to_dev(np.stack(Qs)), T, top_k, idx, scores)
    torch.cuda.synchronize()
    assert eng.device_status() == 0
    got_idx, got_sc = idx.cpu().numpy(), scores.cpu().numpy()
    for s, (ref_idx, ref_sc) in enumerate(refs):
        assert np.array_equal(got_sc[s][:, :nb].view(np.uint32), ref_sc.view(np.uint32)), f"scores of sequence {s}"
        assert np.array_equal(got_idx[s], ref_idx), f"indices of sequence {s}"


def test_sparse_config4_full_size(cuda, qkvlib, oracle):
    """ctx 73728, 64-token blocks, top-32 per KV head, T = 3."""
    sparse_case(cuda, qkvlib, oracle, n_kv=73728, T=3, top_k=32, seed=3)


@pytest.mark.parametrize("T", [1, 3, 4])
def test_fused_append_decode_vs_oracle(cuda, qkvlib, oracle, T):
    """Kernel A fused into kernel C: the appended bytes and the attention both match."""
    # 6334 and 20478: the new rows straddle two tiles of sequences long enough that different
    # units may own them (each unit writes its rows into the page before copying that tile in)
    lens = [1500, 64 - T, 255, 3, 6334, 20478]
    eng = engine(qkvlib, n_slots=6, n_ctx=20608)
    K0, V0, Kn, Vn = {}, {}, {}, {}
    for i, n in enumerate(lens):
        eng.seq_alloc(i)
        K0[i], V0[i] = normal(200 + i, (n, 512)), normal(300 + i, (n, 512))
        append_rows(eng, 0, i, 0, K0[i], V0[i])
        Kn[i], Vn[i] = normal(400 + i, (T, 512)), normal(500 + i, (T, 512))
    import torch
    Q = normal(9, (len(lens), T, 16, HD))
    q = to_dev(Q)
    out = torch.empty_like(q)
    eng.append_attn_decode(0, list(range(len(lens))), lens, to_dev(np.stack([Kn[i] for i in range(len(lens))])),
                           to_dev(np.stack([Vn[i] for i in range(len(lens))])), q, T, 1 / 16, out)
    torch.cuda.synchronize()
    assert eng.device_status() == 0
    got = out.cpu().numpy()
    for i, n in enumerate(lens):
        assert eng.n_past(i) == n + T
        Kall, Vall = np.concatenate([K0[i], Kn[i]]), np.concatenate([V0[i], Vn[i]])
        Kq, Vq = read_rows(eng, 0, i, 0, n + T)
        assert np.array_equal(Kq, oracle.quantize_rows(Kall)) and np.array_equal(Vq, oracle.quantize_rows(Vall))
        ref = oracle.attn(Q[i], Kq, Vq, np.arange(n, n + T), 2, 1 / 16)
        assert_close(got[i], ref, f"fused seq {i}")


def test_decode_many_units_with_merge(cuda, qkvlib, oracle):
    """A long and a short sequence: the long pairs are split over many units (merge kernel), the
    short one runs as single-unit pairs that write their output directly."""
    lens = [40000, 100]
    eng = engine(qkvlib, n_slots=2, n_ctx=40960)
    kv = {}
    for i, n in enumerate(lens):
        eng.seq_alloc(i)
        kv[i] = fill_seq(eng, oracle, 0, i, n, seed=700 + i)
    Q = normal(8, (2, 2, 16, HD))
    for rep in range(2):   # the scratch records are reused by the next launch
        got = decode(eng, 0, [0, 1], [n - 2 for n in lens], Q, 2)
        for i, n in enumerate(lens):
            ref = oracle.attn(Q[i], kv[i][0], kv[i][1], np.arange(n - 2, n), 2, 1 / 16)
            assert_close(got[i], ref, f"rep {rep} seq {i}")


def test_decode_widest_group_t4_g16(cuda, qkvlib, oracle):
    """The largest query group a pair holds: T=4 tokens x 16 q-heads over one KV head (64 rows)."""
    eng = engine(qkvlib, n_head=16, n_head_kv=1)
    eng.seq_alloc(0)
    n, T = 3001, 4
    Kf, Vf = normal(31, (n, HD)), normal(32, (n, HD))
    append_rows(eng, 0, 0, 0, Kf, Vf)
    K, V = read_rows(eng, 0, 0, 0, n, n_head_kv=1)
    Q = normal(33, (T, 16, HD))
    got = decode(eng, 0, [0], [n - T], Q, T)
    ref = oracle.attn(Q, K, V, np.arange(n - T, n), 1, 1 / 16)
    assert_close(got.reshape(ref.shape), ref, "T=4 G=16")
