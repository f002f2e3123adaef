"""GPU parity at the BASELINE configs' own sizes, on the exact paths the benchmark times.

* one layer, 4096 cached tokens + 1 appended, T = 1, seed 0 (fused append + decode).
* 12 layers at context 16384, three 3-token MTP-verify steps replayed from one CUDA
  graph of `qkv_append_attn_decode` calls, exactly as bench.py captures them; every appended q8_0
  row bit-exact and every layer's attention within tolerance of the oracle.
* the whole 16384-token prompt in 32 chunks of 512 (append, then tcgen05 prefill over
  the cache so far), the last chunk (512 queries over 16384 keys) and a middle one checked.
* 16 of the config's ragged contexts restored with `qkv_snapshot_restore_many` from an
  8192-token shared prefix (sequences shorter than 8193 keep part of it and copy the shared page
  on their first write), then one fused 1-token decode over the paged batch.
* value magnitudes: K and V scaled by 1e-3 and 1e2, with the tolerance scaled to the data.

The reference's semantics are ggml's flash_attn_ext over q8_0 views (src/qwfn_graph.cpp:461-471,
697-699) with the chained verify positions of src/qwfn_engine.cpp:2259-2282.
"""
from __future__ import annotations

import numpy as np
import pytest

from helpers import ATOL, HD, RTOL, append_rows, assert_close, engine, normal, read_rows, to_dev

pytestmark = pytest.mark.gpu
SCALE = 1 / 16


def test_config1_exact(cuda, qkvlib, oracle):
    """4096 cached rows, then the step's token appended and attended in one launch (seed 0:
    K [4097, 512], V [4097, 512], Q [1, 16, 256] drawn in that order from numpy default_rng(0))."""
    import torch
    r = np.random.default_rng(0)
    n = 4097
    Kf = r.standard_normal((n, 512), dtype=np.float32)
    Vf = r.standard_normal((n, 512), dtype=np.float32)
    Qf = r.standard_normal((1, 16, HD), dtype=np.float32)
    with engine(qkvlib, n_ctx=4352, n_slots=1) as eng:
        eng.seq_alloc(0)
        append_rows(eng, 0, 0, 0, Kf[:n - 1], Vf[:n - 1])
        out = torch.empty((1, 16, HD), device="cuda")
        eng.append_attn_decode(0, [0], [n - 1], to_dev(Kf[n - 1:]), to_dev(Vf[n - 1:]), to_dev(Qf), 1, SCALE, out)
        torch.cuda.synchronize()
        assert eng.device_status() == 0
        K, V = read_rows(eng, 0, 0, 0, n)
    Kq, Vq = oracle.quantize_rows(Kf), oracle.quantize_rows(Vf)
    assert np.array_equal(K, Kq) and np.array_equal(V, Vq)
    ref = oracle.attn(Qf, Kq, Vq, [n - 1], 2, SCALE)
    assert_close(out.cpu().numpy(), ref, "configs[0]")


def test_config2_graph_replay(cuda, qkvlib, oracle):
    """12 layers at 16384 + 3 per step, three steps captured once and replayed (bench.py's timed path)."""
    import torch
    L, T, CTX, STEPS = 12, 3, 16384, 3
    gen = torch.Generator(device="cuda").manual_seed(1)
    with engine(qkvlib, n_layer=L, n_ctx=CTX + T * (STEPS + 1), n_slots=1) as eng:
        eng.seq_alloc(0)
        for l in range(L):
            for c in range(0, CTX, 4096):
                eng.append(l, 0, c, torch.randn(4096, 512, generator=gen, device="cuda"),
                           torch.randn(4096, 512, generator=gen, device="cuda"))
        eng.reserve(0, CTX + T * STEPS)       # no block-table uploads inside the capture
        Qd = torch.randn(STEPS, L, T, 16, HD, generator=gen, device="cuda")
        Kd = torch.randn(STEPS, L, T, 512, generator=gen, device="cuda")
        Vd = torch.randn(STEPS, L, T, 512, generator=gen, device="cuda")
        out = torch.full((STEPS, L, T, 16, HD), float("nan"), device="cuda")
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(STEPS):
                for l in range(L):
                    eng.append_attn_decode(l, [0], [CTX + T * i], Kd[i, l], Vd[i, l], Qd[i, l], T, SCALE, out[i, l])
        graph.replay()
        torch.cuda.synchronize()
        assert eng.device_status() == 0
        rows = [read_rows(eng, l, 0, 0, CTX + T * STEPS) for l in range(L)]
        del graph
    Qn, Kn, Vn, got = Qd.cpu().numpy(), Kd.cpu().numpy(), Vd.cpu().numpy(), out.cpu().numpy()
    for l in range(L):
        K, V = rows[l]
        for i in range(STEPS):
            n0 = CTX + T * i
            assert np.array_equal(K[n0:n0 + T], oracle.quantize_rows(Kn[i, l])), f"layer {l} step {i}: K rows"
            assert np.array_equal(V[n0:n0 + T], oracle.quantize_rows(Vn[i, l])), f"layer {l} step {i}: V rows"
            ref = oracle.attn(Qn[i, l], K, V, np.arange(n0, n0 + T), 2, SCALE, n_cells=n0 + T)
            assert_close(got[i, l], ref, f"layer {l} step {i}")


def test_config3_whole_prompt(cuda, qkvlib, oracle):
    """The 16384-token prompt in 32 chunks of 512, as bench.py --workload cfg3 runs it."""
    import torch
    N, C = 16384, 512
    gen = torch.Generator(device="cuda").manual_seed(2)
    K = torch.randn(N, 512, generator=gen, device="cuda")
    V = torch.randn(N, 512, generator=gen, device="cuda")
    Qb = torch.randn(N, 16, HD, generator=gen, device="cuda").to(torch.bfloat16)
    out = torch.full((N, 16, HD), float("nan"), device="cuda")
    with engine(qkvlib, n_ctx=N, n_slots=1) as eng:
        eng.seq_alloc(0)
        for c in range(N // C):
            a, b = c * C, (c + 1) * C
            eng.append(0, 0, a, K[a:b], V[a:b])
            eng.attn_prefill(0, 0, a, Qb[a:b].view(torch.int16), C, SCALE, out[a:b])
        torch.cuda.synchronize()
        assert eng.device_status() == 0
        Kq, Vq = read_rows(eng, 0, 0, 0, N)
    assert np.array_equal(Kq, oracle.quantize_rows(K.cpu().numpy()))
    assert np.array_equal(Vq, oracle.quantize_rows(V.cpu().numpy()))
    qv = Qb.float().cpu().numpy()
    got = out.cpu().numpy()
    last = np.arange(N - C, N)                                           # every query of the last chunk
    mid = 15 * C + np.random.default_rng(2).choice(C, 64, replace=False)  # 64 queries of chunk 15
    for rows, what in ((last, "last chunk"), (np.sort(mid), "chunk 15")):
        ref = oracle.attn(qv[rows], Kq, Vq, rows, 2, SCALE, n_cells=int(rows.max()) + 1)
        assert_close(got[rows], ref, what)


def test_config5_restored_ragged_batch(cuda, qkvlib, oracle):
    """16 of configs[4]'s contexts after a shared-prefix restore, decoded in one fused launch."""
    import torch
    r = np.random.default_rng(4)
    ctx = [int(c) for c in np.floor(np.exp(r.uniform(np.log(1024), np.log(65536), 64)))][:16]
    assert sum(c < 8193 for c in ctx) >= 4
    PREFIX, n = 8192, len(ctx)
    pages = sum((c + 255) // 256 for c in ctx) + PREFIX // 256 + n + 8
    gen = torch.Generator(device="cuda").manual_seed(4)
    with engine(qkvlib, n_ctx=max(ctx) + 8, n_slots=n + 1, n_pages=pages) as eng:
        src = n
        eng.seq_alloc(src)
        eng.append(0, src, 0, torch.randn(PREFIX, 512, generator=gen, device="cuda"),
                   torch.randn(PREFIX, 512, generator=gen, device="cuda"))
        snap = eng.snapshot_save(src)
        keep = [min(PREFIX, c - 1) for c in ctx]
        for s in range(n):
            eng.seq_alloc(s)
        eng.snapshot_load_many(snap, list(range(n)), keep)
        for s, c in enumerate(ctx):
            eng.reserve(s, c)
            for p0 in range(keep[s], c - 1, 8192):
                m = min(8192, c - 1 - p0)
                eng.append(0, s, p0, torch.randn(m, 512, generator=gen, device="cuda"),
                           torch.randn(m, 512, generator=gen, device="cuda"))
        Qd = torch.randn(n, 1, 16, HD, generator=gen, device="cuda")
        Kd = torch.randn(n, 1, 512, generator=gen, device="cuda")
        Vd = torch.randn(n, 1, 512, generator=gen, device="cuda")
        out = torch.full((n, 1, 16, HD), float("nan"), device="cuda")
        pos = [c - 1 for c in ctx]
        eng.append_attn_decode(0, list(range(n)), pos, Kd, Vd, Qd, 1, SCALE, out)
        torch.cuda.synchronize()
        assert eng.device_status() == 0
        Kp, Vp = read_rows(eng, 0, src, 0, PREFIX)
        got = out.cpu().numpy()
        Qn, Kn, Vn = Qd.cpu().numpy(), Kd.cpu().numpy(), Vd.cpu().numpy()
        for s, c in enumerate(ctx):
            K, V = read_rows(eng, 0, s, 0, c)
            assert np.array_equal(K[:keep[s]], Kp[:keep[s]]) and np.array_equal(V[:keep[s]], Vp[:keep[s]]), \
                f"seq {s}: restored prefix rows"
            assert np.array_equal(K[c - 1], oracle.quantize_rows(Kn[s])[0]), f"seq {s}: appended K row"
            assert np.array_equal(V[c - 1], oracle.quantize_rows(Vn[s])[0]), f"seq {s}: appended V row"
            ref = oracle.attn(Qn[s], K, V, [c - 1], 2, SCALE)
            assert_close(got[s], ref, f"seq {s} (ctx {c}, {keep[s]} prefix positions kept)")
        snap.release()


@pytest.mark.parametrize("k_scale,v_scale", [(1.0, 1e-3), (1.0, 1e2), (1e-3, 1.0), (1e2, 1.0), (1e-3, 1e-3)])
def test_decode_value_magnitudes(cuda, qkvlib, oracle, k_scale, v_scale):
    """Small and large K/V.  The output scales with V, so the absolute part of the tolerance is
    scaled with it; the relative part stays 1e-3."""
    n, T = 3000, 3
    Kf, Vf = normal(60, (n, 512), k_scale), normal(61, (n, 512), v_scale)
    Q = normal(62, (T, 16, HD))
    with engine(qkvlib, n_slots=1) as eng:
        eng.seq_alloc(0)
        append_rows(eng, 0, 0, 0, Kf, Vf)
        from helpers import decode
        got = decode(eng, 0, [0], [n - T], Q, T)
    K, V = oracle.quantize_rows(Kf), oracle.quantize_rows(Vf)
    ref = oracle.attn(Q, K, V, np.arange(n - T, n), 2, SCALE)
    err = np.abs(got.reshape(ref.shape) - ref)
    bound = ATOL * v_scale + RTOL * np.abs(ref)
    assert (err <= bound).all(), (f"K x{k_scale} V x{v_scale}: {int((err > bound).sum())} outside; "
                                  f"max err {err.max():.3e}, max |ref| {np.abs(ref).max():.3e}")
