"""Kernel D parity: chunked causal prefill (tcgen05) against the CPU oracle.

The reference runs ggml's flash_attn_ext over the whole q8_0 cache for every prefill chunk with a
causal mask (src/qwfn_graph.cpp:417-476, mask src/qwfn_engine.cpp:1238-1274): query t of a chunk
starting at pos0 sees cells 0 .. pos0 + t.  The oracle is that computation (query quantised to
q8_0, exact integer block dots, fp32 softmax).  Q is bf16 as in config 3.
"""
from __future__ import annotations

import numpy as np
import pytest

from helpers import HD, assert_close, engine, normal, read_rows, to_dev

pytestmark = pytest.mark.gpu


def bf16(x: np.ndarray):
    """float32 -> (bf16 bits as int16 torch tensor on cuda, float32 values of those bf16)."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16)
    return t.view(torch.int16).cuda(), t.float().numpy()


def run_prefill(oracle, qkvlib, n_kv: int, pos0: int, Tc: int, seed: int, n_head: int = 16, n_head_kv: int = 2,
                chunks=None):
    """Append n_kv rows, then prefill-attend queries at pos0 .. pos0+Tc-1 (optionally in chunks);
    returns (gpu out, oracle out)."""
    import torch
    r = np.random.default_rng(seed)
    kv_dim = n_head_kv * HD
    Kf = r.standard_normal((n_kv, kv_dim), dtype=np.float32)
    Vf = r.standard_normal((n_kv, kv_dim), dtype=np.float32)
    Qf = r.standard_normal((Tc, n_head, HD), dtype=np.float32)
    qbits, qvals = bf16(Qf)
    out = torch.full((Tc, n_head, HD), float("nan"), dtype=torch.float32, device="cuda")
    with engine(qkvlib, n_head=n_head, n_head_kv=n_head_kv, n_ctx=max(8192, n_kv), n_slots=1) as eng:
        eng.seq_alloc(0)
        eng.append(0, 0, 0, to_dev(Kf), to_dev(Vf))
        for c0, c1 in (chunks or [(0, Tc)]):
            eng.attn_prefill(0, 0, pos0 + c0, qbits[c0:c1], c1 - c0, 1 / 16, out[c0:c1])
        torch.cuda.synchronize()
        assert eng.device_status() == 0
        kq, vq = read_rows(eng, 0, 0, 0, n_kv, n_head_kv)
    got = out.cpu().numpy()
    ref = oracle.attn(qvals, kq, vq, pos0 + np.arange(Tc), n_head_kv, 1 / 16, n_cells=n_kv)
    return got, ref


def test_prefill_first_chunk(oracle, qkvlib):
    got, ref = run_prefill(oracle, qkvlib, n_kv=128, pos0=0, Tc=128, seed=20)
    assert_close(got, ref, "first chunk")


def test_prefill_second_chunk(oracle, qkvlib):
    got, ref = run_prefill(oracle, qkvlib, n_kv=1024, pos0=512, Tc=512, seed=21)
    assert_close(got, ref, "second chunk")


def test_prefill_ragged_offsets(oracle, qkvlib):
    # chunk start and end off every 16/64/256 boundary; keys past n_kv inside the last tile
    got, ref = run_prefill(oracle, qkvlib, n_kv=137, pos0=37, Tc=100, seed=22)
    assert_close(got, ref, "ragged")


def test_prefill_long_context_split(oracle, qkvlib):
    # 4096 keys: tiles are split across CTAs and merged by their last segment
    got, ref = run_prefill(oracle, qkvlib, n_kv=4096, pos0=3584, Tc=512, seed=23)
    assert_close(got, ref, "long context")


def test_prefill_chunked_calls(oracle, qkvlib):
    # the same 768 queries as three chunks (each call sees the whole cache, causal per query)
    got, ref = run_prefill(oracle, qkvlib, n_kv=1500, pos0=732, Tc=768, seed=24,
                           chunks=[(0, 256), (256, 512), (512, 768)])
    assert_close(got, ref, "chunked")


def test_prefill_group_of_two(oracle, qkvlib):
    # 2 q-heads per KV head: tiles of 64 tokens x 2 heads
    got, ref = run_prefill(oracle, qkvlib, n_kv=520, pos0=300, Tc=220, seed=25, n_head=4, n_head_kv=2)
    assert_close(got, ref, "G=2")


def test_prefill_rejects_unappended_and_bad_sizes(qkvlib):
    import torch
    q = torch.zeros((64, 16, HD), dtype=torch.int16, device="cuda")
    out = torch.empty((64, 16, HD), dtype=torch.float32, device="cuda")
    with engine(qkvlib, n_slots=1) as eng:
        eng.seq_alloc(0)
        K = to_dev(normal(26, (32, 2 * HD)))
        eng.append(0, 0, 0, K, K)
        with pytest.raises(qkvlib.QkvError, match="not appended"):
            eng.attn_prefill(0, 0, 0, q, 64, 1 / 16, out)
        with pytest.raises(qkvlib.QkvError):
            eng.attn_prefill(0, 0, 0, q, 0, 1 / 16, out)
        with pytest.raises(qkvlib.QkvError):
            eng.attn_prefill(0, 0, 0, q, 5000, 1 / 16, out)
        eng.attn_prefill(0, 0, 0, q, 32, 1 / 16, out)
        torch.cuda.synchronize()
        assert eng.device_status() == 0


def test_prefill_group_of_sixteen(oracle, qkvlib):
    # 16 q-heads per KV head: tiles of 8 tokens x 16 heads
    got, ref = run_prefill(oracle, qkvlib, n_kv=700, pos0=290, Tc=410, seed=27, n_head=16, n_head_kv=1)
    assert_close(got, ref, "G=16")


def test_prefill_one_head_per_kv_head(oracle, qkvlib):
    # G = 1: tiles of 128 tokens of one head
    got, ref = run_prefill(oracle, qkvlib, n_kv=900, pos0=500, Tc=400, seed=28, n_head=2, n_head_kv=2)
    assert_close(got, ref, "G=1")


@pytest.mark.parametrize("n_kv", [256, 257, 384])
def test_prefill_single_query_at_boundaries(oracle, qkvlib, n_kv):
    # one query token whose position ends a page, starts one, or ends a 128-key tile
    got, ref = run_prefill(oracle, qkvlib, n_kv=n_kv, pos0=n_kv - 1, Tc=1, seed=29 + n_kv)
    assert_close(got, ref, f"Tc=1 at {n_kv - 1}")
