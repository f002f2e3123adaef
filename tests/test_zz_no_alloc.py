"""The allocation-free decode entry point (qkv_attn_decode_static) against qkv_attn_decode.

It serves callers that cannot allocate device memory, such as a custom op running inside ggml's
graph executor, whose memory is planned ahead and may not grow during the graph.  Its split-K
scratch is a fixed array compiled into the library.  This file is collected last on purpose: if it
fails, a run that stops at the first failure has already run every other test.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from helpers import HD, append_rows, assert_close, engine, normal, to_dev

pytestmark = pytest.mark.gpu


def static_decode(qkvlib, eng, layer, n_slots, slots, pos0, Q, T, n_head, out):
    import torch
    L = qkvlib.lib()
    fn = L.qkv_attn_decode_static
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(qkvlib.QkvCacheView), ctypes.c_int32, ctypes.POINTER(ctypes.c_int32),
                   ctypes.POINTER(ctypes.c_int32), ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int32,
                   ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p]
    view = eng.cache_view(layer)
    s = (ctypes.c_int32 * len(slots))(*slots)
    p = (ctypes.c_int32 * len(pos0))(*pos0)
    return fn(ctypes.byref(view), n_slots, s, p, len(slots), n_head, Q.data_ptr(), T, 1 / 16, out.data_ptr(),
              torch.cuda.current_stream().cuda_stream)


def test_static_decode_matches_engine_decode_twice(cuda, qkvlib):
    import torch
    lens, T = [20000, 3000, 129, 5], 3
    eng = engine(qkvlib, n_slots=4, n_ctx=20480)
    for i, n in enumerate(lens):
        eng.seq_alloc(i)
        append_rows(eng, 0, i, 0, normal(900 + i, (n, 512)), normal(950 + i, (n, 512)))
    q = to_dev(normal(77, (len(lens), T, 16, HD)))
    ref = torch.empty_like(q)
    eng.attn_decode(0, list(range(len(lens))), [n - T for n in lens], q, T, 1 / 16, ref)
    torch.cuda.synchronize()
    ref = ref.cpu().numpy()
    for call in range(2):   # the shared scratch keeps the previous call's contents
        out = torch.full_like(q, float("nan"))
        st = static_decode(qkvlib, eng, 0, 4, list(range(len(lens))), [n - T for n in lens], q, T, 16, out)
        assert st == qkvlib.OK, st
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), ref, f"static decode, call {call}")


def test_static_decode_rejects_oversized_groups(cuda, qkvlib):
    import torch
    eng = engine(qkvlib, n_head=24, n_slots=1)
    eng.seq_alloc(0)
    append_rows(eng, 0, 0, 0, normal(1, (100, 512)), normal(2, (100, 512)))
    q = to_dev(normal(3, (1, 3, 24, HD)))   # 3 * 24 / 2 = 36 query rows per KV head > 32
    out = torch.empty_like(q)
    assert static_decode(qkvlib, eng, 0, 1, [0], [97], q, 3, 24, out) == qkvlib.ERR_UNSUPPORTED
    assert static_decode(qkvlib, eng, 0, 1, [1], [0], q[:, :1].contiguous(), 1, 24, out) == qkvlib.ERR_INVALID


def static_status(qkvlib):
    import torch
    code = ctypes.c_int32(-1)
    st = qkvlib.lib().qkv_static_status(torch.cuda.current_stream().cuda_stream, ctypes.byref(code))
    return st, code.value


@pytest.mark.parametrize("lens", [[16000], [300 + 41 * i for i in range(70)]],
                         ids=["one-long-sequence", "70-sequences"])
def test_static_decode_both_modes_twice(cuda, qkvlib, lens):
    """One long sequence: its pairs split into many units, merged by the long-pair merge kernel.
    70 short ones: two launches (at most 64 sequences per launch, so the second offsets Q and the
    output and renumbers its sequences) whose pairs have a few units each, merged by the row
    merge kernel."""
    import torch
    T = 3
    eng = engine(qkvlib, n_slots=len(lens), n_ctx=16384)
    for i, n in enumerate(lens):
        eng.seq_alloc(i)
        append_rows(eng, 0, i, 0, normal(1200 + i, (n, 512)), normal(1300 + i, (n, 512)))
    q = to_dev(normal(78, (len(lens), T, 16, HD)))
    pos = [n - T for n in lens]
    ref = torch.empty_like(q)
    eng.attn_decode(0, list(range(len(lens))), pos, q, T, 1 / 16, ref)
    torch.cuda.synchronize()
    ref = ref.cpu().numpy()
    for call in range(2):
        out = torch.full_like(q, float("nan"))
        st = static_decode(qkvlib, eng, 0, len(lens), list(range(len(lens))), pos, q, T, 16, out)
        assert st == qkvlib.OK, st
        assert static_status(qkvlib) == (qkvlib.OK, 0)
        assert_close(out.cpu().numpy(), ref, f"static decode, call {call}")


def test_static_status_reports_a_bad_page(cuda, qkvlib):
    """A block table entry outside the pool is skipped by the kernel and reported through
    qkv_static_status (bit 1), which also clears the word."""
    import torch
    eng = engine(qkvlib, n_slots=1)
    eng.seq_alloc(0)
    append_rows(eng, 0, 0, 0, normal(5, (300, 512)), normal(6, (300, 512)))
    view = eng.cache_view(0)
    bt = torch.full((1, view.max_pages_per_seq), -1, dtype=torch.int32, device="cuda")
    bt[0, 0] = eng.pages(0)[0]
    bt[0, 1] = view.n_pages + 7                     # not a page of the pool
    view.block_table = bt.data_ptr()
    q = to_dev(normal(7, (1, 1, 16, HD)))
    out = torch.empty_like(q)
    L = qkvlib.lib()
    s, p = (ctypes.c_int32 * 1)(0), (ctypes.c_int32 * 1)(299)
    st = L.qkv_attn_decode_static(ctypes.byref(view), 1, s, p, 1, 16, q.data_ptr(), 1, ctypes.c_float(1 / 16),
                                  out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == qkvlib.OK
    assert static_status(qkvlib) == (qkvlib.ERR_DEVICE, 1)
    assert static_status(qkvlib) == (qkvlib.OK, 0)
