"""GPU: the fused projection + rms-norm + rope + q8_0 append (qkv_project_append) against the CPU
oracle: query outputs and the stored q8_0 K/V bytes bit-exact (graph_builder::qsa_dec_qkv and
qsa_dec_kv_write, src/qwfn_graph.cpp:582-628)."""
from __future__ import annotations

import numpy as np
import pytest

from helpers import append_rows, engine, normal, read_rows, to_dev
from test_oracle_project import bf16_bits

pytestmark = pytest.mark.gpu

N_EMBD = 2560


def weights(seed, n_head=16, n_head_kv=2, n_embd=N_EMBD):
    r = np.random.default_rng(seed)
    s = 1 / np.sqrt(n_embd)
    Wq = bf16_bits(r.standard_normal((2 * n_head * 256, n_embd), dtype=np.float32) * s)
    Wk = bf16_bits(r.standard_normal((n_head_kv * 256, n_embd), dtype=np.float32) * s)
    Wv = bf16_bits(r.standard_normal((n_head_kv * 256, n_embd), dtype=np.float32) * s)
    qn = (1 + 0.1 * r.standard_normal(256)).astype(np.float32)
    kn = (1 + 0.1 * r.standard_normal(256)).astype(np.float32)
    return Wq, Wk, Wv, qn, kn


def dev16(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda()


@pytest.mark.parametrize("T,pos,with_q,n_embd", [(3, 100, True, N_EMBD), (1, 0, False, N_EMBD), (4, 254, True, N_EMBD),
                                                 (4, 17, True, 3072)])   # the last: T x n_embd at its limit
def test_project_append_bit_exact(cuda, qkvlib, oracle, T, pos, with_q, n_embd):
    import torch
    eng = engine(qkvlib, n_layer=2, n_ctx=1024, n_slots=1)
    eng.seq_alloc(0)
    if pos:
        append_rows(eng, 1, 0, 0, normal(90, (pos, 512)), normal(91, (pos, 512)))
    Wq, Wk, Wv, qn, kn = weights(92 + T, n_embd=n_embd)
    x = normal(93 + T, (T, n_embd))
    Qout = torch.full((T, 16, 256), float("nan"), device="cuda") if with_q else None
    eng.project_append(1, 0, pos, to_dev(x), dev16(Wq) if with_q else None, dev16(Wk), dev16(Wv),
                       to_dev(qn) if with_q else None, to_dev(kn), Qout)
    torch.cuda.synchronize()
    assert eng.device_status() == 0 and eng.n_past(0) == pos + T
    Q, K, V = oracle.project(x, Wq if with_q else None, Wk, Wv, 16, 2, qn if with_q else None, kn, 1e-6, 64, 1e7,
                             pos)
    kq, vq = read_rows(eng, 1, 0, pos, T)
    np.testing.assert_array_equal(kq, oracle.quantize_rows(K))
    np.testing.assert_array_equal(vq, oracle.quantize_rows(V))
    if with_q:
        np.testing.assert_array_equal(Qout.cpu().numpy(), Q)


def test_project_append_errors(cuda, qkvlib):
    import torch
    eng = engine(qkvlib, n_ctx=1024, n_slots=1)
    eng.seq_alloc(0)
    Wq, Wk, Wv, qn, kn = weights(99)
    for T, n_embd in ((5, N_EMBD), (2, 2500)):
        x = torch.zeros(T, n_embd, device="cuda")
        with pytest.raises(qkvlib.QkvError) as e:
            eng.project_append(0, 0, 0, x, None, dev16(Wk[:, :n_embd]), dev16(Wv[:, :n_embd]), None, to_dev(kn))
        assert e.value.status == qkvlib.ERR_INVALID
    with pytest.raises(qkvlib.QkvError) as e:           # beyond n_past
        eng.project_append(0, 0, 3, torch.zeros(1, N_EMBD, device="cuda"), None, dev16(Wk), dev16(Wv), None,
                           to_dev(kn))
    assert e.value.status == qkvlib.ERR_INVALID
