"""Helpers shared by the GPU parity tests: seeded inputs, engine setup, oracle comparisons."""
from __future__ import annotations

import numpy as np

HD = 256
ROW = 272          # ggml q8_0 bytes per head row
ATOL, RTOL = 2e-3, 1e-3   # attention tolerance


def normal(seed: int, shape, scale: float = 1.0) -> np.ndarray:
    return (np.random.default_rng(seed).standard_normal(shape, dtype=np.float32) * np.float32(scale)).astype(np.float32)


def to_dev(a: np.ndarray):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def engine(qkvlib, **kw):
    args = dict(n_layer=1, n_head=16, n_head_kv=2, n_ctx=8192, n_slots=4, device=0)
    args.update(kw)
    return qkvlib.Engine(**args)


def append_rows(eng, layer: int, slot: int, pos: int, Kf: np.ndarray, Vf: np.ndarray, chunk: int = 4096):
    for s in range(0, Kf.shape[0], chunk):
        k, v = to_dev(Kf[s:s + chunk]), to_dev(Vf[s:s + chunk])
        eng.append(layer, slot, pos + s, k, v)


def read_rows(eng, layer: int, slot: int, pos: int, n: int, n_head_kv: int = 2):
    import torch
    K = torch.empty((n, n_head_kv * ROW), dtype=torch.uint8, device="cuda")
    V = torch.empty_like(K)
    eng.read_rows(layer, slot, pos, n, K, V)
    torch.cuda.synchronize()
    return K.cpu().numpy(), V.cpu().numpy()


def decode(eng, layer: int, slots, pos0, Q: np.ndarray, T: int, scale: float = 1 / 16, sel=None, n_sel: int = 0):
    import torch
    q = to_dev(Q)
    out = torch.empty_like(q)
    eng.attn_decode(layer, slots, pos0, q, T, scale, out, sel=sel, n_sel=n_sel)
    torch.cuda.synchronize()
    assert eng.device_status() == 0
    return out.cpu().numpy()


def assert_close(got: np.ndarray, ref: np.ndarray, what: str = ""):
    err = np.abs(got - ref)
    bound = ATOL + RTOL * np.abs(ref)
    bad = err > bound
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {bad.size} outside atol {ATOL} + rtol {RTOL}; "
                           f"max err {err.max():.3e}")
