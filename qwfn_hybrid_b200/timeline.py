"""Per-CTA phase timelines of the decode and projection kernels (analysis tool, not the product).

    python -m qwfn_hybrid_b200.build --timeline         # libqkv_timeline.so (-DQKV_TIMELINE)
    python -m qwfn_hybrid_b200.timeline decode           # configs[1]'s layer: 12 layers, T = 3, ctx 16384
    python -m qwfn_hybrid_b200.timeline proj             # qkv_project_append, 12 layers, T = 3
    python -m qwfn_hybrid_b200.timeline prefill          # configs[2]'s last chunk (kernel D roles)

In the timeline build, thread 0 of every CTA notes %globaltimer at fixed points of its kernel and
appends one record per CTA; this tool replays a CUDA graph of the workload once, reads the records
and prints, per kernel, the median (and max) of each phase relative to the launch's earliest
return from griddepcontrol.wait (decode, merge) or its earliest CTA entry (projection), in ns.

Decode phases: 0 entry, 1 dependency wait returned, 9 the sequence's position read, 6 first tile
copies issued, 18 / 19 thread 0's first / all query values arrived, 7 query rows rounded (warp 0),
2 rows in shared memory (CTA barrier), 8 first tile landed, 10-13 first tile: QK done, P barrier,
after the reference move, PV done; 3 first tile finished; 14-17 the same for the second tile; 4 all
tiles done; 5 partial record written.  Merge phases: 0 entry, 1 wait returned, 2 output written.
Projection phases: 0 entry, 1 x staged, 2 dot products done, 3 the cluster's normalised dims
posted (after its second barrier), 4 the CTA's epilogue done (every CTA: each holds 32 dims of
the head).
Prefill: per-role phase durations of kernel D (see `prefill`).
"""
from __future__ import annotations

import ctypes
import os
import statistics
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _engine_lib():
    import qwfn_hybrid_b200 as Q
    from qwfn_hybrid_b200 import build
    Q.LIB_PATH = build.LIB_TL
    if not os.path.exists(Q.LIB_PATH):
        raise SystemExit("libqkv_timeline.so missing: python -m qwfn_hybrid_b200.build --timeline")
    return Q, Q.lib()


def decode(steps: int = 4) -> None:
    import torch
    Q, L = _engine_lib()
    L.qkv_tl_read.argtypes = [ctypes.c_void_p, ctypes.c_int]
    L.qkv_tl_read.restype = ctypes.c_int
    NL, T, CTX = 12, 3, 16384
    dev = torch.device("cuda", 0)
    eng = Q.Engine(n_layer=NL, n_head=16, n_head_kv=2, n_ctx=CTX + T * (steps + 4), n_slots=1, device=0)
    gen = torch.Generator(device=dev).manual_seed(1)
    eng.seq_alloc(0)
    for layer in range(NL):
        eng.append(layer, 0, 0, torch.randn(CTX, 512, generator=gen, device=dev), torch.randn(CTX, 512, generator=gen, device=dev))
    eng.reserve(0, CTX + T * steps)
    Qd = torch.randn(steps, NL, 1, T, 16, 256, generator=gen, device=dev)
    Kd = torch.randn(steps, NL, 1, T, 512, generator=gen, device=dev)
    Vd = torch.randn(steps, NL, 1, T, 512, generator=gen, device=dev)
    out = torch.empty(NL, 1, T, 16, 256, device=dev)

    def step(i):
        for layer in range(NL):
            eng.append_attn_decode(layer, [0], [CTX + T * i], Kd[i, layer], Vd[i, layer], Qd[i, layer], T, 1 / 16, out[layer])

    for i in range(steps):
        step(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(steps):
            step(i)
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    buf = np.zeros((1 << 16, 22), dtype=np.uint64)
    L.qkv_tl_read(buf.ctypes.data, 1 << 16)   # drop the warm-up records
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    n = L.qkv_tl_read(buf.ctypes.data, 1 << 16)
    launches = steps * NL
    print(f"decode: {e0.elapsed_time(e1) * 1e3 / launches:.2f} us per layer (decode + merge launch), {n} CTA records")
    rec = buf[:n].astype(np.int64)
    names = {2: "decode", 3: "merge", 4: "merge_rows"}
    groups = []
    for kid in sorted(set(rec[:, 0].tolist())):
        r = rec[rec[:, 0] == kid]
        per = len(r) // launches
        r = r[np.argsort(r[:, 3])]
        groups += [(kid, r[k * per:(k + 1) * per]) for k in range(launches)]
    groups.sort(key=lambda x: x[1][:, 3].min())
    rows = []
    for kid, r in groups:
        t1 = r[:, 3].min()
        d = {"kernel": names.get(kid, str(kid)), "ctas": len(r)}
        for ph in range(20):
            v = r[:, 2 + ph]
            v = v[v > 0]
            if len(v):
                d[ph] = (statistics.median((v - t1).tolist()), int((v - t1).max()))
        rows.append(d)
    mid = rows[len(rows) // 3: 2 * len(rows) // 3]   # launches away from the graph's ends
    for kname in sorted(set(x["kernel"] for x in mid)):
        xs = [x for x in mid if x["kernel"] == kname]
        phases = sorted(k for k in xs[0] if isinstance(k, int))
        cells = [f"{ph}: {statistics.median([x[ph][0] for x in xs if ph in x]):.0f}/"
                 f"{statistics.median([x[ph][1] for x in xs if ph in x]):.0f}" for ph in phases]
        print(f"{kname} ({xs[0]['ctas']} CTAs) phase: median/max ns -> " + ", ".join(cells))


def proj() -> None:
    import torch
    Q, L = _engine_lib()
    L.qkv_tl_read_k.argtypes = [ctypes.c_void_p, ctypes.c_int]
    L.qkv_tl_read_k.restype = ctypes.c_int
    NL, T, E = 12, 3, 2560
    dev = torch.device("cuda", 0)
    eng = Q.Engine(n_layer=NL, n_head=16, n_head_kv=2, n_ctx=4096, n_slots=1, device=0)
    eng.seq_alloc(0)
    eng.reserve(0, 4096)
    gen = torch.Generator(device=dev).manual_seed(7)
    s = E ** -0.5
    W = [[(torch.randn(rows, E, generator=gen, device=dev) * s).to(torch.bfloat16).view(torch.int16) for _ in range(NL)]
         for rows in (2 * 16 * 256, 2 * 256, 2 * 256)]
    qn, kn = torch.ones(256, device=dev), torch.ones(256, device=dev)
    X = torch.randn(NL, T, E, generator=gen, device=dev)
    Qo = torch.empty(NL, T, 16, 256, device=dev)

    def step():
        for layer in range(NL):
            eng.project_append(layer, 0, 0, X[layer], W[0][layer], W[1][layer], W[2][layer], qn, kn, Qo[layer])

    step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    g.replay()
    torch.cuda.synchronize()
    buf = np.zeros((1 << 14, 8), dtype=np.uint64)
    L.qkv_tl_read_k(buf.ctypes.data, 1 << 14)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    n = L.qkv_tl_read_k(buf.ctypes.data, 1 << 14)
    print(f"proj: {e0.elapsed_time(e1) * 1e3 / NL:.2f} us per layer, {n} CTA records")
    rec = buf[:n].astype(np.int64)
    rec = rec[np.argsort(rec[:, 2])]
    per = n // NL
    for layer in range(NL):
        r = rec[layer * per:(layer + 1) * per]
        t0 = r[:, 2].min()
        last = r[r[:, 6] > 0]
        cells = [f"{ph}: {statistics.median((r[:, 2 + ph] - t0).tolist()):.0f}/{int((r[:, 2 + ph] - t0).max())}" for ph in (1, 2, 3)]
        if len(last):
            cells.append(f"4: {statistics.median((last[:, 6] - t0).tolist()):.0f}/{int((last[:, 6] - t0).max())}")
        print(f"layer {layer} ({len(r)} CTAs) phase: median/max ns -> " + ", ".join(cells))


def prefill(chunk: int = 31) -> None:
    """configs[2]'s chunk `chunk` (512 queries at 512 chunk .. over the 16384 cached keys), called
    eagerly; the table of the last call.  Per role, the median over CTAs of each phase's duration
    in ns, for the first KV tiles of each CTA."""
    import torch
    Q, L = _engine_lib()
    L.qkv_pf_tl_read.argtypes = [ctypes.c_void_p, ctypes.c_int]
    L.qkv_pf_tl_read.restype = ctypes.c_int
    N, C = 16384, 512
    dev = torch.device("cuda", 0)
    eng = Q.Engine(n_layer=1, n_head=16, n_head_kv=2, n_ctx=N, n_slots=1, device=0)
    eng.seq_alloc(0)
    gen = torch.Generator(device=dev).manual_seed(2)
    eng.append(0, 0, 0, torch.randn(N, 512, generator=gen, device=dev), torch.randn(N, 512, generator=gen, device=dev))
    Qb = torch.randn(C, 16, 256, generator=gen, device=dev).to(torch.bfloat16).view(torch.int16)
    out = torch.empty(C, 16, 256, device=dev)
    a = chunk * C
    for _ in range(5):
        eng.attn_prefill(0, 0, a, Qb, C, 1 / 16, out)
    torch.cuda.synchronize()
    n = L.qkv_pf_tl_read(None, 1)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    eng.attn_prefill(0, 0, a, Qb, C, 1 / 16, out)
    e1.record()
    torch.cuda.synchronize()
    buf = np.zeros(n, dtype=np.uint64)
    L.qkv_pf_tl_read(buf.ctypes.data, 0)
    tl = buf.reshape(-1, 5, 16, 6).astype(np.int64)
    print(f"prefill chunk {chunk}: {e0.elapsed_time(e1) * 1e3:.1f} us for the call (3 launches, eager)")

    def med(x):
        x = [v for v in x if v is not None]
        return f"{statistics.median(x):6.0f}" if x else "     -"

    def dur(role, k, p1, k2, p2, rank=None):   # per-CTA durations: stamp (k2, p2) - stamp (k, p1)
        out = []
        for c in range(tl.shape[0]):
            if rank is not None and c % 2 != rank:
                continue
            a, b = tl[c, role, k, p1], tl[c, role, k2, p2]
            out.append(int(b - a) if a > 0 and b > 0 else None)
        return out

    names = ["max pass", "exchange", "P pass", "rescale+st", "arrive", "to next S"]
    for role in (0, 1):
        for rank in (0, 1):
            print(f"softmax half {role}, {('leader', 'follower')[rank]} CTAs: per KV tile j, ns: " + " | ".join(names) + " | period")
            for k in range(15):
                cells = [med(dur(role, k, i, k, i + 1, rank)) for i in range(5)] + \
                        [med(dur(role, k, 5, k + 1, 0, rank)), med(dur(role, k, 0, k + 1, 0, rank))]
                print(f"  j={k:2d} " + " ".join(cells))
    print("MMA issue (leader): per KV tile j, ns: K slot + S_j issue | p_full(j-1) + V slot + PV_{j-1} issue | period")
    for k in range(15):
        print(f"  j={k:2d} {med(dur(2, k, 0, k, 1))} {med(dur(2, k, 1, k, 2))} {med(dur(2, k, 0, k + 1, 0))}")
    for role, nm in ((3, "K"), (4, "V")):
        print(f"{nm} producers: per KV tile j, ns: slot free wait | dequantise + store + arrive | period")
        for u in range(15):
            print(f"  j={u:2d} {med(dur(role, u, 0, u, 1))} {med(dur(role, u, 1, u, 2))} {med(dur(role, u, 0, u + 1, 0))}")

if __name__ == "__main__":
    what = sys.argv[1] if len(sys.argv) > 1 else "decode"
    {"decode": decode, "proj": proj, "prefill": prefill}[what]()
