"""The multi-GPU path's host logic as world_size-2 `gloo` ranks on the CPU.

Independent sequences are sharded across GPUs by slot with no collective on the data path: every
rank computes the same longest-processing-time assignment (qkv_shard_lpt) from the context
lengths, serves only its own sequences from its own engine, and the only collectives are the
timing/throughput reductions the benchmark does after the timed region (max of step times, sum of
bytes).  A rank that leaves between steps must make the others fail within the process-group
timeout instead of hanging.  Engines here are host-only (device < 0): page bookkeeping only.
"""
from __future__ import annotations

import multiprocessing as mp
import os
import socket
import sys
import time
from datetime import timedelta

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WS = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, port: int, timeout_s: float):
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=WS, timeout=timedelta(seconds=timeout_s))
    return dist


def _shard_worker(rank: int, port: int, q) -> None:
    try:
        dist = _init(rank, port, 60)
        import torch
        import bench
        import qwfn_hybrid_b200 as Q
        ctx = bench.config5_contexts()
        owner = Q.shard_lpt(ctx, WS)
        mine = [i for i, o in enumerate(owner) if o == rank]
        pages = sum((ctx[i] + 255) // 256 for i in mine)
        eng = Q.Engine(n_layer=12, n_head=16, n_head_kv=2, n_ctx=max(ctx[i] for i in mine) + 1,
                       n_slots=len(mine), n_pages=pages, device=-1)
        for s, i in enumerate(mine):
            eng.seq_alloc(s)
            eng.reserve(s, ctx[i])
        used = pages - eng.pages_free()
        kv_bytes = sum(ctx[i] for i in mine) * 12 * 2 * 544
        owners = [None] * WS
        shards = [None] * WS
        dist.all_gather_object(owners, owner)
        dist.all_gather_object(shards, mine)
        # the benchmark's reductions: max over ranks of the step time, sum of bytes
        t = torch.tensor([1.5 * (rank + 1)])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        b = torch.tensor([float(kv_bytes)], dtype=torch.float64)
        dist.all_reduce(b, op=dist.ReduceOp.SUM)
        eng.close()
        dist.destroy_process_group()
        q.put((rank, owners, shards, used, pages, t.item(), b.item(), kv_bytes, None))
    except Exception as e:   # reported to the parent, which fails the test
        q.put((rank, None, None, 0, 0, 0.0, 0.0, 0, repr(e)))


def _leaving_worker(rank: int, port: int, q) -> None:
    try:
        dist = _init(rank, port, 10)
        dist.barrier()                      # step 1: both ranks
        if rank == 1:
            os._exit(0)                     # leaves between steps, nothing in flight
        t0 = time.monotonic()
        try:
            dist.barrier()                  # step 2: the peer is gone
            q.put((rank, "completed", time.monotonic() - t0))
        except Exception as e:
            q.put((rank, type(e).__name__, time.monotonic() - t0))
    except Exception as e:
        q.put((rank, "setup: " + repr(e), 0.0))


def _run(target, timeout: float):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, port, q)) for r in range(WS)]
    for p in procs:
        p.start()
    out = []
    deadline = time.monotonic() + timeout
    try:
        while len(out) < WS and time.monotonic() < deadline:
            try:
                out.append(q.get(timeout=max(0.1, deadline - time.monotonic())))
            except Exception:
                break
            if target is _leaving_worker and out and out[-1][0] == 0:
                break
    finally:
        for p in procs:
            p.join(timeout=5)
            if p.is_alive():
                p.kill()
                p.join()
    return sorted(out, key=lambda r: r[0])


def test_sequence_shards_cover_all_and_balance(qkvlib):
    res = _run(_shard_worker, 180)
    assert len(res) == WS, res
    for r in res:
        assert r[8] is None, r[8]
    (_, owners0, shards0, *_), (_, owners1, shards1, *_) = res
    assert owners0 == owners1 and owners0[0] == owners0[1]          # every rank planned the same
    assert shards0 == shards1
    covered = sorted(i for s in shards0 for i in s)
    assert covered == list(range(64))                                # each sequence on exactly one rank
    import bench
    ctx = bench.config5_contexts()
    loads = [sum(ctx[i] for i in s) for s in shards0]
    assert max(loads) <= 1.05 * sum(loads) / WS                      # LPT balance on 64 ragged contexts
    for rank, _, shards, used, pages, tmax, bsum, kv, _err in res:
        assert used == pages                                         # own sequences' pages only
        assert tmax == 1.5 * WS                                      # max over ranks
        assert bsum == pytest.approx(sum(ctx) * 12 * 2 * 544)        # sum over ranks = whole job


def test_rank_leaving_between_steps_fails_the_others_without_hanging():
    res = _run(_leaving_worker, 120)
    assert res and res[0][0] == 0, res
    rank, outcome, waited = res[0]
    assert outcome != "completed" and not outcome.startswith("setup"), res
    assert waited < 60, res
