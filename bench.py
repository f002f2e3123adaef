#!/usr/bin/env python
"""Benchmark of the q8_0 KV-cache attention path (BASELINE.json configs[1] is the headline).

Headline ("step"): MTP-verify decode over 12 full-attention layers, 16 query heads / 2 KV heads /
head_dim 256, q8_0 KV at context 16384 growing by 3 per step; each layer appends the step's 3 K/V
rows and runs causal verify attention for 3 query tokens, in one fused launch (plus the split-K
merge).  Reported: tokens/s = 3 * steps / time, the median of 5 timed replays of one CUDA graph
holding the K steps.  Inputs are seeded N(0,1) synthetic data, the same numbers in both arms
(numpy SeedSequence(1)); the reference's model and prompts are not available.  The 215 MB of KV a
step reads exceeds the 126 MB L2, so no flush is needed between steps.

The same JSON line carries sub-records measured in the same run:
  "ragged"   configs[4] at every N: 64 sequences LPT-sharded over the ranks, restored from an
             8192-token shared-prefix snapshot, one 1-token decode over 12 layers per step
             (aggregate tokens/s, per-rank time and GB/s, imbalance, restore latency);
  "configs"  at N = 1: configs[0] (µs per decode step), configs[2] (chunked prefill, TFLOP/s) and
             configs[3] (select + sparse decode at 73,728, bit-exact indices), each with its CPU
             oracle timing.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload ...]

One process per GPU (torchrun for N > 1); sequences are independent, so there is no collective on
the data path.  `--impl reference` times the reference's CPU algorithm (the C restatement in
oracle/, since ggml itself cannot be built here) on this host's cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "q8_0-KV attention HBM GB/s & decode tokens/s at 16K–73K ctx, 1/2/4/8 B200"
N_LAYER, N_HEAD, N_HEAD_KV, HD, T = 12, 16, 2, 256, 3
CTX0 = 16384
SCALE = 1.0 / 16.0
ROW_BYTES = N_HEAD_KV * 272          # one q8_0 K (or V) row of all KV heads
KV_DIM = N_HEAD_KV * HD
REPLAYS = 5
CONFIG = {"workload": "configs[1]: MTP-verify decode, 12 layers, ctx 16384 (+3/step), T=3, 16q/2kv x 256, q8_0 KV",
          "global_batch": 1, "seq_len": CTX0, "query_tokens": T, "layers": N_LAYER,
          "l2": "inputs larger than L2 (215 MB of KV read per step vs 126 MB L2)"}
DATA = "synthetic N(0,1), numpy SeedSequence(1) (the same numbers in both arms); no model or prompts available"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="headline only: skip the ragged and configs sub-records")
    ap.add_argument("--workload", choices=["cfg2", "cfg1", "cfg3", "cfg4", "cfg5", "qsa", "proj", "append", "long"],
                    default="cfg2",
                    help="cfg2 (default, the headline line with its sub-records): BASELINE configs[1]; cfg1/cfg3/"
                         "cfg4/cfg5: configs[0]/[2]/[3]/[4] alone; qsa: configs[3]'s context and tokens through the "
                         "model's own lightning indexer (select + sparse attention over the kept blocks in place); proj: the fused decode "
                         "projections + norm + rope + q8_0 append of configs[1]'s step; append: kernel A alone; long: "
                         "configs[1]'s step for one sequence at ctx 73728")
    ap.add_argument("--seqs", type=int, default=64, help="cfg5: use the first N of the 64 sequences (profiling)")
    return ap.parse_args()


# ----------------------------------------------------------------------------- clocks sampler
class Clocks:
    FIELDS = ["index", "clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.active",
              "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
              "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.lines: list[str] = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={','.join(self.FIELDS)}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- distributed
def dist_init(backend: str):
    import torch.distributed as dist
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    # NCCL's own messages (its version line among them) go to stderr: stdout carries only the JSON line
    os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
    if ws > 1 and not dist.is_initialized():
        from datetime import timedelta
        dist.init_process_group(backend=backend, timeout=timedelta(seconds=180))
    return int(os.environ.get("RANK", "0")), ws, int(os.environ.get("LOCAL_RANK", "0"))


# ----------------------------------------------------------------------------- shared helpers
def host_threads() -> int:
    """Cores this process may run on (torchrun sets OMP_NUM_THREADS=1; the CPU arms ignore it)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def peaks() -> dict:
    pk = os.path.join(ROOT, "MEASURED_PEAKS.json")
    p = json.load(open(pk)) if os.path.exists(pk) else {}
    out = {"hbm": p.get("hbm_gbs") or 6650.0, "bf16": p.get("bf16_tflops") or 1590.0}
    out["hbm_src"] = "measured (MEASURED_PEAKS.json hbm_gbs)" if p.get("hbm_gbs") else "fallback 6650 GB/s"
    out["bf16_src"] = "measured (MEASURED_PEAKS.json bf16_tflops, burst)" if p.get("bf16_tflops") else \
        "fallback 1590 TFLOP/s"
    return out


def _normals(seed_seq, shape):
    import numpy as np
    return np.random.default_rng(seed_seq).standard_normal(shape, dtype=np.float32)


def cfg2_host_data(n_steps: int):
    """configs[1]'s inputs, seed 1: the 16384-row K and V prefix of every layer (one child stream
    each, generated in parallel) and, from the last child, every step's Q, new K and new V."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor
    ss = np.random.SeedSequence(1).spawn(2 * N_LAYER + 1)
    with ThreadPoolExecutor(max(1, min(2 * N_LAYER, host_threads()))) as ex:
        prefix = list(ex.map(lambda s: _normals(s, (CTX0, KV_DIM)), ss[:2 * N_LAYER]))
    r = np.random.default_rng(ss[-1])
    Qs = r.standard_normal((n_steps, N_LAYER, T, N_HEAD, HD), dtype=np.float32)
    Ks = r.standard_normal((n_steps, N_LAYER, T, KV_DIM), dtype=np.float32)
    Vs = r.standard_normal((n_steps, N_LAYER, T, KV_DIM), dtype=np.float32)
    return [(prefix[2 * l], prefix[2 * l + 1]) for l in range(N_LAYER)], Qs, Ks, Vs


# ----------------------------------------------------------------------------- CPU arms (oracle)
class CpuConfig2:
    """configs[1] on the host's cores through the oracle: q8_0 caches of 12 layers in ggml's row
    layout; a step quantises and writes the 3 new rows of every layer, then runs the 3-token verify."""

    def __init__(self, prefix, Qs, Ks, Vs, threads: int):
        import numpy as np
        from oracle import oracle as O
        O.build()
        self.O, self.threads = O, threads
        n = CTX0 + T * Qs.shape[0]
        self.layers = []
        for Kf, Vf in prefix:
            K = np.zeros((n, ROW_BYTES), np.uint8)
            V = np.zeros((n, ROW_BYTES), np.uint8)
            K[:CTX0] = O.quantize_rows(Kf, threads)
            V[:CTX0] = O.quantize_rows(Vf, threads)
            self.layers.append((K, V))
        self.Qs, self.Ks, self.Vs = Qs, Ks, Vs

    def step(self, i: int):
        import numpy as np
        n0 = CTX0 + T * i
        for l, (K, V) in enumerate(self.layers):
            K[n0:n0 + T] = self.O.quantize_rows(self.Ks[i, l], self.threads)
            V[n0:n0 + T] = self.O.quantize_rows(self.Vs[i, l], self.threads)
            self.O.attn(self.Qs[i, l], K, V, np.arange(n0, n0 + T, dtype=np.int32), N_HEAD_KV, SCALE,
                        n_cells=n0 + T, threads=self.threads)

    def timed(self, first: int, steps: int) -> list[float]:
        times = []
        for i in range(first, first + steps):
            t0 = time.perf_counter()
            self.step(i)
            times.append(time.perf_counter() - t0)
        return times


def run_reference(args) -> None:
    # the CPU arm needs no process group: rank 0 measures, the other ranks have nothing to do
    if int(os.environ.get("RANK", "0")) != 0:
        return
    threads = host_threads()
    total = args.warmup + args.steps
    cpu = CpuConfig2(*cfg2_host_data(total), threads=threads)
    for i in range(args.warmup):
        cpu.step(i)
    times = cpu.timed(args.warmup, args.steps)
    total_s = sum(times)
    value = T * args.steps / total_s
    sample = (f"every step is a full config-2 step: 12 layers, each quantising 3 K/V rows to q8_0 and running "
              f"3-token causal verify attention at ctx {CTX0}+3*step; oracle/qkv_oracle.c (the reference's ggml CPU "
              f"flash_attn_ext + quantize_row_q8_0 restated; ggml itself is not buildable here), OpenMP with "
              f"{threads} threads (the process's CPU affinity)")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total_s / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 dot + f32 softmax/accumulate",
        "data": DATA, "config": CONFIG,
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ----------------------------------------------------------------------------- our arm: configs[1]
def load_traffic() -> tuple[float | None, str | None]:
    """DRAM bytes per decode launch from the committed ncu summary, if present."""
    path = os.path.join(ROOT, "profiles", "decode_cfg2_ncu.md")
    if not os.path.exists(path):
        return None, None
    for line in open(path):
        if line.startswith("dram_bytes_per_launch:"):
            return float(line.split(":")[1].split()[0]), os.path.relpath(path, ROOT)
    return None, None


def _barrier(ws: int, local: int):
    import torch
    if ws > 1:
        torch.distributed.barrier(device_ids=[local])


def _max_over_ranks(ws: int, dev, values: list[float]) -> list[float]:
    import torch
    if ws == 1:
        return values
    t = torch.tensor(values, device=dev, dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return t.tolist()


def _gather(ws: int, dev, values: list[float]) -> list[list[float]]:
    """Every rank's `values` (same length on all ranks), in rank order."""
    import torch
    if ws == 1:
        return [values]
    t = torch.tensor(values, device=dev, dtype=torch.float64)
    out = [torch.empty_like(t) for _ in range(ws)]
    torch.distributed.all_gather(out, t)
    return [o.tolist() for o in out]


def measure_cfg2(args, rank: int, ws: int, local: int) -> dict:
    import numpy as np
    import torch
    import qwfn_hybrid_b200 as Q
    from oracle import oracle as O
    dev = torch.device("cuda", local)
    steps, warm = args.steps, args.warmup
    total_steps = warm + steps
    prefix, Qs, Ks, Vs = cfg2_host_data(total_steps)
    n_ctx = CTX0 + T * (total_steps + 8)
    eng = Q.Engine(n_layer=N_LAYER, n_head=N_HEAD, n_head_kv=N_HEAD_KV, n_ctx=n_ctx, n_slots=1, device=local)
    eng.seq_alloc(0)
    for l, (Kf, Vf) in enumerate(prefix):
        eng.append(l, 0, 0, torch.from_numpy(Kf).to(dev), torch.from_numpy(Vf).to(dev))
    torch.cuda.synchronize()
    snap = eng.snapshot_save(0)                  # the 16384-token prefix, restored for the e2e pass
    eng.reserve(0, CTX0 + T * total_steps)       # pages for every step: no host uploads while timing
    Qd, Kd, Vd = (torch.from_numpy(a).to(dev) for a in (Qs, Ks, Vs))
    out = torch.empty(N_LAYER, T, N_HEAD, HD, device=dev)

    def step(i: int):
        """One config-2 step: per layer one launch that appends the 3 rows and runs the verify attention."""
        n0 = CTX0 + T * i
        for l in range(N_LAYER):
            eng.append_attn_decode(l, [0], [n0], Kd[i, l], Vd[i, l], Qd[i, l], T, SCALE, out[l])

    for i in range(warm):
        step(i)
    torch.cuda.synchronize()
    # The K timed steps, captured once as a CUDA graph (the kernels of every layer and step).
    graph = torch.cuda.CUDAGraph()
    launches0 = Q.launch_count()
    with torch.cuda.graph(graph):
        for i in range(warm, total_steps):
            step(i)
    launches = Q.launch_count() - launches0
    graph.replay()                               # untimed: the same steps, same bytes
    torch.cuda.synchronize()
    _barrier(ws, local)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    clocks = Clocks(local)
    clocks.start()
    region_ms = []
    for _ in range(REPLAYS):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        region_ms.append(e0.elapsed_time(e1))
    _barrier(ws, local)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = statistics.median(region_ms)
    if eng.device_status() != 0:
        raise RuntimeError("device status reported a bounds violation")
    del graph
    # ---- parity of the timed path: the last step's first and last layer against the oracle ----
    last = total_steps - 1
    n0 = CTX0 + T * last
    outh = out.cpu().numpy()
    parity = {"checked": "layers 0 and 11 of the last timed step (appended q8_0 rows bit-exact; attention vs "
                         "oracle/qkv_oracle.c)", "atol": 2e-3, "rtol": 1e-3}
    max_abs, ok = 0.0, True
    for l in (0, N_LAYER - 1):
        Kr = torch.empty((n0 + T, ROW_BYTES), dtype=torch.uint8, device=dev)
        Vr = torch.empty_like(Kr)
        eng.read_rows(l, 0, 0, n0 + T, Kr, Vr)
        torch.cuda.synchronize()
        Kh, Vh = Kr.cpu().numpy(), Vr.cpu().numpy()
        rows_ok = bool(np.array_equal(Kh[n0:], O.quantize_rows(Ks[last, l])) and
                       np.array_equal(Vh[n0:], O.quantize_rows(Vs[last, l])))
        ref = O.attn(Qs[last, l], Kh, Vh, np.arange(n0, n0 + T, dtype=np.int32), N_HEAD_KV, SCALE,
                     threads=host_threads())
        err = np.abs(outh[l] - ref)
        max_abs = max(max_abs, float(err.max()))
        ok = ok and rows_ok and bool((err <= 2e-3 + 1e-3 * np.abs(ref)).all())
    parity.update(max_abs=max_abs, ok=ok)
    # ---- e2e: the same steps through the public API with host buffers -----------------------
    # Each step's inputs (per layer: Q, K, V packed) come from pinned host memory and its outputs go
    # back, every step.  Within a step the copies overlap the attention: layers 0-5's inputs go first,
    # layers 6-11's are copied on a side stream while 0-5 run, and 0-5's outputs come back while
    # 6-11 run.  Nothing crosses steps (a decode step's inputs exist only once the step before ended).
    import ctypes
    qn, kn = T * N_HEAD * HD, T * KV_DIM
    rowf = qn + 2 * kn
    Xh = torch.from_numpy(np.concatenate([Qs.reshape(total_steps, N_LAYER, qn), Ks.reshape(total_steps, N_LAYER, kn),
                                          Vs.reshape(total_steps, N_LAYER, kn)], axis=2)).pin_memory()
    outh_p = torch.empty(N_LAYER, T, N_HEAD, HD).pin_memory()
    xd = torch.empty(N_LAYER, rowf, device=dev)
    eng.snapshot_load(snap, 0)
    # the C ABI as a C++ caller (a ggml custom op) uses it: raw device addresses, argument arrays
    # built once, the position updated in place
    cabi = Q.lib().qkv_append_attn_decode
    h_eng, h_stream = eng.handle, stream.cuda_stream
    slot_arr, pos_arr = (ctypes.c_int32 * 1)(0), (ctypes.c_int32 * 1)(0)
    xp, op = xd.data_ptr(), out.data_ptr()
    c_scale = ctypes.c_float(SCALE)
    cs = torch.cuda.Stream(device=dev)
    HALF = N_LAYER // 2
    ev = {k: torch.cuda.Event() for k in ("inA", "inB", "doneA", "doneB", "outA", "outB")}

    def layers(l0: int, l1: int):
        for l in range(l0, l1):
            base = xp + l * rowf * 4
            st_ = cabi(h_eng, l, slot_arr, pos_arr, 1, base + qn * 4, base + (qn + kn) * 4, base, T, c_scale,
                       op + l * qn * 4, h_stream)
            if st_ != 0:
                raise RuntimeError(f"qkv_append_attn_decode: status {st_}: {Q.lib().qkv_last_error(h_eng)}")

    def step_e2e(i: int):
        pos_arr[0] = CTX0 + T * i
        with torch.cuda.stream(cs):
            cs.wait_event(ev["doneB"])                       # the previous step is done with xd
            xd[:HALF].copy_(Xh[i, :HALF], non_blocking=True)
            ev["inA"].record(cs)
            xd[HALF:].copy_(Xh[i, HALF:], non_blocking=True)
            ev["inB"].record(cs)
        stream.wait_event(ev["inA"])
        stream.wait_event(ev["outA"])                        # out[:HALF] of the previous step copied out
        layers(0, HALF)
        ev["doneA"].record(stream)
        stream.wait_event(ev["inB"])
        stream.wait_event(ev["outB"])
        layers(HALF, N_LAYER)
        ev["doneB"].record(stream)
        with torch.cuda.stream(cs):
            cs.wait_event(ev["doneA"])
            outh_p[:HALF].copy_(out[:HALF], non_blocking=True)
            ev["outA"].record(cs)
            cs.wait_event(ev["doneB"])
            outh_p[HALF:].copy_(out[HALF:], non_blocking=True)
            ev["outB"].record(cs)

    for k in ev.values():
        k.record(stream)
    for i in range(warm):
        step_e2e(i)
    torch.cuda.synchronize()
    _barrier(ws, local)
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for i in range(warm, total_steps):
        step_e2e(i)
    stream.wait_event(ev["outB"])                            # the last step's outputs are on the host
    f1.record(stream)
    torch.cuda.synchronize()
    _barrier(ws, local)
    e2e_ms = f0.elapsed_time(f1)
    ms, e2e_ms = _max_over_ranks(ws, dev, [ms, e2e_ms])
    snap.release()
    eng.close()
    pk = peaks()
    ms_launch = ms / (steps * N_LAYER)
    # algorithmic bytes of one launch: the q8_0 K and V rows it attends, Q and the new K/V rows
    # read, the output and the appended q8_0 rows written
    io_bytes = 2 * T * N_HEAD * HD * 4 + 2 * T * KV_DIM * 4 + 2 * T * ROW_BYTES
    dec_bytes = [(CTX0 + T * (i + 1)) * 2 * ROW_BYTES + io_bytes for i in range(warm, total_steps)]
    achieved = statistics.mean(dec_bytes) / (ms_launch * 1e-3) / 1e9
    traffic, traffic_src = load_traffic()
    tokens = ws * T * steps
    line = {
        "metric": METRIC, "value": tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": ws, "steps": steps,
        "warmup": warm, "ms_per_step": ms / steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8 dot + f32 softmax/accumulate", "data": DATA,
        "config": dict(CONFIG, parallelism=f"sequence-sharded x{ws} (independent sequence per GPU, no collective)",
                       timing=f"the K steps captured once as a CUDA graph (per layer: the fused append+attention "
                              f"kernel and its split-K merge), device-resident inputs; the timed region is one "
                              f"replay of the K steps, repeated {REPLAYS} times, median reported (max over ranks)",
                       region_ms=[round(x, 4) for x in region_ms]),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm"], "unit": "GB/s",
                     "frac": achieved / pk["hbm"], "frac_of_8000": achieved / 8000.0, "peak_source": pk["hbm_src"],
                     "kernel": "k_decode (fused q8_0 append + split-K verify attention) and its merge, per layer",
                     "bytes_per_launch": statistics.mean(dec_bytes), "ms_per_launch": ms_launch,
                     "ms_per_launch_note": "graph time / layers: both kernels of a layer and the gaps between "
                                           "layers",
                     "traffic": traffic, "traffic_source": traffic_src},
        "parity": parity,
        "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": N_LAYER * (T * N_HEAD * HD * 4 + 2 * T * KV_DIM * 4),
                "d2h_bytes_per_step": N_LAYER * T * N_HEAD * HD * 4,
                "path": "qkv_append_attn_decode (C ABI, called through ctypes with raw device addresses as a C++ "
                        "caller would) per layer, no graph; every step copies its inputs in from pinned host "
                        "memory and its outputs out, in two halves of 6 layers so that copies overlap the "
                        "step's own attention (never another step's)"},
        "gpu_launches": launches,
        "clocks": clk,
    }
    if ws == 1 and not args.no_cpu_baseline:
        threads = host_threads()
        cpu = CpuConfig2(prefix, Qs, Ks, Vs, threads)
        cpu.step(0)
        n_cpu = min(steps, 24)
        times = cpu.timed(1, n_cpu)
        line["cpu_baseline"] = {
            "value": T * n_cpu / sum(times), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{n_cpu} full config-2 steps of the same inputs (12 layers x 3-token verify at ctx 16387+) "
                      f"after 1 warm step; oracle/qkv_oracle.c, OpenMP over (token, head) rows, {threads} threads"}
    return line


# ----------------------------------------------------------------------------- ctx 73,728
CTX_LONG = 73728


def measure_long(args, local: int, steps: int = 10) -> dict:
    """configs[1]'s step (12 layers, T = 3, one fused append + verify launch per layer) for one
    sequence at context 73,728, the top of the metric's 16K-73K range.  The prefix is device-seeded
    N(0,1) (torch Philox, seed 73); the K steps are one CUDA graph, median of REPLAYS replays; the
    last step's layer 0 is checked against the oracle."""
    import numpy as np
    import torch
    import qwfn_hybrid_b200 as Q
    from oracle import oracle as O
    dev = torch.device("cuda", local)
    warm = max(args.warmup, 3)
    total = warm + steps
    eng = Q.Engine(n_layer=N_LAYER, n_head=N_HEAD, n_head_kv=N_HEAD_KV, n_ctx=CTX_LONG + T * (total + 8), n_slots=1,
                   device=local)
    eng.seq_alloc(0)
    gen = torch.Generator(device=dev).manual_seed(73)
    for l in range(N_LAYER):
        eng.append(l, 0, 0, torch.randn(CTX_LONG, KV_DIM, generator=gen, device=dev),
                   torch.randn(CTX_LONG, KV_DIM, generator=gen, device=dev))
    eng.reserve(0, CTX_LONG + T * total)
    Qd = torch.randn(total, N_LAYER, T, N_HEAD, HD, generator=gen, device=dev)
    Kd = torch.randn(total, N_LAYER, T, KV_DIM, generator=gen, device=dev)
    Vd = torch.randn(total, N_LAYER, T, KV_DIM, generator=gen, device=dev)
    out = torch.empty(N_LAYER, T, N_HEAD, HD, device=dev)

    def step(i: int):
        for l in range(N_LAYER):
            eng.append_attn_decode(l, [0], [CTX_LONG + T * i], Kd[i, l], Vd[i, l], Qd[i, l], T, SCALE, out[l])

    for i in range(warm):
        step(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(warm, total):
            step(i)
    graph.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    per = []
    for _ in range(REPLAYS):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        per.append(e0.elapsed_time(e1))
    del graph
    if eng.device_status() != 0:
        raise RuntimeError("device status reported a bounds violation")
    ms = statistics.median(per)
    # parity: layer 0 of the last step (its appended rows bit-exact, attention vs the oracle)
    last, l = total - 1, 0
    n0 = CTX_LONG + T * last
    Kr = torch.empty((n0 + T, ROW_BYTES), dtype=torch.uint8, device=dev)
    Vr = torch.empty_like(Kr)
    eng.read_rows(l, 0, 0, n0 + T, Kr, Vr)
    torch.cuda.synchronize()
    Kh, Vh = Kr.cpu().numpy(), Vr.cpu().numpy()
    rows_ok = bool(np.array_equal(Kh[n0:], O.quantize_rows(Kd[last, l].cpu().numpy())) and
                   np.array_equal(Vh[n0:], O.quantize_rows(Vd[last, l].cpu().numpy())))
    ref = O.attn(Qd[last, l].cpu().numpy(), Kh, Vh, np.arange(n0, n0 + T, dtype=np.int32), N_HEAD_KV, SCALE,
                 threads=host_threads())
    err = np.abs(out[l].cpu().numpy() - ref)
    ok = rows_ok and bool((err <= 2e-3 + 1e-3 * np.abs(ref)).all())
    eng.close()
    ms_launch = ms / (steps * N_LAYER)
    io_bytes = 2 * T * N_HEAD * HD * 4 + 2 * T * KV_DIM * 4 + 2 * T * ROW_BYTES
    dec_bytes = statistics.mean([(CTX_LONG + T * (i + 1)) * 2 * ROW_BYTES + io_bytes for i in range(warm, total)])
    gbs = dec_bytes / (ms_launch * 1e-3) / 1e9
    hbm = peaks()["hbm"]
    return {"workload": f"configs[1]'s step at ctx {CTX_LONG}: 1 sequence, 12 layers, T=3, one fused append + decode "
                        "launch (and its merge) per layer; device-seeded N(0,1) prefix (seed 73)",
            "tokens_per_s": T * steps / (ms * 1e-3), "us_per_layer": 1e3 * ms_launch, "steps": steps,
            "timing": f"the {steps} steps as one CUDA graph, median of {REPLAYS} replays",
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                         "bytes_per_launch": dec_bytes},
            "parity": {"checked": "layer 0 of the last step (appended rows bit-exact; attention vs oracle/qkv_oracle.c)",
                       "atol": 2e-3, "rtol": 1e-3, "max_abs": float(err.max()), "ok": ok}}


# ----------------------------------------------------------------------------- configs[4] (ragged)
PREFIX = 8192


def config5_contexts() -> list[int]:
    """64 contexts floor(exp(U(ln 1024, ln 65536))), numpy default_rng(4)."""
    import numpy as np
    r = np.random.default_rng(4)
    return [int(c) for c in np.floor(np.exp(r.uniform(np.log(1024), np.log(65536), 64)))]


def measure_ragged(args, rank: int, ws: int, local: int, n_seqs: int = 64) -> dict:
    """the 64 sequences sharded by slot (LPT on context) over the ranks, each restored
    from the 8192-token shared-prefix snapshot (its first min(8192, ctx-1) positions shared, recurrent
    state of 36 DeltaNet layers copied), then one 1-token decode step over 12 layers per timed step.
    Returns the whole-job record (identical on every rank)."""
    import torch
    import qwfn_hybrid_b200 as Q
    dev = torch.device("cuda", local)
    ctx = config5_contexts()[:n_seqs]
    owner = Q.shard_lpt(ctx, ws)
    mine = [i for i in range(len(ctx)) if owner[i] == rank]
    n = len(mine)
    my_ctx = [ctx[i] for i in mine]
    pages = sum((c + 255) // 256 for c in my_ctx) + PREFIX // 256 + n + 8
    eng = Q.Engine(n_layer=N_LAYER, n_head=N_HEAD, n_head_kv=N_HEAD_KV, n_ctx=max(my_ctx + [PREFIX]) + 8,
                   n_slots=n + 1, n_pages=pages, rec_n_layer=36, rec_head_dim=128, rec_n_head=32,
                   conv_channels=8192, conv_hist=3, device=local)
    gen = torch.Generator(device=dev).manual_seed(4 + 1000 * rank)
    src = n   # the prefix slot
    eng.seq_alloc(src)
    for l in range(N_LAYER):
        eng.append(l, src, 0, torch.randn(PREFIX, KV_DIM, generator=gen, device=dev),
                   torch.randn(PREFIX, KV_DIM, generator=gen, device=dev))
    for l in range(36):
        for kind in (0, 1):
            ptr, nbytes = eng.state_ptr(src, l, kind)
            torch.as_tensor(_DevRange(ptr, nbytes), device=dev).copy_(torch.randn(nbytes // 4, generator=gen, device=dev))
    snap = eng.snapshot_save(src)
    slots = list(range(n))
    keep = [min(PREFIX, c - 1) for c in my_ctx]
    for s_ in slots:
        eng.seq_alloc(s_)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    r0.record(stream)
    eng.snapshot_load_many(snap, slots, keep)
    r1.record(stream)
    torch.cuda.synchronize()
    restore_ms = r0.elapsed_time(r1)
    rec_bytes = 36 * (128 * 128 * 32 * 4 + 3 * 8192 * 4)
    # each sequence's own positions beyond the shared prefix, up to ctx - 1 (random rows drawn once
    # per chunk size and reused: their values do not change the work)
    pool_k = torch.randn(8192, KV_DIM, generator=gen, device=dev)
    pool_v = torch.randn(8192, KV_DIM, generator=gen, device=dev)
    for s_, c in zip(slots, my_ctx):
        eng.reserve(s_, c + 1)
        for l in range(N_LAYER):
            for p0 in range(keep[s_], c - 1, 8192):
                m = min(8192, c - 1 - p0)
                eng.append(l, s_, p0, pool_k[:m], pool_v[:m])
    Qd = torch.randn(N_LAYER, n, 1, N_HEAD, HD, generator=gen, device=dev)
    Kd = torch.randn(N_LAYER, n, 1, KV_DIM, generator=gen, device=dev)
    Vd = torch.randn(N_LAYER, n, 1, KV_DIM, generator=gen, device=dev)
    out = torch.empty(N_LAYER, n, 1, N_HEAD, HD, device=dev)
    pos = [c - 1 for c in my_ctx]

    def step():
        for l in range(N_LAYER):
            eng.append_attn_decode(l, slots, pos, Kd[l], Vd[l], Qd[l], 1, SCALE, out[l])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    _barrier(ws, local)
    torch.cuda.synchronize()
    launches0 = Q.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    launches = Q.launch_count() - launches0
    _barrier(ws, local)
    ms = e0.elapsed_time(e1)
    if eng.device_status() != 0:
        raise RuntimeError("device status reported a bounds violation")
    kv_bytes = sum(my_ctx) * N_LAYER * 2 * ROW_BYTES
    io_bytes = N_LAYER * n * (2 * N_HEAD * HD * 4 + 2 * KV_DIM * 4 + 2 * ROW_BYTES)
    step_bytes = kv_bytes + io_bytes
    per_rank = _gather(ws, dev, [ms, restore_ms, float(step_bytes), float(n), float(sum(my_ctx))])
    snap.release()
    eng.close()
    hbm = peaks()
    rank_ms = [p[0] for p in per_rank]
    rank_gbs = [p[2] * args.steps / (p[0] * 1e-3) / 1e9 for p in per_rank]
    t_max = max(rank_ms)
    return {
        "workload": f"configs[4]: {len(ctx)} ragged sequences (ctx 1219..61356, sum {sum(ctx)}), 12 layers, paged "
                    f"256-token pages, restored from an 8192-token shared-prefix snapshot, T=1, one fused append + "
                    f"decode launch per layer",
        "parallelism": f"strong scaling: the {len(ctx)} sequences LPT-sharded by context over {ws} rank(s), no "
                       f"collective", "scaling": "strong",
        "value": len(ctx) * args.steps / (t_max * 1e-3), "unit": "tokens/s", "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_max / args.steps,
        "per_rank": [{"rank": i, "seqs": int(p[3]), "tokens": int(p[4]), "ms_per_step": p[0] / args.steps,
                      "gbs": g, "frac": g / hbm["hbm"]} for i, (p, g) in enumerate(zip(per_rank, rank_gbs))],
        "imbalance_max_over_min": max(rank_ms) / min(rank_ms),
        "roofline": {"bound": "hbm", "achieved": statistics.mean(rank_gbs), "peak": hbm["hbm"], "unit": "GB/s",
                     "frac": statistics.mean(rank_gbs) / hbm["hbm"], "peak_source": hbm["hbm_src"],
                     "note": "per-GPU GB/s (mean over ranks) of the KV, query, output and appended bytes"},
        "snapshot_restore": {"ms_max_over_ranks": max(p[1] for p in per_rank),
                             "slots_per_rank_max": int(max(p[3] for p in per_rank)),
                             "recurrent_bytes_per_slot": rec_bytes},
        "gpu_launches_per_rank0": launches,
    }


def run_cfg5(args) -> None:
    import torch
    rank, ws, local = dist_init("nccl")
    torch.cuda.set_device(local)
    clocks = Clocks(local)
    clocks.start()
    r = measure_ragged(args, rank, ws, local, n_seqs=args.seqs)
    clk = clocks.stop()
    if rank != 0:
        return
    print(json.dumps({
        "metric": METRIC, "value": r["value"], "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8 dot + f32 softmax/accumulate",
        "data": "synthetic N(0,1) (torch Philox, seed 4+1000*rank); contexts from numpy default_rng(4)",
        "config": {"workload": r["workload"], "parallelism": r["parallelism"],
                   "l2": "inputs larger than L2 (17 GB of KV per step)"},
        "roofline": r["roofline"], "ragged": r, "gpu_launches": r["gpu_launches_per_rank0"], "clocks": clk,
    }), flush=True)


# ----------------------------------------------------------------------------- configs[0]
def measure_cfg1(args, local: int) -> dict:
    """4096 cached rows, then a step appends the token's K/V and attends for its one
    query (seed 0: K [4097, 512], V [4097, 512], Q [16, 256] from numpy default_rng(0)).  A step is
    one fused launch (+ merge); it is captured as a CUDA graph and replayed K times per timed region."""
    import numpy as np
    import torch
    import qwfn_hybrid_b200 as Q
    from oracle import oracle as O
    dev = torch.device("cuda", local)
    r = np.random.default_rng(0)
    n = 4097
    Kf = r.standard_normal((n, KV_DIM), dtype=np.float32)
    Vf = r.standard_normal((n, KV_DIM), dtype=np.float32)
    Qf = r.standard_normal((1, N_HEAD, HD), dtype=np.float32)
    eng = Q.Engine(n_layer=1, n_head=N_HEAD, n_head_kv=N_HEAD_KV, n_ctx=4352, n_slots=1, device=local)
    eng.seq_alloc(0)
    eng.append(0, 0, 0, torch.from_numpy(Kf[:n - 1]).to(dev), torch.from_numpy(Vf[:n - 1]).to(dev))
    eng.reserve(0, n)
    kd, vd, qd = (torch.from_numpy(a).to(dev) for a in (Kf[n - 1:], Vf[n - 1:], Qf))
    out = torch.empty(1, N_HEAD, HD, device=dev)
    for _ in range(max(args.warmup, 3)):
        eng.append_attn_decode(0, [0], [n - 1], kd, vd, qd, 1, SCALE, out)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        eng.append_attn_decode(0, [0], [n - 1], kd, vd, qd, 1, SCALE, out)
    graph.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    per_step = []
    for _ in range(REPLAYS):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        per_step.append(e0.elapsed_time(e1) / args.steps)
    del graph
    assert eng.device_status() == 0
    Kr = torch.empty((n, ROW_BYTES), dtype=torch.uint8, device=dev)
    Vr = torch.empty_like(Kr)
    eng.read_rows(0, 0, 0, n, Kr, Vr)
    torch.cuda.synchronize()
    Kq, Vq = O.quantize_rows(Kf), O.quantize_rows(Vf)
    rows_ok = bool(np.array_equal(Kr.cpu().numpy(), Kq) and np.array_equal(Vr.cpu().numpy(), Vq))
    threads = host_threads()
    ref = O.attn(Qf, Kq, Vq, [n - 1], N_HEAD_KV, SCALE, threads=threads)
    err = np.abs(out.cpu().numpy() - ref)
    eng.close()
    # the same step on the host's cores: quantise the new row, then the 16-head attention
    cpu = []
    for _ in range(20):
        t0 = time.perf_counter()
        O.quantize_rows(Kf[n - 1:], threads)
        O.quantize_rows(Vf[n - 1:], threads)
        O.attn(Qf, Kq, Vq, [n - 1], N_HEAD_KV, SCALE, threads=threads)
        cpu.append(time.perf_counter() - t0)
    us = 1e3 * statistics.median(per_step)
    algo = n * 2 * ROW_BYTES + 2 * N_HEAD * HD * 4 + 2 * KV_DIM * 4 + 2 * ROW_BYTES
    pk = peaks()
    return {"workload": "configs[0]: 1 layer, 4096 cached + 1 appended, T=1, seed 0, one fused append + decode",
            "us_per_step": us, "tokens_per_s": 1e6 / us,
            "roofline": {"bound": "hbm (launch-bound at this size)", "achieved": algo / (us * 1e-6) / 1e9,
                         "peak": pk["hbm"], "unit": "GB/s", "frac": algo / (us * 1e-6) / 1e9 / pk["hbm"],
                         "bytes_per_step": algo},
            "parity": {"rows_bit_exact": rows_ok, "max_abs": float(err.max()),
                       "ok": rows_ok and bool((err <= 2e-3 + 1e-3 * np.abs(ref)).all())},
            "cpu_baseline": {"value": 1e6 * statistics.median(cpu), "unit": "us/step", "cores": threads,
                             "kind": "port", "sample": "20 steps of the same inputs (quantise the new K/V row + "
                                                       "16-head attention over 4097 cells), median"}}


# ----------------------------------------------------------------------------- configs[3]
SP_CTX, SP_BLK, SP_TOPK = 73728, 64, 32


def cfg4_host_data():
    """seed 3: K = N(0,1) + an offset of variance 2 drawn per 64-token block and KV head (added to
    all 256 dims), V = N(0,1); then the step's Q [3, 16, 256]."""
    import numpy as np
    r = np.random.default_rng(3)
    nb = SP_CTX // SP_BLK
    off = (r.standard_normal((nb, N_HEAD_KV, 1), dtype=np.float32) * np.float32(np.sqrt(2.0)))
    Kf = (r.standard_normal((nb, SP_BLK, N_HEAD_KV, HD), dtype=np.float32) + off[:, None]).reshape(SP_CTX, KV_DIM)
    Vf = r.standard_normal((SP_CTX, KV_DIM), dtype=np.float32)
    Qf = r.standard_normal((T, N_HEAD, HD), dtype=np.float32)
    return Kf, Vf, Qf


def measure_cfg4(args, local: int) -> dict:
    """a step appends its 3 tokens' K/V rows (positions 73725..73727), scores the 1152
    64-token blocks per KV head against the 3 query tokens, keeps the top 32 (block 0 and the last
    two forced) and attends to the selected blocks in place."""
    import numpy as np
    import torch
    import qwfn_hybrid_b200 as Q
    from oracle import oracle as O
    dev = torch.device("cuda", local)
    Kf, Vf, Qf = cfg4_host_data()
    p0 = SP_CTX - T
    eng = Q.Engine(n_layer=1, n_head=N_HEAD, n_head_kv=N_HEAD_KV, n_ctx=SP_CTX, n_slots=1, select_block=SP_BLK,
                   device=local)
    eng.seq_alloc(0)
    for c in range(0, p0, 8192):
        m = min(8192, p0 - c)
        eng.append(0, 0, c, torch.from_numpy(Kf[c:c + m]).to(dev), torch.from_numpy(Vf[c:c + m]).to(dev))
    eng.reserve(0, SP_CTX)
    kd, vd, qd = (torch.from_numpy(a).to(dev) for a in (Kf[p0:], Vf[p0:], Qf))
    idx = torch.empty((1, N_HEAD_KV, SP_TOPK), dtype=torch.int32, device=dev)
    out = torch.empty(T, N_HEAD, HD, device=dev)
    stream = torch.cuda.current_stream()

    def step(ev=None):
        eng.append(0, 0, p0, kd, vd)
        if ev:
            ev[0].record(stream)
        eng.select_blocks(0, [0], [p0], qd, T, SP_TOPK, idx)
        eng.attn_decode(0, [0], [p0], qd, T, SCALE, out, sel=idx, n_sel=SP_TOPK)
        if ev:
            ev[1].record(stream)

    for _ in range(max(args.warmup, 3)):     # the first select computes the 1150 whole-block summaries
        step()
    torch.cuda.synchronize()
    # timed as replays of CUDA graphs (the step, and select + attend alone), so no host time sits
    # between the launches; eager steps with per-step events if capture is refused
    timing = "replays of CUDA graphs of a step and of its select + attend, median of 5"
    try:
        g_step, g_sel = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_step):
            step()
        with torch.cuda.graph(g_sel):
            eng.select_blocks(0, [0], [p0], qd, T, SP_TOPK, idx)
            eng.attn_decode(0, [0], [p0], qd, T, SCALE, out, sel=idx, n_sel=SP_TOPK)
        g_step.replay()
        torch.cuda.synchronize()

        def timed(g):
            per = []
            for _ in range(REPLAYS):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                for _ in range(args.steps):
                    g.replay()
                b.record(stream)
                torch.cuda.synchronize()
                per.append(a.elapsed_time(b) / args.steps)
            return 1e3 * statistics.median(per)

        step_us, sel_us = timed(g_step), timed(g_sel)
        del g_step, g_sel
    except RuntimeError:
        timing = "eager steps, CUDA events around each step's select + attend"
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(args.steps):
            step(evs[i])
        t1.record(stream)
        torch.cuda.synchronize()
        sel_us = 1e3 * statistics.median(a.elapsed_time(b) for a, b in evs)
        step_us = 1e3 * t0.elapsed_time(t1) / args.steps
    assert eng.device_status() == 0
    Kr = torch.empty((SP_CTX, ROW_BYTES), dtype=torch.uint8, device=dev)
    Vr = torch.empty_like(Kr)
    eng.read_rows(0, 0, 0, SP_CTX, Kr, Vr)
    torch.cuda.synchronize()
    Kq, Vq = Kr.cpu().numpy(), Vr.cpu().numpy()
    got_idx, got = idx.cpu().numpy()[0], out.cpu().numpy()
    eng.close()
    threads = host_threads()
    nb = SP_CTX // SP_BLK
    rows_ok = bool(np.array_equal(Kq, O.quantize_rows(Kf, threads)) and np.array_equal(Vq, O.quantize_rows(Vf, threads)))
    summ = np.zeros((N_HEAD_KV, nb, HD), np.uint16)
    summ[:, :nb - 2] = O.block_summary(Kq, N_HEAD_KV, HD, SP_BLK, nb - 2, threads)
    c0 = time.perf_counter()
    ref_idx, _ = O.select_blocks(Qf, N_HEAD_KV, summ, nb, SP_TOPK)
    cells = [O.blocks_to_cells(ref_idx[h], SP_BLK, SP_CTX) for h in range(N_HEAD_KV)]
    ref = O.attn_sparse(Qf, Kq, Vq, np.arange(p0, SP_CTX), N_HEAD_KV, SCALE, cells, threads=threads)
    cpu_us = 1e6 * (time.perf_counter() - c0)
    err = np.abs(got - ref)
    algo = N_HEAD_KV * (nb - 2) * HD * 2 + N_HEAD_KV * SP_TOPK * SP_BLK * 2 * 272 + N_HEAD_KV * SP_TOPK * 4 \
        + 2 * T * N_HEAD * HD * 4
    pk = peaks()
    return {"workload": "configs[3]: ctx 73728 (1152 blocks of 64), seed 3 (K offset variance 2 per block and KV "
                        "head), T=3; per step: append 3 rows, score + top-32 per KV head (block 0 and the last two "
                        "forced), sparse attention over the 2048 selected tokens read in place",
            "us_per_select_attend": sel_us, "us_per_step_with_append": step_us, "timing": timing,
            "tokens_per_s": T * 1e6 / step_us,
            "roofline": {"bound": "hbm (latency-bound)", "achieved": algo / (sel_us * 1e-6) / 1e9, "peak": pk["hbm"],
                         "unit": "GB/s", "frac": algo / (sel_us * 1e-6) / 1e9 / pk["hbm"],
                         "bytes_per_select_attend": algo},
            "parity": {"indices_bit_exact": bool(np.array_equal(got_idx, ref_idx)), "rows_bit_exact": rows_ok,
                       "max_abs": float(err.max()),
                       "ok": bool(np.array_equal(got_idx, ref_idx)) and rows_ok and
                       bool((err <= 2e-3 + 1e-3 * np.abs(ref)).all())},
            "cpu_baseline": {"value": cpu_us, "unit": "us/select+attend", "cores": threads, "kind": "port",
                             "sample": "one select (1150 scored summaries per KV head, top-32) + sparse attention "
                                       "over the 2048 selected cells of 3 tokens x 16 heads"}}


def run_single(args, fn) -> None:
    import torch
    rank, ws, local = dist_init("nccl")
    torch.cuda.set_device(local)
    if rank == 0:
        print(json.dumps(fn(args, local)), flush=True)


# ----------------------------------------------------------------------------- the default line
def run_ours(args) -> None:
    import torch
    rank, ws, local = dist_init("nccl")
    torch.cuda.set_device(local)
    line = measure_cfg2(args, rank, ws, local)
    if not args.no_extras:
        line["ragged"] = measure_ragged(args, rank, ws, local)
        if ws == 1:
            extras = {"configs[0]": measure_cfg1(args, local)}
            c3 = measure_cfg3(args, rank, ws, local, e2e=False)
            extras["configs[2]"] = c3
            extras["configs[3]"] = measure_cfg4(args, local)
            extras["ctx73728"] = measure_long(args, local)
            line["configs"] = extras
    if rank == 0:
        print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- config 3
PF_N, PF_C = 16384, 512


def prefill_flops() -> float:
    """Causal QK^T + PV flops of the whole 16384-token prompt: 4 * H_q * d * sum_t (t + 1)."""
    return 4.0 * N_HEAD * HD * (PF_N * (PF_N + 1) / 2)


def cpu_prefill_baseline(chunks=(8, 15, 16, 23)) -> dict:
    """The oracle on a sample of config-3 chunks whose mean work equals the mean chunk's."""
    import numpy as np
    from oracle import oracle as O
    O.build()
    threads = host_threads()
    r = np.random.default_rng(2)
    n_kv = (max(chunks) + 1) * PF_C
    K = O.quantize_rows(r.standard_normal((n_kv, N_HEAD_KV * HD), dtype=np.float32), threads)
    V = O.quantize_rows(r.standard_normal((n_kv, N_HEAD_KV * HD), dtype=np.float32), threads)
    import torch
    Qf = torch.from_numpy(r.standard_normal((len(chunks), PF_C, N_HEAD, HD), dtype=np.float32)).to(torch.bfloat16).float().numpy()
    t0 = time.perf_counter()
    for i, c in enumerate(chunks):
        O.attn(Qf[i], K, V, c * PF_C + np.arange(PF_C, dtype=np.int32), N_HEAD_KV, SCALE, n_cells=(c + 1) * PF_C,
               threads=threads)
    dt = time.perf_counter() - t0
    return {"value": len(chunks) * PF_C / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"config-3 chunks {list(chunks)} (512 queries each over {[(c + 1) * PF_C for c in chunks]} "
                      f"cached keys; mean work = the mean chunk's); oracle/qkv_oracle.c, {threads} threads"}


def run_cfg3(args) -> None:
    import torch
    rank, ws, local = dist_init("nccl")
    torch.cuda.set_device(local)
    line = measure_cfg3(args, rank, ws, local)
    if rank == 0:
        print(json.dumps(line), flush=True)


def measure_cfg3(args, rank: int, ws: int, local: int, e2e: bool = True) -> dict:
    """a 16384-token prompt prefilled in 32 chunks of 512 on one layer; every chunk
    appends its 512 K/V rows (kernel A) and runs causal attention of its bf16 queries over the whole
    cache so far (kernel D, tcgen05).  One step = the whole prompt."""
    import torch
    dev = torch.device("cuda", local)
    import qwfn_hybrid_b200 as Q
    gen = torch.Generator(device=dev).manual_seed(2 + 1000 * rank)
    K = torch.randn(PF_N, N_HEAD_KV * HD, generator=gen, device=dev)
    V = torch.randn(PF_N, N_HEAD_KV * HD, generator=gen, device=dev)
    Qb = torch.randn(PF_N, N_HEAD, HD, generator=gen, device=dev).to(torch.bfloat16).view(torch.int16)
    out = torch.empty(PF_N, N_HEAD, HD, device=dev)
    eng = Q.Engine(n_layer=1, n_head=N_HEAD, n_head_kv=N_HEAD_KV, n_ctx=PF_N, n_slots=1, device=local)
    eng.seq_alloc(0)
    nch = PF_N // PF_C
    stream = torch.cuda.current_stream()

    def step():
        for c in range(nch):
            a, b = c * PF_C, (c + 1) * PF_C
            eng.append(0, 0, a, K[a:b], V[a:b])
            eng.attn_prefill(0, 0, a, Qb[a:b], PF_C, SCALE, out[a:b])

    def barrier():
        if ws > 1:
            torch.distributed.barrier(device_ids=[local])

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    # kernel-D time alone: the prompt's 32 prefill calls (the cache already holds every row) as one
    # CUDA graph, so no host time sits between them; median of 5 replays
    attn_timing = "the 32 prefill calls of a prompt as one CUDA graph, median of 5 replays"
    try:
        pf_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(pf_graph):
            for c in range(nch):
                a, b = c * PF_C, (c + 1) * PF_C
                eng.attn_prefill(0, 0, a, Qb[a:b], PF_C, SCALE, out[a:b])
        pf_graph.replay()
        torch.cuda.synchronize()
        per = []
        for _ in range(5):
            x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            x0.record(stream)
            pf_graph.replay()
            x1.record(stream)
            torch.cuda.synchronize()
            per.append(x0.elapsed_time(x1))
        del pf_graph
        attn_ms = statistics.median(per)
    except RuntimeError:   # capture refused: CUDA events around each call of one eager prompt
        attn_timing = "CUDA events around each prefill call of one eager prompt"
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(nch)]
        for c in range(nch):
            a, b = c * PF_C, (c + 1) * PF_C
            evs[c][0].record(stream)
            eng.attn_prefill(0, 0, a, Qb[a:b], PF_C, SCALE, out[a:b])
            evs[c][1].record(stream)
        torch.cuda.synchronize()
        attn_ms = sum(e0.elapsed_time(e1) for e0, e1 in evs)
    barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    clocks.start()
    # the timed prompts: replays of one CUDA graph of a whole prompt (32 appends + 32 prefill calls),
    # so no host time sits between the launches (eager prompts if capture is refused)
    launches0 = Q.launch_count()
    try:
        step_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(step_graph):
            step()
        per_prompt = (Q.launch_count() - launches0)
        step_graph.replay()
        torch.cuda.synchronize()
    except RuntimeError:
        step_graph, per_prompt = None, 0
        torch.cuda.synchronize()
    launches0 = Q.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        if step_graph is not None:
            step_graph.replay()
        else:
            step()
    e1.record(stream)
    torch.cuda.synchronize()
    launches = per_prompt * args.steps if step_graph is not None else Q.launch_count() - launches0
    del step_graph
    barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    if eng.device_status() != 0:
        raise RuntimeError("device status reported a bounds violation")
    # kernel A alone: appends of 4096 rows (F32 K and V in, q8_0 rows out) rewriting the prompt's
    # rows, four per replay of one CUDA graph (back to back, no host time between them)
    ap_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(ap_graph):
        for a in range(0, PF_N, 4096):
            eng.append(0, 0, a, K[a:a + 4096], V[a:a + 4096])
    ap_graph.replay()
    torch.cuda.synchronize()
    ap_ms = []
    for _ in range(5):
        x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        x0.record(stream)
        ap_graph.replay()
        x1.record(stream)
        torch.cuda.synchronize()
        ap_ms.append(x0.elapsed_time(x1) / (PF_N // 4096))
    del ap_graph
    ap_bytes = 4096 * N_HEAD_KV * HD * 4 * 2 + 4096 * 2 * ROW_BYTES
    append_rec = {"rows": 4096, "us_per_append": 1e3 * statistics.median(ap_ms),
                  "gbs": ap_bytes / (statistics.median(ap_ms) * 1e-3) / 1e9, "bytes_per_append": ap_bytes,
                  "kernel": "k_append (F32 K/V rows in, q8_0 rows out)",
                  "timing": "4 appends per replay of one CUDA graph, median of 5 replays"}
    e2e_ms = None
    if e2e:
        # end to end through the API: each chunk's K, V and Q from pinned host memory, its output back.
        # A prefill knows its whole prompt, so the copies run on two side streams and overlap the
        # attention of other chunks of the same prompt: inputs ahead, each chunk's output as soon as
        # that chunk is done; every copy of the prompt stays inside the timed region.
        hK, hV, hQ = K.cpu().pin_memory(), V.cpu().pin_memory(), Qb.cpu().pin_memory()
        hO = torch.empty(out.shape, dtype=out.dtype).pin_memory()
        dK, dV, dQ, dO = torch.empty_like(K), torch.empty_like(V), torch.empty_like(Qb), torch.empty_like(out)
        e2e_steps = max(1, min(args.steps, 3))
        cin, cout = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        ev_in = [torch.cuda.Event() for _ in range(nch)]
        ev_done = [torch.cuda.Event() for _ in range(nch)]
        ev_out = [torch.cuda.Event() for _ in range(nch)]
        for c in range(nch):
            ev_done[c].record(stream)
            ev_out[c].record(stream)
        torch.cuda.synchronize()
        x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        x0.record(stream)
        for _ in range(e2e_steps):
            with torch.cuda.stream(cin):
                for c in range(nch):
                    a, b = c * PF_C, (c + 1) * PF_C
                    cin.wait_event(ev_done[c])               # the previous prompt is done with these rows
                    dK[a:b].copy_(hK[a:b], non_blocking=True)
                    dV[a:b].copy_(hV[a:b], non_blocking=True)
                    dQ[a:b].copy_(hQ[a:b], non_blocking=True)
                    ev_in[c].record(cin)
            for c in range(nch):
                a, b = c * PF_C, (c + 1) * PF_C
                stream.wait_event(ev_in[c])
                stream.wait_event(ev_out[c])                 # the previous prompt's output rows are out
                eng.append(0, 0, a, dK[a:b], dV[a:b])
                eng.attn_prefill(0, 0, a, dQ[a:b], PF_C, SCALE, dO[a:b])
                ev_done[c].record(stream)
                with torch.cuda.stream(cout):
                    cout.wait_event(ev_done[c])
                    hO[a:b].copy_(dO[a:b], non_blocking=True)
                    ev_out[c].record(cout)
        stream.wait_event(ev_out[nch - 1])
        for c in range(nch):
            stream.wait_event(ev_out[c])
        x1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = x0.elapsed_time(x1) / e2e_steps
    eng.close()
    ms, attn_ms, e2e_ms = _max_over_ranks(ws, dev, [ms, attn_ms, e2e_ms or 0.0])
    pk = peaks()
    peak, peak_src = pk["bf16"], pk["bf16_src"]
    tflops = prefill_flops() / (attn_ms * 1e-3) / 1e12
    line = {
        "metric": "chunked-prefill tokens/s over q8_0 KV (16384-token prompt, 512-token chunks)",
        "value": ws * PF_N * args.steps / (ms * 1e-3), "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp16 tcgen05 (q8_0-rounded operands) + f32 softmax/accumulate",
        "data": "synthetic N(0,1) (torch Philox, seed 2+1000*rank), Q bf16",
        "config": {"workload": "configs[2]: 16384-token prompt, 32 chunks of 512, 1 layer, 16q/2kv x 256, q8_0 KV, "
                               "each chunk appends 512 rows then attends causally over the whole cache",
                   "parallelism": f"independent prompts x{ws} (replicas, no collective)",
                   "l2": "inputs larger than L2 (134 MB of bf16 queries + 268 MB of outputs per step)",
                   "timing": "replays of one CUDA graph of a whole prompt" if per_prompt else "eager prompts"},
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": peak, "unit": "TFLOP/s", "frac": tflops / peak,
                     "peak_source": peak_src, "traffic": None,
                     "kernel": "k_prefill_q + k_prefill + k_prefill_merge per chunk", "attn_timing": attn_timing,
                     "flops_per_step": prefill_flops(), "attn_ms_per_step": attn_ms},
        "gpu_launches": launches, "clocks": clk,
        "append": dict(append_rec, frac=append_rec["gbs"] / peaks()["hbm"]),
    }
    if e2e:
        line["e2e"] = {"value": ws * PF_N / (e2e_ms * 1e-3), "unit": "tokens/s",
                       "h2d_bytes_per_step": (K.numel() + V.numel()) * 4 + Qb.numel() * 2,
                       "d2h_bytes_per_step": out.numel() * 4}
    if not args.no_cpu_baseline and rank == 0:
        line["cpu_baseline"] = cpu_prefill_baseline()
    return line


QSA_CTX, QSA_LAYERS = 73728, 1


def qsa_inputs(r, n: int):
    """Indexer raw keys with a per-block offset (N(0,1) plus an offset of variance 2 drawn per
    4-cell block), so that blocks differ in relevance as configs[3]'s K does per 64-token block."""
    import numpy as np
    kr = r.standard_normal((n, 128), dtype=np.float32)
    kr += np.repeat(r.standard_normal(((n + 3) // 4, 128), dtype=np.float32) * np.float32(np.sqrt(2.0)), 4, axis=0)[:n]
    return kr


def cpu_qsa_baseline(steps: int = 2) -> dict:
    """The oracle's indexer + sparse attention for the same step on the host's cores."""
    import numpy as np
    from oracle import oracle as O
    O.build()
    threads = host_threads()
    r = np.random.default_rng(33)
    n = QSA_CTX
    K = O.quantize_rows(r.standard_normal((n, N_HEAD_KV * HD), dtype=np.float32))
    V = O.quantize_rows(r.standard_normal((n, N_HEAD_KV * HD), dtype=np.float32))
    keys16 = qsa_inputs(r, n).astype(np.float16).view(np.uint16)
    w = np.ones(128, np.float32)
    t0 = time.perf_counter()
    pooled = O.idx_pool(keys16, n // 4, w, 1e-6, 64, 1e7)      # maintained incrementally on the GPU
    t_pool = time.perf_counter() - t0
    t0 = time.perf_counter()
    for _ in range(steps):
        for t in range(T):
            pos = n - T + t
            q = r.standard_normal((4, 128), dtype=np.float32)
            kept, _ = O.idx_select(q, pooled, pos, 513)
            cells = (4 * kept[:, None] + np.arange(4)[None, :]).reshape(-1)
            cells = cells[cells <= pos].astype(np.int32)
            Qt = r.standard_normal((1, N_HEAD, HD), dtype=np.float32)
            O.attn(Qt, K, V, [pos], N_HEAD_KV, SCALE, cells=cells, threads=threads)
    dt = (time.perf_counter() - t0) / steps
    return {"value": T / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{steps} steps of 3 tokens at ctx {n}: score all whole blocks, top-513, attention over the "
                      f"kept cells (oracle/qkv_oracle.c, {threads} threads); pooling all {n // 4} blocks once took "
                      f"{t_pool * 1e3:.0f} ms and is not counted"}


def run_qsa(args) -> None:
    """configs[3]'s context (73728) and 3 MTP tokens, decoded through the model's own selector:
    each step appends the 3 tokens' K/V rows and indexer keys, then qkv_attn_decode_qsa scores
    every whole 4-cell block, keeps 513 per token (2052 cells) and attends over them in place."""
    import numpy as np
    import torch
    rank, ws, local = dist_init("nccl")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import qwfn_hybrid_b200 as Q
    steps, warm = args.steps, max(args.warmup, 3)
    total = warm + steps
    n0 = QSA_CTX - T * (total + 1)
    eng = Q.Engine(n_layer=QSA_LAYERS, n_head=N_HEAD, n_head_kv=N_HEAD_KV, n_ctx=QSA_CTX, n_slots=1, device=local)
    eng.indexer_enable(4, 2048, 64, 1e7, 1e-6)
    eng.seq_alloc(0)
    r = np.random.default_rng(3 + 1000 * rank)
    kr = torch.from_numpy(qsa_inputs(r, QSA_CTX)).to(dev)
    gen = torch.Generator(device=dev).manual_seed(3 + 1000 * rank)
    for c in range(0, n0, 4096):
        m = min(4096, n0 - c)
        eng.append(0, 0, c, torch.randn(m, N_HEAD_KV * HD, generator=gen, device=dev),
                   torch.randn(m, N_HEAD_KV * HD, generator=gen, device=dev))
        eng.idx_append(0, 0, c, kr[c:c + m])
    eng.reserve(0, QSA_CTX)
    Kd = torch.randn(total, T, N_HEAD_KV * HD, generator=gen, device=dev)
    Vd = torch.randn(total, T, N_HEAD_KV * HD, generator=gen, device=dev)
    Qd = torch.randn(total, T, N_HEAD, HD, generator=gen, device=dev)
    qi = torch.randn(total, T, 4, 128, generator=gen, device=dev)
    out = torch.empty(T, N_HEAD, HD, device=dev)
    stream = torch.cuda.current_stream()

    def step(i: int, attn_ev=None):
        p = n0 + T * i
        eng.append(0, 0, p, Kd[i], Vd[i])
        eng.idx_append(0, 0, p, kr[p:p + T])
        if attn_ev:
            attn_ev[0].record(stream)
        eng.attn_decode_qsa(0, [0], [p], qi[i], Qd[i], T, SCALE, out)
        if attn_ev:
            attn_ev[1].record(stream)

    for i in range(warm):
        step(i)
    torch.cuda.synchronize()
    clocks = Clocks(local)
    clocks.start()
    # timed as replays of CUDA graphs (a step -- the last warm-up step's, rewriting its rows -- and
    # its select + attend alone), so no host time sits between launches; eager steps with events
    # around each attend if capture is refused
    timing = "replays of CUDA graphs of a step and of its select + attend, median of 5"
    try:
        i_fix = warm - 1
        launches0 = Q.launch_count()
        g_step, g_attn = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_step):
            step(i_fix)
        per_step = Q.launch_count() - launches0
        with torch.cuda.graph(g_attn):
            eng.attn_decode_qsa(0, [0], [n0 + T * i_fix], qi[i_fix], Qd[i_fix], T, SCALE, out)
        g_step.replay()
        torch.cuda.synchronize()

        def timed(g):
            per = []
            for _ in range(REPLAYS):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                for _ in range(steps):
                    g.replay()
                b.record(stream)
                torch.cuda.synchronize()
                per.append(a.elapsed_time(b))
            return statistics.median(per)

        ms = timed(g_step)
        attn_us = 1e3 * timed(g_attn) / steps
        launches = per_step * steps
        del g_step, g_attn
    except RuntimeError:
        timing = "eager steps, CUDA events around each select + attend"
        torch.cuda.synchronize()
        launches0 = Q.launch_count()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(steps):
            step(warm + i, evs[i])
        e1.record(stream)
        torch.cuda.synchronize()
        launches = Q.launch_count() - launches0
        ms = e0.elapsed_time(e1)
        attn_us = 1e3 * statistics.median(a.elapsed_time(b) for a, b in evs)
    clk = clocks.stop()
    if eng.device_status() != 0:
        raise RuntimeError("device status reported a bounds violation")
    if ws > 1:
        t = torch.tensor([ms, attn_us], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, attn_us = t.tolist()
    if rank != 0:
        return
    n_whole = (QSA_CTX - 1) // 4
    algo = n_whole * 128 * 2 + T * 2052 * N_HEAD_KV * 2 * 272 + 2 * T * N_HEAD * HD * 4 + T * 4 * 128 * 4
    hbm, hbm_src = 6650.0, "fallback 6650 GB/s"
    pk = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pk):
        hbm, hbm_src = json.load(open(pk)).get("hbm_gbs", hbm), "measured hbm_gbs"
    gbs = algo / (attn_us * 1e-6) / 1e9
    line = {
        "metric": "QSA sparse decode (model's indexer) tokens/s and µs per select+attend step, ctx 73728, T=3",
        "value": ws * T * steps / (ms * 1e-3), "unit": "tokens/s", "n_gpus": ws, "steps": steps, "warmup": warm,
        "ms_per_step": ms / steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "q8_0 KV (int8 QK / f16 PV, f32 softmax); fp16 indexer keys, f32 scores",
        "data": "synthetic N(0,1) (torch Philox / numpy PCG64, seed 3+1000*rank); indexer keys with a per-block "
                "offset of variance 2",
        "config": {"workload": "configs[3]'s context and tokens through the model's own lightning indexer: ctx 73728, "
                               "1 layer, T=3, 4 indexer heads x 128, 4-cell blocks, 513 kept per token; each step "
                               "appends 3 K/V rows + 3 indexer keys, then select + attention over the kept blocks",
                   "parallelism": f"independent sequences x{ws} (replicas, no collective)",
                   "l2": "working set 4.7 MB of pooled keys + 6.7 MB of kept KV per step fits L2: latency-bound",
                   "timing": timing},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                     "peak_source": hbm_src, "traffic": None,
                     "kernel": "qkv_attn_decode_qsa: k_idx_score + k_idx_topk + k_decode in QSA mode (kept blocks read in place) + merge",
                     "algorithmic_bytes_per_step": algo, "attn_us_per_step": attn_us},
        "gpu_launches": launches, "clocks": clk,
    }
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_qsa_baseline()
    print(json.dumps(line), flush=True)


PJ_EMBD = 2560


def run_proj(args) -> None:
    """configs[1]'s step ahead of attention: per layer, the 3 tokens' query/key/value projections
    (n_embd 2560 -> 16 query heads, 2 KV heads of 256, bf16 weights), rms-norm + rope of Q and K and
    the q8_0 append of K and V, in one qkv_project_append call.  Weights of 12 layers (315 MB)
    exceed L2, so every layer streams its weights from HBM."""
    import torch
    rank, ws, local = dist_init("nccl")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import qwfn_hybrid_b200 as Q
    steps, warm = args.steps, max(args.warmup, 3)
    total = warm + steps
    n_ctx = CTX0 + T * (total + 2)
    eng = Q.Engine(n_layer=N_LAYER, n_head=N_HEAD, n_head_kv=N_HEAD_KV, n_ctx=n_ctx, n_slots=1, device=local)
    eng.seq_alloc(0)
    gen = torch.Generator(device=dev).manual_seed(7 + 1000 * rank)
    s = PJ_EMBD ** -0.5
    Wq = [(torch.randn(2 * N_HEAD * HD, PJ_EMBD, generator=gen, device=dev) * s).to(torch.bfloat16).view(torch.int16)
          for _ in range(N_LAYER)]
    Wk = [(torch.randn(N_HEAD_KV * HD, PJ_EMBD, generator=gen, device=dev) * s).to(torch.bfloat16).view(torch.int16)
          for _ in range(N_LAYER)]
    Wv = [(torch.randn(N_HEAD_KV * HD, PJ_EMBD, generator=gen, device=dev) * s).to(torch.bfloat16).view(torch.int16)
          for _ in range(N_LAYER)]
    qn = torch.ones(HD, device=dev)
    kn = torch.ones(HD, device=dev)
    X = torch.randn(total, N_LAYER, T, PJ_EMBD, generator=gen, device=dev)
    Qo = torch.empty(N_LAYER, T, N_HEAD, HD, device=dev)
    eng.reserve(0, n_ctx)
    stream = torch.cuda.current_stream()

    def step(i: int):
        p = T * i
        for l in range(N_LAYER):
            eng.project_append(l, 0, p, X[i, l], Wq[l], Wk[l], Wv[l], qn, kn, Qo[l])

    for i in range(warm):
        step(i)
    torch.cuda.synchronize()
    # the timed steps are one CUDA graph (12 launches per step), so host launch time is not in them
    graph = torch.cuda.CUDAGraph()
    launches0 = Q.launch_count()
    with torch.cuda.graph(graph):
        for i in range(steps):
            step(warm + i)
    launches = Q.launch_count() - launches0
    graph.replay()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    clocks.start()
    per = []
    for _ in range(REPLAYS):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        per.append(e0.elapsed_time(e1))
    clk = clocks.stop()
    del graph
    ms = statistics.median(per)
    if eng.device_status() != 0:
        raise RuntimeError("device status reported a bounds violation")
    if ws > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = t.item()
    if rank != 0:
        return
    per_layer = (2 * N_HEAD * HD // 2 + 2 * N_HEAD_KV * HD) * PJ_EMBD * 2     # weight rows read (query, K, V)
    per_layer += T * PJ_EMBD * 4 + T * N_HEAD * HD * 4 + 2 * T * ROW_BYTES    # x in, Q out, q8_0 rows out
    hbm, hbm_src = 6650.0, "fallback 6650 GB/s"
    pk = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pk):
        hbm, hbm_src = json.load(open(pk)).get("hbm_gbs", hbm), "measured hbm_gbs"
    ms_layer = ms / (steps * N_LAYER)
    gbs = per_layer / (ms_layer * 1e-3) / 1e9
    line = {
        "metric": "fused decode projections + norm + rope + q8_0 append: µs per layer and GB/s of weights streamed",
        "value": ms_layer * 1e3, "unit": "us/layer", "n_gpus": ws, "steps": steps, "warmup": warm,
        "ms_per_step": ms / steps, "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 weights, f32 accumulate / norm / rope, q8_0 K/V",
        "data": "synthetic N(0, 1/n_embd) weights and N(0,1) inputs (torch Philox, seed 7+1000*rank)",
        "config": {"workload": "configs[1]'s 3 tokens per step, 12 layers: n_embd 2560 -> 16 query heads (of the "
                               "query/gate interleave), 2 K and 2 V heads of 256",
                   "parallelism": f"independent sequences x{ws} (replicas, no collective)",
                   "l2": "12 layers of weights (315 MB) exceed L2: each layer's 26 MB come from HBM"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                     "peak_source": hbm_src, "traffic": None, "kernel": "k_project (one launch per layer)",
                     "bytes_per_launch": per_layer},
        "gpu_launches": launches, "clocks": clk,
    }
    print(json.dumps(line), flush=True)


def run_append(args) -> None:
    """Kernel A alone (BASELINE configs[2]'s append step at 4096 rows per call): F32 K and V rows
    into a 2-head q8_0 engine.  16 launches fill 65536 positions, then a CUDA graph of 16
    back-to-back 4096-row appends (rewriting those positions) is replayed."""
    import torch
    rank, ws, local = dist_init("nccl")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import qwfn_hybrid_b200 as Q
    n, R = 65536, 4096
    eng = Q.Engine(n_layer=1, n_head=N_HEAD, n_head_kv=N_HEAD_KV, n_ctx=n, n_slots=1, device=local)
    eng.seq_alloc(0)
    gen = torch.Generator(device=dev).manual_seed(5 + 1000 * rank)
    K = torch.randn(n, KV_DIM, generator=gen, device=dev)
    V = torch.randn(n, KV_DIM, generator=gen, device=dev)
    for a in range(0, n, R):
        eng.append(0, 0, a, K[a:a + R], V[a:a + R])
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for a in range(0, n, R):
            eng.append(0, 0, a, K[a:a + R], V[a:a + R])
    for _ in range(max(args.warmup, 3)):
        g.replay()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    clocks.start()
    per = []
    for _ in range(args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        per.append(e0.elapsed_time(e1) / (n // R))
    clk = clocks.stop()
    del g
    assert eng.device_status() == 0
    us = 1e3 * statistics.median(per)
    nbytes = R * (2 * KV_DIM * 4 + 2 * ROW_BYTES)
    pk = peaks()
    gbs = nbytes / (us * 1e-6) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": "q8_0 append (kernel A): µs per 4096-row append of F32 K and V rows", "value": us,
            "unit": "us/append", "n_gpus": ws, "steps": args.steps, "warmup": max(args.warmup, 3),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32 in, q8_0 out",
            "data": "synthetic N(0,1) (torch Philox, seed 5+1000*rank)",
            "config": {"workload": "4096-row appends, 2 KV heads x 256, 16 per CUDA-graph replay (median of the steps)",
                       "parallelism": f"independent engines x{ws} (replicas)"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": pk["hbm"], "unit": "GB/s", "frac": gbs / pk["hbm"],
                         "peak_source": pk["hbm_src"], "bytes_per_launch": nbytes, "kernel": "k_append"},
            "gpu_launches": n // R, "clocks": clk,
        }), flush=True)


class _DevRange:
    """A device address range as a float32 tensor (CUDA array interface)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes // 4,), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "cfg5":
        run_cfg5(args)
    elif args.workload == "cfg3":
        run_cfg3(args)
    elif args.workload == "cfg1":
        run_single(args, measure_cfg1)
    elif args.workload == "cfg4":
        run_single(args, measure_cfg4)
    elif args.workload == "qsa":
        run_qsa(args)
    elif args.workload == "proj":
        run_proj(args)
    elif args.workload == "append":
        run_append(args)
    elif args.workload == "long":
        run_single(args, measure_long)
    else:
        run_ours(args)
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
