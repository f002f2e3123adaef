"""qwfn_hybrid_b200 -- B200-native q8_0 KV-cache and attention engine for QwFN-hybrid's
full-attention layers.

The product is libqkv.so (C++ host engine + sm_100a CUDA kernels) behind the C ABI of
include/qkv.h.  This module is a thin ctypes front of that ABI for Python callers (tests,
bench.py): method names follow the reference's qwfn::state / qwfn::engine surface
(src/qwfn_state.h:39-92, src/qwfn_engine.h:226-312).  There is no fallback: if libqkv.so is
missing or fails to load, importing the engine raises.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqkv.so")

OK, ERR_INVALID, ERR_NO_MEMORY, ERR_CUDA, ERR_STATE, ERR_MISMATCH, ERR_DEVICE, ERR_UNSUPPORTED = range(8)

# Every symbol include/qkv.h declares (checked by tests/test_abi.py).
EXPORTS = [
    "qkv_create", "qkv_destroy", "qkv_last_error", "qkv_status_string", "qkv_bytes", "qkv_summary",
    "qkv_seq_alloc", "qkv_seq_free", "qkv_seq_reset", "qkv_seq_length", "qkv_seq_reserve", "qkv_seq_pages", "qkv_page_refcount",
    "qkv_pages_free", "qkv_append", "qkv_attn_decode", "qkv_append_attn_decode", "qkv_block_summary", "qkv_select_blocks",
    "qkv_gather_rows", "qkv_read_rows", "qkv_write_rows", "qkv_attn_prefill", "qkv_snapshot_save",
    "qkv_snapshot_restore", "qkv_snapshot_restore_many", "qkv_snapshot_release", "qkv_snapshot_info",
    "qkv_snapshot_to_host", "qkv_snapshot_from_host", "qkv_rollback", "qkv_rollback_arm", "qkv_state_ptr",
    "qkv_cache_view_get", "qkv_attn_decode_static", "qkv_device_status", "qkv_launch_count", "qkv_shard_lpt",
    "qkv_store_create", "qkv_store_destroy", "qkv_store_save", "qkv_store_restore_or_reset",
    "qkv_store_prefix_split", "qkv_store_evict", "qkv_store_info", "qkv_store_entry",
    "qkv_indexer_enable", "qkv_idx_append", "qkv_idx_select", "qkv_attn_decode_qsa", "qkv_idx_read",
    "qkv_project_append", "qkv_static_status", "qkv_debug_decode_wait", "qkv_attn_prefill_qsa",
    "qkv_debug_check_q8_scale",
]


class QkvError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status


class QkvConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "n_layer", "n_head", "n_head_kv", "head_dim", "n_ctx", "n_slots", "n_pages", "rec_n_layer",
        "rec_head_dim", "rec_n_head", "conv_channels", "conv_hist", "n_rollback", "select_block",
        "attn_interval")]


class QkvIndexerConfig(ctypes.Structure):
    _fields_ = [("n_head", ctypes.c_int32), ("key_len", ctypes.c_int32), ("ratio", ctypes.c_int32),
                ("top_k", ctypes.c_int32), ("rope_dim", ctypes.c_int32), ("rope_freq_base", ctypes.c_float),
                ("rms_eps", ctypes.c_float)]


class QkvCacheView(ctypes.Structure):
    _fields_ = [("pool", ctypes.c_void_p), ("page_bytes", ctypes.c_size_t), ("tile_bytes", ctypes.c_size_t),
                ("page_tokens", ctypes.c_int32), ("tile_tokens", ctypes.c_int32), ("n_pages", ctypes.c_int32),
                ("n_head_kv", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("block_table", ctypes.c_void_p),
                ("max_pages_per_seq", ctypes.c_int32)]


_lib = None


def lib() -> ctypes.CDLL:
    """Loads libqkv.so; raises if it was not built (no fallback path exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: run `python -m qwfn_hybrid_b200.build` (nvcc, sm_100a)")
    L = ctypes.CDLL(LIB_PATH)
    P, I32, I64, F32, SZ = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
    pI32 = ctypes.POINTER(ctypes.c_int32)
    sig = {
        "qkv_create": [ctypes.POINTER(QkvConfig), ctypes.c_int, ctypes.POINTER(P)],
        "qkv_destroy": [P], "qkv_last_error": [P], "qkv_status_string": [ctypes.c_int],
        "qkv_bytes": [P, ctypes.POINTER(SZ)], "qkv_summary": [P, ctypes.c_char_p, SZ],
        "qkv_seq_alloc": [P, I32], "qkv_seq_free": [P, I32], "qkv_seq_reset": [P, I32, P],
        "qkv_seq_length": [P, I32, pI32], "qkv_seq_pages": [P, I32, pI32, I32, pI32],
        "qkv_seq_reserve": [P, I32, I32, P],
        "qkv_page_refcount": [P, I32, pI32], "qkv_pages_free": [P, pI32],
        "qkv_append": [P, I32, I32, I32, P, P, I32, P],
        "qkv_attn_decode": [P, I32, pI32, pI32, I32, P, I32, F32, P, I32, P, P],
        "qkv_append_attn_decode": [P, I32, pI32, pI32, I32, P, P, P, I32, F32, P, P],
        "qkv_block_summary": [P, I32, I32, I32, I32, P],
        "qkv_select_blocks": [P, I32, pI32, pI32, I32, P, I32, I32, P, P, P],
        "qkv_gather_rows": [P, I32, I32, P, I32, P, P, P],
        "qkv_read_rows": [P, I32, I32, I32, I32, P, P, P],
        "qkv_write_rows": [P, I32, I32, I32, I32, P, P, P],
        "qkv_attn_prefill": [P, I32, I32, I32, P, I32, F32, P, P],
        "qkv_snapshot_save": [P, I32, ctypes.POINTER(P), P],
        "qkv_snapshot_restore": [P, P, I32, I32, P],
        "qkv_snapshot_restore_many": [P, P, pI32, pI32, I32, P],
        "qkv_snapshot_release": [P, P],
        "qkv_snapshot_info": [P, pI32, ctypes.POINTER(SZ)],
        "qkv_snapshot_to_host": [P, P, P, SZ, P],
        "qkv_snapshot_from_host": [P, P, SZ, I32, ctypes.POINTER(P), P],
        "qkv_rollback": [P, I32, I32, P], "qkv_rollback_arm": [P, I32, I32],
        "qkv_state_ptr": [P, I32, I32, I32, I32, ctypes.POINTER(P), ctypes.POINTER(SZ)],
        "qkv_cache_view_get": [P, I32, ctypes.POINTER(QkvCacheView)],
        "qkv_device_status": [P, P, pI32],
        "qkv_shard_lpt": [ctypes.POINTER(I64), I32, I32, pI32],
        "qkv_launch_count": [ctypes.POINTER(ctypes.c_uint64)],
        "qkv_store_create": [P, SZ, I32, ctypes.POINTER(P)], "qkv_store_destroy": [P],
        "qkv_store_save": [P, I32, pI32, I32, pI32, P],
        "qkv_store_restore_or_reset": [P, I32, pI32, I32, pI32, P],
        "qkv_store_prefix_split": [P, pI32, I32, I32, I32, pI32], "qkv_store_evict": [P, I32],
        "qkv_store_info": [P, pI32, ctypes.POINTER(SZ)], "qkv_store_entry": [P, I32, pI32, ctypes.POINTER(SZ)],
        "qkv_indexer_enable": [P, ctypes.POINTER(QkvIndexerConfig), P],
        "qkv_idx_append": [P, I32, I32, I32, P, I32, P],
        "qkv_idx_select": [P, I32, pI32, pI32, I32, P, I32, P, P, P, P],
        "qkv_attn_decode_qsa": [P, I32, pI32, pI32, I32, P, P, I32, F32, P, P],
        "qkv_idx_read": [P, I32, I32, I32, I32, P, I32, I32, P, P],
        "qkv_project_append": [P, I32, I32, I32, P, I32, I32, P, P, P, P, P, F32, I32, F32, P, P],
        "qkv_attn_decode_static": [ctypes.POINTER(QkvCacheView), I32, pI32, pI32, I32, I32, P, I32, F32, P, P],
        "qkv_static_status": [P, pI32],
        "qkv_debug_decode_wait": [P, I64, I32],
        "qkv_attn_prefill_qsa": [P, I32, I32, I32, P, P, I32, F32, P, P, P, P],
        "qkv_debug_check_q8_scale": [ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)],
    }
    for name, args in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int
    L.qkv_destroy.restype = None
    L.qkv_snapshot_release.restype = None
    L.qkv_store_destroy.restype = None
    L.qkv_last_error.restype = ctypes.c_char_p
    L.qkv_status_string.restype = ctypes.c_char_p
    _lib = L
    return L


def _i32_array(values) -> ctypes.Array:
    vals = [int(v) for v in values]
    return (ctypes.c_int32 * max(1, len(vals)))(*vals)


def _ptr(x) -> int | None:
    """Device pointer of a torch tensor (contiguous) or a raw integer address; None -> NULL."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if not x.is_contiguous():
        raise ValueError("tensor must be contiguous")
    return x.data_ptr()


_cur_stream = None   # () -> raw cudaStream_t of torch's current stream on the current device, or None


def _stream(stream) -> int | None:
    """Raw stream handle: torch's current stream when None (looked up without building a Stream
    object, a few microseconds per call otherwise), an int as is, else `stream.cuda_stream`."""
    global _cur_stream
    if stream is None:
        if _cur_stream is None:
            import torch
            if not torch.cuda.is_available():
                _cur_stream = lambda: None
            else:
                raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
                dev = torch.cuda.current_device
                _cur_stream = (lambda: raw(dev())) if raw else (lambda: torch.cuda.current_stream().cuda_stream)
        return _cur_stream()
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def shard_lpt(costs, n_ranks: int) -> list[int]:
    """Longest-processing-time owner rank for each independent sequence (include/qkv.h)."""
    n = len(costs)
    c = (ctypes.c_int64 * max(1, n))(*[int(v) for v in costs])
    owner = (ctypes.c_int32 * max(1, n))()
    st = lib().qkv_shard_lpt(c, n, n_ranks, owner)
    if st != OK:
        raise QkvError(st, "qkv_shard_lpt")
    return [owner[i] for i in range(n)]


def launch_count() -> int:
    """Kernels launched through libqkv.so by this process so far."""
    c = ctypes.c_uint64()
    st = lib().qkv_launch_count(ctypes.byref(c))
    if st != OK:
        raise QkvError(st, "qkv_launch_count")
    return c.value


@dataclass
class Snapshot:
    engine: "Engine"
    handle: int
    released: bool = field(default=False)

    def info(self) -> tuple[int, int]:
        n = ctypes.c_int32()
        b = ctypes.c_size_t()
        self.engine._check(lib().qkv_snapshot_info(self.handle, ctypes.byref(n), ctypes.byref(b)))
        return n.value, b.value

    @property
    def n_past(self) -> int:
        return self.info()[0]

    def release(self) -> None:
        if not self.released:
            lib().qkv_snapshot_release(self.engine.handle, self.handle)
            self.released = True


class Store:
    """Saved sequences on the device keyed by token ids: the reference server's saved_seq list with
    restore_or_reset and shared_prefix_split (tools/qwfn_server.cpp:764-800, 1380-1430)."""

    def __init__(self, engine: "Engine", cap_bytes: int, max_entries: int = 4):
        self.engine = engine
        h = ctypes.c_void_p()
        engine._check(lib().qkv_store_create(engine.handle, cap_bytes, max_entries, ctypes.byref(h)))
        self.handle = h.value

    def _s(self, stream):
        return _stream(stream) if self.engine.device >= 0 else None

    def close(self) -> None:
        if getattr(self, "handle", None):
            lib().qkv_store_destroy(self.handle)
            self.handle = None

    def save(self, slot: int, tokens, stream=None) -> bool:
        kept = ctypes.c_int32()
        self.engine._check(lib().qkv_store_save(self.handle, slot, _i32_array(tokens), len(tokens),
                                                ctypes.byref(kept), self._s(stream)))
        return bool(kept.value)

    def restore_or_reset(self, slot: int, prompt, stream=None) -> int:
        n = ctypes.c_int32()
        self.engine._check(lib().qkv_store_restore_or_reset(self.handle, slot, _i32_array(prompt), len(prompt),
                                                            ctypes.byref(n), self._s(stream)))
        return n.value

    def prefix_split(self, prompt, n_consumed: int, min_prefix: int = 2048) -> int:
        at = ctypes.c_int32()
        self.engine._check(lib().qkv_store_prefix_split(self.handle, _i32_array(prompt), len(prompt), n_consumed,
                                                        min_prefix, ctypes.byref(at)))
        return at.value

    def evict(self, n: int = 1) -> None:
        self.engine._check(lib().qkv_store_evict(self.handle, n))

    def info(self) -> tuple[int, int]:
        n, b = ctypes.c_int32(), ctypes.c_size_t()
        self.engine._check(lib().qkv_store_info(self.handle, ctypes.byref(n), ctypes.byref(b)))
        return n.value, b.value

    def entries(self) -> list[tuple[int, int]]:
        """(token count, device bytes) per entry, least recently used first."""
        out = []
        for i in range(self.info()[0]):
            n, b = ctypes.c_int32(), ctypes.c_size_t()
            self.engine._check(lib().qkv_store_entry(self.handle, i, ctypes.byref(n), ctypes.byref(b)))
            out.append((n.value, b.value))
        return out


class Engine:
    """One engine per GPU (device < 0: host-only bookkeeping engine, no kernels)."""

    def __init__(self, *, n_layer: int, n_head: int, n_head_kv: int, n_ctx: int, n_slots: int, head_dim: int = 256,
                 n_pages: int = 0, rec_n_layer: int = 0, rec_head_dim: int = 128, rec_n_head: int = 32,
                 conv_channels: int = 8192, conv_hist: int = 3, n_rollback: int = 0, select_block: int = 0,
                 attn_interval: int = 0, device: int = 0):
        self.cfg = QkvConfig(n_layer, n_head, n_head_kv, head_dim, n_ctx, n_slots, n_pages, rec_n_layer,
                             rec_head_dim, rec_n_head, conv_channels, conv_hist, n_rollback, select_block,
                             attn_interval)
        self.device = device
        h = ctypes.c_void_p()
        st = lib().qkv_create(ctypes.byref(self.cfg), device, ctypes.byref(h))
        if st != OK:
            raise QkvError(st, f"qkv_create: {lib().qkv_status_string(st).decode()}")
        self.handle = h.value

    # -- lifetime ---------------------------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "handle", None):
            lib().qkv_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, st: int) -> None:
        if st != OK:
            msg = lib().qkv_last_error(self.handle).decode(errors="replace") if self.handle else ""
            raise QkvError(st, msg)

    # -- state (qwfn::state surface) ---------------------------------------------------------
    def bytes(self) -> int:
        b = ctypes.c_size_t()
        self._check(lib().qkv_bytes(self.handle, ctypes.byref(b)))
        return b.value

    def summary(self) -> str:
        buf = ctypes.create_string_buffer(512)
        self._check(lib().qkv_summary(self.handle, buf, 512))
        return buf.value.decode()

    def seq_alloc(self, slot: int) -> None:
        self._check(lib().qkv_seq_alloc(self.handle, slot))

    def seq_free(self, slot: int) -> None:
        self._check(lib().qkv_seq_free(self.handle, slot))

    def reset(self, slot: int, stream=None) -> None:
        self._check(lib().qkv_seq_reset(self.handle, slot, _stream(stream) if self.device >= 0 else None))

    def n_past(self, slot: int) -> int:
        n = ctypes.c_int32()
        self._check(lib().qkv_seq_length(self.handle, slot, ctypes.byref(n)))
        return n.value

    def reserve(self, slot: int, n_tokens: int, stream=None) -> None:
        self._check(lib().qkv_seq_reserve(self.handle, slot, n_tokens, _stream(stream) if self.device >= 0 else None))

    def pages(self, slot: int) -> list[int]:
        n = ctypes.c_int32()
        self._check(lib().qkv_seq_pages(self.handle, slot, None, 0, ctypes.byref(n)))
        buf = (ctypes.c_int32 * max(1, n.value))()
        self._check(lib().qkv_seq_pages(self.handle, slot, buf, n.value, ctypes.byref(n)))
        return [buf[i] for i in range(n.value)]

    def refcount(self, page: int) -> int:
        n = ctypes.c_int32()
        self._check(lib().qkv_page_refcount(self.handle, page, ctypes.byref(n)))
        return n.value

    def pages_free(self) -> int:
        n = ctypes.c_int32()
        self._check(lib().qkv_pages_free(self.handle, ctypes.byref(n)))
        return n.value

    def cache_view(self, layer: int) -> QkvCacheView:
        v = QkvCacheView()
        self._check(lib().qkv_cache_view_get(self.handle, layer, ctypes.byref(v)))
        return v

    def state_ptr(self, slot: int, rec_layer: int, kind: int, which: int = 0) -> tuple[int, int]:
        p = ctypes.c_void_p()
        b = ctypes.c_size_t()
        self._check(lib().qkv_state_ptr(self.handle, slot, rec_layer, kind, which, ctypes.byref(p), ctypes.byref(b)))
        return p.value, b.value

    def debug_decode_wait(self, limit_ns: int, withhold_unit: int = -1) -> None:
        """Failure tests: bounded-wait limit of the decode kernels, and a unit whose first tile copy
        the next decode launch withholds (include/qkv.h qkv_debug_decode_wait)."""
        self._check(lib().qkv_debug_decode_wait(self.handle, int(limit_ns), int(withhold_unit)))

    def device_status(self, stream=None) -> int:
        c = ctypes.c_int32()
        st = lib().qkv_device_status(self.handle, _stream(stream), ctypes.byref(c))
        if st not in (OK, ERR_DEVICE):
            self._check(st)
        return c.value

    # -- kernels -----------------------------------------------------------------------------
    def append(self, layer: int, slot: int, pos: int, K, V, n_rows: int | None = None, stream=None) -> None:
        n = n_rows if n_rows is not None else K.shape[0]
        self._check(lib().qkv_append(self.handle, layer, slot, pos, _ptr(K), _ptr(V), n,
                                     _stream(stream) if self.device >= 0 else None))

    def attn_decode(self, layer: int, slots, pos0, Q, T: int, scale: float, out, sel=None, n_sel: int = 0,
                    stream=None) -> None:
        n = len(slots)
        self._check(lib().qkv_attn_decode(self.handle, layer, _i32_array(slots), _i32_array(pos0), n, _ptr(Q), T,
                                          scale, _ptr(sel), n_sel, _ptr(out), _stream(stream)))

    def append_attn_decode(self, layer: int, slots, pos0, K, V, Q, T: int, scale: float, out, stream=None) -> None:
        """Fused kernel A + C: append T rows per sequence at pos0 and attend (one launch)."""
        self._check(lib().qkv_append_attn_decode(self.handle, layer, _i32_array(slots), _i32_array(pos0), len(slots),
                                                 _ptr(K), _ptr(V), _ptr(Q), T, scale, _ptr(out), _stream(stream)))

    def block_summary(self, layer: int, slot: int, b0: int, b1: int, stream=None) -> None:
        self._check(lib().qkv_block_summary(self.handle, layer, slot, b0, b1, _stream(stream)))

    def select_blocks(self, layer: int, slots, pos0, Q, T: int, top_k: int, idx_out, scores_out=None,
                      stream=None) -> None:
        self._check(lib().qkv_select_blocks(self.handle, layer, _i32_array(slots), _i32_array(pos0), len(slots),
                                            _ptr(Q), T, top_k, _ptr(idx_out), _ptr(scores_out), _stream(stream)))

    def gather_rows(self, layer: int, slot: int, cells, K_out, V_out, stream=None) -> None:
        self._check(lib().qkv_gather_rows(self.handle, layer, slot, _ptr(cells), cells.numel(), _ptr(K_out),
                                          _ptr(V_out), _stream(stream)))

    def read_rows(self, layer: int, slot: int, pos: int, n: int, K_out, V_out, stream=None) -> None:
        self._check(lib().qkv_read_rows(self.handle, layer, slot, pos, n, _ptr(K_out), _ptr(V_out), _stream(stream)))

    def write_rows(self, layer: int, slot: int, pos: int, n: int, K_in, V_in, stream=None) -> None:
        self._check(lib().qkv_write_rows(self.handle, layer, slot, pos, n, _ptr(K_in), _ptr(V_in), _stream(stream)))

    def attn_prefill(self, layer: int, slot: int, pos0: int, Q, Tc: int, scale: float, out, stream=None) -> None:
        self._check(lib().qkv_attn_prefill(self.handle, layer, slot, pos0, _ptr(Q), Tc, scale, _ptr(out),
                                           _stream(stream)))

    def project_append(self, layer: int, slot: int, pos: int, x, Wq, Wk, Wv, q_norm, k_norm, Q_out=None,
                       rms_eps: float = 1e-6, rope_dim: int = 64, rope_freq_base: float = 1e7, stream=None) -> None:
        """x: F32 [T, n_embd]; W*: bf16 bits (int16 tensors) [rows, n_embd]; Wq/q_norm/Q_out may be None."""
        T, n_embd = int(x.shape[0]), int(x.shape[1])
        self._check(lib().qkv_project_append(self.handle, layer, slot, pos, _ptr(x), n_embd, T, _ptr(Wq), _ptr(Wk),
                                             _ptr(Wv), _ptr(q_norm), _ptr(k_norm), rms_eps, rope_dim, rope_freq_base,
                                             _ptr(Q_out), _stream(stream)))

    # -- QSA lightning indexer ------------------------------------------------------------------
    def indexer_enable(self, n_head: int = 4, top_k: int = 2048, rope_dim: int = 64, rope_freq_base: float = 1e7,
                       rms_eps: float = 1e-6, k_norm=None) -> int:
        """Returns k_blocks (blocks kept per token).  k_norm: numpy float32 [n_layer, 128] or None."""
        c = QkvIndexerConfig(n_head, 128, 4, top_k, rope_dim, rope_freq_base, rms_eps)
        w = None
        if k_norm is not None:
            import numpy as np
            self._knorm = np.ascontiguousarray(k_norm, dtype=np.float32)
            w = self._knorm.ctypes.data
        self._check(lib().qkv_indexer_enable(self.handle, ctypes.byref(c), w))
        self.k_blocks = (top_k + 3 + 3) // 4
        return self.k_blocks

    def idx_append(self, layer: int, slot: int, pos: int, k_raw, n_rows: int | None = None, stream=None) -> None:
        n = n_rows if n_rows is not None else int(k_raw.shape[0])
        self._check(lib().qkv_idx_append(self.handle, layer, slot, pos, _ptr(k_raw), n, _stream(stream)))

    def idx_select(self, layer: int, slots, pos0, q_idx, T: int, blocks_out, n_out, scores_out=None,
                   stream=None) -> None:
        self._check(lib().qkv_idx_select(self.handle, layer, _i32_array(slots), _i32_array(pos0), len(slots),
                                          _ptr(q_idx), T, _ptr(blocks_out), _ptr(n_out), _ptr(scores_out),
                                          _stream(stream)))

    def attn_decode_qsa(self, layer: int, slots, pos0, q_idx, Q, T: int, scale: float, out, stream=None) -> None:
        self._check(lib().qkv_attn_decode_qsa(self.handle, layer, _i32_array(slots), _i32_array(pos0), len(slots),
                                               _ptr(q_idx), _ptr(Q), T, scale, _ptr(out), _stream(stream)))

    def attn_prefill_qsa(self, layer: int, slot: int, pos0: int, q_idx, Q, Tc: int, scale: float, out,
                         blocks_out=None, n_out=None, stream=None) -> None:
        """Sparse prefill: each query row attends to the cells of its kept indexer blocks."""
        self._check(lib().qkv_attn_prefill_qsa(self.handle, layer, slot, pos0, _ptr(q_idx), _ptr(Q), Tc, scale, _ptr(out),
                                                _ptr(blocks_out), _ptr(n_out), _stream(stream)))

    def idx_read(self, layer: int, slot: int, pos: int = 0, n: int = 0, keys_out=None, b0: int = 0, n_blk: int = 0,
                 pooled_out=None, stream=None) -> None:
        self._check(lib().qkv_idx_read(self.handle, layer, slot, pos, n, _ptr(keys_out), b0, n_blk, _ptr(pooled_out),
                                        _stream(stream)))

    # -- snapshots / rollback (engine::snapshot_* surface) -------------------------------------
    def snapshot_save(self, slot: int, stream=None) -> Snapshot:
        h = ctypes.c_void_p()
        self._check(lib().qkv_snapshot_save(self.handle, slot, ctypes.byref(h),
                                            _stream(stream) if self.device >= 0 else None))
        return Snapshot(self, h.value)

    def snapshot_load(self, snap: Snapshot, slot: int, n_keep: int = -1, stream=None) -> None:
        self._check(lib().qkv_snapshot_restore(self.handle, snap.handle, slot, n_keep,
                                               _stream(stream) if self.device >= 0 else None))

    def snapshot_load_many(self, snap: Snapshot, slots, n_keep=None, stream=None) -> None:
        keep = _i32_array(n_keep) if n_keep is not None else None
        self._check(lib().qkv_snapshot_restore_many(self.handle, snap.handle, _i32_array(slots), keep, len(slots),
                                                    _stream(stream) if self.device >= 0 else None))

    def snapshot_to_host(self, snap: Snapshot, stream=None) -> bytearray:
        _, nbytes = snap.info()
        buf = bytearray(nbytes)
        cbuf = (ctypes.c_char * max(1, nbytes)).from_buffer(buf) if nbytes else ctypes.create_string_buffer(1)
        self._check(lib().qkv_snapshot_to_host(self.handle, snap.handle, ctypes.addressof(cbuf), nbytes,
                                               _stream(stream)))
        return buf

    def snapshot_from_host(self, blob: bytes | bytearray, n_past: int, stream=None) -> Snapshot:
        b = bytearray(blob)
        cbuf = (ctypes.c_char * max(1, len(b))).from_buffer(b)
        h = ctypes.c_void_p()
        self._check(lib().qkv_snapshot_from_host(self.handle, ctypes.addressof(cbuf), len(blob), n_past,
                                                 ctypes.byref(h), _stream(stream)))
        return Snapshot(self, h.value)

    def rollback_arm(self, slot: int, depth: int) -> None:
        self._check(lib().qkv_rollback_arm(self.handle, slot, depth))

    def rollback_n(self, slot: int, n_back: int, stream=None) -> None:
        self._check(lib().qkv_rollback(self.handle, slot, n_back, _stream(stream) if self.device >= 0 else None))
