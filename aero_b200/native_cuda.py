"""ctypes binding for libaero_cuda_moe.so, the B200 MoE library.

Same shape as the reference's engine/native.py and engine/native_ssm.py: a
plain C ABI, argtypes declared once in `_load()`, which catches
(OSError, AttributeError) so a stale library that lacks a symbol is reported
instead of crashing the caller (engine/native_ssm.py:104-109).

Unlike the reference there is no fallback: when the library or a GPU is
missing, every compute entry point raises CudaMoeUnavailable.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import (CFUNCTYPE, POINTER, Structure, c_char_p, c_double, c_float, c_int, c_int32, c_int64,
                    c_long, c_size_t, c_uint, c_uint8, c_void_p)

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libaero_cuda_moe.so")

DTYPE_F32 = 0
DTYPE_F16 = 1
DTYPE_Q8_0 = 8
DTYPE_Q4_K = 12

# memory classes (src/memory_guard.cpp MemClass order)
MEM_WEIGHTS_RESIDENT, MEM_WEIGHTS_CACHE, MEM_KV_CACHE, MEM_SCRATCH, MEM_RUNTIME = range(5)

OPT_GEMM_MIN_TOKENS = 1
OPT_ROUTER_TC = 2
OPT_PEER_WAIT_MS = 3
OPT_DECODE_FUSED = 4


class CudaMoeUnavailable(RuntimeError):
    """The CUDA library is not built or no GPU is present. There is no CPU path."""


class Tensor(Structure):
    _fields_ = [("dtype", c_int32), ("reserved", c_int32), ("data", c_void_p), ("nbytes", c_int64)]


class Desc(Structure):
    _fields_ = [
        ("n_embd", c_int32), ("n_expert", c_int32), ("n_expert_used", c_int32), ("ffn_len", c_int32),
        ("norm_topk_prob", c_int32), ("has_shared", c_int32), ("ffn_len_shared", c_int32), ("device", c_int32),
        ("expert_begin", c_int32), ("expert_end", c_int32), ("n_resident", c_int32), ("reserved", c_int32 * 5),
        ("gate_exps", Tensor), ("up_exps", Tensor), ("down_exps", Tensor),
        ("router", c_void_p), ("router_bias", c_void_p), ("shexp_gate_inp", c_void_p),
        ("shexp_gate", Tensor), ("shexp_up", Tensor), ("shexp_down", Tensor),
        ("resident_ids", c_void_p),
    ]


class DecoderLayer(Structure):
    """aero_cuda_decoder_layer (include/aero_cuda_decoder.h)."""
    _fields_ = [("attn_q", Tensor), ("attn_k", Tensor), ("attn_v", Tensor), ("attn_output", Tensor),
                ("attn_norm", c_void_p), ("ffn_norm", c_void_p), ("q_norm", c_void_p), ("k_norm", c_void_p),
                ("moe", c_void_p)]


class DecoderDesc(Structure):
    """aero_cuda_decoder_desc (include/aero_cuda_decoder.h)."""
    _fields_ = [("n_layer", c_int32), ("n_embd", c_int32), ("n_head", c_int32), ("n_head_kv", c_int32),
                ("head_dim", c_int32), ("vocab", c_int32), ("n_seq", c_int32), ("n_ctx", c_int32),
                ("device", c_int32), ("reserved", c_int32), ("eps", c_float), ("rope_base", c_float),
                ("token_embd", Tensor), ("output", Tensor), ("output_norm", c_void_p), ("layers", POINTER(DecoderLayer))]


EVICT_FN = CFUNCTYPE(c_size_t, c_void_p, c_size_t)
BREACH_FN = CFUNCTYPE(None, c_void_p, c_size_t, c_size_t)

_lib = None
_load_error: str | None = None

# (name, restype, argtypes) for every symbol include/aero_cuda_moe.h declares
_P = c_void_p
SYMBOLS = [
    ("aero_cuda_moe_open", c_void_p, [POINTER(Desc), c_char_p, c_int]),
    ("aero_cuda_moe_open_gguf", c_void_p, [c_char_p, c_int, c_int, c_int, c_int, c_char_p, c_int]),
    ("aero_cuda_moe_gguf_info", c_int, [c_char_p, c_int, _P, c_char_p, c_int]),
    ("aero_cuda_moe_close", None, [_P]),
    ("aero_cuda_moe_plan_bytes", c_int64, [POINTER(Desc)]),
    ("aero_cuda_moe_page_in", c_int, [_P, c_int, c_int, _P, _P, _P]),
    ("aero_cuda_moe_resident", c_int, [_P, _P, c_int]),
    ("aero_cuda_moe_model_open_gguf", c_void_p, [c_char_p, c_int, c_int, c_char_p, c_int]),
    ("aero_cuda_moe_model_forward", c_int, [_P, c_int, _P, c_int, c_int, _P]),
    ("aero_cuda_moe_model_layer", c_void_p, [_P, c_int]),
    ("aero_cuda_moe_model_close", None, [_P]),
    ("aero_cuda_decoder_open", c_void_p, [POINTER(DecoderDesc), c_char_p, c_int]),
    ("aero_cuda_decoder_open_gguf", c_void_p, [c_char_p, c_int, c_int, c_int, c_char_p, c_int]),
    ("aero_cuda_decoder_plan_bytes", c_int64, [POINTER(DecoderDesc), _P]),
    ("aero_cuda_decoder_forward", c_int, [_P, _P, c_int, _P, _P]),
    ("aero_cuda_decoder_step", c_int, [_P, _P, _P, _P, c_int, _P]),
    ("aero_cuda_decoder_set_stream", c_int, [_P, _P]),
    ("aero_cuda_decoder_kv", c_int, [_P, c_int, POINTER(c_void_p), POINTER(c_void_p)]),
    ("aero_cuda_decoder_profile", c_int, [_P, c_int, _P]),
    ("aero_cuda_decoder_info", c_int, [_P, _P]),
    ("aero_cuda_decoder_last_error", c_char_p, [_P]),
    ("aero_cuda_decoder_close", None, [_P]),
    ("aero_cuda_moe_forward", c_int, [_P, c_int, _P, c_int, c_int, _P]),
    ("aero_cuda_moe_submit", c_int, [_P, c_int, _P, c_int, _P]),
    ("aero_cuda_moe_wait", c_int, [_P, c_int]),
    ("aero_cuda_moe_ffn_block", c_int, [_P, _P, _P, c_int, _P]),
    ("aero_cuda_moe_router_logits", c_int, [_P, _P, c_int, _P]),
    ("aero_cuda_moe_route", c_int, [_P, _P, c_int, _P, _P]),
    ("aero_cuda_route", c_int, [_P, c_int, c_int, c_int, c_int, _P, _P]),
    ("aero_cuda_dispatch", c_int, [_P, c_int, c_int, c_int, _P, _P]),
    ("aero_cuda_dispatch_noalloc", c_int, [_P, c_int, c_int, c_int, _P, _P, _P]),
    ("aero_cuda_dequant", c_int, [c_int, _P, c_int64, _P, c_int64]),
    ("aero_cuda_quantize", c_int, [c_int, _P, c_int64, _P, c_int64]),
    ("aero_cuda_moe_set_profiling", c_int, [_P, c_int]),
    ("aero_cuda_moe_stage_times", c_int, [_P, _P, _P, c_int]),
    ("aero_cuda_moe_set_option", c_int, [_P, c_int, c_int64]),
    ("aero_cuda_moe_status", c_int, [_P]),
    ("aero_cuda_ep_meta_ld", c_int, [_P]),
    ("aero_cuda_ep_dispatch", c_int, [_P, _P, c_int, c_int, c_int, POINTER(c_int32), c_int, _P, _P, _P, _P, c_int,
                                      _P, _P]),
    ("aero_cuda_ep_expert_block", c_int, [_P, _P, c_int, _P, c_int, c_int, _P, c_int]),
    ("aero_cuda_ep_combine", c_int, [_P, _P, _P, c_int, _P, c_int, c_int, c_int, _P]),
    ("aero_cuda_ep_bad_ids", c_int, [_P]),
    ("aero_cuda_ep_peer_open", c_int, [_P, c_int, c_int, POINTER(c_int32), c_int, c_int, _P]),
    ("aero_cuda_ep_peer_connect", c_int, [_P, _P]),
    ("aero_cuda_ep_peer_step", c_int, [_P, _P, c_int, _P]),
    ("aero_cuda_ep_peer_status", c_int, [_P]),
    ("aero_cuda_ep_peer_counts", c_int, [_P, POINTER(c_int32), POINTER(c_int32)]),
    ("aero_cuda_ep_peer_profile", c_int, [_P, c_int, POINTER(c_double)]),
    ("aero_cuda_ep_peer_close", c_int, [_P]),
    ("aero_cuda_moe_set_stream", c_int, [_P, _P]),
    ("aero_cuda_moe_info", c_int, [_P, POINTER(c_int32)]),
    ("aero_cuda_moe_last_error", c_char_p, [_P]),
    ("aero_cuda_moe_stats", c_int, [_P, c_char_p, c_int]),
    ("aero_cuda_device_count", c_int, []),
    ("aero_cuda_guard_set_budget", None, [c_size_t]),
    ("aero_cuda_guard_budget", c_size_t, []),
    ("aero_cuda_guard_committed", c_size_t, [c_int]),
    ("aero_cuda_guard_headroom", c_size_t, []),
    ("aero_cuda_guard_try_reserve", c_int, [c_size_t, c_int]),
    ("aero_cuda_guard_release", None, [c_size_t, c_int]),
    ("aero_cuda_guard_admit_plan", c_int, [c_size_t, c_char_p, c_int]),
    ("aero_cuda_guard_set_evictor", None, [EVICT_FN, c_void_p]),
    ("aero_cuda_guard_fail_nth_alloc", None, [c_long]),
    ("aero_cuda_guard_own_footprint", c_size_t, [c_int]),
    ("aero_cuda_guard_device_free", c_size_t, [c_int]),
    ("aero_cuda_guard_preflight", c_int, [c_int, c_size_t]),
    ("aero_cuda_guard_set_on_breach", None, [BREACH_FN, c_void_p]),
    ("aero_cuda_guard_exceeded", c_int, []),
    ("aero_cuda_guard_peak_footprint", c_size_t, []),
    ("aero_cuda_guard_reset_exceeded", None, []),
    ("aero_cuda_guard_start_monitor", None, [c_int, c_uint]),
    ("aero_cuda_guard_stop_monitor", None, []),
    ("aero_cuda_loadgate_open", c_void_p, [c_size_t, c_int]),
    ("aero_cuda_loadgate_close", None, [_P]),
    ("aero_cuda_loadgate_set_pause_ms", None, [_P, c_uint]),
    ("aero_cuda_loadgate_next_chunk", c_int, [_P, c_size_t, c_int]),
    ("aero_cuda_loadgate_pause_and_check", c_int, [_P]),
    ("aero_cuda_loadgate_ok", c_int, [_P]),
    ("aero_cuda_loadgate_done", c_int, [_P]),
    ("aero_cuda_loadgate_taken", c_size_t, [_P]),
    ("aero_cuda_loadgate_reserved", c_size_t, [_P]),
    ("aero_cuda_loadgate_remaining", c_size_t, [_P]),
    ("aero_cuda_loadgate_reason", c_int, [_P, c_char_p, c_int]),
]


def _load():
    """Load once; remember the failure so callers get a clear reason."""
    global _lib, _load_error
    if _lib is not None or _load_error is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        _load_error = (f"{LIB_PATH} not found; build it with `python -m aero_b200.build` "
                       "(or __graft_entry__.build())")
        return None
    try:
        lib = ctypes.CDLL(LIB_PATH)
        for name, res, args in SYMBOLS:
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    except (OSError, AttributeError) as e:
        _load_error = f"{LIB_PATH}: {e}"
    return _lib


def available() -> bool:
    return _load() is not None


def unavailable_reason() -> str:
    _load()
    return _load_error or ""


def lib():
    """The loaded library, or CudaMoeUnavailable."""
    l = _load()
    if l is None:
        raise CudaMoeUnavailable(unavailable_reason())
    return l


def gpu_count() -> int:
    return int(lib().aero_cuda_device_count())


def require_gpu() -> None:
    if gpu_count() <= 0:
        raise CudaMoeUnavailable("no CUDA device is visible; aero_b200 has no CPU path")


def last_error(handle=None) -> str:
    r = lib().aero_cuda_moe_last_error(handle)
    return r.decode() if r else ""


# ---- buffers ----------------------------------------------------------------
def ptr(a) -> int:
    """Address of a numpy array or a torch tensor (host or device)."""
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    raise TypeError(f"expected a numpy array or torch tensor, got {type(a)}")


def f32c(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _is_torch(a) -> bool:
    return hasattr(a, "data_ptr") and hasattr(a, "is_cuda")


# ---- thin wrappers ------------------------------------------------------------
def route(logits, n_expert: int, k: int, norm_topk_prob: bool = True):
    """Batched top-k on the GPU. logits (E,) or (T, E) -> idx int64, w f32 of
    shape (k,) or (T, k), matching engine/native_ssm.py route()."""
    L = lib()
    require_gpu()
    lg = f32c(logits)
    single = lg.ndim == 1
    lg2 = lg.reshape(1, -1) if single else lg.reshape(lg.shape[0], -1)
    T = lg2.shape[0]
    if lg2.shape[1] != n_expert:
        raise ValueError(f"logits have width {lg2.shape[1]}, expected {n_expert}")
    idx = np.empty((T, max(k, 0)), dtype=np.int64)
    w = np.empty((T, max(k, 0)), dtype=np.float32)
    rc = L.aero_cuda_route(ptr(lg2), T, int(n_expert), int(k), 1 if norm_topk_prob else 0, ptr(idx), ptr(w))
    if rc != 0:
        raise ValueError(f"route refused k={k} for n_expert={n_expert}: {last_error()}")
    return (idx[0], w[0]) if single else (idx, w)


def dispatch(idx, n_expert: int):
    """(offsets (E+1,), perm (T*k,)) for routed expert indices idx (T, k)."""
    L = lib()
    require_gpu()
    ix = np.ascontiguousarray(idx, dtype=np.int64)
    T, k = ix.shape
    offsets = np.empty(n_expert + 1, dtype=np.int32)
    perm = np.empty(T * k, dtype=np.int32)
    if L.aero_cuda_dispatch(ptr(ix), T, k, int(n_expert), ptr(offsets), ptr(perm)) != 0:
        raise ValueError(f"dispatch refused: {last_error()}")
    return offsets, perm


def dequant(dtype: int, raw: bytes, n_values: int) -> np.ndarray:
    """GGUF bytes -> f32 on the GPU (bit-identical to aero_dequant_ref)."""
    L = lib()
    require_gpu()
    buf = np.frombuffer(raw, dtype=np.uint8)
    out = np.empty(n_values, dtype=np.float32)
    if L.aero_cuda_dequant(int(dtype), ptr(buf), buf.size, ptr(out), int(n_values)) != 1:
        raise ValueError(f"dequant refused (type {dtype}, {buf.size} bytes for {n_values} values)")
    return out


def quantize(dtype: int, x) -> bytes:
    """f32 -> GGUF bytes on the GPU (equal to aero_b200.quant.quantize). x may be
    a numpy array or a CUDA torch tensor; the bytes come back to the host."""
    L = lib()
    require_gpu()
    from .quant import type_size
    if _is_torch(x):
        n = x.numel()
        out = np.empty(type_size(dtype, n), dtype=np.uint8)
        rc = L.aero_cuda_quantize(int(dtype), x.data_ptr(), n, ptr(out), out.size)
    else:
        xa = f32c(x).reshape(-1)
        out = np.empty(type_size(dtype, xa.size), dtype=np.uint8)
        rc = L.aero_cuda_quantize(int(dtype), ptr(xa), xa.size, ptr(out), out.size)
    if rc != 1:
        raise ValueError(f"quantize refused (type {dtype})")
    return out.tobytes()


class MemoryGuard:
    """Process-wide device memory guard (the reference's engine/native.py:297-353
    MemoryGuard, backed here by the CUDA library's guard)."""

    def __init__(self) -> None:
        self._lib = lib()
        self._cbs = []

    def set_budget(self, n: int) -> None:
        self._lib.aero_cuda_guard_set_budget(int(n))

    def budget(self) -> int:
        return int(self._lib.aero_cuda_guard_budget())

    def committed(self, cls: int = -1) -> int:
        return int(self._lib.aero_cuda_guard_committed(int(cls)))

    def headroom(self) -> int:
        return int(self._lib.aero_cuda_guard_headroom())

    def try_reserve(self, n: int, cls: int = MEM_SCRATCH) -> bool:
        return bool(self._lib.aero_cuda_guard_try_reserve(int(n), int(cls)))

    def release(self, n: int, cls: int = MEM_SCRATCH) -> None:
        self._lib.aero_cuda_guard_release(int(n), int(cls))

    def admit_plan(self, n: int):
        buf = ctypes.create_string_buffer(256)
        ok = bool(self._lib.aero_cuda_guard_admit_plan(int(n), buf, 256))
        return ok, buf.value.decode()

    def set_evictor(self, fn) -> None:
        if fn is None:
            self._lib.aero_cuda_guard_set_evictor(EVICT_FN(), None)
            return
        cb = EVICT_FN(lambda ctx, need: int(fn(int(need))))
        self._cbs.append(cb)
        self._lib.aero_cuda_guard_set_evictor(cb, None)

    def fail_nth_alloc(self, n: int) -> None:
        self._lib.aero_cuda_guard_fail_nth_alloc(int(n))

    def own_footprint(self, device: int = 0) -> int:
        return int(self._lib.aero_cuda_guard_own_footprint(int(device)))

    def preflight(self, device: int = 0, headroom: int = 0) -> bool:
        return bool(self._lib.aero_cuda_guard_preflight(int(device), int(headroom)))

    def exceeded(self) -> bool:
        return bool(self._lib.aero_cuda_guard_exceeded())


class LoadGate:
    """Chunked-load gate (src/memory_guard.cpp:314-378)."""

    def __init__(self, planned: int, device: int = 0) -> None:
        self._lib = lib()
        self._h = self._lib.aero_cuda_loadgate_open(int(planned), int(device))

    def __del__(self):
        h, self._h = getattr(self, "_h", None), None
        if h and _lib is not None:
            _lib.aero_cuda_loadgate_close(h)

    def next_chunk(self, n: int, cls: int = MEM_WEIGHTS_CACHE) -> bool:
        return bool(self._lib.aero_cuda_loadgate_next_chunk(self._h, int(n), int(cls)))

    def set_chunk_pause_ms(self, ms: int) -> None:
        self._lib.aero_cuda_loadgate_set_pause_ms(self._h, int(ms))

    def pause_and_check(self) -> bool:
        return bool(self._lib.aero_cuda_loadgate_pause_and_check(self._h))

    def ok(self) -> bool:
        return bool(self._lib.aero_cuda_loadgate_ok(self._h))

    def done(self) -> bool:
        return bool(self._lib.aero_cuda_loadgate_done(self._h))

    def taken(self) -> int:
        return int(self._lib.aero_cuda_loadgate_taken(self._h))

    def reserved(self) -> int:
        return int(self._lib.aero_cuda_loadgate_reserved(self._h))

    def remaining(self) -> int:
        return int(self._lib.aero_cuda_loadgate_remaining(self._h))

    def reason(self) -> str:
        buf = ctypes.create_string_buffer(512)
        self._lib.aero_cuda_loadgate_reason(self._h, buf, 512)
        return buf.value.decode()
