"""Python access to the parity oracle — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs may import this module, and only as the checker or the timed CPU
baseline. The product (aero_b200/) never imports it.

Two oracles:
  * liboracle_moe.so — the C restatement in moe_oracle.c (always buildable);
  * _ref/librefdrive.so + _ref/libaero_ssm.so — the reference's OWN
    src/moe.cpp / src/kernels.cpp, compiled from the reference tree by the
    Makefile here when that tree is present (this container); the GPU box only
    sees the prebuilt files.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import c_int, c_int64, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "liboracle_moe.so")
REF_DIR = os.path.join(HERE, "_ref")
REFDRIVE_LIB = os.path.join(REF_DIR, "librefdrive.so")
REF_SSM_LIB = os.path.join(REF_DIR, "libaero_ssm.so")

_orc = None
_ref = None


def reference_root() -> str:
    """The reference checkout: $AERO_REF, else a "reference" directory beside this repository."""
    return os.environ.get("AERO_REF") or os.path.abspath(os.path.join(HERE, "..", "..", "reference"))


def build(ref_root: str = "") -> None:
    """make the oracle (and the reference objects when the reference tree exists)."""
    args = ["make", "-s", "-C", HERE, "all", f"REF={ref_root or reference_root()}"]
    subprocess.run(args, check=True, capture_output=True)


def lib():
    global _orc
    if _orc is None:
        if not os.path.exists(ORACLE_LIB):
            subprocess.run(["make", "-s", "-C", HERE, "oracle"], check=True, capture_output=True)
        L = ctypes.CDLL(ORACLE_LIB)
        P = c_void_p
        L.orc_dequant.argtypes = [c_int, P, c_int64, P, c_int64]
        L.orc_dequant.restype = c_int
        L.orc_route.argtypes = [P, c_int, c_int, c_int, c_int, P, P]
        L.orc_route.restype = c_int
        L.orc_argsort_desc.argtypes = [P, c_int, P]
        L.orc_expert_accum.argtypes = [P, c_int, P, P, P, c_int, ctypes.c_float, P]
        L.orc_shared_accum.argtypes = [P, c_int, c_int, P, P, P, P, c_int, P]
        L.orc_router_logits.argtypes = [P, c_int, c_int, P, c_int, P, c_int, P]
        L.orc_dispatch.argtypes = [P, c_int, c_int, c_int, P, P]
        L.orc_moe_block_q.argtypes = [P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_int, P, P, P,
                                      c_int, P, c_int, P, P, P, c_int, c_int, P]
        L.orc_moe_block_q.restype = c_int
        _orc = L
    return _orc


def ref_available() -> bool:
    return os.path.exists(REFDRIVE_LIB) and os.path.exists(REF_SSM_LIB)


def ref_lib():
    """The reference's own MoE block (compiled from its sources) + our fetch driver."""
    global _ref
    if _ref is None:
        if not ref_available():
            raise FileNotFoundError(f"{REFDRIVE_LIB} not built (needs the reference sources at build time)")
        ssm = ctypes.CDLL(REF_SSM_LIB, mode=ctypes.RTLD_GLOBAL)
        L = ctypes.CDLL(REFDRIVE_LIB)
        P = c_void_p
        L.refdrive_block.argtypes = [P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_int, P, P, P, c_int,
                                     P, P, P, P, c_int, P]
        L.refdrive_block.restype = c_int
        ssm.aero_moe_route.argtypes = [P, c_int, c_int, c_int, P, P]
        ssm.aero_moe_route.restype = c_int
        ssm.aero_dequant_ref.argtypes = [c_int, P, c_int64, P, c_int64]
        ssm.aero_dequant_ref.restype = c_int
        _ref = (L, ssm)
    return _ref


def _p(a):
    return None if a is None else a.ctypes.data


def _f(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _u8(b):
    return np.frombuffer(b, dtype=np.uint8) if isinstance(b, (bytes, bytearray)) else np.ascontiguousarray(b)


# ------------------------------------------------------------ restatement
def dequant(dtype: int, raw, n: int) -> np.ndarray:
    r = _u8(raw)
    out = np.empty(n, dtype=np.float32)
    if lib().orc_dequant(dtype, r.ctypes.data, r.size, out.ctypes.data, n) != 1:
        raise ValueError("dequant refused")
    return out


def route(logits, k: int, norm: bool = True):
    lg = _f(logits)
    single = lg.ndim == 1
    lg2 = lg.reshape(1, -1) if single else lg
    T, E = lg2.shape
    idx = np.empty((T, k), dtype=np.int64)
    w = np.empty((T, k), dtype=np.float32)
    if lib().orc_route(lg2.ctypes.data, T, E, k, 1 if norm else 0, idx.ctypes.data, w.ctypes.data) != 0:
        raise ValueError(f"route refused k={k} for n_expert={E}")
    return (idx[0], w[0]) if single else (idx, w)


def argsort_desc(logits) -> np.ndarray:
    lg = _f(logits)
    out = np.empty(lg.size, dtype=np.int32)
    lib().orc_argsort_desc(lg.ctypes.data, lg.size, out.ctypes.data)
    return out


def dispatch(idx, E: int):
    ix = np.ascontiguousarray(idx, dtype=np.int64)
    T, k = ix.shape
    off = np.empty(E + 1, dtype=np.int32)
    perm = np.empty(T * k, dtype=np.int32)
    lib().orc_dispatch(ix.ctypes.data, T, k, E, off.ctypes.data, perm.ctypes.data)
    return off, perm


def router_logits(h, W, bias=None, f64: bool = False) -> np.ndarray:
    h = _f(h)
    W = _f(W)
    T, d = h.shape
    E = W.shape[0]
    out = np.empty((T, E), dtype=np.float32)
    b = None if bias is None else _f(bias)
    lib().orc_router_logits(h.ctypes.data, T, d, W.ctypes.data, E, _p(b), 1 if f64 else 0, out.ctypes.data)
    return out


def moe_block(layer, h, logits, nthreads: int = 1) -> np.ndarray:
    """The block over the layer's quantised bytes (aero_b200.synth.SynthLayer)."""
    sp = layer.spec
    h = _f(h)
    lg = _f(logits)
    T = h.shape[0]
    out = np.zeros((T, sp.d), dtype=np.float32)
    sh = layer.shexp
    g, u, dn = _u8(layer.gate), _u8(layer.up), _u8(layer.down)
    if sp.dtype == 0:
        g, u, dn = (np.ascontiguousarray(v, dtype=np.float32) for v in (layer.gate, layer.up, layer.down))
    args = [h.ctypes.data, lg.ctypes.data, T, sp.d, sp.E, sp.k, sp.F, 1 if sp.norm_topk_prob else 0, sp.dtype,
            g.ctypes.data, u.ctypes.data, dn.ctypes.data]
    keep = []
    if sh:
        gi = _f(sh["gate_inp"]).reshape(-1)
        sg, su, sd = (_u8(sh[k]) if sh["dtype"] != 0 else _f(sh[k]) for k in ("gate", "up", "down"))
        keep += [gi, sg, su, sd]
        args += [1, gi.ctypes.data, sh["dtype"], sg.ctypes.data, su.ctypes.data, sd.ctypes.data, sh["ffn_len"]]
    else:
        args += [0, None, 0, None, None, None, 0]
    args += [nthreads, out.ctypes.data]
    if lib().orc_moe_block_q(*args) != 0:
        raise ValueError("oracle block refused")
    return out


# ------------------------------------------------------------ reference itself
def ref_route(logits, k: int, norm: bool = True):
    _L, ssm = ref_lib()
    lg = _f(logits).reshape(-1)
    idx = np.empty(k, dtype=np.int64)
    w = np.empty(k, dtype=np.float32)
    rc = ssm.aero_moe_route(lg.ctypes.data, lg.size, k, 1 if norm else 0, idx.ctypes.data, w.ctypes.data)
    if rc != 0:
        raise ValueError("reference route refused")
    return idx, w


def ref_block(layer, h, logits, nthreads: int = 1) -> np.ndarray:
    """The reference's aero_moe_ffn_block over the layer (shared expert passed
    as fp32 dequantised by the reference's own aero_dequant_ref)."""
    L, ssm = ref_lib()
    sp = layer.spec
    h = _f(h)
    lg = _f(logits)
    T = h.shape[0]
    out = np.zeros((T, sp.d), dtype=np.float32)
    keep = []
    shp = [0, None, None, None, None]
    if layer.shexp:
        sh = layer.shexp
        if sh["ffn_len"] != sp.F:
            raise ValueError("the reference ABI needs ffn_len_shared == ffn_len (src/moe.cpp:156-159)")
        mats = []
        for key in ("gate", "up", "down"):
            raw = _u8(sh[key])
            m = np.empty(sp.F * sp.d, dtype=np.float32)
            if ssm.aero_dequant_ref(sh["dtype"], raw.ctypes.data, raw.size, m.ctypes.data, m.size) != 1:
                raise ValueError("reference dequant refused")
            mats.append(m)
        gi = _f(sh["gate_inp"]).reshape(-1)
        keep += [gi] + mats
        shp = [1, gi.ctypes.data, mats[0].ctypes.data, mats[1].ctypes.data, mats[2].ctypes.data]
    g, u, dn = _u8(layer.gate), _u8(layer.up), _u8(layer.down)
    rc = L.refdrive_block(h.ctypes.data, lg.ctypes.data, T, sp.d, sp.E, sp.k, sp.F, 1 if sp.norm_topk_prob else 0,
                          sp.dtype, g.ctypes.data, u.ctypes.data, dn.ctypes.data, *shp, nthreads, out.ctypes.data)
    if rc != 0:
        raise ValueError("reference block refused")
    return out
