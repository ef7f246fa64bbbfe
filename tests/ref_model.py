"""ctypes binding of the reference's native block loop (include/aero/model.hpp:170-215),
compiled from the reference's own sources into oracle/_ref/libaero_model.so by
oracle/Makefile. Test infrastructure: the golden generator drives it with the
reference's MoE block as the MoE hook; the block-loop tests drive it with this
library's aero_cuda_moe_model_forward as the hook."""

import ctypes
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_MODEL = os.path.join(ROOT, "oracle", "_ref", "libaero_model.so")


class Geom(ctypes.Structure):
    """aero_geom (include/aero/model.hpp:180-186)."""
    _fields_ = [("arch", ctypes.c_int32), ("n_layer", ctypes.c_int32), ("n_embd", ctypes.c_int32),
                ("vocab", ctypes.c_int32), ("eps", ctypes.c_float), ("tied_output", ctypes.c_int32),
                ("softcap", ctypes.c_float), ("embed_scale", ctypes.c_float),
                ("block_on_output", ctypes.c_int32), ("gemma_out_scale", ctypes.c_int32),
                ("threads", ctypes.c_int32), ("block_rows", ctypes.c_int32)]


class LayerGeom(ctypes.Structure):
    """aero_layer_geom (include/aero/model.hpp:188-191)."""
    _fields_ = [("kind", ctypes.c_int32), ("is_moe", ctypes.c_int32), ("out_scale", ctypes.c_float)]


MOE_HOOK = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_float), ctypes.c_int,
                            ctypes.c_int, ctypes.POINTER(ctypes.c_float))


def available() -> bool:
    return os.path.exists(REF_MODEL)


def load():
    lib = ctypes.CDLL(REF_MODEL)
    lib.aero_model_open.restype = ctypes.c_void_p
    lib.aero_model_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(Geom), ctypes.POINTER(LayerGeom),
                                    ctypes.c_char_p, ctypes.c_int]
    lib.aero_model_free.argtypes = [ctypes.c_void_p]
    lib.aero_model_prepare_state.argtypes = [ctypes.c_void_p, ctypes.c_int64]
    lib.aero_model_use_native_hooks.argtypes = [ctypes.c_void_p]
    lib.aero_model_set_moe.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    lib.aero_model_forward.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                       ctypes.c_void_p]
    return lib


def open_model(lib, path: str, spec, n_ctx: int = 64, threads: int = 1):
    """A qwen block loop (arch 1) over a decoder GGUF: every layer attention with its FFN
    through the MoE hook (is_moe = 1), the reference's C++ attention hooks installed."""
    g = Geom(1, spec.n_layer, spec.d, spec.vocab, spec.eps, 1 if spec.tied else 0, 0.0, 0.0, 0, 0, threads, 64)
    lg = (LayerGeom * spec.n_layer)(*[LayerGeom(0, 1, 1.0) for _ in range(spec.n_layer)])
    err = ctypes.create_string_buffer(256)
    m = lib.aero_model_open(path.encode(), ctypes.byref(g), lg, err, 256)
    if not m:
        raise RuntimeError(f"reference model open: {err.value.decode()}")
    if lib.aero_model_prepare_state(m, n_ctx) != 1 or lib.aero_model_use_native_hooks(m) != 1:
        lib.aero_model_free(m)
        raise RuntimeError("reference model state / hooks refused")
    return m
