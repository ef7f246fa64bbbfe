"""Minimal GGUF writer, for building synthetic MoE layers with known bytes.

The device loader that reads GGUF files lives in the CUDA library
(csrc/gguf_loader.cpp, an mmap parser); this writer exists so tests and the
benchmark can produce files in the layout the reference reads
(engine/gguf.py:1-19 describes the container):

    "GGUF" | u32 version=3 | u64 n_tensors | u64 n_kv
    n_kv    x (string key, u32 value type, value)
    n_tensors x (string name, u32 n_dims, u64 dims[n_dims] fastest-first,
                 u32 ggml type, u64 offset relative to the data section)
    zero padding to general.alignment, then the tensor data, each tensor
    starting on an alignment boundary.

Strings are u64 length + UTF-8. Shapes passed to add_tensor are row-major and
are reversed on write, as GGUF stores the fastest-varying dimension first
(engine/gguf.py:72-75).
"""

from __future__ import annotations

import struct
from typing import Any, List, Tuple

GGUF_UINT32 = 4
GGUF_FLOAT32 = 6
GGUF_STRING = 8
GGUF_UINT64 = 10

DEFAULT_ALIGNMENT = 32

_FMT = {GGUF_UINT32: "<I", GGUF_FLOAT32: "<f", GGUF_UINT64: "<Q"}


def _pack_str(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


class GGUFWriter:
    def __init__(self, arch: str, alignment: int = DEFAULT_ALIGNMENT) -> None:
        if alignment <= 0 or alignment & (alignment - 1):
            raise ValueError("alignment must be a power of two")
        self.arch = arch
        self.alignment = alignment
        self._kv: List[Tuple[str, int, Any]] = [
            ("general.architecture", GGUF_STRING, arch),
            ("general.alignment", GGUF_UINT32, alignment),
        ]
        self._tensors: List[Tuple[str, Tuple[int, ...], int, bytes]] = []

    def add_kv(self, key: str, vtype: int, value: Any) -> None:
        self._kv.append((key, vtype, value))

    def add_u32(self, key: str, value: int) -> None:
        self.add_kv(key, GGUF_UINT32, int(value))

    def add_tensor(self, name: str, shape: Tuple[int, ...], raw: bytes, ggml_type: int) -> None:
        self._tensors.append((name, tuple(int(d) for d in shape), int(ggml_type), bytes(raw)))

    def to_bytes(self) -> bytes:
        head = bytearray(b"GGUF")
        head += struct.pack("<IQQ", 3, len(self._tensors), len(self._kv))
        for key, vt, v in self._kv:
            head += _pack_str(key) + struct.pack("<I", vt)
            head += _pack_str(v) if vt == GGUF_STRING else struct.pack(_FMT[vt], v)
        offsets, cur = [], 0
        for _n, _s, _t, raw in self._tensors:
            offsets.append(cur)
            cur += len(raw)
            cur += (-cur) % self.alignment
        for (name, shape, t, _raw), off in zip(self._tensors, offsets):
            head += _pack_str(name) + struct.pack("<I", len(shape))
            for d in reversed(shape):
                head += struct.pack("<Q", d)
            head += struct.pack("<IQ", t, off)
        head += b"\0" * ((-len(head)) % self.alignment)
        data = bytearray()
        for (_n, _s, _t, raw), off in zip(self._tensors, offsets):
            data += b"\0" * (off - len(data))
            data += raw
        data += b"\0" * ((-len(data)) % self.alignment)
        return bytes(head + data)

    def write(self, path: str) -> None:
        with open(path, "wb") as f:
            f.write(self.to_bytes())


def moe_tensor_names(layer: int) -> dict:
    """The qwen35moe per-layer MoE tensor names (engine/moe.py:5-12)."""
    p = f"blk.{layer}."
    return {
        "router": p + "ffn_gate_inp.weight",
        "shexp_gate_inp": p + "ffn_gate_inp_shexp.weight",
        "gate": p + "ffn_gate_exps.weight",
        "up": p + "ffn_up_exps.weight",
        "down": p + "ffn_down_exps.weight",
        "shexp_gate": p + "ffn_gate_shexp.weight",
        "shexp_up": p + "ffn_up_shexp.weight",
        "shexp_down": p + "ffn_down_shexp.weight",
    }
