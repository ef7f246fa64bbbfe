"""GGUF Q8_0 / Q4_K block formats: sizes and numpy quantisers.

The reference engine only reads these formats (engine/quant.py:133-181 decodes
them); this module writes them, so synthetic layers can be built with known
bytes. The CUDA library decodes the same bytes on the device, and its own
quantiser kernel (aero_cuda_quantize) produces bit-identical blocks for large
tensors.

Q8_0 (34 bytes / 32 values): fp16 d, then 32 int8. The quantiser is ggml's
published Q8_0 rule: d = amax/127, q = round-half-away(x / d) using the f32 d
(gguf-py 0.19.0 `Q8_0.quantize_blocks` states the same rule).

Q4_K (144 bytes / 256 values): fp16 d, fp16 dmin, 12 bytes of 6-bit sub-block
scales/mins, 128 bytes of nibbles; value = d*sc_j*q - dmin*m_j. Low nibbles of
bytes [32g, 32g+32) are sub-block 2g, high nibbles sub-block 2g+1. ggml's own
Q4_K search (make_qkx2_quants) is not part of the reference; this module uses a
simple, fully specified min/max rule instead:
    per 32-value sub-block j:  lo_j = min(0, min x), span_j = (max x - lo_j) / 15,
                               mval_j = -lo_j
    per super-block:           d = max_j span_j / 63, dmin = max_j mval_j / 63,
                               both stored as fp16 (dq, dminq = their f32 values)
    sc_j = min(63, rnd(span_j / dq)) (0 when dq == 0); m_j likewise with dminq
    q = clamp(rnd((x + dminq*m_j) / (dq*sc_j)), 0, 15) (0 when dq*sc_j == 0)
where rnd rounds half away from zero. All arithmetic is single IEEE f32
operations, so the CUDA quantiser reproduces it exactly.
"""

from __future__ import annotations

import numpy as np

DTYPE_F32 = 0
DTYPE_F16 = 1
DTYPE_Q8_0 = 8
DTYPE_Q4_K = 12

QK_K = 256

# (block_bytes, values_per_block)
BLOCK = {DTYPE_F32: (4, 1), DTYPE_Q8_0: (34, 32), DTYPE_Q4_K: (144, QK_K)}

TYPE_NAMES = {DTYPE_F32: "F32", DTYPE_Q8_0: "Q8_0", DTYPE_Q4_K: "Q4_K"}


def type_size(dtype: int, n_values: int) -> int:
    """Bytes occupied by n_values of `dtype` (whole blocks only)."""
    if dtype not in BLOCK:
        raise NotImplementedError(f"unsupported ggml type {dtype}")
    bb, bv = BLOCK[dtype]
    if n_values % bv:
        raise ValueError(f"type {dtype}: {n_values} is not a multiple of {bv}")
    return (n_values // bv) * bb


def _rnd(v: np.ndarray) -> np.ndarray:
    """Round half away from zero, in f32."""
    a = np.abs(v)
    f = np.floor(a)
    return (np.sign(v) * (f + np.floor(np.float32(2) * (a - f)))).astype(np.float32)


def quantize_q8_0(x: np.ndarray) -> bytes:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, 32)
    d = (np.abs(x).max(axis=1, keepdims=True) / np.float32(127)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    q = _rnd((x * inv).astype(np.float32)).astype(np.int8)
    out = np.empty((x.shape[0], 34), dtype=np.uint8)
    out[:, :2] = d.astype(np.float16).view(np.uint8)
    out[:, 2:] = q.view(np.uint8)
    return out.tobytes()


def quantize_q4_k(x: np.ndarray) -> bytes:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, 8, 32)
    nb = x.shape[0]
    lo = np.minimum(x.min(axis=2), np.float32(0))                  # (nb, 8)
    span = ((x.max(axis=2) - lo) / np.float32(15)).astype(np.float32)
    mval = (-lo).astype(np.float32)
    d = (span.max(axis=1) / np.float32(63)).astype(np.float32)     # (nb,)
    dmin = (mval.max(axis=1) / np.float32(63)).astype(np.float32)
    d16 = d.astype(np.float16)
    dm16 = dmin.astype(np.float16)
    dq = d16.astype(np.float32)[:, None]
    dmq = dm16.astype(np.float32)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(dq > 0, np.minimum(_rnd(span / dq), 63), 0).astype(np.uint8)
        mn = np.where(dmq > 0, np.minimum(_rnd(mval / dmq), 63), 0).astype(np.uint8)
        eff_s = (dq * sc.astype(np.float32)).astype(np.float32)[:, :, None]
        eff_m = (dmq * mn.astype(np.float32)).astype(np.float32)[:, :, None]
        num = (x + eff_m).astype(np.float32)
        qf = np.where(eff_s > 0, _rnd((num / eff_s).astype(np.float32)), 0)
    q = np.clip(qf, 0, 15).astype(np.uint8)                         # (nb, 8, 32)

    out = np.zeros((nb, 144), dtype=np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = dm16.view(np.uint8).reshape(nb, 2)
    for j in range(4):
        out[:, 4 + j] = (sc[:, j] & 63) | ((sc[:, j + 4] >> 4) << 6)
        out[:, 8 + j] = (mn[:, j] & 63) | ((mn[:, j + 4] >> 4) << 6)
        out[:, 12 + j] = (sc[:, j + 4] & 15) | ((mn[:, j + 4] & 15) << 4)
    for g in range(4):
        out[:, 16 + 32 * g:16 + 32 * g + 32] = q[:, 2 * g, :] | (q[:, 2 * g + 1, :] << 4)
    return out.tobytes()


def quantize(x: np.ndarray, dtype: int) -> bytes:
    """Quantise a row-major f32 array to GGUF bytes of `dtype`."""
    if dtype == DTYPE_F32:
        return np.ascontiguousarray(x, dtype=np.float32).tobytes()
    if dtype == DTYPE_Q8_0:
        return quantize_q8_0(x)
    if dtype == DTYPE_Q4_K:
        return quantize_q4_k(x)
    raise NotImplementedError(f"quantize: unsupported type {dtype}")
