"""The decoder around the MoE layer on the GPU (include/aero_cuda_decoder.h).

`CudaDecoder.forward(tokens, positions)` keeps the reference's
aero_model_forward contract (src/model.cpp:389-392; ModelNative::forward,
src/model.cpp:290-330): the tokens of sequence 0 at their positions, the logits
of the last one. `step(tokens, seqs, positions)` runs tokens of several
sequences at once (batched decode, or a prompt in one call) and returns one
logits row per token. The cache is f16, one region per sequence.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np

from . import native_cuda as nc
from .moe import CudaMoeLayer


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a).reshape(-1), dtype=np.int32)


def _i64(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a).reshape(-1), dtype=np.int64)


def plan_footprint(spec, n_seq: int = 1, n_ctx: int = 4096) -> dict:
    """Device bytes the decoder of a synth.DecoderSpec holds once open, as the memory
    guard charges them: the decoder's weights and caches (aero_cuda_decoder_plan_bytes)
    and every layer's MoE handle (aero_cuda_moe_plan_bytes: router rows, the
    tensor-core router's split copy, the quantised expert planes). Replaces the
    reference's plan_footprint (engine/model.py:776-840), whose expert term
    (:828-832) counts the fp32 bytes of the active experts, for this device layout.
    The descriptions passed to the library carry shapes and types only (their
    pointers are tested for presence, never read)."""
    L = nc.lib()
    present = ctypes.c_void_p(1).value
    layers = (nc.DecoderLayer * spec.n_layer)()
    for ly in layers:
        ly.attn_q.dtype = ly.attn_k.dtype = ly.attn_v.dtype = ly.attn_output.dtype = spec.attn_dtype
        if spec.qk_norm:
            ly.q_norm = ly.k_norm = present
    d = nc.DecoderDesc()
    d.n_layer, d.n_embd, d.n_head, d.n_head_kv, d.head_dim, d.vocab = (spec.n_layer, spec.d, spec.n_head, spec.n_kv,
                                                                      spec.head_dim, spec.vocab)
    d.n_seq, d.n_ctx = int(n_seq), int(n_ctx)
    d.token_embd.dtype = spec.embd_dtype
    if not spec.tied:
        d.output.dtype, d.output.data = spec.embd_dtype, present
    d.layers = layers
    by = (ctypes.c_int64 * 2)()
    if L.aero_cuda_decoder_plan_bytes(ctypes.byref(d), by) < 0:
        raise ValueError("invalid decoder description")
    m = spec.moe
    md = nc.Desc()
    md.n_embd, md.n_expert, md.n_expert_used, md.ffn_len = m.d, m.E, m.k, m.F
    md.router = present
    md.gate_exps.dtype = md.up_exps.dtype = md.down_exps.dtype = m.dtype
    if m.Fs:
        md.has_shared, md.ffn_len_shared = 1, m.Fs
        md.shexp_gate.dtype = md.shexp_up.dtype = md.shexp_down.dtype = m.dtype
    moe = L.aero_cuda_moe_plan_bytes(ctypes.byref(md))
    if moe < 0:
        raise ValueError("invalid MoE description")
    weights = int(by[0]) + spec.n_layer * int(moe)
    return {"weights_resident": weights, "kv_cache": int(by[1]), "moe_weights": spec.n_layer * int(moe),
            "total": weights + int(by[1])}


class CudaDecoder:
    def __init__(self, handle: int, keep=None) -> None:
        if not handle:
            raise RuntimeError("null decoder")
        self._lib = nc.lib()
        self.handle = handle
        info = (ctypes.c_int64 * 8)()
        self._lib.aero_cuda_decoder_info(handle, info)
        (self.n_layer, self.n_embd, self.n_head, self.n_head_kv, self.head_dim, self.vocab, self.n_seq,
         self.n_ctx) = (int(v) for v in info)
        self._keep = keep or []

    # ---- construction
    @classmethod
    def from_gguf(cls, path: str, n_seq: int = 1, n_ctx: int = 4096, device: int = 0) -> "CudaDecoder":
        L = nc.lib()
        nc.require_gpu()
        err = ctypes.create_string_buffer(512)
        h = L.aero_cuda_decoder_open_gguf(str(path).encode(), int(device), int(n_seq), int(n_ctx), err, 512)
        if not h:
            raise RuntimeError(f"decoder open ({path}): {err.value.decode()}")
        return cls(h)

    @classmethod
    def from_synth(cls, dec, n_seq: int = 1, n_ctx: int = 4096, device: int = 0) -> "CudaDecoder":
        """Open a synth.SynthDecoder: its MoE layers as CudaMoeLayer handles (kept alive
        by the decoder object), the rest from its tensors (host or device bytes)."""
        from .synth import open_layer
        L = nc.lib()
        nc.require_gpu()
        sp = dec.spec
        keep = []
        moes = [open_layer(m, device=device) for m in dec.moe]
        keep.extend(moes)

        def tensor(name):
            shape, dt, raw = dec.tensors[name]
            if hasattr(raw, "data_ptr"):
                t = raw.contiguous()
                keep.append(t)
                return nc.Tensor(dt, 0, t.data_ptr(), t.numel() * t.element_size())
            a = np.ascontiguousarray(raw)
            keep.append(a)
            return nc.Tensor(dt, 0, a.ctypes.data, a.nbytes)

        def f32(name):
            if name not in dec.tensors:
                return None
            a = np.ascontiguousarray(dec.tensors[name][2], dtype=np.float32)
            keep.append(a)
            return a.ctypes.data

        layers = (nc.DecoderLayer * sp.n_layer)()
        for i in range(sp.n_layer):
            p = f"blk.{i}."
            ly = layers[i]
            ly.attn_q, ly.attn_k = tensor(p + "attn_q.weight"), tensor(p + "attn_k.weight")
            ly.attn_v, ly.attn_output = tensor(p + "attn_v.weight"), tensor(p + "attn_output.weight")
            ly.attn_norm, ly.ffn_norm = f32(p + "attn_norm.weight"), f32(p + "post_attention_norm.weight")
            ly.q_norm, ly.k_norm = f32(p + "attn_q_norm.weight"), f32(p + "attn_k_norm.weight")
            ly.moe = moes[i].handle
        d = nc.DecoderDesc()
        d.n_layer, d.n_embd, d.n_head, d.n_head_kv, d.head_dim, d.vocab = (sp.n_layer, sp.d, sp.n_head, sp.n_kv,
                                                                          sp.head_dim, sp.vocab)
        d.n_seq, d.n_ctx, d.device = int(n_seq), int(n_ctx), int(device)
        d.eps, d.rope_base = float(sp.eps), float(sp.rope_base)
        d.token_embd = tensor("token_embd.weight")
        if not sp.tied:
            d.output = tensor("output.weight")
        d.output_norm = f32("output_norm.weight")
        d.layers = layers
        err = ctypes.create_string_buffer(512)
        h = L.aero_cuda_decoder_open(ctypes.byref(d), err, 512)
        if not h:
            for m in moes:
                m.close()
            raise RuntimeError(f"decoder open: {err.value.decode()}")
        # the weights are on the device now; the MoE handles stay borrowed by the decoder
        return cls(h, list(moes))

    # ---- compute
    def forward(self, tokens, positions, logits=None) -> np.ndarray:
        """aero_model_forward on sequence 0: logits (vocab,) of the last token."""
        tk, ps = _i32(tokens), _i64(positions)
        if tk.size != ps.size:
            raise ValueError("tokens and positions differ in length")
        out = np.empty(self.vocab, np.float32) if logits is None else logits
        ptr = out.data_ptr() if hasattr(out, "data_ptr") else out.ctypes.data
        if self._lib.aero_cuda_decoder_forward(self.handle, tk.ctypes.data, tk.size, ps.ctypes.data, ptr) != 1:
            raise RuntimeError(f"decoder forward refused: {self.last_error()}")
        return out

    def step(self, tokens, seqs, positions, logits: Optional[object] = "host"):
        """One step over T tokens of their sequences; logits (T, vocab) on the host, or
        into a given device tensor, or None (the cache is filled, no head)."""
        tk, sq, ps = _i32(tokens), _i32(seqs), _i64(positions)
        if not (tk.size == sq.size == ps.size):
            raise ValueError("tokens, seqs and positions differ in length")
        out, ptr = None, None
        if isinstance(logits, str):
            out = np.empty((tk.size, self.vocab), np.float32)
            ptr = out.ctypes.data
        elif logits is not None:
            out, ptr = logits, logits.data_ptr()
        if self._lib.aero_cuda_decoder_step(self.handle, tk.ctypes.data, sq.ctypes.data, ps.ctypes.data, tk.size,
                                            ptr) != 0:
            raise RuntimeError(f"decoder step refused: {self.last_error()}")
        return out

    def set_stream(self, stream) -> None:
        """Run on a cudaStream_t (int) or torch.cuda.Stream; None restores the decoder's own."""
        st = getattr(stream, "cuda_stream", stream)
        self._lib.aero_cuda_decoder_set_stream(self.handle, st or None)

    def kv(self, layer: int):
        """Device addresses of the layer's key and value caches."""
        k, v = ctypes.c_void_p(), ctypes.c_void_p()
        if self._lib.aero_cuda_decoder_kv(self.handle, int(layer), ctypes.byref(k), ctypes.byref(v)) != 0:
            raise ValueError(f"no layer {layer}")
        return k.value, v.value

    PHASES = ("embed_norm", "projections", "attention", "moe", "head")

    def profile(self, on: bool = True) -> dict:
        """Switch phase timing; returns (and resets) the device ms accumulated so far."""
        ms = np.zeros(5, np.float64)
        self._lib.aero_cuda_decoder_profile(self.handle, 1 if on else 0, ms.ctypes.data)
        return dict(zip(self.PHASES, (float(v) for v in ms)))

    def last_error(self) -> str:
        r = self._lib.aero_cuda_decoder_last_error(self.handle)
        return r.decode() if r else ""

    def close(self) -> None:
        h, self.handle = self.handle, None
        if h:
            self._lib.aero_cuda_decoder_close(h)
        for m in self._keep:
            if isinstance(m, CudaMoeLayer):
                m.close()
        self._keep = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
