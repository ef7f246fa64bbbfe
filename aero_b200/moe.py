"""Mixture-of-Experts FFN on the B200: the drop-in for the reference's MoE API.

Mirrors engine/moe.py (MoeConfig :46-57, route :60-94, moe_ffn :117-177,
expert_plan :201-213) and engine/native_ssm.py (route :237-250,
ffn_block :265-314), with the same names, argument meaning and errors
(ValueError for a bad width, a missing router, or k out of range). Every call
runs on the GPU through libaero_cuda_moe.so; there is no numpy fallback, and a
missing library or GPU raises CudaMoeUnavailable.

Two ways to give moe_ffn its experts:
  * a CudaMoeLayer (experts uploaded once, quantised, device-resident) — the
    fast path. With its own router (`layer.router`) the whole block, router
    included, runs on the device; with any other router_fn the logits are
    computed on the host per token, as the reference does, and handed over.
  * any `expert_rows(name, expert, block_rows)` callable returning fp32
    matrices, as in the reference. Only the selected experts are fetched (the
    reference's memory argument), uploaded as f32 for this call, and the block
    runs on the device.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from typing import Optional, Tuple

import numpy as np

from . import native_cuda as nc
from .quant import BLOCK, DTYPE_F32, DTYPE_Q4_K, DTYPE_Q8_0

_NAMES = ("ffn_gate_exps.weight", "ffn_up_exps.weight", "ffn_down_exps.weight")


@dataclass
class MoeConfig:
    n_expert: int
    n_expert_used: int
    n_embd: int
    ffn_len: int
    has_shared: bool = True
    norm_topk_prob: bool = True

    @property
    def routed_width(self) -> int:
        return self.n_expert_used * self.ffn_len


def _check_k(cfg: MoeConfig) -> None:
    k = cfg.n_expert_used
    if k <= 0 or k > cfg.n_expert:
        raise ValueError(f"n_expert_used={k} out of range for {cfg.n_expert} experts")


def route(logits: np.ndarray, cfg: MoeConfig) -> Tuple[np.ndarray, np.ndarray]:
    """Top-k routing of one token's logits (or a (T, E) batch) on the GPU.

    Returns (expert_index int64, weight f32). Ties go to the lower expert index;
    weights are the softmax over the selected logits when norm_topk_prob is set,
    else the full-softmax probability (f64 denominator)."""
    _check_k(cfg)
    return nc.route(logits, cfg.n_expert, cfg.n_expert_used, cfg.norm_topk_prob)


# ---------------------------------------------------------------- device layer
def _as_bytes_view(x):
    """(address, nbytes, keepalive) for bytes / numpy / CUDA torch tensors."""
    if isinstance(x, (bytes, bytearray, memoryview)):
        a = np.frombuffer(x, dtype=np.uint8)
        return a.ctypes.data, a.nbytes, a
    if isinstance(x, np.ndarray):
        a = np.ascontiguousarray(x)
        return a.ctypes.data, a.nbytes, a
    if hasattr(x, "data_ptr"):
        t = x.contiguous()
        return t.data_ptr(), t.numel() * t.element_size(), t
    raise TypeError(f"unsupported tensor source {type(x)}")


class _SharedMarker(dict):
    """Truthy stand-in for the `shexp` dict when the shared expert lives on the device."""


class CudaMoeLayer:
    """One MoE layer's weights resident on a GPU (an aero_cuda_moe handle)."""

    def __init__(self, handle: int, device: int = 0) -> None:
        if not handle:
            raise RuntimeError("null handle")
        self._lib = nc.lib()
        self.handle = handle
        self.device = device
        info = (nc.c_int32 * 8)()
        self._lib.aero_cuda_moe_info(handle, info)
        d, E, k, F, Fs, has_sh, dt, norm = list(info)
        self.cfg = MoeConfig(n_expert=E, n_expert_used=k, n_embd=d, ffn_len=F, has_shared=bool(has_sh),
                             norm_topk_prob=bool(norm))
        self.ffn_len_shared = Fs
        self.dtype = dt
        self.shexp = _SharedMarker(device=True) if has_sh else None
        self.router = DeviceRouter(self)

    # ---- construction
    @classmethod
    def from_gguf(cls, path: str, layer: int, device: int = 0, expert_range=None) -> "CudaMoeLayer":
        L = nc.lib()
        nc.require_gpu()
        b, e = expert_range or (0, 0)
        err = nc.ctypes.create_string_buffer(512)
        h = L.aero_cuda_moe_open_gguf(path.encode(), int(layer), int(device), int(b), int(e), err, 512)
        if not h:
            raise RuntimeError(f"open_gguf({path}, layer {layer}): {err.value.decode()}")
        return cls(h, device)

    @classmethod
    def from_tensors(cls, cfg: MoeConfig, gate, up, down, dtype: int, router=None, router_bias=None,
                     shexp: Optional[dict] = None, device: int = 0, expert_range=None,
                     resident_ids=None) -> "CudaMoeLayer":
        """Open a layer from GGUF-format bytes (or f32 arrays for DTYPE_F32).

        gate/up are (E, F, d), down (E, d, F); shexp holds gate_inp (d,), gate,
        up, down and optionally dtype / ffn_len for the shared expert. With
        resident_ids (ascending global expert ids) the expert tensors hold only
        those experts, in that order (E = len(resident_ids)); routing stays over
        all cfg.n_expert logits, and a call that selects another expert fails."""
        L = nc.lib()
        nc.require_gpu()
        _check_k(cfg)
        keep = []
        desc = nc.Desc()
        desc.n_embd, desc.n_expert, desc.n_expert_used, desc.ffn_len = (cfg.n_embd, cfg.n_expert,
                                                                        cfg.n_expert_used, cfg.ffn_len)
        desc.norm_topk_prob = 1 if cfg.norm_topk_prob else 0
        desc.device = device
        if expert_range:
            desc.expert_begin, desc.expert_end = expert_range
        if resident_ids is not None:
            ids = np.ascontiguousarray(resident_ids, dtype=np.int32).reshape(-1)
            keep.append(ids)
            desc.n_resident = int(ids.size)
            desc.resident_ids = ids.ctypes.data

        def tensor(src, dt):
            addr, n, k = _as_bytes_view(src)
            keep.append(k)
            return nc.Tensor(dt, 0, addr, n)

        def f32(src):
            if src is None:
                return None
            if hasattr(src, "data_ptr"):
                t = src.contiguous().float()
                keep.append(t)
                return t.data_ptr()
            a = nc.f32c(src)
            keep.append(a)
            return a.ctypes.data

        desc.gate_exps, desc.up_exps, desc.down_exps = (tensor(gate, dtype), tensor(up, dtype), tensor(down, dtype))
        desc.router = f32(router)
        desc.router_bias = f32(router_bias)
        if shexp:
            sdt = int(shexp.get("dtype", dtype))
            desc.has_shared = 1
            desc.ffn_len_shared = int(shexp.get("ffn_len", 0))
            desc.shexp_gate_inp = f32(shexp["gate_inp"])
            desc.shexp_gate, desc.shexp_up, desc.shexp_down = (tensor(shexp["gate"], sdt), tensor(shexp["up"], sdt),
                                                               tensor(shexp["down"], sdt))
        err = nc.ctypes.create_string_buffer(512)
        h = L.aero_cuda_moe_open(nc.ctypes.byref(desc), err, 512)
        if not h:
            raise RuntimeError(f"aero_cuda_moe_open: {err.value.decode()}")
        return cls(h, device)

    # ---- compute
    def _io(self, h, width):
        if hasattr(h, "data_ptr"):
            import torch
            if h.dim() != 2 or h.shape[1] != width:
                raise ValueError(f"hidden width {h.shape[-1]} != n_embd {width}")
            t = h.contiguous().float()
            out = torch.empty_like(t)
            return t, out, t.data_ptr(), out.data_ptr()
        a = nc.f32c(h)
        if a.ndim != 2 or a.shape[1] != width:
            raise ValueError(f"hidden width {a.shape[-1]} != n_embd {width}")
        out = np.empty_like(a)
        return a, out, a.ctypes.data, out.ctypes.data

    def forward(self, h):
        """The whole block (router on the device). h (T, d) numpy or torch."""
        a, out, pa, po = self._io(h, self.cfg.n_embd)
        if self._lib.aero_cuda_moe_forward(self.handle, 0, pa, a.shape[0], self.cfg.n_embd, po) != 1:
            raise RuntimeError(f"moe forward refused: {nc.last_error(self.handle)}")
        return out

    def ffn_block(self, h, router_logits):
        """The block with caller-supplied (T, n_expert) router logits."""
        a, out, pa, po = self._io(h, self.cfg.n_embd)
        if hasattr(router_logits, "data_ptr"):
            lg = router_logits.contiguous().float()
            plg = lg.data_ptr()
        else:
            lg = nc.f32c(router_logits)
            plg = lg.ctypes.data
        if tuple(lg.shape) != (a.shape[0], self.cfg.n_expert):
            raise ValueError(f"router produced {tuple(lg.shape)} logits for {self.cfg.n_expert} experts")
        if self._lib.aero_cuda_moe_ffn_block(self.handle, pa, plg, a.shape[0], po) != 0:
            raise ValueError(f"moe ffn block refused: {nc.last_error(self.handle)}")
        return out

    def router_logits(self, h) -> np.ndarray:
        a = nc.f32c(h).reshape(-1, self.cfg.n_embd)
        out = np.empty((a.shape[0], self.cfg.n_expert), dtype=np.float32)
        if self._lib.aero_cuda_moe_router_logits(self.handle, a.ctypes.data, a.shape[0], out.ctypes.data) != 0:
            raise RuntimeError(f"router refused: {nc.last_error(self.handle)}")
        return out

    def route(self, logits):
        lg = nc.f32c(logits)
        single = lg.ndim == 1
        lg2 = lg.reshape(-1, self.cfg.n_expert)
        T, k = lg2.shape[0], self.cfg.n_expert_used
        idx = np.empty((T, k), dtype=np.int64)
        w = np.empty((T, k), dtype=np.float32)
        if self._lib.aero_cuda_moe_route(self.handle, lg2.ctypes.data, T, idx.ctypes.data, w.ctypes.data) != 0:
            raise ValueError(f"route refused: {nc.last_error(self.handle)}")
        return (idx[0], w[0]) if single else (idx, w)

    def set_gemm_min_tokens(self, n: int) -> None:
        """Calls with at least n tokens use the tcgen05 grouped-GEMM path."""
        if self._lib.aero_cuda_moe_set_option(self.handle, nc.OPT_GEMM_MIN_TOKENS, int(n)) != 0:
            raise ValueError(nc.last_error(self.handle))

    def set_router_tc(self, on: bool) -> None:
        """Project the router of >= 128-token calls on the tensor cores (default) or on the SIMT kernels."""
        if self._lib.aero_cuda_moe_set_option(self.handle, nc.OPT_ROUTER_TC, 1 if on else 0) != 0:
            raise ValueError(nc.last_error(self.handle))

    def set_decode_fused(self, on: bool) -> None:
        """Calls of up to 32 tokens as one fused kernel (default) or as separate kernels."""
        if self._lib.aero_cuda_moe_set_option(self.handle, nc.OPT_DECODE_FUSED, 1 if on else 0) != 0:
            raise ValueError(nc.last_error(self.handle))

    def set_peer_wait_ms(self, ms: int) -> None:
        """How long a peer-exchange kernel waits for a peer before giving up (code 21 / 22)."""
        if self._lib.aero_cuda_moe_set_option(self.handle, nc.OPT_PEER_WAIT_MS, int(ms)) != 0:
            raise ValueError(nc.last_error(self.handle))

    def status(self) -> int:
        """0, or the code of the first bounded device wait of this layer's kernels that gave up
        since the last read (synchronises)."""
        rc = self._lib.aero_cuda_moe_status(self.handle)
        if rc < 0:
            raise RuntimeError(nc.last_error(self.handle))
        return int(rc)

    def set_stream(self, stream) -> None:
        """Run on a cudaStream_t (int) or a torch.cuda.Stream; None restores the handle's own."""
        s = getattr(stream, "cuda_stream", stream)
        self._lib.aero_cuda_moe_set_stream(self.handle, s or None)

    STAGES = ("router", "topk", "dispatch", "gate_up", "down", "combine")

    def set_profiling(self, on: bool) -> None:
        if self._lib.aero_cuda_moe_set_profiling(self.handle, 1 if on else 0) != 0:
            raise RuntimeError("profiling could not be enabled")

    def stage_times(self) -> dict:
        """Accumulated device milliseconds and call counts per stage."""
        n = len(self.STAGES)
        ms = np.zeros(n, np.float64)
        cnt = np.zeros(n, np.int64)
        self._lib.aero_cuda_moe_stage_times(self.handle, ms.ctypes.data, cnt.ctypes.data, n)
        return {s: (float(ms[i]), int(cnt[i])) for i, s in enumerate(self.STAGES)}

    def stats(self) -> dict:
        buf = nc.ctypes.create_string_buffer(1024)
        self._lib.aero_cuda_moe_stats(self.handle, buf, 1024)
        return json.loads(buf.value.decode())

    def close(self) -> None:
        h, self.handle = self.handle, None
        if h:
            self._lib.aero_cuda_moe_close(h)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __call__(self, name, expert, block_rows=64):
        raise TypeError("CudaMoeLayer keeps experts quantised on the device; pass it to moe_ffn as expert_rows")


def _u8(b) -> np.ndarray:
    return np.ascontiguousarray(np.frombuffer(memoryview(b).cast("B"), dtype=np.uint8))


class PagedMoeLayer:
    """A MoE layer whose experts live in host memory, with n_slots of them resident on
    the device: router-ahead expert paging (the reference's design, ENGINE_DESIGN.md
    §3.3, ENGINE_DESIGN.md:99-101: the router result for a layer is known before its
    experts are needed, so the prefetch is exact). A call computes the routing on the
    device, pages in the experts it selects that are not resident (evicting the least
    recently used ones it does not need; aero_cuda_moe_page_in), then runs the block
    on the same logits (aero_cuda_moe_ffn_block), so every selected expert is resident.

    expert_bytes(e) -> (gate, up, down): expert e's GGUF bytes of each tensor (host
    bytes / numpy, e.g. slices of an mmap). A call that selects more experts than
    n_slots is refused (ValueError)."""

    def __init__(self, cfg: MoeConfig, expert_bytes, dtype: int, router, n_slots: int, router_bias=None,
                 shexp: Optional[dict] = None, device: int = 0) -> None:
        _check_k(cfg)
        if not 0 < n_slots < cfg.n_expert:
            raise ValueError(f"n_slots {n_slots} must be in [1, {cfg.n_expert})")
        self.cfg, self.n_slots, self._bytes = cfg, int(n_slots), expert_bytes
        first = [[_u8(b) for b in expert_bytes(e)] for e in range(n_slots)]
        gate, up, down = (np.concatenate([f[i] for f in first]) for i in range(3))
        self.layer = CudaMoeLayer.from_tensors(cfg, gate, up, down, dtype, router=router, router_bias=router_bias,
                                               shexp=shexp, device=device, resident_ids=list(range(n_slots)))
        self.slot_expert = list(range(n_slots))
        self._last = [0] * n_slots
        self._clock = 0
        self.pages = 0  # experts paged in since open

    def _page(self, slot: int, expert: int) -> None:
        g, u, d = (_u8(b) for b in self._bytes(expert))
        lib = nc.lib()
        if lib.aero_cuda_moe_page_in(self.layer.handle, slot, expert, g.ctypes.data, u.ctypes.data,
                                     d.ctypes.data) != 0:
            raise RuntimeError(f"page-in of expert {expert}: {nc.last_error(self.layer.handle)}")
        self.slot_expert[slot] = expert
        self.pages += 1

    def forward(self, h) -> np.ndarray:
        h = nc.f32c(h)
        cfg = self.cfg
        lg = self.layer.router_logits(h)
        idx, _ = nc.route(lg, cfg.n_expert, cfg.n_expert_used, cfg.norm_topk_prob)
        need = sorted({int(e) for e in np.asarray(idx).reshape(-1)})
        if len(need) > self.n_slots:
            raise ValueError(f"the call routes to {len(need)} experts; the device holds {self.n_slots}")
        self._clock += 1
        where = {e: s for s, e in enumerate(self.slot_expert)}
        free = sorted((s for s, e in enumerate(self.slot_expert) if e not in need), key=lambda s: self._last[s])
        for e in need:
            if e not in where:
                self._page(free.pop(0), e)
        for s, e in enumerate(self.slot_expert):
            if e in need:
                self._last[s] = self._clock
        return self.layer.ffn_block(h, lg)

    def close(self) -> None:
        self.layer.close()


def gguf_layer_info(path: str, layer: int) -> dict:
    """One MoE layer's description read from a GGUF file without opening it on a
    device (the metadata and tensor-shape reads of engine/model.py:193-224)."""
    out = (nc.c_int64 * 8)()
    err = nc.ctypes.create_string_buffer(512)
    if nc.lib().aero_cuda_moe_gguf_info(str(path).encode(), int(layer), out, err, 512) != 0:
        raise ValueError(f"gguf layer {layer} of {path}: {err.value.decode()}")
    d, E, k, F, Fs, has_sh, dt, has_router = (int(v) for v in out)
    return {"config": MoeConfig(n_expert=E, n_expert_used=k, n_embd=d, ffn_len=F, has_shared=bool(has_sh)),
            "ffn_len_shared": Fs, "dtype": dt, "has_router": bool(has_router)}


class DeviceRouter:
    """The layer's own router as a router_fn: moe_ffn recognises it and keeps
    the projection on the device; called directly it returns one token's logits."""

    def __init__(self, layer: CudaMoeLayer) -> None:
        self.layer = layer

    def __call__(self, hv):
        return self.layer.router_logits(np.asarray(hv, dtype=np.float32).reshape(1, -1))[0]


# ---------------------------------------------------------------- the block
def _host_logits(h: np.ndarray, cfg: MoeConfig, router_fn) -> np.ndarray:
    """Per-token router projection on the host, with the reference's width check
    (engine/moe.py:104-110)."""
    T = h.shape[0]
    out = np.empty((T, cfg.n_expert), dtype=np.float32)
    for t in range(T):
        rl = np.asarray(router_fn(h[t]), dtype=np.float32).reshape(-1)
        if rl.shape[-1] != cfg.n_expert:
            raise ValueError(f"router produced {rl.shape[-1]} logits for {cfg.n_expert} experts")
        out[t] = rl
    return out


def ffn_block(h, router_logits, n_expert, n_expert_used, ffn_len, norm_topk_prob, shexp, expert_rows,
              block_rows=64, device: int = 0):
    """engine/native_ssm.py ffn_block on the GPU: the experts come from the
    `expert_rows(name, expert, block_rows)` reader (full fp32 matrices); only the
    experts the routing selects are fetched. A reader exception propagates."""
    h = nc.f32c(h)
    lg = nc.f32c(router_logits)
    T, d = h.shape
    cfg = MoeConfig(n_expert=int(n_expert), n_expert_used=int(n_expert_used), n_embd=d, ffn_len=int(ffn_len),
                    has_shared=bool(shexp), norm_topk_prob=bool(norm_topk_prob))
    _check_k(cfg)
    if lg.shape != (T, cfg.n_expert):
        raise ValueError(f"router_logits shape {lg.shape} != ({T}, {cfg.n_expert})")
    if T == 0:
        return np.zeros((0, d), dtype=np.float32)
    # the routing on the device, then only the selected experts are fetched and
    # uploaded (a compact (n_sel, ...) layer whose slots map the global ids)
    idx, _ = nc.route(lg, cfg.n_expert, cfg.n_expert_used, cfg.norm_topk_prob)
    sel = np.unique(idx.reshape(-1)).astype(np.int32)
    F = cfg.ffn_len
    gate = np.empty((sel.size, F, d), dtype=np.float32)
    up = np.empty_like(gate)
    down = np.empty((sel.size, d, F), dtype=np.float32)
    for i, e in enumerate(int(v) for v in sel):
        gate[i] = nc.f32c(expert_rows(_NAMES[0], e, block_rows)).reshape(F, d)
        up[i] = nc.f32c(expert_rows(_NAMES[1], e, block_rows)).reshape(F, d)
        down[i] = nc.f32c(expert_rows(_NAMES[2], e, block_rows)).reshape(d, F)
    sh = None
    if shexp:
        sg = nc.f32c(shexp["gate"])
        sh = {"gate_inp": nc.f32c(shexp["gate_inp"]).reshape(-1), "gate": sg, "up": nc.f32c(shexp["up"]),
              "down": nc.f32c(shexp["down"]), "dtype": DTYPE_F32, "ffn_len": sg.shape[0]}
    layer = CudaMoeLayer.from_tensors(cfg, gate, up, down, DTYPE_F32, router=None, shexp=sh, device=device,
                                      resident_ids=sel)
    try:
        return layer.ffn_block(h, lg)
    finally:
        layer.close()


def moe_ffn(h: np.ndarray, cfg: MoeConfig, expert_rows, shexp: Optional[dict] = None, block_rows: int = 64,
            router_fn=None) -> np.ndarray:
    """The MoE FFN for a (T, n_embd) block, on the GPU (engine/moe.py:117-177)."""
    T, E = h.shape
    if E != cfg.n_embd:
        raise ValueError(f"hidden width {E} != n_embd {cfg.n_embd}")
    if router_fn is None:
        raise ValueError(
            "moe_ffn requires router_fn (a callable mapping a hidden vector to n_expert router logits); "
            "routing on the hidden state would be wrong")
    _check_k(cfg)
    if isinstance(expert_rows, CudaMoeLayer):
        layer = expert_rows
        use_shared = bool(cfg.has_shared and shexp)
        if use_shared != layer.cfg.has_shared:
            raise ValueError("the device layer was opened %s a shared expert; open it to match shexp"
                             % ("with" if layer.cfg.has_shared else "without"))
        if isinstance(router_fn, DeviceRouter) and router_fn.layer is layer:
            return layer.forward(h)
        return layer.ffn_block(h, _host_logits(nc.f32c(h), cfg, router_fn))
    use_shared = bool(cfg.has_shared and shexp)
    lg = _host_logits(nc.f32c(h), cfg, router_fn)
    return ffn_block(h, lg, cfg.n_expert, cfg.n_expert_used, cfg.ffn_len, cfg.norm_topk_prob,
                     shexp if use_shared else None, expert_rows, block_rows)


def expert_plan(cfg: MoeConfig, dtype: int = DTYPE_F32) -> dict:
    """Footprint plan (engine/moe.py:201-213), plus the device bytes the
    quantised, repacked planes occupy for `dtype` (all experts resident)."""
    per = cfg.n_embd * cfg.ffn_len * 4
    out = {
        "one_expert_fp32_bytes": 3 * per,
        "active_experts_fp32_bytes": 3 * per * cfg.n_expert_used,
        "all_experts_fp32_bytes": 3 * per * cfg.n_expert,
        "saving_factor": float(cfg.n_expert) / max(cfg.n_expert_used, 1),
    }
    if dtype in (DTYPE_Q8_0, DTYPE_Q4_K):
        bb, bv = BLOCK[dtype]
        one = 3 * cfg.n_embd * cfg.ffn_len // bv * bb
        out["one_expert_quant_bytes"] = one
        out["all_experts_quant_bytes"] = one * cfg.n_expert
    return out
