"""Seeded synthetic MoE layers and inputs for the benchmark configurations.

No datasets or checkpoints are involved: weights are N(0, 0.02), quantised to
the configuration's GGUF type; inputs are N(0, 1). Tensors are generated in a
fixed order, each from its own seeded stream, so any one of them can be
regenerated alone:

    0 router (E, d) f32      1 gate (E, F, d)      2 up (E, F, d)
    3 down (E, d, F)         4 shexp gate_inp (d,) 5 shexp gate (Fs, d)
    6 shexp up (Fs, d)       7 shexp down (d, Fs)

Three generators produce the weights: numpy (default_rng(seed * 1000 + i)) for
the small layers the tests use; the GPU (torch.randn with a seeded CUDA
generator, quantised by aero_cuda_quantize) for benchmark-size layers; and, for
benchmark-size layers that must not touch the GPU (the CPU reference arm of
bench.py), numpy over blocks of experts in worker processes, block b of tensor
i drawn from PCG64(seed * 1000 + i) jumped b times. The router, bias and inputs
always come from numpy, so the routing of a configuration does not depend on
the generator.

Zipf-skewed routing (configs 2 and 5): a per-expert logit bias
b_e = tau * log p_rank(e), p_r proportional to r^-s over a seeded random
ranking of the experts. tau is bisected until the measured load curve (expert
loads sorted descending, log load vs log rank, least squares over ranks
2 .. E/2) has slope -s. Top-k routing caps an expert at one pick per token,
which rules out matching the Zipf head exactly; the slope criterion matches
the skew of the body of the distribution.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from .quant import DTYPE_F32, DTYPE_Q4_K, DTYPE_Q8_0, quantize


@dataclass
class LayerSpec:
    d: int
    E: int
    k: int
    F: int
    Fs: int = 0                 # 0 = no shared expert
    dtype: int = DTYPE_Q8_0
    norm_topk_prob: bool = True


@dataclass
class Workload:
    name: str
    spec: LayerSpec
    T: int                       # tokens per call
    calls: int = 1               # calls per step (config 1 decodes 64 tokens one at a time)
    zipf_s: float = 0.0          # 0 = uniform routing
    bf16_x: bool = False         # round x to bf16-representable values
    note: str = ""


CONFIGS = {
    "c1": Workload("c1_decode_q8_0", LayerSpec(2048, 128, 8, 768, 0, DTYPE_Q8_0), T=1, calls=64,
                   note="single MoE layer, Q8_0, 64 tokens decoded one at a time"),
    "c2": Workload("c2_prefill_q4_k_zipf1.1", LayerSpec(2048, 128, 8, 768, 0, DTYPE_Q4_K), T=512, zipf_s=1.1,
                   bf16_x=True, note="Q4_K prefill, 512 tokens, Zipf(1.1) expert load"),
    "c3": Workload("c3_decode_q4_k_shared", LayerSpec(2048, 512, 10, 512, 512, DTYPE_Q4_K), T=32,
                   note="512 experts top-10 + sigmoid-gated shared expert, 32-token decode batch"),
    "c4b1": Workload("c4_moe_decode_b1_q4_k", LayerSpec(2048, 128, 8, 768, 0, DTYPE_Q4_K), T=1, calls=64,
                     note="config-4 decoder's MoE layer (Q4_K, 128 experts top-8, F=768), batch 1, 64 calls"),
    "c4b16": Workload("c4_moe_decode_b16_q4_k", LayerSpec(2048, 128, 8, 768, 0, DTYPE_Q4_K), T=16, calls=4,
                      note="config-4 decoder's MoE layer, batch 16, 4 calls"),
    "c5": Workload("c5_prefill_q4_k_shared", LayerSpec(2048, 512, 10, 512, 512, DTYPE_Q4_K), T=8192,
                   note="512 experts top-10 + shared expert, 8192-token prefill, uniform routing"),
    "c5z": Workload("c5_prefill_q4_k_shared_zipf1.2", LayerSpec(2048, 512, 10, 512, 512, DTYPE_Q4_K), T=8192,
                    zipf_s=1.2, note="config 5 with Zipf(1.2) expert load"),
}


@dataclass
class SynthLayer:
    spec: LayerSpec
    router: np.ndarray                      # (E, d) f32
    gate: np.ndarray                        # GGUF bytes as uint8 (or f32 for DTYPE_F32)
    up: np.ndarray
    down: np.ndarray
    router_bias: Optional[np.ndarray] = None
    shexp: Optional[dict] = None            # gate_inp f32 (d,), gate/up/down bytes, dtype, ffn_len
    meta: dict = field(default_factory=dict)


def _rng(seed: int, i: int) -> np.random.Generator:
    return np.random.default_rng(seed * 1000 + i)


def _normal_np(seed: int, i: int, n: int, scale: float) -> np.ndarray:
    return (_rng(seed, i).standard_normal(n, dtype=np.float32) * np.float32(scale)).astype(np.float32)


def _quant_np(seed, i, n, dtype):
    w = _normal_np(seed, i, n, 0.02)
    if dtype == DTYPE_F32:
        return w
    return np.frombuffer(quantize(w, dtype), dtype=np.uint8)


def _quant_gpu(seed, i, n, dtype, scale=0.02):
    import torch

    from . import native_cuda as nc
    g = torch.Generator(device="cuda")
    g.manual_seed(seed * 1000 + i)
    w = torch.randn(n, generator=g, device="cuda", dtype=torch.float32) * scale
    if dtype == DTYPE_F32:
        return w.cpu().numpy()
    b = nc.quantize(dtype, w)
    del w
    return np.frombuffer(b, dtype=np.uint8)


def _host_block(args):
    seed, i, b, n, dtype = args
    g = np.random.Generator(np.random.PCG64(seed * 1000 + i).jumped(b))
    w = (g.standard_normal(n, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    return w if dtype == DTYPE_F32 else np.frombuffer(quantize(w, dtype), dtype=np.uint8)


_HOST_POOL = None


def _quant_host_parallel(seed, i, n, dtype, block=1 << 24):
    """N(0, 0.02) values in blocks of `block` values (a multiple of 256), each
    block from its own jumped PCG64 stream, quantised in a spawn process pool."""
    global _HOST_POOL
    import multiprocessing as mp
    import os
    nb = (n + block - 1) // block
    jobs = [(seed, i, b, min(block, n - b * block), dtype) for b in range(nb)]
    if nb == 1:
        return _host_block(jobs[0])
    if _HOST_POOL is None:
        _HOST_POOL = mp.get_context("spawn").Pool(min(16, os.cpu_count() or 1))
    return np.concatenate(_HOST_POOL.map(_host_block, jobs))


def make_layer(spec: LayerSpec, seed: int = 0, device_gen: bool = False, host_parallel: bool = False) -> SynthLayer:
    """device_gen: weights from the GPU generator; host_parallel: from the
    block-parallel numpy generator (no GPU); neither: the single-stream numpy
    generator."""
    gen = _quant_gpu if device_gen else (_quant_host_parallel if host_parallel else _quant_np)
    d, E, F, Fs = spec.d, spec.E, spec.F, spec.Fs
    router = _normal_np(seed, 0, E * d, 0.02).reshape(E, d)
    gate = gen(seed, 1, E * F * d, spec.dtype)
    up = gen(seed, 2, E * F * d, spec.dtype)
    down = gen(seed, 3, E * d * F, spec.dtype)
    shexp = None
    if Fs:
        shexp = {
            "gate_inp": _normal_np(seed, 4, d, 0.02),
            "gate": gen(seed, 5, Fs * d, spec.dtype),
            "up": gen(seed, 6, Fs * d, spec.dtype),
            "down": gen(seed, 7, d * Fs, spec.dtype),
            "dtype": spec.dtype,
            "ffn_len": Fs,
        }
    return SynthLayer(spec, router, gate, up, down, None, shexp,
                      {"seed": seed, "device_gen": device_gen, "host_parallel": host_parallel})


def make_x(T: int, d: int, seed: int = 0, bf16: bool = False) -> np.ndarray:
    x = np.random.default_rng(seed * 1000 + 99).standard_normal((T, d), dtype=np.float32)
    if bf16:
        u = x.view(np.uint32)
        # round to nearest even at bit 16
        u = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
        x = u.view(np.float32)
    return np.ascontiguousarray(x)


def _topk_loads(logits: np.ndarray, k: int) -> np.ndarray:
    idx = np.argpartition(-logits, k - 1, axis=1)[:, :k]
    return np.bincount(idx.reshape(-1), minlength=logits.shape[1])


def _slope(loads: np.ndarray) -> float:
    E = loads.size
    l = np.sort(loads)[::-1].astype(np.float64)
    r = np.arange(1, E + 1, dtype=np.float64)
    sel = slice(1, max(3, E // 2))
    return float(np.polyfit(np.log(r[sel]), np.log(l[sel] + 1.0), 1)[0])


def zipf_bias(base_logits: np.ndarray, k: int, s: float, seed: int = 0, iters: int = 40):
    """(bias (E,) f32, tau, loads) giving a Zipf(s)-shaped expert load."""
    E = base_logits.shape[1]
    order = np.random.default_rng(seed * 1000 + 77).permutation(E)
    rank = np.empty(E, dtype=np.int64)
    rank[order] = np.arange(1, E + 1)
    logp = (-s * np.log(rank.astype(np.float64))).astype(np.float32)
    logp -= logp.max()
    lo, hi = 0.0, 1.0
    while _slope(_topk_loads(base_logits + np.float32(hi) * logp, k)) > -s and hi < 1e4:
        hi *= 2.0
    for _ in range(iters):
        mid = 0.5 * (lo + hi)
        if _slope(_topk_loads(base_logits + np.float32(mid) * logp, k)) > -s:
            lo = mid
        else:
            hi = mid
    tau = 0.5 * (lo + hi)
    bias = (np.float32(tau) * logp).astype(np.float32)
    return bias, tau, _topk_loads(base_logits + bias, k)


def attach_zipf(layer: SynthLayer, x: np.ndarray, s: float, seed: int = 0) -> SynthLayer:
    """Calibrate and attach the Zipf router bias for inputs x."""
    base = x @ layer.router.T
    bias, tau, loads = zipf_bias(base, layer.spec.k, s, seed)
    layer.router_bias = bias
    E, k = layer.spec.E, layer.spec.k
    # the Zipf(s) head share 1 / H(E, s) against top-k's cap: a token picks an expert at
    # most once, so no expert can take more than 1 / k of the assignments
    zipf_top = float(1.0 / np.sum(np.arange(1, E + 1, dtype=np.float64) ** -s))
    layer.meta.update({"zipf_s": s, "zipf_tau": tau, "top_load_share": float(loads.max() / loads.sum()),
                       "zipf_top_share": zipf_top, "top_share_cap": 1.0 / k, "load_slope": float(_slope(loads)),
                       "max_load": int(loads.max()), "min_load": int(loads.min())})
    return layer


def open_layer(layer: SynthLayer, device: int = 0, expert_range=None):
    """Upload a synthetic layer to the GPU as a CudaMoeLayer."""
    from .moe import CudaMoeLayer, MoeConfig
    sp = layer.spec
    cfg = MoeConfig(n_expert=sp.E, n_expert_used=sp.k, n_embd=sp.d, ffn_len=sp.F, has_shared=bool(sp.Fs),
                    norm_topk_prob=sp.norm_topk_prob)
    return CudaMoeLayer.from_tensors(cfg, layer.gate, layer.up, layer.down, sp.dtype, router=layer.router,
                                     router_bias=layer.router_bias, shexp=layer.shexp, device=device,
                                     expert_range=expert_range)


def write_gguf(layer: SynthLayer, path: str, layer_index: int = 0, arch: str = "qwen35moe") -> None:
    """Write the layer as a GGUF file in the qwen35moe tensor naming."""
    from .gguf import GGUFWriter, moe_tensor_names
    sp = layer.spec
    names = moe_tensor_names(layer_index)
    w = GGUFWriter(arch)
    w.add_u32(f"{arch}.expert_count", sp.E)
    w.add_u32(f"{arch}.expert_used_count", sp.k)
    w.add_u32(f"{arch}.embedding_length", sp.d)
    w.add_tensor(names["router"], (sp.E, sp.d), layer.router.astype(np.float32).tobytes(), DTYPE_F32)
    w.add_tensor(names["gate"], (sp.E, sp.F, sp.d), np.asarray(layer.gate).tobytes(), sp.dtype)
    w.add_tensor(names["up"], (sp.E, sp.F, sp.d), np.asarray(layer.up).tobytes(), sp.dtype)
    w.add_tensor(names["down"], (sp.E, sp.d, sp.F), np.asarray(layer.down).tobytes(), sp.dtype)
    if layer.shexp:
        sh = layer.shexp
        w.add_tensor(names["shexp_gate_inp"], (1, sp.d), np.asarray(sh["gate_inp"], np.float32).tobytes(), DTYPE_F32)
        w.add_tensor(names["shexp_gate"], (sp.Fs, sp.d), np.asarray(sh["gate"]).tobytes(), sh["dtype"])
        w.add_tensor(names["shexp_up"], (sp.Fs, sp.d), np.asarray(sh["up"]).tobytes(), sh["dtype"])
        w.add_tensor(names["shexp_down"], (sp.d, sp.Fs), np.asarray(sh["down"]).tobytes(), sh["dtype"])
    w.write(path)


# ---------------------------------------------------------------- decoder
@dataclass
class DecoderSpec:
    """A qwen-style decoder around the MoE layer (the reference's block loop,
    src/model.cpp:234-330): per layer RMSNorm -> GQA attention (q/k RMSNorm per
    head, neox RoPE) -> residual -> RMSNorm (post_attention_norm) -> MoE FFN ->
    residual; then output_norm and the LM head on the last position."""
    n_layer: int
    d: int
    n_head: int
    n_kv: int
    head_dim: int
    vocab: int
    moe: LayerSpec
    rope_base: float = 1e6
    eps: float = 1e-6
    attn_dtype: int = DTYPE_Q8_0
    embd_dtype: int = DTYPE_Q8_0
    tied: bool = False
    qk_norm: bool = True


# config 4 (the 48-layer decoder): GQA 32 q / 4 kv heads of 128, RoPE 1e6, every FFN the
# 128-expert top-8 Q4_K MoE (F 768), vocab 151936 with Q8_0 embedding and head
DECODER_C4 = DecoderSpec(48, 2048, 32, 4, 128, 151936, LayerSpec(2048, 128, 8, 768, 0, DTYPE_Q4_K))


@dataclass
class SynthDecoder:
    spec: DecoderSpec
    tensors: dict                           # name -> (row-major shape, ggml type, bytes as uint8 / f32 array)
    moe: list                               # SynthLayer per layer


def _norm_weight(seed: int, i: int, n: int) -> np.ndarray:
    return (np.float32(1.0) + _normal_np(seed, i, n, 0.1)).astype(np.float32)


def make_decoder(spec: DecoderSpec, seed: int = 0, device_gen: bool = False) -> SynthDecoder:
    """Seeded random-init weights of the decoder: projections N(0, 0.02) quantised to
    attn_dtype, the embedding N(0, 1) quantised to embd_dtype, norm weights 1 + N(0, 0.1),
    the MoE layers from make_layer (seed * 100 + layer)."""
    gen = _quant_gpu if device_gen else _quant_np
    d, H, HK, D = spec.d, spec.n_head, spec.n_kv, spec.head_dim
    t = {}

    def q(name, shape, i, dt, scale=0.02):
        n = int(np.prod(shape))
        if scale == 0.02:
            raw = gen(seed, i, n, dt)
        elif device_gen:
            raw = _quant_gpu(seed, i, n, dt, scale)
        else:
            w = _normal_np(seed, i, n, scale)
            raw = w if dt == DTYPE_F32 else np.frombuffer(quantize(w, dt), dtype=np.uint8)
        t[name] = (tuple(shape), dt, raw)

    q("token_embd.weight", (spec.vocab, d), 900, spec.embd_dtype, scale=1.0)
    if not spec.tied:
        q("output.weight", (spec.vocab, d), 901, spec.embd_dtype)
    t["output_norm.weight"] = ((d,), DTYPE_F32, _norm_weight(seed, 902, d))
    moe = []
    for L in range(spec.n_layer):
        p, b = f"blk.{L}.", 1000 + 20 * L
        t[p + "attn_norm.weight"] = ((d,), DTYPE_F32, _norm_weight(seed, b, d))
        t[p + "post_attention_norm.weight"] = ((d,), DTYPE_F32, _norm_weight(seed, b + 1, d))
        q(p + "attn_q.weight", (H * D, d), b + 2, spec.attn_dtype)
        q(p + "attn_k.weight", (HK * D, d), b + 3, spec.attn_dtype)
        q(p + "attn_v.weight", (HK * D, d), b + 4, spec.attn_dtype)
        q(p + "attn_output.weight", (d, H * D), b + 5, spec.attn_dtype)
        if spec.qk_norm:
            t[p + "attn_q_norm.weight"] = ((D,), DTYPE_F32, _norm_weight(seed, b + 6, D))
            t[p + "attn_k_norm.weight"] = ((D,), DTYPE_F32, _norm_weight(seed, b + 7, D))
        moe.append(make_layer(spec.moe, seed * 100 + L, device_gen=device_gen))
    return SynthDecoder(spec, t, moe)


def write_decoder_gguf(dec: SynthDecoder, path: str, arch: str = "qwen3moe") -> None:
    """The decoder as a GGUF file: the reference's metadata keys (arch-prefixed) and
    tensor names, the MoE tensors per layer in the qwen35moe naming."""
    from .gguf import GGUF_FLOAT32, GGUFWriter, moe_tensor_names
    sp = dec.spec
    w = GGUFWriter(arch)
    for key, v in (("block_count", sp.n_layer), ("embedding_length", sp.d), ("attention.head_count", sp.n_head),
                   ("attention.head_count_kv", sp.n_kv), ("attention.key_length", sp.head_dim),
                   ("attention.value_length", sp.head_dim), ("expert_count", sp.moe.E),
                   ("expert_used_count", sp.moe.k), ("vocab_size", sp.vocab)):
        w.add_u32(f"{arch}.{key}", v)
    w.add_kv(f"{arch}.rope.freq_base", GGUF_FLOAT32, float(sp.rope_base))
    w.add_kv(f"{arch}.attention.layer_norm_rms_epsilon", GGUF_FLOAT32, float(sp.eps))
    for name, (shape, dt, raw) in dec.tensors.items():
        w.add_tensor(name, shape, np.asarray(raw).tobytes(), dt)
    for L, layer in enumerate(dec.moe):
        names = moe_tensor_names(L)
        m = layer.spec
        w.add_tensor(names["router"], (m.E, m.d), layer.router.astype(np.float32).tobytes(), DTYPE_F32)
        w.add_tensor(names["gate"], (m.E, m.F, m.d), np.asarray(layer.gate).tobytes(), m.dtype)
        w.add_tensor(names["up"], (m.E, m.F, m.d), np.asarray(layer.up).tobytes(), m.dtype)
        w.add_tensor(names["down"], (m.E, m.d, m.F), np.asarray(layer.down).tobytes(), m.dtype)
        if layer.shexp:
            sh = layer.shexp
            w.add_tensor(names["shexp_gate_inp"], (m.d,), np.asarray(sh["gate_inp"], np.float32).tobytes(), DTYPE_F32)
            w.add_tensor(names["shexp_gate"], (m.Fs, m.d), np.asarray(sh["gate"]).tobytes(), sh["dtype"])
            w.add_tensor(names["shexp_up"], (m.Fs, m.d), np.asarray(sh["up"]).tobytes(), sh["dtype"])
            w.add_tensor(names["shexp_down"], (m.d, m.Fs), np.asarray(sh["down"]).tobytes(), sh["dtype"])
    w.write(path)
