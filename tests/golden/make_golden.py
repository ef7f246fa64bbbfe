#!/usr/bin/env python3
"""Generate tests/golden/golden.npz from the REFERENCE ITSELF.

Run where the reference checkout exists (its root given by --ref), after
`make -C oracle all` built oracle/_ref/libaero_ssm.so from the reference's own
src/ssm.cpp, src/moe.cpp, src/kernels.cpp:

    python tests/golden/make_golden.py [--ref REFERENCE_ROOT]

What it records, each produced by the reference's code:
  * dequant vectors: engine/quant.py dequantize AND the C++ aero_dequant_ref on
    the same Q8_0 / Q4_K bytes (asserted bit-identical to each other), including
    the hand-built blocks of tests/test_quant.py:71-93,126-131;
  * routing cases: aero_moe_route (src/moe.cpp:26-66) and engine.moe.route on
    fixed logits, including the tie cases of tests/test_moe_cpp.cpp:95-109,
    tests/test_ssm_cpp.cpp:154-168 and tests/test_arch.py:92-97;
  * MoE blocks: engine.moe.moe_ffn with the native library (src/moe.cpp via
    engine/native_ssm.py), fed by an expert reader that dequantises the layer's
    GGUF bytes with engine.quant.dequantize and caches per call the way
    engine/model.py:651-678 does, and a router_fn h @ W_r^T (+ bias)
    (engine/model.py:665-666). Layer bytes are NOT stored: they are regenerated
    by aero_b200.synth with the stored seed and checked against a stored
    SHA-256, which keeps the fixture small.
  * GGUF files written by the reference's own GGUFWriter (engine/gguf.py:448-526)
    around synth layers, with the reference block's outputs on them
    (ref_writer_<name>.gguf beside the .npz, their SHA-256 in it).
The GPU box has no reference tree; the tests read only the .npz and the .gguf files.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from aero_b200 import synth  # noqa: E402
from aero_b200.quant import DTYPE_Q4_K, DTYPE_Q8_0, quantize  # noqa: E402

REF_SSM = os.path.join(ROOT, "oracle", "_ref", "libaero_ssm.so")


def sha(*arrs) -> str:
    h = hashlib.sha256()
    for a in arrs:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def load_reference(ref_root: str):
    sys.path.insert(0, ref_root)
    from engine import moe as M  # noqa: E402
    from engine import native_ssm as NS  # noqa: E402
    from engine import quant as Q  # noqa: E402
    NS._LIB_CANDIDATES = (REF_SSM,)
    if not NS.available():
        raise SystemExit(f"reference native MoE library not loadable: {NS.unavailable_reason()}")
    import ctypes
    lib = ctypes.CDLL(REF_SSM)
    lib.aero_dequant_ref.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64]
    lib.aero_dequant_ref.restype = ctypes.c_int
    return M, NS, Q, lib


def f16(v: float) -> bytes:
    return struct.pack("<e", v)


def dequant_cases(Q, lib):
    rng = np.random.default_rng(20261201)
    cases = {}
    # Q8_0: random bytes with sane scales; the 0.5*index block (tests/test_quant.py:126-131)
    q8 = bytearray(rng.integers(0, 256, size=34 * 16, dtype=np.uint8).tobytes())
    for b in range(16):
        q8[34 * b:34 * b + 2] = f16(0.02 * (b + 1) * (-1 if b % 3 == 0 else 1))
    q8[34 * 15:34 * 16] = f16(0.5) + bytes(range(32))
    q8[34 * 14:34 * 14 + 2] = struct.pack("<H", 0x0001)  # subnormal fp16 scale
    cases["q8_random"] = (DTYPE_Q8_0, bytes(q8))
    # Q4_K: random bytes with sane d/dmin; the hand block of tests/test_quant.py:71-93
    q4 = bytearray(rng.integers(0, 256, size=144 * 8, dtype=np.uint8).tobytes())
    for b in range(8):
        q4[144 * b:144 * b + 2] = f16(0.01 * (b + 1))
        q4[144 * b + 2:144 * b + 4] = f16(0.003 * (b + 1))
    scales = bytes([1, 1, 1, 1, 0, 0, 0, 0, 1, 1, 1, 1])
    qs = bytes([(i & 0x0F) | (((31 - i) & 0x0F) << 4) for i in range(128)])
    q4[144 * 7:144 * 8] = f16(1.0) + f16(0.0) + scales + qs
    q4[144 * 6:144 * 7] = f16(1.0) + f16(2.0) + scales + qs
    cases["q4k_random"] = (DTYPE_Q4_K, bytes(q4))
    # quantised from N(0, 0.02) by this repo's quantisers
    w = (rng.standard_normal(4096) * 0.02).astype(np.float32)
    cases["q8_quantised"] = (DTYPE_Q8_0, quantize(w, DTYPE_Q8_0))
    cases["q4k_quantised"] = (DTYPE_Q4_K, quantize(w, DTYPE_Q4_K))
    out = {}
    for name, (dt, raw) in cases.items():
        n = len(raw) // (34 if dt == DTYPE_Q8_0 else 144) * (32 if dt == DTYPE_Q8_0 else 256)
        py = np.asarray(Q.dequantize(raw, dt, (n,)), dtype=np.float32)
        c = np.empty(n, dtype=np.float32)
        buf = np.frombuffer(raw, dtype=np.uint8)
        assert lib.aero_dequant_ref(dt, buf.ctypes.data, buf.size, c.ctypes.data, n) == 1
        assert np.array_equal(py.view(np.uint32), c.view(np.uint32)), f"{name}: python and C++ reference disagree"
        out[f"deq_{name}_raw"] = np.frombuffer(raw, dtype=np.uint8).copy()
        out[f"deq_{name}_dtype"] = np.int32(dt)
        out[f"deq_{name}_out"] = c
    return out


def route_cases(M, NS):
    rng = np.random.default_rng(7)
    cases = []
    lg = (0.1 * np.arange(24)).astype(np.float32)
    lg[3] = lg[7] = 5.0
    cases.append(("tie_3_7", lg, 2))                                                   # test_moe_cpp [1]
    cases.append(("fixed_1_4", np.array([0.1, 3.0, -2.0, 1.5, 2.9, 0.0], np.float32), 2))  # test_ssm_cpp [3]
    cases.append(("all_zero", np.zeros(8, np.float32), 3))                              # test_arch ties
    cases.append(("k_equals_E", rng.standard_normal(4).astype(np.float32), 4))          # test_moe_cpp [7]
    z = np.zeros(16, np.float32)
    z[5] = -0.0
    z[2] = 0.0
    z[9] = 1.0
    cases.append(("signed_zero", z, 3))
    cases.append(("coarse_128_8", (np.round(rng.standard_normal(128) * 2) / 2).astype(np.float32), 8))
    cases.append(("coarse_512_10", (np.round(rng.standard_normal(512)) / 1).astype(np.float32), 10))
    for i in range(4):
        cases.append((f"rand_128_8_{i}", rng.standard_normal(128).astype(np.float32) * 2, 8))
        cases.append((f"rand_512_10_{i}", rng.standard_normal(512).astype(np.float32) * 2, 10))
    out = {"route_names": np.array([c[0] for c in cases])}
    for name, lg, k in cases:
        for norm in (1, 0):
            idx, w = NS.route(lg, lg.size, k, bool(norm))
            cfg = M.MoeConfig(n_expert=lg.size, n_expert_used=k, n_embd=1, ffn_len=1, norm_topk_prob=bool(norm))
            i2, w2 = M.route(lg, cfg)
            assert np.array_equal(idx, i2)
            out[f"route_{name}_logits"] = lg
            out[f"route_{name}_k"] = np.int32(k)
            out[f"route_{name}_n{norm}_idx"] = idx
            out[f"route_{name}_n{norm}_w"] = w
    return out


def block_case(M, Q, spec, T, seed, zipf_s=0.0):
    layer = synth.make_layer(spec, seed)
    x = synth.make_x(T, spec.d, seed)
    if zipf_s:
        synth.attach_zipf(layer, x, zipf_s, seed)
    d, E, F = spec.d, spec.E, spec.F
    names = {"ffn_gate_exps.weight": (layer.gate, (F, d)), "ffn_up_exps.weight": (layer.up, (F, d)),
             "ffn_down_exps.weight": (layer.down, (d, F))}
    per = {k: v[0].size // E for k, v in names.items()}
    cache = {}
    calls = {"n": 0}

    def rows(name, expert, block_rows):
        key = (name, expert)
        if key not in cache:
            raw, shape = names[name]
            b = raw[expert * per[name]:(expert + 1) * per[name]].tobytes()
            cache[key] = Q.dequantize(b, spec.dtype, shape)
        calls["n"] += 1
        return cache[key]

    W = layer.router
    bias = layer.router_bias

    def router_fn(hv):
        lg = (hv @ W.T).reshape(-1)
        return lg + bias if bias is not None else lg

    shexp = None
    if layer.shexp:
        sh = layer.shexp
        shexp = {"gate_inp": sh["gate_inp"].reshape(1, d),
                 "gate": Q.dequantize(sh["gate"].tobytes(), sh["dtype"], (spec.Fs, d)),
                 "up": Q.dequantize(sh["up"].tobytes(), sh["dtype"], (spec.Fs, d)),
                 "down": Q.dequantize(sh["down"].tobytes(), sh["dtype"], (d, spec.Fs))}
    cfg = M.MoeConfig(n_expert=E, n_expert_used=spec.k, n_embd=d, ffn_len=F, has_shared=bool(spec.Fs),
                      norm_topk_prob=spec.norm_topk_prob)
    out = M.moe_ffn(x, cfg, rows, shexp, 64, router_fn=router_fn)
    # the reference's numpy path must agree (tests/test_ssm_native.py:316-330)
    saved = M._native_ssm
    M._native_ssm = None
    try:
        out_np = M.moe_ffn(x, cfg, rows, shexp, 64, router_fn=router_fn)
    finally:
        M._native_ssm = saved
    assert np.abs(out - out_np).max() < 1e-5 * max(1.0, float(np.abs(out_np).max())), "reference native != numpy"
    logits = np.stack([router_fn(x[t]) for t in range(T)]).astype(np.float32)
    sh_bytes = [layer.shexp[k] for k in ("gate", "up", "down")] if layer.shexp else []
    return {
        "spec": np.array([d, E, spec.k, F, spec.Fs, spec.dtype, int(spec.norm_topk_prob), T, seed], np.int64),
        "zipf_s": np.float64(zipf_s),
        "sha": np.array(sha(layer.router, layer.gate, layer.up, layer.down, *sh_bytes)),
        "x": x,
        "logits": logits,
        "bias": bias if bias is not None else np.zeros(0, np.float32),
        "out": out.astype(np.float32),
        "fetches": np.int64(calls["n"]),
    }


GGUF_CASES = {
    # name: (spec, tokens, seed, layer index)
    "g_q8_shared": (synth.LayerSpec(256, 4, 2, 64, 64, DTYPE_Q8_0), 5, 31, 1),
    "g_q4k": (synth.LayerSpec(256, 2, 1, 256, 0, DTYPE_Q4_K), 3, 32, 0),
}


def gguf_case(G, M, Q, name, spec, T, seed, layer_index):
    """The layer's bytes written by the reference's own GGUFWriter (engine/gguf.py:448-526),
    with metadata of every value kind around the MoE tensors, and the reference block's
    output on it (block_case on the same seed)."""
    layer = synth.make_layer(spec, seed)
    arch = "qwen3moe"
    w = G.GGUFWriter(arch)
    w.add_kv(f"{arch}.block_count", G.GGUF_UINT32, layer_index + 1)
    w.add_kv(f"{arch}.expert_count", G.GGUF_UINT32, spec.E)
    w.add_kv(f"{arch}.expert_used_count", G.GGUF_UINT32, spec.k)
    w.add_kv(f"{arch}.embedding_length", G.GGUF_UINT32, spec.d)
    w.add_kv(f"{arch}.rope.freq_base", G.GGUF_FLOAT32, 1000000.0)
    w.add_kv("general.name", G.GGUF_STRING, f"aero-b200 fixture {name}")
    w.add_kv("tokenizer.ggml.tokens", G.GGUF_ARRAY, (G.GGUF_STRING, ["<s>", "</s>", "a", "b"]))
    w.add_kv("tokenizer.ggml.scores", G.GGUF_ARRAY, (G.GGUF_FLOAT32, [0.0, -1.0, -2.5, -3.0]))
    w.add_kv("general.file_type", G.GGUF_UINT64, 7)
    d, E, F = spec.d, spec.E, spec.F
    w.add_tensor("token_embd.weight", (4, d), np.ones((4, d), np.float32).tobytes(), G.T_F32)
    p = f"blk.{layer_index}."
    w.add_tensor(p + "ffn_gate_inp.weight", (E, d), layer.router.astype(np.float32).tobytes(), G.T_F32)
    w.add_tensor(p + "ffn_gate_exps.weight", (E, F, d), np.asarray(layer.gate).tobytes(), spec.dtype)
    w.add_tensor(p + "ffn_up_exps.weight", (E, F, d), np.asarray(layer.up).tobytes(), spec.dtype)
    w.add_tensor(p + "ffn_down_exps.weight", (E, d, F), np.asarray(layer.down).tobytes(), spec.dtype)
    if layer.shexp:
        sh = layer.shexp
        w.add_tensor(p + "ffn_gate_inp_shexp.weight", (d,), np.asarray(sh["gate_inp"], np.float32).tobytes(), G.T_F32)
        w.add_tensor(p + "ffn_gate_shexp.weight", (spec.Fs, d), np.asarray(sh["gate"]).tobytes(), sh["dtype"])
        w.add_tensor(p + "ffn_up_shexp.weight", (spec.Fs, d), np.asarray(sh["up"]).tobytes(), sh["dtype"])
        w.add_tensor(p + "ffn_down_shexp.weight", (d, spec.Fs), np.asarray(sh["down"]).tobytes(), sh["dtype"])
    w.add_tensor(p + "attn_norm.weight", (d,), np.ones(d, np.float32).tobytes(), G.T_F32)
    path = os.path.join(HERE, f"ref_writer_{name}.gguf")
    w.write(path)
    with open(path, "rb") as fh:
        file_sha = hashlib.sha256(fh.read()).hexdigest()
    case = block_case(M, Q, spec, T, seed)
    return {"layer": np.int64(layer_index), "file_sha": np.array(file_sha), "spec": case["spec"],
            "x": case["x"], "logits": case["logits"], "out": case["out"]}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("AERO_REF") or os.path.abspath(
        os.path.join(os.path.dirname(__file__), "..", "..", "..", "reference")),
        help="the reference checkout (default: $AERO_REF, else a 'reference' directory beside this repository)")
    args = ap.parse_args()
    M, NS, Q, lib = load_reference(args.ref)
    out = {}
    out.update(dequant_cases(Q, lib))
    out.update(route_cases(M, NS))
    blocks = {
        "b_q8": (synth.LayerSpec(256, 16, 4, 64, 64, DTYPE_Q8_0), 6, 11, 0.0),
        "b_q8_noshared": (synth.LayerSpec(256, 12, 3, 96, 0, DTYPE_Q8_0), 5, 12, 0.0),
        "b_q4k": (synth.LayerSpec(256, 6, 2, 256, 256, DTYPE_Q4_K), 4, 13, 0.0),
        "b_q8_norm0": (synth.LayerSpec(256, 10, 3, 64, 0, DTYPE_Q8_0, norm_topk_prob=False), 3, 14, 0.0),
        "b_q4k_zipf": (synth.LayerSpec(512, 16, 4, 256, 0, DTYPE_Q4_K), 24, 15, 1.1),
    }
    for name, (spec, T, seed, zs) in blocks.items():
        for key, v in block_case(M, Q, spec, T, seed, zs).items():
            out[f"{name}_{key}"] = v
    out["block_names"] = np.array(list(blocks))
    sys.path.insert(0, args.ref)
    from engine import gguf as G  # noqa: E402
    for name, (spec, T, seed, li) in GGUF_CASES.items():
        for key, v in gguf_case(G, M, Q, name, spec, T, seed, li).items():
            out[f"{name}_{key}"] = v
    out["gguf_names"] = np.array(list(GGUF_CASES))
    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()
