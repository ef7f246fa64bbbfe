"""Host-side checks that need no GPU: quantisers, GGUF writer, the C-ABI
library's exports, the memory guard's accounting, and the GGUF parser's
refusals."""

import glob
import os
import re
import struct

import numpy as np
import pytest

import oracle as O
from aero_b200 import quant as Q
from aero_b200 import synth
from aero_b200.gguf import GGUFWriter

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_q8_0_matches_gguf_py():
    gguf = pytest.importorskip("gguf")
    x = (np.random.default_rng(0).standard_normal((16, 2048)) * 0.02).astype(np.float32)
    x[0, :32] = 0.0  # an all-zero block (d = 0)
    want = gguf.quants.quantize(x, gguf.GGMLQuantizationType.Q8_0).tobytes()
    assert Q.quantize(x, Q.DTYPE_Q8_0) == want


def test_q4_k_roundtrip_error():
    x = (np.random.default_rng(1).standard_normal(256 * 64) * 0.02).astype(np.float32)
    raw = Q.quantize(x, Q.DTYPE_Q4_K)
    assert len(raw) == 64 * 144
    y = O.dequant(Q.DTYPE_Q4_K, raw, x.size)
    rel = np.sqrt(np.mean((y - x) ** 2)) / np.sqrt(np.mean(x ** 2))
    assert rel < 0.12
    # all-zero super-block quantises to d = dmin = 0 and decodes to zeros
    z = Q.quantize(np.zeros(256, np.float32), Q.DTYPE_Q4_K)
    assert np.all(O.dequant(Q.DTYPE_Q4_K, z, 256) == 0)


def test_type_sizes():
    assert Q.type_size(Q.DTYPE_Q8_0, 32) == 34
    assert Q.type_size(Q.DTYPE_Q4_K, 512) == 288
    with pytest.raises(ValueError):
        Q.type_size(Q.DTYPE_Q4_K, 100)


def test_gguf_writer_layout(tmp_path):
    w = GGUFWriter("qwen35moe")
    w.add_u32("qwen35moe.expert_count", 4)
    w.add_tensor("t0", (3, 32), Q.quantize(np.ones(96, np.float32), Q.DTYPE_Q8_0), Q.DTYPE_Q8_0)
    w.add_tensor("t1", (2,), np.arange(2, dtype=np.float32).tobytes(), Q.DTYPE_F32)
    b = w.to_bytes()
    assert b[:4] == b"GGUF"
    version, n_t, n_kv = struct.unpack_from("<IQQ", b, 4)
    assert (version, n_t, n_kv) == (3, 2, 3)
    assert len(b) % 32 == 0


# ---------------------------------------------------------------- the C ABI
def _headers():
    """Every header under include/, comments removed."""
    srcs = [open(p).read() for p in sorted(glob.glob(os.path.join(ROOT, "include", "*.h")))]
    return re.sub(r"/\*.*?\*/", "", "\n".join(srcs), flags=re.S)


def _header_functions():
    src = _headers()
    names = re.findall(r"\b(aero_cuda_\w+)\s*\(", src)
    return sorted(set(n for n in names if not n.endswith("_fn")))


def test_library_exports_every_header_symbol(cuda_lib):
    from aero_b200 import native_cuda as nc
    names = _header_functions()
    assert len(names) >= 40
    for n in names:
        assert hasattr(cuda_lib, n), n
    declared = {s[0] for s in nc.SYMBOLS}
    assert set(names) == declared


def test_compute_refuses_without_gpu(cuda_lib):
    """With no visible GPU every compute entry point refuses (no CPU fallback)."""
    from aero_b200 import native_cuda as nc
    if nc.gpu_count() > 0:
        pytest.skip("a GPU is visible")
    with pytest.raises(nc.CudaMoeUnavailable):
        nc.route(np.zeros(8, np.float32), 8, 2)
    lg = np.zeros(8, np.float32)
    idx = np.zeros(2, np.int64)
    w = np.zeros(2, np.float32)
    assert cuda_lib.aero_cuda_route(lg.ctypes.data, 1, 8, 2, 1, idx.ctypes.data, w.ctypes.data) == -1
    assert "no CUDA device" in nc.last_error()


def test_guard_accounting(cuda_lib):
    from aero_b200 import native_cuda as nc
    g = nc.MemoryGuard()
    base = g.committed()
    g.set_budget(0)
    assert g.try_reserve(1 << 40, nc.MEM_SCRATCH)  # budget 0 = unbounded
    g.release(1 << 40, nc.MEM_SCRATCH)
    g.set_budget(base + 1000)
    try:
        assert g.try_reserve(600, nc.MEM_WEIGHTS_RESIDENT)
        assert not g.try_reserve(600, nc.MEM_SCRATCH)
        assert g.committed(nc.MEM_WEIGHTS_RESIDENT) >= 600
        assert g.headroom() == 400
        ok, why = g.admit_plan(2000)
        assert not ok and "exceeds" in why
        ok, why = g.admit_plan(500)
        assert not ok and "already committed" in why
        # evictor frees cache bytes on a refusal (src/memory_guard.cpp:172-182)
        assert g.try_reserve(300, nc.MEM_WEIGHTS_CACHE)

        def evict(need):
            g.release(300, nc.MEM_WEIGHTS_CACHE)
            return 300

        g.set_evictor(evict)
        assert g.try_reserve(250, nc.MEM_SCRATCH)
        g.set_evictor(None)
        g.release(250, nc.MEM_SCRATCH)
        g.release(600, nc.MEM_WEIGHTS_RESIDENT)
        g.release(10 ** 9, nc.MEM_KV_CACHE)  # never below zero
        assert g.committed(nc.MEM_KV_CACHE) == 0
    finally:
        g.set_budget(0)
    assert g.committed() == base


def test_loadgate_semantics(cuda_lib):
    from aero_b200 import native_cuda as nc
    g = nc.MemoryGuard()
    base = g.committed()
    g.set_budget(base + 1000)
    try:
        gate = nc.LoadGate(700)
        assert gate.ok()
        assert gate.next_chunk(300) and gate.next_chunk(300)
        assert not gate.next_chunk(300)          # 600 + 300 > 700: the plan is complete
        assert gate.ok() and gate.done()          # completion, not failure
        assert gate.reserved() == 600
        g.release(600, nc.MEM_WEIGHTS_CACHE)
        big = nc.LoadGate(5000)
        assert not big.ok() and "exceeds" in big.reason()
        assert g.try_reserve(600, nc.MEM_RUNTIME)
        stop = nc.LoadGate(300)                  # 600 + 300 <= 1000: admitted
        assert stop.next_chunk(150)
        assert g.try_reserve(200, nc.MEM_RUNTIME)  # someone else takes memory mid-load
        assert not stop.next_chunk(100) and not stop.ok()
        assert "would exceed" in stop.reason()
        g.release(150, nc.MEM_WEIGHTS_CACHE)
        g.release(800, nc.MEM_RUNTIME)
    finally:
        g.set_budget(0)
    assert g.committed() == base


def test_gguf_open_refuses_bad_files(cuda_lib, tmp_path):
    import ctypes
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOPE" + b"\0" * 64)
    err = ctypes.create_string_buffer(256)
    assert not cuda_lib.aero_cuda_moe_open_gguf(str(bad).encode(), 0, 0, 0, 0, err, 256)
    assert b"bad magic" in err.value
    # a real layer file, truncated in the middle of its data
    spec = synth.LayerSpec(256, 4, 2, 64, 0, Q.DTYPE_Q8_0)
    p = tmp_path / "layer.gguf"
    synth.write_gguf(synth.make_layer(spec, 1), str(p))
    data = p.read_bytes()
    t = tmp_path / "trunc.gguf"
    t.write_bytes(data[: len(data) // 2])
    assert not cuda_lib.aero_cuda_moe_open_gguf(str(t).encode(), 0, 0, 0, 0, err, 256)
    assert b"past the end" in err.value or b"truncated" in err.value
    # wrong layer index: not a MoE layer
    assert not cuda_lib.aero_cuda_moe_open_gguf(str(p).encode(), 3, 0, 0, 0, err, 256)
    assert b"missing" in err.value


def test_zipf_calibration():
    spec = synth.LayerSpec(256, 64, 4, 64, 0, Q.DTYPE_Q8_0)
    layer = synth.make_layer(spec, 2)
    x = synth.make_x(512, 256, 2)
    synth.attach_zipf(layer, x, 1.1, 2)
    lg = x @ layer.router.T + layer.router_bias
    loads = np.bincount(np.argsort(-lg, axis=1)[:, :4].reshape(-1), minlength=64)
    assert abs(synth._slope(loads) + 1.1) < 0.05
    assert loads.max() > 3 * np.median(loads)
    # the recorded calibration: the measured head share stays under top-k's 1/k cap, which
    # the Zipf(1.1) head share over 64 experts exceeds (the reason the slope is matched)
    m = layer.meta
    assert m["top_share_cap"] == 1 / 4
    assert abs(m["zipf_top_share"] - 1 / np.sum(np.arange(1, 65, dtype=np.float64) ** -1.1)) < 1e-12
    assert m["top_load_share"] <= m["top_share_cap"] < m["zipf_top_share"]
    assert abs(m["load_slope"] + 1.1) < 0.05


def test_bf16_inputs_representable():
    x = synth.make_x(4, 64, 0, bf16=True)
    assert np.all((x.view(np.uint32) & 0xFFFF) == 0)


def test_bench_gemm_roofline_bound():
    """bench.py's prefill roofline takes the larger of the tensor and HBM times as the bound:
    config 5's gate/up GEMM is tensor-bound, config 2's (512 tokens, 128 experts) HBM-bound.
    The tensor fraction is against the burst peak (the GEMM runs inside a ~1 ms step)."""
    import bench
    from aero_b200 import synth

    pk = {"bf16_tflops": 1641.0, "bf16_tflops_sustained": 1392.6, "hbm_gbs": 6545.0, "source": "measured"}
    for key, stats, st, bound, frac in (
            ("c5", {"last_pairs": 81920, "last_shared_rows": 8192, "last_active": 512},
             {"gate_up": 0.559, "down": 0.315}, "tensor", 0.4120),
            ("c2", {"last_pairs": 4096, "last_shared_rows": 0, "last_active": 126},
             {"gate_up": 0.193, "down": 0.1065}, "hbm", 0.1765)):
        spec = synth.CONFIGS[key].spec
        per_expert, shared = bench.layer_bytes(spec)
        r = bench.gemm_roofline(spec, stats, st, pk, per_expert // 3, shared)
        assert r["kernel"] == "grouped_gemm_gate_up"
        assert r["bound"] == bound and r["other_bound"]["bound"] != bound
        assert abs(r["frac"] - frac) < 2e-3, (key, r["frac"])
        assert abs(r["frac"] - r["achieved"] / r["peak"]) < 1e-12
        tc = r if r["bound"] == "tensor" else r["other_bound"]
        assert tc["peak"] == pk["bf16_tflops"]
        assert abs(tc["frac_of_sustained"] - tc["achieved"] / pk["bf16_tflops_sustained"]) < 1e-12


def test_bench_decode_bytes_and_config():
    """Decode HBM bytes count each call's distinct experts once, plus router, shared expert and
    activations; both bench arms print the same config record."""
    import bench
    from aero_b200 import synth

    spec = synth.LayerSpec(64, 8, 2, 32, 32, synth.DTYPE_Q4_K)
    router = np.eye(8, 64, dtype=np.float32)
    x = np.zeros((4, 64), np.float32)
    x[0, 0] = x[1, 0] = 5.0  # calls of 2 tokens: both tokens pick expert 0 (+ a tie-broken partner)
    x[2, 3], x[3, 4] = 5.0, 5.0
    per_expert, shared = bench.layer_bytes(spec)
    got = bench.decode_bytes(spec, x, router, None, 2, 2)
    lg = x @ router.T
    want = 0
    for c in range(2):
        sel = np.argpartition(-lg[2 * c:2 * c + 2], 1, axis=1)[:, :2]
        want += len(np.unique(sel)) * per_expert + shared + 9 * 64 * 4 + 2 * 2 * 64 * 4
    assert got == want
    wl = synth.CONFIGS["c5"]
    assert bench.config_dict(wl, 1) == bench.config_dict(wl, 1) and bench.config_dict(wl, 8)["parallelism"] == "ep8"
    assert bench.config_dict(wl, 1)["tokens_per_step"] == 8192


def test_bench_clock_window():
    """The clock sampler keeps running; a timed region reads the samples around it only, and
    flags hardware slowdowns seen there."""
    import bench

    c = bench.Clocks(0)
    line = lambda mhz, slow: f"{mhz}, 1965, 700.0, {slow}, Not Active, Not Active, Not Active"  # noqa: E731
    c.lines = [(9.0, line(1200, "Not Active")), (10.1, line(1965, "Not Active")), (10.3, line(1950, "Active")),
               (11.5, line(1000, "Not Active"))]
    r = c.summary(10.2, 10.25, pad=0.3)
    assert r["samples"] == 2 and r["sm_mhz"] == 1957.5 and r["sm_max_mhz"] == 1965.0
    assert r["reasons"] == ["hw_slowdown"]
    assert c.summary(20.0, 20.1)["reasons"] == ["unsampled"]


def test_ctypes_signatures_match_header():
    """Every ctypes declaration has as many arguments as the header's prototype."""
    from aero_b200 import native_cuda as nc

    src = _headers()
    protos = {}
    for m in re.finditer(r"\b(aero_cuda_\w+)\s*\(([^;{]*?)\)\s*;", src, flags=re.S):
        name, params = m.group(1), " ".join(m.group(2).split())
        if name.endswith("_fn"):
            continue
        protos[name] = 0 if params in ("", "void") else params.count(",") + 1
    assert len(protos) >= 40
    for name, _restype, argtypes in nc.SYMBOLS:
        assert name in protos, name
        assert len(argtypes) == protos[name], (name, len(argtypes), protos[name])


def test_decoder_plan_footprint_config4(cuda_lib):
    """The config-4 decoder's device plan (no device work): the f16 caches of 16 sequences
    of 4096 positions, Q8_0 projections / embedding / head, and 48 MoE layers in
    quantised planes (the reference's fp32 active-expert term would be 8 x 3 x 2048 x
    768 x 4 B per layer)."""
    from aero_b200.decoder import plan_footprint
    sp = synth.DECODER_C4
    p = plan_footprint(sp, n_seq=16, n_ctx=4096)
    assert p["kv_cache"] == 2 * 16 * 4 * 128 * 4096 * 2 * 48
    q8 = lambda n: n // 32 * 34  # noqa: E731
    attn = q8((32 * 128 + 2 * 4 * 128) * 2048) + q8(2048 * 32 * 128)
    expert = 3 * 768 * 2048 // 256 * 144
    # device planes hold the GGUF bytes (plus 128-byte alignment per plane); the router f32
    assert 48 * 128 * expert < p["moe_weights"] < 48 * (128 * expert + 129 * 2048 * 4 * 3 + 1 << 16)
    assert 48 * attn + 2 * q8(151936 * 2048) < p["weights_resident"] - p["moe_weights"] < \
        48 * attn + 2 * q8(151936 * 2048) + (1 << 22)
    assert p["total"] == p["weights_resident"] + p["kv_cache"]
    assert 23e9 < p["total"] < 26e9
