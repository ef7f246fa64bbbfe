"""GPU parity: the CUDA library through its C ABI against the oracle and the
reference's golden vectors.

Bars (from the task's north star): routed expert indices and the dispatch
permutation are bit-exact on identical logits; dequantised values are
bit-exact; layer outputs are within max-abs-error 2e-3 x RMS(output) for the
fp32-accumulated decode path and 1e-2 x RMS for the bf16-dequantised prefill
path.
"""

import os

import numpy as np
import pytest

import oracle as O
from aero_b200 import moe as M
from aero_b200 import native_cuda as nc
from aero_b200 import quant as Q
from aero_b200 import synth
from golden_blocks import block

pytestmark = pytest.mark.gpu

DECODE_TOL = 2e-3
PREFILL_TOL = 1e-2


def rms(a):
    return float(np.sqrt(np.mean(np.asarray(a, np.float64) ** 2)))


def rel_err(got, want):
    return float(np.abs(np.asarray(got, np.float64) - want).max()) / max(rms(want), 1e-12)


@pytest.fixture(scope="module", autouse=True)
def _lib(cuda_lib):
    nc.require_gpu()


# ---------------------------------------------------------------- dequant / quant
def test_dequant_bit_exact_vs_reference(golden):
    for name in ("q8_random", "q4k_random", "q8_quantised", "q4k_quantised"):
        raw = golden[f"deq_{name}_raw"].tobytes()
        want = golden[f"deq_{name}_out"]
        got = nc.dequant(int(golden[f"deq_{name}_dtype"]), raw, want.size)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), name


def test_dequant_refuses_short_buffer():
    with pytest.raises(ValueError):
        nc.dequant(Q.DTYPE_Q4_K, b"\0" * 100, 256)


def test_quantize_gpu_equals_host():
    rng = np.random.default_rng(5)
    x = (rng.standard_normal(256 * 300) * 0.02).astype(np.float32)
    x[:256] = 0.0
    x[256:512] = np.abs(x[256:512])  # a super-block with no negative values
    x[512:768] *= 50.0
    for dt in (Q.DTYPE_Q8_0, Q.DTYPE_Q4_K):
        assert nc.quantize(dt, x) == Q.quantize(x, dt), dt


# ---------------------------------------------------------------- routing
def test_route_matches_reference_cases(golden):
    for name in golden["route_names"]:
        lg = golden[f"route_{name}_logits"]
        k = int(golden[f"route_{name}_k"])
        for norm in (1, 0):
            idx, w = nc.route(lg, lg.size, k, bool(norm))
            assert np.array_equal(idx, golden[f"route_{name}_n{norm}_idx"]), (name, norm)
            np.testing.assert_allclose(w, golden[f"route_{name}_n{norm}_w"], rtol=2e-6, atol=1e-7)


def test_route_batched_bit_exact_with_ties():
    rng = np.random.default_rng(6)
    for T, E, k in ((1, 128, 8), (33, 128, 8), (257, 512, 10), (40, 24, 24), (5, 1024, 32)):
        lg = (np.round(rng.standard_normal((T, E)) * 4) / 4).astype(np.float32)  # heavy ties
        lg[0, :] = 0.0
        for norm in (True, False):
            idx, w = nc.route(lg, E, k, norm)
            ridx, rw = O.route(lg, k, norm)
            assert np.array_equal(idx, ridx), (T, E, k, norm)
            np.testing.assert_allclose(w, rw, rtol=2e-6, atol=1e-7)


def test_route_refusals():
    with pytest.raises(ValueError):
        nc.route(np.zeros(4, np.float32), 4, 0)
    with pytest.raises(ValueError):
        nc.route(np.zeros(4, np.float32), 4, 5)
    idx, _ = nc.route(np.zeros(4, np.float32), 4, 4)
    assert list(idx) == [0, 1, 2, 3]


def test_dispatch_bit_exact():
    rng = np.random.default_rng(7)
    for T, k, E in ((1, 8, 128), (32, 10, 512), (512, 8, 128), (8192, 10, 512), (3, 2, 1000)):
        idx = rng.integers(0, E, size=(T, k))
        if T >= 512:  # skewed load, an empty expert and a dominant one
            idx[: T // 2, 0] = 3
            idx[idx == 5] = 6
        off, perm = nc.dispatch(idx, E)
        roff, rperm = O.dispatch(idx, E)
        assert np.array_equal(off, roff) and np.array_equal(perm, rperm), (T, k, E)


# ---------------------------------------------------------------- blocks
def test_golden_blocks_ffn_block(golden):
    """Caller logits (identical to the reference's) -> the reference's outputs."""
    for name in golden["block_names"]:
        layer, g = block(golden, name)
        L = synth.open_layer(layer)
        try:
            out = L.ffn_block(g["x"], g["logits"])
        finally:
            L.close()
        assert rel_err(out, g["out"]) <= DECODE_TOL, name


def test_golden_blocks_device_router(golden):
    """Router on the device: idx must equal the reference's on its logits
    unless a near-tie flips (checked against f64 logits), then outputs match."""
    for name in golden["block_names"]:
        layer, g = block(golden, name)
        L = synth.open_layer(layer)
        try:
            lg = L.router_logits(g["x"])
            np.testing.assert_allclose(lg, g["logits"], rtol=1e-5, atol=1e-5)
            idx_dev, _ = nc.route(lg, layer.spec.E, layer.spec.k, layer.spec.norm_topk_prob)
            idx_ref, _ = O.route(g["logits"], layer.spec.k, layer.spec.norm_topk_prob)
            if np.array_equal(idx_dev, idx_ref):
                out = L.forward(g["x"])
                assert rel_err(out, g["out"]) <= DECODE_TOL, name
        finally:
            L.close()


def test_forward_deterministic_and_device_pointers(golden):
    torch = pytest.importorskip("torch")
    layer, g = block(golden, "b_q8")
    L = synth.open_layer(layer)
    try:
        a = L.forward(g["x"])
        b = L.forward(g["x"])
        assert np.array_equal(a, b)
        xt = torch.from_numpy(g["x"]).cuda()
        c = L.forward(xt)
        torch.cuda.synchronize()
        assert np.array_equal(c.cpu().numpy(), a)
        # an unaligned device view is staged, not read with vector loads
        big = torch.zeros(g["x"].size + 1, device="cuda")
        big[1:] = xt.reshape(-1)
        d = L.forward(big[1:].view(g["x"].shape))
        torch.cuda.synchronize()
        assert np.array_equal(d.cpu().numpy(), a)
    finally:
        L.close()


def _config_check(key, T, seed=0, tol=DECODE_TOL, calls=1):
    wl = synth.CONFIGS[key]
    layer = synth.make_layer(wl.spec, seed, device_gen=True)
    # the device-generated bytes must decode to N(0, 0.02)-like weights
    w = O.dequant(wl.spec.dtype, layer.gate[: 34 * 64 if wl.spec.dtype == Q.DTYPE_Q8_0 else 144 * 8],
                  2048)
    assert 0.015 < float(np.std(w)) < 0.025
    x = synth.make_x(T * calls, wl.spec.d, seed, bf16=wl.bf16_x)
    if wl.zipf_s:
        synth.attach_zipf(layer, x, wl.zipf_s, seed)
    L = synth.open_layer(layer)
    try:
        lg = L.router_logits(x)
        outs = [L.ffn_block(x[i * T:(i + 1) * T], lg[i * T:(i + 1) * T]) for i in range(calls)]
    finally:
        L.close()
    out = np.concatenate(outs)
    ref = O.moe_block(layer, x, lg, nthreads=os.cpu_count() or 1)
    assert rms(ref) > 1e-3, "degenerate reference output (weights or routing broken)"
    err = rel_err(out, ref)
    assert err <= tol, (key, err)
    return err


def test_config1_decode_q8_0():
    """All 64 tokens of config 1, one call each."""
    _config_check("c1", T=1, calls=64)


def test_config4_moe_layer_batch1():
    """Config 4's MoE layer (Q4_K, 128 experts top-8, F=768) at decode batch 1: 64 calls."""
    _config_check("c4b1", T=1, calls=64)


def test_config4_moe_layer_batch16():
    """Config 4's MoE layer at decode batch 16: 4 calls of 16 tokens."""
    _config_check("c4b16", T=16, calls=4)


def test_config3_decode_q4_k_shared():
    _config_check("c3", T=32)


def test_config2_prefill_q4_k_zipf_subset():
    # routing over all 512 tokens of the config, outputs checked on all of them
    _config_check("c2", T=512, tol=PREFILL_TOL)


def test_gguf_open_equals_tensors(tmp_path):
    spec = synth.LayerSpec(512, 8, 2, 256, 256, Q.DTYPE_Q4_K)
    layer = synth.make_layer(spec, 21)
    p = str(tmp_path / "l.gguf")
    synth.write_gguf(layer, p, layer_index=3)
    x = synth.make_x(7, 512, 21)
    A = M.CudaMoeLayer.from_gguf(p, 3)
    B = synth.open_layer(layer)
    try:
        assert A.cfg.n_expert == 8 and A.cfg.n_expert_used == 2 and A.cfg.has_shared
        assert np.array_equal(A.forward(x), B.forward(x))
    finally:
        A.close()
        B.close()


# ---------------------------------------------------------------- drop-in API
def test_moe_ffn_dropin_matches_loop_reference():
    """tests/test_arch.py:129-195, run through the GPU path."""
    rng = np.random.default_rng(9)
    E, F, NX = 8, 4, 6
    cfg = M.MoeConfig(n_expert=NX, n_expert_used=2, n_embd=E, ffn_len=F)
    Gt = rng.standard_normal((NX, F, E)).astype(np.float32) * 0.5
    Ut = rng.standard_normal((NX, F, E)).astype(np.float32) * 0.5
    Dt = rng.standard_normal((NX, E, F)).astype(np.float32) * 0.5
    fetched = []

    def rows(name, expert, block_rows):
        fetched.append((name, expert))
        return {"ffn_gate_exps.weight": Gt, "ffn_up_exps.weight": Ut, "ffn_down_exps.weight": Dt}[name][expert]

    Rout = rng.standard_normal((NX, E)).astype(np.float32) * 0.5
    router_fn = lambda hv: (hv @ Rout.T).reshape(-1)  # noqa: E731
    h = rng.standard_normal((3, E)).astype(np.float32)
    out = M.moe_ffn(h, cfg, rows, shexp=None, router_fn=router_fn)
    with pytest.raises(ValueError):
        M.moe_ffn(h, cfg, rows, shexp=None)
    with pytest.raises(ValueError):
        M.moe_ffn(h, cfg, rows, shexp=None, router_fn=lambda hv: np.zeros(3, dtype=np.float32))

    def ref_one(ht):
        idx, w = O.route(router_fn(ht), 2)
        acc = np.zeros(E, dtype=np.float32)
        for e, wt in zip(idx, w):
            a = (ht @ Gt[e].T) / (1 + np.exp(-(ht @ Gt[e].T))) * (ht @ Ut[e].T)
            acc += wt * (a @ Dt[e].T)
        return acc

    ref = np.stack([ref_one(h[t]) for t in range(3)])
    assert np.allclose(out, ref, atol=1e-5)
    assert {e for _, e in fetched} <= set(int(i) for t in range(3) for i in O.route(router_fn(h[t]), 2)[0])
    sh = {"gate_inp": rng.standard_normal((1, E)).astype(np.float32), "gate": rng.standard_normal((F, E)).astype(np.float32),
          "up": rng.standard_normal((F, E)).astype(np.float32), "down": rng.standard_normal((E, F)).astype(np.float32)}
    with_sh = M.moe_ffn(h, cfg, rows, shexp=sh, router_fn=router_fn)
    assert not np.allclose(out, with_sh)
    g = 1 / (1 + np.exp(-(h @ sh["gate_inp"].T)))
    want = ref.copy()
    for t in range(3):
        a = (h[t] @ sh["gate"].T) / (1 + np.exp(-(h[t] @ sh["gate"].T))) * (h[t] @ sh["up"].T)
        want[t] += g[t, 0] * (a @ sh["down"].T)
    assert np.allclose(with_sh, want, atol=1e-5)


def test_fetch_failure_propagates():
    """tests/test_moe_cpp.cpp:252-268: a failing reader aborts the block."""
    cfg = M.MoeConfig(n_expert=6, n_expert_used=2, n_embd=16, ffn_len=16, has_shared=False)

    def rows(name, expert, block_rows):
        if name == "ffn_up_exps.weight":
            raise KeyError("up missing")
        return np.zeros((16, 16), np.float32)

    with pytest.raises(KeyError):
        M.moe_ffn(np.ones((1, 16), np.float32), cfg, rows, router_fn=lambda hv: np.arange(6, dtype=np.float32))


def _loop_reference(h, lg, k, norm, rows, sh=None):
    """engine/native_ssm.py ffn_block as a plain f64 loop over the routed experts."""
    out = np.zeros(h.shape, np.float64)
    for t in range(h.shape[0]):
        idx, w = O.route(lg[t], k, norm)
        x = h[t].astype(np.float64)
        for e, wt in zip(idx, w):
            g = rows("ffn_gate_exps.weight", int(e), 64) @ x
            u = rows("ffn_up_exps.weight", int(e), 64) @ x
            out[t] += float(wt) * (rows("ffn_down_exps.weight", int(e), 64) @ (g / (1 + np.exp(-g)) * u))
        if sh is not None:
            gs = sh["gate"] @ x
            a = gs / (1 + np.exp(-gs)) * (sh["up"] @ x)
            out[t] += (1 / (1 + np.exp(-(sh["gate_inp"].reshape(-1) @ x)))) * (sh["down"] @ a)
    return out


@pytest.mark.parametrize("norm,T,shared", [(True, 1, False), (False, 2, True)])
def test_generic_block_uploads_only_the_selected_experts(monkeypatch, norm, T, shared):
    """A c1-shaped call (128 experts, k = 8, n_embd 2048, ffn 768) through a host reader of
    fp32 matrices: the reader is asked for the routed experts only and the device layer
    holds only those (a compact layer whose slot map keeps the global ids), while the
    routing is over all 128 logits, so norm_topk_prob = 0 keeps the full-softmax weights."""
    d, F, E, k = 2048, 768, 128, 8
    cache = {}

    def rows(name, expert, block_rows):
        key = (name, expert)
        if key not in cache:
            r = np.random.default_rng([7, expert, len(name)])
            shape = (d, F) if name == "ffn_down_exps.weight" else (F, d)
            cache[key] = (r.standard_normal(shape) * 0.03).astype(np.float32)
        return cache[key]

    fetched = []

    def reader(name, expert, block_rows):
        fetched.append(expert)
        return rows(name, expert, block_rows)

    rng = np.random.default_rng(11 + T)
    h = rng.standard_normal((T, d)).astype(np.float32)
    lg = (rng.standard_normal((T, E)) * 2).astype(np.float32)
    sh = None
    if shared:
        sh = {"gate_inp": (rng.standard_normal((1, d)) * 0.05).astype(np.float32),
              "gate": (rng.standard_normal((F, d)) * 0.03).astype(np.float32),
              "up": (rng.standard_normal((F, d)) * 0.03).astype(np.float32),
              "down": (rng.standard_normal((d, F)) * 0.03).astype(np.float32)}
    guard = nc.MemoryGuard()
    base = guard.committed(nc.MEM_WEIGHTS_RESIDENT)
    seen = {}
    orig = M.CudaMoeLayer.from_tensors.__func__

    def spy(cls, cfg, gate, up, down, *a, **kw):
        layer = orig(cls, cfg, gate, up, down, *a, **kw)
        seen["experts"] = gate.shape[0]
        seen["ids"] = np.asarray(kw["resident_ids"]).tolist()
        seen["weights"] = guard.committed(nc.MEM_WEIGHTS_RESIDENT) - base
        return layer

    monkeypatch.setattr(M.CudaMoeLayer, "from_tensors", classmethod(spy))
    out = M.ffn_block(h, lg, E, k, F, norm, sh, reader)
    routed = sorted({int(e) for t in range(T) for e in O.route(lg[t], k, norm)[0]})
    assert sorted(set(fetched)) == routed and len(fetched) == 3 * len(routed)
    assert seen["ids"] == routed and seen["experts"] == len(routed)
    per_expert = 3 * F * d * 4
    assert seen["weights"] < (len(routed) + 4) * per_expert, seen
    ref = _loop_reference(h, lg, k, norm, rows, sh)
    assert rel_err(out, ref) <= 1e-4, rel_err(out, ref)


def test_resident_subset_refuses_an_expert_it_does_not_hold():
    """A layer holding experts {1, 4} of 6: routing to them works; routing that selects
    another expert fails the call (status code 41), and the next call runs."""
    d, F, E = 64, 32, 6
    rng = np.random.default_rng(5)
    gate = (rng.standard_normal((2, F, d)) * 0.1).astype(np.float32)
    up = (rng.standard_normal((2, F, d)) * 0.1).astype(np.float32)
    down = (rng.standard_normal((2, d, F)) * 0.1).astype(np.float32)
    cfg = M.MoeConfig(n_expert=E, n_expert_used=2, n_embd=d, ffn_len=F, has_shared=False)
    L = M.CudaMoeLayer.from_tensors(cfg, gate, up, down, Q.DTYPE_F32, resident_ids=[1, 4])
    try:
        x = rng.standard_normal((3, d)).astype(np.float32)
        good = np.full((3, E), -5.0, np.float32)
        good[:, 1], good[:, 4] = 1.0, 0.5
        a = L.ffn_block(x, good)
        full = {"ffn_gate_exps.weight": {1: gate[0], 4: gate[1]}, "ffn_up_exps.weight": {1: up[0], 4: up[1]},
                "ffn_down_exps.weight": {1: down[0], 4: down[1]}}
        ref = _loop_reference(x, good, 2, True, lambda n, e, b: full[n][e])
        assert rel_err(a, ref) <= 1e-5
        bad = good.copy()
        bad[1, 2] = 3.0
        with pytest.raises(ValueError, match="does not hold"):
            L.ffn_block(x, bad)
        assert np.array_equal(L.ffn_block(x, good), a)
        assert L.status() == 0
    finally:
        L.close()
    with pytest.raises(RuntimeError, match="ascending"):
        M.CudaMoeLayer.from_tensors(cfg, gate, up, down, Q.DTYPE_F32, resident_ids=[4, 1])


def test_device_layer_with_its_router(golden):
    layer, g = block(golden, "b_q8")
    L = synth.open_layer(layer)
    try:
        cfg = L.cfg
        a = M.moe_ffn(g["x"], cfg, L, shexp=L.shexp, router_fn=L.router)
        b = L.forward(g["x"])
        assert np.array_equal(a, b)
        c = M.moe_ffn(g["x"], cfg, L, shexp=L.shexp, router_fn=lambda hv: hv @ layer.router.T)
        assert rel_err(c, g["out"]) <= DECODE_TOL
    finally:
        L.close()


# ---------------------------------------------------------------- guard on the device
def test_guard_refuses_oversized_layer():
    g = nc.MemoryGuard()
    base = g.committed()
    spec = synth.LayerSpec(256, 16, 4, 64, 0, Q.DTYPE_Q8_0)
    layer = synth.make_layer(spec, 3)
    g.set_budget(base + 4096)
    try:
        with pytest.raises(RuntimeError) as e:
            synth.open_layer(layer)
        assert "refused" in str(e.value)
    finally:
        g.set_budget(0)
    assert g.committed() == base


def test_guard_injected_allocation_failure_leaks_nothing():
    g = nc.MemoryGuard()
    base = g.committed()
    spec = synth.LayerSpec(256, 16, 4, 64, 64, Q.DTYPE_Q8_0)
    layer = synth.make_layer(spec, 4)
    for n in (1, 2, 3, 5, 8):
        g.fail_nth_alloc(n)
        with pytest.raises(RuntimeError):
            synth.open_layer(layer)
        assert g.committed() == base, n
    g.fail_nth_alloc(0)
    L = synth.open_layer(layer)
    assert g.committed() > base
    L.close()
    assert g.committed() == base


def test_asynchronous_submit_wait_equals_forward():
    """aero_cuda_moe_submit / _wait over slots 0 and 1 give the synchronous call's outputs,
    for a decode-size and a prefill-size call (GEMM path) interleaved, pinned and pageable
    host buffers; device buffers are refused."""
    torch = pytest.importorskip("torch")
    spec = synth.LayerSpec(512, 16, 4, 256, 256, Q.DTYPE_Q4_K)
    layer = synth.make_layer(spec, 61)
    L = synth.open_layer(layer)
    lib = nc.lib()
    try:
        xs = [synth.make_x(T, spec.d, 61 + T) for T in (3, 200, 1, 96)]
        want = [L.forward(x) for x in xs]
        ins = [torch.from_numpy(x).pin_memory() if i % 2 else torch.from_numpy(x.copy()) for i, x in enumerate(xs)]
        outs = [torch.empty_like(t).pin_memory() if i % 2 else torch.empty_like(t) for i, t in enumerate(ins)]
        for rnd in range(2):
            for i, (xi, oi) in enumerate(zip(ins, outs)):
                assert lib.aero_cuda_moe_submit(L.handle, i % 2, xi.data_ptr(), xi.shape[0], oi.data_ptr()) == 0, \
                    nc.last_error(L.handle)
            for slot in (0, 1):
                assert lib.aero_cuda_moe_wait(L.handle, slot) == 0
            # the first two calls were waited for by the later submits to their slots
            for i in range(4):
                assert np.array_equal(outs[i].numpy(), want[i]), (rnd, i)
        xd = torch.from_numpy(xs[0]).cuda()
        assert lib.aero_cuda_moe_submit(L.handle, 0, xd.data_ptr(), 3, outs[0].data_ptr()) == -1
        assert "host buffers" in nc.last_error(L.handle)
        assert lib.aero_cuda_moe_submit(L.handle, 4, ins[0].data_ptr(), 3, outs[0].data_ptr()) == -1
    finally:
        L.close()
