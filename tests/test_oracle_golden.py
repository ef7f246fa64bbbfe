"""Pin the CPU oracle to the reference's own outputs (CPU only).

The golden file was produced by the reference itself (tests/golden/make_golden.py):
engine/quant.py + src/kernels.cpp dequantisation, src/moe.cpp routing and the
engine/moe.py -> src/moe.cpp MoE block. The oracle (oracle/moe_oracle.c) must
reproduce them: bit-exact for dequantised values and routed indices, within
fp32 rounding for weights and block outputs.
"""

import hashlib

import numpy as np
import pytest

import oracle as O
from golden_blocks import block


def _names(golden, prefix):
    return sorted({k[len(prefix):].rsplit("_", 1)[0] for k in golden if k.startswith(prefix) and k.endswith("_raw")})


def test_dequant_bit_exact(golden):
    names = _names(golden, "deq_")
    assert len(names) >= 4
    for n in names:
        raw = golden[f"deq_{n}_raw"]
        want = golden[f"deq_{n}_out"]
        got = O.dequant(int(golden[f"deq_{n}_dtype"]), raw, want.size)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), n


def test_dequant_refuses_short_buffer(golden):
    raw = golden["deq_q8_random_raw"]
    with pytest.raises(ValueError):
        O.dequant(8, raw[:33], 32)


def test_hand_blocks(golden):
    # tests/test_quant.py:126-131: Q8_0 with d=0.5 over 0..31 -> 0.5*index
    out = golden["deq_q8_random_out"][15 * 32:16 * 32]
    assert np.array_equal(out, 0.5 * np.arange(32, dtype=np.float32))
    # tests/test_quant.py:71-93: Q4_K d=1, dmin=0, sc=1 -> the quants themselves
    out = golden["deq_q4k_random_out"][7 * 256:8 * 256]
    lo = np.array([i & 15 for i in range(128)], np.float32)
    hi = np.array([(31 - i) & 15 for i in range(128)], np.float32)
    want = np.concatenate([np.concatenate([lo[32 * j:32 * j + 32], hi[32 * j:32 * j + 32]]) for j in range(4)])
    assert np.array_equal(out, want)


def test_route_matches_reference(golden):
    for name in golden["route_names"]:
        lg = golden[f"route_{name}_logits"]
        k = int(golden[f"route_{name}_k"])
        for norm in (1, 0):
            idx, w = O.route(lg, k, bool(norm))
            assert np.array_equal(idx, golden[f"route_{name}_n{norm}_idx"]), (name, norm)
            np.testing.assert_allclose(w, golden[f"route_{name}_n{norm}_w"], rtol=1e-6, atol=1e-7)


def test_route_tie_rules(golden):
    assert list(golden["route_tie_3_7_n0_idx"]) == [3, 7]
    assert list(golden["route_fixed_1_4_n1_idx"]) == [1, 4]
    assert list(golden["route_all_zero_n1_idx"]) == [0, 1, 2]


def test_route_refuses_bad_k():
    lg = np.zeros(4, np.float32)
    for k in (0, 5):
        with pytest.raises(ValueError):
            O.route(lg, k)


def test_route_scan_equals_sort():
    rng = np.random.default_rng(3)
    for E, k in ((128, 8), (512, 10)):
        lg = np.round(rng.standard_normal(E) * 3).astype(np.float32)  # many ties
        idx, _ = O.route(lg, k)
        assert np.array_equal(idx, O.argsort_desc(lg)[:k].astype(np.int64))


def test_dispatch_is_stable_sort():
    rng = np.random.default_rng(4)
    for T, k, E in ((1, 8, 128), (32, 10, 512), (700, 4, 16)):
        idx = rng.integers(0, E, size=(T, k))
        off, perm = O.dispatch(idx, E)
        flat = idx.reshape(-1)
        assert np.array_equal(perm, np.argsort(flat, kind="stable"))
        assert np.array_equal(off, np.concatenate([[0], np.cumsum(np.bincount(flat, minlength=E))]))


def test_blocks_regenerate_and_match(golden):
    for name in golden["block_names"]:
        layer, g = block(golden, name)
        sh = [layer.shexp[k] for k in ("gate", "up", "down")] if layer.shexp else []
        h = hashlib.sha256()
        for a in (layer.router, layer.gate, layer.up, layer.down, *sh):
            h.update(np.ascontiguousarray(a).tobytes())
        assert h.hexdigest() == str(g["sha"]), f"{name}: synthetic layer bytes changed"
        out = O.moe_block(layer, g["x"], g["logits"])
        scale = float(np.sqrt(np.mean(g["out"].astype(np.float64) ** 2)))
        err = float(np.abs(out - g["out"]).max())
        assert err <= 1e-5 * max(scale, 1e-6), (name, err, scale)


def test_block_threads_identical(golden):
    layer, g = block(golden, "b_q8")
    a = O.moe_block(layer, g["x"], g["logits"], nthreads=1)
    b = O.moe_block(layer, g["x"], g["logits"], nthreads=3)
    assert np.array_equal(a, b)


def test_router_logits_close_to_reference(golden):
    layer, g = block(golden, "b_q4k_zipf")
    lg = O.router_logits(g["x"], layer.router, layer.router_bias)
    np.testing.assert_allclose(lg, g["logits"], rtol=1e-5, atol=1e-5)


@pytest.mark.skipif(not O.ref_available(), reason="reference objects not built here")
def test_reference_build_matches_oracle(golden):
    """The reference's own block (oracle/_ref) against the restatement."""
    for name in ("b_q8", "b_q4k"):
        layer, g = block(golden, name)
        ref = O.ref_block(layer, g["x"], g["logits"], nthreads=2)
        orc = O.moe_block(layer, g["x"], g["logits"])
        np.testing.assert_allclose(ref, g["out"], rtol=0, atol=1e-6)
        np.testing.assert_allclose(orc, ref, rtol=0, atol=1e-6)
