"""The fused decode kernel (calls of up to 32 tokens in one cooperative launch)
against the oracle and against the separate-kernel path of the same library.

Bar: max-abs-error <= 2e-3 x RMS(output) (the decode bar: f32 accumulation over
integer-coded inputs); repeated calls bit-identical."""

import os

import numpy as np
import pytest

import oracle as O
from aero_b200 import native_cuda as nc
from aero_b200 import quant as Q
from aero_b200 import synth

pytestmark = pytest.mark.gpu
DECODE_TOL = 2e-3


def rms(a):
    return float(np.sqrt(np.mean(np.asarray(a, np.float64) ** 2)))


def rel_err(got, want):
    return float(np.abs(np.asarray(got, np.float64) - want).max()) / max(rms(want), 1e-12)


@pytest.fixture(scope="module", autouse=True)
def _lib(cuda_lib):
    nc.require_gpu()


def _min_gap(lg, k):
    top = -np.sort(-lg.astype(np.float64), axis=1)[:, :k + 1]
    return float(np.min(top[:, :-1] - top[:, 1:]))


@pytest.mark.parametrize("dt", [Q.DTYPE_Q4_K, Q.DTYPE_Q8_0])
@pytest.mark.parametrize("T", [1, 2, 3, 17, 32])
def test_fused_decode_matches_oracle_and_separate_kernels(dt, T):
    spec = synth.LayerSpec(512, 24, 4, 256, 256, dt)
    layer = synth.make_layer(spec, 51)
    x = synth.make_x(T, spec.d, 51 + T)
    L = synth.open_layer(layer)
    try:
        lg = L.router_logits(x)
        a = L.ffn_block(x, lg)
        b = L.ffn_block(x, lg)
        f = L.forward(x)  # the fused kernel's own router
        assert L.status() == 0
        L.set_decode_fused(False)
        c = L.ffn_block(x, lg)
    finally:
        L.close()
    ref = O.moe_block(layer, x, lg, nthreads=os.cpu_count() or 1)
    assert rms(ref) > 1e-3
    assert np.array_equal(a, b), "fused decode is not deterministic"
    assert rel_err(a, ref) <= DECODE_TOL, rel_err(a, ref)
    assert rel_err(c, ref) <= DECODE_TOL
    if _min_gap(lg, spec.k) > 1e-4:  # no near-tie: the in-kernel router selects the same experts
        assert rel_err(f, ref) <= DECODE_TOL


@pytest.mark.parametrize("case", ["no_shared_norm0", "wide", "k32_E1024"])
def test_fused_decode_shapes(case):
    """No shared expert with norm_topk_prob = 0 (full-softmax weights); a 2048-wide layer
    with F = 768 (16-lane row groups with idle lanes in the down product); k = 32 of 1024
    experts at 32 tokens with F = 192 (the dispatch tables at their limit, 3 of 4 lanes
    active per down row)."""
    if case == "no_shared_norm0":
        spec = synth.LayerSpec(256, 40, 6, 256, 0, Q.DTYPE_Q8_0, norm_topk_prob=False)
        T = 9
    elif case == "wide":
        spec = synth.LayerSpec(2048, 16, 4, 768, 768, Q.DTYPE_Q4_K)
        T = 5
    else:
        spec = synth.LayerSpec(256, 1024, 32, 192, 192, Q.DTYPE_Q8_0)
        T = 32
    layer = synth.make_layer(spec, 52)
    x = synth.make_x(T, spec.d, 52)
    L = synth.open_layer(layer)
    try:
        lg = L.router_logits(x)
        a = L.ffn_block(x, lg)
        L.set_decode_fused(False)
        c = L.ffn_block(x, lg)
    finally:
        L.close()
    ref = O.moe_block(layer, x, lg, nthreads=os.cpu_count() or 1)
    assert rms(ref) > 1e-4
    assert rel_err(a, ref) <= DECODE_TOL, (case, rel_err(a, ref))
    assert rel_err(c, ref) <= DECODE_TOL


def test_fused_decode_host_and_device_buffers_and_many_calls():
    """Host and device pointers give the same result; a few hundred calls in a row keep the
    grid-barrier counter in step (every call's result equal to the first)."""
    torch = pytest.importorskip("torch")
    spec = synth.LayerSpec(512, 16, 4, 256, 256, Q.DTYPE_Q4_K)
    layer = synth.make_layer(spec, 53)
    x = synth.make_x(4, spec.d, 53)
    L = synth.open_layer(layer)
    try:
        a = L.forward(x)
        xd = torch.from_numpy(x).cuda()
        outs = [L.forward(xd) for _ in range(300)]
        torch.cuda.synchronize()
        assert all(np.array_equal(o.cpu().numpy(), a) for o in outs[::37])
        assert np.array_equal(outs[-1].cpu().numpy(), a)
        assert L.status() == 0
    finally:
        L.close()
