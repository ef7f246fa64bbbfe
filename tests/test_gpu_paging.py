"""Router-ahead expert paging (PagedMoeLayer, aero_cuda_moe_page_in): a layer whose
16 experts live on the host with 6 resident on the device. Every call's output equals
the whole layer's block on the same logits (the separate-kernel path, bit for bit:
the same kernels over the same expert bytes) and the oracle's within the decode bar;
experts are paged in only when a call needs them, least recently used first."""

import os

import numpy as np
import pytest

import oracle as O
from aero_b200 import moe as M
from aero_b200 import native_cuda as nc
from aero_b200 import quant as Q
from aero_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib(cuda_lib):
    nc.require_gpu()


def _layer(dt=Q.DTYPE_Q8_0):
    spec = synth.LayerSpec(256, 16, 2, 256, 256, dt)
    layer = synth.make_layer(spec, 71)
    per = layer.gate.size // spec.E

    def expert_bytes(e):
        return (layer.gate[e * per:(e + 1) * per], layer.up[e * per:(e + 1) * per], layer.down[e * per:(e + 1) * per])

    return spec, layer, expert_bytes


@pytest.mark.parametrize("dt", [Q.DTYPE_Q8_0, Q.DTYPE_Q4_K])
def test_paged_layer_matches_the_whole_layer(dt):
    spec, layer, expert_bytes = _layer(dt)
    cfg = M.MoeConfig(n_expert=spec.E, n_expert_used=spec.k, n_embd=spec.d, ffn_len=spec.F, has_shared=True)
    P = M.PagedMoeLayer(cfg, expert_bytes, dt, layer.router, n_slots=6, shexp=layer.shexp)
    full = synth.open_layer(layer)
    full.set_decode_fused(False)
    try:
        for i in range(8):
            x = synth.make_x(2, spec.d, 100 + i)
            got = P.forward(x)
            lg = full.router_logits(x)
            assert np.array_equal(got, full.ffn_block(x, lg)), i
            ref = O.moe_block(layer, x, lg, nthreads=os.cpu_count() or 1)
            err = float(np.abs(got - ref).max()) / float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
            assert err <= 2e-3, (i, err)
            idx, _ = nc.route(lg, spec.E, spec.k)
            assert set(int(e) for e in idx.reshape(-1)) <= set(P.slot_expert)
        assert P.pages > 0
        resident = np.zeros(6, np.int32)
        assert nc.lib().aero_cuda_moe_resident(P.layer.handle, resident.ctypes.data, 6) == 6
        assert resident.tolist() == P.slot_expert
    finally:
        P.close()
        full.close()


def test_paging_refusals_and_lru():
    spec, layer, expert_bytes = _layer()
    cfg = M.MoeConfig(n_expert=spec.E, n_expert_used=spec.k, n_embd=spec.d, ffn_len=spec.F, has_shared=True)
    P = M.PagedMoeLayer(cfg, expert_bytes, Q.DTYPE_Q8_0, layer.router, n_slots=3, shexp=layer.shexp)
    lib = nc.lib()
    try:
        g, u, d = (np.ascontiguousarray(b) for b in expert_bytes(9))
        h = P.layer.handle
        assert lib.aero_cuda_moe_page_in(h, 3, 9, g.ctypes.data, u.ctypes.data, d.ctypes.data) == -1  # no slot 3
        assert lib.aero_cuda_moe_page_in(h, 0, 16, g.ctypes.data, u.ctypes.data, d.ctypes.data) == -1  # no expert 16
        assert lib.aero_cuda_moe_page_in(h, 0, 1, g.ctypes.data, u.ctypes.data, d.ctypes.data) == -1  # 1 is in slot 1
        assert "resident in slot 1" in nc.last_error(h)
        # a call routing to more experts than the device holds is refused
        x = synth.make_x(8, spec.d, 5)
        lg = P.layer.router_logits(x)
        idx, _ = nc.route(lg, spec.E, spec.k)
        if len(set(idx.reshape(-1).tolist())) > 3:
            with pytest.raises(ValueError, match="the device holds 3"):
                P.forward(x)
        # one token: two experts; the slot paged over is the least recently used one
        x1 = synth.make_x(1, spec.d, 6)
        P.forward(x1)
        before = list(P.slot_expert)
        x2 = synth.make_x(1, spec.d, 7)
        need2 = set(nc.route(P.layer.router_logits(x2), spec.E, spec.k)[0].reshape(-1).tolist())
        P.forward(x2)
        kept = [e for e in before if e in P.slot_expert]
        assert need2 <= set(P.slot_expert) and len(kept) >= 1
    finally:
        P.close()
