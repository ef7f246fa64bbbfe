"""The CUDA decoder (include/aero_cuda_decoder.h) against the logits of the
reference's own native block loop (src/model.cpp with its C++ attention and the
reference MoE block as the MoE hook; tests/golden/make_golden.py) on the same
synthetic decoder files, prompts then single-token steps.

The reference's cache is fp32 and ours f16 (its native slots hold fp32, int8 or
int4 only, src/kv.cpp), the attention projections take the integer-coded input
rows (2^-15 of each 32-value block's largest input) and each MoE layer is within
the decode bar of the reference's. Bar: per call, max-abs-error of the logits
<= 2e-3 x RMS(logits) (measured: 1.3e-4 and 6.9e-5); every logit row's argmax equal."""

import numpy as np
import pytest

from aero_b200 import native_cuda as nc
from aero_b200 import synth
from aero_b200.decoder import CudaDecoder
from test_gpu_block_loop import calls_of, decoder_fixture

pytestmark = pytest.mark.gpu
TOL = 2e-3


@pytest.fixture(scope="module", autouse=True)
def _lib(cuda_lib):
    nc.require_gpu()


def rel(got, want):
    want = np.asarray(want, np.float64)
    return float(np.abs(np.asarray(got, np.float64) - want).max()) / float(np.sqrt(np.mean(want ** 2)))


@pytest.mark.parametrize("name", ["dec_q8", "dec_q4k_tied"])
def test_decoder_forward_matches_reference_block_loop(golden, tmp_path, name):
    spec, path = decoder_fixture(golden, name, tmp_path)
    errs = []
    for s in range(int(golden[f"{name}_n_seq"])):
        toks, calls = calls_of(golden, name, s)
        want = golden[f"{name}_s{s}_logits"]
        dec = CudaDecoder.from_gguf(path, n_seq=1, n_ctx=64)
        try:
            for ci, (a, b) in enumerate(calls):
                got = dec.forward(toks[a:b], np.arange(a, b))
                e = rel(got, want[ci])
                errs.append(e)
                assert e <= TOL, (name, s, ci, e)
                assert int(np.argmax(got)) == int(np.argmax(want[ci])), (name, s, ci)
        finally:
            dec.close()
    print(f"{name}: max logit error / RMS per call {max(errs):.2e}")


def test_decoder_batched_sequences(golden, tmp_path):
    """Both sequences of dec_q8 in one decoder: their prompts in one step (each prompt's
    tokens attend causally within it, not across sequences), then both single tokens per
    step; every row equals the reference's call for its sequence."""
    name = "dec_q8"
    spec, path = decoder_fixture(golden, name, tmp_path)
    seqs = [calls_of(golden, name, s) for s in range(2)]
    wants = [golden[f"{name}_s{s}_logits"] for s in range(2)]
    dec = CudaDecoder.from_gguf(path, n_seq=2, n_ctx=64)
    try:
        (t0, c0), (t1, c1) = seqs
        p0, p1 = c0[0][1], c1[0][1]
        tokens = np.concatenate([t0[:p0], t1[:p1]])
        sq = np.array([0] * p0 + [1] * p1)
        pos = np.concatenate([np.arange(p0), np.arange(p1)])
        out = dec.step(tokens, sq, pos)
        assert rel(out[p0 - 1], wants[0][0]) <= TOL and rel(out[p0 + p1 - 1], wants[1][0]) <= TOL
        n = min(len(c0), len(c1)) - 1
        for i in range(n):
            a0, a1 = c0[1 + i][0], c1[1 + i][0]
            out = dec.step([t0[a0], t1[a1]], [0, 1], [a0, a1])
            assert rel(out[0], wants[0][1 + i]) <= TOL, (0, i)
            assert rel(out[1], wants[1][1 + i]) <= TOL, (1, i)
    finally:
        dec.close()


def test_decoder_from_tensors_equals_from_gguf_and_device_logits(golden, tmp_path):
    torch = pytest.importorskip("torch")
    name = "dec_q8"
    spec, path = decoder_fixture(golden, name, tmp_path)
    sp = [int(v) for v in golden[f"{name}_spec"]]
    dec_s = synth.make_decoder(spec, sp[-1])
    A = CudaDecoder.from_gguf(path, n_seq=1, n_ctx=64)
    B = CudaDecoder.from_synth(dec_s, n_seq=1, n_ctx=64)
    try:
        toks, calls = calls_of(golden, name, 0)
        for a, b in calls:
            la = A.forward(toks[a:b], np.arange(a, b))
            dev = torch.empty(spec.vocab, device="cuda")
            B.forward(toks[a:b], np.arange(a, b), logits=dev)
            torch.cuda.synchronize()
            assert np.array_equal(la, dev.cpu().numpy())
        # no head: the step only fills the cache
        assert B.step([1], [0], [calls[-1][1]], logits=None) is None
    finally:
        A.close()
        B.close()


def test_decoder_refusals(golden, tmp_path):
    spec, path = decoder_fixture(golden, "dec_q8", tmp_path)
    dec = CudaDecoder.from_gguf(path, n_seq=2, n_ctx=16)
    try:
        for args in (([1], [0], [16]),          # position outside the cache
                     ([1, 2], [0, 0], [3, 3]),  # one (sequence, position) twice
                     ([spec.vocab], [0], [0]),  # token outside the vocabulary
                     ([1], [2], [0])):          # sequence outside the cache
            with pytest.raises(RuntimeError):
                dec.step(*args)
        dec.step([1, 2], [0, 1], [0, 0])  # still usable
    finally:
        dec.close()
    with pytest.raises(RuntimeError):
        CudaDecoder.from_gguf(str(tmp_path / "missing.gguf"))


def test_decoder_graph_replay_equals_eager(golden, tmp_path, monkeypatch):
    """Decode steps replayed from the captured CUDA graph (from a key's third call on)
    give the same logits as eager steps, batched and single, with host and device logits."""
    torch = pytest.importorskip("torch")
    spec, path = decoder_fixture(golden, "dec_q8", tmp_path)
    monkeypatch.setenv("AERO_DECODER_GRAPHS", "0")
    E = CudaDecoder.from_gguf(path, n_seq=3, n_ctx=64)
    monkeypatch.setenv("AERO_DECODER_GRAPHS", "1")
    G = CudaDecoder.from_gguf(path, n_seq=3, n_ctx=64)
    try:
        rng = np.random.default_rng(8)
        prompt = rng.integers(0, spec.vocab, 12)
        seqs = np.repeat(np.arange(3), 4)
        pos = np.tile(np.arange(4), 3)
        assert np.array_equal(E.step(prompt, seqs, pos), G.step(prompt, seqs, pos))
        dev_e = torch.empty((3, spec.vocab), device="cuda")
        dev_g = torch.empty((3, spec.vocab), device="cuda")
        for i in range(6):
            tok = rng.integers(0, spec.vocab, 3)
            p = np.full(3, 4 + i)
            a, b = E.step(tok, [0, 1, 2], p), G.step(tok, [0, 1, 2], p)
            assert np.array_equal(a, b), i
            E.step(tok[:1], [0], [20 + i], logits=dev_e[:1])
            G.step(tok[:1], [0], [20 + i], logits=dev_g[:1])
            torch.cuda.synchronize()
            assert torch.equal(dev_e[:1], dev_g[:1]), i
    finally:
        E.close()
        G.close()


def test_decoder_open_charges_exactly_its_plan(golden, tmp_path):
    """Opening a decoder (its MoE handles and its own weights and caches) adds exactly
    plan_footprint's bytes to the guard's resident-weights and KV-cache classes, and
    closing it returns them."""
    from aero_b200.decoder import plan_footprint
    spec, _ = decoder_fixture(golden, "dec_q8", tmp_path)
    seed = int(golden["dec_q8_spec"][-1])
    g = nc.MemoryGuard()

    def held():
        return g.committed(nc.MEM_WEIGHTS_RESIDENT) + g.committed(nc.MEM_KV_CACHE)

    before = held()
    plan = plan_footprint(spec, n_seq=3, n_ctx=48)
    D = CudaDecoder.from_synth(synth.make_decoder(spec, seed), n_seq=3, n_ctx=48)
    try:
        assert held() - before == plan["total"], (held() - before, plan)
        assert g.committed(nc.MEM_KV_CACHE) >= plan["kv_cache"]
    finally:
        D.close()
    assert held() == before


@pytest.mark.parametrize("attn_dtype", [synth.DTYPE_Q8_0, synth.DTYPE_Q4_K])
def test_decoder_batched_steps_match_single_steps_at_full_width(attn_dtype):
    """At the config-4 widths (d 2048, 32 x 128 query heads, 4 kv heads; Q8_0 head,
    Q4_K experts, Q8_0 or Q4_K projections), steps of 16 sequences at once (Q8_0: the
    dense projections and head on the integer tensor-core kernel; Q4_K projections:
    the multi-token CUDA-core kernel) give the logits of the same tokens run one at a
    time (the single-token kernels, the 4096-wide output projection split over two
    warps per row), within the decode bar of their RMS; every argmax equal."""
    spec = synth.DecoderSpec(2, 2048, 32, 4, 128, 4096, synth.LayerSpec(2048, 16, 4, 768, 0, synth.DTYPE_Q4_K),
                             attn_dtype=attn_dtype)
    dec = synth.make_decoder(spec, 5, device_gen=True)
    B = CudaDecoder.from_synth(dec, n_seq=16, n_ctx=32)
    S = CudaDecoder.from_synth(dec, n_seq=16, n_ctx=32)
    try:
        rng = np.random.default_rng(6)
        errs = []
        for p in range(3):
            tok = rng.integers(0, spec.vocab, 16)
            batched = B.step(tok, np.arange(16), np.full(16, p))
            for sq in range(16):
                one = S.step(tok[sq:sq + 1], [sq], [p])[0]
                e = rel(batched[sq], one)
                errs.append(e)
                assert e <= TOL, (p, sq, e)
                assert int(np.argmax(batched[sq])) == int(np.argmax(one)), (p, sq)
        print(f"batched vs single steps: max logit error / RMS {max(errs):.2e}")
    finally:
        B.close()
        S.close()


class _Dev:
    """A device buffer (address, shape, numpy type string) for torch.as_tensor."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape), "typestr": typestr, "version": 3}


def test_decoder_long_cache_merged_chunks_match_single_steps():
    """Over a 2048-position cache (the same N(0, 1) f16 keys and values in two
    decoders), a step of 16 sequences at position 1900 (attention CTAs merge several
    64-position chunks online before the combine) gives the logits of the same
    tokens stepped one at a time (one chunk per CTA), within the decode bar."""
    torch = pytest.importorskip("torch")
    spec = synth.DecoderSpec(1, 2048, 32, 4, 128, 2048, synth.LayerSpec(2048, 8, 2, 256, 0, synth.DTYPE_Q4_K))
    dec = synth.make_decoder(spec, 9, device_gen=True)
    n_ctx, p = 2048, 1900
    B = CudaDecoder.from_synth(dec, n_seq=16, n_ctx=n_ctx)
    S = CudaDecoder.from_synth(dec, n_seq=16, n_ctx=n_ctx)
    try:
        g = torch.Generator(device="cuda").manual_seed(3)
        shape = (16, spec.n_kv, n_ctx, spec.head_dim)
        for li in range(spec.n_layer):
            for pb, ps in zip(B.kv(li), S.kv(li)):
                vals = torch.randn(shape, generator=g, device="cuda").half()
                torch.as_tensor(_Dev(pb, shape, "<f2"), device="cuda").copy_(vals)
                torch.as_tensor(_Dev(ps, shape, "<f2"), device="cuda").copy_(vals)
        torch.cuda.synchronize()
        tok = np.random.default_rng(4).integers(0, spec.vocab, 16)
        batched = B.step(tok, np.arange(16), np.full(16, p))
        errs = []
        for sq in range(16):
            one = S.step(tok[sq:sq + 1], [sq], [p])[0]
            e = rel(batched[sq], one)
            errs.append(e)
            assert e <= TOL, (sq, e)
        print(f"long cache, merged chunks vs single steps: max logit error / RMS {max(errs):.2e}")
    finally:
        B.close()
        S.close()
