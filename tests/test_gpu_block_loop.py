"""The reference's native block loop driving this library (the drop-in of
src/model.cpp:166-170, 385-387): the loop compiled from the reference's sources
(oracle/_ref/libaero_model.so) runs its own C++ attention, and its MoE hook is
aero_cuda_moe_model_forward from this library with the whole file's MoE layers
in one table, called from C with no Python in the loop.

Against the logits the same loop produced with the reference's own MoE block as
the hook (tests/golden/make_golden.py). Bar: per call, max-abs-error of the
logits <= 2e-3 x RMS(logits) x n_layer (each layer's MoE output is within the
decode bar 2e-3 x RMS of the reference's; the residual stream carries them)."""

import ctypes
import hashlib

import numpy as np
import pytest

import ref_model as R
from aero_b200 import native_cuda as nc
from aero_b200 import synth

pytestmark = pytest.mark.gpu


def decoder_fixture(golden, name, tmp_path):
    sp = [int(v) for v in golden[f"{name}_spec"]]
    fs = golden[f"{name}_fspec"]
    n_layer, d, H, HK, D, vocab, md, E, k, F, Fs, mdt, adt, edt, tied, qkn, seed = sp
    spec = synth.DecoderSpec(n_layer, d, H, HK, D, vocab, synth.LayerSpec(md, E, k, F, Fs, mdt),
                             rope_base=float(fs[0]), eps=float(fs[1]), attn_dtype=adt, embd_dtype=edt,
                             tied=bool(tied), qk_norm=bool(qkn))
    path = str(tmp_path / f"{name}.gguf")
    synth.write_decoder_gguf(synth.make_decoder(spec, seed), path)
    with open(path, "rb") as fh:
        assert hashlib.sha256(fh.read()).hexdigest() == str(golden[f"{name}_file_sha"]), name
    return spec, path


def calls_of(golden, name, s):
    toks = golden[f"{name}_s{s}_tokens"]
    n_prompt = int(golden[f"{name}_s{s}_prompt"])
    calls = [(0, n_prompt)] + [(i, i + 1) for i in range(n_prompt, toks.size)]
    return toks, calls


@pytest.mark.parametrize("name", ["dec_q8", "dec_q4k_tied"])
def test_reference_block_loop_with_cuda_moe_hook(golden, cuda_lib, tmp_path, name):
    if not R.available():
        pytest.skip("the reference's block loop was not built (make -C oracle ref)")
    nc.require_gpu()
    spec, path = decoder_fixture(golden, name, tmp_path)
    ours = nc.lib()
    err = ctypes.create_string_buffer(512)
    table = ours.aero_cuda_moe_model_open_gguf(path.encode(), 0, 0, err, 512)
    assert table, err.value.decode()
    ref = R.load()
    try:
        assert ours.aero_cuda_moe_model_layer(table, spec.n_layer) is None
        for s in range(int(golden[f"{name}_n_seq"])):
            toks, calls = calls_of(golden, name, s)
            want = golden[f"{name}_s{s}_logits"]
            m = R.open_model(ref, path, spec)
            try:
                fn = ctypes.cast(ours.aero_cuda_moe_model_forward, ctypes.c_void_p)
                ref.aero_model_set_moe(m, fn, table)
                for ci, (a, b) in enumerate(calls):
                    tk = np.ascontiguousarray(toks[a:b])
                    pos = np.arange(a, b, dtype=np.int64)
                    got = np.empty(spec.vocab, np.float32)
                    assert ref.aero_model_forward(m, tk.ctypes.data, b - a, pos.ctypes.data, got.ctypes.data) == 1
                    rms = float(np.sqrt(np.mean(want[ci].astype(np.float64) ** 2)))
                    e = float(np.abs(got - want[ci]).max()) / rms
                    assert e <= 2e-3 * spec.n_layer, (name, s, ci, e)
            finally:
                ref.aero_model_free(m)
    finally:
        ours.aero_cuda_moe_model_close(table)


def test_model_table_refuses_dense_layers_and_bad_files(cuda_lib, tmp_path):
    nc.require_gpu()
    ours = nc.lib()
    err = ctypes.create_string_buffer(512)
    # a GGUF with one MoE layer at index 1: layer 0 is empty, its hook call returns 0
    layer = synth.make_layer(synth.LayerSpec(256, 4, 2, 64, 0), 3)
    p = str(tmp_path / "one.gguf")
    synth.write_gguf(layer, p, layer_index=1)
    table = ours.aero_cuda_moe_model_open_gguf(p.encode(), 2, 0, err, 512)
    assert table, err.value.decode()
    try:
        x = synth.make_x(2, 256, 3)
        out = np.zeros_like(x)
        assert ours.aero_cuda_moe_model_forward(table, 0, x.ctypes.data, 2, 256, out.ctypes.data) == 0
        assert ours.aero_cuda_moe_model_forward(table, 1, x.ctypes.data, 2, 256, out.ctypes.data) == 1
        assert ours.aero_cuda_moe_model_forward(table, 7, x.ctypes.data, 2, 256, out.ctypes.data) == 0
        assert float(np.abs(out).max()) > 0
    finally:
        ours.aero_cuda_moe_model_close(table)
    p2 = str(tmp_path / "none.gguf")
    with open(p2, "wb") as fh:
        fh.write(b"not a gguf file")
    assert not ours.aero_cuda_moe_model_open_gguf(p2.encode(), 1, 0, err, 512)
