"""GGUF files written by the reference's own GGUFWriter (engine/gguf.py:448-526),
read through this library's loader (tests/golden/make_golden.py writes them
around synth layers and records the reference block's output on each).

CPU: the files are the recorded ones, and aero_cuda_moe_gguf_info reads each
layer's description (metadata of every value kind and unrelated tensors around
it). GPU: aero_cuda_moe_open_gguf opens the layer and its block output matches
the reference's at the decode bar."""

import hashlib
import os

import numpy as np
import pytest

from aero_b200 import moe as M

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DECODE_TOL = 2e-3


def _path(name):
    return os.path.join(HERE, f"ref_writer_{name}.gguf")


def test_fixture_files_are_the_recorded_ones(golden):
    for name in golden["gguf_names"]:
        with open(_path(name), "rb") as fh:
            assert hashlib.sha256(fh.read()).hexdigest() == str(golden[f"{name}_file_sha"]), name


def test_layer_info_from_reference_written_files(golden):
    for name in golden["gguf_names"]:
        d, E, k, F, Fs, dtype, norm, _, _ = (int(v) for v in golden[f"{name}_spec"])
        info = M.gguf_layer_info(_path(name), int(golden[f"{name}_layer"]))
        cfg = info["config"]
        assert (cfg.n_embd, cfg.n_expert, cfg.n_expert_used, cfg.ffn_len) == (d, E, k, F), name
        assert info["ffn_len_shared"] == Fs and cfg.has_shared == bool(Fs), name
        assert info["dtype"] == dtype and info["has_router"], name
        with pytest.raises(ValueError, match="not a MoE layer"):
            M.gguf_layer_info(_path(name), int(golden[f"{name}_layer"]) + 5)
    with pytest.raises(ValueError):
        M.gguf_layer_info(os.path.join(HERE, "golden.npz"), 0)  # not a GGUF file


@pytest.mark.gpu
def test_open_reference_written_gguf_matches_reference_block(golden, cuda_lib):
    from aero_b200 import native_cuda as nc

    nc.require_gpu()
    for name in golden["gguf_names"]:
        x, lg = golden[f"{name}_x"], golden[f"{name}_logits"]
        L = M.CudaMoeLayer.from_gguf(_path(name), int(golden[f"{name}_layer"]))
        try:
            outs = [L.ffn_block(x, lg)]
            # the router read from the file: same logits (f32), so the same routing
            np.testing.assert_allclose(L.router_logits(x), lg, rtol=1e-5, atol=1e-5)
            outs.append(L.forward(x))
        finally:
            L.close()
        want = golden[f"{name}_out"].astype(np.float64)
        rms = float(np.sqrt(np.mean(want ** 2)))
        for out in outs:
            err = float(np.abs(out - want).max()) / rms
            assert err <= DECODE_TOL, (name, err)
