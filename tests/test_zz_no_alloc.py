"""aero_cuda_dispatch_noalloc against aero_cuda_dispatch, through the C ABI.

The no-alloc variant serves callers that must not allocate device memory while
they route tokens (a fully committed device budget, or a pipeline that cannot
take cudaMalloc's implicit synchronisation); it runs on a fixed scratch array
inside the library. This file is collected last on purpose: if it fails, a run
that stops at the first failure has already run every other test. It must pass
both alone in a fresh process and after the other tests.
"""

import numpy as np
import pytest

import oracle as O
from aero_b200 import native_cuda as nc

pytestmark = pytest.mark.gpu


def _noalloc(lib, torch, idx, E, stream=None):
    T, k = idx.shape
    d_idx = torch.from_numpy(np.ascontiguousarray(idx, dtype=np.int64)).cuda()
    d_off = torch.full((E + 1,), -7, dtype=torch.int32, device="cuda")
    d_perm = torch.full((max(T * k, 1),), -7, dtype=torch.int32, device="cuda")
    rc = lib.aero_cuda_dispatch_noalloc(d_idx.data_ptr(), T, k, E, d_off.data_ptr(), d_perm.data_ptr(), stream)
    return rc, d_off.cpu().numpy(), d_perm.cpu().numpy()[: T * k]


def test_noalloc_dispatch_matches_allocating_dispatch(cuda_lib):
    torch = pytest.importorskip("torch")
    nc.require_gpu()
    lib = cuda_lib
    g = nc.MemoryGuard()
    rng = np.random.default_rng(11)
    # two calls in a row with different shapes: the second must not see the
    # first call's leftovers in the shared scratch
    cases = [(8192, 8, 128), (37, 10, 512)]
    for T, k, E in cases:
        idx = rng.integers(0, E, size=(T, k))
        idx[: T // 3, 0] = 5  # a dominant expert
        committed = g.committed()
        rc, off, perm = _noalloc(lib, torch, idx, E)
        assert rc == 0, nc.last_error()
        assert g.committed() == committed  # nothing was charged to the guard
        ref_off, ref_perm = nc.dispatch(idx, E)  # the existing, allocating entry point
        assert np.array_equal(off, ref_off) and np.array_equal(perm, ref_perm), (T, k, E)
        o_off, o_perm = O.dispatch(idx, E)
        assert np.array_equal(off, o_off) and np.array_equal(perm, o_perm)


def test_noalloc_dispatch_refusals(cuda_lib):
    torch = pytest.importorskip("torch")
    nc.require_gpu()
    lib = cuda_lib
    # beyond the stated maximum: refused with a clear reason
    rc, _, _ = _noalloc(lib, torch, np.zeros((8193, 8), np.int64), 128)
    assert rc == -1 and "at most 65536" in nc.last_error()
    rc, _, _ = _noalloc(lib, torch, np.zeros((4, 2), np.int64), 2048)
    assert rc == -1 and "1024 experts" in nc.last_error()
    # host buffers are refused (staging them would need an allocation)
    idx = np.zeros((2, 2), np.int64)
    off = np.zeros(5, np.int32)
    perm = np.zeros(4, np.int32)
    assert lib.aero_cuda_dispatch_noalloc(idx.ctypes.data, 2, 2, 4, off.ctypes.data, perm.ctypes.data, None) == -1
    assert "device pointers" in nc.last_error()
    # an out-of-range expert id is reported, and the next call is clean again
    rc, _, _ = _noalloc(lib, torch, np.array([[0, 9]], np.int64), 4)
    assert rc == -1 and "out of range" in nc.last_error()
    rc, off, perm = _noalloc(lib, torch, np.array([[3, 1], [1, 0]], np.int64), 4)
    assert rc == 0 and list(off) == [0, 1, 3, 3, 4] and list(perm) == [3, 1, 2, 0]
