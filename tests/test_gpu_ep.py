"""Expert-parallel layer on the GPU.

One GPU: the ranks are threads, each with its own handle holding its expert
range and its own stream, exchanging through device copies in place of NCCL
(the kernels and the host protocol are the same as over NCCL). The sharded
result must match the single-handle layer over all tokens. With two or more
GPUs, the same over NCCL with one process per GPU.
"""

import os
import socket
import threading

import numpy as np
import pytest

import oracle as O
from aero_b200 import ep
from aero_b200 import native_cuda as nc
from aero_b200 import quant as Q
from aero_b200 import synth

pytestmark = pytest.mark.gpu
PREFILL_TOL = 1e-2


def rms(a):
    return float(np.sqrt(np.mean(np.asarray(a, np.float64) ** 2)))


def rel_err(got, want):
    return float(np.max(np.abs(np.asarray(got, np.float64) - want))) / max(rms(want), 1e-30)


class ThreadExchange:
    """all_to_all_single between threads of one process (device copies)."""

    def __init__(self, world):
        self.world = world
        self.board = [None] * world
        self.bar = threading.Barrier(world, timeout=120)

    def for_rank(self, rank):
        import torch

        def a2a(out, inp, out_splits, in_splits):
            n = self.world
            out_splits = out_splits or [out.shape[0] // n] * n
            in_splits = in_splits or [inp.shape[0] // n] * n
            torch.cuda.current_stream().synchronize()
            self.board[rank] = (inp, in_splits)
            self.bar.wait()
            off = 0
            for src in range(n):
                sinp, ss = self.board[src]
                assert ss[rank] == out_splits[src]
                so = sum(ss[:rank])
                c = out_splits[src]
                if c:
                    out[off:off + c].copy_(sinp[so:so + c])
                off += c
            torch.cuda.current_stream().synchronize()
            self.bar.wait()

        return a2a


def _run_threads(layer, x, world, row_f16, gemm_min=None):
    import torch

    T = x.shape[0]
    shards = ep.token_shards(T, world)
    begin = ep.expert_ranges(layer.spec.E, world)
    handles = [synth.open_layer(layer, expert_range=(begin[r], begin[r + 1])) for r in range(world)]
    if gemm_min is not None:
        for h in handles:
            h.set_gemm_min_tokens(gemm_min)
    xg = torch.from_numpy(x).cuda()
    xch = ThreadExchange(world)
    outs, errs = [None] * world, []

    def work(r):
        try:
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                m = ep.ExpertParallelMoe(ep.CudaEpOps(handles[r]), layer.spec.d, layer.spec.E, layer.spec.k, world, r,
                                         max_tokens=max(shards[i + 1] - shards[i] for i in range(world)),
                                         row_f16=row_f16, exchange=xch.for_rank(r))
                mine = xg[shards[r]:shards[r + 1]]
                o = m.forward(mine)
                o2 = m.forward(mine)  # a second step reuses the buffers
                s.synchronize()
                outs[r] = (o.cpu().numpy(), o2.cpu().numpy())
                m.close()
        except Exception as e:  # surfaced below
            errs.append(f"rank {r}: {e!r}")
            xch.bar.abort()

    th = [threading.Thread(target=work, args=(r,)) for r in range(world)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=300)
    try:
        assert not errs, errs
        for h in handles:
            assert ep.CudaEpOps(h).lib.aero_cuda_ep_bad_ids(h.handle) == 0
    finally:
        for h in handles:
            h.close()
    a = np.concatenate([o[0] for o in outs], 0)
    b = np.concatenate([o[1] for o in outs], 0)
    return a, b


@pytest.mark.parametrize("world", [2, 4])
def test_ep_prefill_matches_single_gpu(world):
    """c5-shaped layer (512 experts, top-10, shared expert, Q4_K), 2048 tokens, f16 rows."""
    nc.require_gpu()
    wl = synth.CONFIGS["c5"]
    layer = synth.make_layer(wl.spec, 0, device_gen=True)
    x = synth.make_x(2048, wl.spec.d, 4)
    L = synth.open_layer(layer)
    try:
        L.set_gemm_min_tokens(1)
        single = L.forward(x)
        lg = L.router_logits(x)
    finally:
        L.close()
    a, b = _run_threads(layer, x, world, row_f16=True)
    assert np.array_equal(a, b), "second step differs"
    # same f16 expert products; the per-rank partial sums are rounded to f16 once
    # for the return exchange
    assert rel_err(a, single) <= 5e-3
    sel = np.sort(np.random.default_rng(9).choice(x.shape[0], 128, replace=False))
    ref = O.moe_block(layer, x[sel], lg[sel], nthreads=os.cpu_count() or 1)
    assert rel_err(a[sel], ref) <= PREFILL_TOL


def test_ep_gemv_rows_uneven_experts():
    """Q8_0 layer, 24 experts over 5 ranks (5,5,5,5,4), f32 rows on the GEMV path."""
    nc.require_gpu()
    spec = synth.LayerSpec(1024, 24, 4, 256, 256, Q.DTYPE_Q8_0)
    layer = synth.make_layer(spec, 33)
    x = synth.make_x(45, spec.d, 33)
    L = synth.open_layer(layer)
    try:
        L.set_gemm_min_tokens(1 << 20)
        lg = L.router_logits(x)
    finally:
        L.close()
    a, _ = _run_threads(layer, x, 5, row_f16=False, gemm_min=1 << 20)
    ref = O.moe_block(layer, x, lg)
    assert rms(ref) > 1e-3
    assert rel_err(a, ref) <= 2e-3


def test_ep_refusals():
    nc.require_gpu()
    import torch

    spec = synth.LayerSpec(1024, 24, 4, 256, 0, Q.DTYPE_Q8_0)
    layer = synth.make_layer(spec, 34)
    L = synth.open_layer(layer, expert_range=(0, 12))
    lib = nc.lib()
    try:
        x = torch.zeros((4, 1024), device="cuda")
        slab = 32
        selfb = torch.zeros((4, 1024), device="cuda")
        selfm = torch.zeros((4, 10), dtype=torch.int32, device="cuda")
        buf = torch.zeros((2 * slab, 1024), device="cuda")  # two slabs
        meta = torch.zeros((2 * slab, 10), dtype=torch.int32, device="cuda")
        cnt = torch.zeros(3, dtype=torch.int32, device="cuda")
        pos = torch.zeros((4, 2), dtype=torch.int32, device="cuda")
        tab = (nc.c_int32 * 3)(0, 12, 24)

        def disp(rank, table, slab_rows=slab):
            return lib.aero_cuda_ep_dispatch(L.handle, x.data_ptr(), 4, 2, rank, table, 0, selfb.data_ptr(),
                                             selfm.data_ptr(), buf.data_ptr(), meta.data_ptr(), slab_rows,
                                             cnt.data_ptr(), pos.data_ptr())

        assert disp(0, tab) == 0
        torch.cuda.synchronize()
        # every row of the other rank's slab past its count names no expert
        c1 = int(cnt[1])
        assert bool((meta[slab + c1:, :4] == -1).all())
        assert disp(1, tab) == -1 and "this handle holds [0, 12)" in nc.last_error(L.handle)
        assert disp(0, (nc.c_int32 * 3)(0, 12, 20)) == -1 and "from 0 to 24" in nc.last_error(L.handle)
        assert disp(0, tab, slab_rows=3) == -1 and "slab_rows" in nc.last_error(L.handle)
        # a forward on a ranged handle is refused: it holds only some experts
        with pytest.raises(Exception):
            L.forward(np.zeros((2, 1024), np.float32))
        # ids this rank does not own are skipped and counted
        bad = torch.full((2, 10), -1, dtype=torch.int32, device="cuda")
        bad[0, 0] = 20
        out = torch.empty((2, 1024), device="cuda")
        assert lib.aero_cuda_ep_expert_block(L.handle, selfb.data_ptr(), 0, bad.data_ptr(), 2, 0, out.data_ptr(), 0) == 0
        assert lib.aero_cuda_ep_bad_ids(L.handle) == 1
        assert lib.aero_cuda_ep_bad_ids(L.handle) == 0
        assert float(out.abs().max()) == 0.0
    finally:
        L.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, q):
    try:
        import datetime

        import torch
        import torch.distributed as dist

        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        wl = synth.CONFIGS["c5"]
        layer = synth.make_layer(wl.spec, 0, device_gen=True)
        x = synth.make_x(1024, wl.spec.d, 4)
        shards = ep.token_shards(1024, world)
        begin = ep.expert_ranges(wl.spec.E, world)
        h = synth.open_layer(layer, device=rank, expert_range=(begin[rank], begin[rank + 1]))
        m = ep.ExpertParallelMoe(ep.CudaEpOps(h), wl.spec.d, wl.spec.E, wl.spec.k, world, rank,
                                 max_tokens=shards[1] - shards[0] + 1, device=f"cuda:{rank}")
        o = m.forward(torch.from_numpy(x[shards[rank]:shards[rank + 1]]).cuda())
        outs = [torch.empty((shards[r + 1] - shards[r], wl.spec.d), device=f"cuda:{rank}") for r in range(world)]
        dist.all_gather(outs, o)
        if rank == 0:
            q.put(("ok", torch.cat(outs).cpu().numpy()))
        dist.barrier()
        m.close()
        h.close()
        dist.destroy_process_group()
    except Exception as e:
        import traceback

        q.put(("err", f"rank {rank}: {e}\n{traceback.format_exc()}"))


def test_ep_nccl_two_gpus():
    import torch
    import torch.multiprocessing as mp

    nc.require_gpu()
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    msg = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert msg[0] == "ok", msg[1]
    wl = synth.CONFIGS["c5"]
    layer = synth.make_layer(wl.spec, 0, device_gen=True)
    x = synth.make_x(1024, wl.spec.d, 4)
    L = synth.open_layer(layer)
    try:
        L.set_gemm_min_tokens(1)
        single = L.forward(x)
    finally:
        L.close()
    assert rel_err(msg[1], single) <= 5e-3  # f16 partial rows cross the network


def _peer_worker(rank, world, port, q):
    try:
        import datetime

        import torch
        import torch.distributed as dist

        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        wl = synth.CONFIGS["c5"]
        layer = synth.make_layer(wl.spec, 0, device_gen=True)
        T = 1024
        x = synth.make_x(T, wl.spec.d, 4)
        shards = ep.token_shards(T, world)
        begin = ep.expert_ranges(wl.spec.E, world)
        dev = f"cuda:{rank}"
        h = synth.open_layer(layer, device=rank, expert_range=(begin[rank], begin[rank + 1]))
        mine = torch.from_numpy(x[shards[rank]:shards[rank + 1]]).to(dev)

        def gather(o):
            outs = [torch.empty((shards[r + 1] - shards[r], wl.spec.d), device=dev) for r in range(world)]
            dist.all_gather(outs, o.contiguous())
            return torch.cat(outs).cpu().numpy()

        # the all-to-all path first, as the reference for the peer path
        m = ep.ExpertParallelMoe(ep.CudaEpOps(h), wl.spec.d, wl.spec.E, wl.spec.k, world, rank, max_tokens=T,
                                 device=dev)
        ref = gather(m.forward(mine))
        torch.cuda.synchronize()
        m.close()
        p = ep.PeerExpertParallelMoe(h, wl.spec.d, wl.spec.E, wl.spec.k, world, rank, max_tokens=T, device=dev)
        o1 = gather(p.forward(mine))
        o2 = gather(p.forward(mine))  # second step: flags of the next epoch, buffers reused
        sent, recv = p.last_split
        # third step: every token on rank 0, none on the others
        x0 = torch.from_numpy(x).to(dev) if rank == 0 else torch.empty((0, wl.spec.d), device=dev)
        o3 = p.forward(x0)
        torch.cuda.synchronize()
        o3 = o3.cpu().numpy() if rank == 0 else None
        st = p.status()
        p.close()
        if rank == 0:
            q.put(("ok", (ref, o1, o2, o3, st, sent, recv)))
        dist.barrier()
        h.close()
        dist.destroy_process_group()
    except Exception as e:
        import traceback

        q.put(("err", f"rank {rank}: {e}\n{traceback.format_exc()}"))


def _peer_f32_worker(rank, world, port, q):
    """Decode-sized steps with f32 rows over peer memory: the GEMV path (16 tokens)
    and the GEMM path with f32 rows and f32 partials (128 tokens)."""
    try:
        import datetime

        import torch
        import torch.distributed as dist

        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        wl = synth.CONFIGS["c3"]
        layer = synth.make_layer(wl.spec, 1, device_gen=True)
        begin = ep.expert_ranges(wl.spec.E, world)
        dev = f"cuda:{rank}"
        h = synth.open_layer(layer, device=rank, expert_range=(begin[rank], begin[rank + 1]))
        # the SIMT router computes each token's logits the same way at any batch size, so
        # the sharded and the single-handle runs route identically
        h.set_router_tc(False)
        res = {}
        for T in (16, 128):
            x = synth.make_x(T, wl.spec.d, 6)
            shards = ep.token_shards(T, world)
            p = ep.PeerExpertParallelMoe(h, wl.spec.d, wl.spec.E, wl.spec.k, world, rank,
                                         max_tokens=shards[1] - shards[0], device=dev, row_f16=False)
            o = p.forward(torch.from_numpy(x[shards[rank]:shards[rank + 1]]).to(dev))
            outs = [torch.empty((shards[r + 1] - shards[r], wl.spec.d), device=dev) for r in range(world)]
            dist.all_gather(outs, o)
            res[T] = (torch.cat(outs).cpu().numpy(), p.status())
            p.close()
        if rank == 0:
            q.put(("ok", res))
        dist.barrier()
        h.close()
        dist.destroy_process_group()
    except Exception as e:
        import traceback

        q.put(("err", f"rank {rank}: {e}\n{traceback.format_exc()}"))


def test_ep_peer_two_gpus_f32_rows():
    import torch
    import torch.multiprocessing as mp

    nc.require_gpu()
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_f32_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    msg = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert msg[0] == "ok", msg[1]
    wl = synth.CONFIGS["c3"]
    layer = synth.make_layer(wl.spec, 1, device_gen=True)
    L = synth.open_layer(layer)
    try:
        L.set_router_tc(False)
        L.set_decode_fused(False)  # the separate-kernel arithmetic the exchange path runs
        for T, (got, st) in msg[1].items():
            assert st == 0
            single = L.forward(synth.make_x(T, wl.spec.d, 6))
            assert rel_err(got, single) <= 1e-4, T  # f32 rows and partials
    finally:
        L.close()


def test_ep_peer_two_gpus():
    """Rows and partial outputs cross by peer stores; the result matches the all-to-all path's."""
    import torch
    import torch.multiprocessing as mp

    nc.require_gpu()
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    msg = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert msg[0] == "ok", msg[1]
    ref, o1, o2, o3, st, sent, recv = msg[1]
    assert st == 0
    # same partial rows added in the same order as the all-to-all path; the
    # expert products see the rows at other positions of their tiles
    assert rel_err(o1, ref) <= 1e-3
    assert np.array_equal(o1, o2)
    assert sent[0] == 0 and recv[0] == 0 and 0 < sent[1] <= 512 and 0 < recv[1] <= 512
    wl = synth.CONFIGS["c5"]
    layer = synth.make_layer(wl.spec, 0, device_gen=True)
    x = synth.make_x(1024, wl.spec.d, 4)
    L = synth.open_layer(layer)
    try:
        L.set_gemm_min_tokens(1)
        single = L.forward(x)
    finally:
        L.close()
    assert rel_err(o1, single) <= 5e-3
    assert rel_err(o3, single) <= 5e-3


def test_peer_connect_refuses_a_different_window_layout():
    """Two ranks' windows opened on one GPU (no kernel runs): connect compares the
    layouts in the blobs before it maps anything, so a rank that opened larger slabs
    is refused on both sides; with equal layouts the shared GPU is refused."""
    import ctypes

    nc.require_gpu()
    spec = synth.LayerSpec(512, 16, 4, 256, 256, Q.DTYPE_Q4_K)
    layer = synth.make_layer(spec, 41)
    begin = ep.expert_ranges(spec.E, 2)
    lib = nc.lib()
    hs = [synth.open_layer(layer, expert_range=(begin[r], begin[r + 1])) for r in range(2)]
    tab = (nc.c_int32 * 3)(*begin)
    try:
        for slabs, want in (((16, 32), "different exchange window layout"), ((16, 16), "one GPU per rank")):
            blobs = []
            for r in range(2):
                ipc = (ctypes.c_char * ep.IPC_BYTES)()
                assert lib.aero_cuda_ep_peer_open(hs[r].handle, 2, r, tab, slabs[r], ep.ROWS_F32, ipc) == 0, \
                    nc.last_error(hs[r].handle)
                blobs.append(bytes(ipc))
            allb = b"".join(blobs)
            for r in range(2):
                assert lib.aero_cuda_ep_peer_connect(hs[r].handle, allb) == -1
                assert want in nc.last_error(hs[r].handle), (slabs, nc.last_error(hs[r].handle))
                assert lib.aero_cuda_ep_peer_close(hs[r].handle) == 0
    finally:
        for h in hs:
            h.close()


def _peer_skip_worker(rank, world, port, q):
    """Rank 1 leaves one step out (between steps, nothing of its own in flight): rank 0's
    wait for its rows gives up after the handle's 50 ms limit with code 21, its later
    waits of that step return at once, every later call is refused with the code, and both
    ranks still close their windows."""
    try:
        import datetime

        import torch
        import torch.distributed as dist

        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        spec = synth.LayerSpec(512, 16, 4, 256, 256, Q.DTYPE_Q4_K)
        layer = synth.make_layer(spec, 42)
        begin = ep.expert_ranges(spec.E, world)
        dev = f"cuda:{rank}"
        h = synth.open_layer(layer, device=rank, expert_range=(begin[rank], begin[rank + 1]))
        h.set_peer_wait_ms(50)
        p = ep.PeerExpertParallelMoe(h, spec.d, spec.E, spec.k, world, rank, max_tokens=8, device=dev, row_f16=False)
        x = torch.from_numpy(synth.make_x(8, spec.d, 42 + rank)).to(dev)
        p.forward(x)
        torch.cuda.synchronize()
        st1 = p.status()
        dist.barrier()
        refused = None
        if rank == 0:
            import time
            t0 = time.time()
            p.forward(x)  # rank 1 does not step: this rank's waits give up
            torch.cuda.synchronize()
            waited = time.time() - t0
            st2 = p.status()
            st_layer = h.status()
            try:
                p.forward(x)
            except RuntimeError as e:
                refused = str(e)
            try:
                p.forward(x)
            except RuntimeError as e:
                refused = (refused, str(e))
        else:
            waited, st2, st_layer = 0.0, p.status(), h.status()
        dist.barrier()
        p.close()
        res = (st1, st2, st_layer, refused, waited)
        outs = [None] * world
        dist.all_gather_object(outs, res)
        if rank == 0:
            q.put(("ok", outs))
        h.close()
        dist.destroy_process_group()
    except Exception as e:
        import traceback

        q.put(("err", f"rank {rank}: {e}\n{traceback.format_exc()}"))


def test_ep_peer_wait_gives_up_when_a_rank_skips_a_step():
    import torch
    import torch.multiprocessing as mp

    nc.require_gpu()
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_skip_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    msg = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert msg[0] == "ok", msg[1]
    (a1, a2, a_layer, a_refused, a_wait), (b1, b2, b_layer, _, _) = msg[1]
    assert a1 == 0 and b1 == 0
    assert a2 == 21 and a_layer == 21  # rows wait (kEpErrRowsWait)
    assert isinstance(a_refused, tuple) and all("code 21" in m for m in a_refused), a_refused
    assert a_wait < 5.0  # the 50 ms limit, not the 5 s default
    assert b2 == 0 and b_layer == 0
