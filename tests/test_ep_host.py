"""Expert-parallel host protocol over gloo on CPU (world sizes 2 and 3).

Each rank runs aero_b200.ep.ExpertParallelMoe with the CPU stand-in ops over
its token shard; the gathered outputs must equal the oracle's single-process
block over all tokens. Covers uneven expert ranges (8 experts over 3 ranks),
uneven and empty token shards, f32 and f16 rows, and the split bookkeeping.
"""

import os
import socket
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer():
    from aero_b200 import quant as Q
    from aero_b200 import synth

    spec = synth.LayerSpec(256, 8, 3, 256, 256, Q.DTYPE_Q4_K)
    return synth.make_layer(spec, 7)


def _worker(rank, world, port, shards, row_f16, q):
    try:
        sys.path.insert(0, HERE)
        sys.path.insert(0, os.path.dirname(HERE))
        import torch
        import torch.distributed as dist

        from aero_b200 import ep
        from aero_b200 import synth
        from ep_cpu_ops import CpuEpOps

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        layer = _layer()
        begin = ep.expert_ranges(layer.spec.E, world)
        ops = CpuEpOps(layer, begin[rank], begin[rank + 1])
        T_all = shards[-1]
        x = synth.make_x(T_all, layer.spec.d, 3)
        mine = torch.from_numpy(x[shards[rank]:shards[rank + 1]].copy())
        m = ep.ExpertParallelMoe(ops, layer.spec.d, layer.spec.E, layer.spec.k, world, rank,
                                 max_tokens=max(shards[r + 1] - shards[r] for r in range(world)), device="cpu",
                                 row_f16=row_f16, guard=False)
        out = m.forward(mine)
        send, recv = m.last_split
        assert send[rank] == 0 and recv[rank] == 0
        # what each rank sends is what the others receive
        allsend = [None] * world
        dist.all_gather_object(allsend, send)
        for r in range(world):
            assert allsend[r][rank] == recv[r]
        outs = [None] * world
        dist.all_gather_object(outs, out.numpy())
        if rank == 0:
            q.put(("ok", np.concatenate(outs, 0)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        import traceback

        q.put(("err", f"rank {rank}: {e}\n{traceback.format_exc()}"))


def _run(world, shards, row_f16):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, shards, row_f16, q)) for r in range(world)]
    for p in procs:
        p.start()
    msg = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert msg[0] == "ok", msg[1]
    return msg[1]


def _reference(shards, row_f16):
    import oracle as O
    from aero_b200 import synth

    layer = _layer()
    x = synth.make_x(shards[-1], layer.spec.d, 3)
    lg = O.router_logits(x, layer.router, layer.router_bias)
    # f16 rows: the experts see f16-rounded inputs, the router the f32 ones
    xe = x.astype(np.float16).astype(np.float32) if row_f16 else x
    return O.moe_block(layer, xe, lg)


@pytest.mark.parametrize("world,shards,row_f16", [
    (2, [0, 19, 37], False),
    (2, [0, 0, 12], True),     # rank 0 has no tokens this step
    (3, [0, 9, 20, 26], False),  # 8 experts over 3 ranks: 3, 3, 2
])
def test_ep_protocol_matches_single_process(world, shards, row_f16):
    got = _run(world, shards, row_f16)
    want = _reference(shards, row_f16)
    scale = float(np.sqrt(np.mean(want.astype(np.float64) ** 2)))
    assert scale > 1e-4
    # f16 rows: the partial outputs also cross back as f16 (one more rounding of
    # ~5e-4 relative per element), so the prefill bar applies
    tol = 1e-2 if row_f16 else 1e-4
    assert float(np.max(np.abs(got - want))) <= tol * scale


def test_expert_ranges_and_shards():
    from aero_b200 import ep

    assert ep.expert_ranges(512, 8) == [64 * i for i in range(9)]
    assert ep.expert_ranges(8, 3) == [0, 3, 6, 8]
    assert ep.token_shards(10, 4) == [0, 3, 6, 8, 10]
    with pytest.raises(ValueError):
        ep.expert_ranges(4, 5)


class _FakePeerLib:
    """The aero_cuda_ep_peer_* calls of the C ABI, failing where told (host logic only).
    Like the library, each blob carries the window layout (here the slab rows) and
    connect refuses a blob set whose layouts differ."""

    def __init__(self, rank, fail_open=(), fail_connect=()):
        self.rank, self.fail_open, self.fail_connect = rank, fail_open, fail_connect
        self.calls = []
        self.why = "refused by the fake"

    def aero_cuda_ep_peer_open(self, h, world, rank, tab, slab, row_dtype, ipc):
        self.calls.append("open")
        if rank in self.fail_open:
            return -1
        ipc[:8] = bytes([rank + 1] * 8)
        ipc[8:12] = int(slab).to_bytes(4, "little")
        return 0

    def aero_cuda_ep_peer_connect(self, h, blobs):
        self.calls.append("connect")
        self.blobs = blobs
        ipc = len(blobs) // self.world if hasattr(self, "world") else 128
        slabs = {bytes(blobs[r * ipc + 8:r * ipc + 12]) for r in range(len(blobs) // ipc)}
        if len(slabs) > 1:
            self.why = "a different exchange window layout"
            return -1
        return -1 if self.rank in self.fail_connect else 0

    def aero_cuda_ep_peer_close(self, h):
        self.calls.append("close")
        return 0

    def last_error(self, h):
        return self.why


def _peer_setup_worker(rank, world, port, case, q):
    try:
        sys.path.insert(0, os.path.dirname(HERE))
        import torch.distributed as dist

        from aero_b200 import ep

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)

        class Layer:
            handle = 1

            def set_stream(self, s):
                raise AssertionError("no stream on the CPU")

        lib = _FakePeerLib(rank, fail_open=case.get("fail_open", ()), fail_connect=case.get("fail_connect", ()))
        lib.world = world
        max_tokens = case.get("max_tokens", {}).get(rank, 16)
        try:
            m = ep.PeerExpertParallelMoe(Layer(), 256, 8, 2, world, rank, max_tokens=max_tokens, device="cpu", lib=lib)
        except RuntimeError as e:
            res = ("raised", str(e), lib.calls)
        else:
            ipc = ep.IPC_BYTES
            got = [lib.blobs[r * ipc] for r in range(world)]
            m.close()
            res = ("ok", got, lib.calls)
        outs = [None] * world
        dist.all_gather_object(outs, res)
        if rank == 0:
            q.put(("ok", outs))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        import traceback

        q.put(("err", f"rank {rank}: {e}\n{traceback.format_exc()}"))


@pytest.mark.parametrize("case", [{}, {"fail_open": (1,)}, {"fail_connect": (0,)}, {"max_tokens": {2: 32}}])
def test_peer_exchange_setup_is_collective(case):
    """Every rank gets every rank's window blob in rank order; when one rank
    cannot open or map, all ranks raise together (and release what they opened)."""
    import torch.multiprocessing as mp

    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_setup_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    msg = q.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert msg[0] == "ok", msg[1]
    outs = msg[1]
    if not case:
        for kind, got, calls in outs:
            assert kind == "ok"
            assert got == [r + 1 for r in range(world)]
            assert calls == ["open", "connect", "close"]
    else:
        for r, (kind, why, calls) in enumerate(outs):
            assert kind == "raised" and "peer exchange unavailable" in why
            assert calls[-1] == "close"
        if "fail_open" in case:
            assert all("connect" not in c for _, _, c in outs)
            assert "refused by the fake" in outs[1][1]
        if "max_tokens" in case:  # every rank sees the mismatch and raises with the reason
            assert all("different exchange window layout" in why for _, why, _ in outs)
