"""Expert-parallel MoE layer: one process per GPU, NCCL all-to-all between them.

The reference runs a layer in one process (engine/moe.py:117-177,
src/moe.cpp:122-161); this is the sharded form of the same computation.
Rank r holds experts [begin[r], begin[r+1]) of the layer (begin from
`expert_ranges`), the full router and the shared expert, and owns T_r of the
step's tokens. A step on each rank:

1. `aero_cuda_ep_dispatch` routes the local tokens over all experts and writes
   the self rows (every local token, straight into the head of the receive
   buffer) and, for every rank, a slab of `max_tokens` send rows: one row per
   (token, that rank owning one of its experts), tokens in order, each with a
   metadata row (expert ids owned by the destination, weights, shared gate),
   then padding rows whose metadata names no expert;
2. the slabs and their metadata cross with `all_to_all_single` in equal splits,
   so no host synchronisation is needed; received slabs land after the self
   rows;
3. `aero_cuda_ep_expert_block` runs this rank's experts over all R rows (the
   self rows also take the shared expert) and writes one f32 row per row;
4. rows [T_r, R) of that output go back with the reverse `all_to_all_single`,
   arriving in the send slabs' layout;
5. `aero_cuda_ep_combine` adds, per token, the self part and then the remote
   parts in rank order.

Every rank takes the same collective steps in the same order, also for T_r = 0.
The device work and the collectives are ordered on one stream; the host never
waits inside a step.
"""

from __future__ import annotations

import ctypes
from typing import List

ROWS_F32 = 0
ROWS_F16 = 1
IPC_BYTES = 128  # AERO_EP_IPC_BYTES


def expert_ranges(n_expert: int, world: int) -> List[int]:
    """begin[0..world]: rank r holds experts [begin[r], begin[r+1]) (E/world each,
    the first E % world ranks one more)."""
    if world < 1 or world > n_expert:
        raise ValueError(f"world size {world} must be in [1, n_expert={n_expert}]")
    base, extra = divmod(n_expert, world)
    begin = [0]
    for r in range(world):
        begin.append(begin[-1] + base + (1 if r < extra else 0))
    return begin


def token_shards(T: int, world: int) -> List[int]:
    """Token offsets[0..world] of a T-token batch split over the ranks."""
    base, extra = divmod(T, world)
    off = [0]
    for r in range(world):
        off.append(off[-1] + base + (1 if r < extra else 0))
    return off


class CudaEpOps:
    """The device side of a step, through the library's C ABI (device pointers)."""

    def __init__(self, layer) -> None:
        from . import native_cuda as nc

        self.nc = nc
        self.lib = nc.lib()
        self.layer = layer
        self.h = layer.handle
        self.meta_ld = int(self.lib.aero_cuda_ep_meta_ld(self.h))

    def _check(self, rc: int, what: str) -> None:
        if rc != 0:
            raise RuntimeError(f"{what}: {self.nc.last_error(self.h)}")

    def set_stream(self, stream) -> None:
        self.layer.set_stream(stream)

    def dispatch(self, x, T, world, rank, begin, row_dtype, self_rows, self_meta, send_rows, send_meta, counts, pos):
        tab = (self.nc.c_int32 * len(begin))(*begin)
        rc = self.lib.aero_cuda_ep_dispatch(self.h, x.data_ptr(), T, world, rank, tab, row_dtype, self_rows.data_ptr(),
                                            self_meta.data_ptr(), send_rows.data_ptr(), send_meta.data_ptr(),
                                            send_rows.shape[0] // world, counts.data_ptr(), pos.data_ptr())
        self._check(rc, "aero_cuda_ep_dispatch")

    def expert_block(self, rows, row_dtype, meta, R, n_shared, out):
        out_dtype = ROWS_F16 if out.element_size() == 2 else ROWS_F32
        rc = self.lib.aero_cuda_ep_expert_block(self.h, rows.data_ptr(), row_dtype, meta.data_ptr(), R, n_shared,
                                                out.data_ptr(), out_dtype)
        self._check(rc, "aero_cuda_ep_expert_block")

    def combine(self, self_out, back, pos, T, world, rank, out):
        parts = ROWS_F16 if back.element_size() == 2 else ROWS_F32
        rc = self.lib.aero_cuda_ep_combine(self.h, self_out.data_ptr(), back.data_ptr(), parts, pos.data_ptr(), T,
                                           world, rank, out.data_ptr())
        self._check(rc, "aero_cuda_ep_combine")


class ExpertParallelMoe:
    """One rank's share of an expert-parallel MoE layer.

    `ops` does the device work (CudaEpOps for a CudaMoeLayer opened with this
    rank's expert range); `forward(x)` takes this rank's tokens (T_r, n_embd)
    f32 on `device` and returns their layer output. `max_tokens` bounds T_r on
    every rank (it sizes the exchange buffers once). With `row_f16` the rows
    cross as f16 (the GEMM path's operand type; halves the bytes), and so do the
    partial outputs coming back; otherwise both are f32.
    `exchange(out, inp, out_splits, in_splits)` replaces
    torch.distributed.all_to_all_single over `group` (None splits: equal).
    """

    def __init__(self, ops, n_embd: int, n_expert: int, k: int, world: int, rank: int, max_tokens: int,
                 device="cuda", group=None, row_f16: bool = True, guard: bool = True, exchange=None) -> None:
        import torch
        import torch.distributed as dist

        self.torch, self.dist = torch, dist
        self.ops, self.d, self.E, self.k = ops, n_embd, n_expert, k
        self.world, self.rank, self.group = world, rank, group
        self.exchange = exchange
        self.begin = expert_ranges(n_expert, world)
        self.row_dtype = ROWS_F16 if row_f16 else ROWS_F32
        self.device = torch.device(device)
        rdt = torch.float16 if row_f16 else torch.float32
        ml = ops.meta_ld
        self.max_tokens = int(max_tokens)
        # one slab of max_tokens rows per rank (a rank sends a token at most once)
        self.slab = max(1, self.max_tokens)
        send_cap = world * self.slab
        recv_cap = self.max_tokens + world * self.slab  # self rows + a slab from every rank
        dev = self.device
        self.send_rows = torch.empty((send_cap, n_embd), dtype=rdt, device=dev)
        self.send_meta = torch.empty((send_cap, ml), dtype=torch.int32, device=dev)
        self.recv_rows = torch.empty((recv_cap, n_embd), dtype=rdt, device=dev)
        self.recv_meta = torch.empty((recv_cap, ml), dtype=torch.int32, device=dev)
        # partial outputs cross back in the rows' type (f16 for prefill: the GEMM's
        # per-expert results are f16 already)
        self.y = torch.empty((recv_cap, n_embd), dtype=rdt, device=dev)
        self.back = torch.empty((send_cap, n_embd), dtype=rdt, device=dev)
        self.counts = torch.zeros(world + 1, dtype=torch.int32, device=dev)
        self.recv_counts = torch.zeros(world, dtype=torch.int32, device=dev)
        self.pos = torch.empty((max(1, self.max_tokens), world), dtype=torch.int32, device=dev)
        self._reserved = 0
        self.stream = None
        if self.device.type == "cuda":
            # the library's kernels and the collectives run on one side stream,
            # ordered after the caller's stream at entry and before it at exit
            # (a handle given the legacy default stream would use its own)
            self.stream = torch.cuda.Stream(device=self.device)
            ops.set_stream(self.stream)
        if guard and self.device.type == "cuda":
            # the exchange buffers are torch allocations; charge them to the
            # library's memory guard so its accounting covers them
            from . import native_cuda as nc

            nbytes = sum(t.numel() * t.element_size() for t in (self.send_rows, self.send_meta, self.recv_rows,
                                                                 self.recv_meta, self.y, self.back, self.pos))
            g = nc.MemoryGuard()
            if not g.try_reserve(nbytes, nc.MEM_SCRATCH):
                raise RuntimeError(f"expert-parallel exchange buffers ({nbytes} bytes) refused by the memory guard")
            self._guard, self._reserved = g, nbytes
        # per-phase device times (set_profiling): dispatch, counts (exchange), rows
        # (row + metadata exchange), experts, back (return exchange), combine
        self.PHASES = ("dispatch", "counts", "rows", "experts", "back", "combine")
        self._prof = None
        self.phase_ms = {k: 0.0 for k in self.PHASES}
        self.phase_n = 0

    def set_profiling(self, on: bool) -> None:
        """Time the step's phases with CUDA events on the layer's stream (synchronises each step)."""
        torch = self.torch
        self._prof = [torch.cuda.Event(enable_timing=True) for _ in range(len(self.PHASES) + 1)] if on else None
        self.phase_ms = {k: 0.0 for k in self.PHASES}
        self.phase_n = 0

    def _mark(self, i: int) -> None:
        if self._prof is not None:
            self._prof[i].record(self.stream)

    def close(self) -> None:
        if self._reserved:
            from . import native_cuda as nc

            self._guard.release(self._reserved, nc.MEM_SCRATCH)
            self._reserved = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _a2a(self, out, inp, out_splits, in_splits) -> None:
        if self.exchange is not None:
            self.exchange(out, inp, out_splits, in_splits)
        else:
            self.dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def forward(self, x):
        torch = self.torch
        T = int(x.shape[0])
        if x.dim() != 2 or x.shape[1] != self.d:
            raise ValueError(f"hidden width {tuple(x.shape)} != n_embd {self.d}")
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens on rank {self.rank} > max_tokens {self.max_tokens}")
        x = x.contiguous().float()
        out = torch.empty((T, self.d), dtype=torch.float32, device=self.device)
        if self.stream is None:
            self._step(x, out)
            return out
        caller = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(caller)
        with torch.cuda.stream(self.stream):
            self._step(x, out)
        caller.wait_stream(self.stream)
        x.record_stream(self.stream)
        out.record_stream(self.stream)
        return out

    @property
    def last_split(self):
        """(rows sent to each rank, rows received from each rank) in the last step
        (reads the device counters: synchronises)."""
        both = self.torch.cat([self.counts[:self.world], self.recv_counts]).cpu().tolist()
        return [int(v) for v in both[:self.world]], [int(v) for v in both[self.world:]]

    def _step(self, x, out):
        T = int(x.shape[0])
        n, r, C = self.world, self.rank, self.slab
        R = T + n * C
        self._mark(0)
        self.ops.dispatch(x, T, n, r, self.begin, self.row_dtype, self.recv_rows, self.recv_meta, self.send_rows,
                          self.send_meta, self.counts, self.pos)
        self._mark(1)
        self._a2a(self.recv_counts, self.counts[:n], None, None)  # for last_split only; stays on the device
        self._mark(2)
        self._a2a(self.recv_rows[T:R], self.send_rows, None, None)
        self._a2a(self.recv_meta[T:R], self.send_meta, None, None)
        self._mark(3)
        self.ops.expert_block(self.recv_rows, self.row_dtype, self.recv_meta, R, T, self.y)
        self._mark(4)
        self._a2a(self.back, self.y[T:R], None, None)
        self._mark(5)
        self.ops.combine(self.y, self.back, self.pos, T, n, r, out)
        self._mark(6)
        if self._prof is not None:
            self._prof[6].synchronize()
            for i, k in enumerate(self.PHASES):
                self.phase_ms[k] += self._prof[i].elapsed_time(self._prof[i + 1])
            self.phase_n += 1

    __call__ = forward


class PeerExpertParallelMoe:
    """One rank's share of an expert-parallel MoE layer, exchanging over peer memory.

    Same step as ExpertParallelMoe (same partial sums, added in the same rank
    order), with no collective library inside it: every rank's exchange window
    is mapped into the other ranks' processes (CUDA IPC), the dispatch kernel
    stores the rows straight into their owners' windows, the owners' return
    kernel stores the partial outputs straight back, and the kernels wait for
    the peers' step flags (aero_cuda_ep_peer_* in the C ABI). One GPU per rank.
    Construction and `close` are collective over `group` (all-gather of the
    window handles, barriers); every rank must run the same number of steps.
    When any rank cannot open or map the windows, every rank raises
    RuntimeError("peer exchange unavailable: ...") (callers fall back together).
    `gather(bytes) -> list of bytes in rank order` replaces the all-gather;
    `lib` replaces the library (an object with the aero_cuda_ep_peer_* calls and
    last_error(handle)).
    """

    PHASES = ("route", "plan", "pack", "rows_wait", "experts", "return", "combine")

    def __init__(self, layer, n_embd: int, n_expert: int, k: int, world: int, rank: int, max_tokens: int,
                 device="cuda", group=None, row_f16: bool = True, gather=None, lib=None) -> None:
        import torch
        import torch.distributed as dist

        from . import native_cuda as nc

        self.torch, self.dist, self.nc = torch, dist, nc
        self.lib = lib if lib is not None else nc.lib()
        self._last_error = (lambda: lib.last_error(self.h)) if lib is not None else (lambda: nc.last_error(self.h))
        self.layer, self.h = layer, layer.handle
        self.d, self.E, self.k = n_embd, n_expert, k
        self.world, self.rank, self.group = world, rank, group
        self.begin = expert_ranges(n_expert, world)
        self.row_dtype = ROWS_F16 if row_f16 else ROWS_F32
        self.device = torch.device(device)
        self.max_tokens = max(1, int(max_tokens))
        self.cuda = self.device.type == "cuda"
        self.stream = torch.cuda.Stream(device=self.device) if self.cuda else None
        if self.cuda:
            layer.set_stream(self.stream)
        tab = (nc.c_int32 * len(self.begin))(*self.begin)
        ipc = (ctypes.c_char * IPC_BYTES)()
        rc = self.lib.aero_cuda_ep_peer_open(self.h, world, rank, tab, self.max_tokens, self.row_dtype, ipc)
        self.opened = rc == 0
        err = "" if self.opened else self._last_error()
        blobs = (gather or self._gather)(bytes(ipc) if self.opened else b"")
        if not all(len(b) == IPC_BYTES for b in blobs):
            self.close(barrier=False)
            raise RuntimeError(f"peer exchange unavailable: rank {rank}: {err or 'another rank failed to open'}")
        allh = b"".join(blobs)
        rc = self.lib.aero_cuda_ep_peer_connect(self.h, allh)
        ok = self._all_ok(rc == 0)
        if not ok:
            why = self._last_error() if rc != 0 else "another rank failed to connect"
            self.close(barrier=False)
            raise RuntimeError(f"peer exchange unavailable: rank {rank}: {why}")
        if self.cuda:
            torch.cuda.synchronize(self.device)
        if dist.is_initialized():
            dist.barrier(group=group)
        self.phase_ms = {k: 0.0 for k in self.PHASES}
        self.phase_n = 0

    def _gather(self, blob: bytes):
        dist, torch = self.dist, self.torch
        if self.world == 1:
            return [blob]
        t = torch.zeros(IPC_BYTES + 1, dtype=torch.uint8, device=self.device)
        if blob:
            t[:IPC_BYTES] = torch.frombuffer(bytearray(blob), dtype=torch.uint8)
            t[IPC_BYTES] = 1
        out = torch.empty(self.world * (IPC_BYTES + 1), dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(out, t, group=self.group)
        rows = out.view(self.world, IPC_BYTES + 1).cpu()
        return [bytes(r[:IPC_BYTES].numpy().tobytes()) if int(r[IPC_BYTES]) else b"" for r in rows]

    def _all_ok(self, ok: bool) -> bool:
        dist, torch = self.dist, self.torch
        if not dist.is_initialized() or self.world == 1:
            return ok
        f = torch.tensor([1 if ok else 0], dtype=torch.int32, device=self.device)
        dist.all_reduce(f, op=dist.ReduceOp.MIN, group=self.group)
        return bool(int(f.item()))

    def forward(self, x):
        torch = self.torch
        T = int(x.shape[0])
        if x.dim() != 2 or x.shape[1] != self.d:
            raise ValueError(f"hidden width {tuple(x.shape)} != n_embd {self.d}")
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens on rank {self.rank} > max_tokens {self.max_tokens}")
        x = x.contiguous().float()
        out = torch.empty((T, self.d), dtype=torch.float32, device=self.device)
        caller = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(caller)
        rc = self.lib.aero_cuda_ep_peer_step(self.h, x.data_ptr() if T else None, T, out.data_ptr() if T else None)
        if rc != 0:
            raise RuntimeError(f"aero_cuda_ep_peer_step: {self.nc.last_error(self.h)}")
        caller.wait_stream(self.stream)
        x.record_stream(self.stream)
        out.record_stream(self.stream)
        return out

    __call__ = forward

    def status(self) -> int:
        """0, or the code of the first wait that gave up (synchronises)."""
        return int(self.lib.aero_cuda_ep_peer_status(self.h))

    @property
    def last_split(self):
        """(rows sent to each rank, rows received from each rank) in the last step (synchronises)."""
        sent = (self.nc.c_int32 * self.world)()
        recv = (self.nc.c_int32 * self.world)()
        if self.lib.aero_cuda_ep_peer_counts(self.h, sent, recv) != 0:
            raise RuntimeError(self.nc.last_error(self.h))
        return list(sent), list(recv)

    def set_profiling(self, on: bool) -> None:
        """Time the step's phases (synchronises each step); read them with `read_phases`."""
        self.lib.aero_cuda_ep_peer_profile(self.h, 1 if on else 0, None)

    def read_phases(self):
        """Mean device ms per phase since the last read."""
        ms = (ctypes.c_double * len(self.PHASES))()
        n = self.lib.aero_cuda_ep_peer_profile(self.h, 1, ms)
        return {k: float(v) for k, v in zip(self.PHASES, ms)}, int(n)

    def close(self, barrier: bool = True) -> None:
        """Collective: waits for this rank's work, then for every rank, then frees the window."""
        if self.h is None:
            return
        if self.cuda:
            self.torch.cuda.synchronize(self.device)
        if barrier and self.dist.is_initialized() and self.world > 1:
            self.dist.barrier(group=self.group)
        self.lib.aero_cuda_ep_peer_close(self.h)
        self.h = None


def open_rank_layer(layer_src, world: int, rank: int, device: int = 0):
    """Open rank `rank`'s share of a synthetic layer (aero_b200.synth.SynthLayer)."""
    from . import synth

    begin = expert_ranges(layer_src.spec.E, world)
    return synth.open_layer(layer_src, device=device, expert_range=(begin[rank], begin[rank + 1]))
