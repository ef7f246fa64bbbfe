#!/usr/bin/env python3
"""Benchmark of the B200 MoE FFN layer (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c5] [--impl ours|reference]
    python bench.py --profile --workload c5 [--tokens T] [--calls C] [--gemm-min N]

Metric: MoE-layer tokens/s. The default workload is config 5
(512 experts top-10 + shared expert, Q4_K, 8192-token prefill): the metric is
quoted at 1/2/4/8 GPUs and config 5 is the configuration defined at those
counts. A step is one layer call over the workload's tokens (config 1: 64
one-token calls). Inputs are synthetic (seeded N(0,1) activations, N(0,0.02)
weights quantised to GGUF blocks); no datasets or checkpoints exist here.
With N > 1 (torchrun, one process per GPU) the layer runs expert parallel:
E/N experts and T/N tokens per rank; the rows and partial outputs cross by
stores into the peers' exchange windows (CUDA IPC over NVLink, no collective
library in the step; --exchange nccl uses NCCL all-to-all instead,
aero_b200.ep); the step's token count stays T (strong scaling).

  value        tokens/s over K steps, inputs already in HBM, device time by
               CUDA events on the layer's stream (max over ranks)
  roofline     prefill: the larger grouped GEMM (tensor-bound: algorithmic
               FLOPs / its CUDA-event time vs the measured burst bf16 peak,
               the step being ~1 ms); decode: the whole layer call (HBM-bound:
               GGUF bytes of the experts it streams + router + activations)
  traffic      ncu DRAM read + write bytes per launch of that kernel (TRAFFIC
               below, from the capture its comment names)
  e2e          the same through the public API with host buffers: every
               step's pinned host input -> device, layer, device -> pinned
               host output; one GPU: the asynchronous calls
               (aero_cuda_moe_submit / _wait, three slots in turn, so calls'
               copies in both directions overlap another call's block), host wall clock from the
               first submit to the last wait; N GPUs: the exchange's forward
               with the copies on the layer's stream, CUDA events
  decode       at N = 1, the decode configurations (c1, c4 batch 1 and 16,
               c3) timed the same way, with their HBM bytes and fraction
  cpu_baseline the reference's own MoE block (oracle/_ref, built from its
               sources) on the host cores, over a bounded token sample
The working set (weights >= 340 MB) exceeds the 126 MB L2, so no flush runs
between steps.

--impl reference times the reference's own CPU block (oracle/_ref) on rank 0
with all host threads, on the same workload and config, with weights from the
host generator (no GPU and none of this package's native code on that arm).
--profile runs a few layer calls with device-resident inputs and prints the
per-stage device times: the command the profile summaries are captured from.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        d["source"] = "measured"
        return d
    return dict(PEAKS_FALLBACK)


class Clocks:
    """nvidia-smi sampling (every 200 ms), started once before any timed work so
    that the sampler's start-up never lands in a timed region; summary(t0, t1)
    reads the samples of a window around one."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []  # (host time, csv line)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.proc = None

    def summary(self, t0: float, t1: float, pad: float = 0.3):
        """Samples from pad seconds before t0 to pad seconds after t1 (regions
        shorter than the sampling period get the samples that bracket them)."""
        if self.proc:
            time.sleep(max(0.0, t1 + pad - time.time()))
        sm, mx, reasons = [], 0.0, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ts, ln in list(self.lines):
            if ts < t0 - pad or ts > t1 + pad:
                continue
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = max(mx, float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return ws, rank, local


def layer_bytes(spec):
    from aero_b200.quant import type_size
    per_expert = 3 * type_size(spec.dtype, spec.F * spec.d)
    shared = 3 * type_size(spec.dtype, spec.Fs * spec.d) if spec.Fs else 0
    return per_expert, shared


# DRAM read + write bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum)
# of the dominant kernel of a workload, keyed (workload, kernel). Each entry
# names the capture it comes from; a kernel changed since its capture has no
# entry (traffic: null) until it is captured again.
TRAFFIC = {
    # profiles/traffic_c5_8192tok.md (ncu launch list of bench.py --profile --workload c5 --tokens 8192)
    ("c5_prefill_q4_k_shared", "grouped_gemm_gate_up"): (1052660224, "profiles/traffic_c5_8192tok.md"),
    ("c5_prefill_q4_k_shared", "grouped_gemm_down"): (707158528, "profiles/traffic_c5_8192tok.md"),
    # profiles/decode_kernel_c1.md, profiles/decode_kernel_c3.md (one call of the fused decode kernel)
    ("c1_decode_q8_0", "decode_layer"): (41298176, "profiles/decode_kernel_c1.md"),
    ("c3_decode_q4_k_shared", "decode_layer"): (539513856, "profiles/decode_kernel_c3.md"),
}


def traffic_record(workload: str, kernel: str):
    rec = TRAFFIC.get((workload, kernel))
    return None if rec is None else rec[0]


def config_dict(wl, ws: int) -> dict:
    """The workload's config record, identical on both arms."""
    spec = wl.spec
    return {"workload": wl.name, "tokens_per_step": wl.T * wl.calls, "tokens_per_call": wl.T, "experts": spec.E,
            "top_k": spec.k, "d": spec.d, "ffn": spec.F, "shared_ffn": spec.Fs,
            "quant": "Q8_0" if spec.dtype == 8 else "Q4_K",
            "routing": f"zipf{wl.zipf_s}" if wl.zipf_s else "uniform",
            "parallelism": f"ep{ws}" if ws > 1 else "single",
            "l2": "no flush: expert weights exceed the 126 MB L2"}


def decode_bytes(spec, x, router, bias, T: int, calls: int) -> int:
    """Algorithmic HBM bytes of `calls` layer calls of T tokens: GGUF bytes of the
    distinct experts each call selects (top-k of x @ router^T + bias, computed
    here on the host), the shared expert, the f32 router (+ shared gate row)
    and the activations in and out."""
    per_expert, shared = layer_bytes(spec)
    lg = x @ router.T + (bias if bias is not None else 0)
    total = 0
    for c in range(calls):
        sel = np.argpartition(-lg[c * T:(c + 1) * T], spec.k - 1, axis=1)[:, :spec.k]
        total += len(np.unique(sel)) * per_expert + shared
        total += (spec.E + (1 if spec.Fs else 0)) * spec.d * 4 + 2 * T * spec.d * 4
    return int(total)


def cpu_reference(wl, layer, x, logits, budget_s: float, threads: int):
    """Time the reference's own block (or the C restatement when the reference
    objects are absent) on a bounded token sample. Returns (tokens/s, kind, sample, threads)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    kind = "reference" if O.ref_available() else "port"
    fn = O.ref_block if kind == "reference" else O.moe_block
    if kind == "reference" and layer.shexp and layer.shexp["ffn_len"] != wl.spec.F:
        kind, fn = "port", O.moe_block
    n = min(max(threads, 1), x.shape[0])
    t0 = time.perf_counter()
    fn(layer, x[:n], logits[:n], nthreads=threads)
    dt = time.perf_counter() - t0
    # grow the sample towards the time budget
    while dt < budget_s / 4 and n < x.shape[0]:
        n = min(x.shape[0], n * 4)
        t0 = time.perf_counter()
        fn(layer, x[:n], logits[:n], nthreads=threads)
        dt = time.perf_counter() - t0
    return n / dt, kind, n, dt


def gemm_roofline(spec, stats, stage_avg, pk, per_mat, shared):
    """Roofline of the larger grouped GEMM of a prefill call (gate/up or down). Its bound is the
    larger of the tensor time (algorithmic FLOPs, 2 * rows * n per weight row, at the measured
    burst bf16 peak: the GEMM runs inside a ~1 ms step, and f16 operands run at the bf16 rate)
    and the HBM time (GGUF bytes of the expert matrices it streams, at the measured copy
    bandwidth); the other is reported beside it."""
    pairs, srows = stats["last_pairs"], stats["last_shared_rows"]
    active = stats["last_active"]
    dom = max(("gate_up", "down"), key=lambda k: stage_avg[k])
    mult = 2 if dom == "gate_up" else 1
    flops = 2.0 * mult * spec.d * (spec.F * pairs + spec.Fs * srows)
    nbytes = active * mult * per_mat + (mult * shared // 3 if shared else 0)
    t_s = stage_avg[dom] / 1000.0
    peak_tc = pk["bf16_tflops"]
    tc = {"bound": "tensor", "achieved": flops / t_s / 1e12, "peak": peak_tc, "unit": "TFLOP/s",
          "peak_source": f"{pk['source']} bf16 burst (f16 operands run at the same rate)"}
    if "bf16_tflops_sustained" in pk:
        tc["frac_of_sustained"] = tc["achieved"] / pk["bf16_tflops_sustained"]
    hbm = {"bound": "hbm", "achieved": nbytes / t_s / 1e9, "peak": pk["hbm_gbs"], "unit": "GB/s",
           "peak_source": f"{pk['source']} HBM copy"}
    for r in (tc, hbm):
        r["frac"] = r["achieved"] / r["peak"]
    tensor_bound = flops / (peak_tc * 1e12) >= nbytes / (pk["hbm_gbs"] * 1e9)
    main, other = (tc, hbm) if tensor_bound else (hbm, tc)
    roof = {"kernel": f"grouped_gemm_{dom}", **main, "traffic": None, "algorithmic_flops": flops,
            "algorithmic_bytes": int(nbytes), "other_bound": other, "avg_ms": stage_avg[dom], "pairs": pairs,
            "shared_rows": srows, "active_experts": active}
    return roof


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="c5")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the decode sub-record")
    ap.add_argument("--no-decoder", action="store_true", help="skip the config-4 decoder sub-record")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="expert parallel (N > 1): rows cross by peer-memory stores (default) or NCCL all-to-all")
    ap.add_argument("--profile", action="store_true",
                    help="run --calls layer calls of --tokens tokens and print the per-stage device times")
    ap.add_argument("--tokens", type=int, default=0, help="--profile: tokens per call (default: the workload's)")
    ap.add_argument("--calls", type=int, default=3, help="--profile: layer calls")
    ap.add_argument("--gemm-min", type=int, default=0, help="--profile: GEMM path threshold (0: library default)")
    ap.add_argument("--decoder-layers", type=int, default=0,
                    help="--profile --workload decoder: layers of the config-4 decoder (0: all 48)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    ws, rank, local = dist_env()
    from aero_b200 import synth

    if args.profile and args.workload == "decoder":
        run_profile_decoder(args)
        return
    wl = synth.CONFIGS[args.workload]
    if args.impl == "reference":
        if rank == 0:
            run_reference(args, ws, wl)
        return
    if args.profile:
        run_profile(args, wl)
        return

    import torch
    from aero_b200 import native_cuda as nc

    nc.lib()
    nc.require_gpu()
    torch.cuda.set_device(local)
    if ws > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    dev = local
    cuda = f"cuda:{dev}"
    clk = Clocks(dev).start()  # runs until the end, so its start-up is outside every timed region
    try:
        run_ours(args, ws, rank, dev, cuda, wl, wl.spec, wl.T, 0, clk)
    finally:
        clk.stop()


def run_reference(args, ws, wl):
    """The reference's own CPU block (oracle/_ref) on this host's cores, on the
    workload's config, each step a bounded token sample; weights come from the
    host generator, so nothing on this arm uses the GPU or this package's
    native library."""
    from aero_b200 import synth
    spec, T = wl.spec, wl.T
    x = synth.make_x(T * wl.calls, spec.d, 0, bf16=wl.bf16_x)
    layer = synth.make_layer(spec, 0, host_parallel=True)
    if wl.zipf_s:
        synth.attach_zipf(layer, x, wl.zipf_s, 0)
    lg = (x @ layer.router.T + (layer.router_bias if layer.router_bias is not None else 0)).astype(np.float32)
    threads = os.cpu_count() or 1
    per_step = max(1.0, 120.0 / (args.steps + args.warmup))
    times = []
    kind = "reference"
    for i in range(args.warmup + args.steps):
        _, kind, n, dt = cpu_reference(wl, layer, x, lg, per_step, threads)
        if i >= args.warmup:
            times.append((n, dt))
    n_tot = sum(n for n, _ in times)
    t_tot = sum(dt for _, dt in times)
    v = n_tot / t_tot
    tokens_per_step = T * wl.calls
    print(json.dumps({
        "impl": "reference", "metric": "moe_layer_tokens_per_s", "value": v, "unit": "tokens/s",
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * tokens_per_step / v,
        "ms_per_step_note": f"a full {tokens_per_step}-token step at the measured rate; each timed step ran a "
                            f"{times[-1][0]}-token sample",
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(wl, ws),
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": kind,
                         "sample": f"{times[-1][0]} tokens of {tokens_per_step} per step"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_profile(args, wl):
    """A few layer calls with device-resident inputs; prints the per-stage
    device times of the last one (the command profile captures run)."""
    import torch
    from aero_b200 import native_cuda as nc
    from aero_b200 import synth

    nc.require_gpu()
    T = args.tokens or wl.T
    layer = synth.make_layer(wl.spec, 0, device_gen=True)
    x_host = synth.make_x(T, wl.spec.d, 0, bf16=wl.bf16_x)
    if wl.zipf_s:
        synth.attach_zipf(layer, x_host, wl.zipf_s, 0)
    L = synth.open_layer(layer)
    if args.gemm_min:
        L.set_gemm_min_tokens(args.gemm_min)
    x = torch.from_numpy(x_host).cuda()
    out = torch.empty_like(x)
    lib = nc.lib()
    for i in range(args.calls):
        if i == args.calls - 1:
            L.set_profiling(True)
        if lib.aero_cuda_moe_forward(L.handle, 0, x.data_ptr(), T, wl.spec.d, out.data_ptr()) != 1:
            raise RuntimeError(nc.last_error(L.handle))
    torch.cuda.synchronize()
    st = L.stage_times()
    L.close()
    print(json.dumps({"workload": wl.name, "tokens": T, "stages_ms": {k: v[0] / max(v[1], 1) for k, v in st.items()},
                      "checksum": float(np.abs(out.cpu().numpy()).sum())}))


def run_profile_decoder(args):
    """The config-4 decoder (--decoder-layers of its 48 layers) with a 4096-position
    cache: --calls eager decode steps of --tokens sequences (default 1), then the
    phase times of one more (the command the decoder profile captures run)."""
    import dataclasses

    import torch
    from aero_b200 import synth
    from aero_b200.decoder import CudaDecoder

    os.environ["AERO_DECODER_GRAPHS"] = "0"  # every kernel its own launch in the capture
    spec = synth.DECODER_C4
    if args.decoder_layers:
        spec = dataclasses.replace(spec, n_layer=args.decoder_layers)
    B = args.tokens or 1
    n_kv = 4096
    D = CudaDecoder.from_synth(synth.make_decoder(spec, 0, device_gen=True), n_seq=B, n_ctx=n_kv + args.calls + 2)
    shape = (B, spec.n_kv, D.n_ctx, spec.head_dim)
    for li in range(spec.n_layer):
        for ptr in D.kv(li):
            t = torch.as_tensor(_CudaArray(ptr, shape, "<f2"), device="cuda")
            t[:, :, :n_kv].normal_()
    logits = torch.empty((B, spec.vocab), device="cuda")
    rng = np.random.default_rng(3)
    for i in range(args.calls):
        D.step(rng.integers(0, spec.vocab, B), np.arange(B), np.full(B, n_kv + i), logits=logits)
    D.profile(True)
    D.step(rng.integers(0, spec.vocab, B), np.arange(B), np.full(B, n_kv + args.calls), logits=logits)
    torch.cuda.synchronize()
    ph = D.profile(False)
    D.close()
    print(json.dumps({"workload": f"decoder_{spec.n_layer}l", "batch": B, "phases_ms": ph,
                      "checksum": float(logits.abs().sum().item())}))


class _CudaArray:
    """A device buffer (address, shape, numpy type string) for torch.as_tensor."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape), "typestr": typestr, "version": 3}


def run_ours(args, ws, rank, dev, cuda, wl, spec, T, seed, clk):
    import torch
    from aero_b200 import synth
    from aero_b200 import native_cuda as nc

    x_host = synth.make_x(T * wl.calls, spec.d, seed, bf16=wl.bf16_x)
    layer = synth.make_layer(spec, seed, device_gen=True)
    if wl.zipf_s:
        synth.attach_zipf(layer, x_host, wl.zipf_s, seed)
    stream = torch.cuda.Stream(device=dev)
    lib = nc.lib()
    ep_mode = ws > 1
    if ep_mode:
        # expert parallel: experts E/n per rank, tokens T/n per rank, NCCL
        # all-to-all for the rows (ranks = processes, one GPU each)
        from aero_b200 import ep
        if wl.calls != 1:
            raise SystemExit(f"{wl.name}: expert parallel applies to batched workloads (one call per step)")
        begin = ep.expert_ranges(spec.E, ws)
        shards = ep.token_shards(T, ws)
        L = synth.open_layer(layer, device=dev, expert_range=(begin[rank], begin[rank + 1]))
        row_f16 = T >= 64  # prefill: rows cross in the GEMM operand type
        max_tok = max(shards[r + 1] - shards[r] for r in range(ws))
        moe = None
        exchange = args.exchange
        if exchange == "peer":
            try:
                moe = ep.PeerExpertParallelMoe(L, spec.d, spec.E, spec.k, ws, rank, max_tokens=max_tok, device=cuda,
                                               row_f16=row_f16)
            except RuntimeError as e:  # collective: every rank falls back together
                if rank == 0:
                    print(f"# {e}; using the NCCL all-to-all exchange", file=sys.stderr, flush=True)
                exchange = "nccl"
        if moe is None:
            with torch.cuda.stream(stream):
                moe = ep.ExpertParallelMoe(ep.CudaEpOps(L), spec.d, spec.E, spec.k, ws, rank, max_tokens=max_tok,
                                           device=cuda, row_f16=row_f16)
        x_mine = x_host[shards[rank]:shards[rank + 1]]
    else:
        L = synth.open_layer(layer, device=dev)
        L.set_stream(stream)
        x_mine = x_host
    x_dev = torch.from_numpy(x_mine).to(cuda)
    out_dev = torch.empty_like(x_dev)
    Tm = x_mine.shape[0] // wl.calls  # tokens per call on this rank

    def step_device():
        if ep_mode:
            out_dev.copy_(moe.forward(x_dev))
            return
        for c in range(wl.calls):
            xs = x_dev[c * Tm:(c + 1) * Tm]
            os_ = out_dev[c * Tm:(c + 1) * Tm]
            if lib.aero_cuda_moe_forward(L.handle, 0, xs.data_ptr(), Tm, spec.d, os_.data_ptr()) != 1:
                raise RuntimeError(nc.last_error(L.handle))

    def max_over_ranks(v):
        if ws == 1:
            return v
        t = torch.tensor([v], device=cuda)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    # ---- value: device-resident inputs
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step_device()
    stream.synchronize()
    launches0 = L.stats()["launches"]
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        ev0.record(stream)
        t_start = time.time()
        for _ in range(args.steps):
            step_device()
        ev1.record(stream)
        ev1.synchronize()
        t_end = time.time()
    torch.cuda.synchronize()
    clocks = clk.summary(t_start, t_end)
    launches = L.stats()["launches"] - launches0
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    if ws > 1:
        torch.distributed.barrier()
    tokens_per_step = T * wl.calls
    value = tokens_per_step * args.steps / (ms / 1000.0)

    # ---- e2e: host buffers through the public API every step
    n_slots = 3  # asynchronous slots in turn: one input in, one block, one output out at a time
    xh = [torch.from_numpy(x_mine).pin_memory() for _ in range(n_slots)]
    oh = [torch.empty_like(xh[0]).pin_memory() for _ in range(n_slots)]

    if ep_mode:
        def step_host():
            xd = xh[0].to(cuda, non_blocking=True)
            oh[0].copy_(moe.forward(xd), non_blocking=True)

        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                step_host()
        stream.synchronize()
        torch.distributed.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(args.steps):
                step_host()
            e1.record(stream)
            e1.synchronize()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1))
        e2e_mode = "exchange forward, copies on the layer's stream, CUDA events"
    else:
        n_sub = [0]

        def submit(c):
            """The step's call c into the next slot, after that slot's previous call has landed."""
            slot = n_sub[0] % n_slots
            if lib.aero_cuda_moe_submit(L.handle, slot, xh[slot][c * Tm:(c + 1) * Tm].data_ptr(), Tm,
                                        oh[slot][c * Tm:(c + 1) * Tm].data_ptr()) != 0:
                raise RuntimeError(nc.last_error(L.handle))
            n_sub[0] += 1

        def drain():
            for slot in range(n_slots):
                if lib.aero_cuda_moe_wait(L.handle, slot) != 0:
                    raise RuntimeError(nc.last_error(L.handle))

        for _ in range(args.warmup):
            for c in range(wl.calls):
                submit(c)
        drain()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            for c in range(wl.calls):
                submit(c)
        drain()
        e2e_ms = (time.perf_counter() - t0) * 1000.0
        e2e_mode = "asynchronous calls (aero_cuda_moe_submit / _wait, three slots in turn), host wall clock"
    e2e_value = tokens_per_step * args.steps / (e2e_ms / 1000.0)

    # ---- per-stage device times (a separate profiled pass)
    L.set_profiling(True)
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.steps // 2)):
            step_device()
    stream.synchronize()
    st = L.stage_times()
    stats = L.stats()
    L.set_profiling(False)
    stage_avg = {k: (v[0] / v[1] if v[1] else 0.0) for k, v in st.items()}
    pk = peaks()
    per_expert, shared = layer_bytes(spec)
    per_mat = per_expert // 3
    active = stats["last_active"]
    if stats.get("last_gemm"):
        roof = gemm_roofline(spec, stats, stage_avg, pk, per_mat, shared)
        dtype = "f16"
    else:
        # decode: the whole layer call streams the selected experts' blocks once
        alg = decode_bytes(spec, x_mine, layer.router, layer.router_bias, Tm, wl.calls)
        achieved = alg / (ms / args.steps / 1000.0) / 1e9
        roof = {"kernel": "decode_layer", "bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / pk["hbm_gbs"], "traffic": None, "peak_source": f"{pk['source']} HBM copy",
                "algorithmic_bytes": alg, "avg_ms": ms / args.steps}
        dtype = "f32"
    tr = traffic_record(wl.name, roof["kernel"])
    if tr is not None:
        roof["traffic"] = tr
    result = {
        "metric": "moe_layer_tokens_per_s",
        "value": value,
        "unit": "tokens/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": dtype,
        "data": "synthetic",
        "config": config_dict(wl, ws),
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": int(x_host.nbytes),
                "d2h_bytes_per_step": int(x_host.nbytes), "ms_per_step": e2e_ms / args.steps, "mode": e2e_mode},
        "gpu_launches": int(launches),
        "clocks": clocks,
        "roofline": roof,
        "stages_ms": {k: round(v, 5) for k, v in stage_avg.items()},
    }
    if ep_mode:
        result["exchange"] = "peer memory (CUDA IPC, NVLink stores)" if exchange == "peer" else "NCCL all-to-all"
        result["exchange_rows"] = {"sent": moe.last_split[0], "received": moe.last_split[1]}
        # per-phase device times of rank 0's step (a separate profiled pass, the
        # ranks lined up first: a phase that waits for peers also times their lag)
        torch.distributed.barrier()
        moe.set_profiling(True)
        with torch.cuda.stream(stream):
            for _ in range(3):
                step_device()
        stream.synchronize()
        if exchange == "peer":
            ph, _ = moe.read_phases()
            result["ep_phases_ms"] = {k: round(v, 5) for k, v in ph.items()}
            result["exchange_status"] = moe.status()
        else:
            result["ep_phases_ms"] = {k: round(v / max(moe.phase_n, 1), 5) for k, v in moe.phase_ms.items()}
        moe.set_profiling(False)
    if ws == 1 and not args.no_decode and wl.name == synth.CONFIGS["c5"].name:
        result["zipf"] = zipf_record(args, dev, stream)
    if ws == 1 and not args.no_decode and not wl.name.startswith(("c1", "c3", "c4")):
        result["decode"] = decode_records(args, dev, stream, pk)
    if ws == 1 and not args.no_decoder and not wl.name.startswith(("c1", "c3", "c4")):
        result["decoder"] = decoder_records(args, dev, stream, pk)
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        lg = x_host @ layer.router.T + (layer.router_bias if layer.router_bias is not None else 0)
        threads = os.cpu_count() or 1
        tps, kind, n, dt = cpu_reference(wl, layer, x_host, lg.astype(np.float32), args.cpu_seconds, threads)
        # the reference block itself is single-threaded (tokens shard over processes / threads)
        tps1, _, n1, dt1 = cpu_reference(wl, layer, x_host, lg.astype(np.float32), args.cpu_seconds / 5, 1)
        result["cpu_baseline"] = {"value": tps, "unit": "tokens/s", "cores": threads, "kind": kind,
                                  "sample": f"{n} of {T * wl.calls} tokens, {dt:.1f} s",
                                  "single_thread": {"value": tps1, "sample": f"{n1} tokens, {dt1:.1f} s"}}
    if rank == 0:
        print(json.dumps(result), flush=True)
    if ep_mode:
        moe.close()
    L.close()
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def zipf_record(args, dev, stream) -> dict:
    """Config 5 with Zipf(s = 1.2)-skewed routing (workload c5z) at N = 1, timed like
    the headline line (device-resident inputs, CUDA events over `args.steps` steps),
    with the calibration of its router bias: tau, the measured top-expert share and
    load-curve slope, and the Zipf head share against top-k's 1 / k cap."""
    import torch
    from aero_b200 import native_cuda as nc
    from aero_b200 import synth

    lib = nc.lib()
    wl = synth.CONFIGS["c5z"]
    spec, T = wl.spec, wl.T
    x_host = synth.make_x(T, spec.d, 0, bf16=wl.bf16_x)
    layer = synth.make_layer(spec, 0, device_gen=True)
    synth.attach_zipf(layer, x_host, wl.zipf_s, 0)
    L = synth.open_layer(layer, device=dev)
    L.set_stream(stream)
    x = torch.from_numpy(x_host).to(f"cuda:{dev}")
    o = torch.empty_like(x)

    def step():
        if lib.aero_cuda_moe_forward(L.handle, 0, x.data_ptr(), T, spec.d, o.data_ptr()) != 1:
            raise RuntimeError(nc.last_error(L.handle))

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    L.close()
    m = layer.meta
    return {"workload": wl.name, "tokens_per_step": T, "ms_per_step": ms, "tokens_per_s": T / (ms / 1000.0),
            "routing": {k: m[k] for k in ("zipf_s", "zipf_tau", "top_load_share", "zipf_top_share", "top_share_cap",
                                          "load_slope", "max_load", "min_load")}}


def decode_records(args, dev, stream, pk) -> dict:
    """The decode configurations at N = 1: one step = the workload's calls with
    device-resident inputs, timed by CUDA events over `args.steps` steps; HBM
    bytes as in decode_bytes, fraction of the measured copy bandwidth."""
    import torch
    from aero_b200 import native_cuda as nc
    from aero_b200 import synth

    lib = nc.lib()
    out = {}
    for key in ("c1", "c4b1", "c4b16", "c3"):
        wl = synth.CONFIGS[key]
        spec, T = wl.spec, wl.T
        x_host = synth.make_x(T * wl.calls, spec.d, 0, bf16=wl.bf16_x)
        layer = synth.make_layer(spec, 0, device_gen=True)
        L = synth.open_layer(layer, device=dev)
        L.set_stream(stream)
        x = torch.from_numpy(x_host).to(f"cuda:{dev}")
        o = torch.empty_like(x)

        def step():
            for c in range(wl.calls):
                if lib.aero_cuda_moe_forward(L.handle, 0, x[c * T:].data_ptr(), T, spec.d, o[c * T:].data_ptr()) != 1:
                    raise RuntimeError(nc.last_error(L.handle))

        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                step()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                step()
            e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        nbytes = decode_bytes(spec, x_host, layer.router, layer.router_bias, T, wl.calls)
        gbs = nbytes / (ms / 1000.0) / 1e9
        out[key] = {"workload": wl.name, "tokens_per_call": T, "calls_per_step": wl.calls, "ms_per_step": ms,
                    "us_per_call": 1000.0 * ms / wl.calls, "tokens_per_s": T * wl.calls / (ms / 1000.0),
                    "hbm_bytes_per_step": nbytes, "achieved_gbs": gbs, "frac_of_hbm": gbs / pk["hbm_gbs"],
                    "traffic_per_call": traffic_record(wl.name, "decode_layer")}
        L.close()
        del x, o
    return out


def decoder_step_bytes(spec, B: int, kv_len: int, experts_per_layer: float) -> int:
    """Algorithmic HBM bytes of one decoder step over B sequences whose caches hold
    kv_len positions: every layer's q/k/v/o projections and f32 router once, the
    distinct experts the step routes to (gate, up, down), each sequence's K and V
    rows read (and the new ones written), the embedding rows and the head once."""
    from aero_b200 import synth
    H, HK, D, d = spec.n_head, spec.n_kv, spec.head_dim, spec.d
    m = spec.moe
    q8 = lambda n: n // 32 * 34  # noqa: E731
    attn = q8((H * D + 2 * HK * D) * d) + q8(d * H * D)
    per_expert = layer_bytes(synth.LayerSpec(m.d, 1, 1, m.F, 0, m.dtype))[0]
    kv = B * (kv_len + 1) * HK * D * 2 * 2
    layer = attn + int(round(experts_per_layer * per_expert)) + m.E * m.d * 4 + kv
    head = q8(spec.vocab * d) if not spec.tied else 0
    return spec.n_layer * layer + head + B * q8(d)


def decoder_records(args, dev, stream, pk) -> dict:
    """Config 4: the 48-layer decoder (GQA 32/4 x 128, RoPE 1e6, the Q4_K 128-expert
    MoE in every layer, vocab 151936 Q8_0), decode steps at batch 1 and 16 over a
    4096-position f16 cache per sequence (filled with N(0, 1) values: a synthetic
    stand-in for a prefilled cache, the step's cost does not depend on them), random
    token ids. One step = one token per sequence through the whole model and the head;
    timed by CUDA events on the decoder's stream over `args.steps` steps."""
    import torch
    from aero_b200 import synth
    from aero_b200.decoder import CudaDecoder

    spec = synth.DECODER_C4
    n_kv = 4096
    n_ctx = n_kv + 2 * (args.warmup + args.steps) + 2
    t0 = time.time()
    dec_s = synth.make_decoder(spec, 0, device_gen=True)
    D = CudaDecoder.from_synth(dec_s, n_seq=16, n_ctx=n_ctx, device=dev)
    del dec_s
    build_s = time.time() - t0

    g = torch.Generator(device=f"cuda:{dev}")
    g.manual_seed(4)
    shape = (16, spec.n_kv, n_ctx, spec.head_dim)
    for li in range(spec.n_layer):
        for ptr in D.kv(li):
            t = torch.as_tensor(_CudaArray(ptr, shape, "<f2"), device=f"cuda:{dev}")
            t[:, :, :n_kv].normal_(generator=g)
    torch.cuda.synchronize(dev)
    D.set_stream(stream)
    rng = np.random.default_rng(3)
    out = {"config": "c4_decoder_48l_gqa32x4_q4k128e_top8_vocab151936", "kv_positions": n_kv,
           "build_s": round(build_s, 1), "data": "synthetic weights and cache, random token ids"}
    try:
        for B in (1, 16):
            pos = n_kv  # every batch size decodes after the same 4096 cached positions
            logits = torch.empty((B, spec.vocab), device=f"cuda:{dev}")
            seqs = np.arange(B)

            def step(p):
                D.step(rng.integers(0, spec.vocab, B), seqs, np.full(B, p), logits=logits)

            # distinct experts per layer: read once from the MoE layers' profiled call
            for m in D._keep:
                m.set_profiling(True)
            step(pos)
            pos += 1
            stream.synchronize()
            active = [m.stats()["last_active"] for m in D._keep]
            for m in D._keep:
                m.set_profiling(False)
            for _ in range(args.warmup):
                step(pos)
                pos += 1
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            p0 = pos
            e0.record(stream)
            for _ in range(args.steps):
                step(pos)
                pos += 1
            e1.record(stream)
            e1.synchronize()
            ms = e0.elapsed_time(e1) / args.steps
            D.profile(True)
            step(pos)
            pos += 1
            stream.synchronize()
            phases = D.profile(False)
            ex = float(np.mean(active))
            nbytes = decoder_step_bytes(spec, B, (p0 + pos) // 2, ex)
            gbs = nbytes / (ms / 1000.0) / 1e9
            out[f"batch{B}"] = {"ms_per_step": round(ms, 4), "tokens_per_s": round(B / (ms / 1000.0), 1),
                                "hbm_bytes_per_step": nbytes, "achieved_gbs": round(gbs, 1),
                                "frac_of_hbm": round(gbs / pk["hbm_gbs"], 4), "experts_per_layer": round(ex, 2),
                                "phases_ms": {k: round(v, 4) for k, v in phases.items()}}
            del logits
    finally:
        D.close()
    return out


if __name__ == "__main__":
    main()
