"""Run one synthetic MoE layer a few times, for profilers (ncu) and quick timing.

    python -m aero_b200.prof --workload c5 --tokens 1024 --calls 3 [--gemm-min 64]

Builds the workload's layer on the GPU (seeded, as bench.py does), then makes
`calls` forward calls on `tokens` tokens with device-resident inputs and
prints the per-stage device times of the last calls.
"""

from __future__ import annotations

import argparse
import json

import numpy as np


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="c5")
    ap.add_argument("--tokens", type=int, default=0, help="tokens per call (default: the workload's)")
    ap.add_argument("--calls", type=int, default=3)
    ap.add_argument("--gemm-min", type=int, default=0, help="GEMM path threshold (0: library default)")
    args = ap.parse_args()

    import torch

    from . import synth
    from . import native_cuda as nc

    nc.require_gpu()
    wl = synth.CONFIGS[args.workload]
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


if __name__ == "__main__":
    main()
