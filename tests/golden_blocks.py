"""Rebuild the golden MoE blocks' layers from their recorded seeds."""

import numpy as np

from aero_b200 import synth


def block(golden, name):
    g = {k[len(name) + 1:]: v for k, v in golden.items() if k.startswith(name + "_")}
    d, E, k, F, Fs, dt, norm, T, seed = (int(v) for v in g["spec"])
    spec = synth.LayerSpec(d, E, k, F, Fs, dt, bool(norm))
    layer = synth.make_layer(spec, seed)
    if g["bias"].size:
        layer.router_bias = g["bias"]
    return layer, g
