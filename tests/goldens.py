"""Loaders for the golden fixtures and the synthetic inputs they name.

The fixtures store the reference's outputs plus the (seed, stream) of every
input; this module regenerates those inputs with ``nurostream_b200.synth``.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

from nurostream_b200 import synth
from nurostream_b200.ggml import GGMLType, row_bytes

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name: str):
    return np.load(GOLDEN / f"{name}.npz")


def cases(npz) -> dict:
    out = {}
    for key in npz.files:
        if key.endswith("__meta"):
            name = key[: -len("__meta")]
            out[name] = json.loads(bytes(npz[key]).decode())
    return out


def gemv_inputs(meta: dict):
    t = GGMLType(meta["type"])
    n, K, T = meta["n_rows"], meta["K"], meta["T"]
    raw = synth.quant_bytes(t, meta["seed"], meta["w_stream"], 0, n * row_bytes(t, K))
    x = synth.float_values(meta["seed"], meta["x_stream"], 0, T * K).reshape(T, K)
    return raw, x


class SynthLayer:
    """Host copy of one synthetic MoE layer, as written by make_golden.layer_tensors."""

    def __init__(self, c: dict, layer: int = 0):
        self.c = c
        self.t = GGMLType(c["type"])
        self.E, self.H, self.F, self.k, self.T = c["E"], c["H"], c["F"], c["k"], c["T"]
        seed = c["seed"]
        s = synth.LayerStreams(layer)
        self.s = s
        self.seed = seed
        E, H, F = self.E, self.H, self.F
        self.x = synth.float_values(seed, s.x, 0, self.T * H).reshape(self.T, H)
        self.router_w = synth.float_values(seed, s.router_w, 0, E * H, 0.02).reshape(E, H)
        gptoss = c["arch"] == "gpt-oss"
        self.gptoss = gptoss
        if gptoss:
            bias = c["bias"]
            z = lambda n: np.zeros(n, np.float32)
            self.router_b = synth.float_values(seed, s.router_b, 0, E, 0.02) if bias else z(E)
            self.biases = {
                "gate": (synth.float_values(seed, s.gate_b, 0, E * F, 0.02) if bias else z(E * F)).reshape(E, F),
                "up": (synth.float_values(seed, s.up_b, 0, E * F, 0.02) if bias else z(E * F)).reshape(E, F),
                "down": (synth.float_values(seed, s.down_b, 0, E * H, 0.02) if bias else z(E * H)).reshape(E, H),
            }
            self.norm_w = (np.ones(H, np.float32) if c["norm"] == "ones"
                           else synth.float_values(seed, s.norm_w, 0, H, 0.1))
        else:
            self.router_b = None
            self.biases = None
            self.norm_w = None
        self.rb_in = row_bytes(self.t, H)     # gate/up rows span H
        self.rb_ff = row_bytes(self.t, F)     # down rows span F

    def stream_of(self, kind):
        return {"gate": self.s.gate, "up": self.s.up, "down": self.s.down}[kind]

    def expert_bytes(self, kind: str, e: int) -> np.ndarray:
        rows, rb = (self.F, self.rb_in) if kind in ("gate", "up") else (self.H, self.rb_ff)
        return synth.quant_bytes(self.t, self.seed, self.stream_of(kind), e * rows * rb, rows * rb)

    def tensor_bytes(self, kind: str) -> np.ndarray:
        rows, rb = (self.F, self.rb_in) if kind in ("gate", "up") else (self.H, self.rb_ff)
        return synth.quant_bytes(self.t, self.seed, self.stream_of(kind), 0, self.E * rows * rb)

    def rows_fn(self):
        from oracle import quant

        cache = {}

        def rows(kind, e):
            key = (kind, e)
            if key not in cache:
                out, K = (self.F, self.H) if kind in ("gate", "up") else (self.H, self.F)
                cache[key] = quant.dequantize(self.expert_bytes(kind, e), self.t, out * K).reshape(out, K)
            return cache[key]

        return rows
