"""Host twin of the synthetic GPT-OSS model that ``nurostream_b200.gptoss.GptOssDecoder`` builds in HBM.

``model_tensors`` names every tensor of the model as the reference's GGUF loader would, with a
producer of its bytes that reproduces the device generator bit for bit (``nurostream_b200.synth``
with the decoder's seeds, streams and float arithmetic).  ``tests/golden/make_golden.py`` feeds
it to the reference's own ``GptOssModel``; the GPU tests feed it to the oracle.
"""
from __future__ import annotations

import numpy as np

from nurostream_b200 import synth
from nurostream_b200.ggml import GGMLType, row_bytes
from nurostream_b200.shapes import GptOssShape


def _f32_producer(values_fn):
    cache = {}

    def prod(start, n):
        if "v" not in cache:
            cache["v"] = values_fn().astype(np.float32).view(np.uint8)
        return cache["v"][start:start + n]
    return prod


def _bf16_producer(seed, stream, sigma):
    def prod(start, n):
        assert start % 2 == 0 and n % 2 == 0
        return synth.float_values(seed, stream, start // 2, n // 2, sigma, dtype="bf16").astype(np.uint16).view(np.uint8)
    return prod


def _quant_producer(t, seed, stream):
    return lambda start, n: synth.quant_bytes(t, seed, stream, start, n)


def model_tensors(shape: GptOssShape, seed: int = 0, bias_sigma: float = 0.02) -> dict:
    """name -> (torch_shape, GGMLType, producer(start_byte, nbytes) -> uint8 array)."""
    H, V, qd, kvd = shape.n_embd, shape.vocab_size, shape.q_dim, shape.kv_dim
    E, F = shape.n_expert, shape.n_ffn_expert
    ms = synth.ModelStreams
    one = np.float32(1.0)
    T = {
        "token_embd.weight": ((V, H), GGMLType.BF16, _bf16_producer(seed, ms.token_embd, 1.0)),
        "output_norm.weight": ((H,), GGMLType.F32,
                               _f32_producer(lambda: synth.float_values(seed, ms.output_norm, 0, H, 0.1) + one)),
        "output.weight": ((V, H), GGMLType.BF16, _bf16_producer(seed, ms.output, 0.02)),
    }
    for l in range(shape.n_layer):
        s = synth.LayerStreams(l)
        p = f"blk.{l}."
        T[p + "attn_norm.weight"] = ((H,), GGMLType.F32,
                                     _f32_producer(lambda s=s: synth.float_values(seed, s.attn_norm, 0, H, 0.1) + one))
        for nm, rows, cols, ws, bs in (("attn_q", qd, H, s.q_w, s.q_b), ("attn_k", kvd, H, s.k_w, s.k_b),
                                       ("attn_v", kvd, H, s.v_w, s.v_b), ("attn_output", H, qd, s.o_w, s.o_b)):
            T[p + nm + ".weight"] = ((rows, cols), GGMLType.BF16, _bf16_producer(seed, ws, 0.02))
            T[p + nm + ".bias"] = ((rows,), GGMLType.F32,
                                   _f32_producer(lambda bs=bs, rows=rows: synth.float_values(seed, bs, 0, rows, 0.02)))
        T[p + "attn_sinks.weight"] = ((shape.n_head,), GGMLType.F32,
                                      _f32_producer(lambda s=s: synth.float_values(seed, s.sinks, 0, shape.n_head, 1.0)))
        T[p + "post_attention_norm.weight"] = ((H,), GGMLType.F32,
                                               _f32_producer(lambda s=s: synth.float_values(seed, s.norm_w, 0, H, 0.1) + one))
        T[p + "ffn_gate_inp.weight"] = ((E, H), GGMLType.BF16, _bf16_producer(seed, s.router_w, 0.02))
        T[p + "ffn_gate_inp.bias"] = ((E,), GGMLType.F32,
                                      _f32_producer(lambda s=s: synth.float_values(seed, s.router_b, 0, E, 0.02)))
        for kind, rows, cols, ws, bs in (("gate", F, H, s.gate, s.gate_b), ("up", F, H, s.up, s.up_b),
                                         ("down", H, F, s.down, s.down_b)):
            T[p + f"ffn_{kind}_exps.weight"] = ((E, rows, cols), GGMLType.MXFP4, _quant_producer(GGMLType.MXFP4, seed, ws))
            T[p + f"ffn_{kind}_exps.bias"] = ((E, rows), GGMLType.F32, _f32_producer(
                lambda bs=bs, rows=rows: synth.float_values(seed, bs, 0, E * rows, bias_sigma)))
    return T


def kv_history(shape: GptOssShape, seed: int, ctx: int) -> dict:
    """layer -> [k, v] (n_kv, ctx, head_dim) fp32: the synthetic history the decoder's caches start with."""
    out = {}
    n = shape.n_head_kv * ctx * shape.head_dim
    for l in range(shape.n_layer):
        s = synth.LayerStreams(l)
        k = synth.float_values(seed, s.k_cache, 0, n, 1.0).reshape(shape.n_head_kv, ctx, shape.head_dim)
        v = synth.float_values(seed, s.v_cache, 0, n, 1.0).reshape(shape.n_head_kv, ctx, shape.head_dim)
        out[l] = [k, v]
    return out


class TwinWeights:
    """``oracle.model`` weight accessor over ``model_tensors`` (fp32 values, dequantized experts)."""

    def __init__(self, shape: GptOssShape, seed: int = 0):
        from oracle import quant
        self.shape, self.seed = shape, seed
        self.T = model_tensors(shape, seed)
        self._w = {}
        self._rows = {}
        self._quant = quant

    def w(self, name):
        if name not in self._w:
            shp, t, prod = self.T[name]
            n = int(np.prod(shp))
            if t == GGMLType.BF16:
                raw = prod(0, 2 * n).view(np.uint16)
                self._w[name] = synth.bf16_to_f32(raw).reshape(shp)
            else:
                self._w[name] = prod(0, 4 * n).view(np.float32).reshape(shp)
        return self._w[name]

    def rows(self, layer):
        sh = self.shape
        H, F = sh.n_embd, sh.n_ffn_expert

        def rows(kind, e):
            key = (layer, kind, e)
            if key not in self._rows:
                out, K = (F, H) if kind in ("gate", "up") else (H, F)
                rb = row_bytes(GGMLType.MXFP4, K)
                _, _, prod = self.T[f"blk.{layer}.ffn_{kind}_exps.weight"]
                raw = prod(e * out * rb, out * rb)
                self._rows[key] = self._quant.dequantize(raw, GGMLType.MXFP4, out * K).reshape(out, K)
            return self._rows[key]
        return rows

    def biases(self, layer):
        return {kind: self.w(f"blk.{layer}.ffn_{kind}_exps.bias") for kind in ("gate", "up", "down")}

    def config(self) -> dict:
        return self.shape.reference_config()
