"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container where the reference tree and gguf-py are importable:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference <reference checkout>

It calls the reference's OWN code (``neurostream.compute.quant.dequantize``,
``compute.blockffn.stream_linear``, ``model.gpt_oss.GptOssModel._ffn_block`` /
``_route`` and ``moe.router.moe_ffn``) on seeded synthetic inputs from
``nurostream_b200.synth`` and stores inputs-by-seed plus the reference outputs
in ``tests/golden/*.npz``.  Large weight tensors are not stored: tests
regenerate them from the recorded (seed, stream) with the same generator.

Dequantization is additionally cross-checked here against gguf-py's
``gguf.dequantize`` (an independent implementation of the GGML formats).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from nurostream_b200 import synth  # noqa: E402
from nurostream_b200.ggml import TYPE_LAYOUT, GGMLType, row_bytes  # noqa: E402


def _import_reference(path: str):
    sys.path.insert(0, path)
    import torch  # noqa: F401
    import neurostream  # noqa: F401
    return path


# --------------------------------------------------------------------------- sources

class SynthSource:
    """A weight source whose tensor bytes come from ``nurostream_b200.synth``.

    Presents the method names the reference's TieredCache and stream_linear
    call on a source (the ``MmapSource`` surface in
    ``neurostream/io/source.py:65-133``), decoding with the reference's own
    ``dequantize`` -- so the reference math runs unmodified on top of it.
    """

    def __init__(self, tensors: dict):
        # tensors: name -> (torch_shape, GGMLType, producer(start_byte, nbytes) -> np.uint8)
        from neurostream.format.gguf import GGMLType as RefType, TensorInfo, nbytes_for

        self._prod = {}
        infos = {}
        for name, (shape, dtype, prod) in tensors.items():
            n = int(np.prod(shape))
            rt = RefType(int(dtype))
            infos[name] = TensorInfo(name, tuple(reversed(shape)), rt, 0, nbytes_for(rt, n))
            self._prod[name] = prod
        self.gguf = SimpleNamespace(tensors=infos)

    def _raw(self, name, start, nbytes):
        import torch
        return torch.from_numpy(np.ascontiguousarray(self._prod[name](start, nbytes)))

    def raw_bytes(self, name):
        return self._raw(name, 0, self.gguf.tensors[name].nbytes)

    def fetch(self, name, device="cpu", dtype=None):
        import torch
        from neurostream.compute.quant import dequantize
        info = self.gguf.tensors[name]
        flat = dequantize(self.raw_bytes(name), info.dtype, info.n_elements,
                          out_dtype=dtype or torch.float32)
        return flat.reshape(info.torch_shape).to(device)

    def raw_rows(self, name, start, end):
        from neurostream.io.source import row_geometry
        n_rows, _, rb = row_geometry(self.gguf.tensors[name])
        start, end = max(0, start), min(n_rows, end)
        return self._raw(name, start * rb, (end - start) * rb)

    def fetch_rows(self, name, start, end, device="cpu", dtype=None):
        import torch
        from neurostream.compute.quant import dequantize
        from neurostream.io.source import row_geometry
        info = self.gguf.tensors[name]
        n_rows, elems, rb = row_geometry(info)
        start, end = max(0, start), min(n_rows, end)
        raw = self.raw_rows(name, start, end)
        flat = dequantize(raw, info.dtype, (end - start) * elems, out_dtype=dtype or torch.float32)
        return flat.reshape(end - start, elems).to(device)


def quant_producer(dtype, seed, stream):
    return lambda start, n: synth.quant_bytes(dtype, seed, stream, start, n)


def f32_producer(seed, stream, sigma, const=None):
    def prod(start, n):
        assert start % 4 == 0 and n % 4 == 0
        if const is not None:
            v = np.full(n // 4, const, dtype=np.float32)
        else:
            v = synth.float_values(seed, stream, start // 4, n // 4, sigma)
        return v.view(np.uint8)
    return prod


# --------------------------------------------------------------------------- dequant

def golden_dequant(out_path: Path):
    import gguf
    import torch
    from neurostream.compute.quant import dequantize
    from neurostream.format.gguf import GGMLType as RefType

    rng = np.random.default_rng(20261201)
    arrays = {}
    for t in (GGMLType.MXFP4, GGMLType.Q4_K, GGMLType.Q5_K, GGMLType.Q6_K, GGMLType.Q8_0, GGMLType.Q4_0):
        be, bb = TYPE_LAYOUT[t]
        nb = 256 if t == GGMLType.MXFP4 else 24
        raw = rng.integers(0, 256, (nb, bb), dtype=np.uint8)
        if t == GGMLType.MXFP4:
            raw[:, 0] = np.arange(256, dtype=np.uint8)       # every E8M0 exponent, 255 included
        else:
            # finite fp16 scales spanning normals and subnormals, both signs
            lo = {GGMLType.Q6_K: 208}.get(t, 0)
            fields = [lo] + ([2] if t in (GGMLType.Q4_K, GGMLType.Q5_K) else [])
            for f in fields:
                mag = rng.uniform(-18, 4, nb)
                val = (np.sign(rng.uniform(-1, 1, nb)) * 2.0 ** mag).astype(np.float16)
                val[:3] = np.array([0.0, 6.0e-8, -65504.0], dtype=np.float16)
                raw[:, f:f + 2] = val.view(np.uint8).reshape(nb, 2)
        flat = raw.reshape(-1)
        ref = dequantize(torch.from_numpy(flat.copy()), RefType(int(t)), nb * be).numpy()
        g = gguf.dequantize(raw, gguf.GGMLQuantizationType(int(t))).reshape(-1).astype(np.float32)
        assert np.array_equal(ref.view(np.uint32) & 0x7FFFFFFF, g.view(np.uint32) & 0x7FFFFFFF) or \
            np.array_equal(ref, g), f"reference and gguf-py disagree on {t.name}"
        arrays[f"raw_{t.name}"] = flat
        arrays[f"out_{t.name}"] = ref.view(np.uint32)
        print(f"dequant {t.name}: {nb} blocks, matches gguf-py")
    np.savez_compressed(out_path, **arrays)


# --------------------------------------------------------------------------- gemv

GEMV_CASES = [
    # name, type, n_rows, K, T, seed, block_rows
    ("mxfp4_19x2880", GGMLType.MXFP4, 19, 2880, 1, 11, 512),
    ("q8_0_19x2880", GGMLType.Q8_0, 19, 2880, 1, 12, 512),
    ("q4_k_37x4096", GGMLType.Q4_K, 37, 4096, 1, 13, 512),
    ("q6_k_13x512", GGMLType.Q6_K, 13, 512, 1, 14, 512),
    ("mxfp4_t3_600x1024", GGMLType.MXFP4, 600, 1024, 3, 15, 512),
    ("q4_k_t2_1x256", GGMLType.Q4_K, 1, 256, 2, 16, 512),
    ("q5_k_29x1024", GGMLType.Q5_K, 29, 1024, 1, 17, 512),
    ("q4_0_21x2880", GGMLType.Q4_0, 21, 2880, 1, 18, 512),
    ("q5_k_t3_300x512", GGMLType.Q5_K, 300, 512, 3, 19, 128),
    ("q4_0_t2_70x1024", GGMLType.Q4_0, 70, 1024, 2, 20, 32),
]


def golden_gemv(out_path: Path):
    import torch
    from neurostream.compute.blockffn import stream_linear
    from neurostream.residency.cache import TieredCache

    arrays = {}
    for name, t, n, K, T, seed, br in GEMV_CASES:
        src = SynthSource({"w": ((n, K), t, quant_producer(t, seed, 1))})
        cache = TieredCache(src, ram_budget=1 << 40)
        assert cache.admit_ram("w")
        x = synth.float_values(seed, 2, 0, T * K).reshape(T, K)
        y = stream_linear(cache, "w", torch.from_numpy(x.copy()), block_rows=br).numpy()
        meta = dict(type=int(t), n_rows=n, K=K, T=T, seed=seed, w_stream=1, x_stream=2)
        arrays[f"{name}__meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
        arrays[f"{name}__y"] = y.astype(np.float32)
        print(f"gemv {name}: y[0,:3]={y[0, :3]}")
    np.savez_compressed(out_path, **arrays)


# --------------------------------------------------------------------------- MoE layers

MOE_CASES = [
    # config 1 of the benchmark: 32 experts, H=F=2880, top-4, MXFP4, zero biases, norm = ones
    dict(name="gptoss_cfg1", arch="gpt-oss", type=int(GGMLType.MXFP4), E=32, H=2880, F=2880,
         k=4, T=1, seed=0, bias=False, norm="ones", block_rows=512),
    # small GPT-OSS layer with nonzero biases and a random norm weight, 3 tokens
    dict(name="gptoss_small_bias_t3", arch="gpt-oss", type=int(GGMLType.MXFP4), E=8, H=256, F=192,
         k=2, T=3, seed=5, bias=True, norm="random", block_rows=64),
    # Qwen3-MoE layer, Q4_K experts, top-8 of 16, 2 tokens
    dict(name="qwen_q4k_t2", arch="qwen3moe", type=int(GGMLType.Q4_K), E=16, H=512, F=256,
         k=8, T=2, seed=7, bias=False, norm=None, block_rows=0),
]


def layer_tensors(c: dict, layer: int = 0) -> dict:
    """Tensor name -> (shape, type, producer) for one synthetic MoE layer."""
    t = GGMLType(c["type"])
    E, H, F, seed = c["E"], c["H"], c["F"], c["seed"]
    s = synth.LayerStreams(layer)
    p = f"blk.{layer}."
    tensors = {
        p + "ffn_gate_inp.weight": ((E, H), GGMLType.F32, f32_producer(seed, s.router_w, 0.02)),
        p + "ffn_gate_exps.weight": ((E, F, H), t, quant_producer(t, seed, s.gate)),
        p + "ffn_up_exps.weight": ((E, F, H), t, quant_producer(t, seed, s.up)),
        p + "ffn_down_exps.weight": ((E, H, F), t, quant_producer(t, seed, s.down)),
    }
    if c["arch"] == "gpt-oss":
        bias = c["bias"]
        tensors[p + "ffn_gate_inp.bias"] = ((E,), GGMLType.F32,
                                            f32_producer(seed, s.router_b, 0.02, None if bias else 0.0))
        for kind, width, stream in (("gate", F, s.gate_b), ("up", F, s.up_b), ("down", H, s.down_b)):
            tensors[p + f"ffn_{kind}_exps.bias"] = ((E, width), GGMLType.F32,
                                                     f32_producer(seed, stream, 0.02, None if bias else 0.0))
        norm_const = 1.0 if c["norm"] == "ones" else None
        tensors[p + "post_attention_norm.weight"] = ((H,), GGMLType.F32,
                                                      f32_producer(seed, s.norm_w, 0.1, norm_const))
    return tensors


def golden_moe(out_path: Path):
    import torch
    from neurostream.model.gpt_oss import GptOssConfig, GptOssModel
    from neurostream.model.qwen3 import Qwen3Config, Qwen3Model
    from neurostream.moe.router import moe_ffn
    from neurostream.residency.cache import TieredCache

    arrays = {}
    for c in MOE_CASES:
        src = SynthSource(layer_tensors(c))
        cache = TieredCache(src)
        common = dict(n_layer=1, n_embd=c["H"], n_head=1, n_head_kv=1, head_dim=c["H"],
                      n_ffn=c["F"], vocab_size=8, rms_eps=1e-5, rope_base=10000.0,
                      context_length=4096, n_expert=c["E"], n_expert_used=c["k"],
                      n_ffn_expert=c["F"])
        x = synth.float_values(c["seed"], synth.LayerStreams(0).x, 0, c["T"] * c["H"]).reshape(c["T"], c["H"])
        xt = torch.from_numpy(x.copy())
        with torch.no_grad():
            if c["arch"] == "gpt-oss":
                model = GptOssModel(cache, GptOssConfig(**common), block_rows=c["block_rows"])
                out = model._ffn_block(xt, 0).numpy()
                from neurostream.compute.ops import rms_norm
                h = rms_norm(xt, model.w("blk.0.post_attention_norm.weight"), 1e-5)
                _, ids, weights = model._route(h, 0)
            else:
                model = Qwen3Model(cache, Qwen3Config(**common), block_rows=c["block_rows"])
                out = moe_ffn(model, xt, 0).numpy()           # x is used directly as h
                from neurostream.moe.router import route
                ids, weights = route(model, xt, 0)
        meta = {k: v for k, v in c.items()}
        arrays[f"{c['name']}__meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
        arrays[f"{c['name']}__out"] = out.astype(np.float32)
        arrays[f"{c['name']}__ids"] = ids.numpy().astype(np.int64)
        arrays[f"{c['name']}__weights"] = weights.numpy().astype(np.float32)
        print(f"moe {c['name']}: ids={ids.numpy().tolist()} out[0,:3]={out[0, :3]}")
    np.savez_compressed(out_path, **arrays)


# --------------------------------------------------------------------------- whole decode steps

MODEL_CASE = dict(name="gptoss_2layer", n_layer=2, vocab_size=4096, seed=3, ctx=300,
                  tokens=[17, 4000, 123])


def golden_model(out_path: Path):
    """The reference's own ``GptOssModel.forward`` decoding 3 tokens on a 2-layer GPT-OSS-120B-wide model.

    Widths are GPT-OSS-120B's (hidden 2880, 64 query / 8 kv heads of 64, 128 experts top-4, expert
    ffn 2880, YaRN RoPE, sliding window 128 on even layers) with 2 layers and a 4096-token
    vocabulary; every tensor comes from ``tests.model_twin.model_tensors`` (the device generator's
    host twin).  The KV cache starts with ``ctx`` synthetic positions; the tokens are decoded at
    positions ctx, ctx+1, ctx+2 (each appending to the cache).  Stores the logits and, per token and
    layer, the routed expert ids the reference's ``_route`` chose.
    """
    import torch
    from neurostream.model.gpt_oss import GptOssConfig, GptOssModel
    from neurostream.model.qwen3 import KVCache
    from neurostream.residency.cache import TieredCache

    from nurostream_b200.shapes import GptOssShape
    from tests.model_twin import kv_history, model_tensors

    c = MODEL_CASE
    shape = GptOssShape(n_layer=c["n_layer"], vocab_size=c["vocab_size"])
    src = SynthSource(model_tensors(shape, c["seed"]))
    cache = TieredCache(src, vram_budget=1 << 40)
    for name, info in src.gguf.tensors.items():
        if info.dtype.name in ("F32", "BF16"):
            assert cache.admit_vram(name)
    model = GptOssModel(cache, GptOssConfig(**shape.reference_config()), block_rows=512)
    routed = []
    orig_route = GptOssModel._route

    def recording_route(self, h, layer):
        out = orig_route(self, h, layer)
        routed.append(out[1].numpy().astype(np.int64).copy())
        return out

    kv = KVCache(shape.n_layer)
    for l, (k, v) in kv_history(shape, c["seed"], c["ctx"]).items():
        kv.k[l], kv.v[l] = torch.from_numpy(k.copy()), torch.from_numpy(v.copy())
    kv.length = c["ctx"]
    logits = []
    GptOssModel._route = recording_route
    try:
        with torch.no_grad():
            for i, tok in enumerate(c["tokens"]):
                y = model.forward(tokens=[tok], kv=kv, start_pos=c["ctx"] + i)
                logits.append(y.numpy().astype(np.float32).reshape(-1))
    finally:
        GptOssModel._route = orig_route
    meta = dict(c)
    arrays = {
        f"{c['name']}__meta": np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8),
        f"{c['name']}__logits": np.stack(logits),
        f"{c['name']}__ids": np.stack(routed).reshape(len(c["tokens"]), shape.n_layer, -1),
    }
    np.savez_compressed(out_path, **arrays)
    print(f"model {c['name']}: logits[0,:3]={logits[0][:3]} ids={arrays[c['name'] + '__ids'].tolist()}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--only", choices=["dequant", "gemv", "moe", "model"], default=None)
    args = ap.parse_args()
    _import_reference(args.reference)
    import torch
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    if args.only in (None, "dequant"):
        golden_dequant(HERE / "dequant.npz")
    if args.only in (None, "gemv"):
        golden_gemv(HERE / "gemv.npz")
    if args.only in (None, "moe"):
        golden_moe(HERE / "moe.npz")
    if args.only in (None, "model"):
        golden_model(HERE / "model.npz")


if __name__ == "__main__":
    main()
