"""Install the B200 kernels into the reference package, in place.

The reference looks its kernels up as module attributes at call time, so
replacing those attributes reroutes every caller without touching the
reference's source:

* ``neurostream.compute.triton_kernels.can_fuse / fused_gemv`` -> ``nurostream_b200.fused``
  (callers: ``compute/blockffn.py:139,166,197,215``, ``moe/router.py:365-383``,
  ``model/qwen3.py:174-185``);
* ``neurostream.compute.quant.dequantize`` and the name bound in
  ``neurostream.residency.cache`` -> the bit-exact device dequantizer for CUDA
  inputs (CPU inputs still go to the reference's own function);
* ``GptOssModel._route / _ffn_block`` (``model/gpt_oss.py:116-205``) and
  ``moe.router.moe_ffn`` (``moe/router.py:173-219``) -> ``nurostream_b200.moe``.

``NeuroStream.load/generate``, ``stream_linear``, ``BlockPrefetcher`` and
``TieredCache`` are left untouched: they are the contracts the drop-in keeps.
"""
from __future__ import annotations

import importlib

from . import fused, moe


class Installation:
    def __init__(self, patches):
        self._patches = patches  # (object, attribute, original)

    def uninstall(self) -> None:
        for obj, attr, orig in reversed(self._patches):
            setattr(obj, attr, orig)
        self._patches = []
        moe._ORIGINALS.clear()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.uninstall()


def install(package: str = "neurostream", streamed: bool = False) -> Installation:
    """Patch an importable reference package; returns a handle that undoes it.

    streamed=True also routes ``compute.blockffn.stream_linear`` calls on RAM-tier quantized tensors
    (CUDA device, fused type, up to NS_MAX_TOKENS rows, no callback or shared prefetcher) to
    ``nurostream_b200.stream.streamed_linear``, which overlaps each block's upload with the previous
    block's GEMV; every other call keeps the reference's own ``stream_linear``.
    """
    tk = importlib.import_module(f"{package}.compute.triton_kernels")
    quant = importlib.import_module(f"{package}.compute.quant")
    cache_mod = importlib.import_module(f"{package}.residency.cache")
    gpt_oss = importlib.import_module(f"{package}.model.gpt_oss")
    router = importlib.import_module(f"{package}.moe.router")

    patches = []

    def patch(obj, attr, new):
        patches.append((obj, attr, getattr(obj, attr)))
        setattr(obj, attr, new)

    ref_dequant = quant.dequantize

    def dequantize(raw, dtype, n_elements, out_dtype=None):
        import torch
        out_dtype = torch.float32 if out_dtype is None else out_dtype
        if raw.is_cuda and raw.dtype == torch.uint8:
            return fused.dequantize(raw, dtype, n_elements, out_dtype)
        return ref_dequant(raw, dtype, n_elements, out_dtype=out_dtype)

    moe._ORIGINALS["gptoss_route"] = gpt_oss.GptOssModel._route
    moe._ORIGINALS["gptoss_ffn_block"] = gpt_oss.GptOssModel._ffn_block
    moe._ORIGINALS["moe_ffn"] = router.moe_ffn

    patch(tk, "can_fuse", fused.can_fuse)
    patch(tk, "fused_gemv", fused.fused_gemv)
    patch(quant, "dequantize", dequantize)
    patch(cache_mod, "dequantize", dequantize)
    patch(gpt_oss.GptOssModel, "_route", lambda self, h, layer: moe.gptoss_route(self, h, layer))
    patch(gpt_oss.GptOssModel, "_ffn_block", lambda self, x, layer: moe.gptoss_ffn_block(self, x, layer))
    patch(router, "moe_ffn", moe.moe_ffn)
    if streamed:
        from . import stream
        blockffn = importlib.import_module(f"{package}.compute.blockffn")
        ref_stream_linear = blockffn.stream_linear

        def stream_linear(provider, name, x, block_rows=1024, device="cpu", dtype=None, callback=None, out=None,
                          row_start=0, row_end=None, lookahead=2, prefetcher=None):
            import torch
            dt = torch.float32 if dtype is None else dtype
            if (callback is None and prefetcher is None and x.is_cuda and fused.can_fuse_rows(x)
                    and torch.device(device).type == "cuda"):
                y = stream.streamed_linear(provider, name, x, block_rows, device, dt, out, row_start, row_end)
                if y is not None:
                    return y
            return ref_stream_linear(provider, name, x, block_rows, device, dt, callback, out, row_start, row_end,
                                     lookahead, prefetcher)

        patch(blockffn, "stream_linear", stream_linear)
    return Installation(patches)
