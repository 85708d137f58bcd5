"""Drop-in replacement of ``neurostream/compute/triton_kernels.py``.

Same names and argument meaning as the reference (``can_fuse``,
``fused_gemv``), backed by the hand-written sm_100a kernel ``ns_gemv`` instead
of Triton.  Callers that look these up as module attributes at call time
(``neurostream/compute/blockffn.py:137-139``, ``neurostream/moe/router.py:22``,
``neurostream/model/qwen3.py:174``) are rerouted by ``nurostream_b200.install``.

Differences from the reference, all deliberate:
* ``can_fuse`` accepts 1..NS_MAX_TOKENS activation rows (the reference: exactly
  one); the kernel handles a small batch in one pass over the weights.
* ``fused_gemv`` writes ``out_dtype`` directly (no fp32 temporary + cast) and
  validates the byte count; ``block_n`` / ``num_warps`` are accepted and
  ignored because the library picks its own launch shape.
* Unsupported types raise ``KeyError`` like the reference's ``_KERNELS[dtype]``.
"""
from __future__ import annotations

import torch

from . import _lib
from .ggml import FUSED_TYPES, GGMLType, as_ggml_type, row_bytes

_TORCH_TO_NS = {torch.float32: _lib.NS_F32, torch.float16: _lib.NS_F16, torch.bfloat16: _lib.NS_BF16}


def ns_dtype(dt: torch.dtype) -> int:
    try:
        return _TORCH_TO_NS[dt]
    except KeyError:
        raise TypeError(f"unsupported float dtype {dt}; expected float32, float16 or bfloat16") from None


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


_HAVE: bool | None = None


def kernels_available() -> bool:
    """True once libns_b200.so loads; the first call loads it (not at import time)."""
    global _HAVE
    if _HAVE is None:
        try:
            _lib.load()
            _HAVE = True
        except Exception:
            _HAVE = False
    return _HAVE


MAX_TOKENS = _lib.NS_MAX_TOKENS


def can_fuse(dtype, x: torch.Tensor) -> bool:
    """Fused path applies to decode-sized activations on CUDA in a fused format."""
    try:
        t = GGMLType(int(dtype))
    except ValueError:
        return False
    return (
        x.is_cuda
        and x.dim() >= 1
        and 1 <= (x.shape[0] if x.dim() > 1 else 1) <= MAX_TOKENS
        and t in FUSED_TYPES
        and x.dtype in _TORCH_TO_NS
        and kernels_available()
    )


def can_fuse_rows(x: torch.Tensor) -> bool:
    """x has 1..NS_MAX_TOKENS activation rows of a supported float type (the GEMV's batch limit)."""
    return x.dim() >= 1 and 1 <= (x.shape[0] if x.dim() > 1 else 1) <= MAX_TOKENS and x.dtype in _TORCH_TO_NS


def fused_gemv(
    raw: torch.Tensor,
    dtype,
    x: torch.Tensor,
    n_rows: int,
    K: int,
    out_dtype: torch.dtype = torch.float16,
    block_n: int = 16,
    num_warps: int = 2,
) -> torch.Tensor:
    """y = x @ dequant(raw).T without materialising the weights.

    raw: (n_rows * row_bytes,) uint8 on CUDA (a view with a storage offset is
    fine).  x: (T, K) with 1 <= T <= NS_MAX_TOKENS.  Returns (T, n_rows).
    """
    t = GGMLType(int(dtype))
    if t not in FUSED_TYPES:
        raise KeyError(t)
    if raw.dtype != torch.uint8 or not raw.is_cuda:
        raise TypeError(f"raw must be a uint8 CUDA tensor, got {raw.dtype} on {raw.device}")
    if not raw.is_contiguous():
        raw = raw.contiguous()
    xf = x.reshape(-1, K)
    if not xf.is_contiguous():
        xf = xf.contiguous()
    T = xf.shape[0]
    rb = row_bytes(t, K)
    if raw.numel() < n_rows * rb:
        raise ValueError(f"raw has {raw.numel()} bytes; {n_rows} rows of {t.name} K={K} need {n_rows * rb}")
    y = torch.empty((T, n_rows), device=xf.device, dtype=out_dtype)
    _lib.call(
        "ns_gemv", raw.data_ptr(), raw.numel(), int(t), n_rows, K,
        xf.data_ptr(), ns_dtype(xf.dtype), K, T,
        y.data_ptr(), ns_dtype(out_dtype), n_rows, stream_of(xf),
    )
    return y


def dequantize(raw: torch.Tensor, dtype, n_elements: int, out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Device mirror of ``neurostream/compute/quant.py:153-184`` (bit-exact).

    Expands ``raw`` (uint8, 1-D, on CUDA) into the first ``n_elements`` values.
    """
    if raw.dtype != torch.uint8:
        raise TypeError(f"expected uint8 byte buffer, got {raw.dtype}")
    if not raw.is_cuda:
        raise RuntimeError("nurostream_b200.dequantize runs on CUDA tensors only (no CPU fallback)")
    t = as_ggml_type(dtype)
    raw = raw.reshape(-1)
    if not raw.is_contiguous():
        raw = raw.contiguous()
    out = torch.empty(n_elements, device=raw.device, dtype=out_dtype)
    _lib.call("ns_dequant", raw.data_ptr(), raw.numel(), int(t), n_elements, out.data_ptr(),
              ns_dtype(out_dtype), stream_of(raw))
    return out
