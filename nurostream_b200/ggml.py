"""GGML tensor type codes and block layouts used on the decode hot path.

The numeric codes are the on-disk GGUF type ids, so a ``GGMLType`` from the
reference's own GGUF parser (``neurostream/format/gguf.py:19-35``) converts to
this enum by value, and ``int(dtype)`` is what crosses the C ABI.  The block
layouts restate ``TYPE_LAYOUT`` (``neurostream/format/gguf.py:39-55``): they are
fixed by the GGUF format, not a design choice.
"""
from __future__ import annotations

from enum import IntEnum


class GGMLType(IntEnum):
    F32 = 0
    F16 = 1
    Q4_0 = 2
    Q8_0 = 8
    Q4_K = 12
    Q5_K = 13
    Q6_K = 14
    BF16 = 30
    MXFP4 = 39


# (elements per block, bytes per block), per the GGUF format.
TYPE_LAYOUT: dict[GGMLType, tuple[int, int]] = {
    GGMLType.F32: (1, 4),
    GGMLType.F16: (1, 2),
    GGMLType.BF16: (1, 2),
    GGMLType.MXFP4: (32, 17),
    GGMLType.Q4_0: (32, 18),
    GGMLType.Q8_0: (32, 34),
    GGMLType.Q4_K: (256, 144),
    GGMLType.Q5_K: (256, 176),
    GGMLType.Q6_K: (256, 210),
}

# Quantized formats the fused GEMV reads directly: the reference's Triton set
# (``neurostream/compute/triton_kernels.py:177-186``: MXFP4, Q8_0, Q4_K, Q6_K) plus Q5_K and Q4_0,
# which the reference can only dequantize (``neurostream/compute/quant.py:59-81, 118-126``).
FUSED_TYPES = frozenset({GGMLType.MXFP4, GGMLType.Q8_0, GGMLType.Q4_K, GGMLType.Q6_K, GGMLType.Q5_K,
                         GGMLType.Q4_0})

# Expert formats of the fused MoE layer (ns_moe_decode_layer).
MOE_TYPES = frozenset({GGMLType.MXFP4, GGMLType.Q8_0, GGMLType.Q4_K, GGMLType.Q6_K})

# Formats the device dequantizer expands (``neurostream/compute/quant.py:143-150``
# plus the three float types handled inline at ``quant.py:166-171``).
DEQUANT_TYPES = frozenset(TYPE_LAYOUT)


def as_ggml_type(dtype) -> GGMLType:
    """Accept this enum, the reference's enum, or a plain int."""
    try:
        return GGMLType(int(dtype))
    except ValueError:
        raise NotImplementedError(f"unsupported ggml type: {dtype!r}") from None


def row_bytes(dtype, row_elems: int) -> int:
    """Bytes of one row of ``row_elems`` elements (rows span whole blocks)."""
    t = as_ggml_type(dtype)
    block_elems, block_bytes = TYPE_LAYOUT[t]
    if row_elems % block_elems:
        raise ValueError(
            f"{row_elems} elements is not a multiple of {t.name} block size {block_elems}"
        )
    return (row_elems // block_elems) * block_bytes
