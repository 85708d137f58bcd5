"""CPU oracle: numpy restatement of the reference's GGML block decoders.

TEST INFRASTRUCTURE ONLY.  This module is the checker that the CUDA kernels are
compared against.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it; the
product package ``nurostream_b200`` never does.

Parity pin: every decoder here is checked bit for bit against outputs of the
reference's own ``neurostream.compute.quant.dequantize`` (and, where gguf-py
implements the format, against ``gguf.dequantize``), stored as fixtures under
``tests/golden/`` by ``tests/golden/make_golden.py``.

Each function follows the reference file:line it cites, in the same fp32
operation order, so the decoded floats are identical bit for bit.
"""
from __future__ import annotations

import numpy as np

from nurostream_b200.ggml import TYPE_LAYOUT, GGMLType

_F32 = np.float32


def _f16_field(blocks: np.ndarray, lo: int) -> np.ndarray:
    """Little-endian fp16 at byte ``lo`` of each block, widened to fp32 (nb, 1).

    Follows ``neurostream/compute/quant.py:19-21``.
    """
    raw = np.ascontiguousarray(blocks[:, lo:lo + 2])
    return raw.view(np.float16).astype(_F32)


def _k_scales_mins(scales: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """6-bit scale/min pairs of Q4_K/Q5_K: (nb, 8) each, as fp32.

    Follows ``neurostream/compute/quant.py:24-38`` (ggml get_scale_min_k4):
    sub-blocks 0..3 take the low 6 bits of bytes 0..3 / 4..7; sub-blocks 4..7
    take 4 bits from bytes 8..11 and borrow the top 2 bits of bytes 0..7.
    """
    q = scales.astype(np.int32)
    sc = np.concatenate([q[:, 0:4] & 63, (q[:, 8:12] & 0x0F) | ((q[:, 0:4] >> 6) << 4)], axis=1)
    mn = np.concatenate([q[:, 4:8] & 63, (q[:, 8:12] >> 4) | ((q[:, 4:8] >> 6) << 4)], axis=1)
    return sc.astype(_F32), mn.astype(_F32)


def dequant_q4_k(blocks: np.ndarray) -> np.ndarray:
    """Q4_K, 144 B -> 256 values: ``d*sc*q - dmin*mn``.

    Follows ``neurostream/compute/quant.py:41-56``.  Group g of 64 values reads
    ``qs[32g:32g+32]``: low nibbles are sub-block 2g, high nibbles 2g+1.
    """
    nb = blocks.shape[0]
    d = _f16_field(blocks, 0)
    dmin = _f16_field(blocks, 2)
    sc, mn = _k_scales_mins(blocks[:, 4:16])
    qs = blocks[:, 16:144].reshape(nb, 4, 32).astype(np.int32)
    q = np.stack([qs & 0x0F, qs >> 4], axis=2).reshape(nb, 8, 32).astype(_F32)
    scale = (d * sc)[:, :, None]
    offset = (dmin * mn)[:, :, None]
    return (scale * q - offset).reshape(nb, 256)


def dequant_q5_k(blocks: np.ndarray) -> np.ndarray:
    """Q5_K, 176 B -> 256 values; the 5th bit of group g is bit (2g, 2g+1) of qh.

    Follows ``neurostream/compute/quant.py:59-81``.
    """
    nb = blocks.shape[0]
    d = _f16_field(blocks, 0)
    dmin = _f16_field(blocks, 2)
    sc, mn = _k_scales_mins(blocks[:, 4:16])
    qh = blocks[:, 16:48].astype(np.int32)[:, None, :]          # (nb, 1, 32)
    qs = blocks[:, 48:176].reshape(nb, 4, 32).astype(np.int32)
    g = np.arange(4, dtype=np.int32)[None, :, None]
    lo = (qs & 0x0F) + (((qh >> (2 * g)) & 1) << 4)
    hi = (qs >> 4) + (((qh >> (2 * g + 1)) & 1) << 4)
    q = np.stack([lo, hi], axis=2).reshape(nb, 8, 32).astype(_F32)
    return ((d * sc)[:, :, None] * q - (dmin * mn)[:, :, None]).reshape(nb, 256)


def dequant_q6_k(blocks: np.ndarray) -> np.ndarray:
    """Q6_K, 210 B -> 256 values: ``(d*sc)*(q-32)``, left to right as the reference.

    Follows ``neurostream/compute/quant.py:84-107``: per 128-value half h, the
    four 32-wide lanes take ql low/high nibbles and 2-bit slices of qh; lane i
    of half h, element l uses scale ``sc[h, l//16 + 2i]``.
    """
    nb = blocks.shape[0]
    ql = blocks[:, 0:128].reshape(nb, 2, 64).astype(np.int32)
    qh = blocks[:, 128:192].reshape(nb, 2, 32).astype(np.int32)
    sc = blocks[:, 192:208].view(np.int8).reshape(nb, 2, 8).astype(_F32)
    d = _f16_field(blocks, 208)[:, :, None]                      # (nb, 1, 1)
    lanes = (
        (ql[:, :, 0:32] & 0x0F) | (((qh >> 0) & 3) << 4),
        (ql[:, :, 32:64] & 0x0F) | (((qh >> 2) & 3) << 4),
        (ql[:, :, 0:32] >> 4) | (((qh >> 4) & 3) << 4),
        (ql[:, :, 32:64] >> 4) | (((qh >> 6) & 3) << 4),
    )
    l16 = np.arange(32) // 16
    out = np.empty((nb, 2, 128), dtype=_F32)
    for i, qv in enumerate(lanes):
        s = sc[:, :, l16 + 2 * i]                                # (nb, 2, 32)
        out[:, :, 32 * i:32 * (i + 1)] = (d * s) * (qv - 32).astype(_F32)
    return out.reshape(nb, 256)


def dequant_q8_0(blocks: np.ndarray) -> np.ndarray:
    """Q8_0, 34 B -> 32 values: ``d*q``.  Follows ``neurostream/compute/quant.py:110-115``."""
    d = _f16_field(blocks, 0)
    q = np.ascontiguousarray(blocks[:, 2:34]).view(np.int8).astype(_F32)
    return d * q


def dequant_q4_0(blocks: np.ndarray) -> np.ndarray:
    """Q4_0, 18 B -> 32 values: ``d*(q-8)``, low nibbles first.

    Follows ``neurostream/compute/quant.py:118-126``.
    """
    d = _f16_field(blocks, 0)
    qs = blocks[:, 2:18].astype(np.int32)
    q = np.concatenate([(qs & 0x0F) - 8, (qs >> 4) - 8], axis=1).astype(_F32)
    return d * q


# GGML's MXFP4 code table: e2m1 values doubled, +0 for the negative-zero code.
MXFP4_VALUES = np.array([0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12], dtype=_F32)


def e8m0_half_scale(e: np.ndarray) -> np.ndarray:
    """GGML's E8M0 'half' scale 2**(e-128) as fp32 (e=0,1 are subnormals).

    Follows ``neurostream/compute/quant.py:131-134``; e=255 is 2**127, not NaN.
    """
    e = e.astype(np.int64)
    bits = np.where(e < 2, np.int64(0x00200000) << e, (e - 1) << 23).astype(np.uint32)
    return bits.view(_F32)


def dequant_mxfp4(blocks: np.ndarray) -> np.ndarray:
    """MXFP4, 17 B -> 32 values: ``scale(e) * table[code]``.

    Follows ``neurostream/compute/quant.py:129-140``: byte 0 is the exponent;
    value j<16 is the low nibble of payload byte j, value j>=16 the high nibble
    of payload byte j-16.
    """
    scale = e8m0_half_scale(blocks[:, :1])
    packed = blocks[:, 1:].astype(np.int64)
    codes = np.concatenate([packed & 15, packed >> 4], axis=1)
    with np.errstate(over="ignore"):                  # e=255 times 12 overflows to inf, as in the reference
        return scale * MXFP4_VALUES[codes]


_DECODERS = {
    GGMLType.MXFP4: dequant_mxfp4,
    GGMLType.Q4_K: dequant_q4_k,
    GGMLType.Q5_K: dequant_q5_k,
    GGMLType.Q6_K: dequant_q6_k,
    GGMLType.Q8_0: dequant_q8_0,
    GGMLType.Q4_0: dequant_q4_0,
}


def dequantize(raw: np.ndarray, dtype, n_elements: int) -> np.ndarray:
    """Flat uint8 bytes -> first ``n_elements`` values as fp32.

    Follows ``neurostream/compute/quant.py:153-184``: float types are
    reinterpreted, block types decoded block by block, the tail truncated.
    """
    raw = np.asarray(raw)
    if raw.dtype != np.uint8:
        raise TypeError(f"expected uint8 byte buffer, got {raw.dtype}")
    t = GGMLType(int(dtype))
    raw = np.ascontiguousarray(raw.reshape(-1))
    if t == GGMLType.F32:
        return raw[: (raw.size // 4) * 4].view(_F32)[:n_elements].copy()
    if t == GGMLType.F16:
        return raw[: (raw.size // 2) * 2].view(np.float16)[:n_elements].astype(_F32)
    if t == GGMLType.BF16:
        h = raw[: (raw.size // 2) * 2].view(np.uint16)[:n_elements].astype(np.uint32)
        return (h << 16).view(_F32)
    block_elems, block_bytes = TYPE_LAYOUT[t]
    nb = raw.size // block_bytes
    blocks = raw[: nb * block_bytes].reshape(nb, block_bytes)
    return _DECODERS[t](blocks).reshape(-1)[:n_elements].astype(_F32, copy=False)
