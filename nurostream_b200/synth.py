"""Seeded, counter-based synthetic GGUF tensors (host side).

The benchmark configurations are synthetic: random quantized expert weights
and near-normal float weights and activations.  Every byte and value is a pure
function of ``(seed, stream, index)``, so the device generator
(``ns_synth_fill`` in ``csrc/synth.cu``) fills a 60 GB expert store in seconds
while this numpy twin regenerates any slice of it bit for bit on the host.

Generator: splitmix64 (Steele, Lea & Flood, "Fast splittable pseudorandom
number generators", 2014): word i of a stream with key k is
``mix64(k + (i + 1) * 0x9E3779B97F4A7C15)``.

Distributions:
* quantized payload bytes: uniform over 0..255 (codes uniform);
* MXFP4 E8M0 exponents: ``lo + byte % (hi - lo + 1)`` (default 118..124);
* fp16 block scales (d, dmin): ``fp16((0.5 + u) * scale_mult)``, u uniform on
  [0, 1) with 23 bits (exact in fp32), default ``scale_mult = 1e-3``;
* float values: Irwin-Hall sum of 12 uniform 24-bit draws minus 6 (mean 0,
  variance 1, bounded to +-6), times ``sigma``.  The sum is exact in fp64, so
  host and device agree to the bit after the same fp32 rounding.
"""
from __future__ import annotations

import numpy as np

from .ggml import TYPE_LAYOUT, GGMLType

GAMMA = 0x9E3779B97F4A7C15
_M1 = 0xBF58476D1CE4E5B9
_M2 = 0x94D049BB133111EB
AUX_SALT = 0xA5A5A5A5A5A5A5A5
STREAM_SALT = 0x632BE59BD9B4E019

_U64 = np.uint64


def _mix64(z: np.ndarray) -> np.ndarray:
    z = z ^ (z >> _U64(30))
    z = z * _U64(_M1)
    z = z ^ (z >> _U64(27))
    z = z * _U64(_M2)
    return z ^ (z >> _U64(31))


def _mix64_int(z: int) -> int:
    mask = (1 << 64) - 1
    z &= mask
    z ^= z >> 30
    z = (z * _M1) & mask
    z ^= z >> 27
    z = (z * _M2) & mask
    return z ^ (z >> 31)


def stream_key(seed: int, stream: int) -> int:
    """64-bit key of one tensor's stream."""
    return _mix64_int(((seed * GAMMA) & ((1 << 64) - 1)) ^ ((stream + STREAM_SALT) & ((1 << 64) - 1)))


def words(key: int, start: int, count: int) -> np.ndarray:
    """Words ``start .. start+count-1`` of the stream with this key (in-place uint64 passes)."""
    z = np.arange(start + 1, start + count + 1, dtype=np.uint64)
    t = np.empty_like(z)
    with np.errstate(over="ignore"):
        np.multiply(z, _U64(GAMMA), out=z)
        np.add(z, _U64(key), out=z)
        for shift, mult in ((30, _M1), (27, _M2), (31, None)):
            np.right_shift(z, _U64(shift), out=t)
            np.bitwise_xor(z, t, out=z)
            if mult is not None:
                np.multiply(z, _U64(mult), out=z)
    return z


def _scale_fp16(key: int, idx: np.ndarray, scale_mult: float) -> np.ndarray:
    """fp16 block scales for aux indices ``idx`` (see module doc)."""
    aux = key ^ AUX_SALT
    i = idx.astype(np.uint64)
    with np.errstate(over="ignore"):
        w = _mix64(_U64(aux) + (i + _U64(1)) * _U64(GAMMA))
    u = (w >> _U64(41)).astype(np.float64) * 2.0 ** -23          # exact
    v = (0.5 + u).astype(np.float32) * np.float32(scale_mult)     # one fp32 rounding
    return v.astype(np.float16)


def quant_bytes(dtype, seed: int, stream: int, start: int, count: int,
                e_lo: int = 118, e_hi: int = 124, scale_mult: float = 1e-3) -> np.ndarray:
    """Bytes ``[start, start+count)`` of a synthetic tensor of GGML type ``dtype``."""
    t = GGMLType(int(dtype))
    key = stream_key(seed, stream)
    w0 = start >> 3
    nw = ((start + count + 7) >> 3) - w0
    raw = words(key, w0, nw).view(np.uint8)                       # little-endian bytes
    out = raw[start - (w0 << 3): start - (w0 << 3) + count].copy()
    pos = np.arange(start, start + count, dtype=np.int64)
    _, bb = TYPE_LAYOUT[t]
    off = pos % bb
    blk = pos // bb

    def put_fp16(field_lo: int, field: int):
        sel = (off == field_lo) | (off == field_lo + 1)
        if not sel.any():
            return
        h = _scale_fp16(key, blk[sel] * 2 + field, scale_mult).view(np.uint16)
        hi_byte = off[sel] == field_lo + 1
        out[sel] = np.where(hi_byte, h >> 8, h & 0xFF).astype(np.uint8)

    if t == GGMLType.MXFP4:
        sel = off == 0
        out[sel] = (e_lo + out[sel].astype(np.int64) % (e_hi - e_lo + 1)).astype(np.uint8)
    elif t in (GGMLType.Q8_0, GGMLType.Q4_0):
        put_fp16(0, 0)
    elif t in (GGMLType.Q4_K, GGMLType.Q5_K):
        put_fp16(0, 0)
        put_fp16(2, 1)
    elif t == GGMLType.Q6_K:
        put_fp16(208, 0)
    else:
        raise NotImplementedError(f"no synthetic generator for {t.name}")
    return out


def float_values(seed: int, stream: int, start: int, count: int, sigma: float = 1.0,
                 dtype=np.float32) -> np.ndarray:
    """Values ``[start, start+count)`` of a synthetic near-normal float tensor."""
    key = stream_key(seed, stream)
    v = np.empty(count, dtype=np.float32)
    chunk = 1 << 16                                               # values per pass (cache-sized)
    for c0 in range(0, count, chunk):
        n = min(chunk, count - c0)
        w = words(key, 12 * (start + c0), 12 * n)
        np.right_shift(w, _U64(40), out=w)
        s = w.reshape(n, 12).sum(axis=1, dtype=np.uint64)        # exact integer sum
        v[c0:c0 + n] = (s.astype(np.float64) * 2.0 ** -24 - 6.0).astype(np.float32)
    v = v * np.float32(sigma)
    if dtype == np.float32:
        return v
    if dtype == "bf16":
        b = v.view(np.uint32).astype(np.uint64)
        b = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
        return b.astype(np.uint16)
    return v.astype(dtype)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


class LayerStreams:
    """Stream ids of one synthetic MoE layer's tensors (layer-major, disjoint)."""

    def __init__(self, layer: int):
        base = 1000 * (layer + 1)
        self.x = base + 0          # activations entering the layer
        self.norm_w = base + 1     # post-attention RMSNorm weight
        self.router_w = base + 2   # router weight (E, H)
        self.router_b = base + 3   # router bias (E,)
        self.gate = base + 10      # ffn_gate_exps (E, F, H), quantized
        self.up = base + 11        # ffn_up_exps (E, F, H), quantized
        self.down = base + 12      # ffn_down_exps (E, H, F), quantized
        self.gate_b = base + 13    # ffn_gate_exps.bias (E, F)
        self.up_b = base + 14      # ffn_up_exps.bias (E, F)
        self.down_b = base + 15    # ffn_down_exps.bias (E, H)
        self.attn_norm = base + 20  # attn_norm.weight (H,)
        self.q_w = base + 21        # attn_q.weight (n_head*hd, H), bf16
        self.q_b = base + 22        # attn_q.bias
        self.k_w = base + 23        # attn_k.weight (n_kv*hd, H), bf16
        self.k_b = base + 24
        self.v_w = base + 25        # attn_v.weight (n_kv*hd, H), bf16
        self.v_b = base + 26
        self.o_w = base + 27        # attn_output.weight (H, n_head*hd), bf16
        self.o_b = base + 28
        self.sinks = base + 29      # attn_sinks.weight (n_head,)
        self.k_cache = base + 30    # synthetic key history (n_kv, ctx, hd)
        self.v_cache = base + 31    # synthetic value history


class ModelStreams:
    """Stream ids of a synthetic model's tensors outside the layers."""

    token_embd = 1       # token_embd.weight (vocab, H), bf16
    output_norm = 2      # output_norm.weight (H,)
    output = 3           # output.weight (vocab, H), bf16


# ----------------------------------------------------------------------------- device fill

def fill_quant(dst, dtype, seed: int, stream: int, start: int = 0, e_lo: int = 118, e_hi: int = 124,
               scale_mult: float = 1e-3) -> None:
    """Fill a uint8 CUDA tensor with bytes [start, start+numel) of a synthetic tensor."""
    import torch

    from . import _lib
    assert dst.dtype == torch.uint8 and dst.is_cuda and dst.is_contiguous()
    _lib.call("ns_synth_fill", dst.data_ptr(), dst.numel(), int(GGMLType(int(dtype))), seed, stream, start,
              1.0, e_lo, e_hi, scale_mult, torch.cuda.current_stream(dst.device).cuda_stream)


def fill_float(dst, seed: int, stream: int, start: int = 0, sigma: float = 1.0) -> None:
    """Fill a float32 or bfloat16 CUDA tensor with values [start, start+numel) of a synthetic stream."""
    import torch

    from . import _lib
    assert dst.is_cuda and dst.is_contiguous()
    kind = {torch.float32: _lib.NS_SYNTH_F32, torch.bfloat16: _lib.NS_SYNTH_BF16}[dst.dtype]
    _lib.call("ns_synth_fill", dst.data_ptr(), dst.numel(), kind, seed, stream, start, sigma, 0, 0, 0.0,
              torch.cuda.current_stream(dst.device).cuda_stream)
