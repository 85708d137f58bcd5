"""CPU oracle: numpy restatement of the reference's MoE decode step.

TEST INFRASTRUCTURE ONLY (see ``oracle/quant.py`` for who may import it).

Covers the router (GPT-OSS top-k-then-softmax and Qwen3 softmax-top-k-renorm),
the two activations, one expert's gate/up/down walk and the weighted combine,
in the reference's fp32 order of operations.  Parity pin: checked against
outputs of the reference's own ``GptOssModel._ffn_block`` / ``_route`` and
``moe.router.moe_ffn`` on seeded synthetic layers, stored under
``tests/golden/`` by ``tests/golden/make_golden.py``.
"""
from __future__ import annotations

from typing import Callable

import numpy as np

from . import quant

_F32 = np.float32


def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float) -> np.ndarray:
    """``x * rsqrt(mean(x^2) + eps) * w`` in fp32 (``neurostream/compute/ops.py:14-20``)."""
    x = x.astype(_F32)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=_F32)
    r = (_F32(1.0) / np.sqrt(var + _F32(eps))).astype(_F32)
    return (x * r) * weight.astype(_F32)


def linear(x: np.ndarray, w: np.ndarray, acc=_F32) -> np.ndarray:
    """``x @ w.T``; ``acc=np.float64`` gives a tighter truth for tolerance checks."""
    return (x.astype(acc) @ w.astype(acc).T).astype(_F32)


def quant_linear(x: np.ndarray, raw: np.ndarray, dtype, n_rows: int, K: int, acc=_F32) -> np.ndarray:
    """``x @ dequant(raw).T`` -- what the reference's fused GEMV computes.

    Follows ``neurostream/compute/triton_kernels.py:199-228`` (result) via the
    reference CPU path ``neurostream/compute/blockffn.py:171-176``: dequantize
    the row block, then multiply.
    """
    w = quant.dequantize(raw, dtype, n_rows * K).reshape(n_rows, K)
    return linear(np.atleast_2d(x), w, acc)


def _softmax(v: np.ndarray) -> np.ndarray:
    v = v.astype(_F32)
    e = np.exp(v - v.max(axis=-1, keepdims=True)).astype(_F32)
    return (e / e.sum(axis=-1, keepdims=True, dtype=_F32)).astype(_F32)


def topk(v: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    """Largest k per row, descending; exact ties resolve to the lower index."""
    ids = np.argsort(-v, axis=-1, kind="stable")[:, :k]
    return np.take_along_axis(v, ids, axis=-1), ids


def route_gptoss(h: np.ndarray, w: np.ndarray, b: np.ndarray | None, k: int, acc=_F32):
    """GPT-OSS router: biased logits -> top-k -> softmax over the k.

    Follows ``neurostream/model/gpt_oss.py:116-121`` (``_biased_linear`` at
    :97-99).  Returns (ids (T,k) int64, weights (T,k) fp32, logits (T,E)).
    """
    logits = linear(h, w, acc)
    if b is not None:
        logits = (logits + b.astype(_F32)).astype(_F32)
    top, ids = topk(logits, k)
    return ids, _softmax(top), logits


def route_qwen(h: np.ndarray, w: np.ndarray, k: int, acc=_F32):
    """Qwen3-MoE router: softmax over all experts -> top-k -> renormalise.

    Follows ``neurostream/moe/router.py:59-69``.
    """
    logits = linear(h, w, acc)
    probs = _softmax(logits)
    top, ids = topk(probs, k)
    weights = (top / top.sum(axis=-1, keepdims=True, dtype=_F32)).astype(_F32)
    return ids, weights, logits


def sigmoid(x: np.ndarray) -> np.ndarray:
    x = x.astype(_F32)
    return (_F32(1.0) / (_F32(1.0) + np.exp(-x))).astype(_F32)


def clamped_swiglu(gate: np.ndarray, up: np.ndarray, alpha: float = 1.702, limit: float = 7.0):
    """GPT-OSS activation (``neurostream/model/gpt_oss.py:61-70``)."""
    gate = np.minimum(gate.astype(_F32), _F32(limit))
    up = np.clip(up.astype(_F32), _F32(-limit), _F32(limit))
    return ((up + _F32(1.0)) * (gate * sigmoid(gate * _F32(alpha)))).astype(_F32)


def silu_mul(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """Qwen3 activation ``silu(gate) * up`` (``neurostream/moe/router.py:208``)."""
    gate = gate.astype(_F32)
    return ((gate * sigmoid(gate)) * up.astype(_F32)).astype(_F32)


ExpertRows = Callable[[str, int], np.ndarray]
"""``rows(kind, e)`` -> dequantized (out, in) fp32 matrix of expert e, kind in gate/up/down."""


def expert_ffn(rows: ExpertRows, e: int, x: np.ndarray, act, biases: dict | None, acc=_F32):
    """One expert's gate/up -> activation -> down walk.

    Follows ``neurostream/compute/blockffn.py:396-449`` (``stream_expert_ffn``),
    including the per-expert bias row added after each projection.
    """
    def project(kind, v):
        y = linear(v, rows(kind, e), acc)
        if biases is not None:
            y = (y + biases[kind][e].astype(_F32)).astype(_F32)
        return y

    a = act(project("gate", x), project("up", x))
    return project("down", a)


def combine(ids: np.ndarray, weights: np.ndarray, expert_out) -> np.ndarray:
    """Weighted combine in ascending expert order.

    Follows ``neurostream/model/gpt_oss.py:139-173`` / ``neurostream/moe/router.py:183-211``:
    for each distinct expert (sorted), ``out[rows] += w_rows * expert(h[rows])``.
    ``expert_out(e, rows)`` returns the (len(rows), H) expert output.
    """
    out = None
    for e in np.unique(ids):
        mask = ids == e
        rows = np.nonzero(mask.any(axis=-1))[0]
        w = (weights * mask).sum(axis=-1, dtype=_F32)[rows, None].astype(_F32)
        y = expert_out(int(e), rows)
        if out is None:
            out = np.zeros((ids.shape[0], y.shape[1]), dtype=_F32)
        out[rows] = (out[rows] + w * y).astype(_F32)
    return out


def gptoss_ffn_block(x, norm_w, eps, router_w, router_b, rows: ExpertRows, biases, k,
                     alpha=1.702, limit=7.0, acc=_F32):
    """GPT-OSS MoE FFN block: ``x + sum_e w_e * expert_e(rms_norm(x))``.

    Follows ``neurostream/model/gpt_oss.py:123-177``.  Returns (out, ids, weights).
    """
    x = np.atleast_2d(x).astype(_F32)
    h = rms_norm(x, norm_w, eps)
    ids, weights, _ = route_gptoss(h, router_w, router_b, k, acc)
    act = lambda g, u: clamped_swiglu(g, u, alpha, limit)
    moe = combine(ids, weights, lambda e, r: expert_ffn(rows, e, h[r], act, biases, acc))
    return (x + moe).astype(_F32), ids, weights


def qwen_moe_ffn(h, router_w, rows: ExpertRows, k, acc=_F32):
    """Qwen3 sparse FFN on already-normalised ``h``; returns (moe_out, ids, weights).

    Follows ``neurostream/moe/router.py:173-219`` (no shared expert, no biases).
    """
    h = np.atleast_2d(h).astype(_F32)
    ids, weights, _ = route_qwen(h, router_w, k, acc)
    moe = combine(ids, weights, lambda e, r: expert_ffn(rows, e, h[r], silu_mul, None, acc))
    return moe, ids, weights


def stacked_rows(raw_by_kind: dict, dtype, F: int, H: int) -> ExpertRows:
    """Expert-row accessor over stacked (E, out, in) GGUF byte tensors.

    Expert e of a stacked tensor owns rows [e*out, (e+1)*out)
    (``neurostream/io/source.py:38-62``).  ``raw_by_kind[kind]`` is either a
    flat uint8 array or a callable ``(row_start, row_end) -> bytes``.
    """
    from nurostream_b200.ggml import row_bytes

    shape = {"gate": (F, H), "up": (F, H), "down": (H, F)}

    def rows(kind, e):
        out, K = shape[kind]
        rb = row_bytes(dtype, K)
        src = raw_by_kind[kind]
        if callable(src):
            raw = src(e * out, (e + 1) * out)
        else:
            raw = src[e * out * rb:(e + 1) * out * rb]
        return quant.dequantize(raw, dtype, out * K).reshape(out, K)

    return rows
