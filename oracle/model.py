"""CPU oracle: numpy restatement of the reference's GPT-OSS decode step (attention + MoE + LM head).

TEST INFRASTRUCTURE ONLY (see ``oracle/quant.py`` for who may import it).

Covers ``GptOssModel.forward`` for decode tokens (``neurostream/model/gpt_oss.py:189-228``): the
embedding row, per layer ``_attention_block`` (:101-114 -- RMSNorm, biased q/k/v projections, YaRN
RoPE from ``yarn_tables`` :44-58 with ``apply_rope`` ``neurostream/compute/ops.py:136-151``, the
KV-cache append ``neurostream/model/qwen3.py:74-85``, ``repeat_kv`` ops.py:154-159 and
``sink_attention`` gpt_oss.py:73-87 with the sliding window on even layers, the biased output
projection and the residual) and ``_ffn_block`` (``oracle.moe.gptoss_ffn_block``), then the final
RMSNorm and the LM head.  Parity pin: ``tests/golden/model.npz`` holds the logits and routing of the
reference's own ``forward`` on the same synthetic model (``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import math

import numpy as np

from . import moe

_F32 = np.float32


def yarn_tables(head_dim, rope_base, factor, original_context, beta_fast, beta_slow, positions):
    """cos/sin tables (len(positions), head_dim), fp32 (``neurostream/model/gpt_oss.py:44-58``)."""
    half = head_dim // 2
    dims = np.arange(half, dtype=_F32)
    inv = (_F32(1.0) / (_F32(rope_base) ** (dims / _F32(half)))).astype(_F32)
    if factor != 1:
        def correction(rotations):
            return head_dim * math.log(original_context / (rotations * 2 * math.pi)) / (2 * math.log(rope_base))
        low = max(correction(beta_fast), 0)
        high = min(correction(beta_slow), head_dim - 1)
        ramp = np.clip((dims - _F32(low)) / _F32(high - low if high != low else 0.001), 0, 1).astype(_F32)
        inv = (inv * (_F32(1) - ramp) + inv / _F32(factor) * ramp).astype(_F32)
    freqs = np.asarray(positions, dtype=_F32)[:, None] * inv[None, :]
    freqs = np.concatenate([freqs, freqs], axis=-1).astype(_F32)
    amp = _F32(1 + 0.1 * math.log(factor) if factor > 1 else 1.0)
    return (np.cos(freqs) * amp).astype(_F32), (np.sin(freqs) * amp).astype(_F32)


def apply_rope(x, cos, sin):
    """x (heads, T, hd): ``x * cos + rotate_half(x) * sin`` (``neurostream/compute/ops.py:130-151``)."""
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return (x * cos[None] + rot * sin[None]).astype(_F32)


def sink_attention(q, k, v, sinks, window, acc=_F32):
    """Causal attention of the last q rows over k/v with one sink logit per head.

    q (H, Tq, D), k/v (H, Tk, D) (kv already repeated per query head); follows
    ``neurostream/model/gpt_oss.py:73-87``: visible keys kp <= qp (and kp > qp - window when
    window > 0), scores / sqrt(D), softmax over [scores, sink], sink column dropped.
    """
    tq, tk = q.shape[1], k.shape[1]
    qp = np.arange(tk - tq, tk)[:, None]
    kp = np.arange(tk)[None, :]
    vis = kp <= qp
    if window:
        vis &= kp > qp - window
    scores = (q.astype(acc) @ np.swapaxes(k.astype(acc), -1, -2)) / math.sqrt(q.shape[-1])
    scores = np.where(vis[None], scores, -np.inf)
    sink = np.broadcast_to(sinks.astype(acc)[:, None, None], (q.shape[0], tq, 1))
    allv = np.concatenate([scores, sink], axis=-1)
    m = allv.max(axis=-1, keepdims=True)
    e = np.exp(allv - m)
    probs = (e / e.sum(axis=-1, keepdims=True))[..., :-1]
    return (probs @ v.astype(acc)).astype(_F32)


class Weights:
    """Accessor protocol of the oracle model: ``w(name)`` -> fp32 array of a float tensor,
    ``rows(layer)`` -> ``ExpertRows`` of that layer's experts, ``biases(layer)`` -> {kind: [e] -> row}."""


def attention_block(x, W, layer, cfg, kv, pos, acc=_F32):
    """One decode token's ``_attention_block`` (``neurostream/model/gpt_oss.py:101-114``).

    x (1, H); kv: dict layer -> [k (n_kv, T, hd), v] history (the new key/value are appended, as
    ``KVCache.append`` does); pos: the token's position.  Returns x + o_proj(attention).
    """
    p = f"blk.{layer}."
    hd, nh, nkv = cfg["head_dim"], cfg["n_head"], cfg["n_head_kv"]
    h = moe.rms_norm(x, W.w(p + "attn_norm.weight"), cfg["rms_eps"])

    def biased(name, v):
        return (moe.linear(v, W.w(p + name + ".weight"), acc) + W.w(p + name + ".bias")).astype(_F32)

    q = biased("attn_q", h).reshape(1, nh, hd).transpose(1, 0, 2)
    k = biased("attn_k", h).reshape(1, nkv, hd).transpose(1, 0, 2)
    v = biased("attn_v", h).reshape(1, nkv, hd).transpose(1, 0, 2)
    cos, sin = yarn_tables(hd, cfg["rope_base"], cfg["rope_factor"], cfg["original_context"], cfg["beta_fast"],
                           cfg["beta_slow"], [pos])
    q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
    kh, vh = kv[layer]
    kh = np.concatenate([kh, k], axis=1)
    vh = np.concatenate([vh, v], axis=1)
    kv[layer] = [kh, vh]
    rep = nh // nkv
    window = cfg["sliding_window"] if layer % 2 == 0 else 0
    out = sink_attention(q, np.repeat(kh, rep, axis=0), np.repeat(vh, rep, axis=0), W.w(p + "attn_sinks.weight"),
                         window, acc)
    out = out.transpose(1, 0, 2).reshape(1, nh * hd)
    return (x + biased("attn_output", out)).astype(_F32)


def forward_token(token, W, cfg, kv, pos, acc=_F32, trace=None):
    """Logits (1, vocab) of one decode token at ``pos`` (``GptOssModel.forward``, gpt_oss.py:189-228).

    ``trace``: optional list that receives per layer (ids, x after attention, x after the MoE block).
    """
    x = W.w("token_embd.weight")[token][None, :].astype(_F32)
    for layer in range(cfg["n_layer"]):
        x = attention_block(x, W, layer, cfg, kv, pos, acc)
        xa = x
        p = f"blk.{layer}."
        x, ids, _ = moe.gptoss_ffn_block(x, W.w(p + "post_attention_norm.weight"), cfg["rms_eps"],
                                         W.w(p + "ffn_gate_inp.weight"), W.w(p + "ffn_gate_inp.bias"),
                                         W.rows(layer), W.biases(layer), cfg["n_expert_used"], acc=acc)
        if trace is not None:
            trace.append((ids, xa, x))
    h = moe.rms_norm(x, W.w("output_norm.weight"), cfg["rms_eps"])
    return moe.linear(h, W.w("output.weight"), acc)
