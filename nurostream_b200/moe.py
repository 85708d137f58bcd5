"""MoE decode step on the B200: router and the fused one-launch layer.

``MoeLayer`` holds one layer's device tensors (router, norm, the stacked
GGUF expert byte slabs -- used exactly as the reference's VRAM-Q cache keeps
them, never repacked -- and the per-expert biases) plus the kernel workspace,
and runs ``ns_moe_decode_layer``.

The reference-facing functions mirror the reference's own operators:
* ``gptoss_route(model, h, layer)``     -> ``GptOssModel._route`` (gpt_oss.py:116-121)
* ``gptoss_ffn_block(model, x, layer)`` -> ``GptOssModel._ffn_block`` (gpt_oss.py:123-205)
* ``moe_ffn(model, h, layer)``          -> ``moe.router.moe_ffn`` (router.py:173-219)
They take the fused path when every expert slab of the layer is resident in
VRAM (quantized) and the token count fits one launch; otherwise they hand the
call to the reference's own streaming implementation (saved by
``nurostream_b200.install``), whose per-block GEMVs then run on ``ns_gemv``.
"""
from __future__ import annotations

import ctypes as C
from collections import Counter
from dataclasses import dataclass, field

import torch

from . import _lib
from .fused import ns_dtype, stream_of
from .ggml import MOE_TYPES, GGMLType, as_ggml_type, row_bytes


@dataclass
class RouterStats:
    """Counters the reference's ``pin_hot_experts`` reads (``neurostream/moe/router.py:27-56``)."""

    tokens_routed: int = 0
    expert_reads: int = 0
    hits: Counter = field(default_factory=Counter)


def route(h: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None, k: int,
          mode: int = _lib.NS_ROUTE_TOPK_SOFTMAX):
    """Router on device: returns (ids (T,k) int64, weights (T,k) fp32, logits (T,E) fp32).

    mode NS_ROUTE_TOPK_SOFTMAX follows ``neurostream/model/gpt_oss.py:116-121``;
    NS_ROUTE_SOFTMAX_TOPK_NORM follows ``neurostream/moe/router.py:59-69``.
    """
    h2 = h.reshape(-1, h.shape[-1]).contiguous()
    T, H = h2.shape
    E = w.shape[0]
    w = w.contiguous()
    bf = None if b is None else b.to(torch.float32).contiguous()
    ids = torch.empty((T, k), device=h.device, dtype=torch.int32)
    weights = torch.empty((T, k), device=h.device, dtype=torch.float32)
    logits = torch.empty((T, E), device=h.device, dtype=torch.float32)
    _lib.call("ns_moe_route", h2.data_ptr(), ns_dtype(h2.dtype), T, H, w.data_ptr(), ns_dtype(w.dtype),
              None if bf is None else bf.data_ptr(), E, k, mode, ids.data_ptr(), weights.data_ptr(),
              logits.data_ptr(), stream_of(h2))
    return ids.long(), weights, logits


def _ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


class MoeLayer:
    """One MoE layer's device tensors + workspace, run by ``ns_moe_decode_layer``.

    gate/up/down: flat uint8 CUDA tensors of stacked experts [expert_lo, expert_hi)
    (gate/up: (n_local*F) rows over H; down: (n_local*H) rows over F).
    """

    def __init__(self, *, H: int, F: int, n_expert: int, k: int, ggml_type, router_w: torch.Tensor,
                 gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor,
                 router_b: torch.Tensor | None = None, norm_w: torch.Tensor | None = None,
                 gate_b: torch.Tensor | None = None, up_b: torch.Tensor | None = None,
                 down_b: torch.Tensor | None = None, expert_lo: int = 0, expert_hi: int | None = None,
                 route_mode: int = _lib.NS_ROUTE_TOPK_SOFTMAX, act_mode: int = _lib.NS_ACT_CLAMPED_SWIGLU,
                 alpha: float = 1.702, limit: float = 7.0, rms_eps: float = 1e-5, max_tokens: int = 1):
        self.t = as_ggml_type(ggml_type)
        if self.t not in MOE_TYPES:
            raise NotImplementedError(f"no fused MoE kernel for {self.t.name}")
        self.H, self.F, self.E, self.k = H, F, n_expert, k
        self.lo = expert_lo
        self.hi = n_expert if expert_hi is None else expert_hi
        n_local = self.hi - self.lo
        dev = router_w.device
        self.device = dev
        self._src = {}
        self.bind_small(router_w=router_w, router_b=router_b, norm_w=norm_w, gate_b=gate_b, up_b=up_b,
                        down_b=down_b)
        self.n_local = n_local
        self.bind(gate, up, down)
        self.route_mode, self.act_mode = route_mode, act_mode
        self.alpha, self.limit, self.rms_eps = alpha, limit, rms_eps
        self.max_tokens = max_tokens
        self._slice = 0  # rows per launch that prefill settled on
        self._pf_ws = None  # workspace of the grouped prefill (grown on demand)
        self.l2_prefetch: list = []  # tensors whose bytes the layer kernel asks L2 to fetch (a hint)
        p = self._params(max_tokens, None, None, True, None, None)
        n = C.c_size_t(0)
        _lib.call("ns_moe_workspace_bytes", C.byref(p), C.byref(n))
        self.workspace = torch.empty(n.value + 256, device=dev, dtype=torch.uint8)
        off = (-self.workspace.data_ptr()) % 256
        self._ws_ptr = self.workspace.data_ptr() + off
        self._ws_bytes = n.value
        _lib.call("ns_moe_workspace_init", self._ws_ptr, self._ws_bytes, stream_of(self.workspace))

    def bind(self, gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor) -> None:
        """Point the layer at (new) stacked expert byte tensors; sizes are checked."""
        H, F, n_local = self.H, self.F, self.n_local
        for name, t, rows, K in (("gate", gate, F, H), ("up", up, F, H), ("down", down, H, F)):
            need = n_local * rows * row_bytes(self.t, K)
            if t.dtype != torch.uint8 or not t.is_cuda or t.numel() < need:
                raise ValueError(f"{name}: expected >= {need} uint8 CUDA bytes, got {t.numel()} {t.dtype} {t.device}")
        self.gate, self.up, self.down = gate.contiguous(), up.contiguous(), down.contiguous()

    def bind_small(self, **tensors) -> None:
        """(Re)bind router / norm / bias tensors; a tensor is converted (fp32, contiguous) only when
        the caller hands a different tensor than last time."""
        for name, v in tensors.items():
            key = None if v is None else (v.data_ptr(), v.dtype, tuple(v.shape))
            if name in self._src and self._src[name] == key:
                continue
            if v is None:
                conv = None
            elif name == "router_w":
                conv = v.contiguous()
            else:
                conv = v.to(device=self.device, dtype=torch.float32).contiguous()
            setattr(self, name, conv)
            self._src[name] = key

    def release_weights(self) -> None:
        """Drop the references to the expert bytes (stream-ordered use already enqueued stays valid:
        the caching allocator reuses freed blocks in stream order)."""
        self.gate = self.up = self.down = None

    def _params(self, T, x, out, add_residual, ids, weights) -> _lib.MoeLayerParams:
        p = _lib.MoeLayerParams()
        p.T, p.H, p.F, p.n_expert = T, self.H, self.F, self.E
        p.expert_lo, p.expert_hi, p.k = self.lo, self.hi, self.k
        p.route_mode, p.act_mode, p.ggml_type = self.route_mode, self.act_mode, int(self.t)
        p.alpha, p.limit, p.rms_eps = self.alpha, self.limit, self.rms_eps
        p.add_residual = 1 if add_residual else 0
        p.x, p.norm_w = _ptr(x), _ptr(self.norm_w)
        p.router_w, p.router_dtype, p.router_b = self.router_w.data_ptr(), ns_dtype(self.router_w.dtype), _ptr(self.router_b)
        p.gate_w, p.up_w, p.down_w = self.gate.data_ptr(), self.up.data_ptr(), self.down.data_ptr()
        p.gate_b, p.up_b, p.down_b = _ptr(self.gate_b), _ptr(self.up_b), _ptr(self.down_b)
        p.out, p.ids, p.weights = _ptr(out), _ptr(ids), _ptr(weights)
        p.l2.set(getattr(self, "l2_prefetch", []))
        return p

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None, add_residual: bool = True,
                 ids: torch.Tensor | None = None, weights: torch.Tensor | None = None) -> torch.Tensor:
        """out = x + sum_e w_e expert_e(norm(x)) (fp32, (T, H)); ids/weights optional (T,k) outputs."""
        if x.dtype != torch.float32 or not x.is_contiguous():
            raise TypeError("x must be a contiguous float32 tensor")
        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"T={T} exceeds the layer's max_tokens={self.max_tokens}")
        if out is None:
            out = torch.empty_like(x)
        p = self._params(T, x, out, add_residual, ids, weights)
        _lib.call("ns_moe_decode_layer", C.byref(p), self._ws_ptr, self._ws_bytes, stream_of(x))
        return out

    def prefill_grouped(self, x: torch.Tensor, out: torch.Tensor | None = None, add_residual: bool = True,
                        ids: torch.Tensor | None = None, weights: torch.Tensor | None = None) -> torch.Tensor:
        """T tokens (any T) through ``ns_moe_prefill_grouped``: the routed experts as a grouped GEMM on
        the tensor cores, each expert's rows streamed once per group of up to 16 of its tokens.

        The prefill of ``blockffn.py:171-176, 220-229`` / ``router.py:158-166`` (per-expert dequantize
        and matmul) with the same results as the per-token layer; MXFP4 experts only.  The workspace
        is allocated on the first call for a larger T (outside any graph capture).
        """
        if x.dtype != torch.float32 or not x.is_contiguous() or x.dim() != 2:
            raise TypeError("x must be a contiguous (T, H) float32 tensor")
        T = x.shape[0]
        if out is None:
            out = torch.empty_like(x)
        p = self._params(T, x, out, add_residual, ids, weights)
        n = C.c_size_t(0)
        _lib.call("ns_moe_prefill_workspace_bytes", C.byref(p), C.byref(n))
        if self._pf_ws is None or self._pf_ws.numel() < n.value + 256:
            self._pf_ws = torch.empty(n.value + 256, device=self.device, dtype=torch.uint8)
        ptr = self._pf_ws.data_ptr() + (-self._pf_ws.data_ptr()) % 256
        _lib.call("ns_moe_prefill_grouped", C.byref(p), ptr, n.value, stream_of(x))
        return out

    def prefill(self, x: torch.Tensor, out: torch.Tensor | None = None, add_residual: bool = True,
                ids: torch.Tensor | None = None, weights: torch.Tensor | None = None) -> torch.Tensor:
        """Any number of token rows (prefill, T > max_tokens): the fused layer on successive slices
        of ``max_tokens`` rows, stream-ordered, no host synchronisation.

        Tokens are independent through RMSNorm, routing, the experts and the combine, so the slices
        give exactly the rows of one T-row call.  Each slice streams the experts its tokens route
        to, so an expert shared by several slices is read once per slice: the prefill of
        ``blockffn.py:171-176`` / ``router.py:158-166`` without a grouped GEMM.
        """
        if x.dtype != torch.float32 or not x.is_contiguous() or x.dim() != 2:
            raise TypeError("x must be a contiguous (T, H) float32 tensor")
        T = x.shape[0]
        if out is None:
            out = torch.empty_like(x)
        # MXFP4: slices of 2 rows on the tensor-core layer kernel.  Other types run on the CUDA-core
        # layer kernel, whose one-row launches measured faster per token than wider ones (Qwen3-235B
        # shape, Q4_K: 119 us for one row, 370 us for two).  A slice the library refuses is halved
        # once and for all.
        size = self._slice or (min(2, self.max_tokens) if self.t == GGMLType.MXFP4 else 1)
        t0 = 0
        while t0 < T:
            t1 = min(T, t0 + size)
            try:
                self(x[t0:t1], out=out[t0:t1], add_residual=add_residual,
                     ids=None if ids is None else ids[t0:t1], weights=None if weights is None else weights[t0:t1])
            except _lib.NsError as e:
                if e.status != -2 or t0 > 0 or size == 1:
                    raise
                size //= 2
                continue
            self._slice = size
            t0 = t1
        return out


# ----------------------------------------------------------------------------- reference-facing drop-ins

_ORIGINALS: dict = {}   # filled by nurostream_b200.install


def _vram_payload(cache, name):
    """(device bytes, type) of a VRAM-Q resident tensor, else None (never uploads host bytes).

    Called on every layer call, like the reference's own ``_linear`` calls ``raw_quantized`` per
    projection (``neurostream/model/qwen3.py:176-180``): the lookup refreshes the tensor's LRU position
    and counts a VRAM hit (``neurostream/residency/cache.py:411-420``), so eviction sees hot expert
    slabs as hot, and an evicted tensor is simply no longer found.
    """
    vram = getattr(cache, "_vram", None)
    if vram is None or name not in vram:
        return None
    hit = cache.raw_quantized(name)
    if hit is None or not hit[0].is_cuda:
        return None
    return hit


class DeferredRouterStats:
    """``router_stats`` whose expert counts arrive from the device without stalling the host.

    The reference's ``RouterStats`` (``neurostream/moe/router.py:27-56``) is updated inside every MoE
    call with host-side ids, which costs one device->host synchronisation per layer.  Here each fused
    layer call queues a non-blocking copy of its (T, k) ids into pinned host memory behind an event;
    finished copies are folded into the counters at the next call (``event.query()``, no wait), and
    every read of ``hits`` / ``tokens_routed`` / ``expert_reads`` (``pin_hot_experts``,
    ``speculative_prefetch``, ``summary``) first folds everything still pending, waiting only for
    copies not yet done.  The counts are the reference's: per layer call ``tokens_routed += T``, and
    per distinct expert e ``hits[(layer, e)] += rows routed to e`` and ``expert_reads += 1``.
    """

    MAX_PENDING = 4096

    def __init__(self, base=None):
        if base is None:
            try:
                from neurostream.moe.router import RouterStats as RefStats  # the reference's own class
                base = RefStats()
            except Exception:
                base = RouterStats()
        object.__setattr__(self, "_base", base)
        object.__setattr__(self, "_pending", [])

    # -- queueing (fused path)
    def defer(self, layer: int, ids: torch.Tensor) -> None:
        host = torch.empty(ids.shape, dtype=ids.dtype, pin_memory=True)
        host.copy_(ids, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(ids.device))
        self._pending.append((layer, host, ev))
        self.poll()

    def poll(self, wait: bool = False) -> None:
        pend = self._pending
        n = 0
        while n < len(pend):
            layer, host, ev = pend[n]
            if not (wait or len(pend) - n > self.MAX_PENDING or ev.query()):
                break
            ev.synchronize()
            self._fold(layer, host.numpy())
            n += 1
        del pend[:n]

    def _fold(self, layer, ids) -> None:
        b = self._base
        b.tokens_routed += int(ids.shape[0])
        for e in sorted(set(ids.reshape(-1).tolist())):
            b.hits[(layer, int(e))] += int((ids == e).any(axis=-1).sum())
            b.expert_reads += 1

    # -- the RouterStats surface
    def __getattr__(self, name):
        if name in ("hits", "tokens_routed", "expert_reads"):
            self.poll(wait=True)
        return getattr(self._base, name)

    def __setattr__(self, name, value):
        if name in ("hits", "tokens_routed", "expert_reads"):
            self.poll(wait=True)
        setattr(self._base, name, value)

    def top_experts(self, layer: int, k: int = 8):
        self.poll(wait=True)
        return self._base.top_experts(layer, k)

    def skew(self) -> float:
        self.poll(wait=True)
        return self._base.skew()

    def summary(self) -> str:
        self.poll(wait=True)
        return self._base.summary()


def _stats(model) -> DeferredRouterStats:
    stats = getattr(model, "router_stats", None)
    if not isinstance(stats, DeferredRouterStats):
        stats = DeferredRouterStats(stats)
        model.router_stats = stats
    return stats


def _lookup(model, layer: int, gptoss: bool):
    """This call's tensors of ``layer`` from the cache, in the order the reference touches them.

    The reference's neuron-block ``_ffn_block`` reads, per call: the norm weight, the router weight
    and bias, then per routed expert gate rows, gate bias, up rows, up bias, down rows, down bias
    (``neurostream/model/gpt_oss.py:123-170``, ``neurostream/compute/blockffn.py:434-449``).  Each
    lookup refreshes that tensor's LRU position in the cache, so the fused path leaves the cache's
    eviction order as the reference leaves it.  Returns (expert hits or None, small tensors).
    """
    p = f"blk.{layer}."
    small = {}
    if gptoss:
        small["norm_w"] = model.w(p + "post_attention_norm.weight")
    small["router_w"] = model.w(p + "ffn_gate_inp.weight")
    if gptoss:
        small["router_b"] = model.w(p + "ffn_gate_inp.bias")
    hits = []
    for kind in ("gate", "up", "down"):
        hits.append(_vram_payload(model.cache, p + f"ffn_{kind}_exps.weight"))
        if gptoss:
            small[f"{kind}_b"] = model.w(p + f"ffn_{kind}_exps.bias")
    if any(h is None for h in hits) or len({int(h[1]) for h in hits}) != 1:
        return None, small
    return hits, small


def _layer_for(model, layer: int, gptoss: bool) -> MoeLayer | None:
    """The fused layer of ``layer``, bound to this call's VRAM-Q expert bytes, or None.

    The tensors are looked up in the cache on every call (``_lookup``) and the MoeLayer is rebound
    to them: between calls it keeps only converted copies of the small tensors and its workspace,
    never the expert bytes, so an eviction frees them and the next call falls back to the
    reference's streaming path.  Nothing is cached for a layer that is not resident.
    """
    c = model.cfg
    hits, small = _lookup(model, layer, gptoss)
    if hits is None:
        return None
    t = GGMLType(int(hits[0][1]))
    if t not in MOE_TYPES:
        return None
    cache = getattr(model, "_ns_layers", None)
    if cache is None:
        cache = model._ns_layers = {}
    lay = cache.get(layer)
    if lay is not None and lay.t == t:
        try:
            lay.bind(hits[0][0], hits[1][0], hits[2][0])
            lay.bind_small(**small)
            return lay
        except ValueError:
            cache.pop(layer, None)
    kw = dict(small)
    if gptoss:
        kw.update(rms_eps=c.rms_eps, route_mode=_lib.NS_ROUTE_TOPK_SOFTMAX, act_mode=_lib.NS_ACT_CLAMPED_SWIGLU)
    else:
        kw.update(route_mode=_lib.NS_ROUTE_SOFTMAX_TOPK_NORM, act_mode=_lib.NS_ACT_SILU_MUL)
    try:
        lay = MoeLayer(H=c.n_embd, F=c.n_ffn_expert, n_expert=c.n_expert, k=c.n_expert_used,
                       ggml_type=t, gate=hits[0][0], up=hits[1][0], down=hits[2][0],
                       max_tokens=_lib.NS_MAX_TOKENS, **kw)
    except (_lib.NsError, ValueError):
        return None
    cache[layer] = lay
    return lay


def _run_fused(model, layer_obj: MoeLayer, x: torch.Tensor, layer: int, add_residual: bool):
    T = x.shape[0]
    xf = x.to(torch.float32).contiguous()
    ids = torch.empty((T, layer_obj.k), device=x.device, dtype=torch.int32)
    try:
        out = layer_obj.prefill(xf, add_residual=add_residual, ids=ids)
    except _lib.NsError as e:
        if e.status == -2:  # shape outside the fused kernel: use the streaming path
            return None
        raise
    finally:
        layer_obj.release_weights()
    _stats(model).defer(layer, ids)
    return out.to(x.dtype)


def gptoss_route(model, h: torch.Tensor, layer: int):
    """Drop-in for ``GptOssModel._route``: (chosen list, ids (T,k), weights (T,k)).

    The reference's contract returns the chosen experts as a Python list, which needs the ids on the
    host; the fused ``_ffn_block`` does not call this.
    """
    p = f"blk.{layer}."
    if not h.is_cuda:
        return _ORIGINALS["gptoss_route"](model, h, layer)
    ids, w, _ = route(h, model.w(p + "ffn_gate_inp.weight"), model.w(p + "ffn_gate_inp.bias"),
                      model.cfg.n_expert_used, _lib.NS_ROUTE_TOPK_SOFTMAX)
    return torch.unique(ids).tolist(), ids, w.to(h.dtype)


def gptoss_ffn_block(model, x: torch.Tensor, layer: int):
    """Drop-in for ``GptOssModel._ffn_block``: ``x + MoE(rms_norm(x))``."""
    if x.is_cuda and x.shape[0] >= 1:
        lay = _layer_for(model, layer, gptoss=True)
        if lay is not None:
            out = _run_fused(model, lay, x, layer, add_residual=True)
            if out is not None:
                return out
    return _ORIGINALS["gptoss_ffn_block"](model, x, layer)


def moe_ffn(model, h: torch.Tensor, layer: int) -> torch.Tensor:
    """Drop-in for ``neurostream.moe.router.moe_ffn`` (Qwen3-MoE; returns the MoE output only)."""
    if h.is_cuda and h.shape[0] >= 1:
        lay = _layer_for(model, layer, gptoss=False)
        if lay is not None:
            out = _run_fused(model, lay, h, layer, add_residual=False)
            if out is not None:
                p = f"blk.{layer}."
                if model.has(p + "ffn_gate_shexp.weight"):   # shared expert, as router.py:215-218
                    import torch.nn.functional as F
                    sg = model._linear(p + "ffn_gate_shexp.weight", h)
                    su = model._linear(p + "ffn_up_shexp.weight", h)
                    out = out + model._linear(p + "ffn_down_shexp.weight", F.silu(sg) * su)
                return out
    return _ORIGINALS["moe_ffn"](model, h, layer)
