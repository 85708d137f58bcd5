"""GPT-OSS decode on the B200: one whole token step on device.

``GptOssDecoder`` holds a GPT-OSS model in HBM -- bf16 embedding, attention projections and LM
head, fp32 norms / biases / sinks, MXFP4 expert slabs as GGUF bytes, an fp32 KV cache per layer --
and runs one decode token as the reference's ``GptOssModel.forward`` does
(``neurostream/model/gpt_oss.py:189-228``):

    x = embed(token)
    for each layer:  x = x + o_proj(sink_attention(rope(q), rope(k), v))      (_attention_block)
                     x = x + sum_e w_e expert_e(rms_norm(x))                    (_ffn_block)
    logits = output(rms_norm(x))

with two launches per layer -- ``ns_attn_block`` (RMSNorm, q/k/v, RoPE, KV append, sink attention,
o-proj and residual as one cooperative kernel) and ``ns_moe_decode_layer`` -- plus the embedding and
the LM head, all chained with programmatic dependent launch and captured once into a CUDA graph.
(``fused_attention=False`` runs the attention block as its three separate kernels instead:
``ns_dense_gemv`` q/k/v, ``ns_attn_decode``, ``ns_dense_gemv`` o-proj.)  The token id and its position live in device memory, so the same graph decodes
any token at any position.

Expert parallelism (``world > 1``): rank r holds experts [r*E/world, (r+1)*E/world) of every
layer; everything else is replicated.  Each rank adds its local experts' weighted outputs (rank 0
also the residual) and one sum over the ranks per layer combines them: ``ns_peer_allreduce`` over
NVLink peer memory (``combine="peer"``, the default) or NCCL's all-reduce (``combine="nccl"``).
"""
from __future__ import annotations

import ctypes as C
import math

import torch

from . import _lib, synth
from .decoder import expert_range, synth_moe_layer
from .shapes import GptOssShape


def yarn_tables(shape: GptOssShape, n_pos: int) -> tuple[torch.Tensor, torch.Tensor]:
    """RoPE cos/sin tables (n_pos, head_dim) fp32 for positions 0..n_pos-1, on the host.

    Restates ``yarn_tables`` (``neurostream/model/gpt_oss.py:44-58``) with the same torch CPU
    operations in the same order, so every row equals what the reference computes for that
    position: YaRN frequency interpolation over the untruncated correction range, NeoX half-split
    layout (the frequencies repeated), amplitude 1 + 0.1 ln(factor).
    """
    hd = shape.head_dim
    half = hd // 2
    dims = torch.arange(half, dtype=torch.float32)
    inv = 1.0 / shape.rope_base ** (dims / half)
    factor = shape.rope_factor
    if factor != 1:
        def correction(rotations):
            return hd * math.log(shape.original_context / (rotations * 2 * math.pi)) / (2 * math.log(shape.rope_base))

        low = max(correction(shape.beta_fast), 0)
        high = min(correction(shape.beta_slow), hd - 1)
        ramp = ((dims - low) / (high - low if high != low else 0.001)).clamp(0, 1)
        inv = inv * (1 - ramp) + inv / factor * ramp
    positions = torch.arange(n_pos)
    freqs = positions.float()[:, None] * inv[None, :]
    freqs = torch.cat((freqs, freqs), -1)
    amplitude = 1 + 0.1 * math.log(factor) if factor > 1 else 1.0
    return (freqs.cos() * amplitude).to(torch.float32), (freqs.sin() * amplitude).to(torch.float32)


def _f32(n: int, seed: int, stream: int, sigma: float, dev, start: int = 0) -> torch.Tensor:
    buf = torch.empty(n, dtype=torch.float32, device=dev)
    synth.fill_float(buf, seed, stream, start, sigma)
    return buf


def _bf16(n: int, seed: int, stream: int, sigma: float, dev) -> torch.Tensor:
    buf = torch.empty(n, dtype=torch.bfloat16, device=dev)
    synth.fill_float(buf, seed, stream, 0, sigma)
    return buf


class AttnLayer:
    """One layer's attention block on device: weights, KV cache and the three launches."""

    def __init__(self, shape: GptOssShape, l: int, dev, seed: int, max_ctx: int, ctx: int):
        s = synth.LayerStreams(l)
        H, qd, kvd = shape.n_embd, shape.q_dim, shape.kv_dim
        self.shape, self.l, self.window = shape, l, shape.window(l)
        self.norm_w = _f32(H, seed, s.attn_norm, 0.1, dev) + 1.0
        self.q_w = _bf16(qd * H, seed, s.q_w, 0.02, dev).reshape(qd, H)
        self.k_w = _bf16(kvd * H, seed, s.k_w, 0.02, dev).reshape(kvd, H)
        self.v_w = _bf16(kvd * H, seed, s.v_w, 0.02, dev).reshape(kvd, H)
        self.o_w = _bf16(H * qd, seed, s.o_w, 0.02, dev).reshape(H, qd)
        self.q_b = _f32(qd, seed, s.q_b, 0.02, dev)
        self.k_b = _f32(kvd, seed, s.k_b, 0.02, dev)
        self.v_b = _f32(kvd, seed, s.v_b, 0.02, dev)
        self.o_b = _f32(H, seed, s.o_b, 0.02, dev)
        self.sinks = _f32(shape.n_head, seed, s.sinks, 1.0, dev)
        # fp32 key/value history, (n_kv, max_ctx, hd); positions 0..ctx-1 hold synthetic N(0, 1)
        # values (head g = values [g*ctx*hd, (g+1)*ctx*hd) of the layer's stream)
        self.k_cache = torch.zeros((shape.n_head_kv, max_ctx, shape.head_dim), dtype=torch.float32, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        n = ctx * shape.head_dim
        if n:
            for g in range(shape.n_head_kv):
                synth.fill_float(self.k_cache[g, :ctx].reshape(-1), seed, s.k_cache, g * n, 1.0)
                synth.fill_float(self.v_cache[g, :ctx].reshape(-1), seed, s.v_cache, g * n, 1.0)

    def qkv_params(self, x, qkv) -> _lib.DenseGemvParams:
        sh = self.shape
        p = _lib.DenseGemvParams()
        p.K, p.w_dtype, p.n_seg = sh.n_embd, _lib.NS_BF16, 3
        qd, kvd = sh.q_dim, sh.kv_dim
        outs = (qkv[:qd], qkv[qd:qd + kvd], qkv[qd + kvd:])
        for i, (w, b, y) in enumerate(((self.q_w, self.q_b, outs[0]), (self.k_w, self.k_b, outs[1]),
                                       (self.v_w, self.v_b, outs[2]))):
            p.seg[i].w, p.seg[i].rows, p.seg[i].bias, p.seg[i].residual, p.seg[i].y = (
                w.data_ptr(), w.shape[0], b.data_ptr(), None, y.data_ptr())
        p.x, p.norm_w, p.rms_eps = x.data_ptr(), self.norm_w.data_ptr(), sh.rms_eps
        return p

    def attn_params(self, pos, qkv, rope_cos, rope_sin, out) -> _lib.AttnDecodeParams:
        sh = self.shape
        a = _lib.AttnDecodeParams()
        a.n_head, a.n_head_kv, a.head_dim = sh.n_head, sh.n_head_kv, sh.head_dim
        a.max_ctx, a.window, a.scale = self.k_cache.shape[1], self.window, 1.0 / math.sqrt(sh.head_dim)
        a.pos, a.qkv, a.rope_cos, a.rope_sin = pos.data_ptr(), qkv.data_ptr(), rope_cos.data_ptr(), rope_sin.data_ptr()
        a.sinks, a.k_cache, a.v_cache, a.out = (self.sinks.data_ptr(), self.k_cache.data_ptr(),
                                                self.v_cache.data_ptr(), out.data_ptr())
        return a

    def block_params(self, x, pos, rope_cos, rope_sin, out) -> _lib.AttnBlockParams:
        """Parameters of the whole block as one launch (ns_attn_block): x -> out."""
        sh = self.shape
        b = _lib.AttnBlockParams()
        b.H, b.n_head, b.n_head_kv, b.head_dim = sh.n_embd, sh.n_head, sh.n_head_kv, sh.head_dim
        b.max_ctx, b.window, b.rms_eps, b.scale = self.k_cache.shape[1], self.window, sh.rms_eps, 1.0 / math.sqrt(sh.head_dim)
        b.x, b.norm_w = x.data_ptr(), self.norm_w.data_ptr()
        b.wq, b.wk, b.wv = self.q_w.data_ptr(), self.k_w.data_ptr(), self.v_w.data_ptr()
        b.bq, b.bk, b.bv = self.q_b.data_ptr(), self.k_b.data_ptr(), self.v_b.data_ptr()
        b.wo, b.bo, b.sinks = self.o_w.data_ptr(), self.o_b.data_ptr(), self.sinks.data_ptr()
        b.pos, b.rope_cos, b.rope_sin = pos.data_ptr(), rope_cos.data_ptr(), rope_sin.data_ptr()
        b.k_cache, b.v_cache, b.out = self.k_cache.data_ptr(), self.v_cache.data_ptr(), out.data_ptr()
        return b

    def oproj_params(self, attn_out, residual, y) -> _lib.DenseGemvParams:
        sh = self.shape
        p = _lib.DenseGemvParams()
        p.K, p.w_dtype, p.n_seg = sh.q_dim, _lib.NS_BF16, 1
        p.seg[0].w, p.seg[0].rows, p.seg[0].bias, p.seg[0].residual, p.seg[0].y = (
            self.o_w.data_ptr(), sh.n_embd, self.o_b.data_ptr(), residual.data_ptr(), y.data_ptr())
        p.x, p.norm_w, p.rms_eps = attn_out.data_ptr(), None, 0.0
        return p


class GptOssDecoder:
    """A synthetic GPT-OSS model in HBM, decoding one token per ``step`` (see the module doc).

    shape: the model's dimensions (``GptOssShape``, GPT-OSS-120B by default).
    ctx: positions 0..ctx-1 of every layer's KV cache hold synthetic history; ``max_ctx`` bounds the
    positions a token may take.  Weights are generated in HBM by ``ns_synth_fill``; their host twin is
    ``nurostream_b200.synth`` (token_embd N(0,1), dense weights bf16 N(0, 0.02), biases N(0, 0.02),
    sinks N(0,1), norm weights 1 + 0.1 N(0,1), MXFP4 experts as ``decoder.synth_moe_layer``).
    """

    def __init__(self, shape: GptOssShape | None = None, device="cuda", seed: int = 0, ctx: int = 2048,
                 max_ctx: int | None = None, rank: int = 0, world: int = 1, group=None, use_graph: bool = True,
                 keep_layer_outputs: bool = False, l2_prefetch: bool = False, fused_attention: bool = False,
                 combine: str = "peer"):
        self.shape = shape = shape or GptOssShape()
        self.device = dev = torch.device(device)
        self.seed, self.ctx = seed, ctx
        self.max_ctx = max_ctx or max(ctx + 64, 256)
        if ctx >= self.max_ctx:
            raise ValueError(f"ctx={ctx} leaves no room below max_ctx={self.max_ctx}")
        self.rank, self.world, self.group = rank, world, group
        self.lo, self.hi = expert_range(rank, world, shape.n_expert)
        H, V = shape.n_embd, shape.vocab_size
        ms = synth.ModelStreams
        self.embd = _bf16(V * H, seed, ms.token_embd, 1.0, dev).reshape(V, H)
        self.out_norm = _f32(H, seed, ms.output_norm, 0.1, dev) + 1.0
        self.out_w = _bf16(V * H, seed, ms.output, 0.02, dev).reshape(V, H)
        self.moe_shape = shape.moe_shape(seed=seed)
        self.attn = [AttnLayer(shape, l, dev, seed, self.max_ctx, ctx) for l in range(shape.n_layer)]
        self.moe = [synth_moe_layer(self.moe_shape, l, dev, self.lo, self.hi) for l in range(shape.n_layer)]
        cos, sin = yarn_tables(shape, self.max_ctx)
        self.rope_cos, self.rope_sin = cos.to(dev), sin.to(dev)
        # device state of one step
        self.token = torch.zeros(1, dtype=torch.int32, device=dev)
        self.pos = torch.full((1,), ctx, dtype=torch.int32, device=dev)
        nbuf = shape.n_layer + 1 if keep_layer_outputs else 2
        self.xs = [torch.zeros(H, dtype=torch.float32, device=dev) for _ in range(nbuf)]
        self.xa = [torch.zeros(H, dtype=torch.float32, device=dev) for _ in range(shape.n_layer if keep_layer_outputs else 1)]
        self.qkv = torch.zeros(shape.q_dim + 2 * shape.kv_dim, dtype=torch.float32, device=dev)
        self.attn_out = torch.zeros(shape.q_dim, dtype=torch.float32, device=dev)
        self.logits = torch.zeros(V, dtype=torch.float32, device=dev)
        self.ids = torch.zeros((shape.n_layer, shape.n_expert_used), dtype=torch.int32, device=dev)
        n = C.c_size_t(0)
        _lib.call("ns_attn_workspace_bytes", C.byref(self.attn[0].attn_params(self.pos, self.qkv, self.rope_cos,
                                                                             self.rope_sin, self.attn_out)),
                  C.byref(n))
        # sliding and full layers plan different split counts: size for the larger
        n2 = C.c_size_t(0)
        _lib.call("ns_attn_workspace_bytes", C.byref(self.attn[min(1, shape.n_layer - 1)].attn_params(
            self.pos, self.qkv, self.rope_cos, self.rope_sin, self.attn_out)), C.byref(n2))
        self.attn_ws_bytes = max(n.value, n2.value)
        self.attn_ws = torch.zeros(self.attn_ws_bytes + 256, dtype=torch.uint8, device=dev)
        self._attn_ws_ptr = self.attn_ws.data_ptr() + (-self.attn_ws.data_ptr()) % 256
        self.l2_prefetch = l2_prefetch
        self.fused_attention = fused_attention
        self._build_params()
        self.graph = None
        self.use_graph = use_graph
        self.launches_per_step = 2 + (2 if fused_attention else 4) * shape.n_layer
        self.peer = None
        if world > 1 and combine == "peer":
            from .peer import PeerReduce
            self.peer = PeerReduce(H, group, dev)
            self.launches_per_step += shape.n_layer

    # ------------------------------------------------------------------ launches of one step

    def _build_params(self):
        """ctypes parameter blocks of every launch, built once (the pointers never change).

        L2 prefetch hints chain the weight stream across kernels: the MoE block of layer l asks
        L2 for layer l+1's q/k/v weights (the last layer for the head of the LM head) while it
        routes, and the attention kernel of layer l for the o-proj weights that follow it; HBM
        then works while those kernels are latency-bound, and the dense kernels find their
        weights in L2.
        """
        sh = self.shape
        for l in range(sh.n_layer):
            if not self.l2_prefetch:
                self.moe[l].l2_prefetch = []
            elif l + 1 < sh.n_layer:
                nxt = self.attn[l + 1]
                self.moe[l].l2_prefetch = [nxt.q_w, nxt.k_w, nxt.v_w]
            else:
                self.moe[l].l2_prefetch = [self.out_w.view(-1)[: 32 << 20]]
        self._p = []
        self._blk = []
        cur = self.xs[0]
        for l in range(sh.n_layer):
            A = self.attn[l]
            xa = self.xa[l % len(self.xa)]
            nxt = self.xs[(l + 1) % len(self.xs)]
            pa = A.attn_params(self.pos, self.qkv, self.rope_cos, self.rope_sin, self.attn_out)
            if self.l2_prefetch:
                pa.l2.set([A.o_w])
            self._p.append((A.qkv_params(cur, self.qkv), pa, A.oproj_params(self.attn_out, cur, xa), xa, nxt))
            self._blk.append(A.block_params(cur, self.pos, self.rope_cos, self.rope_sin, xa))
            cur = nxt
        n = C.c_size_t(0)
        if self.fused_attention:
            ws = 0
            for b in self._blk:
                _lib.call("ns_attn_block_workspace_bytes", C.byref(b), C.byref(n))
                ws = max(ws, n.value)
            self.block_ws = torch.zeros(ws + 256, dtype=torch.uint8, device=self.device)
            self._block_ws_ptr = self.block_ws.data_ptr() + (-self.block_ws.data_ptr()) % 256
            self._block_ws_bytes = ws
        self.x_final = cur
        head = _lib.DenseGemvParams()
        head.K, head.w_dtype, head.n_seg = sh.n_embd, _lib.NS_BF16, 1
        head.seg[0].w, head.seg[0].rows, head.seg[0].bias, head.seg[0].residual, head.seg[0].y = (
            self.out_w.data_ptr(), sh.vocab_size, None, None, self.logits.data_ptr())
        head.x, head.norm_w, head.rms_eps = cur.data_ptr(), self.out_norm.data_ptr(), sh.rms_eps
        self._head = head

    def _run(self) -> torch.Tensor:
        stream = torch.cuda.current_stream(self.device).cuda_stream
        sh = self.shape
        _lib.call("ns_embed", self.embd.data_ptr(), _lib.NS_BF16, sh.vocab_size, sh.n_embd, self.token.data_ptr(),
                  self.xs[0].data_ptr(), stream)
        for l, (pq, pa, po, xa, nxt) in enumerate(self._p):
            if self.fused_attention:
                _lib.call("ns_attn_block", C.byref(self._blk[l]), self._block_ws_ptr, self._block_ws_bytes, stream)
            else:
                _lib.call("ns_dense_gemv", C.byref(pq), stream)
                _lib.call("ns_attn_decode", C.byref(pa), self._attn_ws_ptr, self.attn_ws_bytes, stream)
                _lib.call("ns_dense_gemv", C.byref(po), stream)
            self.moe[l](xa.view(1, -1), out=nxt.view(1, -1), add_residual=(self.rank == 0), ids=self.ids[l:l + 1])
            if self.peer is not None:
                self.peer(nxt)
            elif self.world > 1:
                torch.distributed.all_reduce(nxt, group=self.group)
        _lib.call("ns_dense_gemv", C.byref(self._head), stream)
        return self.logits

    def capture(self) -> bool:
        """Capture one step into a CUDA graph (False if capture is refused)."""
        if not self.use_graph:
            return False
        torch.cuda.synchronize(self.device)
        self._run()                      # outside capture: NCCL communicator, kernel attributes
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(g):
                self._run()
        except Exception:
            self.graph = None
            torch.cuda.synchronize(self.device)
            return False
        self.graph = g
        return True

    def step(self) -> torch.Tensor:
        """One token (self.token at self.pos, both on device) through the model; returns the logits."""
        if self.graph is not None:
            self.graph.replay()
            return self.logits
        return self._run()

    def set_token(self, token: int, pos: int | None = None) -> None:
        """Set the next step's token (and position) from the host (stream-ordered copies)."""
        self.token.fill_(int(token))
        if pos is not None:
            if not 0 <= pos < self.max_ctx:
                raise ValueError(f"position {pos} outside 0..{self.max_ctx - 1}")
            self.pos.fill_(int(pos))

    def decode(self, token_host: torch.Tensor, logits_host: torch.Tensor | None = None,
               pos_host: torch.Tensor | None = None) -> torch.Tensor:
        """End to end from host memory: token id (and position) in, logits out (pinned int32 / fp32)."""
        self.token.copy_(token_host, non_blocking=True)
        if pos_host is not None:
            self.pos.copy_(pos_host, non_blocking=True)
        y = self.step()
        if logits_host is None:
            logits_host = torch.empty(y.shape, dtype=y.dtype, pin_memory=True)
        logits_host.copy_(y, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return logits_host

    def release(self) -> None:
        """Drop the graph (it may hold NCCL work) and the peer areas before the process group goes away."""
        self.graph = None
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def check_device_errors(self) -> None:
        bits = _lib.device_error()
        if bits:
            raise RuntimeError(f"device error bits {bits:#x} (bounded wait ran out)")

    def bytes_per_token(self) -> dict:
        """Algorithmic bytes one decode token reads and writes, by part (the roofline numerator)."""
        sh = self.shape
        H, V, hd, nkv = sh.n_embd, sh.vocab_size, sh.head_dim, sh.n_head_kv
        pos = int(self.pos.item()) if self.pos.is_cuda else self.ctx
        kv = 0
        for l in range(sh.n_layer):
            w = sh.window(l)
            keys = min(pos + 1, w) if w else pos + 1
            kv += 2 * nkv * (keys - 1) * hd * 4 + 2 * nkv * hd * 4   # history read + the new slot written
        moe = sh.n_layer * self.moe_shape.layer_bytes_per_token()
        attn = sh.n_layer * (sh.attn_weight_bytes() + 4 * (2 * H + (sh.q_dim + 2 * sh.kv_dim) + sh.q_dim) * 2)
        head = V * H * 2 + H * 4 + V * 4
        return {"experts+router": moe, "attention weights": attn, "kv": kv, "lm_head": head + H * 2,
                "total": moe + attn + kv + head + H * 2}
