"""GPT-OSS-shaped MoE decode stack on device (the benchmark and EP harness).

A ``MoeDecoder`` holds ``n_layer`` MoE layers of one model shape with seeded
synthetic weights generated directly in HBM (``nurostream_b200.synth``): the
stacked MXFP4 expert slabs, a bf16 router with fp32 bias, fp32 expert biases
and the post-attention RMSNorm weight.  ``step`` runs one decode token through
every layer (x <- layer(x)); ``decode`` does the same from and to host memory.
Per-token launches are captured once into a CUDA graph.

Expert parallelism (``world > 1``): rank r holds experts
[r*E/world, (r+1)*E/world) of every layer -- a contiguous row window of each
stacked tensor -- and dense state is replicated.  Every rank computes the
identical router; each adds its local experts' weighted outputs (rank 0 also
adds the residual), and one all-reduce(sum) per layer over NCCL combines them.
"""
from __future__ import annotations

import torch

from . import _lib, synth
from .ggml import GGMLType, row_bytes
from .moe import MoeLayer
from .shapes import MoeShape, expert_range  # noqa: F401  (re-exported)


def synth_moe_layer(sh: MoeShape, l: int, dev, lo: int, hi: int, max_tokens: int = 1) -> MoeLayer:
    """MoE layer ``l`` of the synthetic model ``sh``, generated in HBM, holding experts [lo, hi).

    Norm weight 1 + 0.1 N(0,1) and router (``sh.router_dtype``) N(0, 0.02); GPT-OSS adds an fp32
    router bias and fp32 expert biases N(0, ``sh.bias_sigma``).  The host twin of every tensor is
    ``nurostream_b200.synth`` with the same (seed, stream, offset).
    """
    s = synth.LayerStreams(l)
    H, F, E, t = sh.hidden, sh.expert_ffn, sh.n_expert, GGMLType(sh.ggml_type)
    n_local = hi - lo

    def quant(stream, rows, K):
        rb = row_bytes(t, K)
        buf = torch.empty(n_local * rows * rb, dtype=torch.uint8, device=dev)
        synth.fill_quant(buf, t, sh.seed, stream, start=lo * rows * rb)
        return buf

    def flt(n, stream, sigma, dtype=torch.float32, start=0):
        buf = torch.empty(n, dtype=dtype, device=dev)
        synth.fill_float(buf, sh.seed, stream, start, sigma)
        return buf

    norm = flt(H, s.norm_w, 0.1) + 1.0
    if sh.arch == "qwen3":
        # the decoder layer's post-attention RMSNorm feeds moe_ffn (neurostream/model/qwen3.py); the
        # MoE itself has no biases
        return MoeLayer(
            H=H, F=F, n_expert=E, k=sh.top_k, ggml_type=t, norm_w=norm, rms_eps=1e-6,
            router_w=flt(E * H, s.router_w, 0.02, sh.router_dtype).reshape(E, H),
            gate=quant(s.gate, F, H), up=quant(s.up, F, H), down=quant(s.down, H, F),
            expert_lo=lo, expert_hi=hi, max_tokens=max_tokens,
            route_mode=_lib.NS_ROUTE_SOFTMAX_TOPK_NORM, act_mode=_lib.NS_ACT_SILU_MUL,
        )
    return MoeLayer(
        H=H, F=F, n_expert=E, k=sh.top_k, ggml_type=t,
        router_w=flt(E * H, s.router_w, 0.02, sh.router_dtype).reshape(E, H),
        router_b=flt(E, s.router_b, 0.02),
        norm_w=norm,
        gate=quant(s.gate, F, H), up=quant(s.up, F, H), down=quant(s.down, H, F),
        gate_b=flt(n_local * F, s.gate_b, sh.bias_sigma, start=lo * F).reshape(n_local, F),
        up_b=flt(n_local * F, s.up_b, sh.bias_sigma, start=lo * F).reshape(n_local, F),
        down_b=flt(n_local * H, s.down_b, sh.bias_sigma, start=lo * H).reshape(n_local, H),
        expert_lo=lo, expert_hi=hi, rms_eps=1e-5, max_tokens=max_tokens,
    )


class MoeDecoder:
    def __init__(self, shape: MoeShape, device: torch.device | str = "cuda", rank: int = 0, world: int = 1,
                 group=None, use_graph: bool = True, max_tokens: int = 1, keep_layer_outputs: bool = False,
                 batch: int = 1, combine: str = "peer"):
        self.shape = shape
        self.batch = batch            # token rows of one decode step (each layer one fused launch over all)
        max_tokens = max(max_tokens, batch)
        self.max_tokens = max_tokens  # rows per fused launch (prefill runs slices of this many)
        self.device = torch.device(device)
        self.rank, self.world, self.group = rank, world, group
        self.lo, self.hi = expert_range(rank, world, shape.n_expert)
        self.layers = [self._make_layer(l) for l in range(shape.n_layer)]
        H = shape.hidden
        self.x = torch.zeros((batch, H), device=self.device, dtype=torch.float32)
        # two ping-pong output buffers, or one per layer when every layer's output is kept (tests)
        nbuf = shape.n_layer if keep_layer_outputs else 2
        self.bufs = [torch.empty((batch, H), device=self.device, dtype=torch.float32) for _ in range(nbuf)]
        ids_shape = (shape.n_layer, shape.top_k) if batch == 1 else (shape.n_layer, batch, shape.top_k)
        self.ids = torch.zeros(ids_shape, device=self.device, dtype=torch.int32)
        self.out = None
        self.graph = None
        self.use_graph = use_graph
        self.launches_per_step = shape.n_layer
        # expert-parallel combine of the decode step: "peer" (ns_peer_allreduce over NVLink peer
        # memory) or "nccl" (torch.distributed.all_reduce); prefill always uses NCCL
        self.peer = None
        if world > 1 and combine == "peer":
            from .peer import PeerReduce
            self.peer = PeerReduce(batch * H, group, self.device)
            self.launches_per_step = 2 * shape.n_layer

    def _combine(self, t: torch.Tensor) -> None:
        if self.peer is not None:
            self.peer(t)
        else:
            torch.distributed.all_reduce(t, group=self.group)

    def _make_layer(self, l: int) -> MoeLayer:
        return synth_moe_layer(self.shape, l, self.device, self.lo, self.hi, self.max_tokens)

    # ------------------------------------------------------------------ one token

    def _run_layers(self) -> torch.Tensor:
        cur = self.x
        for l, layer in enumerate(self.layers):
            nxt = self.bufs[l % len(self.bufs)]
            if self.batch == 1:
                layer(cur, out=nxt, add_residual=(self.rank == 0), ids=self.ids[l])
            else:  # as many rows per launch as the layer's kernel takes (halved if its activations overflow)
                layer.prefill(cur, out=nxt, add_residual=(self.rank == 0), ids=self.ids[l])
            if self.world > 1:
                self._combine(nxt)
            cur = nxt
        return cur

    def capture(self) -> bool:
        """Capture the per-token launches into a CUDA graph (returns False if capture is refused)."""
        if not self.use_graph:
            return False
        torch.cuda.synchronize(self.device)
        self._run_layers()                       # warm-up outside capture (NCCL communicator, attributes)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(g):
                self.out = self._run_layers()
        except Exception:
            self.graph = None
            torch.cuda.synchronize(self.device)
            return False
        self.graph = g
        return True

    def step(self, x: torch.Tensor | None = None) -> torch.Tensor:
        """One decode step (``batch`` token rows) through all layers; x (batch, H) fp32 on device (copied
        into the input buffer)."""
        if x is not None:
            self.x.copy_(x, non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
            return self.out
        return self._run_layers()

    def decode(self, x_host: torch.Tensor, out_host: torch.Tensor | None = None) -> torch.Tensor:
        """End to end from host memory: copy x in, run every layer, copy the result out."""
        self.x.copy_(x_host, non_blocking=True)
        y = self.step()
        if out_host is None:
            out_host = torch.empty(y.shape, dtype=y.dtype, pin_memory=True)
        out_host.copy_(y, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return out_host

    # ------------------------------------------------------------------ many tokens

    def prefill(self, x: torch.Tensor, bufs: list[torch.Tensor] | None = None, grouped: bool = True) -> torch.Tensor:
        """T tokens (T, H) fp32 on device through every layer; bufs: two (T, H) fp32 ping-pong buffers
        (allocated if None).  grouped: each layer as one grouped expert GEMM
        (``MoeLayer.prefill_grouped``, MXFP4 experts); otherwise, or for other expert types, as slices
        of max_tokens rows through the decode layer kernel (``MoeLayer.prefill``)."""
        if bufs is None:
            bufs = [torch.empty_like(x) for _ in range(2)]
        cur = x
        for l, layer in enumerate(self.layers):
            nxt = bufs[l % 2]
            if grouped and layer.t == GGMLType.MXFP4:
                layer.prefill_grouped(cur, out=nxt, add_residual=(self.rank == 0))
            else:
                layer.prefill(cur, out=nxt, add_residual=(self.rank == 0))
            if self.world > 1:
                torch.distributed.all_reduce(nxt, group=self.group)
            cur = nxt
        return cur

    def release(self) -> None:
        """Drop the graph (it may hold NCCL work) and the peer areas before the process group goes away."""
        self.graph = None
        self.out = None
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def check_device_errors(self) -> None:
        bits = _lib.device_error()
        if bits:
            raise RuntimeError(f"device error bits {bits:#x} (bounded wait ran out)")
