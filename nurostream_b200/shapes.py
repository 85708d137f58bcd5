"""Shapes of the benchmarked MoE stacks, with no dependency on the native library.

``MoeShape`` and ``expert_range`` describe a model's MoE layers and how experts
split over ranks.  They live apart from ``decoder``/``moe`` so that code which
must not map ``libns_b200.so`` (the reference arm of the benchmark, CPU-only
host logic) can use them.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .ggml import GGMLType, row_bytes


@dataclass
class MoeShape:
    n_layer: int = 36
    hidden: int = 2880
    expert_ffn: int = 2880
    n_expert: int = 128
    top_k: int = 4
    ggml_type: int = int(GGMLType.MXFP4)
    router_dtype: torch.dtype = torch.bfloat16
    seed: int = 0
    bias_sigma: float = 0.02
    # "gpt-oss": RMSNorm, biased router, top-k then softmax, clamped SwiGLU, expert biases.
    # "qwen3": no norm or biases, softmax then top-k renormalised, silu(gate) * up.
    arch: str = "gpt-oss"

    @property
    def expert_bytes(self) -> int:
        """Bytes of one expert's gate + up + down matrices."""
        t = GGMLType(self.ggml_type)
        return 2 * self.expert_ffn * row_bytes(t, self.hidden) + self.hidden * row_bytes(t, self.expert_ffn)

    def layer_bytes_per_token(self) -> int:
        """Algorithmic bytes one layer reads/writes for one token (the roofline numerator)."""
        H, F, E, k = self.hidden, self.expert_ffn, self.n_expert, self.top_k
        gptoss = self.arch == "gpt-oss"
        router = E * H * (2 if self.router_dtype == torch.bfloat16 else 4) + (4 * E if gptoss else 0)
        experts = k * self.expert_bytes
        biases = k * 4 * (2 * F + H) if gptoss else 0
        acts = 4 * H * (3 if gptoss else 2)  # x in, norm weight (GPT-OSS), out
        return router + experts + biases + acts


def expert_range(rank: int, world: int, n_expert: int) -> tuple[int, int]:
    """Experts [lo, hi) that rank `rank` of `world` holds: an even, contiguous split by index.

    Each rank's share is one row window of every stacked expert tensor.  Rank 0 also adds the
    residual, so summing the ranks' layer outputs gives the full layer.
    """
    if n_expert % world:
        raise ValueError(f"{n_expert} experts do not split evenly over {world} ranks")
    return rank * n_expert // world, (rank + 1) * n_expert // world


@dataclass
class GptOssShape:
    """A GPT-OSS model's dimensions (GPT-OSS-120B by default): the full-decode workload.

    The field names are the reference's ``GptOssConfig`` fields
    (``neurostream/model/gpt_oss.py:22-41``, ``neurostream/model/qwen3.py:27-47``), so
    ``reference_config()`` can build the reference's own config from them.
    """

    n_layer: int = 36
    n_embd: int = 2880
    n_head: int = 64
    n_head_kv: int = 8
    head_dim: int = 64
    n_ffn: int = 2880
    vocab_size: int = 201088
    rms_eps: float = 1e-5
    rope_base: float = 150000.0
    context_length: int = 131072
    n_expert: int = 128
    n_expert_used: int = 4
    n_ffn_expert: int = 2880
    sliding_window: int = 128
    rope_factor: float = 32.0
    original_context: int = 4096
    beta_fast: float = 32.0
    beta_slow: float = 1.0

    def reference_config(self) -> dict:
        return {f: getattr(self, f) for f in self.__dataclass_fields__}

    @property
    def q_dim(self) -> int:
        return self.n_head * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_head_kv * self.head_dim

    def moe_shape(self, **kw) -> MoeShape:
        return MoeShape(n_layer=self.n_layer, hidden=self.n_embd, expert_ffn=self.n_ffn_expert,
                        n_expert=self.n_expert, top_k=self.n_expert_used, **kw)

    def window(self, layer: int) -> int:
        """Sliding window of ``layer`` (0 = full attention): even layers slide (gpt_oss.py:91-92)."""
        return self.sliding_window if layer % 2 == 0 else 0

    def attn_weight_bytes(self, wbytes: int = 2) -> int:
        """Dense attention weights + biases + sinks + norm of one layer (bf16 weights)."""
        H, q, kv = self.n_embd, self.q_dim, self.kv_dim
        return (q + 2 * kv) * H * wbytes + (q + 2 * kv) * 4 + H * q * wbytes + H * 4 + self.n_head * 4 + H * 4
