"""B200-native (sm_100a) decode hot path of neurostream.

Fused dequant-GEMV straight from GGUF bytes (MXFP4, Q8_0, Q4_K, Q5_K, Q6_K, Q4_0), the MoE decode
step around it (router top-k/softmax, gate/up activation, down, weighted combine) and the rest of
a GPT-OSS decode token (bf16 projections, attention with sinks, LM head) as hand-written CUDA behind
a C ABI (include/ns_b200.h), with Python mirrors of the reference's operators on top:

* ``nurostream_b200.fused``   -- can_fuse / fused_gemv / dequantize
* ``nurostream_b200.moe``     -- route, MoeLayer, the GPT-OSS / Qwen3 MoE drop-ins
* ``nurostream_b200.gptoss``  -- GptOssDecoder: a whole decode token in one CUDA graph
* ``nurostream_b200.install`` -- patch an importable reference package in place

Importing the package loads no native code; the library is loaded on first use.
"""
from .ggml import GGMLType, TYPE_LAYOUT, row_bytes  # noqa: F401
# bound eagerly: importing the submodule of the same name later must not replace the function
from .install import install  # noqa: F401

__version__ = "0.2.0"
