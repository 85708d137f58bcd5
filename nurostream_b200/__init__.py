"""B200-native (sm_100a) decode hot path of neurostream.

Fused dequant-GEMV straight from GGUF bytes (MXFP4, Q8_0, Q4_K, Q6_K) and the
MoE decode step around it (router top-k/softmax, gate/up activation, down,
weighted combine) as hand-written CUDA behind a C ABI (include/ns_b200.h),
with Python mirrors of the reference's operators on top:

* ``nurostream_b200.fused``   -- can_fuse / fused_gemv / dequantize
* ``nurostream_b200.moe``     -- route, MoeLayer, the GPT-OSS / Qwen3 MoE drop-ins
* ``nurostream_b200.install`` -- patch an importable reference package in place
"""
from .ggml import GGMLType, TYPE_LAYOUT, row_bytes  # noqa: F401

__version__ = "0.1.0"


def install(package: str = "neurostream"):
    from .install import install as _install
    return _install(package)
