"""ctypes binding of libns_b200.so (the C ABI in include/ns_b200.h).

There is no CPU fallback: if the library is missing or a call fails, the
caller gets an exception.  Loading happens after torch (when torch is
imported) so that both share one CUDA runtime.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libns_b200.so"
HEADER = PKG.parent / "include" / "ns_b200.h"

NS_OK = 0
ABI_VERSION = 2
NS_L2_PREFETCH_RANGES = 4
NS_F32, NS_F16, NS_BF16 = 0, 1, 2
NS_ROUTE_TOPK_SOFTMAX, NS_ROUTE_SOFTMAX_TOPK_NORM = 0, 1
NS_ACT_CLAMPED_SWIGLU, NS_ACT_SILU_MUL = 0, 1
NS_SYNTH_F32, NS_SYNTH_BF16 = 1000, 1001
NS_MAX_TOKENS, NS_MAX_TOPK, NS_MAX_EXPERTS = 8, 16, 512
NS_MOE_STATIC_SCRATCH_BYTES = 1024 * 1024
DEVERR_GRID_WAIT, DEVERR_COPY_WAIT, DEVERR_ROUTE = 1, 2, 4

_STATUS = {-1: "invalid argument", -2: "unsupported", -3: "buffer too small", -4: "CUDA error", -5: "timeout"}


class NsError(RuntimeError):
    """A failed ns_b200 call; ``status`` is the negative ns_status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{message} [{_STATUS.get(status, status)}]")
        self.status = status


class L2Prefetch(C.Structure):
    """Mirror of ns_l2_prefetch_t."""

    _fields_ = [("ptr", C.c_void_p * NS_L2_PREFETCH_RANGES), ("bytes", C.c_uint64 * NS_L2_PREFETCH_RANGES)]

    def set(self, tensors) -> "L2Prefetch":
        """Prefetch these tensors' bytes (at most NS_L2_PREFETCH_RANGES)."""
        for i, t in enumerate(list(tensors)[:NS_L2_PREFETCH_RANGES]):
            self.ptr[i] = t.data_ptr()
            self.bytes[i] = t.numel() * t.element_size()
        return self


class MoeLayerParams(C.Structure):
    """Mirror of ns_moe_layer_t."""

    _fields_ = [
        ("T", C.c_int), ("H", C.c_int), ("F", C.c_int), ("n_expert", C.c_int),
        ("expert_lo", C.c_int), ("expert_hi", C.c_int), ("k", C.c_int),
        ("route_mode", C.c_int), ("act_mode", C.c_int), ("ggml_type", C.c_int),
        ("alpha", C.c_float), ("limit", C.c_float), ("rms_eps", C.c_float),
        ("add_residual", C.c_int),
        ("x", C.c_void_p), ("norm_w", C.c_void_p),
        ("router_w", C.c_void_p), ("router_dtype", C.c_int), ("router_b", C.c_void_p),
        ("gate_w", C.c_void_p), ("up_w", C.c_void_p), ("down_w", C.c_void_p),
        ("gate_b", C.c_void_p), ("up_b", C.c_void_p), ("down_b", C.c_void_p),
        ("out", C.c_void_p), ("ids", C.c_void_p), ("weights", C.c_void_p), ("l2", L2Prefetch),
    ]


NS_DENSE_MAX_SEG = 4


class DenseSeg(C.Structure):
    """Mirror of ns_dense_seg_t."""

    _fields_ = [("w", C.c_void_p), ("rows", C.c_int), ("bias", C.c_void_p), ("residual", C.c_void_p),
                ("y", C.c_void_p)]


class DenseGemvParams(C.Structure):
    """Mirror of ns_dense_gemv_t."""

    _fields_ = [("K", C.c_int), ("w_dtype", C.c_int), ("n_seg", C.c_int), ("seg", DenseSeg * NS_DENSE_MAX_SEG),
                ("x", C.c_void_p), ("norm_w", C.c_void_p), ("rms_eps", C.c_float), ("l2", L2Prefetch)]


class AttnDecodeParams(C.Structure):
    """Mirror of ns_attn_decode_t."""

    _fields_ = [("n_head", C.c_int), ("n_head_kv", C.c_int), ("head_dim", C.c_int), ("max_ctx", C.c_int),
                ("window", C.c_int), ("scale", C.c_float), ("pos", C.c_void_p), ("qkv", C.c_void_p),
                ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p), ("sinks", C.c_void_p),
                ("k_cache", C.c_void_p), ("v_cache", C.c_void_p), ("out", C.c_void_p), ("l2", L2Prefetch)]


class AttnBlockParams(C.Structure):
    """Mirror of ns_attn_block_t."""

    _fields_ = [("H", C.c_int), ("n_head", C.c_int), ("n_head_kv", C.c_int), ("head_dim", C.c_int),
                ("max_ctx", C.c_int), ("window", C.c_int), ("rms_eps", C.c_float), ("scale", C.c_float),
                ("x", C.c_void_p), ("norm_w", C.c_void_p), ("wq", C.c_void_p), ("wk", C.c_void_p),
                ("wv", C.c_void_p), ("bq", C.c_void_p), ("bk", C.c_void_p), ("bv", C.c_void_p),
                ("wo", C.c_void_p), ("bo", C.c_void_p), ("sinks", C.c_void_p), ("pos", C.c_void_p),
                ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p), ("k_cache", C.c_void_p),
                ("v_cache", C.c_void_p), ("out", C.c_void_p)]


NS_MAX_PEERS, NS_PEER_MAX_CTAS = 8, 32


class PeerReduceParams(C.Structure):
    """Mirror of ns_peer_reduce_t."""

    _fields_ = [("world", C.c_int), ("rank", C.c_int), ("n", C.c_int64), ("cap", C.c_int64), ("data", C.c_void_p),
                ("slots", C.c_void_p * NS_MAX_PEERS), ("ctr", C.c_void_p)]


_P, _I, _I64, _U64, _SZ, _F = C.c_void_p, C.c_int, C.c_int64, C.c_uint64, C.c_size_t, C.c_float

SIGNATURES = {
    "ns_last_error": (C.c_char_p, []),
    "ns_abi_version": (_I, []),
    "ns_type_layout": (_I, [_I, C.POINTER(_I), C.POINTER(_I)]),
    "ns_device_error": (_I, [C.POINTER(C.c_uint32), _I]),
    "ns_dequant": (_I, [_P, _SZ, _I, _I64, _P, _I, _P]),
    "ns_gemv": (_I, [_P, _SZ, _I, _I, _I, _P, _I, _I64, _I, _P, _I, _I64, _P]),
    "ns_moe_route": (_I, [_P, _I, _I, _I, _P, _I, _P, _I, _I, _I, _P, _P, _P, _P]),
    "ns_moe_workspace_bytes": (_I, [C.POINTER(MoeLayerParams), C.POINTER(_SZ)]),
    "ns_moe_workspace_init": (_I, [_P, _SZ, _P]),
    "ns_moe_decode_layer": (_I, [C.POINTER(MoeLayerParams), _P, _SZ, _P]),
    "ns_moe_decode_layer_static": (_I, [C.POINTER(MoeLayerParams), _P]),
    "ns_moe_prefill_workspace_bytes": (_I, [C.POINTER(MoeLayerParams), C.POINTER(_SZ)]),
    "ns_moe_prefill_grouped": (_I, [C.POINTER(MoeLayerParams), _P, _SZ, _P]),
    "ns_peer_allreduce": (_I, [C.POINTER(PeerReduceParams), _P]),
    "ns_peer_alloc": (_I, [_SZ, C.POINTER(C.c_void_p)]),
    "ns_peer_free": (_I, [_P]),
    "ns_ipc_handle": (_I, [_P, C.c_char_p]),
    "ns_ipc_open": (_I, [C.c_char_p, C.POINTER(C.c_void_p)]),
    "ns_ipc_close": (_I, [_P]),
    "ns_synth_fill": (_I, [_P, _U64, _I, _U64, _U64, _U64, _F, _I, _I, _F, _P]),
    "ns_moe_set_trace": (_I, [_P, _SZ]),
    "ns_moe_select_kernel": (_I, [_I]),
    "ns_dense_gemv": (_I, [C.POINTER(DenseGemvParams), _P]),
    "ns_attn_workspace_bytes": (_I, [C.POINTER(AttnDecodeParams), C.POINTER(_SZ)]),
    "ns_attn_decode": (_I, [C.POINTER(AttnDecodeParams), _P, _SZ, _P]),
    "ns_embed": (_I, [_P, _I, _I64, _I, _P, _P, _P]),
    "ns_attn_block_workspace_bytes": (_I, [C.POINTER(AttnBlockParams), C.POINTER(_SZ)]),
    "ns_attn_block": (_I, [C.POINTER(AttnBlockParams), _P, _SZ, _P]),
}

_lib = None


def load(path: Path | str | None = None) -> C.CDLL:
    """Load libns_b200.so (once); raises if it is absent or out of ABI version."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"{p} is missing: build it with `python -m nurostream_b200.build` "
            "(the decode path has no CPU fallback)"
        )
    try:
        import torch  # noqa: F401  -- load torch's CUDA runtime first so both share it
    except ImportError:
        pass
    lib = C.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.ns_abi_version() != ABI_VERSION:
        raise RuntimeError(f"{p}: ABI version {lib.ns_abi_version()} != {ABI_VERSION}")
    if path is None:
        _lib = lib
    return lib


def check(status: int) -> None:
    if status != NS_OK:
        raise NsError(status, load().ns_last_error().decode(errors="replace"))


def call(name: str, *args) -> None:
    """Call an ns_* entry point and raise NsError on a negative status."""
    check(getattr(load(), name)(*args))


def device_error(clear: bool = True) -> int:
    """Error bits raised by kernels on the current device (synchronises)."""
    v = C.c_uint32(0)
    call("ns_device_error", C.byref(v), 1 if clear else 0)
    return int(v.value)


def header_symbols() -> list[str]:
    """Function names declared in include/ns_b200.h."""
    import re

    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\**(ns_\w+)\s*\(", text, re.M)))
