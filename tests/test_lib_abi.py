"""The C-ABI library loads, exports every declared symbol and validates
arguments on the host (no GPU work is launched by these tests)."""
import ctypes as C

import pytest

from nurostream_b200 import _lib
from nurostream_b200.ggml import TYPE_LAYOUT, GGMLType


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


def test_exports_every_header_symbol(lib):
    names = _lib.header_symbols()
    assert len(names) >= 11
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures must cover the header exactly"


def test_abi_version(lib):
    assert lib.ns_abi_version() == _lib.ABI_VERSION == 2


def test_type_layouts_match_gguf(lib):
    for t, (be, bb) in TYPE_LAYOUT.items():
        e, b = C.c_int(0), C.c_int(0)
        assert lib.ns_type_layout(int(t), C.byref(e), C.byref(b)) == 0
        assert (e.value, b.value) == (be, bb), t
    assert lib.ns_type_layout(99, C.byref(C.c_int()), C.byref(C.c_int())) == -2


def _err(lib):
    return lib.ns_last_error().decode()


def test_gemv_rejects_bad_arguments_before_launching(lib):
    # unsupported type (a float type has no fused GEMV, like the reference's _KERNELS)
    assert lib.ns_gemv(1, 512, int(GGMLType.BF16), 1, 256, 1, 0, 256, 1, 1, 0, 1, None) == -2
    assert "no fused GEMV" in _err(lib)
    # T outside 1..8
    assert lib.ns_gemv(1, 4352, int(GGMLType.Q8_0), 1, 4096, 1, 0, 4096, 9, 1, 0, 1, None) == -1
    # K not a whole number of blocks
    assert lib.ns_gemv(1, 4352, int(GGMLType.Q8_0), 1, 4010, 1, 0, 4010, 1, 1, 0, 1, None) == -1
    # buffer too small for n_rows rows
    assert lib.ns_gemv(1, 100, int(GGMLType.MXFP4), 2, 2880, 1, 0, 2880, 1, 1, 0, 2, None) == -3
    assert "weight buffer" in _err(lib)
    # zero rows is a no-op
    assert lib.ns_gemv(None, 0, int(GGMLType.MXFP4), 0, 2880, None, 0, 2880, 1, None, 0, 0, None) == 0


def test_dequant_rejects_bad_arguments(lib):
    assert lib.ns_dequant(1, 17, 7, 32, 1, 0, None) == -2
    assert lib.ns_dequant(1, 17, int(GGMLType.MXFP4), 64, 1, 0, None) == -3
    assert lib.ns_dequant(1, 17, int(GGMLType.MXFP4), 32, 1, 5, None) == -1
    assert lib.ns_dequant(None, 0, int(GGMLType.MXFP4), 0, None, 0, None) == 0


def _params(**kw):
    p = _lib.MoeLayerParams()
    base = dict(T=1, H=2880, F=2880, n_expert=32, expert_lo=0, expert_hi=32, k=4, route_mode=0, act_mode=0,
                ggml_type=int(GGMLType.MXFP4), alpha=1.702, limit=7.0, rms_eps=1e-5, add_residual=1,
                router_dtype=0)
    base.update(kw)
    for k, v in base.items():
        setattr(p, k, v)
    return p


def test_moe_workspace_bytes_and_validation(lib):
    n = C.c_size_t(0)
    assert lib.ns_moe_workspace_bytes(C.byref(_params()), C.byref(n)) == 0
    # MXFP4, T <= 2: the larger of the two kernels' workspaces.  CUDA-core kernel: header
    # (barrier word, activation maxima) + logits (T*E fp32) + activations (T*k*F fp32).
    # Tensor-core kernel: header with counters + logits + split-tile partials (160 SMs x (one gate/up
    # slot of 2T x 128 + one down slot of 128) fp32) + activation image per pair (90 blocks x 128 B of
    # planes, then 23 scale atoms x 128 B, 256-aligned) + down outputs per pair.
    v2 = 1024 + 256 + 4 * 2880 * 4
    tc = 8192 + 256 + 160 * 3 * 128 * 4 + 4 * 14592 + 4 * 2880 * 4
    assert n.value == max(v2, tc)
    assert lib.ns_moe_workspace_bytes(C.byref(_params(ggml_type=int(GGMLType.Q8_0))), C.byref(n)) == 0
    assert n.value == v2
    # sized for up to 8 tokens: also covers the tensor-core kernel's scratch of the 1- and 2-token calls
    n8 = C.c_size_t(0)
    assert lib.ns_moe_workspace_bytes(C.byref(_params(T=8)), C.byref(n8)) == 0
    assert n8.value >= max(v2, tc)
    bad = [dict(T=0), dict(T=9), dict(k=0), dict(k=33), dict(n_expert=600), dict(expert_lo=4, expert_hi=4),
           dict(H=100), dict(route_mode=7), dict(act_mode=3), dict(ggml_type=int(GGMLType.Q5_K)),
           dict(router_dtype=9)]
    for kw in bad:
        assert lib.ns_moe_workspace_bytes(C.byref(_params(**kw)), C.byref(n)) < 0, kw


def test_moe_route_validation(lib):
    assert lib.ns_moe_route(1, 0, 1, 64, 1, 0, None, 4, 5, 0, 1, 1, 1, None) == -1  # k > E
    assert lib.ns_moe_route(1, 0, 1, 64, 1, 0, None, 4, 2, 3, 1, 1, 1, None) == -1  # bad mode


def test_synth_fill_validation(lib):
    assert lib.ns_synth_fill(1, 16, 7, 0, 0, 0, 1.0, 118, 124, 1e-3, None) == -2
    assert lib.ns_synth_fill(1, 16, int(GGMLType.MXFP4), 0, 0, 0, 1.0, 124, 118, 1e-3, None) == -1
    assert lib.ns_synth_fill(None, 0, int(GGMLType.MXFP4), 0, 0, 0, 1.0, 118, 124, 1e-3, None) == 0


def test_errors_raise_with_message():
    with pytest.raises(_lib.NsError, match="no fused GEMV"):
        _lib.call("ns_gemv", 1, 512, int(GGMLType.BF16), 1, 256, 1, 0, 256, 1, 1, 0, 1, None)


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.load(tmp_path / "libns_b200.so")
