"""ns_moe_decode_layer_static: the fused MoE decode layer on the library's
static device scratch (no caller workspace, no allocation), called through the
C ABI and compared with ns_moe_decode_layer on the same layer.

The file is named to be collected last, so that it also runs after every other
test has used the device; it passes alone in a fresh process as well.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from nurostream_b200 import _lib
from tests import goldens
from tests.gpu_util import assert_rel_close, layer_from_synth


def _layer_params(name):
    g = goldens.load("moe")
    c = goldens.cases(g)[name]
    L = goldens.SynthLayer(c)
    layer = layer_from_synth(L)
    x = torch.from_numpy(np.ascontiguousarray(L.x, dtype=np.float32)).cuda()
    return g, L, layer, x


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["gptoss_cfg1", "qwen_q4k_t2"])
def test_static_scratch_matches_workspace_entry_point(name):
    g, L, layer, x = _layer_params(name)
    T, k = x.shape[0], layer.k
    stream = torch.cuda.current_stream().cuda_stream

    # the existing entry point, with the layer's own workspace
    want = torch.empty_like(x)
    want_ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
    p = layer._params(T, x, want, L.gptoss, want_ids, None)
    _lib.call("ns_moe_decode_layer", C.byref(p), layer._ws_ptr, layer._ws_bytes, stream)
    torch.cuda.synchronize()
    want_np = want.cpu().numpy()

    # the allocation-free entry point, twice in a row on one stream
    outs = []
    for _ in range(2):
        out = torch.full_like(x, float("nan"))
        ids = torch.full((T, k), -1, dtype=torch.int32, device="cuda")
        p = layer._params(T, x, out, L.gptoss, ids, None)
        _lib.call("ns_moe_decode_layer_static", C.byref(p), stream)
        outs.append((out, ids))
    torch.cuda.synchronize()
    assert _lib.device_error() == 0

    for i, (out, ids) in enumerate(outs):
        got = out.cpu().numpy()
        assert_rel_close(got, want_np, 1e-3, f"{name} static call {i}")        # the layer-output tolerance
        assert_rel_close(got, g[f"{name}__out"], 1e-3, f"{name} static call {i} vs golden")
        np.testing.assert_array_equal(ids.cpu().numpy(), want_ids.cpu().numpy())


def test_static_scratch_rejects_layers_beyond_its_size():
    """T x k x F activations beyond NS_MOE_STATIC_SCRATCH_BYTES: NS_ERR_SIZE before any device work."""
    p = _lib.MoeLayerParams()
    for f, v in dict(T=8, H=2880, F=2880, n_expert=64, expert_lo=0, expert_hi=64, k=16, route_mode=0,
                     act_mode=0, ggml_type=39, alpha=1.702, limit=7.0, rms_eps=1e-5, add_residual=1,
                     router_dtype=0).items():
        setattr(p, f, v)
    need = C.c_size_t(0)
    _lib.call("ns_moe_workspace_bytes", C.byref(p), C.byref(need))
    assert need.value > _lib.NS_MOE_STATIC_SCRATCH_BYTES
    with pytest.raises(_lib.NsError, match="NS_MOE_STATIC_SCRATCH_BYTES") as e:
        _lib.call("ns_moe_decode_layer_static", C.byref(p), None)
    assert e.value.status == -3


@pytest.mark.gpu
@pytest.mark.parametrize("order", [(1, 3, 1), (3, 1, 3)])
def test_static_scratch_alternates_tensor_core_and_cuda_core_kernels(order):
    """The two layer kernels share the one static array (T <= 2: tensor-core kernel, T = 3: CUDA-core
    kernel); alternating them on it, in either order, matches the workspace entry point each time."""
    c = dict(name="alt", arch="gpt-oss", type=39, E=16, H=512, F=512, k=4, T=3, seed=31, bias=True,
             norm="random", block_rows=512)
    layer = layer_from_synth(goldens.SynthLayer(c), max_tokens=3)
    stream = torch.cuda.current_stream().cuda_stream
    for T in order:
        x = torch.from_numpy(goldens.SynthLayer(dict(c, T=T)).x.copy()).cuda()
        want = torch.empty_like(x)
        p = layer._params(T, x, want, True, None, None)
        _lib.call("ns_moe_decode_layer", C.byref(p), layer._ws_ptr, layer._ws_bytes, stream)
        got = torch.full_like(x, float("nan"))
        p = layer._params(T, x, got, True, None, None)
        _lib.call("ns_moe_decode_layer_static", C.byref(p), stream)
        torch.cuda.synchronize()
        assert _lib.device_error() == 0
        assert_rel_close(got.cpu().numpy(), want.cpu().numpy(), 1e-3, f"static T={T} in order {order}")
