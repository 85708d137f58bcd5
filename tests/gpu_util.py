"""Helpers shared by the GPU parity tests."""
from __future__ import annotations

import numpy as np
import torch

from nurostream_b200 import _lib, synth
from nurostream_b200.ggml import GGMLType, row_bytes
from nurostream_b200.moe import MoeLayer


def assert_rel_close(got, want, tol=1e-3, what=""):
    """max |got - want| <= tol * max |want|, the layer-output criterion (normwise)."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    scale = max(np.abs(want).max(), 1e-30)
    err = np.abs(got - want).max() / scale
    assert err <= tol, f"{what}: max relative error {err:.3e} > {tol:.1e}"
    return err


def device_quant(t, seed, stream, nbytes, start=0):
    buf = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    synth.fill_quant(buf, t, seed, stream, start)
    return buf


def device_float(n, seed, stream, sigma=1.0, dtype=torch.float32):
    buf = torch.empty(n, dtype=dtype, device="cuda")
    synth.fill_float(buf, seed, stream, 0, sigma)
    return buf


def layer_from_synth(L, router_dtype=torch.float32, lo=0, hi=None, max_tokens=None) -> MoeLayer:
    """Device MoeLayer holding the same synthetic tensors as a tests.goldens.SynthLayer."""
    hi = L.E if hi is None else hi
    n_local = hi - lo
    s, seed, t = L.s, L.seed, L.t
    rb_h, rb_f = row_bytes(t, L.H), row_bytes(t, L.F)

    def q(stream, rows_per_expert, rb):
        nbytes = n_local * rows_per_expert * rb
        return device_quant(t, seed, stream, nbytes, start=lo * rows_per_expert * rb)

    gate, up, down = q(s.gate, L.F, rb_h), q(s.up, L.F, rb_h), q(s.down, L.H, rb_f)
    rw = torch.from_numpy(L.router_w).cuda().to(router_dtype)
    kw = {}
    if L.gptoss:
        kw = dict(router_b=torch.from_numpy(L.router_b).cuda(), norm_w=torch.from_numpy(L.norm_w).cuda(),
                  gate_b=torch.from_numpy(L.biases["gate"][lo:hi].copy()).cuda(),
                  up_b=torch.from_numpy(L.biases["up"][lo:hi].copy()).cuda(),
                  down_b=torch.from_numpy(L.biases["down"][lo:hi].copy()).cuda(),
                  route_mode=_lib.NS_ROUTE_TOPK_SOFTMAX, act_mode=_lib.NS_ACT_CLAMPED_SWIGLU)
    else:
        kw = dict(route_mode=_lib.NS_ROUTE_SOFTMAX_TOPK_NORM, act_mode=_lib.NS_ACT_SILU_MUL)
    return MoeLayer(H=L.H, F=L.F, n_expert=L.E, k=L.k, ggml_type=t, router_w=rw, gate=gate, up=up, down=down,
                    expert_lo=lo, expert_hi=hi, max_tokens=max_tokens or L.T, **kw)


def run_layer(layer: MoeLayer, x: np.ndarray, add_residual=True):
    xt = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
    ids = torch.empty((xt.shape[0], layer.k), dtype=torch.int32, device="cuda")
    w = torch.empty((xt.shape[0], layer.k), dtype=torch.float32, device="cuda")
    out = layer(xt, add_residual=add_residual, ids=ids, weights=w)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    return out.cpu().numpy(), ids.cpu().numpy().astype(np.int64), w.cpu().numpy()
