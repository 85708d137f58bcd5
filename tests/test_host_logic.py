"""Host-side logic that runs without a GPU: the synthetic generator, the
drop-in operator surface and the installer."""
import importlib.util
import os
from pathlib import Path
import sys

import numpy as np
import pytest
import torch

from nurostream_b200 import fused, synth
from nurostream_b200.ggml import FUSED_TYPES, GGMLType, TYPE_LAYOUT, row_bytes
from oracle import quant as oquant


@pytest.mark.parametrize("t", [GGMLType.MXFP4, GGMLType.Q8_0, GGMLType.Q4_K, GGMLType.Q6_K, GGMLType.Q5_K,
                               GGMLType.Q4_0])
def test_synth_slices_are_consistent(t):
    whole = synth.quant_bytes(t, 3, 17, 0, 4096)
    for a, b in [(0, 1), (5, 700), (1023, 2049), (4000, 4096)]:
        np.testing.assert_array_equal(synth.quant_bytes(t, 3, 17, a, b - a), whole[a:b])
    assert not np.array_equal(whole, synth.quant_bytes(t, 4, 17, 0, 4096))


def test_synth_distributions():
    be, bb = TYPE_LAYOUT[GGMLType.MXFP4]
    raw = synth.quant_bytes(GGMLType.MXFP4, 0, 1, 0, bb * 2000).reshape(2000, bb)
    assert raw[:, 0].min() == 118 and raw[:, 0].max() == 124
    vals = oquant.dequantize(raw.reshape(-1), GGMLType.MXFP4, 2000 * 32)
    assert np.isfinite(vals).all()
    q8 = synth.quant_bytes(GGMLType.Q8_0, 0, 2, 0, 34 * 1000).reshape(1000, 34)
    d = q8[:, :2].copy().view(np.float16).astype(np.float32).ravel()
    assert (d >= 0.5e-3 * 0.999).all() and (d <= 1.5e-3 * 1.001).all()
    x = synth.float_values(0, 3, 0, 20000)
    assert abs(float(x.mean())) < 0.03 and abs(float(x.std()) - 1.0) < 0.03
    assert np.abs(x).max() <= 6.0
    np.testing.assert_array_equal(synth.float_values(0, 3, 100, 50), x[100:150])
    bf = synth.float_values(0, 3, 0, 100, 0.02, dtype="bf16")
    np.testing.assert_allclose(synth.bf16_to_f32(bf), x[:100] * np.float32(0.02), rtol=2 ** -8)


def test_can_fuse_gates_on_device_and_type():
    x = torch.zeros(1, 64)
    assert not fused.can_fuse(GGMLType.MXFP4, x)            # CPU tensor
    assert not fused.can_fuse(GGMLType.Q5_K, x)
    assert not fused.can_fuse(12345, x)
    assert FUSED_TYPES == {GGMLType.MXFP4, GGMLType.Q8_0, GGMLType.Q4_K, GGMLType.Q6_K, GGMLType.Q5_K,
                           GGMLType.Q4_0}


def test_fused_gemv_errors_like_reference():
    with pytest.raises(KeyError):
        fused.fused_gemv(torch.zeros(512, dtype=torch.uint8), GGMLType.BF16, torch.zeros(1, 256), 1, 256)
    with pytest.raises(TypeError):
        fused.fused_gemv(torch.zeros(17, dtype=torch.uint8), GGMLType.MXFP4, torch.zeros(1, 32), 1, 32)


def test_dequantize_refuses_cpu_tensors():
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        fused.dequantize(torch.zeros(17, dtype=torch.uint8), GGMLType.MXFP4, 32)
    with pytest.raises(TypeError):
        fused.dequantize(torch.zeros(17, dtype=torch.int8), GGMLType.MXFP4, 32)


def test_row_bytes():
    assert row_bytes(GGMLType.MXFP4, 2880) == 1530
    assert row_bytes(GGMLType.Q4_K, 4096) == 2304
    assert row_bytes(GGMLType.Q8_0, 4096) == 4352
    with pytest.raises(ValueError):
        row_bytes(GGMLType.Q4_K, 1000)


# the reference package: NS_REFERENCE_PATH, else the copy installed into baseline/_ref
REF = os.environ.get("NS_REFERENCE_PATH") or str(Path(__file__).resolve().parents[1] / "baseline" / "_ref")


def _reference_importable():
    return os.path.isdir(os.path.join(REF, "neurostream"))


@pytest.mark.skipif(not _reference_importable(), reason="reference package not present on this machine")
def test_install_patches_and_restores_reference(monkeypatch):
    monkeypatch.syspath_prepend(REF)
    monkeypatch.setenv("PYTHONDONTWRITEBYTECODE", "1")
    sys.dont_write_bytecode = True
    import nurostream_b200
    from nurostream_b200 import moe
    import neurostream.compute.triton_kernels as tk
    import neurostream.compute.quant as q
    import neurostream.residency.cache as cache_mod
    import neurostream.model.gpt_oss as go
    import neurostream.moe.router as rt
    originals = (tk.can_fuse, tk.fused_gemv, q.dequantize, cache_mod.dequantize, go.GptOssModel._route,
                 go.GptOssModel._ffn_block, rt.moe_ffn)
    with nurostream_b200.install():
        assert tk.can_fuse is fused.can_fuse and tk.fused_gemv is fused.fused_gemv
        assert rt.moe_ffn is moe.moe_ffn
        assert go.GptOssModel._ffn_block is not originals[5]
        # CPU tensors still take the reference's own path, unchanged
        raw = synth.quant_bytes(GGMLType.Q4_K, 1, 1, 0, 2 * row_bytes(GGMLType.Q4_K, 256))
        got = q.dequantize(torch.from_numpy(raw.copy()), GGMLType.Q4_K, 512)
        np.testing.assert_array_equal(got.numpy(), oquant.dequantize(raw, GGMLType.Q4_K, 512))
        assert not tk.can_fuse(GGMLType.MXFP4, torch.zeros(1, 32))
    assert (tk.can_fuse, tk.fused_gemv, q.dequantize, cache_mod.dequantize, go.GptOssModel._route,
            go.GptOssModel._ffn_block, rt.moe_ffn) == originals


def test_prefill_slices_cover_every_row_and_halve_on_refusal():
    """MoeLayer.prefill: slices of the launch size in order, halved once when the library refuses
    a slice (status -2) before anything ran; the settled size is kept for later calls."""
    from nurostream_b200 import _lib
    from nurostream_b200.moe import MoeLayer

    calls = []

    class Fake(MoeLayer):
        def __init__(self, t, max_tokens, limit):
            self.t, self.max_tokens, self._slice, self.limit = t, max_tokens, 0, limit

        def __call__(self, x, out=None, add_residual=True, ids=None, weights=None):
            if x.shape[0] > self.limit:
                raise _lib.NsError(-2, "does not fit")
            calls.append((x.shape[0], int(x[0, 0]), ids.shape[0] if ids is not None else None))
            out.copy_(x + 1.0)
            return out

    x = torch.arange(20, dtype=torch.float32).reshape(20, 1).contiguous()
    ids = torch.zeros((20, 4), dtype=torch.int32)
    lay = Fake(GGMLType.MXFP4, 8, 1)          # 2-row slices refused -> halved to 1 for good
    out = lay.prefill(x, ids=ids)
    assert [c[0] for c in calls] == [1] * 20 and [c[1] for c in calls] == list(range(20))
    assert all(c[2] == c[0] for c in calls)
    assert torch.equal(out, x + 1.0) and lay._slice == 1
    calls.clear()
    lay = Fake(GGMLType.MXFP4, 8, 8)          # MXFP4: slices of 2 rows
    lay.prefill(x[:5].contiguous())
    assert [c[0] for c in calls] == [2, 2, 1]
    calls.clear()
    Fake(GGMLType.Q4_K, 8, 8).prefill(x[:3].contiguous())   # CUDA-core types: one row per launch
    assert [c[0] for c in calls] == [1, 1, 1]
    with pytest.raises(_lib.NsError):         # a refusal at one row is an error, not a loop
        Fake(GGMLType.Q8_0, 8, 0).prefill(x)


def test_dropin_touches_cache_in_reference_order(reference):
    """The fused drop-in looks its tensors up in the order the reference's neuron-block _ffn_block
    does, so the VRAM-Q LRU order after a call is the reference's."""
    import torch as _t
    from neurostream.model.gpt_oss import GptOssConfig, GptOssModel
    from neurostream.residency.cache import TieredCache

    from nurostream_b200 import moe
    from tests import goldens
    from tests.golden.make_golden import SynthSource, layer_tensors

    c = goldens.cases(goldens.load("moe"))["gptoss_small_bias_t3"]
    common = dict(n_layer=1, n_embd=c["H"], n_head=1, n_head_kv=1, head_dim=c["H"], n_ffn=c["F"], vocab_size=8,
                  rms_eps=1e-5, rope_base=10000.0, context_length=4096, n_expert=c["E"], n_expert_used=c["k"],
                  n_ffn_expert=c["F"])
    orders = []
    for use_dropin in (False, True):
        src = SynthSource(layer_tensors(c))
        cache = TieredCache(src, vram_budget=1 << 40)
        for name in sorted(src.gguf.tensors, reverse=True):
            assert cache.admit_vram(name)
        model = GptOssModel(cache, GptOssConfig(**common), block_rows=c["block_rows"])
        x = _t.from_numpy(goldens.SynthLayer(c).x.copy())
        if use_dropin:
            moe._lookup(model, 0, gptoss=True)
        else:
            model._ffn_block(x, 0)
        orders.append(list(cache._vram))
    assert orders[0] == orders[1]


def test_deferred_router_stats_fold_like_the_reference():
    """Folding (T, k) ids gives the reference's counters (moe/router.py:183-198)."""
    from nurostream_b200.moe import DeferredRouterStats, RouterStats

    st = DeferredRouterStats(RouterStats())
    st._fold(3, np.array([[5, 1], [1, 7], [5, 1]]))
    assert st.tokens_routed == 3
    assert dict(st.hits) == {(3, 1): 3, (3, 5): 2, (3, 7): 1}
    assert st.expert_reads == 3
    st.tokens_routed += 2                      # what the reference's fallback path does
    assert st.tokens_routed == 5
