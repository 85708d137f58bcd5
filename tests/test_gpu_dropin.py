"""The drop-in through the reference's own API, on a GPU.

``nurostream_b200.install()`` patches the reference package in place; these tests then call the
reference's own ``GptOssModel._ffn_block``, ``moe.router.moe_ffn``, ``stream_linear`` and
``Qwen3Model._linear`` on CUDA tensors over a ``TieredCache`` whose tensors are admitted to VRAM
(quantized experts stay GGUF bytes: the VRAM-Q tier), and compare with the golden outputs the
reference itself produced on CPU (``tests/golden/make_golden.py``).
"""
import numpy as np
import pytest
import torch

from tests import goldens
from tests.gpu_util import assert_rel_close

pytestmark = pytest.mark.gpu


def _vram_cache(src):
    from neurostream.residency.cache import TieredCache
    cache = TieredCache(src, device="cuda", compute_dtype=torch.float32, vram_budget=1 << 40)
    for name in src.gguf.tensors:
        assert cache.admit_vram(name), name
    return cache


def _model(kind, c, cache):
    from neurostream.model.gpt_oss import GptOssConfig, GptOssModel
    from neurostream.model.qwen3 import Qwen3Config, Qwen3Model
    common = dict(n_layer=1, n_embd=c["H"], n_head=1, n_head_kv=1, head_dim=c["H"], n_ffn=c["F"], vocab_size=8,
                  rms_eps=1e-5, rope_base=10000.0, context_length=4096, n_expert=c["E"], n_expert_used=c["k"],
                  n_ffn_expert=c["F"])
    if kind == "gpt-oss":
        return GptOssModel(cache, GptOssConfig(**common), device="cuda", dtype=torch.float32,
                           block_rows=c["block_rows"])
    return Qwen3Model(cache, Qwen3Config(**common), device="cuda", dtype=torch.float32, block_rows=c["block_rows"])


def _expected_hits(ids):
    hits = {}
    for e in sorted(set(ids.reshape(-1).tolist())):
        hits[(0, e)] = int((ids == e).any(-1).sum())
    return hits


@pytest.mark.parametrize("name", ["gptoss_cfg1", "gptoss_small_bias_t3"])
def test_reference_ffn_block_runs_fused_and_matches_golden(reference, name):
    import nurostream_b200
    from nurostream_b200 import _lib
    from tests.golden.make_golden import SynthSource, layer_tensors

    g = goldens.load("moe")
    c = goldens.cases(g)[name]
    cache = _vram_cache(SynthSource(layer_tensors(c)))
    model = _model("gpt-oss", c, cache)
    x = torch.from_numpy(goldens.SynthLayer(c).x.copy()).cuda()
    with nurostream_b200.install():
        out = model._ffn_block(x, 0)
        assert 0 in model._ns_layers, "the fused layer did not run"
        torch.cuda.synchronize()
        assert _lib.device_error() == 0
        assert_rel_close(out.cpu().numpy(), g[f"{name}__out"], 1e-3, name)
        assert_rel_close(out.cpu().numpy(), g[f"{name}__out"], 2e-5, name + " (tight)")
        stats = model.router_stats
        assert stats.tokens_routed == c["T"]
        assert dict(stats.hits) == _expected_hits(g[f"{name}__ids"])
        assert stats.expert_reads == len(set(g[f"{name}__ids"].reshape(-1).tolist()))
        # the layer keeps no reference to the cache's expert bytes between calls
        assert model._ns_layers[0].gate is None


def test_evicted_experts_fall_back_to_streaming(reference):
    """An expert slab evicted from VRAM is not used by a stale pointer: the next call runs the
    reference's streaming walk (its GEMVs on ns_gemv) and still matches the golden layer."""
    import nurostream_b200
    from tests.golden.make_golden import SynthSource, layer_tensors

    g = goldens.load("moe")
    name = "gptoss_small_bias_t3"
    c = goldens.cases(g)[name]
    cache = _vram_cache(SynthSource(layer_tensors(c)))
    model = _model("gpt-oss", c, cache)
    x = torch.from_numpy(goldens.SynthLayer(c).x.copy()).cuda()
    with nurostream_b200.install():
        first = model._ffn_block(x, 0).cpu().numpy()
        victim = "blk.0.ffn_down_exps.weight"
        e = cache._vram.pop(victim)
        cache.stats.vram_bytes -= e.nbytes
        cache.stats.evictions += 1
        del e
        second = model._ffn_block(x, 0).cpu().numpy()
        assert cache.stats.vram_bytes == sum(v.nbytes for v in cache._vram.values())
    assert_rel_close(first, g[f"{name}__out"], 2e-5, "fused")
    assert_rel_close(second, g[f"{name}__out"], 1e-4, "after eviction (reference streaming path)")


def test_reference_moe_ffn_runs_fused_and_matches_golden(reference):
    import nurostream_b200
    import neurostream.moe.router as router
    from tests.golden.make_golden import SynthSource, layer_tensors

    g = goldens.load("moe")
    name = "qwen_q4k_t2"
    c = goldens.cases(g)[name]
    cache = _vram_cache(SynthSource(layer_tensors(c)))
    model = _model("qwen3moe", c, cache)
    h = torch.from_numpy(goldens.SynthLayer(c).x.copy()).cuda()
    with nurostream_b200.install():
        out = router.moe_ffn(model, h, 0)
        assert 0 in model._ns_layers
        assert_rel_close(out.cpu().numpy(), g[f"{name}__out"], 1e-3, name)
        assert dict(model.router_stats.hits) == _expected_hits(g[f"{name}__ids"])


@pytest.mark.parametrize("case", ["mxfp4_19x2880", "q8_0_19x2880", "q4_k_37x4096", "q6_k_13x512", "q5_k_29x1024",
                                  "q4_0_21x2880", "q5_k_t3_300x512",
                                  "mxfp4_t3_600x1024"])
def test_reference_stream_linear_and_linear_on_ns_gemv(reference, case):
    import nurostream_b200
    from neurostream.compute.blockffn import stream_linear
    from neurostream.model.qwen3 import Qwen3Config, Qwen3Model
    from tests.golden.make_golden import SynthSource, quant_producer

    g = goldens.load("gemv")
    meta = goldens.cases(g)[case]
    from nurostream_b200.ggml import GGMLType
    t = GGMLType(meta["type"])
    src = SynthSource({"w": ((meta["n_rows"], meta["K"]), t, quant_producer(t, meta["seed"], meta["w_stream"]))})
    cache = _vram_cache(src)
    _, x = goldens.gemv_inputs(meta)
    xt = torch.from_numpy(x.copy()).cuda()
    want = g[f"{case}__y"]
    with nurostream_b200.install():
        for br in (7, 512):
            y = stream_linear(cache, "w", xt, block_rows=br, device="cuda", dtype=torch.float32)
            assert_rel_close(y.cpu().numpy(), want, 1e-4, f"{case} stream_linear block_rows={br}")
        cfg = Qwen3Config(n_layer=1, n_embd=meta["K"], n_head=1, n_head_kv=1, head_dim=meta["K"], n_ffn=8,
                          vocab_size=8, rms_eps=1e-6, rope_base=1e4, context_length=64)
        model = Qwen3Model(cache, cfg, device="cuda", dtype=torch.float32)
        y = model._linear("w", xt)
        assert_rel_close(y.cpu().numpy(), want, 1e-4, f"{case} Qwen3Model._linear")


@pytest.mark.parametrize("case", ["mxfp4_t3_600x1024", "q4_k_37x4096", "q5_k_t3_300x512"])
def test_streamed_path_for_ram_tier_tensors(reference, case):
    """install(streamed=True): the reference's stream_linear on a RAM-tier (host-resident, quantized)
    tensor goes through the copy-stream executor -- blocks uploaded while the previous block's GEMV
    runs -- and gives the reference's golden result; the RAM-tier hit is counted as the reference does."""
    import nurostream_b200
    from neurostream.compute import blockffn
    from neurostream.residency.cache import TieredCache
    from nurostream_b200 import stream
    from nurostream_b200.ggml import GGMLType
    from tests.golden.make_golden import SynthSource, quant_producer

    g = goldens.load("gemv")
    meta = goldens.cases(g)[case]
    t = GGMLType(meta["type"])
    src = SynthSource({"w": ((meta["n_rows"], meta["K"]), t, quant_producer(t, meta["seed"], meta["w_stream"]))})
    cache = TieredCache(src, device="cuda", compute_dtype=torch.float32, ram_budget=1 << 40)
    assert cache.admit_ram("w")
    _, x = goldens.gemv_inputs(meta)
    xt = torch.from_numpy(x.copy()).cuda()
    want = g[f"{case}__y"]
    with nurostream_b200.install(streamed=True):
        for br in (7, 64, 512):
            hits = cache.stats.ram_hits
            y = blockffn.stream_linear(cache, "w", xt, block_rows=br, device="cuda", dtype=torch.float32)
            torch.cuda.synchronize()
            assert cache.stats.ram_hits == hits + 1
            assert_rel_close(y.cpu().numpy(), want, 1e-5, f"{case} streamed block_rows={br}")
        # a row window, as stream_expert_ffn asks for one expert
        n = meta["n_rows"]
        lo, hi = n // 3, n - n // 4
        y = blockffn.stream_linear(cache, "w", xt, block_rows=16, device="cuda", dtype=torch.float32,
                                   row_start=lo, row_end=hi)
        assert_rel_close(y.cpu().numpy(), want[:, lo:hi], 1e-5, f"{case} window")
    assert torch.device("cuda", torch.cuda.current_device()).index in {k[1] for k in stream._EXECUTORS}
