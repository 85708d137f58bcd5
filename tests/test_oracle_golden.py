"""The CPU oracle against golden vectors produced by the reference's own code.

Bit-exact for dequantization (every E8M0 exponent, fp16 scales across the
normal and subnormal range); fp32-rounding-level agreement for the GEMV and
the MoE layer (summation order differs between numpy and torch); exact
equality of the routed expert ids.
"""
import numpy as np
import pytest

from nurostream_b200.ggml import GGMLType, TYPE_LAYOUT
from oracle import moe as omoe
from oracle import quant as oquant
from tests import goldens


@pytest.mark.parametrize("t", ["MXFP4", "Q4_K", "Q5_K", "Q6_K", "Q8_0", "Q4_0"])
def test_dequant_bit_exact(t):
    g = goldens.load("dequant")
    raw = g[f"raw_{t}"]
    want = g[f"out_{t}"]
    be, bb = TYPE_LAYOUT[GGMLType[t]]
    got = oquant.dequantize(raw, GGMLType[t], raw.size // bb * be)
    assert got.dtype == np.float32
    np.testing.assert_array_equal(got.view(np.uint32), want)


def test_mxfp4_covers_every_exponent():
    raw = goldens.load("dequant")["raw_MXFP4"].reshape(-1, 17)
    assert sorted(set(raw[:, 0].tolist())) == list(range(256))


def test_q8_0_known_answer():
    """fp16 scale 1.0, codes 1..32, dot with ones = 528 (reference tests/test_tuning.py:104-153)."""
    row = np.concatenate([np.array([1.0], np.float16).view(np.uint8), np.arange(1, 33, dtype=np.uint8)])
    y = omoe.quant_linear(np.ones((2, 32), np.float32), np.tile(row, 4), GGMLType.Q8_0, 4, 32)
    np.testing.assert_array_equal(y, np.full((2, 4), 528.0, np.float32))


def test_float_types_reinterpret():
    v = np.array([1.5, -2.25, 3.0e-8], np.float32)
    np.testing.assert_array_equal(oquant.dequantize(v.view(np.uint8), GGMLType.F32, 3), v)
    h = v.astype(np.float16)
    np.testing.assert_array_equal(oquant.dequantize(h.view(np.uint8), GGMLType.F16, 3), h.astype(np.float32))
    bf = (v.view(np.uint32) >> 16).astype(np.uint16)
    np.testing.assert_array_equal(oquant.dequantize(bf.view(np.uint8), GGMLType.BF16, 3),
                                  (bf.astype(np.uint32) << 16).view(np.float32))


def test_gemv_matches_reference_stream_linear():
    g = goldens.load("gemv")
    for name, meta in goldens.cases(g).items():
        raw, x = goldens.gemv_inputs(meta)
        got = omoe.quant_linear(x, raw, meta["type"], meta["n_rows"], meta["K"])
        want = g[f"{name}__y"]
        np.testing.assert_allclose(got, want, rtol=2e-5, atol=2e-5 * np.abs(want).max(), err_msg=name)


@pytest.mark.parametrize("name", ["gptoss_cfg1", "gptoss_small_bias_t3", "qwen_q4k_t2"])
def test_moe_layer_matches_reference(name):
    g = goldens.load("moe")
    c = goldens.cases(g)[name]
    L = goldens.SynthLayer(c)
    if L.gptoss:
        out, ids, w = omoe.gptoss_ffn_block(L.x, L.norm_w, 1e-5, L.router_w, L.router_b,
                                            L.rows_fn(), L.biases, L.k)
    else:
        out, ids, w = omoe.qwen_moe_ffn(L.x, L.router_w, L.rows_fn(), L.k)
    np.testing.assert_array_equal(ids, g[f"{name}__ids"])
    np.testing.assert_allclose(w, g[f"{name}__weights"], rtol=1e-6, atol=1e-7)
    want = g[f"{name}__out"]
    np.testing.assert_allclose(out, want, rtol=1e-5, atol=1e-5 * np.abs(want).max())


def test_oracle_model_matches_reference_forward():
    """The oracle's whole decode step against the reference's own GptOssModel.forward: 3 tokens
    on a 2-layer GPT-OSS-120B-wide model with a 300-position KV history (tests/golden/model.npz)."""
    import time

    from nurostream_b200.shapes import GptOssShape
    from oracle import model as omodel
    from tests import goldens
    from tests.model_twin import TwinWeights, kv_history

    g = goldens.load("model")
    c = goldens.cases(g)["gptoss_2layer"]
    shape = GptOssShape(n_layer=c["n_layer"], vocab_size=c["vocab_size"])
    W = TwinWeights(shape, c["seed"])
    kv = kv_history(shape, c["seed"], c["ctx"])
    cfg = W.config()
    t0 = time.time()
    for i, tok in enumerate(c["tokens"]):
        trace = []
        logits = omodel.forward_token(tok, W, cfg, kv, c["ctx"] + i, trace=trace)
        for l, (ids, _, _) in enumerate(trace):
            np.testing.assert_array_equal(ids[0], g["gptoss_2layer__ids"][i, l], err_msg=f"token {i} layer {l}")
        want = g["gptoss_2layer__logits"][i]
        err = np.abs(logits[0] - want).max() / np.abs(want).max()
        assert err < 1e-5, f"token {i}: oracle logits differ from the reference by {err:.2e}"
    assert time.time() - t0 < 300
