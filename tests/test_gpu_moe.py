"""GPU parity of the MoE decode step: router and the fused one-launch layer,
against the reference's golden layer outputs and the CPU oracle."""
import numpy as np
import pytest
import torch

from nurostream_b200 import _lib
from nurostream_b200.moe import MoeLayer, route
from oracle import moe as omoe
from tests import goldens
from tests.gpu_util import assert_rel_close, layer_from_synth, run_layer

pytestmark = pytest.mark.gpu


def _margin_ok(logits, ids, k):
    """Gap between the k-th and (k+1)-th logit, to flag near-ties instead of hiding them."""
    s = np.sort(logits, axis=-1)[:, ::-1]
    return (s[:, k - 1] - s[:, k]) if s.shape[1] > k else np.full(s.shape[0], np.inf)


@pytest.mark.parametrize("mode", [_lib.NS_ROUTE_TOPK_SOFTMAX, _lib.NS_ROUTE_SOFTMAX_TOPK_NORM])
@pytest.mark.parametrize("E,k,T", [(32, 4, 1), (128, 4, 3), (128, 8, 8), (16, 16, 2)])
def test_route_matches_oracle(mode, E, k, T):
    rng = np.random.default_rng(E * 100 + k * 10 + T)
    H = 2880
    h = rng.standard_normal((T, H)).astype(np.float32)
    w = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    b = (rng.standard_normal(E) * 0.02).astype(np.float32) if mode == 0 else None
    ids, weights, logits = route(torch.from_numpy(h).cuda(), torch.from_numpy(w).cuda(),
                                 None if b is None else torch.from_numpy(b).cuda(), k, mode)
    if mode == 0:
        oid, ow, ol = omoe.route_gptoss(h, w, b, k, acc=np.float64)
    else:
        oid, ow, ol = omoe.route_qwen(h, w, k, acc=np.float64)
    assert_rel_close(logits.cpu().numpy(), ol, 1e-6, "logits")
    assert (_margin_ok(ol, oid, k) > 1e-5).all(), "near-tie in the random draw; pick another seed"
    np.testing.assert_array_equal(ids.cpu().numpy(), oid)
    np.testing.assert_allclose(weights.cpu().numpy(), ow, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("name", ["gptoss_cfg1", "gptoss_small_bias_t3", "qwen_q4k_t2"])
def test_fused_layer_matches_reference_golden(name):
    g = goldens.load("moe")
    c = goldens.cases(g)[name]
    L = goldens.SynthLayer(c)
    layer = layer_from_synth(L)
    out, ids, w = run_layer(layer, L.x, add_residual=L.gptoss)
    np.testing.assert_array_equal(ids, g[f"{name}__ids"])
    np.testing.assert_allclose(w, g[f"{name}__weights"], rtol=2e-6, atol=1e-7)
    assert_rel_close(out, g[f"{name}__out"], 1e-3, name)
    assert_rel_close(out, g[f"{name}__out"], 2e-5, name + " (tight)")


def _oracle_layer(L):
    if L.gptoss:
        return omoe.gptoss_ffn_block(L.x, L.norm_w, 1e-5, L.router_w, L.router_b, L.rows_fn(), L.biases, L.k,
                                     acc=np.float64)
    return omoe.qwen_moe_ffn(L.x, L.router_w, L.rows_fn(), L.k, acc=np.float64)


def _cfg(**kw):
    c = dict(name="t", arch="gpt-oss", type=39, E=128, H=2880, F=2880, k=4, T=1, seed=11, bias=True,
             norm="random", block_rows=512)
    c.update(kw)
    return c


def test_fused_layer_gpt_oss_120b_shape():
    """A layer of the GPT-OSS-120B shape: 128 experts, top-4, H=F=2880, MXFP4, biases."""
    L = goldens.SynthLayer(_cfg())
    out, ids, w = run_layer(layer_from_synth(L), L.x)
    o_out, o_ids, o_w = _oracle_layer(L)
    np.testing.assert_array_equal(ids, o_ids)
    assert_rel_close(out, o_out, 2e-5, "gpt-oss-120b layer")


@pytest.mark.parametrize("T", [1, 2, 8])
def test_fused_layer_qwen3_235b_shape(T):
    """A layer of the Qwen3-235B-A22B shape: 128 experts, top-8, H=4096, F=1536, Q4_K; T=8 is the
    batch-8 decode step (up to 64 distinct experts in one launch; its 64 activation rows of 1536
    floats exceed shared memory, so phase 2 reads them from the workspace)."""
    L = goldens.SynthLayer(_cfg(arch="qwen3moe", type=12, H=4096, F=1536, k=8, T=T, bias=False, norm=None))
    layer = layer_from_synth(L)
    out, ids, w = run_layer(layer, L.x, add_residual=False)
    o_out, o_ids, o_w = _oracle_layer(L)
    np.testing.assert_array_equal(ids, o_ids)
    assert_rel_close(out, o_out, 2e-5, f"qwen3 layer T={T}")
    if T == 8:  # the slice walk of MoeLayer.prefill gives the same rows
        xt = torch.from_numpy(L.x.copy()).cuda()
        idt = torch.empty((T, L.k), dtype=torch.int32, device="cuda")
        out2 = layer.prefill(xt, add_residual=False, ids=idt).cpu().numpy()
        np.testing.assert_array_equal(idt.cpu().numpy().astype(np.int64), o_ids)
        assert_rel_close(out2, o_out, 2e-5, "qwen3 layer T=8 via prefill")
    assert _lib.device_error() == 0


def test_fused_layer_bf16_router_and_q8_0_experts():
    L = goldens.SynthLayer(_cfg(type=8, E=16, H=1024, F=512, k=2, T=2, seed=3))
    layer = layer_from_synth(L, router_dtype=torch.bfloat16)
    out, ids, _ = run_layer(layer, L.x)
    Lb = L
    Lb.router_w = torch.from_numpy(L.router_w).to(torch.bfloat16).float().numpy()
    o_out, o_ids, _ = _oracle_layer(Lb)
    np.testing.assert_array_equal(ids, o_ids)
    assert_rel_close(out, o_out, 2e-5, "q8_0 + bf16 router")


def test_expert_parallel_shards_sum_to_full_layer():
    """Experts split by index over shards; the sum of shard outputs (residual on one) is the layer."""
    L = goldens.SynthLayer(_cfg(E=64, T=2, seed=21))
    full, ids, w = run_layer(layer_from_synth(L), L.x)
    parts = []
    for r, (lo, hi) in enumerate([(0, 16), (16, 32), (32, 48), (48, 64)]):
        out, sids, sw = run_layer(layer_from_synth(L, lo=lo, hi=hi), L.x, add_residual=(r == 0))
        np.testing.assert_array_equal(sids, ids)      # every shard routes identically
        parts.append(out)
    assert_rel_close(sum(parts), full, 1e-5, "sum of 4 shards")


def test_repeated_launches_reuse_the_workspace():
    """The grid barrier's epoch counter carries over launches; outputs stay identical."""
    L = goldens.SynthLayer(_cfg(E=32, seed=4))
    layer = layer_from_synth(L)
    first, _, _ = run_layer(layer, L.x)
    xt = torch.from_numpy(L.x).cuda()
    out = torch.empty_like(xt)
    for _ in range(50):
        layer(xt, out=out)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert np.array_equal(out.cpu().numpy(), first)


def test_too_many_activation_rows_is_reported_not_run():
    L = goldens.SynthLayer(_cfg(E=64, k=16, T=8, F=2880, seed=2))
    layer = layer_from_synth(L, max_tokens=8)
    with pytest.raises(_lib.NsError) as e:
        layer(torch.from_numpy(L.x).cuda())
    assert e.value.status == -2


@pytest.mark.parametrize("kw", [
    dict(T=20),                                                                       # GPT-OSS, 8 + 8 + 4
    dict(arch="qwen3moe", type=12, E=32, k=8, H=1024, F=512, T=11, bias=False, norm=None),
])
def test_prefill_slices_match_oracle(kw):
    """T > max_tokens runs as slices of max_tokens rows; rows equal the oracle's T-row layer."""
    c = _cfg(E=32, H=1024, F=1024, seed=31)
    c.update(kw)
    L = goldens.SynthLayer(c)
    layer = layer_from_synth(L, max_tokens=8)
    xt = torch.from_numpy(np.ascontiguousarray(L.x, dtype=np.float32)).cuda()
    ids = torch.empty((L.T, L.k), dtype=torch.int32, device="cuda")
    w = torch.empty((L.T, L.k), dtype=torch.float32, device="cuda")
    out = layer.prefill(xt, add_residual=L.gptoss, ids=ids, weights=w)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    o_out, o_ids, _ = _oracle_layer(L)
    np.testing.assert_array_equal(ids.cpu().numpy().astype(np.int64), o_ids)
    assert_rel_close(out.cpu().numpy(), o_out, 2e-5, f"prefill {kw}")


def test_decoder_batch8_qwen3_shape_matches_per_token_layers():
    """MoeDecoder at batch 8 (each layer as 2-row slices of the fused kernel) equals running each row
    alone through the same layers: tokens are independent through the MoE step."""
    from nurostream_b200.decoder import MoeDecoder, MoeShape
    from nurostream_b200.ggml import GGMLType
    from nurostream_b200 import synth

    shape = MoeShape(n_layer=3, hidden=4096, expert_ffn=1536, n_expert=128, top_k=8, ggml_type=int(GGMLType.Q4_K),
                     arch="qwen3")
    dec8 = MoeDecoder(shape, "cuda", use_graph=True, batch=8)
    assert dec8.capture()
    x = torch.empty((8, 4096), device="cuda")
    synth.fill_float(x.view(-1), 91, 2)
    y8 = dec8.step(x).clone()
    ids8 = dec8.ids.clone()
    dec1 = MoeDecoder(shape, "cuda", use_graph=False, batch=1)
    for t in range(8):
        y1 = dec1.step(x[t:t + 1])
        torch.cuda.synchronize()
        np.testing.assert_array_equal(dec1.ids.cpu().numpy(), ids8[:, t].cpu().numpy())
        assert_rel_close(y8[t].cpu().numpy(), y1[0].cpu().numpy(), 1e-5, f"row {t}")
    assert _lib.device_error() == 0
    dec8.release()
