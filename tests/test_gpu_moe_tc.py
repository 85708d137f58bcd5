"""GPU parity of the tensor-core (tcgen05, block-scaled MXFP4) fused MoE layer.

The kernel is forced with ns_moe_select_kernel(2) and compared with the
reference's golden layer outputs, the fp64 CPU oracle and the CUDA-core kernel
on the same inputs."""
import numpy as np
import pytest
import torch

from nurostream_b200 import _lib
from oracle import moe as omoe
from tests import goldens
from tests.gpu_util import assert_rel_close, layer_from_synth, run_layer

pytestmark = pytest.mark.gpu


@pytest.fixture
def path():
    def use(p):
        _lib.call("ns_moe_select_kernel", p)
    yield use
    _lib.call("ns_moe_select_kernel", 0)


def _cfg(**kw):
    c = dict(name="t", arch="gpt-oss", type=39, E=128, H=2880, F=2880, k=4, T=1, seed=11, bias=True,
             norm="random", block_rows=512)
    c.update(kw)
    return c


def _oracle_layer(L):
    if L.gptoss:
        return omoe.gptoss_ffn_block(L.x, L.norm_w, 1e-5, L.router_w, L.router_b, L.rows_fn(), L.biases, L.k,
                                     acc=np.float64)
    return omoe.qwen_moe_ffn(L.x, L.router_w, L.rows_fn(), L.k, acc=np.float64)


def test_tc_layer_matches_reference_golden(path):
    g = goldens.load("moe")
    name = "gptoss_cfg1"
    L = goldens.SynthLayer(goldens.cases(g)[name])
    path(2)
    out, ids, w = run_layer(layer_from_synth(L), L.x, add_residual=L.gptoss)
    np.testing.assert_array_equal(ids, g[f"{name}__ids"])
    np.testing.assert_allclose(w, g[f"{name}__weights"], rtol=2e-6, atol=1e-7)
    assert_rel_close(out, g[f"{name}__out"], 1e-3, name)
    assert_rel_close(out, g[f"{name}__out"], 2e-5, name + " (tight)")


@pytest.mark.parametrize("kw", [
    dict(),                                                    # GPT-OSS-120B layer shape
    dict(T=2, E=64, seed=5),
    dict(E=8, k=2, H=256, F=256, seed=7),
    dict(E=16, k=4, T=2, H=512, F=768, seed=8),
    dict(arch="qwen3moe", E=32, k=8, H=1024, F=512, bias=False, norm=None, T=2, seed=9),
    dict(E=4, k=1, H=2880, F=2880, seed=10),                   # one expert: tiles split over many CTAs
    dict(E=4, k=1, H=64, F=64, seed=11),                       # 4 K blocks: the sharers of a tile lie far apart
    dict(E=8, k=2, T=2, H=128, F=192, seed=12),
])
def test_tc_layer_matches_oracle_and_cuda_core_kernel(path, kw):
    L = goldens.SynthLayer(_cfg(**kw))
    layer = layer_from_synth(L)
    path(2)
    out, ids, w = run_layer(layer, L.x, add_residual=L.gptoss)
    path(1)
    ref_out, ref_ids, _ = run_layer(layer, L.x, add_residual=L.gptoss)
    o_out, o_ids, _ = _oracle_layer(L)
    np.testing.assert_array_equal(ids, o_ids)
    np.testing.assert_array_equal(ids, ref_ids)
    assert_rel_close(out, o_out, 2e-5, f"tc vs fp64 oracle {kw}")
    assert_rel_close(out, ref_out, 2e-5, f"tc vs cuda-core kernel {kw}")


def test_tc_expert_parallel_shards_sum_to_full_layer(path):
    L = goldens.SynthLayer(_cfg(E=64, T=2, seed=21))
    path(2)
    full, ids, _ = run_layer(layer_from_synth(L), L.x)
    parts = []
    for r, (lo, hi) in enumerate([(0, 16), (16, 32), (32, 48), (48, 64)]):
        out, sids, _ = run_layer(layer_from_synth(L, lo=lo, hi=hi), L.x, add_residual=(r == 0))
        np.testing.assert_array_equal(sids, ids)
        parts.append(out)
    assert_rel_close(sum(parts), full, 1e-5, "sum of 4 shards")


def test_tc_repeated_launches_are_identical(path):
    """Split tiles are finished in a fixed order: 50 launches give the same bits."""
    L = goldens.SynthLayer(_cfg(E=32, seed=4))
    layer = layer_from_synth(L)
    path(2)
    first, _, _ = run_layer(layer, L.x)
    xt = torch.from_numpy(L.x).cuda()
    out = torch.empty_like(xt)
    for _ in range(50):
        layer(xt, out=out)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert np.array_equal(out.cpu().numpy(), first)


def test_tc_path_refuses_layers_it_does_not_take(path):
    L = goldens.SynthLayer(_cfg(E=16, T=3, H=512, F=512, seed=2))
    layer = layer_from_synth(L, max_tokens=3)
    path(2)
    with pytest.raises(_lib.NsError) as e:
        layer(torch.from_numpy(L.x).cuda())
    assert e.value.status == -2


def _bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).float().numpy()


@pytest.mark.parametrize("kw", [
    dict(),                                                    # the benchmarked layer: E=128, H=F=2880, top-4
    dict(T=2, E=64, seed=5),
    dict(E=32, k=4, H=1024, F=512, seed=13),
    dict(arch="qwen3moe", E=32, k=8, H=1024, F=512, bias=False, norm=None, T=2, seed=9),
])
def test_tc_layer_with_bf16_router_matches_oracle(path, kw):
    """bf16 router weights (what the benchmark's decoder holds) on the tensor-core kernel; the oracle
    routes with the same bf16-rounded weights widened to fp32."""
    L = goldens.SynthLayer(_cfg(**kw))
    layer = layer_from_synth(L, router_dtype=torch.bfloat16)
    path(2)
    out, ids, w = run_layer(layer, L.x, add_residual=L.gptoss)
    L.router_w = _bf16(L.router_w)
    o_out, o_ids, o_w = _oracle_layer(L)
    np.testing.assert_array_equal(ids, o_ids)
    np.testing.assert_allclose(w, o_w, rtol=2e-6, atol=1e-7)
    assert_rel_close(out, o_out, 1e-3, f"bf16 router {kw}")
    assert_rel_close(out, o_out, 2e-5, f"bf16 router {kw} (tight)")


@pytest.mark.parametrize("order", [(1, 3, 1, 3), (3, 1, 3, 1)])
def test_tensor_core_and_cuda_core_kernels_alternate_on_one_workspace(order):
    """T <= 2 takes the tensor-core kernel and T = 3 the CUDA-core kernel; their scratch layouts
    overlap in one workspace (barrier word, counters vs logits), so alternating them in either
    order must leave every call correct."""
    c = _cfg(E=16, k=4, H=512, F=512, T=3, seed=31)
    L = goldens.SynthLayer(c)
    layer = layer_from_synth(L, max_tokens=3)
    for T in order:
        sub = goldens.SynthLayer(dict(c, T=T))
        out, ids, _ = run_layer(layer, sub.x, add_residual=True)
        o_out, o_ids, _ = _oracle_layer(sub)
        np.testing.assert_array_equal(ids, o_ids)
        assert_rel_close(out, o_out, 2e-5, f"T={T} in order {order}")
