"""GPU parity: synthetic generator, dequant (bit-exact) and the fused GEMV,
called through the C ABI and compared with the CPU oracle and the reference's
golden outputs."""
import numpy as np
import pytest
import torch

from nurostream_b200 import _lib, fused, synth
from nurostream_b200.ggml import GGMLType, TYPE_LAYOUT, row_bytes
from oracle import moe as omoe
from oracle import quant as oquant
from tests import goldens
from tests.gpu_util import assert_rel_close, device_float, device_quant

pytestmark = pytest.mark.gpu

QTYPES = [GGMLType.MXFP4, GGMLType.Q8_0, GGMLType.Q4_K, GGMLType.Q6_K, GGMLType.Q5_K, GGMLType.Q4_0]


@pytest.mark.parametrize("t", QTYPES)
def test_synth_device_matches_host(t):
    for start, n in [(0, 4096), (3, 1001), (123457, 5000)]:
        dev = device_quant(t, 9, 31, n, start).cpu().numpy()
        np.testing.assert_array_equal(dev, synth.quant_bytes(t, 9, 31, start, n))


def test_synth_float_device_matches_host():
    x = device_float(5000, 2, 7, 0.02).cpu().numpy()
    np.testing.assert_array_equal(x, synth.float_values(2, 7, 0, 5000, 0.02))
    b = torch.empty(777, dtype=torch.bfloat16, device="cuda")
    synth.fill_float(b, 2, 8, 5, 0.5)
    np.testing.assert_array_equal(b.cpu().view(torch.int16).numpy().view(np.uint16),
                                  synth.float_values(2, 8, 5, 777, 0.5, dtype="bf16"))


@pytest.mark.parametrize("name", [t.name for t in QTYPES])
def test_dequant_bit_exact_against_reference(name):
    g = goldens.load("dequant")
    raw = g[f"raw_{name}"]
    want = g[f"out_{name}"]
    t = GGMLType[name]
    be, bb = TYPE_LAYOUT[t]
    n = raw.size // bb * be
    got = fused.dequantize(torch.from_numpy(raw).cuda(), t, n).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint32), want)
    # truncation to n_elements and narrower outputs follow torch's rounding of the fp32 value
    for od in (torch.float16, torch.bfloat16):
        got = fused.dequantize(torch.from_numpy(raw).cuda(), t, n - 5, od).cpu()
        ref = torch.from_numpy(want.view(np.float32)[: n - 5].copy()).to(od)
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16))


def test_dequant_float_types():
    v = np.array([1.5, -2.25, 3.0e-8, 65504.0], np.float32)
    for t, raw in ((GGMLType.F32, v.view(np.uint8)), (GGMLType.F16, v.astype(np.float16).view(np.uint8))):
        got = fused.dequantize(torch.from_numpy(raw.copy()).cuda(), t, 4).cpu().numpy()
        np.testing.assert_array_equal(got, oquant.dequantize(raw, t, 4))


def test_q8_0_known_answer():
    """fp16 scale 1.0, codes 1..32, dot with ones = 528 (reference tests/test_tuning.py:104-153)."""
    row = np.concatenate([np.array([1.0], np.float16).view(np.uint8), np.arange(1, 33, dtype=np.uint8)])
    raw = torch.from_numpy(np.tile(row, 4)).cuda()
    y = fused.fused_gemv(raw, GGMLType.Q8_0, torch.ones(2, 32, device="cuda"), 4, 32, out_dtype=torch.float32)
    assert torch.equal(y.cpu(), torch.full((2, 4), 528.0))


def test_gemv_golden_cases():
    g = goldens.load("gemv")
    for name, meta in goldens.cases(g).items():
        raw, x = goldens.gemv_inputs(meta)
        y = fused.fused_gemv(torch.from_numpy(raw).cuda(), meta["type"], torch.from_numpy(x).cuda(),
                             meta["n_rows"], meta["K"], out_dtype=torch.float32).cpu().numpy()
        assert_rel_close(y, g[f"{name}__y"], 1e-5, name)
        truth = omoe.quant_linear(x, raw, meta["type"], meta["n_rows"], meta["K"], acc=np.float64)
        assert_rel_close(y, truth, 1e-5, name + " vs fp64")


def _gemv_case(t, n, K, T, seed=1, offset=0, x_dtype=torch.float32, y_dtype=torch.float32):
    rb = row_bytes(t, K)
    raw = synth.quant_bytes(t, seed, 5, 0, n * rb)
    raw_all = np.zeros(n * rb + offset + 16, np.uint8)
    raw_all[offset:offset + n * rb] = raw          # valid blocks starting off a 16-byte boundary
    x = synth.float_values(seed, 6, 0, T * K).reshape(T, K)
    dev_all = torch.from_numpy(raw_all).cuda()
    dev = dev_all[offset:offset + n * rb]          # a view with a storage offset
    xt = torch.from_numpy(x).cuda().to(x_dtype)
    y = fused.fused_gemv(dev, t, xt, n, K, out_dtype=y_dtype).float().cpu().numpy()
    truth = omoe.quant_linear(xt.float().cpu().numpy(), raw, t, n, K, acc=np.float64)
    return y, truth


@pytest.mark.parametrize("t", [GGMLType.MXFP4, GGMLType.Q8_0, GGMLType.Q4_K, GGMLType.Q6_K])
@pytest.mark.parametrize("T", [1, 2, 3, 5, 8])
def test_gemv_tokens(t, T):
    for n, K in [(1, 256), (37, 2880 if t in (GGMLType.MXFP4, GGMLType.Q8_0) else 2816), (600, 1024)]:
        y, truth = _gemv_case(t, n, K, T)
        assert_rel_close(y, truth, 1e-5, f"{t.name} n={n} K={K} T={T}")


@pytest.mark.parametrize("t", [GGMLType.MXFP4, GGMLType.Q8_0, GGMLType.Q4_K, GGMLType.Q6_K])
def test_gemv_unaligned_views(t):
    """Buffers that start off a 16-byte boundary take the ragged-edge path."""
    for off in (1, 3, 7, 13):
        y, truth = _gemv_case(t, 19, 512, 1, offset=off)
        assert_rel_close(y, truth, 1e-5, f"{t.name} offset {off}")


def test_gemv_activation_and_output_dtypes():
    for xd in (torch.float16, torch.bfloat16):
        for yd in (torch.float32, torch.float16, torch.bfloat16):
            y, truth = _gemv_case(GGMLType.MXFP4, 300, 2880, 2, x_dtype=xd, y_dtype=yd)
            assert_rel_close(y, truth, 1e-5 if yd == torch.float32 else 1e-2, f"x {xd} y {yd}")


@pytest.mark.parametrize("t", [GGMLType.Q8_0, GGMLType.Q4_K, GGMLType.MXFP4])
def test_gemv_benchmark_sweep_sizes(t):
    """The dense sweep of the benchmark: N in {4096, 11008, 14336}, K = 4096."""
    for n in (4096, 11008, 14336):
        y, truth = _gemv_case(t, n, 4096, 1, seed=n)
        assert_rel_close(y, truth, 1e-5, f"{t.name} N={n}")
    assert _lib.device_error() == 0


def test_gemv_stream_linear_blocks_match_whole():
    """Row blocks of one tensor (stream_linear's walk) give the same rows as one call."""
    t, n, K = GGMLType.MXFP4, 2880, 2880
    rb = row_bytes(t, K)
    dev = device_quant(t, 3, 4, n * rb)
    x = device_float(K, 3, 5).reshape(1, K)
    whole = fused.fused_gemv(dev, t, x, n, K, out_dtype=torch.float32)
    for br in (1, 7, 512):
        parts = [fused.fused_gemv(dev[s * rb:min(n, s + br) * rb], t, x, min(n, s + br) - s, K,
                                  out_dtype=torch.float32) for s in range(0, n, br)]
        assert torch.equal(torch.cat(parts, dim=1), whole), br
