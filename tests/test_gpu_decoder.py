"""Parity of exactly what the benchmark times: ``MoeDecoder`` at the GPT-OSS-120B layer shape.

The decoder generates its weights in HBM (bf16 router + fp32 bias, fp32 norm and expert biases,
MXFP4 experts), runs every layer on the tensor-core layer kernel, chains the layers through
ping-pong buffers and captures one token in a CUDA graph with programmatic dependent launch.
Here it runs at a reduced depth of 4 layers on 3 different tokens, keeping every layer's output,
and each layer is compared with the fp64 oracle run on the host twin of the same synthetic bytes
(``nurostream_b200.synth``), fed with the decoder's own input to that layer.
"""
import numpy as np
import pytest
import torch

from nurostream_b200 import _lib, synth
from nurostream_b200.decoder import MoeDecoder, MoeShape
from nurostream_b200.ggml import GGMLType, row_bytes
from oracle import moe as omoe
from oracle import quant as oquant
from tests.gpu_util import assert_rel_close

pytestmark = pytest.mark.gpu


class HostLayer:
    """Host twin of ``MoeDecoder._make_layer(l)`` (same seeds, streams and float arithmetic)."""

    def __init__(self, shape: MoeShape, l: int):
        self.sh, self.s = shape, synth.LayerStreams(l)
        sh, s = shape, self.s
        H, F, E = sh.hidden, sh.expert_ffn, sh.n_expert
        self.t = GGMLType(sh.ggml_type)
        self.norm_w = synth.float_values(sh.seed, s.norm_w, 0, H, 0.1) + np.float32(1.0)
        bits = synth.float_values(sh.seed, s.router_w, 0, E * H, 0.02, dtype="bf16")
        self.router_w = synth.bf16_to_f32(bits).reshape(E, H)
        self.router_b = synth.float_values(sh.seed, s.router_b, 0, E, 0.02)
        self._rows = {}

        class _Bias:
            def __init__(self, stream, n):
                self.stream, self.n = stream, n

            def __getitem__(self, e):
                return synth.float_values(sh.seed, self.stream, e * self.n, self.n, sh.bias_sigma)

        self.biases = {"gate": _Bias(s.gate_b, F), "up": _Bias(s.up_b, F), "down": _Bias(s.down_b, H)}

    def rows(self, kind, e):
        key = (kind, e)
        if key not in self._rows:
            sh, s = self.sh, self.s
            H, F = sh.hidden, sh.expert_ffn
            out, K, stream = {"gate": (F, H, s.gate), "up": (F, H, s.up), "down": (H, F, s.down)}[kind]
            rb = row_bytes(self.t, K)
            raw = synth.quant_bytes(self.t, sh.seed, stream, e * out * rb, out * rb)
            self._rows[key] = oquant.dequantize(raw, self.t, out * K).reshape(out, K)
        return self._rows[key]

    def __call__(self, x):
        return omoe.gptoss_ffn_block(x, self.norm_w, 1e-5, self.router_w, self.router_b, self.rows, self.biases,
                                     self.sh.top_k, acc=np.float64)


def _margin(h, w, b, k):
    logits = h.astype(np.float64) @ w.astype(np.float64).T + b
    s = np.sort(logits, axis=-1)[:, ::-1]
    return s[:, k - 1] - s[:, k]


@pytest.mark.parametrize("use_graph", [True, False])
def test_decoder_chain_matches_oracle_layer_by_layer(use_graph):
    shape = MoeShape(n_layer=4)
    dec = MoeDecoder(shape, "cuda", use_graph=use_graph, keep_layer_outputs=True)
    graphed = dec.capture()
    assert graphed == use_graph
    twins = [HostLayer(shape, l) for l in range(shape.n_layer)]
    for step in range(3):
        x0 = synth.float_values(4242, 7, step * shape.hidden, shape.hidden).reshape(1, shape.hidden)
        dec.step(torch.from_numpy(x0).cuda())
        torch.cuda.synchronize()
        assert _lib.device_error() == 0
        ids = dec.ids.cpu().numpy()
        outs = [b.cpu().numpy() for b in dec.bufs]
        x = x0
        for l, twin in enumerate(twins):
            want, oid, _ = twin(x)
            h = omoe.rms_norm(x, twin.norm_w, 1e-5)
            assert (_margin(h, twin.router_w, twin.router_b, shape.top_k) > 1e-6).all(), \
                f"step {step} layer {l}: near-tie in the draw; routing equality would be luck"
            np.testing.assert_array_equal(ids[l], oid[0], err_msg=f"step {step} layer {l} routing")
            assert_rel_close(outs[l], want, 1e-3, f"step {step} layer {l}")
            assert_rel_close(outs[l], want, 2e-5, f"step {step} layer {l} (tight)")
            x = outs[l]                      # the next layer's input is what the decoder fed it
        if graphed:
            np.testing.assert_array_equal(dec.out.cpu().numpy(), outs[-1])
    dec.release()


def test_decoder_end_to_end_matches_chained_oracle():
    """The whole 4-layer chain from one input against the oracle chained on its own outputs."""
    shape = MoeShape(n_layer=4)
    dec = MoeDecoder(shape, "cuda", use_graph=True)
    assert dec.capture()
    twins = [HostLayer(shape, l) for l in range(shape.n_layer)]
    x0 = synth.float_values(4243, 7, 0, shape.hidden).reshape(1, shape.hidden)
    host = torch.from_numpy(x0).pin_memory()
    got = dec.decode(host).numpy().copy()
    x = x0
    for twin in twins:
        x, _, _ = twin(x)
    assert_rel_close(got, x, 1e-3, "4-layer chain")
    dec.release()
