"""GPU parity of the whole GPT-OSS decode step and of its new kernels.

* ``ns_dense_gemv`` (bf16 projection with fused RMSNorm / bias / residual) against an fp64 numpy
  product of the same bf16 values;
* ``ns_attn_decode`` (RoPE, KV append, sink attention, sliding window) against the oracle's
  ``sink_attention`` on the same history;
* ``GptOssDecoder`` -- embedding, 2 x (attention + MoE), LM head, in one CUDA graph -- against the
  logits and routing of the reference's own ``GptOssModel.forward`` (``tests/golden/model.npz``).
"""
import ctypes as C
import math

import numpy as np
import pytest
import torch

from nurostream_b200 import _lib, synth
from nurostream_b200.gptoss import GptOssDecoder, yarn_tables
from nurostream_b200.shapes import GptOssShape
from oracle import model as omodel
from tests import goldens
from tests.gpu_util import assert_rel_close

pytestmark = pytest.mark.gpu


def _bf16_dev(shape, seed, stream, sigma):
    t = torch.empty(int(np.prod(shape)), dtype=torch.bfloat16, device="cuda")
    synth.fill_float(t, seed, stream, 0, sigma)
    return t.reshape(shape)


def _f32(n, seed, stream, sigma=1.0):
    return torch.from_numpy(synth.float_values(seed, stream, 0, n, sigma)).cuda()


@pytest.mark.parametrize("K,rows,norm,bias,residual", [
    (2880, [4096, 512, 512], True, True, False),    # GPT-OSS q/k/v in one launch
    (4096, [2880], False, True, True),              # GPT-OSS output projection + residual
    (2880, [4096], True, False, False),             # LM head shape (fewer rows)
    (256, [19], False, False, False),               # fewer rows than one tile per CTA
    (8192, [300, 5], True, True, True),             # widest K, ragged second segment
    (1032, [1, 2, 3, 4], True, True, False),        # K = 129 chunks: partial chunk coverage
])
def test_dense_gemv_matches_fp64(K, rows, norm, bias, residual):
    seed = K + sum(rows)
    x = _f32(K, seed, 1)
    nw = (_f32(K, seed, 2, 0.1) + 1.0) if norm else None
    ws = [_bf16_dev((r, K), seed, 10 + i, 0.02) for i, r in enumerate(rows)]
    bs = [_f32(r, seed, 20 + i, 0.02) if bias else None for i, r in enumerate(rows)]
    rs = [_f32(r, seed, 30 + i) if residual else None for i, r in enumerate(rows)]
    ys = [torch.full((r,), float("nan"), device="cuda") for r in rows]
    p = _lib.DenseGemvParams()
    p.K, p.w_dtype, p.n_seg = K, _lib.NS_BF16, len(rows)
    for i in range(len(rows)):
        p.seg[i].w, p.seg[i].rows, p.seg[i].y = ws[i].data_ptr(), rows[i], ys[i].data_ptr()
        p.seg[i].bias = bs[i].data_ptr() if bias else None
        p.seg[i].residual = rs[i].data_ptr() if residual else None
    p.x, p.norm_w, p.rms_eps = x.data_ptr(), nw.data_ptr() if norm else None, 1e-5
    _lib.call("ns_dense_gemv", C.byref(p), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    xh = x.cpu().numpy().astype(np.float64)
    if norm:
        xh = xh / np.sqrt(np.mean(xh * xh) + 1e-5) * nw.cpu().numpy()
    for i in range(len(rows)):
        want = ws[i].float().cpu().numpy().astype(np.float64) @ xh
        if bias:
            want = want + bs[i].cpu().numpy()
        if residual:
            want = want + rs[i].cpu().numpy()
        assert_rel_close(ys[i].cpu().numpy(), want, 1e-5, f"segment {i} K={K}")


def _attn_case(n_head, n_kv, window, pos, max_ctx, seed):
    shape = GptOssShape(n_layer=1, n_head=n_head, n_head_kv=n_kv)
    hd = 64
    qkv = _f32((n_head + 2 * n_kv) * hd, seed, 1)
    k_hist = synth.float_values(seed, 2, 0, n_kv * max_ctx * hd).reshape(n_kv, max_ctx, hd)
    v_hist = synth.float_values(seed, 3, 0, n_kv * max_ctx * hd).reshape(n_kv, max_ctx, hd)
    kc = torch.from_numpy(k_hist.copy()).cuda()
    vc = torch.from_numpy(v_hist.copy()).cuda()
    sinks = _f32(n_head, seed, 4)
    cos, sin = yarn_tables(shape, max_ctx)
    cos_d, sin_d = cos.cuda(), sin.cuda()
    posd = torch.tensor([pos], dtype=torch.int32, device="cuda")
    out = torch.full((n_head * hd,), float("nan"), device="cuda")
    a = _lib.AttnDecodeParams()
    a.n_head, a.n_head_kv, a.head_dim, a.max_ctx, a.window, a.scale = n_head, n_kv, hd, max_ctx, window, 0.125
    a.pos, a.qkv, a.rope_cos, a.rope_sin, a.sinks = posd.data_ptr(), qkv.data_ptr(), cos_d.data_ptr(), sin_d.data_ptr(), sinks.data_ptr()
    a.k_cache, a.v_cache, a.out = kc.data_ptr(), vc.data_ptr(), out.data_ptr()
    n = C.c_size_t(0)
    _lib.call("ns_attn_workspace_bytes", C.byref(a), C.byref(n))
    ws = torch.zeros(n.value, dtype=torch.uint8, device="cuda")
    return dict(a=a, ws=ws, out=out, kc=kc, vc=vc, qkv=qkv, sinks=sinks, k_hist=k_hist, v_hist=v_hist, cos=cos,
                sin=sin, shape=shape, keep=(posd, cos_d, sin_d))


def _attn_oracle(c, pos, window, n_head, n_kv):
    hd = 64
    qkv = c["qkv"].cpu().numpy()
    q = qkv[:n_head * hd].reshape(n_head, 1, hd)
    k = qkv[n_head * hd:(n_head + n_kv) * hd].reshape(n_kv, 1, hd)
    v = qkv[(n_head + n_kv) * hd:].reshape(n_kv, 1, hd)
    cos, sin = c["cos"][pos:pos + 1].numpy(), c["sin"][pos:pos + 1].numpy()
    q, k = omodel.apply_rope(q, cos, sin), omodel.apply_rope(k, cos, sin)
    kh = np.concatenate([c["k_hist"][:, :pos], k], axis=1)
    vh = np.concatenate([c["v_hist"][:, :pos], v], axis=1)
    rep = n_head // n_kv
    o = omodel.sink_attention(q, np.repeat(kh, rep, 0), np.repeat(vh, rep, 0), c["sinks"].cpu().numpy(), window,
                              acc=np.float64)
    return o.reshape(-1), k[:, 0], v[:, 0]


@pytest.mark.parametrize("n_head,n_kv,window,pos,max_ctx", [
    (64, 8, 0, 2048, 2304),       # GPT-OSS full layer at 2k context
    (64, 8, 128, 2048, 2304),     # GPT-OSS sliding layer
    (64, 8, 128, 100, 512),       # window longer than the history
    (64, 8, 0, 0, 64),            # the first token: only its own key
    (64, 8, 0, 63, 256),          # block boundaries
    (64, 8, 0, 64, 256),
    (64, 8, 0, 65, 256),
    (16, 2, 0, 7, 64),            # fewer keys than splits
    (32, 8, 128, 500, 1024),      # 4 query heads per kv head
])
def test_attention_matches_oracle(n_head, n_kv, window, pos, max_ctx):
    c = _attn_case(n_head, n_kv, window, pos, max_ctx, seed=pos + 7 * n_head + window)
    _lib.call("ns_attn_decode", C.byref(c["a"]), c["ws"].data_ptr(), c["ws"].numel(),
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    want, k_new, v_new = _attn_oracle(c, pos, window, n_head, n_kv)
    assert_rel_close(c["out"].cpu().numpy(), want, 2e-5, f"attention pos={pos} window={window}")
    # the token's key (rotated) and value were appended at slot pos
    assert_rel_close(c["kc"][:, pos].cpu().numpy(), k_new, 1e-6, "appended key")
    np.testing.assert_array_equal(c["vc"][:, pos].cpu().numpy(), v_new)
    # history untouched
    np.testing.assert_array_equal(c["kc"][:, :pos].cpu().numpy(), c["k_hist"][:, :pos])
    # a second launch (counters reset by the first) gives the same bits
    out1 = c["out"].clone()
    _lib.call("ns_attn_decode", C.byref(c["a"]), c["ws"].data_ptr(), c["ws"].numel(),
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(out1, c["out"])


def test_embedding_row_is_exact():
    V, H = 1000, 2880
    tab = _bf16_dev((V, H), 9, 1, 1.0)
    tok = torch.tensor([777], dtype=torch.int32, device="cuda")
    out = torch.empty(H, device="cuda")
    _lib.call("ns_embed", tab.data_ptr(), _lib.NS_BF16, V, H, tok.data_ptr(), out.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(out, tab[777].float())


def _golden_decoder(use_graph, fused=True):
    g = goldens.load("model")
    c = goldens.cases(g)["gptoss_2layer"]
    shape = GptOssShape(n_layer=c["n_layer"], vocab_size=c["vocab_size"])
    dec = GptOssDecoder(shape, "cuda", seed=c["seed"], ctx=c["ctx"], max_ctx=512, use_graph=use_graph,
                        fused_attention=fused)
    assert dec.capture() == use_graph
    return g, c, dec


@pytest.mark.parametrize("use_graph,fused", [(True, True), (False, True), (True, False)])
def test_decoder_matches_reference_forward(use_graph, fused):
    """Three consecutive tokens (each appending to the KV cache) against the reference's own forward,
    with the attention block as one cooperative kernel (fused) or as its three kernels."""
    g, c, dec = _golden_decoder(use_graph, fused)
    for i, tok in enumerate(c["tokens"]):
        dec.set_token(tok, c["ctx"] + i)
        logits = dec.step().cpu().numpy()
        assert _lib.device_error() == 0
        np.testing.assert_array_equal(dec.ids.cpu().numpy(), g["gptoss_2layer__ids"][i], err_msg=f"token {i} routing")
        want = g["gptoss_2layer__logits"][i]
        assert_rel_close(logits, want, 1e-3, f"token {i} logits")
        assert_rel_close(logits, want, 1e-4, f"token {i} logits (tight)")
    dec.release()


def test_decoder_end_to_end_from_host_and_repeatable():
    """decode() from pinned host memory; re-decoding a token at the same position gives the same bits."""
    g, c, dec = _golden_decoder(True)
    tok = torch.tensor([c["tokens"][0]], dtype=torch.int32).pin_memory()
    pos = torch.tensor([c["ctx"]], dtype=torch.int32).pin_memory()
    first = dec.decode(tok, pos_host=pos).numpy().copy()
    assert_rel_close(first, g["gptoss_2layer__logits"][0], 1e-4, "decode()")
    again = dec.decode(tok, pos_host=pos).numpy()
    assert np.array_equal(first, again)
    dec.release()


@pytest.mark.parametrize("window,pos,max_ctx,n_head,n_kv", [
    (0, 2048, 2112, 64, 8),       # GPT-OSS full layer at 2k context
    (128, 2048, 2112, 64, 8),     # GPT-OSS sliding layer
    (128, 50, 128, 64, 8),        # fewer keys than the window
    (0, 0, 64, 64, 8),            # the first token
    (0, 5, 64, 16, 2),            # fewer keys than splits
    (0, 700, 1024, 32, 8),        # 4 query heads per kv head
])
def test_attention_block_matches_oracle(window, pos, max_ctx, n_head, n_kv):
    """ns_attn_block (one cooperative launch) against the oracle's attention block on the same
    weights and history: the output row, the appended key/value and an untouched history."""
    from tests.model_twin import TwinWeights, kv_history

    H = 2880
    shape = GptOssShape(n_layer=1, n_embd=H, n_head=n_head, n_head_kv=n_kv, sliding_window=max(window, 1))
    seed = 40 + pos
    from nurostream_b200.gptoss import AttnLayer
    A = AttnLayer(shape, 0, torch.device("cuda"), seed, max_ctx, pos)
    A.window = window
    x = _f32(H, seed, 99)
    out = torch.full((H,), float("nan"), device="cuda")
    cos, sin = yarn_tables(shape, max_ctx)
    cos_d, sin_d = cos.cuda(), sin.cuda()
    posd = torch.tensor([pos], dtype=torch.int32, device="cuda")
    b = A.block_params(x, posd, cos_d, sin_d, out)
    n = C.c_size_t(0)
    _lib.call("ns_attn_block_workspace_bytes", C.byref(b), C.byref(n))
    ws = torch.zeros(n.value + 256, dtype=torch.uint8, device="cuda")
    wp = ws.data_ptr() + (-ws.data_ptr()) % 256
    _lib.call("ns_attn_block", C.byref(b), wp, n.value, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    W = TwinWeights(shape, seed)
    kv = kv_history(shape, seed, pos)
    cfg = W.config()
    cfg["sliding_window"] = window  # the oracle's layer 0 slides by this window (0: full attention)
    want = omodel.attention_block(x.cpu().numpy()[None, :], W, 0, cfg, kv, pos, acc=np.float64)[0]
    assert_rel_close(out.cpu().numpy(), want, 2e-5, f"block pos={pos} window={window}")
    k_new = kv[0][0][:, pos]
    assert_rel_close(A.k_cache[:, pos].cpu().numpy(), k_new, 1e-4, "appended key (a projection output)")
    if pos:
        np.testing.assert_array_equal(A.k_cache[:, :pos].cpu().numpy(), kv_history(shape, seed, pos)[0][0])
    # a second launch from the same state gives the same bits
    first = out.clone()
    _lib.call("ns_attn_block", C.byref(b), wp, n.value, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(first, out)
