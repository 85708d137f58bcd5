"""Benchmark: batch-1 decode of a GPT-OSS-120B-shaped model on one B200 (or expert-parallel on N).

One step = one decode token through the whole model (config 3): embedding, 36 x (RMSNorm + bf16
q/k/v + YaRN RoPE + sink attention over a 2048-position KV cache, sliding window 128 on even
layers, + bf16 output projection + the MoE block: RMSNorm, router top-4 of 128, MXFP4 gate/up
2880x2880, clamped SwiGLU, down, weighted combine) and the LM head over a 201,088-token
vocabulary: 146 kernel launches captured in one CUDA graph.  About 5 GB of weights are read per
step against 126 MB of L2, so no flush is needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--ctx C]
  python bench.py --workload moe     [--layers L]   # the 36 MoE blocks only
  python bench.py --workload gemv                    # config 2: dense dequant-GEMV sweep
  python bench.py --workload qwen3   [--layers L]   # config 4 MoE blocks (Q4_K, top-8)
  python bench.py --workload prefill [--layers L]   # config 5: 512-token prefill of the MoE blocks

``--workload gemv`` prints one JSON line per case (batch 1, K = 4096, N in {4096, 11008, 14336},
MXFP4 / Q4_K / Q8_0), HBM GB/s against the measured copy peak, weight copies rotated so that every
launch streams from HBM.

N > 1 runs expert parallel under torchrun (experts split by index, one NCCL all-reduce per layer,
everything else replicated).  ``--impl reference`` times the reference's own CPU implementation
(``GptOssModel.forward`` of the installed reference package, all layers every step) on the host
cores; when the package is not installed it times the numpy oracle port instead.  Prints ONE JSON
line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tok/s at batch 1 (GPT-OSS-120B shape); dequant-GEMV HBM GB/s vs 8 TB/s"
UNIT = "tok/s"
KERNEL = "moe_tc_kernel"


def workload_config(shape, world, batch=1):
    if shape.arch == "qwen3":
        return {
            "workload": (f"qwen3-235b-a22b-shape MoE decode path: {shape.n_layer} layers x (RMSNorm + router softmax "
                         f"top-{shape.top_k}/{shape.n_expert} renormalised + Q4_K gate/up/down "
                         f"{shape.hidden}x{shape.expert_ffn} + silu*up + weighted combine + residual), batch {batch}"),
            "layers": shape.n_layer, "experts": shape.n_expert, "top_k": shape.top_k, "hidden": shape.hidden,
            "expert_ffn": shape.expert_ffn, "expert_format": "Q4_K (GGUF bytes, HBM-resident)",
            "router": "bf16 weight, no bias", "global_batch": batch, "seq_len": 1,
            "parallelism": f"ep{world}" if world > 1 else "single",
            "l2": "inputs larger than L2 (expert bytes per step far above L2 126 MB)",
        }
    return {
        "workload": (f"gpt-oss-120b-shape MoE decode path: {shape.n_layer} layers x (RMSNorm + router "
                     f"top-{shape.top_k}/{shape.n_expert} + MXFP4 gate/up/down {shape.hidden}x{shape.expert_ffn} "
                     f"+ clamped SwiGLU + weighted combine + residual), batch 1"),
        "layers": shape.n_layer, "experts": shape.n_expert, "top_k": shape.top_k, "hidden": shape.hidden,
        "expert_ffn": shape.expert_ffn, "expert_format": "MXFP4 (GGUF bytes, HBM-resident)",
        "router": "bf16 weight + fp32 bias", "global_batch": 1, "seq_len": 1,
        "parallelism": f"ep{world}" if world > 1 else "single",
        "l2": "inputs larger than L2 (1.9 GB of expert bytes per step, L2 126 MB)",
    }


# ----------------------------------------------------------------------------- CPU (oracle) leg

class CpuLayer:
    """One layer of the reference's CPU MoE path (oracle port), ready to time.

    Per call: RMSNorm, fp32 router (bf16 weights widened), top-4 + softmax,
    then for each routed expert dequantize its MXFP4 gate/up/down rows and
    multiply (numpy), combining in ascending expert order -- the reference's
    CPU path (``neurostream/model/gpt_oss.py:123-177`` on ``device='cpu'``).
    The routed experts' bytes are generated at construction (they stand in for
    the RAM-resident GGUF bytes); everything in ``run`` is timed.  The 8
    gate/up and the 4 down matrices run on a thread pool.
    """

    def __init__(self, shape, l: int):
        from nurostream_b200 import synth
        from nurostream_b200.ggml import GGMLType, row_bytes
        from oracle import moe as omoe

        t = self.t = GGMLType(shape.ggml_type)
        H, F, E, k = shape.hidden, shape.expert_ffn, shape.n_expert, shape.top_k
        self.H, self.F, self.k = H, F, k
        rb_h, rb_f = row_bytes(t, H), row_bytes(t, F)
        s = synth.LayerStreams(l)
        self.x = synth.float_values(777, 1, 0, H).reshape(1, H)
        self.rw = synth.bf16_to_f32(synth.float_values(shape.seed, s.router_w, 0, E * H, 0.02,
                                                       dtype="bf16")).reshape(E, H)
        self.rbias = synth.float_values(shape.seed, s.router_b, 0, E, 0.02)
        self.norm = synth.float_values(shape.seed, s.norm_w, 0, H, 0.1) + np.float32(1.0)
        h = omoe.rms_norm(self.x, self.norm, 1e-5)
        ids, _, _ = omoe.route_gptoss(h, self.rw, self.rbias, k)
        self.raw, self.bias = {}, {"gate": {}, "up": {}, "down": {}}
        for e in sorted(set(ids.reshape(-1).tolist())):
            self.raw[("gate", e)] = synth.quant_bytes(t, shape.seed, s.gate, e * F * rb_h, F * rb_h)
            self.raw[("up", e)] = synth.quant_bytes(t, shape.seed, s.up, e * F * rb_h, F * rb_h)
            self.raw[("down", e)] = synth.quant_bytes(t, shape.seed, s.down, e * H * rb_f, H * rb_f)
            self.bias["gate"][e] = synth.float_values(shape.seed, s.gate_b, e * F, F, shape.bias_sigma)
            self.bias["up"][e] = synth.float_values(shape.seed, s.up_b, e * F, F, shape.bias_sigma)
            self.bias["down"][e] = synth.float_values(shape.seed, s.down_b, e * H, H, shape.bias_sigma)

    def _proj(self, kind, e, v):
        from oracle import moe as omoe
        from oracle import quant as oquant
        rows, K = (self.F, self.H) if kind != "down" else (self.H, self.F)
        w = oquant.dequantize(self.raw[(kind, e)], self.t, rows * K).reshape(rows, K)
        return (omoe.linear(v, w) + self.bias[kind][e]).astype(np.float32)

    def run(self, pool) -> float:
        """Seconds for one token through this layer."""
        from oracle import moe as omoe
        t0 = time.perf_counter()
        h = omoe.rms_norm(self.x, self.norm, 1e-5)
        ids, w, _ = omoe.route_gptoss(h, self.rw, self.rbias, self.k)
        es = sorted(set(ids.reshape(-1).tolist()))
        gu = {(kind, e): pool.submit(self._proj, kind, e, h) for e in es for kind in ("gate", "up")}
        act = {e: omoe.clamped_swiglu(gu[("gate", e)].result(), gu[("up", e)].result()) for e in es}
        dn = {e: pool.submit(self._proj, "down", e, act[e]) for e in es}
        out = np.zeros((1, self.H), np.float32)
        for e in es:
            we = np.float32((w * (ids == e)).sum())
            out = (out + we * dn[e].result()).astype(np.float32)
        _ = self.x + out
        return time.perf_counter() - t0


def cpu_layer_sample(shape, n_layers: int, threads: int, reps: int = 3):
    """tok/s of the CPU path from the median layer time over `n_layers` layers x `reps`."""
    layers = [CpuLayer(shape, l) for l in range(n_layers)]
    with ThreadPoolExecutor(max_workers=threads) as pool:
        layers[0].run(pool)                                  # warm-up
        times = [L.run(pool) for _ in range(reps) for L in layers]
    per_layer = statistics.median(times)
    return 1.0 / (per_layer * shape.n_layer), per_layer, times


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


# ----------------------------------------------------------------------------- clocks

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.f = None

    def start(self):
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def wait_first(self, timeout: float = 5.0) -> None:
        """Block until the sampler has written its first row (so that short timed regions are covered)."""
        if self.proc is None:
            return
        t0 = time.time()
        while time.time() - t0 < timeout:
            try:
                if os.path.getsize(self.f.name) > 0:
                    return
            except OSError:
                return
            time.sleep(0.05)

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.flush()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [c.strip() for c in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
            except ValueError:
                continue
            for name, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- arms

def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def bench_shape(args):
    from nurostream_b200.decoder import MoeShape
    from nurostream_b200.ggml import GGMLType

    if args.workload == "qwen3":
        return MoeShape(n_layer=args.layers, hidden=4096, expert_ffn=1536, n_expert=128, top_k=8,
                        ggml_type=int(GGMLType.Q4_K), arch="qwen3")
    return MoeShape(n_layer=args.layers)


def run_ours(args, rank, world, local_rank, group):
    import torch
    import torch.distributed as dist

    from nurostream_b200 import _lib, synth
    from nurostream_b200.decoder import MoeDecoder, MoeShape
    from nurostream_b200.ggml import GGMLType

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    shape = bench_shape(args)
    B = args.batch
    dec = MoeDecoder(shape, dev, rank, world, group, use_graph=not args.no_graph, batch=B, combine=args.combine)
    H = shape.hidden
    npool = 64
    pool = torch.empty((npool, B, H), device=dev, dtype=torch.float32)
    synth.fill_float(pool.view(-1), 777, 1)
    host_pool = pool.cpu().pin_memory()
    out_host = torch.empty((B, H), dtype=torch.float32, pin_memory=True)
    graphed = dec.capture()

    def barrier():
        if world > 1:
            dist.barrier(group=group)

    for i in range(args.warmup):
        dec.step(pool[i % npool])
    torch.cuda.synchronize()
    dec.check_device_errors()

    clocks = ClockSampler(local_rank)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(args.steps):
        dec.step(pool[i % npool])
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    ms = ev0.elapsed_time(ev1)

    # end to end through the public API: host x in, host result out, every step
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record()
    for i in range(args.steps):
        dec.decode(host_pool[i % npool], out_host)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    ms_e2e = e0.elapsed_time(e1)
    clk = clocks.stop()
    dec.check_device_errors()

    # routing must agree on every rank (dense state is replicated)
    ids_ok = True
    if world > 1:
        t = torch.tensor([ms, ms_e2e], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        ms, ms_e2e = float(t[0]), float(t[1])
        gathered = [torch.empty_like(dec.ids) for _ in range(world)]
        dist.all_gather(gathered, dec.ids, group=group)
        ids_ok = all(torch.equal(g, gathered[0]) for g in gathered)
    # launches of one step: each layer's fused launches (slices of B rows), plus a combine per layer
    launches_per_layer = 1 if B == 1 else -(-B // max(1, dec.layers[0]._slice))
    launches = shape.n_layer * (launches_per_layer + (1 if dec.peer is not None else 0))
    dec.release()

    if rank != 0:
        return None
    step_ms = ms / args.steps
    tok_s = 1000.0 * B / step_ms
    peak, peak_kind = measured_peaks()
    bytes_layer = shape.layer_bytes_per_token()
    uniq = None
    if B > 1:  # the step reads each distinct routed expert once: count them on the last step's routing
        ids = dec.ids.view(shape.n_layer, -1).cpu()
        uniq = [len(set(r.tolist())) for r in ids]
        bytes_layer += (sum(uniq) / len(uniq) - shape.top_k) * shape.expert_bytes + (B - 1) * 4 * H * 3
    per_launch_s = step_ms / 1000.0 / shape.n_layer
    achieved = bytes_layer / per_launch_s / 1e9 if world == 1 else bytes_layer / per_launch_s / 1e9
    line = {
        "metric": METRIC if shape.arch == "gpt-oss" and B == 1 else
                  f"decode tok/s at batch {B} ({'GPT-OSS-120B' if shape.arch == 'gpt-oss' else 'Qwen3-235B-A22B'} shape, MoE layers)",
        "value": round(tok_s, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(step_ms, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": f"{GGMLType(shape.ggml_type).name.lower()} weights, fp32 accumulate",
        "data": "synthetic (seeded splitmix64 GGUF bytes generated in HBM)",
        "config": workload_config(shape, world, B),
        "e2e": {"value": round(1000.0 * B * args.steps / ms_e2e, 2), "unit": UNIT,
                "h2d_bytes_per_step": B * H * 4, "d2h_bytes_per_step": B * H * 4},
        "gpu_launches": launches * args.steps,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / (peak * (1 if world == 1 else world)), 4),
                     "traffic": None, "peak_kind": peak_kind,
                     "kernel": KERNEL if shape.arch == "gpt-oss" else "moe_layer_kernel",
                     "algorithmic_bytes_per_launch": bytes_layer,
                     "launch_ms": round(per_launch_s * 1000, 5),
                     "launch_ms_from": "CUDA events over the timed region / layers in it (each layer "
                                       f"{launches_per_layer} fused launch(es), back to back in the graph)"},
        "cuda_graph": graphed,
        "routing_identical_on_all_ranks": ids_ok,
    }
    if uniq is not None:
        line["roofline"]["unique_experts_per_layer"] = round(sum(uniq) / len(uniq), 2)
    if world > 1:
        line["config"]["combine"] = ("ns_peer_allreduce (NVLink peer stores, one kernel per layer)"
                                     if args.combine == "peer" else "NCCL all-reduce per layer")
    traffic = ROOT / "profiles" / ("moe_tc_kernel_traffic.json" if shape.arch == "gpt-oss"
                                   else "moe_layer_kernel_traffic.json")
    if traffic.exists():
        try:
            line["roofline"]["traffic"] = json.loads(traffic.read_text()).get("dram_bytes_per_launch")
        except Exception:
            pass
    if clk:
        line["clocks"] = clk
    if world == 1 and not args.no_cpu_baseline and shape.arch == "gpt-oss":
        threads = cpu_cores()
        cpu_tok_s, per_layer, _ = cpu_layer_sample(shape, args.cpu_layers, threads)
        line["cpu_baseline"] = {
            "value": round(cpu_tok_s, 5), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": (f"{args.cpu_layers} of {shape.n_layer} layers x 3 reps of one token (median layer "
                       f"{per_layer * 1000:.1f} ms, scaled to {shape.n_layer} layers); numpy oracle of the "
                       f"reference CPU path, expert matrices on a {threads}-thread pool"),
        }
    return line


def run_stream(args):
    """Streamed (host-resident) weights: x @ W.T with W's GGUF bytes in page-locked host memory.

    One step = one pass over a 1 GiB MXFP4 matrix (K = 4096): blocks uploaded on a copy stream while
    the previous block's GEMV runs (``nurostream_b200.stream.StreamedGemv``).  value: weight GB/s
    through the host link + GEMV; the same pass with upload and GEMV serialised is reported beside it.
    """
    import torch

    from nurostream_b200 import _lib, synth
    from nurostream_b200.ggml import GGMLType, row_bytes
    from nurostream_b200.stream import StreamedGemv

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    t, K = GGMLType.MXFP4, 4096
    rb = row_bytes(t, K)
    n = (1 << 30) // rb
    w_dev = torch.empty(n * rb, dtype=torch.uint8, device=dev)
    synth.fill_quant(w_dev, t, 0, 950, 0)
    host = w_dev.cpu().pin_memory()
    del w_dev
    x = torch.empty((1, K), device=dev)
    synth.fill_float(x.view(-1), 0, 951, 0)
    y = torch.empty((1, n), device=dev)
    ex = StreamedGemv(dev, block_bytes=8 << 20, depth=3)
    for _ in range(args.warmup):
        ex(host, t, x, n, K, out=y)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        ex(host, t, x, n, K, out=y)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    # serialised: the whole upload, then the GEMV over the device copy
    buf = torch.empty(n * rb, dtype=torch.uint8, device=dev)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(args.steps):
        buf.copy_(host, non_blocking=True)
        _lib.call("ns_gemv", buf.data_ptr(), buf.numel(), int(t), n, K, x.data_ptr(), _lib.NS_F32, K, 1,
                  y.data_ptr(), _lib.NS_F32, n, torch.cuda.current_stream(dev).cuda_stream)
    f1.record()
    torch.cuda.synchronize()
    ms_serial = f0.elapsed_time(f1) / args.steps
    gbs = n * rb / (ms / 1000.0) / 1e9
    return {
        "metric": "streamed GEMV GB/s (host-resident MXFP4 weights, batch 1)", "value": round(gbs, 1), "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "dtype": "mxfp4 weights, fp32 accumulate", "data": "synthetic",
        "config": {"workload": f"x @ W.T, W {n}x{K} MXFP4 ({n * rb >> 20} MiB) in page-locked host memory, "
                               "8 MiB blocks on a copy stream, 3 in flight"},
        "serialised_ms_per_step": round(ms_serial, 3),
        "serialised_gbs": round(n * rb / (ms_serial / 1000.0) / 1e9, 1),
    }


def full_decode_config(shape, world, ctx):
    return {
        "workload": (f"gpt-oss-120b-shape full decode: embedding + {shape.n_layer} x (RMSNorm + bf16 q/k/v + YaRN RoPE "
                     f"+ sink attention over {ctx} cached positions (sliding window {shape.sliding_window} on even "
                     f"layers) + bf16 o-proj + MoE: RMSNorm + router top-{shape.n_expert_used}/{shape.n_expert} + "
                     f"MXFP4 gate/up/down {shape.n_embd}x{shape.n_ffn_expert} + clamped SwiGLU + combine) + RMSNorm "
                     f"+ LM head {shape.vocab_size}x{shape.n_embd}, batch 1"),
        "model": "gpt-oss-120b shape (synthetic weights)", "layers": shape.n_layer, "hidden": shape.n_embd,
        "heads": f"{shape.n_head}q/{shape.n_head_kv}kv x {shape.head_dim}", "experts": shape.n_expert,
        "top_k": shape.n_expert_used, "vocab": shape.vocab_size, "context": ctx, "global_batch": 1, "seq_len": 1,
        "expert_format": "MXFP4 (GGUF bytes, HBM-resident)", "dense_format": "bf16", "kv_cache": "fp32",
        "parallelism": f"ep{world}" if world > 1 else "single",
        "l2": "inputs larger than L2 (about 5 GB of weights per step, L2 126 MB)",
    }


def run_full_decode(args, rank, world, local_rank, group):
    """Config 3: one whole GPT-OSS-120B-shaped decode token per step (``GptOssDecoder``, one CUDA graph).

    ``value``: K graph replays back to back, CUDA events on the launching stream, token and position
    already in HBM (the same token at position ``ctx`` every step, so every step is the same work).
    ``e2e``: ``GptOssDecoder.decode`` per step -- token id and position copied in from pinned host
    memory, the logits copied back out.  Roofline: the dominant kernel (``moe_tc_kernel``, timed alone
    after the timed region), with the whole step's algorithmic bytes (every weight byte the token
    needs once, KV history read, activations) over the step time beside it.
    """
    import torch
    import torch.distributed as dist

    from nurostream_b200.gptoss import GptOssDecoder
    from nurostream_b200.shapes import GptOssShape

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    shape = GptOssShape(n_layer=args.layers)
    clocks = ClockSampler(local_rank)
    dec = GptOssDecoder(shape, dev, seed=0, ctx=args.ctx, max_ctx=args.ctx + 64, rank=rank, world=world,
                        group=group, use_graph=not args.no_graph, combine=args.combine)
    token = 1234
    dec.set_token(token, args.ctx)
    graphed = dec.capture()
    tok_host = torch.tensor([token], dtype=torch.int32).pin_memory()
    pos_host = torch.tensor([args.ctx], dtype=torch.int32).pin_memory()
    logits_host = torch.empty(shape.vocab_size, dtype=torch.float32).pin_memory()

    def barrier():
        if world > 1:
            dist.barrier(group=group)

    clocks.start()
    clocks.wait_first()
    for _ in range(args.warmup):
        dec.step()
    torch.cuda.synchronize()
    dec.check_device_errors()
    stream = torch.cuda.current_stream(dev)
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        dec.step()
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = ev0.elapsed_time(ev1)
    # end to end through the public API: token and position in from host memory, logits out, every step
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        dec.decode(tok_host, logits_host, pos_host)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms_e2e = e0.elapsed_time(e1)
    # the dominant kernel alone: the MoE launches (moe_tc_kernel) of up to 20 layers back to back in
    # their own CUDA graph (no host time between launches; each layer's own experts, so no launch
    # finds its weights in L2), CUDA events around one replay
    reps = min(20, shape.n_layer)

    def moe_launches():
        for l in range(reps):
            _, _, _, xa, nxt = dec._p[l]
            dec.moe[l](xa.view(1, -1), out=nxt.view(1, -1), add_residual=(rank == 0), ids=dec.ids[l:l + 1])

    moe_launches()
    torch.cuda.synchronize()
    mg = torch.cuda.CUDAGraph()
    with torch.cuda.graph(mg):
        moe_launches()
    mg.replay()
    torch.cuda.synchronize()
    m0, m1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    m0.record(stream)
    mg.replay()
    m1.record(stream)
    torch.cuda.synchronize()
    moe_ms = m0.elapsed_time(m1) / reps
    mg = None
    clk = clocks.stop()
    dec.check_device_errors()
    ids_ok = True
    if world > 1:
        t = torch.tensor([ms, ms_e2e, moe_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        ms, ms_e2e, moe_ms = float(t[0]), float(t[1]), float(t[2])
        gathered = [torch.empty_like(dec.ids) for _ in range(world)]
        dist.all_gather(gathered, dec.ids, group=group)
        ids_ok = all(torch.equal(g_, gathered[0]) for g_ in gathered)
    parts = dec.bytes_per_token()
    dec.release()
    if rank != 0:
        return None
    step_ms = ms / args.steps
    peak, peak_kind = measured_peaks()
    achieved = parts["total"] / (step_ms / 1000.0) / 1e9
    moe_bytes = parts["experts+router"] / shape.n_layer  # one MoE layer's algorithmic bytes
    moe_achieved = moe_bytes / (moe_ms / 1000.0) / 1e9
    line = {
        "metric": METRIC, "value": round(1000.0 / step_ms, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16 dense + mxfp4 expert weights, fp32 activations and accumulation",
        "data": "synthetic (seeded splitmix64 weights and KV history generated in HBM)",
        "config": full_decode_config(shape, world, args.ctx),
        "e2e": {"value": round(1000.0 * args.steps / ms_e2e, 2), "unit": UNIT, "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": 4 * shape.vocab_size},
        "gpu_launches": dec.launches_per_step * args.steps,
        "roofline": {"bound": "hbm", "achieved": round(moe_achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(moe_achieved / peak, 4), "traffic": None, "peak_kind": peak_kind,
                     "kernel": "moe_tc_kernel (the step's largest share: one launch per layer)",
                     "algorithmic_bytes_per_launch": int(moe_bytes), "launch_ms": round(moe_ms, 5),
                     "launch_ms_from": "CUDA events around one replay of a graph of the MoE launches of layers "
                                       "0..19 back to back, after the timed region",
                     "step": {"achieved": round(achieved, 1), "frac": round(achieved / peak, 4),
                              "kernels": "ns_embed + 36 x (dense_gemv_kernel q/k/v, attn_decode_kernel, "
                                         "dense_gemv_kernel o-proj, moe_tc_kernel) + dense_gemv_kernel LM head, "
                                         "one CUDA graph",
                              "algorithmic_bytes_per_step": parts["total"],
                              "bytes_by_part": {k: v for k, v in parts.items() if k != "total"},
                              "step_ms": round(step_ms, 5),
                              "step_ms_from": "CUDA events around the K graph replays of the timed region / K"}},
        "cuda_graph": graphed,
        "routing_identical_on_all_ranks": ids_ok,
    }
    if world > 1:
        line["config"]["combine"] = ("ns_peer_allreduce (NVLink peer stores, one kernel per layer)"
                                     if args.combine == "peer" else "NCCL all-reduce per layer")
    traffic = ROOT / "profiles" / "moe_tc_kernel_traffic.json"
    if traffic.exists():
        try:
            line["roofline"]["traffic"] = json.loads(traffic.read_text()).get("dram_bytes_per_launch")
        except Exception:
            pass
    if clk:
        line["clocks"] = clk
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_full(shape, args.ctx)
    return line


def cpu_baseline_full(shape, ctx):
    """A bounded sample of the reference's own CPU decode: set-up, one warm-up token, two timed tokens."""
    threads = cpu_cores()
    if import_reference() is None:
        mshape = shape.moe_shape()
        tok_s, per_layer, _ = cpu_layer_sample(mshape, 2, threads)
        return {"value": round(tok_s, 5), "unit": UNIT, "cores": threads, "kind": "port",
                "sample": ("reference package not installed on this box: numpy oracle port of the MoE layers only, "
                           f"2 layers x 3 reps (median layer {per_layer * 1000:.1f} ms) scaled to {mshape.n_layer}")}
    t0 = time.perf_counter()
    ref = ReferenceDecode(shape, ctx=ctx, dense=True, threads=threads)
    ref.step()
    setup = time.perf_counter() - t0
    times = [ref.step() for _ in range(2)]
    v = 1.0 / statistics.mean(times)
    return {"value": round(v, 5), "unit": UNIT, "cores": threads, "kind": "reference",
            "sample": (f"2 whole tokens (mean {statistics.mean(times):.2f} s) through the reference's own "
                       f"GptOssModel.forward at {ctx} context on device='cpu', fp32, block_rows=512, "
                       f"torch.set_num_threads({threads}); set-up + 1 warm-up token {setup:.0f} s untimed")}


def run_gemv_sweep(args):
    """Dense dequant-GEMV at batch 1 (the reference's ``fused_gemv``, ``triton_kernels.py:199-228``).

    Each case rotates over enough copies of the weight matrix (>= 512 MB) that no launch finds its
    rows in the 126 MB L2; one step is one launch through ``ns_gemv``, timed with CUDA events on
    the launching stream.  Algorithmic bytes: the rows, x (fp32) and y (fp32).
    """
    import torch

    from nurostream_b200 import _lib, synth
    from nurostream_b200.ggml import GGMLType, row_bytes

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    peak, peak_kind = measured_peaks()
    K = 4096
    lines = []
    for t in (GGMLType.MXFP4, GGMLType.Q4_K, GGMLType.Q8_0):
        for N in (4096, 11008, 14336):
            if args.gemv_case and args.gemv_case != f"{t.name}:{N}":
                continue
            rb = row_bytes(t, K)
            mbytes = N * rb
            copies = max(2, -(-(512 << 20) // mbytes))
            w = torch.empty(copies * mbytes, dtype=torch.uint8, device=dev)
            synth.fill_quant(w, t, 0, 900 + int(t), 0)
            x = torch.empty((1, K), dtype=torch.float32, device=dev)
            synth.fill_float(x.view(-1), 0, 901, 0)
            y = torch.empty((1, N), dtype=torch.float32, device=dev)

            def launch(i):
                _lib.call("ns_gemv", w.data_ptr() + (i % copies) * mbytes, mbytes, int(t), N, K,
                          x.data_ptr(), _lib.NS_F32, K, 1, y.data_ptr(), _lib.NS_F32, N,
                          torch.cuda.current_stream(dev).cuda_stream)

            # one graph of `copies` back-to-back launches (each on the next copy), replayed: the timing
            # is the kernels', not the host's launch rate
            for i in range(copies):
                launch(i)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for i in range(copies):
                    launch(i)
            reps = max(1, -(-args.steps // copies))
            for _ in range(max(1, args.warmup // copies)):
                g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                g.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            n_launches = reps * copies
            us = e0.elapsed_time(e1) * 1000.0 / n_launches
            nbytes = mbytes + 4 * K + 4 * N
            gbs = nbytes / (us * 1e-6) / 1e9
            lines.append({
                "metric": "dequant-GEMV HBM GB/s at batch 1", "value": round(gbs, 1), "unit": "GB/s",
                "n_gpus": 1, "steps": n_launches, "warmup": args.warmup, "us_per_launch": round(us, 3),
                "higher_is_better": True, "dtype": f"{t.name} weights, fp32 accumulate",
                "data": "synthetic (seeded splitmix64 GGUF bytes generated in HBM)",
                "config": {"workload": f"dense dequant-GEMV {t.name} N={N} K={K} T=1", "type": t.name, "N": N,
                           "K": K, "l2": f"{copies} rotated weight copies ({copies * mbytes >> 20} MiB) per case"},
                "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                             "frac": round(gbs / peak, 4), "peak_kind": peak_kind, "kernel": "gemv_kernel",
                             "algorithmic_bytes_per_launch": nbytes},
            })
            del g, w
            torch.cuda.empty_cache()
    return lines


def run_prefill(args, rank=0, world=1, local_rank=0, group=None):
    """Prefill of ``--prefill-tokens`` prompt tokens through the GPT-OSS-shaped MoE layers (config 5).

    Each layer is one grouped expert GEMM on the tensor cores (``MoeLayer.prefill_grouped``: route,
    bucket, planes, gate/up + activation, down, combine), every launch of a step captured in one CUDA
    graph; at N > 1 every rank holds 1/N of the experts and the layer outputs are summed by one NCCL
    all-reduce per layer.  Algorithmic bytes per layer: every expert that the step's tokens route to,
    read once (at T = 512 that is all 128), plus the router and the activations in and out.
    """
    import torch
    import torch.distributed as dist

    from nurostream_b200 import synth
    from nurostream_b200.decoder import MoeDecoder

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    shape = bench_shape(args)
    T, H = args.prefill_tokens, shape.hidden
    dec = MoeDecoder(shape, dev, rank, world, group, use_graph=False, max_tokens=2)
    x = torch.empty((T, H), device=dev, dtype=torch.float32)
    synth.fill_float(x.view(-1), 778, 1)
    x_host = x.cpu().pin_memory()
    out_host = torch.empty((T, H), dtype=torch.float32, pin_memory=True)
    bufs = [torch.empty_like(x) for _ in range(2)]

    def barrier():
        if world > 1:
            dist.barrier(group=group)

    dec.prefill(x, bufs)                         # warm-up outside capture (workspaces, communicator)
    torch.cuda.synchronize()
    g = None
    if not args.no_graph:
        g = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(g):
                y = dec.prefill(x, bufs)
        except Exception:
            g = None
            torch.cuda.synchronize()

    graphed = g is not None

    def step():
        if g is not None:
            g.replay()
            return y
        return dec.prefill(x, bufs)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dec.check_device_errors()
    clocks = ClockSampler(local_rank)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        yy = step()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    ms = e0.elapsed_time(e1) / args.steps
    # end to end: prompt in from pinned host memory, hidden states back, every step
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    f0.record()
    for _ in range(args.steps):
        x.copy_(x_host, non_blocking=True)
        yy = step()
        out_host.copy_(yy, non_blocking=True)
    f1.record()
    torch.cuda.synchronize()
    barrier()
    ms_e2e = f0.elapsed_time(f1) / args.steps
    # one layer alone, outside the graph: the grouped GEMM's eight launches (CUDA events on this stream)
    layer = dec.layers[0]
    l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 5
    l0.record()
    for _ in range(reps):
        layer.prefill_grouped(x, out=bufs[0], add_residual=(rank == 0))
    l1.record()
    torch.cuda.synchronize()
    layer_ms = l0.elapsed_time(l1) / reps
    clk = clocks.stop()
    dec.check_device_errors()
    if world > 1:
        t = torch.tensor([ms, ms_e2e, layer_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        ms, ms_e2e, layer_ms = float(t[0]), float(t[1]), float(t[2])
    g = None
    dec.release()
    if rank != 0:
        return None
    peak, peak_kind = measured_peaks()
    E = shape.n_expert
    n_local = dec.hi - dec.lo
    expert_bytes = shape.expert_bytes                      # one expert's gate + up + down rows
    # the busiest rank's bytes: its experts (T = 512 touches all of them), the router, x in and out
    layer_bytes = n_local * expert_bytes + E * H * 2 + 2 * T * H * 4
    achieved = layer_bytes / (layer_ms / 1000.0) / 1e9
    flops = 2.0 * T * shape.top_k * 3 * H * shape.expert_ffn * n_local / E
    line = {
        "metric": "prefill tok/s (GPT-OSS-120B shape, 512-token prompt, MoE layers)", "value": round(T * 1000.0 / ms, 1),
        "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "mxfp4 weights x 24-bit activation digit planes (mxf4 tensor cores), fp32 accumulate",
        "data": "synthetic (seeded splitmix64 GGUF bytes generated in HBM)",
        "config": {"workload": f"gpt-oss-120b-shape MoE prefill: {T} tokens x {shape.n_layer} layers, each layer one "
                               f"grouped expert GEMM (8 launches: norm, logits, top-k, bucket, planes, gate/up+SwiGLU, down, combine)"
                               + (f" + NCCL all-reduce of the layer output over {world} ranks" if world > 1 else ""),
                   "tokens": T, "layers": shape.n_layer, "experts": E, "top_k": shape.top_k,
                   "parallelism": f"ep{world}" if world > 1 else "single",
                   "l2": "inputs larger than L2 (every layer streams its experts, 1.7 GB, from HBM)"},
        "e2e": {"value": round(T * 1000.0 / ms_e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": T * H * 4,
                "d2h_bytes_per_step": T * H * 4},
        "gpu_launches": shape.n_layer * 8 * args.steps,
        "cuda_graph": graphed,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None, "peak_kind": peak_kind,
                     "kernel": "pf_gemm_kernel<0>/<1> with norm, logits, top-k, bucket, planes and combine (one layer's eight launches)",
                     "algorithmic_bytes_per_layer": layer_bytes, "layer_ms": round(layer_ms, 4),
                     "layer_ms_from": "CUDA events around 5 back-to-back calls of one layer, outside the graph",
                     "mxf4_tflops": round(flops * 8 / (layer_ms / 1000.0) / 1e12, 1),
                     "mxf4_tflops_note": "8 digit planes per activation: MMA work is 8x the algorithmic 2*T*k*3*H*F"},
    }
    if clk:
        line["clocks"] = clk
    return line


# ----------------------------------------------------------------------------- reference arm

def import_reference():
    """Put the reference package on sys.path (NS_REFERENCE_PATH, else the copy installed in
    baseline/_ref); returns its path, or None when it is not installed on this machine."""
    for p in (os.environ.get("NS_REFERENCE_PATH"), str(ROOT / "baseline" / "_ref")):
        if p and (Path(p) / "neurostream").is_dir():
            sys.dont_write_bytecode = True
            if p not in sys.path:
                sys.path.insert(0, p)
            import neurostream  # noqa: F401
            return p
    return None


class SynthGGUF:
    """A GGUF-shaped synthetic weight source for the reference's own CPU path.

    It presents ``MmapSource``'s surface (``neurostream/io/source.py:65-133``): ``raw_bytes``,
    ``fetch``, ``raw_rows`` and ``fetch_rows`` hand out a fresh copy of the tensor's bytes and decode
    them with the reference's own ``dequantize``, as ``MmapSource`` does over a page-cached file.
    The bytes are generated on first touch and kept (they stand for the model file's pages in the
    host page cache): dense tensors whole, stacked expert tensors one expert window at a time.
    Values follow the configuration's distributions -- bf16 N(0, 0.02) dense weights, fp32
    N(0, 0.02) biases and sinks, unit norm weights, MXFP4 codes uniform with E8M0 exponents uniform
    in [118, 124] -- drawn with seeded torch/numpy generators: the reference's time does not depend on
    the values, so they need not equal the GPU arm's bit for bit.
    """

    def __init__(self, shape, dense: bool = True, n_layer: int | None = None):
        import torch
        from neurostream.format.gguf import GGMLType as T, TensorInfo, nbytes_for

        c = shape
        L = c.n_layer if n_layer is None else n_layer
        H, q, kv, E, F, V = c.n_embd, c.q_dim, c.kv_dim, c.n_expert, c.n_ffn_expert, c.vocab_size
        spec = {}
        if dense:
            spec["token_embd.weight"] = ((V, H), T.BF16, 0.02)
            spec["output_norm.weight"] = ((H,), T.F32, None)
            spec["output.weight"] = ((V, H), T.BF16, 0.02)
        for l in range(L):
            p = f"blk.{l}."
            if dense:
                spec[p + "attn_norm.weight"] = ((H,), T.F32, None)
                for nm, rows, cols in (("attn_q", q, H), ("attn_k", kv, H), ("attn_v", kv, H), ("attn_output", H, q)):
                    spec[p + nm + ".weight"] = ((rows, cols), T.BF16, 0.02)
                    spec[p + nm + ".bias"] = ((rows,), T.F32, 0.02)
                spec[p + "attn_sinks.weight"] = ((c.n_head,), T.F32, 1.0)
            spec[p + "post_attention_norm.weight"] = ((H,), T.F32, None)
            spec[p + "ffn_gate_inp.weight"] = ((E, H), T.BF16, 0.02)
            spec[p + "ffn_gate_inp.bias"] = ((E,), T.F32, 0.02)
            for kind, rows, cols in (("gate", F, H), ("up", F, H), ("down", H, F)):
                spec[p + f"ffn_{kind}_exps.weight"] = ((E, rows, cols), T.MXFP4, "expert")
                spec[p + f"ffn_{kind}_exps.bias"] = ((E, rows), T.F32, 0.02)
        self._spec = spec
        infos = {}
        for name, (shp, dt, _) in spec.items():
            n = int(np.prod(shp))
            infos[name] = TensorInfo(name, tuple(reversed(shp)), dt, 0, nbytes_for(dt, n))
        from types import SimpleNamespace
        self.gguf = SimpleNamespace(tensors=infos)
        self._mem: dict = {}
        self._torch = torch
        self._seed = {name: i + 1 for i, name in enumerate(spec)}

    # bytes -------------------------------------------------------------------
    def _dense(self, name) -> np.ndarray:
        got = self._mem.get(name)
        if got is None:
            torch = self._torch
            shp, dt, sigma = self._spec[name]
            n = int(np.prod(shp))
            if sigma is None:
                v = torch.ones(n, dtype=torch.float32)
            else:
                g = torch.Generator().manual_seed(self._seed[name])
                v = torch.randn(n, generator=g) * sigma
            v = v.to(torch.bfloat16) if dt.name == "BF16" else v
            got = self._mem[name] = v.view(torch.uint8).numpy()
        return got

    def _expert(self, name, e) -> np.ndarray:
        key = (name, e)
        got = self._mem.get(key)
        if got is None:
            info = self.gguf.tensors[name]
            nbytes = info.nbytes // info.torch_shape[0]
            rng = np.random.default_rng((self._seed[name] << 16) + e)
            got = rng.integers(0, 256, nbytes, dtype=np.uint8)
            got[0::17] = 118 + got[0::17] % 7                  # E8M0 scale byte of each 17-byte block
            self._mem[key] = got
        return got

    def _raw(self, name, start, nbytes):
        info = self.gguf.tensors[name]
        if self._spec[name][2] == "expert":
            per = info.nbytes // info.torch_shape[0]
            e = start // per
            if start + nbytes > (e + 1) * per:
                raise ValueError("a read spans two experts")
            arr = self._expert(name, e)[start - e * per: start - e * per + nbytes]
        else:
            arr = self._dense(name)[start:start + nbytes]
        return self._torch.from_numpy(arr.copy())

    # MmapSource surface --------------------------------------------------------
    def raw_bytes(self, name):
        return self._raw(name, 0, self.gguf.tensors[name].nbytes)

    def fetch(self, name, device="cpu", dtype=None):
        from neurostream.compute.quant import dequantize
        info = self.gguf.tensors[name]
        raw = self.raw_bytes(name).to(device)
        flat = dequantize(raw, info.dtype, info.n_elements, out_dtype=dtype or self._torch.float32)
        return flat.reshape(info.torch_shape)

    def raw_rows(self, name, start, end):
        from neurostream.io.source import row_geometry
        n_rows, _, rb = row_geometry(self.gguf.tensors[name])
        start, end = max(0, start), min(n_rows, end)
        return self._raw(name, start * rb, (end - start) * rb)

    def fetch_rows(self, name, start, end, device="cpu", dtype=None):
        from neurostream.compute.quant import dequantize
        from neurostream.io.source import row_geometry
        torch = self._torch
        dtype = dtype or torch.float32
        info = self.gguf.tensors[name]
        n_rows, elems, rb = row_geometry(info)
        start, end = max(0, start), min(n_rows, end)
        if start >= end:
            return torch.empty((0, elems), dtype=dtype, device=device)
        raw = self.raw_rows(name, start, end).to(device)
        return dequantize(raw, info.dtype, (end - start) * elems, out_dtype=dtype).reshape(end - start, elems)


class ReferenceDecode:
    """The reference's own GPT-OSS decode on the host cores, ready to time one token at a time.

    ``GptOssModel`` (``neurostream/model/gpt_oss.py``) over a ``TieredCache`` on ``device='cpu'``,
    fp32, ``block_rows=512``: float tensors (embedding, attention, router, norms, biases, LM head)
    admitted to the cache's resident float tier once, expert tensors served by the source one
    neuron block at a time (``stream_expert_ffn``), exactly the reference's stock neuron-block
    path.  The KV cache holds ``ctx`` synthetic positions per layer; each step decodes one token at
    position ``ctx`` from that same cache (the appended position is dropped after the step), so
    every step is the same work: one token at ``ctx`` context.
    With ``dense=False`` a step is instead one token through the MoE blocks only
    (``GptOssModel._ffn_block`` per layer), the workload of ``--workload moe``.
    """

    def __init__(self, shape, ctx: int = 2048, dense: bool = True, threads: int | None = None):
        import torch
        from neurostream.model.gpt_oss import GptOssConfig, GptOssModel
        from neurostream.model.qwen3 import KVCache
        from neurostream.residency.cache import TieredCache

        if threads:
            torch.set_num_threads(threads)
        self.shape, self.ctx, self.dense = shape, ctx, dense
        self.src = SynthGGUF(shape, dense=dense)
        self.cache = TieredCache(self.src, device="cpu", compute_dtype=torch.float32, vram_budget=1 << 44)
        for name, info in self.src.gguf.tensors.items():
            if info.dtype.name in ("F32", "F16", "BF16"):
                assert self.cache.admit_vram(name), name
        cfg = GptOssConfig(**shape.reference_config())
        self.model = GptOssModel(self.cache, cfg, device="cpu", dtype=torch.float32, block_rows=512)
        g = torch.Generator().manual_seed(5)
        self.k0 = [torch.randn(shape.n_head_kv, ctx, shape.head_dim, generator=g) for _ in range(shape.n_layer)]
        self.v0 = [torch.randn(shape.n_head_kv, ctx, shape.head_dim, generator=g) for _ in range(shape.n_layer)]
        self.kv = KVCache(shape.n_layer)
        self.x = torch.randn(1, shape.n_embd, generator=g)
        self.token = 1234
        self._torch = torch

    def step(self) -> float:
        """Seconds for one token (the reset of the KV cache to ``ctx`` positions is not timed)."""
        torch = self._torch
        self.kv.k, self.kv.v = list(self.k0), list(self.v0)
        self.kv.length = self.ctx
        with torch.no_grad():
            t0 = time.perf_counter()
            if self.dense:
                logits = self.model.forward(tokens=[self.token], kv=self.kv, start_pos=self.ctx)
                _ = float(logits[0, 0])
            else:
                x = self.x
                for l in range(self.shape.n_layer):
                    x = self.model._ffn_block(x, l)
                _ = float(x[0, 0])
            return time.perf_counter() - t0


def run_reference(args, rank, world):
    """``--impl reference``: the reference's own CPU implementation of the workload on the host cores.

    Every step is one whole token through the same model as the GPU arm (all layers, timed in
    full).  Rank 0 alone runs it; other ranks exit without work.  When the reference package is
    not installed on the box, the numpy oracle port of its MoE path is timed instead
    (``kind: port``).
    """
    if rank != 0:
        return None
    from nurostream_b200.shapes import GptOssShape

    shape = GptOssShape(n_layer=args.layers)
    threads = cpu_cores()
    dense = args.workload != "moe"
    cfg = full_decode_config(shape, world, args.ctx) if dense else workload_config(shape.moe_shape(), world)
    metric = METRIC
    if import_reference() is not None:
        t_setup = time.perf_counter()
        ref = ReferenceDecode(shape, ctx=args.ctx, dense=dense, threads=threads)
        for _ in range(args.warmup):
            ref.step()
        setup_s = time.perf_counter() - t_setup
        times = [ref.step() for _ in range(args.steps)]
        kind = "reference"
        sample = (f"every step one whole token through the reference's own GptOssModel "
                  f"({'forward: embedding, ' + str(shape.n_layer) + ' x (attention at ' + str(args.ctx) + ' context + MoE), LM head' if dense else str(shape.n_layer) + ' x _ffn_block'}) "
                  f"on device='cpu', fp32, block_rows=512, torch.set_num_threads({threads}); "
                  f"set-up and {args.warmup} warm-up tokens {setup_s:.0f} s untimed")
    else:
        mshape = shape.moe_shape()
        layers = [CpuLayer(mshape, l) for l in range(mshape.n_layer)]
        times = []
        with ThreadPoolExecutor(max_workers=threads) as pool:
            for i in range(args.warmup):
                layers[i % len(layers)].run(pool)
            for _ in range(args.steps):
                times.append(sum(L.run(pool) for L in layers))
        kind = "port"
        sample = ("reference package not installed on this box: every step one token through the numpy "
                  f"oracle port of the reference's {mshape.n_layer} MoE layers (attention and LM head not "
                  f"included), expert matrices on a {threads}-thread pool")
    step_s = statistics.mean(times)
    v = 1.0 / step_s
    return {
        "metric": metric, "impl": "reference", "value": round(v, 5), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_s * 1000, 2),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic", "config": cfg,
        "cpu_baseline": {"value": round(v, 5), "unit": UNIT, "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": round(v, 5), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=None, help="MoE layers (36 for decode, 94 for qwen3)")
    ap.add_argument("--cpu-layers", type=int, default=4)
    ap.add_argument("--ref-layers", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--combine", choices=["peer", "nccl"], default="peer",
                    help="expert-parallel combine of the decode step (N > 1): NVLink peer memory or NCCL")
    ap.add_argument("--workload", choices=["decode", "moe", "gemv", "qwen3", "prefill", "stream"], default="decode")
    ap.add_argument("--ctx", type=int, default=2048, help="KV-cache positions before the decoded token")
    ap.add_argument("--batch", type=int, default=1, help="token rows per decode step (--workload moe / qwen3)")
    ap.add_argument("--prefill-tokens", type=int, default=512)
    ap.add_argument("--gemv-case", default="", help="run one GEMV case only, e.g. MXFP4:14336")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.layers is None:
        args.layers = 94 if args.workload == "qwen3" else 36

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    group = None
    if args.workload == "gemv":
        for line in run_gemv_sweep(args):
            print(json.dumps(line), flush=True)
        return
    if args.workload == "stream":
        print(json.dumps(run_stream(args)), flush=True)
        return
    if args.impl == "reference":
        line = run_reference(args, rank, world)
    else:
        if world > 1:
            import datetime

            import torch
            import torch.distributed as dist
            torch.cuda.set_device(local_rank)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local_rank))
            group = dist.group.WORLD
        if args.workload == "decode":
            line = run_full_decode(args, rank, world, local_rank, group)
        elif args.workload == "prefill":
            line = run_prefill(args, rank, world, local_rank, group)
        else:
            line = run_ours(args, rank, world, local_rank, group)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
