"""Benchmark: batch-1 decode through the GPT-OSS-120B-shaped MoE hot path.

One step = one decode token through 36 MoE layers (RMSNorm -> router top-4 of
128 -> MXFP4 gate/up (2880x2880) -> clamped SwiGLU -> down -> weighted combine
-> residual), one fused launch per layer, captured in a CUDA graph.  Expert
bytes per step (1.9 GB) are far larger than L2 (126 MB), so no flush is needed.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  python bench.py --workload gemv [--steps K] [--warmup W]
  python bench.py --workload qwen3 [--layers L] [--steps K] [--warmup W]
  python bench.py --workload prefill [--layers L] [--steps K] [--warmup W]

``--workload gemv`` measures the dense dequant-GEMV sweep instead (batch 1,
K = 4096, N in {4096, 11008, 14336}, MXFP4 / Q4_K / Q8_0): one JSON line per
case, HBM GB/s against the measured copy peak, weight copies rotated so that
every launch streams from HBM.  ``--workload qwen3`` runs the decode step on
the Qwen3-235B-A22B shape instead (94 MoE layers, hidden 4096, 128 experts,
top-8, expert ffn 1536, Q4_K experts; MoE layers only).  ``--workload prefill``
runs 512 prompt tokens through the GPT-OSS-shaped MoE layers (config 5), each
layer as slices of a few tokens through the fused layer kernel.

N > 1 runs expert parallel under torchrun (experts split by index, one NCCL
all-reduce per layer).  ``--impl reference`` times the reference's CPU path
(the oracle port of it; the reference is Python and is not shipped to the GPU
box) on the host cores.  Prints ONE JSON line on rank 0.
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


def workload_config(shape, world):
    if shape.arch == "qwen3":
        return {
            "workload": (f"qwen3-235b-a22b-shape MoE decode path: {shape.n_layer} layers x (router softmax "
                         f"top-{shape.top_k}/{shape.n_expert} renormalised + Q4_K gate/up/down "
                         f"{shape.hidden}x{shape.expert_ffn} + silu*up + weighted combine + residual), batch 1"),
            "layers": shape.n_layer, "experts": shape.n_expert, "top_k": shape.top_k, "hidden": shape.hidden,
            "expert_ffn": shape.expert_ffn, "expert_format": "Q4_K (GGUF bytes, HBM-resident)",
            "router": "bf16 weight, no bias", "global_batch": 1, "seq_len": 1,
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
                 "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

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
    dec = MoeDecoder(shape, dev, rank, world, group, use_graph=not args.no_graph)
    H = shape.hidden
    npool = 64
    pool = torch.empty((npool, 1, H), device=dev, dtype=torch.float32)
    synth.fill_float(pool.view(-1), 777, 1)
    host_pool = pool.cpu().pin_memory()
    out_host = torch.empty((1, H), dtype=torch.float32, pin_memory=True)
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
    dec.release()

    if rank != 0:
        return None
    step_ms = ms / args.steps
    tok_s = 1000.0 / step_ms
    peak, peak_kind = measured_peaks()
    bytes_layer = shape.layer_bytes_per_token()
    per_launch_s = step_ms / 1000.0 / shape.n_layer
    achieved = bytes_layer / per_launch_s / 1e9 if world == 1 else bytes_layer / per_launch_s / 1e9
    line = {
        "metric": METRIC if shape.arch == "gpt-oss" else "decode tok/s at batch 1 (Qwen3-235B-A22B shape, MoE layers)",
        "value": round(tok_s, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(step_ms, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": f"{GGMLType(shape.ggml_type).name.lower()} weights, fp32 accumulate",
        "data": "synthetic (seeded splitmix64 GGUF bytes generated in HBM)",
        "config": workload_config(shape, world),
        "e2e": {"value": round(1000.0 * args.steps / ms_e2e, 2), "unit": UNIT,
                "h2d_bytes_per_step": H * 4, "d2h_bytes_per_step": H * 4},
        "gpu_launches": shape.n_layer * args.steps,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / (peak * (1 if world == 1 else world)), 4),
                     "traffic": None, "peak_kind": peak_kind,
                     "kernel": KERNEL if shape.arch == "gpt-oss" else "moe_layer_kernel",
                     "algorithmic_bytes_per_launch": bytes_layer,
                     "launch_ms": round(per_launch_s * 1000, 5),
                     "launch_ms_from": "CUDA events over the timed region / layer launches in it (one kernel "
                                       "per layer, back to back in the graph)"},
        "cuda_graph": graphed,
        "routing_identical_on_all_ranks": ids_ok,
    }
    traffic = ROOT / "profiles" / "moe_tc_kernel_traffic.json"
    if traffic.exists() and shape.arch == "gpt-oss":
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


def run_prefill(args):
    """Prefill of ``--prefill-tokens`` prompt tokens through the GPT-OSS-shaped MoE layers (config 5).

    Each layer runs as slices of 2 tokens through the tensor-core layer kernel (``MoeLayer.prefill``), all
    launches of a step captured in one CUDA graph.  Algorithmic bytes per layer: every expert that the
    step's tokens route to, read once (at T = 512 that is all 128), plus the router and activations.
    """
    import torch

    from nurostream_b200 import synth
    from nurostream_b200.decoder import MoeDecoder

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    shape = bench_shape(args)
    T, H = args.prefill_tokens, shape.hidden
    dec = MoeDecoder(shape, dev, 0, 1, None, use_graph=False, max_tokens=8)
    x = torch.empty((T, H), device=dev, dtype=torch.float32)
    synth.fill_float(x.view(-1), 778, 1)
    x_host = x.cpu().pin_memory()
    out_host = torch.empty((T, H), dtype=torch.float32, pin_memory=True)
    bufs = [torch.empty_like(x) for _ in range(2)]
    dec.prefill(x, bufs)                         # warm-up outside capture (settles the slice size)
    torch.cuda.synchronize()
    sl = dec.layers[0]._slice
    n_launch = -(-T // sl)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y = dec.prefill(x, bufs)
    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize()
    dec.check_device_errors()
    clocks = ClockSampler(0)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    # end to end: prompt in from pinned host memory, hidden states back, every step
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(args.steps):
        x.copy_(x_host, non_blocking=True)
        g.replay()
        out_host.copy_(y, non_blocking=True)
    f1.record()
    torch.cuda.synchronize()
    ms_e2e = f0.elapsed_time(f1) / args.steps
    clk = clocks.stop()
    dec.check_device_errors()
    peak, peak_kind = measured_peaks()
    E = shape.n_expert
    expert_bytes = shape.expert_bytes                      # one expert's gate + up + down rows
    layer_bytes = E * expert_bytes + E * H * 2 + 2 * T * H * 4   # all experts (T = 512 touches all 128)
    per_layer_s = ms / 1000.0 / shape.n_layer
    achieved = layer_bytes / per_layer_s / 1e9
    line = {
        "metric": "prefill tok/s (GPT-OSS-120B shape, 512-token prompt, MoE layers)", "value": round(T * 1000.0 / ms, 1),
        "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "mxfp4 weights, fp32 accumulate", "data": "synthetic (seeded splitmix64 GGUF bytes generated in HBM)",
        "config": {"workload": f"gpt-oss-120b-shape MoE prefill: {T} tokens x {shape.n_layer} layers, each layer as "
                               f"{n_launch} fused launches of {sl} tokens", "tokens": T, "layers": shape.n_layer,
                   "experts": E, "top_k": shape.top_k, "parallelism": "single",
                   "l2": "inputs larger than L2 (every layer streams its experts from HBM)"},
        "e2e": {"value": round(T * 1000.0 / ms_e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": T * H * 4,
                "d2h_bytes_per_step": T * H * 4},
        "gpu_launches": shape.n_layer * n_launch * args.steps,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None, "peak_kind": peak_kind,
                     "kernel": "moe_tc_kernel" if sl <= 2 else "moe_layer_kernel",
                     "algorithmic_bytes_per_layer": layer_bytes,
                     "note": "each slice streams the experts its tokens route to, so an expert is read once per "
                             "slice that uses it: HBM traffic is many times the algorithmic bytes"},
    }
    if clk:
        line["clocks"] = clk
    g = None
    return line


def run_reference(args, rank, world):
    """The reference's own CPU implementation of the path (oracle port), host cores only.

    Each step is a bounded sample: one token through one MoE layer (cycling
    over `--ref-layers` prepared layers), scaled to the full layer count.  The
    number of timed steps is capped so the run ends within a few minutes.
    """
    if rank != 0:
        return None
    from nurostream_b200.decoder import MoeShape

    shape = MoeShape(n_layer=args.layers)
    threads = cpu_cores()
    layers = [CpuLayer(shape, l) for l in range(args.ref_layers)]
    times = []
    budget_s, t_start = 150.0, time.perf_counter()
    with ThreadPoolExecutor(max_workers=threads) as pool:
        for i in range(args.warmup):
            layers[i % len(layers)].run(pool)
        for i in range(args.steps):
            times.append(layers[i % len(layers)].run(pool))
            if time.perf_counter() - t_start > budget_s:
                break
    s_per_tok = statistics.median(times) * shape.n_layer
    v = 1.0 / s_per_tok
    return {
        "metric": METRIC, "impl": "reference", "value": round(v, 5), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "steps_timed": len(times), "warmup": args.warmup,
        "ms_per_step": round(s_per_tok * 1000, 2), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded splitmix64 GGUF bytes)",
        "config": workload_config(shape, world),
        "cpu_baseline": {"value": round(v, 5), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": (f"each step: one token through one of {len(layers)} prepared MoE layers "
                                    f"(median over {len(times)} steps), scaled to {shape.n_layer} layers; "
                                    "numpy oracle of the reference CPU path, expert matrices on a "
                                    f"{threads}-thread pool")},
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
    ap.add_argument("--workload", choices=["decode", "gemv", "qwen3", "prefill"], default="decode")
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
    if args.workload == "prefill" and args.impl == "ours" and world == 1:
        print(json.dumps(run_prefill(args)), flush=True)
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
        line = run_ours(args, rank, world, local_rank, group)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
