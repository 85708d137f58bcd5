"""Expert parallelism across ranks, on CPU: two gloo processes.

Each rank holds the experts ``expert_range`` gives it, computes the identical
routing and only its local experts' weighted outputs (rank 0 adds the
residual), and one all-reduce(sum) combines the ranks -- the decomposition the
multi-GPU decoder uses (``nurostream_b200/decoder.py``), with the numpy oracle
standing in for the layer kernel.  The sum must equal the whole layer
(``neurostream/model/gpt_oss.py:123-177``), and every rank must route alike.
"""
from __future__ import annotations

import os
import socket
import sys
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CASES = [
    dict(E=8, k=2, T=2, H=64, F=64),    # both ranks hold routed experts
    dict(E=8, k=1, T=1, H=64, F=128),   # one routed expert: one rank contributes only zeros (+ residual)
]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, case: dict):
    sys.path.insert(0, ROOT)
    from nurostream_b200.decoder import expert_range
    from nurostream_b200.ggml import GGMLType
    from oracle import moe as omoe
    from tests.goldens import SynthLayer

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        c = dict(type=int(GGMLType.MXFP4), seed=3, arch="gpt-oss", bias=True, norm="synth", **case)
        L = SynthLayer(c)
        rows = L.rows_fn()
        lo, hi = expert_range(rank, world, L.E)

        # this rank's share: identical routing, local experts only, residual on rank 0
        h = omoe.rms_norm(L.x, L.norm_w, 1e-5)
        ids, w, _ = omoe.route_gptoss(h, L.router_w, L.router_b, L.k)
        act = lambda g, u: omoe.clamped_swiglu(g, u)
        part = np.zeros_like(L.x)
        for e in np.unique(ids):
            if not lo <= e < hi:
                continue
            mask = ids == e
            r = np.nonzero(mask.any(axis=-1))[0]
            we = (w * mask).sum(axis=-1, dtype=np.float32)[r, None]
            part[r] += we * omoe.expert_ffn(rows, int(e), h[r], act, L.biases)
        if rank == 0:
            part = part + L.x

        t = torch.from_numpy(part.astype(np.float32))
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        got = t.numpy()

        want, want_ids, _ = omoe.gptoss_ffn_block(L.x, L.norm_w, 1e-5, L.router_w, L.router_b, rows, L.biases, L.k)
        np.testing.assert_array_equal(ids, want_ids)
        gathered = [torch.zeros(ids.shape, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(ids.astype(np.int64)))
        for g in gathered:
            np.testing.assert_array_equal(g.numpy(), ids)
        # the ranks' sum regroups the expert terms: fp32 rounding only
        err = np.abs(got - want).max() / max(np.abs(want).max(), 1e-30)
        assert err <= 1e-5, f"rank {rank}: sum of expert-parallel shares off by {err:.2e}"
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", CASES)
def test_expert_parallel_shares_sum_to_the_layer(case):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), case), nprocs=world, join=True,
                       start_method="spawn")


def test_expert_range_splits_evenly_and_refuses_remainders():
    from nurostream_b200.decoder import expert_range

    spans = [expert_range(r, 4, 128) for r in range(4)]
    assert spans == [(0, 32), (32, 64), (64, 96), (96, 128)]
    with pytest.raises(ValueError):
        expert_range(0, 3, 128)
