"""Expert-parallel combine through NVLink peer memory (ns_peer_allreduce), on 2 GPUs: the sum over
ranks equals the rank-ordered fp32 sum bit for bit on every rank, inside and outside a CUDA graph,
and the 2-rank GPT-OSS decoder with the peer combine gives the 1-rank logits.  Skipped with fewer
than 2 GPUs."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

needs_two = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                               reason="needs 2 GPUs")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    return dist


def _sum_worker(rank, world, port, failures):
    dist = _init(rank, world, port)
    try:
        from nurostream_b200 import _lib
        from nurostream_b200.peer import PeerReduce
        n = 2880
        pr = PeerReduce(4 * n)
        for it, size in enumerate((n, 7, 4 * n, 1)):
            vals = [np.random.default_rng(100 * it + r).standard_normal(size).astype(np.float32) for r in range(world)]
            want = np.zeros(size, np.float32)
            for r in range(world):
                want = (want + vals[r]).astype(np.float32)
            t = torch.from_numpy(vals[rank]).cuda()
            pr(t)
            torch.cuda.synchronize()
            np.testing.assert_array_equal(t.cpu().numpy(), want)
        # captured once, replayed: the per-CTA call counters advance on the device
        t = torch.empty(n, device="cuda")
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            pr(t)
        for rep in range(3):
            vals = [np.full(n, 0.5 * (r + 1) + rep, np.float32) for r in range(world)]
            t.copy_(torch.from_numpy(vals[rank]))
            g.replay()
            torch.cuda.synchronize()
            want = np.zeros(n, np.float32)
            for r in range(world):
                want = (want + vals[r]).astype(np.float32)
            np.testing.assert_array_equal(t.cpu().numpy(), want)
        g = None
        assert _lib.device_error() == 0
        pr.close()
    except Exception as e:  # reported by the parent
        failures.put(f"rank {rank}: {e!r}")
        raise
    finally:
        dist.destroy_process_group()


def _decoder_worker(rank, world, port, failures):
    dist = _init(rank, world, port)
    try:
        from nurostream_b200 import _lib
        from nurostream_b200.gptoss import GptOssDecoder
        from nurostream_b200.shapes import GptOssShape
        shape = GptOssShape(n_layer=2, vocab_size=4096)
        dec = GptOssDecoder(shape, "cuda", ctx=64, max_ctx=128, rank=rank, world=world, group=dist.group.WORLD)
        dec.set_token(77, 64)
        assert dec.capture()
        got = dec.step().cpu().numpy().copy()
        dec.release()
        if rank == 0:
            ref = GptOssDecoder(shape, "cuda", ctx=64, max_ctx=128, use_graph=False)
            ref.set_token(77, 64)
            want = ref.step().cpu().numpy()
            err = np.abs(got - want).max() / np.abs(want).max()
            assert err < 1e-5, f"2-rank logits vs 1-rank: {err:.2e}"
        assert _lib.device_error() == 0
    except Exception as e:
        failures.put(f"rank {rank}: {e!r}")
        raise
    finally:
        dist.destroy_process_group()


def _spawn(fn):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    failures = ctx.Queue()
    mp.spawn(fn, args=(2, _free_port(), failures), nprocs=2, join=True)
    assert failures.empty()


@needs_two
def test_peer_allreduce_two_ranks():
    _spawn(_sum_worker)


@needs_two
def test_gptoss_decoder_two_ranks_peer_combine_matches_one_rank():
    _spawn(_decoder_worker)
