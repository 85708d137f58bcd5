"""Expert-parallel combine through NVLink peer memory (``ns_peer_allreduce``).

Under expert parallelism each rank computes its local experts' partial of a MoE layer's output and
the layer output is the sum over ranks.  ``PeerReduce`` replaces the NCCL all-reduce of that small
vector (one per layer in decode) with one kernel: every rank stores its values into every rank's
receive slots as (value, call epoch) words and sums, in rank order, what arrived in its own memory
(identical bits on every rank).  The receive areas are allocated by their owners and mapped on the other ranks through CUDA
IPC handles exchanged once over the process group; plain peer stores and loads, no multicast
objects.  One process per GPU, all ranks on one node with peer access.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib


class PeerReduce:
    """In-place sum over the ranks of ``group`` of fp32 tensors of up to ``cap`` elements."""

    def __init__(self, cap: int, group=None, device=None):
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _lib.NS_MAX_PEERS:
            raise ValueError(f"world {self.world} > {_lib.NS_MAX_PEERS} peers")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.cap = int(cap)
        W = self.world
        slot_bytes = 2 * W * self.cap * 8  # (value, epoch) words, two parities
        self._own = []
        self._opened = []
        ptrs = []
        for nbytes in (slot_bytes, _lib.NS_PEER_MAX_CTAS * 4):
            p = C.c_void_p()
            _lib.call("ns_peer_alloc", nbytes, C.byref(p))
            self._own.append(p.value)
            ptrs.append(p.value)
        slots, self.ctr = ptrs
        h = C.create_string_buffer(64)
        _lib.call("ns_ipc_handle", slots, h)
        torch.cuda.synchronize(self.device)
        gathered = [None] * W
        dist.all_gather_object(gathered, h.raw, group=group)
        self.slots = [0] * W
        for r in range(W):
            if r == self.rank:
                self.slots[r] = slots
                continue
            p = C.c_void_p()
            _lib.call("ns_ipc_open", C.c_char_p(gathered[r]), C.byref(p))
            self._opened.append(p.value)
            self.slots[r] = p.value
        dist.barrier(group=group)

    def __call__(self, t: torch.Tensor) -> torch.Tensor:
        """t: contiguous fp32 CUDA tensor of <= cap elements; summed over the ranks in place."""
        if t.dtype != torch.float32 or not t.is_contiguous() or t.numel() > self.cap:
            raise ValueError("peer reduce takes a contiguous fp32 tensor within the slot capacity")
        p = _lib.PeerReduceParams()
        p.world, p.rank, p.n, p.cap, p.data, p.ctr = self.world, self.rank, t.numel(), self.cap, t.data_ptr(), self.ctr
        for r in range(self.world):
            p.slots[r] = self.slots[r]
        _lib.call("ns_peer_allreduce", C.byref(p), torch.cuda.current_stream(t.device).cuda_stream)
        return t

    def close(self) -> None:
        """Unmap the peers' areas and free this rank's, once every rank is done with every call (a
        barrier over the group first, while it is alive)."""
        import torch.distributed as dist

        torch.cuda.synchronize(self.device)
        if dist.is_initialized():
            dist.barrier(group=self.group)
        for p in self._opened:
            _lib.call("ns_ipc_close", p)
        for p in self._own:
            _lib.call("ns_peer_free", p)
        self._opened, self._own = [], []
