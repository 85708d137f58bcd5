"""Streamed (non-resident) projections: host-resident GGUF bytes through HBM, overlapped with the GEMV.

The reference streams a weight that is not in VRAM block by block (``stream_linear``,
``neurostream/compute/blockffn.py:57-241``, with ``BlockPrefetcher`` :278-393 queueing the reads):
each block's bytes reach the device with ``raw.to(device, non_blocking=True)`` from pageable host
memory, on the compute stream, and the fused GEMV runs after the copy has finished.  Here a block's
upload and the previous block's GEMV run at the same time:

* the host bytes are page-locked in place (``cudaHostRegister`` on the tensor the cache already
  holds: no second copy in host memory), so the copy engine reads them asynchronously;
* a dedicated copy stream uploads block i into slot i % depth of a ring of device buffers while the
  compute stream runs ``ns_gemv`` on block i - 1;
* CUDA events order the two: a slot is refilled only after the GEMV that read it has run
  (``slot free``), and a GEMV starts only after its block has landed (``slot full``).  Nothing
  synchronises the host.

``StreamedGemv`` is the executor; ``streamed_linear`` is a ``stream_linear``-shaped entry point for
tensors held in a ``TieredCache``'s RAM tier (quantized bytes on the host).  ``install(streamed=True)``
routes the reference's ``stream_linear`` to it for exactly those tensors and leaves every other call
on the reference's own code.
"""
from __future__ import annotations

import torch

from . import _lib
from .fused import ns_dtype
from .ggml import FUSED_TYPES, GGMLType, as_ggml_type, row_bytes

_REGISTERED: dict = {}  # data_ptr -> (tensor, nbytes) page-locked in place by this module


def pin_in_place(t: torch.Tensor) -> torch.Tensor:
    """Page-lock a CPU tensor's memory in place (once per allocation); returns the tensor.

    An already pinned tensor is returned unchanged.  Registration lasts as long as the process (the
    cache that owns the bytes keeps them alive).
    """
    if t.is_cuda:
        raise ValueError("pin_in_place takes host tensors")
    if t.is_pinned():
        return t
    t = t.contiguous()
    key = t.data_ptr()
    if key not in _REGISTERED:
        rt = torch.cuda.cudart()
        err = rt.cudaHostRegister(key, t.numel() * t.element_size(), 0)
        if int(err) != 0:
            raise RuntimeError(f"cudaHostRegister failed ({int(err)})")
        _REGISTERED[key] = (t, t.numel() * t.element_size())
    return t


class StreamedGemv:
    """y = x @ W.T for a weight whose GGUF bytes live in host memory, in blocks of rows.

    device: the CUDA device; block_bytes: the ring's slot size (a block is as many whole rows as fit);
    depth: slots in the ring (blocks in flight).
    """

    def __init__(self, device, block_bytes: int = 8 << 20, depth: int = 3):
        self.device = torch.device(device)
        self.block_bytes = int(block_bytes)
        self.depth = max(2, int(depth))
        self.ring = [torch.empty(self.block_bytes, dtype=torch.uint8, device=self.device) for _ in range(self.depth)]
        self.copy_stream = torch.cuda.Stream(self.device)
        self.full = [torch.cuda.Event() for _ in range(self.depth)]
        self.free = [torch.cuda.Event() for _ in range(self.depth)]
        self._used = [False] * self.depth

    def __call__(self, host_raw: torch.Tensor, dtype, x: torch.Tensor, n_rows: int, K: int,
                 out: torch.Tensor | None = None, row_start: int = 0, row_end: int | None = None,
                 block_rows: int | None = None, out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """x (T, K) on the device; host_raw: the whole tensor's bytes (n_rows rows) in host memory.

        Returns (T, row_end - row_start) in ``out_dtype`` (or writes ``out``), stream-ordered on the
        current stream of the device.
        """
        t = as_ggml_type(dtype)
        if t not in FUSED_TYPES:
            raise KeyError(t)
        rb = row_bytes(t, K)
        row_end = n_rows if row_end is None else min(n_rows, row_end)
        row_start = max(0, row_start)
        if host_raw.numel() < n_rows * rb:
            raise ValueError(f"host buffer has {host_raw.numel()} bytes; {n_rows} rows need {n_rows * rb}")
        host_raw = pin_in_place(host_raw.reshape(-1))
        xf = x.reshape(-1, K)
        if not xf.is_contiguous():
            xf = xf.contiguous()
        T = xf.shape[0]
        window = max(0, row_end - row_start)
        if out is None:
            out = torch.empty((T, window), device=self.device, dtype=out_dtype)
        if window == 0:
            return out
        per = self.block_bytes // rb
        if per < 1:
            raise ValueError(f"one row ({rb} bytes) exceeds the ring slot ({self.block_bytes} bytes)")
        if block_rows:
            per = min(per, int(block_rows))
        compute = torch.cuda.current_stream(self.device)
        # the copy stream may reuse a slot only after the GEMVs issued so far on the compute stream
        base = torch.cuda.Event()
        base.record(compute)
        self.copy_stream.wait_event(base)
        i = 0
        for lo in range(row_start, row_end, per):
            hi = min(lo + per, row_end)
            slot = i % self.depth
            nbytes = (hi - lo) * rb
            with torch.cuda.stream(self.copy_stream):
                if self._used[slot]:
                    self.copy_stream.wait_event(self.free[slot])
                self.ring[slot][:nbytes].copy_(host_raw[lo * rb:hi * rb], non_blocking=True)
                self.full[slot].record(self.copy_stream)
            compute.wait_event(self.full[slot])
            y = out[:, lo - row_start:hi - row_start]
            _lib.call("ns_gemv", self.ring[slot].data_ptr(), nbytes, int(t), hi - lo, K, xf.data_ptr(),
                      ns_dtype(xf.dtype), K, T, y.data_ptr(), ns_dtype(out.dtype), out.stride(0),
                      compute.cuda_stream)
            self.free[slot].record(compute)
            self._used[slot] = True
            i += 1
        return out


_EXECUTORS: dict = {}


def executor(device) -> StreamedGemv:
    dev = torch.device(device)
    if dev.index is None:
        dev = torch.device(dev.type, torch.cuda.current_device())
    key = (dev.type, dev.index)
    if key not in _EXECUTORS:
        _EXECUTORS[key] = StreamedGemv(dev)
    return _EXECUTORS[key]


def ram_tier_bytes(provider, name: str):
    """(host uint8 bytes, GGMLType) of a tensor held quantized in a TieredCache's RAM tier, else None."""
    ram = getattr(provider, "_ram", None)
    if ram is None or name in getattr(provider, "_vram", {}):
        return None
    e = ram.get(name)
    if e is None or e.ready or e.payload.is_cuda:
        return None
    return e.payload, e.dtype


def streamed_linear(provider, name: str, x: torch.Tensor, block_rows: int, device, dtype=torch.float32,
                    out: torch.Tensor | None = None, row_start: int = 0, row_end: int | None = None):
    """``stream_linear`` for a RAM-tier quantized tensor: x @ W[row_start:row_end].T with the blocks
    uploaded on a copy stream while the previous block's GEMV runs; returns None when the tensor is
    not in the RAM tier or its type has no fused GEMV (the caller then takes the reference's path).
    Counts the RAM-tier hit as the reference's ``fetch_rows`` does (``residency/cache.py:390-399``)."""
    hit = ram_tier_bytes(provider, name)
    if hit is None:
        return None
    raw, t = hit
    try:
        gt = GGMLType(int(t))
    except ValueError:
        return None
    if gt not in FUSED_TYPES:
        return None
    from neurostream.io.source import row_geometry  # the reference's own geometry (imported lazily)

    n_rows, row_elems, _ = row_geometry(provider.gguf.tensors[name])
    provider._ram.move_to_end(name)
    provider.stats.ram_hits += 1
    return executor(device)(raw, gt, x, n_rows, row_elems, out=out, row_start=row_start, row_end=row_end,
                            block_rows=block_rows, out_dtype=dtype)
