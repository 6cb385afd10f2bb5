"""Host <-> device copies for the CPU-tensor API.

The six-function API takes and returns ordinary (pageable) CPU tensors.  A
plain .cpu() of a device tensor into fresh pageable memory runs at ~2 GB/s
on the B200 hosts (the driver stages it and faults the destination pages in
one thread); a weight's dict5 (9.5625 B per element) then costs far more than
its calibration.  Here each copy goes through two pinned 32 MiB buffers: the
DMA of one chunk (~50 GB/s) overlaps torch's multi-threaded copy of the other
chunk into (or out of) the pageable tensor, ~10x faster end to end.  The
buffers are per (device, host thread), so concurrent calibrations on several
threads never share one.
"""
from __future__ import annotations

import threading

import torch

CHUNK = 32 << 20          # bytes per pinned buffer
SMALL = 1 << 20           # below this a direct copy is cheaper

_TLS = threading.local()


class _Ring:
    def __init__(self, dev: torch.device):
        self.bufs = [torch.empty(CHUNK, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
        self.events = [torch.cuda.Event() for _ in range(2)]
        self.stream = torch.cuda.Stream(device=dev)


def _ring(dev: torch.device) -> _Ring:
    rings = getattr(_TLS, "rings", None)
    if rings is None:
        rings = _TLS.rings = {}
    key = dev.index
    if key not in rings:
        rings[key] = _Ring(dev)
    return rings[key]


def _bytes(t: torch.Tensor) -> torch.Tensor:
    return t.reshape(-1).view(torch.uint8)


def to_host(t: torch.Tensor) -> torch.Tensor:
    """A pageable CPU copy of a CUDA tensor (contiguous, same shape and dtype),
    ordered after the work already queued on the current stream."""
    if not t.is_cuda:
        return t
    t = t.contiguous()
    n = t.numel() * t.element_size()
    if n < SMALL:
        return t.cpu()
    dev = t.device
    r = _ring(dev)
    out = torch.empty(t.shape, dtype=t.dtype)
    src, dst = _bytes(t), _bytes(out)
    r.stream.wait_stream(torch.cuda.current_stream(dev))
    chunks = (n + CHUNK - 1) // CHUNK

    def fetch(i):
        m = min(CHUNK, n - i * CHUNK)
        with torch.cuda.stream(r.stream):
            r.bufs[i % 2][:m].copy_(src[i * CHUNK:i * CHUNK + m], non_blocking=True)
            r.events[i % 2].record(r.stream)

    fetch(0)
    for i in range(chunks):
        if i + 1 < chunks:
            fetch(i + 1)          # its buffer was drained by the copy of chunk i - 1
        r.events[i % 2].synchronize()
        m = min(CHUNK, n - i * CHUNK)
        dst[i * CHUNK:i * CHUNK + m].copy_(r.bufs[i % 2][:m])
    src.record_stream(r.stream)
    return out


def to_device(t: torch.Tensor, dev: torch.device) -> torch.Tensor:
    """A CUDA copy of a CPU tensor on `dev`, usable by work queued on the
    current stream after this call returns."""
    if t.is_cuda:
        return t.to(dev)
    t = t.contiguous()
    n = t.numel() * t.element_size()
    if n < SMALL or t.is_pinned():
        return t.to(dev, non_blocking=t.is_pinned())
    r = _ring(dev)
    out = torch.empty(t.shape, dtype=t.dtype, device=dev)
    src, dst = _bytes(t), _bytes(out)
    cur = torch.cuda.current_stream(dev)
    r.stream.wait_stream(cur)     # `out` may reuse memory the current stream still reads
    chunks = (n + CHUNK - 1) // CHUNK
    for i in range(chunks):
        b = i % 2
        if i >= 2:
            r.events[b].synchronize()     # the upload of chunk i - 2 has left this buffer
        m = min(CHUNK, n - i * CHUNK)
        r.bufs[b][:m].copy_(src[i * CHUNK:i * CHUNK + m])
        with torch.cuda.stream(r.stream):
            dst[i * CHUNK:i * CHUNK + m].copy_(r.bufs[b][:m], non_blocking=True)
            r.events[b].record(r.stream)
    cur.wait_stream(r.stream)
    out.record_stream(r.stream)
    # the ring buffers are reused by the next call only after its events
    for e in r.events:
        e.synchronize()
    return out
