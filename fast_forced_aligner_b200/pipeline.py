"""Batches that live in host memory, aligned with their copies overlapped.

``align`` and ``align_packed`` take emissions already on the GPU, as the
reference's ``align`` does (alignment.py:346-502).  When batches arrive in
host memory one after another (a decoder's output, files, a network feed),
the PCIe copies of a batch can overlap the alignment of its neighbours.
``AlignStream`` does that with three CUDA streams: batch k+1's inputs cross
host->device on one, batch k aligns on another (waiting only for its own
inputs), and batch k-1's labels, scores and status return on a third.
Device buffers come from PyTorch's caching allocator with ``record_stream``,
so a buffer is reused only once every stream that touched it has passed it;
host results are pinned tensors from PyTorch's caching host allocator.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import torch
from torch import Tensor

from .alignment import Mode, align_packed


@dataclass(frozen=True)
class HostAlignment:
    """Results of one batch in pinned host memory (fields as in AlignmentBatch)."""

    lengths: tuple[int, ...]
    labels: Tensor      # int64 [sum T]
    scores: Tensor      # float32 [sum T]
    status: Tensor      # int32 [B]
    objective: Tensor   # float32 [B]

    @property
    def paths(self) -> tuple[Tensor, ...]:
        return self.labels.split(self.lengths)


class PendingAlignment:
    """A submitted batch; ``result()`` waits for its results to reach the host."""

    def __init__(self, done: torch.cuda.Event, result: HostAlignment):
        self._done = done
        self._result = result

    def ready(self) -> bool:
        return self._done.query()

    def result(self) -> HostAlignment:
        self._done.synchronize()
        return self._result


class AlignStream:
    """Align host-resident packed batches with copy/compute overlap on one GPU.

    ``submit`` enqueues one batch and returns at once; batches complete in
    submission order.  Inputs should be pinned (``Tensor.pin_memory()``) for
    the copies to be asynchronous; they must stay unchanged until the batch's
    ``result()`` returns.
    """

    def __init__(self, device: torch.device | str | int | None = None):
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        elif isinstance(device, int):
            device = torch.device("cuda", device)
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("AlignStream needs a CUDA device")
        with torch.cuda.device(self.device):
            self.copy_in = torch.cuda.Stream()
            self.compute = torch.cuda.Stream()
            self.copy_out = torch.cuda.Stream()

    @torch.inference_mode()
    def submit(self, emissions: Tensor, frames, targets: Tensor, tokens, *,
               blank_id: int | Sequence[int] = 0, mode: Mode = "optimized",
               check_inputs: bool = True, from_logits: bool = False) -> PendingAlignment:
        """Enqueue host emissions ``[N, V]`` fp32 and targets ``[M]`` int64
        (packed as for ``align_packed``; with ``from_logits``, fp32 or bf16
        logits, which halves the host->device bytes in bf16); returns a
        PendingAlignment."""
        for t, what in ((emissions, "emissions"), (targets, "targets")):
            if not isinstance(t, Tensor) or t.device.type != "cpu":
                raise ValueError(f"{what} must be a host tensor")
        dev = self.device
        with torch.cuda.device(dev):
            with torch.cuda.stream(self.copy_in):
                e = emissions.to(dev, non_blocking=True)
                t = targets.to(dev, non_blocking=True)
                inputs_ready = torch.cuda.Event()
                inputs_ready.record(self.copy_in)
            self.compute.wait_event(inputs_ready)
            with torch.cuda.stream(self.compute):
                batch = align_packed(e, frames, t, tokens, blank_id=blank_id, mode=mode,
                                     check_inputs=check_inputs, from_logits=from_logits)
                e.record_stream(self.compute)
                t.record_stream(self.compute)
                aligned = torch.cuda.Event()
                aligned.record(self.compute)
            self.copy_out.wait_event(aligned)
            with torch.cuda.stream(self.copy_out):
                fields = (batch.labels, batch.scores, batch.status, batch.objective)
                host = _copy_to_host(fields, self.copy_out)
                done = torch.cuda.Event()
                done.record(self.copy_out)
        return PendingAlignment(done, HostAlignment(batch.lengths, *host))


def _copy_to_host(fields, stream) -> list[Tensor]:
    """Pinned host copies of device tensors, enqueued on `stream`.  The align
    op carves its outputs from one allocation, so one copy of the span that
    holds them (one pinned buffer, one transfer) replaces a copy per field;
    fields that do not share an allocation are copied one by one."""
    storage = fields[0].untyped_storage()
    spans = []
    for x in fields:
        if x.untyped_storage().data_ptr() != storage.data_ptr() or not x.is_contiguous():
            spans = None
            break
        start = x.storage_offset() * x.element_size()
        spans.append((start, start + x.numel() * x.element_size()))
    if spans is None or any(s % 8 for s, _ in spans):
        host = [torch.empty(x.shape, dtype=x.dtype, pin_memory=True) for x in fields]
        for h, x in zip(host, fields):
            h.copy_(x, non_blocking=True)
            x.record_stream(stream)
        return host
    lo, hi = min(s for s, _ in spans), max(e for _, e in spans)
    span = torch.empty(0, dtype=torch.uint8, device=fields[0].device).set_(storage, lo, (hi - lo,))
    pinned = torch.empty(hi - lo, dtype=torch.uint8, pin_memory=True)
    pinned.copy_(span, non_blocking=True)
    span.record_stream(stream)
    return [pinned[s - lo:e - lo].view(x.dtype).view(x.shape) for (s, e), x in zip(spans, fields)]
