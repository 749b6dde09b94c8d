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

import os
from dataclasses import dataclass
from typing import Sequence

import torch
from torch import Tensor

from .alignment import Mode, _input_format, _mode, _packed_counts, load_extension


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
        if self.device.index is None:  # "cuda": the current device
            self.device = torch.device("cuda", torch.cuda.current_device())
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
        PendingAlignment.  The copies, the align and the copy back are
        enqueued by one native call (``torch.ops.ffa_b200.align_stream``)."""
        for t, what in ((emissions, "emissions"), (targets, "targets")):
            if not isinstance(t, Tensor) or t.device.type != "cpu":
                raise ValueError(f"{what} must be a host tensor")
        code = _mode(mode, check_inputs, from_logits)
        fmt = _input_format(emissions, from_logits)
        frames_t, tokens_t, blanks_t = _packed_counts(frames, tokens, blank_id)
        load_extension()
        labels, scores, status, objective = torch.ops.ffa_b200.align_stream(
            emissions, frames_t, targets, tokens_t, blanks_t, code, check_inputs, fmt, self.device.index,
            self.copy_in.stream_id, self.compute.stream_id, self.copy_out.stream_id)
        done = torch.cuda.Event()
        done.record(self.copy_out)
        return PendingAlignment(done, HostAlignment(tuple(frames_t.tolist()), labels, scores, status, objective))


def parse_cpulist(text: str) -> list[int]:
    """CPUs of a Linux cpulist string ("0-3,8,10-11")."""
    cpus: list[int] = []
    for part in text.strip().split(","):
        if not part:
            continue
        lo, _, hi = part.partition("-")
        cpus.extend(range(int(lo), int(hi or lo) + 1))
    return cpus


def bind_host_to_device(device: torch.device | str | int) -> list[int] | None:
    """Restrict the calling process to the CPUs of the NUMA node that holds
    `device`'s PCIe link (Linux sysfs), so that pinned host batches -- placed
    by the first thread to touch them -- and the thread that submits them sit
    next to the GPU.  With one process per GPU, host-to-device copies then do
    not cross the socket link.  Returns the CPUs, or None (and changes
    nothing) where the node is unknown."""
    try:
        props = torch.cuda.get_device_properties(torch.device(device))
        bdf = f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bdf}/numa_node") as f:
            node = int(f.read())
        if node < 0:
            return None
        with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
            allowed = os.sched_getaffinity(0)
            cpus = [c for c in parse_cpulist(f.read()) if c in allowed]
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return cpus
    except (OSError, ValueError, AttributeError, RuntimeError, AssertionError):
        return None
