"""Records spread over several GPUs of one box, with no collective on the path.

Alignment records are independent: a batch spreads over devices by assigning
whole records, and no data ever moves between GPUs while they align.  Two ways
to run that are provided:

  * one process per GPU (torchrun): every rank computes the same
    length-balanced partition from the batch's host metadata with
    ``shard_of_rank`` and aligns only its own records; ``reduce_over_ranks``
    is the host-side helper a caller uses for a timing or status summary
    (never on the data path);
  * one process driving several GPUs: ``align_sharded`` partitions, stages
    each shard on its device, aligns every shard from its own host thread on
    that device's current stream, and returns the per-device batches, which
    ``ShardedAlignment.gather`` can collect on one device.

The reference runs on one device only (its ``align`` uses the inputs' device,
alignment.py:346-502); this module adds the partition the multi-GPU
configuration asks for: longest-processing-time bin packing on a cost model
of the DP work of each record.
"""
from __future__ import annotations

import threading
from dataclasses import dataclass
from typing import Sequence

import numpy as np
import torch
from torch import Tensor

from .alignment import AlignmentBatch, Mode, align

# A frame costs its trellis cells plus a fixed per-frame share (emission row
# staging, traceback and output writes), in cell units.
_FRAME_COST = 64


def record_costs(frames: Sequence[int], tokens: Sequence[int]) -> np.ndarray:
    """Estimated device work of each record: ``T * (2U + 1) + 64 T`` cells."""
    T = np.asarray(frames, dtype=np.int64)
    U = np.asarray(tokens, dtype=np.int64)
    if T.shape != U.shape or T.ndim != 1:
        raise ValueError("frames and tokens must be matching 1-D sequences")
    return T * (2 * U + 1) + _FRAME_COST * T


def partition_records(costs: Sequence[int], shards: int) -> list[np.ndarray]:
    """Longest-processing-time bin packing of records onto ``shards`` bins.

    Records are taken in decreasing cost (ties by index) and each goes to the
    least-loaded bin (ties to the lowest bin), so every process that calls
    this with the same costs gets the same answer.  The heaviest bin is at
    most 4/3 of the optimum, and at most the mean load plus one record's cost.
    Returns the record indices of each bin in increasing order.
    """
    if shards < 1:
        raise ValueError("shards must be >= 1")
    c = np.asarray(costs, dtype=np.int64)
    order = np.lexsort((np.arange(c.size), -c))
    loads = np.zeros(shards, dtype=np.int64)
    owner = np.empty(c.size, dtype=np.int64)
    if shards == 1:
        owner[:] = 0
    else:
        import heapq
        heap = [(0, b) for b in range(shards)]
        for i in order:
            load, b = heapq.heappop(heap)
            owner[i] = b
            load += int(c[i])
            loads[b] = load
            heapq.heappush(heap, (load, b))
    return [np.flatnonzero(owner == b) for b in range(shards)]


def shard_of_rank(frames: Sequence[int], tokens: Sequence[int], rank: int, world: int) -> np.ndarray:
    """Record indices rank ``rank`` of ``world`` aligns (same on every rank)."""
    if not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    return partition_records(record_costs(frames, tokens), world)[rank]


def reduce_over_ranks(value: float, op: str = "max", device: torch.device | None = None) -> float:
    """Max or sum of a host scalar over the ranks of the default process group.

    Returns ``value`` unchanged when torch.distributed is not initialised.
    ``device`` is where the one-element exchange tensor lives: the rank's GPU
    for NCCL, the CPU (None) for gloo.
    """
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return value
    ops = {"max": dist.ReduceOp.MAX, "sum": dist.ReduceOp.SUM}
    if op not in ops:
        raise ValueError("op must be 'max' or 'sum'")
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=ops[op])
    return float(t.item())


@dataclass(frozen=True)
class Shard:
    device: torch.device
    records: np.ndarray       # indices into the caller's batch, increasing
    batch: AlignmentBatch     # outputs of those records on ``device``


@dataclass(frozen=True)
class ShardedAlignment:
    """Per-device results of ``align_sharded``; outputs stay where computed."""

    count: int
    lengths: tuple[int, ...]
    shards: tuple[Shard, ...]

    def paths(self) -> list[Tensor]:
        """Per-record label tensors in the caller's order (on their devices)."""
        out: list[Tensor | None] = [None] * self.count
        for shard in self.shards:
            for i, p in zip(shard.records.tolist(), shard.batch.paths):
                out[i] = p
        return out  # type: ignore[return-value]

    def status(self) -> Tensor:
        """int32 ``[B]`` statuses in the caller's order, on the CPU (synchronises)."""
        out = torch.empty(self.count, dtype=torch.int32)
        for shard in self.shards:
            out[torch.from_numpy(shard.records)] = shard.batch.status.cpu()
        return out

    def raise_for_status(self) -> None:
        """``AlignmentBatch.raise_for_status`` with the caller's batch indices."""
        self.gather(torch.device("cpu")).raise_for_status()

    def gather(self, device: torch.device | str) -> AlignmentBatch:
        """One AlignmentBatch in the caller's record order on ``device``.

        Copies every shard's outputs to ``device`` (peer copies between GPUs);
        this is the optional gather, off the alignment path.
        """
        device = torch.device(device)
        starts = np.concatenate([[0], np.cumsum(self.lengths)]).astype(np.int64)
        total = int(starts[-1])
        labels = torch.empty(total, dtype=torch.int64, device=device)
        scores = torch.empty(total, dtype=torch.float32, device=device)
        per_record = {
            "status": (torch.int32, ()), "objective": (torch.float32, ()),
            "stitched": (torch.int32, ()), "repair_passes": (torch.int32, ()),
            "repaired_frames": (torch.int64, ()), "shortcut_stats": (torch.int64, (3,)),
            "routing_stats": (torch.int32, (3,)),
        }
        fields = {name: torch.empty((self.count, *shape), dtype=dtype, device=device)
                  for name, (dtype, shape) in per_record.items()}
        any_reuse = any(s.batch.reuse_stats.shape[0] for s in self.shards)
        reuse = torch.zeros((self.count if any_reuse else 0, 4), dtype=torch.int64, device=device)
        for shard in self.shards:
            idx = torch.from_numpy(shard.records).to(device)
            b = shard.batch
            # Frame rows of this shard's records, in the caller's packing.
            spans = [np.arange(starts[i], starts[i + 1]) for i in shard.records.tolist()]
            rows = torch.from_numpy(np.concatenate(spans) if spans else np.zeros(0, np.int64)).to(device)
            labels[rows] = b.labels.to(device)
            scores[rows] = b.scores.to(device)
            for name in per_record:
                fields[name][idx] = getattr(b, name).to(device)
            if b.reuse_stats.shape[0]:
                reuse[idx] = b.reuse_stats.to(device)
        return AlignmentBatch(self.lengths, labels, scores, fields["status"], fields["objective"],
                              fields["stitched"], fields["repair_passes"], fields["repaired_frames"],
                              fields["shortcut_stats"], fields["routing_stats"], reuse)


def align_sharded(
    emissions: Sequence[Tensor], targets: Sequence[Tensor], *,
    blank_id: int | Sequence[int] = 0, mode: Mode = "optimized", check_inputs: bool = True,
    devices: Sequence[torch.device | str | int] | None = None, from_logits: bool = False,
) -> ShardedAlignment:
    """Align a batch over several GPUs of this process, no collective involved.

    With ``devices`` None the records stay where they are: each device that
    holds records aligns those.  Otherwise the batch is partitioned over
    ``devices`` by ``partition_records`` and each record is copied to its
    device (inputs may be CPU tensors; pinned ones copy asynchronously).
    Every device's shard is aligned from its own host thread on that device's
    current stream.  Arguments (``from_logits`` included) and per-record
    results are those of ``align``; errors of any shard are raised here.
    """
    count = len(emissions)
    if count == 0 or len(targets) != count:
        raise ValueError("provide 1..65535 matching emissions, targets, and blank IDs")
    blanks = [int(blank_id)] * count if isinstance(blank_id, int) and not isinstance(blank_id, bool) \
        else list(blank_id)  # type: ignore[arg-type]
    if len(blanks) != count:
        raise ValueError("provide 1..65535 matching emissions, targets, and blank IDs")
    lengths = tuple(int(e.shape[0]) for e in emissions)
    if devices is None:
        groups: dict[torch.device, list[int]] = {}
        for i, e in enumerate(emissions):
            groups.setdefault(e.device, []).append(i)
        plan = [(d, np.asarray(ix, dtype=np.int64)) for d, ix in groups.items()]
    else:
        devs = [torch.device("cuda", d) if isinstance(d, int) else torch.device(d) for d in devices]
        if not devs:
            raise ValueError("devices must name at least one CUDA device")
        costs = record_costs(lengths, [int(t.shape[0]) for t in targets])
        plan = [(d, ix) for d, ix in zip(devs, partition_records(costs, len(devs))) if ix.size]

    results: list[AlignmentBatch | None] = [None] * len(plan)
    errors: list[BaseException | None] = [None] * len(plan)

    def work(k: int) -> None:
        device, ix = plan[k]
        try:
            with torch.cuda.device(device):
                es = [emissions[i].to(device, non_blocking=True) for i in ix.tolist()]
                ts = [targets[i].to(device, non_blocking=True) for i in ix.tolist()]
                results[k] = align(es, ts, blank_id=[blanks[i] for i in ix.tolist()], mode=mode,
                                   check_inputs=check_inputs, from_logits=from_logits)
        except BaseException as error:  # re-raised on the calling thread
            errors[k] = error

    threads = [threading.Thread(target=work, args=(k,)) for k in range(1, len(plan))]
    for t in threads:
        t.start()
    work(0)
    for t in threads:
        t.join()
    for error in errors:
        if error is not None:
            raise error
    shards = tuple(Shard(d, ix, r) for (d, ix), r in zip(plan, results))  # type: ignore[misc]
    return ShardedAlignment(count, lengths, shards)
