"""Public API of the B200-native CTC forced aligner.

A drop-in for the reference's Python surface (brthor/fast-forced-aligner,
src/fast_forced_aligner/alignment.py): the same names, keyword arguments,
result fields, status codes, error classes and messages.  The work happens in
the native library: torch.ops.ffa_b200.* (csrc/ffa_torch.cpp) over the C ABI of
libffa_b200.so (include/ffa_b200.h), whose sm_100a kernels run the DP.  There
is no CPU fallback: without the native library every entry point raises.
"""
from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from functools import lru_cache
from pathlib import Path
from typing import Literal

import numpy as np
import torch
from torch import Tensor

Mode = Literal["optimized", "conventional"]
_PACKAGE = Path(__file__).resolve().parent
_MODES = {"conventional": 0, "optimized": 1}


@lru_cache(maxsize=1)
def load_extension() -> None:
    """Load the native library and register the ``torch.ops.ffa_b200`` ops.

    Mirrors the reference's ``load_extension`` (alignment.py:15-63): the same
    prerequisites and RuntimeError messages.  The native library is built
    in-tree (``python -m fast_forced_aligner_b200.build``); when it is absent
    and a CUDA toolkit is available, the first call builds it, like the
    reference's compile-on-first-use.  Successful calls are memoized.

    Raises:
        RuntimeError: PyTorch lacks CUDA support, no GPU is accessible, or the
            native library is missing and cannot be built (no ``nvcc``), or it
            fails to load.
    """
    from torch.utils import cpp_extension

    if torch.version.cuda is None:
        raise RuntimeError("fast_forced_aligner_b200 requires a CUDA-enabled PyTorch installation")
    if not torch.cuda.is_available():
        raise RuntimeError("fast_forced_aligner_b200 requires an accessible NVIDIA GPU and compatible driver")
    shim = _PACKAGE / "_ffa_torch.so"
    library = _PACKAGE / "libffa_b200.so"
    if not (shim.is_file() and library.is_file()):
        cuda_home = cpp_extension.CUDA_HOME
        if cuda_home is None or not (Path(cuda_home) / "bin" / "nvcc").is_file():
            raise RuntimeError(
                "fast_forced_aligner_b200's native library is not built and cannot be compiled here. "
                "Install the matching CUDA development toolkit (including nvcc) and a C++ compiler; "
                "set CUDA_HOME if the toolkit is installed outside its usual location. "
                "PyTorch's CUDA runtime libraries alone are insufficient."
            )
        from . import build as _build
        _build.build()
    try:
        torch.ops.load_library(str(shim))
    except OSError as error:  # pragma: no cover - depends on the box
        raise RuntimeError(f"fast_forced_aligner_b200 failed to load its native library: {error}") from error


@dataclass(frozen=True)
class AlignmentBatch:
    """Packed frame alignments and per-record diagnostics returned by ``align``.

    Same fields, shapes, dtypes and meanings as the reference's
    ``AlignmentBatch`` (alignment.py:66-148).  Let ``B`` be the batch size and
    ``N = sum(T_i)``; every tensor lives on the input CUDA device.

    Attributes:
        lengths: host-known frame counts ``(T_0, ..., T_{B-1})``.
        labels: int64 ``(N,)`` vocabulary IDs, blanks and repeats retained;
            ``-1`` at every frame of a failed record.
        scores: float32 ``(N,)``: ``emissions[i][t, paths[i][t]]``; ``-inf``
            for failed records.
        status: int32 ``(B,)``: 0 success, 1 no finite complete path, 2 rejected
            by the emission-validity mask, 3 invalid target IDs, 4 insufficient
            CTC frames.  Target errors take precedence over the mask.
        objective: float32 ``(B,)`` native accumulated path score (the
            sequential fp32 sum along the returned path).
        stitched: int32 ``(B,)``: 1 when the optimized route's chunk paths were
            joined, 0 when conventional DP produced the path.
        repair_passes: int32 ``(B,)`` repair rounds of the optimized route.
        repaired_frames: int64 ``(B,)`` frames re-solved by repair rounds.
        shortcut_stats: int64 ``(B, 3)``: accepted greedy chunks, frames in
            them, chunks rejected for ambiguous placement.
        routing_stats: int32 ``(B, 3)``: early-fallback state, budget-rejected
            repair rounds, largest rejected region.
        reuse_stats: int64 ``(B, 4)`` in optimized mode when a record has 2048
            or more frames, else ``(0, 4)``.

    Tensor operations follow PyTorch's CUDA stream semantics; returning this
    object does not imply the GPU work has completed.
    """

    lengths: tuple[int, ...]
    labels: Tensor
    scores: Tensor
    status: Tensor
    objective: Tensor
    stitched: Tensor
    repair_passes: Tensor
    repaired_frames: Tensor
    shortcut_stats: Tensor
    routing_stats: Tensor
    reuse_stats: Tensor

    @property
    def paths(self) -> tuple[Tensor, ...]:
        """Per-record views of ``labels`` (no copy, no synchronisation)."""
        return self.labels.split(self.lengths)

    def raise_for_status(self) -> None:
        """Read ``status`` on the host (synchronises) and raise for failures.

        Raises ValueError listing the batch indices of statuses 1-4 with the
        reference's messages (alignment.py:163-230), RuntimeError for an
        unknown status.
        """
        statuses = self.status.cpu().tolist()
        if not any(statuses):
            return
        unknown = [i for i, value in enumerate(statuses) if value not in (0, 1, 2, 3, 4)]
        if unknown:
            raise RuntimeError(f"unknown alignment status at batch indices {unknown}")
        invalid = [i for i, value in enumerate(statuses) if value == 2]
        failed = [i for i, value in enumerate(statuses) if value == 1]
        messages = []
        if invalid:
            messages.append(f"invalid emissions at batch indices {invalid}")
        if failed:
            messages.append(f"no finite complete CTC path for batch indices {failed}")
        invalid_targets = [i for i, value in enumerate(statuses) if value == 3]
        insufficient_frames = [i for i, value in enumerate(statuses) if value == 4]
        if invalid_targets:
            messages.append(f"invalid target IDs at batch indices {invalid_targets}")
        if insufficient_frames:
            messages.append(f"insufficient CTC frames at batch indices {insufficient_frames}")
        if messages:
            raise ValueError("; ".join(messages))


def _blanks(count: int, blank_id) -> list[int]:
    blanks = [blank_id] * count if type(blank_id) is int else list(blank_id)
    if len(blanks) != count:
        raise ValueError("provide one blank ID per record")
    if not all(type(b) is int for b in blanks):
        raise ValueError("unsupported frame count, vocabulary, target length, or blank ID")
    return blanks


def _metadata(emissions: Sequence[Tensor], targets: Sequence[Tensor], blank_id) -> list[int]:
    """Host-side checks that must precede the op (alignment.py:233-252); the
    per-tensor checks run in C++ with the same messages."""
    count = len(emissions)
    if not 0 < count <= 65535 or len(targets) != count:
        raise ValueError("provide 1..65535 matching emissions and targets")
    blanks = _blanks(count, blank_id)
    first = emissions[0]
    if not isinstance(first, Tensor) or first.device.type != "cuda":
        raise ValueError("inputs must be contiguous CUDA float32 [T,V] and int64 [U] on one device")
    return blanks


def _check_mask(emission_validity, device, count) -> None:
    if emission_validity is not None:
        if (not isinstance(emission_validity, Tensor)
                or emission_validity.device != device
                or emission_validity.dtype != torch.bool or emission_validity.ndim != 1
                or emission_validity.numel() != count
                or not emission_validity.is_contiguous()):
            raise ValueError("emission_validity must be contiguous CUDA bool [batch] on the input device")


@torch.inference_mode()
def validate_inputs(
    emissions: Sequence[Tensor], targets: Sequence[Tensor], *,
    blank_id: int | Sequence[int] = 0,
) -> None:
    """Validate metadata, target IDs and CTC frame feasibility (synchronous).

    Same contract as the reference (alignment.py:255-309): the checks run on
    the GPU (one warp per record, ``torch.ops.ffa_b200.check_targets``) and one
    status per record is copied to the host.  Emission values are not scanned.

    Raises:
        ValueError: metadata violates the input contract, or target IDs /
            minimum frame counts fail; the message lists failing batch indices.
    """
    blanks = _metadata(emissions, targets, blank_id)
    with torch.cuda.device(emissions[0].device):
        load_extension()
        status = torch.ops.ffa_b200.check_targets(list(emissions), list(targets), blanks)
    failures = [i for i, value in enumerate(status.cpu().tolist()) if value]
    if failures:
        raise ValueError(f"invalid target IDs or insufficient CTC frames at batch indices {failures}")


@torch.inference_mode()
def emission_validity(emissions: Sequence[Tensor]) -> Tensor:
    """Return a CUDA bool ``[B]`` mask that rejects NaN/+inf in each record.

    Same contract as the reference (alignment.py:312-343): every element is
    scanned (-inf is valid), the mask stays on the device, and no GPU value is
    read by the host.  Pass it to ``align(..., emission_validity=mask)``.
    """
    if not 0 < len(emissions) <= 65535:
        raise ValueError("provide 1..65535 emission tensors")
    first = emissions[0]
    if not isinstance(first, Tensor) or first.device.type != "cuda":
        raise ValueError("emissions must be contiguous CUDA float32 [T,V] with supported dimensions on one device")
    with torch.cuda.device(first.device):
        load_extension()
        return torch.ops.ffa_b200.emission_validity(list(emissions))


_ROUTES = {"auto": 1, "pieces": 2, "window": 3}


def _mode(mode, check_inputs, from_logits=False, route="auto") -> int:
    """The torch op's mode code: 0 conventional, 1 optimized, 2 optimized on
    the chunked route for every record (``route="pieces"``), 3 on the window
    route wherever it applies (``route="window"``)."""
    if mode not in _MODES:
        raise ValueError("mode must be 'optimized' or 'conventional'")
    if type(check_inputs) is not bool:
        raise TypeError("check_inputs must be bool")
    if type(from_logits) is not bool:
        raise TypeError("from_logits must be bool")
    if route not in _ROUTES:
        raise ValueError("route must be 'auto', 'pieces' or 'window'")
    return _ROUTES[route] if _MODES[mode] == 1 else _MODES[mode]


def _input_format(first, from_logits: bool) -> int:
    """The C ABI's input format (ffa_input_format) for a call's inputs."""
    if not from_logits:
        return 0
    dtype = first.dtype if isinstance(first, Tensor) else None
    if dtype == torch.float32:
        return 1
    if dtype == torch.bfloat16:
        return 2
    raise ValueError("logits must be contiguous CUDA float32 or bfloat16 tensors")


@torch.inference_mode()
def row_logsumexp(logits: Tensor | Sequence[Tensor]) -> Tensor:
    """Each row's log-sum-exp, as ``align(..., from_logits=True)`` uses it.

    ``z[t] = m + log(sum_v exp(x[t, v] - m))`` with ``m`` the row maximum, in
    fp32 on the GPU (``torch.ops.ffa_b200.row_logsumexp``).  A row holding NaN
    or +inf, or only -inf, gets NaN.

    Args:
        logits: one contiguous CUDA float32 or bfloat16 ``(T, V)`` tensor, or a
            sequence of them (one dtype, one device).

    Returns:
        CUDA float32 ``(sum T,)``: the rows of every tensor, in order.
    """
    items = [logits] if isinstance(logits, Tensor) else list(logits)
    if not 0 < len(items) <= 65535 or not isinstance(items[0], Tensor) or items[0].device.type != "cuda":
        raise ValueError("logits must be contiguous CUDA float32 or bfloat16 [T,V] tensors of one dtype on one device")
    with torch.cuda.device(items[0].device):
        load_extension()
        return torch.ops.ffa_b200.row_logsumexp(items)


@torch.inference_mode()
def log_softmax(logits: Tensor | Sequence[Tensor]) -> Tensor | list[Tensor]:
    """The emission matrices ``align(logits, ..., from_logits=True)`` aligns.

    ``x - z[:, None]`` in fp32 (one rounded subtraction per element, bf16
    logits widened exactly first), with ``z`` from ``row_logsumexp``: within
    a few fp32 ulps of ``torch.log_softmax(x.float(), -1)``, and exactly the
    values the fused path reads.  Aligning these log-probabilities gives the
    fused path's results bit for bit.

    Returns:
        A float32 tensor for a tensor argument, else a list of them.
    """
    single = isinstance(logits, Tensor)
    items = [logits] if single else list(logits)
    z = row_logsumexp(items)
    out, row = [], 0
    for x in items:
        out.append(x.float() - z[row:row + x.shape[0], None])
        row += x.shape[0]
    return out[0] if single else out


@torch.inference_mode()
def align(
    emissions: Sequence[Tensor], targets: Sequence[Tensor], *,
    blank_id: int | Sequence[int] = 0, mode: Mode = "optimized",
    check_inputs: bool = True, emission_validity: Tensor | None = None,
    from_logits: bool = False, route: str = "auto",
) -> AlignmentBatch:
    """Align known CTC targets to resident emissions; return CUDA frame paths.

    Same arguments, result and error behaviour as the reference's ``align``
    (alignment.py:346-502):

    Args:
        emissions: ``B`` contiguous CUDA float32 ``(T_i, V_i)`` tensors,
            ``1 <= B <= 65535``, ``1 <= T_i <= 2**31 - 1``, ``1 <= V_i <= 8192``.
        targets: ``B`` contiguous CUDA int64 ``(U_i,)`` tensors on the same
            device, IDs in ``[0, V_i)`` and different from the blank,
            ``0 <= U_i <= 32767`` (the reference stops at 2047; longer
            transcripts run the conventional DP on a thread-block cluster).
        blank_id: one Python int or ``B`` Python ints (bools rejected).
        mode: ``"optimized"`` (default) or ``"conventional"``.  Conventional
            runs the exact max-plus Viterbi DP (stay > step > skip tie rule).
            Optimized has two routes (``route``).  The window route: a
            greedy pass (each frame's best emission over the transcript
            alphabet), then the same DP restricted to 64 states that slide up
            the trellis, certified on the GPU against those bounds -- its
            outputs are then the conventional ones bit for bit, ties included
            -- with a 128-state window and then the full DP where the
            certificate fails; for records of at most 64 labels (16-byte
            aligned rows), 4096 states and 8192 frames.  The chunked route:
            32-frame pieces joined at legal seams (with repairs, and the
            conventional DP as fallback), which returns the conventional
            outputs bit for bit unless the conventional DP meets a tie on its
            path -- equal scores, or scores closer than the fp32 rounding
            step of its running sum -- where it returns a path of at least
            the same exact score.
        check_inputs: validate target IDs (status 3) and frame feasibility
            (status 4) on the GPU; must be a Python bool.
        emission_validity: optional CUDA bool ``[B]`` mask; False gives status
            2 unless target validation fails.
        from_logits: the ``emissions`` are a model's logits (float32 or
            bfloat16, one dtype for the batch), aligned as their log_softmax
            without writing it out: each kernel reads the logits it needs and
            subtracts the row's log-sum-exp (``log_softmax`` returns the same
            matrices, for inspection).  Not in the reference, whose examples
            call ``torch.log_softmax`` first.
        route: which optimized route a record takes.  ``"auto"`` (default):
            the window route for records of at most 2048 frames in batches of
            more than 4 such records per SM, the chunked route for the rest;
            ``"pieces"``: the chunked route for every record (the reference's
            optimized design); ``"window"``: the window route for every
            record it can take.  Not in the reference.

    Returns:
        AlignmentBatch with packed CUDA outputs.  Failures are recorded in
        ``status`` and do not raise; call ``raise_for_status``.  ``scores``
        hold the selected log_softmax values when ``from_logits``.

    Raises:
        ValueError: invalid mode, metadata, blank IDs or mask metadata.
        TypeError: ``check_inputs`` or ``from_logits`` is not a bool.
        RuntimeError: the native library is unavailable or CUDA fails.
    """
    code = _mode(mode, check_inputs, from_logits, route)
    blanks = _metadata(emissions, targets, blank_id)
    fmt = _input_format(emissions[0], from_logits)
    _check_mask(emission_validity, emissions[0].device, len(emissions))
    load_extension()
    # The op runs under a device guard for the inputs' device.
    tensors, lengths = torch.ops.ffa_b200.align(
        list(emissions), list(targets), blanks, code, emission_validity, check_inputs, fmt)
    return AlignmentBatch(tuple(lengths), *tensors)


def _host_counts(values, what: str) -> Tensor:
    """A 1-D CPU int64 tensor of counts from a sequence, array or tensor."""
    if isinstance(values, Tensor):
        if values.ndim != 1 or values.dtype.is_floating_point or values.dtype.is_complex \
                or values.dtype == torch.bool:
            raise ValueError(f"{what} must be a 1-D sequence of ints")
        return values.to("cpu", torch.int64).contiguous()
    array = np.asarray(values)
    if array.ndim != 1 or (array.size and array.dtype.kind not in "iu"):
        raise ValueError(f"{what} must be a 1-D sequence of ints")
    return torch.from_numpy(np.ascontiguousarray(array, dtype=np.int64))


def _packed_counts(frames, tokens, blank_id) -> tuple[Tensor, Tensor, Tensor]:
    """CPU int64 frame counts, token counts and blanks (one, or one per
    record) of a packed batch, with align_packed's checks and messages."""
    frames_t = _host_counts(frames, "frames")
    tokens_t = _host_counts(tokens, "tokens")
    count = frames_t.numel()
    if not 0 < count <= 65535 or tokens_t.numel() != count:
        raise ValueError("provide 1..65535 matching frame counts, token counts and blanks")
    if type(blank_id) is int:
        blanks_t = torch.tensor([blank_id], dtype=torch.int64)
    elif not isinstance(blank_id, (Sequence, np.ndarray, Tensor)):
        raise TypeError("blank_id must be an int or a sequence of ints")  # as align's list(blank_id)
    else:
        blanks_t = _host_counts(blank_id, "blank_id")
        if blanks_t.numel() != count:
            raise ValueError("provide one blank ID per record")
    return frames_t, tokens_t, blanks_t


@torch.inference_mode()
def align_packed(
    emissions: Tensor, frames, targets: Tensor, tokens, *,
    blank_id: int | Sequence[int] = 0, mode: Mode = "optimized",
    check_inputs: bool = True, emission_validity: Tensor | None = None,
    from_logits: bool = False, route: str = "auto",
) -> AlignmentBatch:
    """Packed variable-length form of ``align`` (no per-record tensors).

    Record ``i`` is rows ``[sum(frames[:i]), sum(frames[:i+1]))`` of one
    contiguous CUDA float32 ``(N, V)`` matrix and tokens
    ``[sum(tokens[:i]), sum(tokens[:i+1]))`` of one contiguous CUDA int64
    vector.  ``frames``, ``tokens`` and a per-record ``blank_id`` may be
    Python sequences, NumPy integer arrays or integer tensors (arrays and
    tensors skip the per-record Python work).  Results and errors are those
    of ``align`` on the same records; ``from_logits`` takes a float32 or
    bfloat16 logits matrix.
    """
    code = _mode(mode, check_inputs, from_logits, route)
    fmt = _input_format(emissions, from_logits)
    frames_t, tokens_t, blanks_t = _packed_counts(frames, tokens, blank_id)
    count = frames_t.numel()
    if not isinstance(emissions, Tensor) or emissions.device.type != "cuda":
        raise ValueError("inputs must be contiguous CUDA float32 [N,V] and int64 [M] on one device")
    _check_mask(emission_validity, emissions.device, count)
    load_extension()
    # The op runs under a device guard for the inputs' device.
    tensors = torch.ops.ffa_b200.align_packed(
        emissions, frames_t, targets, tokens_t, blanks_t, code, emission_validity, check_inputs, fmt)
    return AlignmentBatch(tuple(frames_t.tolist()), *tensors)


@torch.inference_mode()
def token_spans(batch: AlignmentBatch, tokens, *, blank_id: int | Sequence[int] = 0) -> Tensor:
    """Frame span of every target token, from an AlignmentBatch's labels.

    The conversion the reference's README describes (README.md:509-517),
    done on the GPU: each record's path is split into runs of equal labels,
    blank runs are dropped, and the k-th remaining run is the k-th target
    token (a repeated token keeps its blank-separated occurrences apart).

    Args:
        batch: the result of ``align``/``align_packed``.
        tokens: the records' target lengths ``U_i`` (sequence, array or tensor).
        blank_id: the blank of every record, or one per record.

    Returns:
        CUDA int64 ``(sum(U), 2)``: ``[start, end)`` frames per token in record
        order (``.split(tokens)`` gives each record's); ``-1`` in every row of
        a record whose path does not hold ``U_i`` non-blank runs (failed
        records).  Stream-ordered; nothing is read back.
    """
    tokens_t = _host_counts(tokens, "tokens")
    count = len(batch.lengths)
    if tokens_t.numel() != count:
        raise ValueError("provide one token count per record")
    if type(blank_id) is int:
        blanks_t = torch.tensor([blank_id], dtype=torch.int64)
    elif not isinstance(blank_id, (Sequence, np.ndarray, Tensor)):
        raise TypeError("blank_id must be an int or a sequence of ints")
    else:
        blanks_t = _host_counts(blank_id, "blank_id")
    frames_t = torch.tensor(batch.lengths, dtype=torch.int64)
    load_extension()
    return torch.ops.ffa_b200.token_spans(batch.labels, frames_t, tokens_t, blanks_t)


def token_timestamps(batch: AlignmentBatch, tokens, frame_seconds: float, *,
                     blank_id: int | Sequence[int] = 0) -> Tensor:
    """``token_spans`` in seconds: float64 ``(sum(U), 2)`` start and end times
    (frames times ``frame_seconds``, e.g. a model's
    ``inputs_to_logits_ratio / sample_rate``); NaN rows for failed records."""
    spans = token_spans(batch, tokens, blank_id=blank_id)
    seconds = spans.to(torch.float64) * float(frame_seconds)
    return torch.where(spans < 0, torch.full_like(seconds, float("nan")), seconds)
