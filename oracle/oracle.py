"""ctypes front end for the CPU oracle and loaders for the reference checkers.

TEST INFRASTRUCTURE ONLY.  The product package never imports this module; it
is used by tests/, ``__graft_entry__.smoke()`` and bench.py's CPU baseline.

``align`` mirrors the reference's conventional path
(src/fast_forced_aligner/csrc/alignment.cu:354-523, 641-667, 818-877) on
host numpy arrays and returns the same packed outputs the GPU path returns.
"""
from __future__ import annotations

import ctypes
import importlib.util
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Sequence

import numpy as np

HERE = Path(__file__).resolve().parent


class _Record(ctypes.Structure):
    _fields_ = [("emissions", ctypes.c_void_p), ("targets", ctypes.c_void_p),
                ("T", ctypes.c_int64), ("V", ctypes.c_int64),
                ("U", ctypes.c_int64), ("blank", ctypes.c_int64)]


_LIB = None


def library() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = HERE / "libffa_oracle.so"
        if not path.exists():
            from . import build  # type: ignore[no-redef]
            build.build_oracle()
        lib = ctypes.CDLL(str(path))
        lib.ffa_oracle_align.argtypes = [
            ctypes.POINTER(_Record), ctypes.c_int64, ctypes.c_int, ctypes.c_void_p,
            ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        lib.ffa_oracle_align.restype = ctypes.c_int
        lib.ffa_oracle_emission_validity.argtypes = [
            ctypes.POINTER(_Record), ctypes.c_int64, ctypes.c_void_p]
        lib.ffa_oracle_emission_validity.restype = ctypes.c_int
        _LIB = lib
    return _LIB


@dataclass
class OracleResult:
    lengths: tuple[int, ...]
    labels: np.ndarray      # int64 [sum T]
    scores: np.ndarray      # float32 [sum T]
    status: np.ndarray      # int32 [B]
    objective: np.ndarray   # float32 [B]

    @property
    def paths(self) -> list[np.ndarray]:
        return np.split(self.labels, np.cumsum(self.lengths)[:-1])


def _records(emissions, targets, blanks):
    keep = []
    recs = (_Record * len(emissions))()
    for i, (e, t, b) in enumerate(zip(emissions, targets, blanks, strict=True)):
        e = np.ascontiguousarray(e, dtype=np.float32)
        t = np.ascontiguousarray(t, dtype=np.int64)
        keep += [e, t]
        recs[i] = _Record(e.ctypes.data, t.ctypes.data if t.size else None,
                          e.shape[0], e.shape[1], t.size, int(b))
    return recs, keep


def align(emissions: Sequence[np.ndarray], targets: Sequence[np.ndarray],
          blank_id: int | Sequence[int] = 0, *, check_inputs: bool = True,
          validity: Sequence[bool] | None = None, threads: int = 0) -> OracleResult:
    """Conventional-mode alignment of host arrays (fp32 [T,V], int64 [U])."""
    count = len(emissions)
    blanks = [blank_id] * count if isinstance(blank_id, int) else list(blank_id)
    recs, keep = _records(emissions, targets, blanks)
    lengths = tuple(int(e.shape[0]) for e in emissions)
    total = sum(lengths)
    labels = np.empty(total, np.int64)
    scores = np.empty(total, np.float32)
    status = np.empty(count, np.int32)
    objective = np.empty(count, np.float32)
    mask = None
    if validity is not None:
        mask = np.ascontiguousarray(np.asarray(validity, dtype=np.uint8))
        keep.append(mask)
    rc = library().ffa_oracle_align(
        recs, count, int(bool(check_inputs)), mask.ctypes.data if mask is not None else None,
        int(threads), labels.ctypes.data, scores.ctypes.data, status.ctypes.data,
        objective.ctypes.data)
    if rc:
        raise ValueError(f"oracle rejected the inputs (code {rc})")
    return OracleResult(lengths, labels, scores, status, objective)


def emission_validity(emissions: Sequence[np.ndarray]) -> np.ndarray:
    recs, keep = _records(emissions, [np.zeros(0, np.int64)] * len(emissions),
                          [0] * len(emissions))
    out = np.empty(len(emissions), np.uint8)
    if library().ffa_oracle_emission_validity(recs, len(emissions), out.ctypes.data):
        raise ValueError("oracle rejected the inputs")
    return out.astype(bool)


def corrected_module():
    """The reference repository's own CPU comparator, compiled in place into
    oracle/_ref (benchmarks/patches/cpu_corrected.cpp), or None if absent."""
    import sysconfig
    path = HERE / "_ref" / ("ffa_corrected_ctc_cpp" + sysconfig.get_config_var("EXT_SUFFIX"))
    if not path.exists():
        return None
    spec = importlib.util.spec_from_file_location("ffa_corrected_ctc_cpp", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


_REF_CUDA_LOADED = False


def load_reference_cuda() -> bool:
    """Register the reference's own CUDA ops (torch.ops.fast_forced_aligner_cuda)
    from oracle/_ref, compiled from the reference source.  False if absent."""
    global _REF_CUDA_LOADED
    if _REF_CUDA_LOADED:
        return True
    path = HERE / "_ref" / "fast_forced_aligner_cuda.so"
    if not path.exists():
        return False
    import torch
    torch.ops.load_library(str(path))
    _REF_CUDA_LOADED = True
    return True


def reference_cuda_align(emissions, targets, blanks, *, mode: str = "conventional",
                         check_inputs: bool = True, emission_validity=None):
    """Call the reference's CUDA op with the exact arguments its public
    ``align`` passes (alignment.py:495-502).  Returns the raw tensors
    (labels, scores, status, objective, stitched, repair_passes,
    repaired_frames, shortcut_stats, routing_stats, reuse_stats) and lengths."""
    import torch
    if not load_reference_cuda():
        raise RuntimeError("reference CUDA extension not built under oracle/_ref")
    optimized = mode == "optimized"
    with torch.cuda.device(emissions[0].device):
        return torch.ops.fast_forced_aligner_cuda.align(
            list(emissions), list(targets), list(blanks),
            128, 2 if optimized else 0, 512, 2, 2, 2,
            512 if optimized else 0, 0, False, True, optimized,
            2048, 2048, optimized, 2048, emission_validity, check_inputs)


def default_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def greedy_chunk_stats(emissions: np.ndarray, targets: np.ndarray, blank: int,
                       chunk: int = 128) -> np.ndarray:
    """The reference's greedy shortcut counts for one record (int64 [3]):
    accepted greedy chunks, the frames in them, and chunks rejected because
    the greedy label sequence had several legal placements
    (src/fast_forced_aligner/csrc/alignment.cu:29-153, reported as
    ``shortcut_stats``, alignment.py:116-121).

    Per chunk of ``chunk`` frames: each frame's greedy label is the unique
    finite maximum over the transcript alphabet, blank included (a NaN never
    compares greater or equal there, so NaN columns drop out), else the chunk
    is rejected (:60-91); the relative state offsets r advance by 0 on a
    repeated label, 1 into or out of a blank, 2 between tokens (:112-117); a
    start s is legal when l[s] is the chunk's first label (s <= 1 for the
    first chunk), its terminal s + r[-1] is a state (>= S-2 for the last
    chunk), and every label change lands on a state with that label
    (:119-128).  Exactly one legal start accepts the chunk (if its fp32 sum of
    maxima is finite); more count as rejected for several placements."""
    e = np.asarray(emissions, np.float32)
    T = e.shape[0]
    tokens = np.asarray(targets, np.int64)
    S = 2 * tokens.size + 1
    labels = np.full(S, blank, np.int64)
    labels[1::2] = tokens
    alphabet = np.unique(labels)
    sub = np.where(np.isnan(e[:, alphabet]), np.float32(-np.inf), e[:, alphabet])
    best = sub.max(axis=1)
    unique = (sub == best[:, None]).sum(axis=1) == 1
    finite = np.isfinite(best)
    greedy = alphabet[sub.argmax(axis=1)]
    stats = np.zeros(3, np.int64)
    for a in range(0, T, chunk):
        b = min(T, a + chunk)
        if not (unique[a:b].all() and finite[a:b].all()):
            continue
        g = greedy[a:b]
        change = np.r_[False, g[1:] != g[:-1]]
        prev = np.r_[g[0], g[:-1]]
        step = np.where(change, np.where((g == blank) | (prev == blank), 1, 2), 0)
        r = np.cumsum(step)
        starts = np.flatnonzero(labels == g[0])
        if a == 0:
            starts = starts[starts <= 1]
        term = starts + r[-1]
        ok = term < S
        if b == T:
            ok &= term >= S - 2
        starts = starts[ok]
        idx = np.flatnonzero(change)
        matches = sum(1 for s in starts if np.all(labels[s + r[idx]] == g[idx]))
        if matches == 1:
            total = np.float32(0)
            for v in best[a:b]:
                total = np.float32(total + v)
            if np.isfinite(total):
                stats[0] += 1
                stats[1] += b - a
        elif matches > 1:
            stats[2] += 1
    return stats
