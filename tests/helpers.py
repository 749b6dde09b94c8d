"""Helpers shared by the GPU parity tests."""
from __future__ import annotations

import numpy as np
import torch

from oracle import oracle


def cuda_records(emissions, targets, device="cuda"):
    es = [torch.from_numpy(np.ascontiguousarray(e)).to(device) for e in emissions]
    ts = [torch.from_numpy(np.ascontiguousarray(t, dtype=np.int64)).to(device) for t in targets]
    return es, ts


def assert_same_bits(actual: np.ndarray, expected: np.ndarray, what: str):
    a = np.ascontiguousarray(actual)
    b = np.ascontiguousarray(expected)
    assert a.shape == b.shape, (what, a.shape, b.shape)
    if a.dtype.kind == "f":
        same = a.view(np.int32 if a.dtype == np.float32 else np.int64) == \
            b.view(np.int32 if b.dtype == np.float32 else np.int64)
        both_nan = np.isnan(a) & np.isnan(b)
        bad = np.flatnonzero(~(same | both_nan))
    else:
        bad = np.flatnonzero(a != b)
    assert bad.size == 0, f"{what}: {bad.size} mismatches, first at {bad[:5]}: {a[bad[:5]]} vs {b[bad[:5]]}"


def assert_matches_oracle(result, ref: oracle.OracleResult, what: str = ""):
    """Bit-exact labels, scores, status and objective (integer/index work and
    the single-rounding fp32 DP are both exact)."""
    assert tuple(result.lengths) == tuple(ref.lengths)
    assert_same_bits(result.status.cpu().numpy(), ref.status, what + " status")
    assert_same_bits(result.labels.cpu().numpy(), ref.labels, what + " labels")
    assert_same_bits(result.scores.cpu().numpy(), ref.scores, what + " scores")
    assert_same_bits(result.objective.cpu().numpy(), ref.objective, what + " objective")


def collapse(path: np.ndarray, blank: int) -> np.ndarray:
    keep = np.r_[True, path[1:] != path[:-1]]
    merged = path[keep]
    return merged[merged != blank]


def sequential_sum(values: np.ndarray) -> np.float32:
    acc = np.float32(values[0])
    for v in values[1:]:
        acc = np.float32(acc + v)
    return acc
