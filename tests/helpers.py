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


def assert_same_optimum(result, ref: oracle.OracleResult, emissions, targets, blanks, what: str = "",
                        exact=None):
    """Optimized-route contract where inputs hold ties: the same status per
    record, and for every aligned record a legal path (it collapses to the
    transcript) whose scores are the selected emissions, whose objective is
    their sequential fp32 sum, and whose score equals the conventional
    optimum (both rescored in fp64).  Records listed in `exact` must also
    match the conventional outputs bit for bit.  Returns how many aligned
    records have the conventional path itself."""
    assert tuple(result.lengths) == tuple(ref.lengths)
    status = result.status.cpu().numpy()
    assert_same_bits(status, ref.status, what + " status")
    labels = result.labels.cpu().numpy()
    scores = result.scores.cpu().numpy()
    objective = result.objective.cpu().numpy()
    offsets = np.concatenate([[0], np.cumsum(ref.lengths)])
    blanks = list(blanks) if np.ndim(blanks) else [blanks] * len(emissions)
    exact = set(exact or ())
    same_path = 0
    for i, (e, t) in enumerate(zip(emissions, targets)):
        lo, hi = offsets[i], offsets[i + 1]
        p, q = labels[lo:hi], ref.labels[lo:hi]
        if i in exact or status[i] != 0:
            assert_same_bits(p, q, f"{what} record {i} labels")
            assert_same_bits(scores[lo:hi], ref.scores[lo:hi], f"{what} record {i} scores")
            assert_same_bits(objective[i:i + 1], ref.objective[i:i + 1], f"{what} record {i} objective")
        if status[i] != 0:
            continue
        same_path += int(np.array_equal(p, q))
        np.testing.assert_array_equal(collapse(p, blanks[i]), t, f"{what} record {i} transcript")
        selected = e[np.arange(len(p)), p]
        assert_same_bits(scores[lo:hi], selected, f"{what} record {i} scores")
        assert sequential_sum(selected) == objective[i], f"{what} record {i} objective"
        # Equal optimum: the fp64 rescorings differ by less than a few fp32
        # rounding steps of the conventional objective (zero for exact ties).
        mine = float(np.sum(selected.astype(np.float64)))
        best = float(np.sum(ref.scores[lo:hi].astype(np.float64)))
        step = float(np.spacing(np.float32(abs(ref.objective[i]))))
        assert abs(mine - best) <= 4 * step, f"{what} record {i}: {mine} vs {best} (fp32 step {step})"
    return same_path


def conventional_scores(e: np.ndarray, targets: np.ndarray, blank: int) -> np.ndarray:
    """The conventional DP's fp32 scores alpha[t, s] of one record (the
    recurrence of alignment.cu:407-429: one fp32 add per cell, stay > step >
    skip by strict '>'), as a [T, S] array.  Small records only."""
    T = e.shape[0]
    S = 2 * len(targets) + 1
    labels = np.full(S, blank, np.int64)
    labels[1::2] = targets
    skip = np.zeros(S, bool)
    skip[3::2] = (labels[3::2] != blank) & (labels[3::2] != labels[1:-2:2])
    alpha = np.full((T, S), -np.inf, np.float32)
    alpha[0, :min(2, S)] = e[0, labels[:min(2, S)]]
    ninf = np.float32(-np.inf)
    for t in range(1, T):
        a = alpha[t - 1]
        step = np.r_[ninf, a[:-1]]
        best = np.where(step > a, step, a)
        if S > 2:
            sk = np.r_[ninf, ninf, a[:-2]]
            best = np.where(skip & (sk > best), sk, best)
        alpha[t] = (best + e[t, labels]).astype(np.float32)
    return alpha


def state_path(labels: np.ndarray, targets: np.ndarray, blank: int) -> np.ndarray:
    """The CTC state of every frame of a legal label path (a repeated label
    stays, a new label steps to the next state that carries it)."""
    S = 2 * len(targets) + 1
    lab = np.full(S, blank, np.int64)
    lab[1::2] = targets
    cur = 0 if labels[0] == blank else 1
    out = [cur]
    for x in labels[1:]:
        if x != lab[cur]:
            cur += 1 if (cur + 1 < S and x == lab[cur + 1]) else 2
        out.append(cur)
    return np.array(out)


def classify_divergence(e: np.ndarray, targets: np.ndarray, blank: int, mine_labels: np.ndarray,
                        conv_labels: np.ndarray) -> str:
    """Why an optimized-route path differs from the conventional one, decided
    exactly, in the spirit of the reference's own accuracy audit
    (benchmarks/accuracy.py:67-105):
      "identical"     the label paths are equal;
      "equal_fp32"    both paths' sequential fp32 sums are bitwise equal;
      "tie_rule"      where the two paths meet, the conventional DP chose
                      between equal fp32 scores (its stay > step > skip or
                      terminal >= rule decided);
      "equal_score"   equal exact (fp64) path sums;
      "better"        the optimized path's exact sum is higher: the
                      conventional choice was decided by fp32 rounding;
      "worse"         a genuine divergence: the optimized path scores lower
                      exactly.
    Only "worse" is a parity failure."""
    if np.array_equal(mine_labels, conv_labels):
        return "identical"
    rows = np.arange(e.shape[0])
    mine = e[rows, mine_labels]
    conv = e[rows, conv_labels]
    if sequential_sum(mine).view(np.int32) == sequential_sum(conv).view(np.int32):
        return "equal_fp32"
    sm, sc = state_path(mine_labels, targets, blank), state_path(conv_labels, targets, blank)
    alpha = conventional_scores(e, targets, blank)
    T = e.shape[0]
    last = int(np.flatnonzero(sm != sc)[-1])
    # The last frame where the state paths differ: there the conventional DP
    # compared both predecessors (or, at the last frame, both terminals).
    if alpha[last, sm[last]] == alpha[last, sc[last]]:
        return "tie_rule"
    a, b = float(np.sum(mine.astype(np.float64))), float(np.sum(conv.astype(np.float64)))
    if a == b:
        return "equal_score"
    return "better" if a > b else "worse"
