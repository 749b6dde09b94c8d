"""Pin the CPU oracle against the reference's known-answer tests and fixtures.

Every case here comes from the reference repository's own tests or examples
(cited per test) or from its CPU comparator (tests/golden).  The oracle is the
checker of the GPU path; these tests run without a GPU.
"""
from itertools import product

import numpy as np
import pytest

from oracle import oracle
from tests.golden.make_golden import load as load_golden


def ctc_states(targets, blank):
    states = np.full(2 * len(targets) + 1, blank)
    states[1::2] = targets
    return states


def dp_optimum(values, targets, blank):
    """Independent fp64 max-plus DP score (the reference's test oracle idea,
    tests/test_core.py:11-26, restated)."""
    states = ctc_states(targets, blank)
    prev = np.full(len(states), -np.inf)
    prev[:2] = values[0, states[:2]]
    for frame in values[1:]:
        cur = np.full_like(prev, -np.inf)
        for s, label in enumerate(states):
            best = prev[s]
            if s >= 1:
                best = max(best, prev[s - 1])
            if s >= 2 and label != blank and label != states[s - 2]:
                best = max(best, prev[s - 2])
            cur[s] = best + frame[label]
        prev = cur
    return max(prev[-2:]) if len(states) > 1 else prev[-1]


def collapse(path, blank):
    path = np.asarray(path)
    keep = np.r_[True, path[1:] != path[:-1]]
    merged = path[keep]
    return merged[merged != blank]


def test_tie_kat_picks_the_optimal_path():
    # benchmarks/tests/test_adapters.py:56-69: optimal score 0; the uncorrected
    # upstream CPU aligner returns a -10 path.
    e = np.array([[0, 0, -10], [0, 0, -10], [-10, -10, 0], [0, -10, -10], [0, -10, -10]], np.float32)
    r = oracle.align([e], [np.array([1, 2])], 0)
    assert r.status.tolist() == [0]
    assert r.scores.sum() == 0
    assert r.labels.tolist() == [1, 0, 2, 0, 0]
    assert r.objective[0] == 0


def test_adapter_fixture_paths():
    # benchmarks/tests/test_adapters.py:19-32: three fixed paths, one with blank=3.
    for labels, targets, blank in [([0, 1, 1, 0, 2, 2], [1, 2], 0),
                                   ([3, 0, 0, 3, 0, 2, 3], [0, 0, 2], 3),
                                   ([0, 1, 0, 1, 2, 0, 0, 0], [1, 1, 2], 0)]:
        e = np.full((len(labels), 4), -8, np.float32)
        e[np.arange(len(labels)), labels] = -0.125
        r = oracle.align([e], [np.array(targets)], blank)
        assert r.labels.tolist() == labels
        np.testing.assert_array_equal(r.scores, e[np.arange(len(labels)), labels])


def test_exhaustive_enumeration_kats():
    # benchmarks/tests/test_adapters.py:237-270: enumerate every label path of
    # 12 tiny cases (seed 1729) independently of any DP recurrence.
    rng = np.random.default_rng(1729)
    for index in range(12):
        blank = index % 3
        vocab = [c for c in range(3) if c != blank]
        tokens = [vocab[index % 2], vocab[(index // 2) % 2]]
        frames = 5 + index % 2
        e = rng.integers(-5, 1, size=(frames, 3)).astype(np.float32)
        legal = [float(e[np.arange(frames), p].sum()) for p in product(range(3), repeat=frames)
                 if collapse(p, blank).tolist() == tokens]
        r = oracle.align([e], [np.array(tokens)], blank)
        assert collapse(r.labels, blank).tolist() == tokens
        assert float(r.scores.sum()) == max(legal)


@pytest.mark.parametrize("blank", [0, 5])
def test_ragged_records_match_independent_optimum(blank):
    # tests/test_core.py:29-48: ragged records (T 7..2305, repeats, empty
    # transcript) with integer-valued emissions: the fp64 path sum equals the
    # DP optimum exactly and scores are the selected emissions.
    rng = np.random.default_rng(32)
    labels = np.array([i for i in range(6) if i != blank])
    values = [rng.integers(-9, 0, (n, 6)).astype(np.float32) for n in (7, 129, 257, 2305)]
    tokens = [rng.choice(labels, n) for n in (0, 11, 44, 120)]
    r = oracle.align(values, tokens, blank)
    assert r.status.tolist() == [0, 0, 0, 0]
    for v, t, p in zip(values, tokens, r.paths):
        np.testing.assert_array_equal(collapse(p, blank), t)
        selected = v[np.arange(len(p)), p]
        assert selected.sum(dtype=np.float64) == dp_optimum(v, t, blank)


def test_example_alignment():
    # examples/align_emissions.py:6-14: blank=0, a=1, b=2, transcript a a b.
    logits = np.array([[0, -4, -4], [-4, 0, -4], [0, -4, -4], [-4, 0, -4], [-4, -4, 0], [0, -4, -4]],
                      np.float32)
    e = logits - np.log(np.exp(logits).sum(1, keepdims=True)).astype(np.float32)
    r = oracle.align([e.astype(np.float32)], [np.array([1, 1, 2])], 0)
    assert r.labels.tolist() == [0, 1, 0, 1, 2, 0]


def test_status_precedence_and_failure_fill():
    # tests/test_async_validation.py:164-178: statuses [3, 4, 2, 3, 1].
    es = [np.zeros((3, 4), np.float32) for _ in range(5)]
    es[-1][:] = -np.inf
    ts = [np.array(t) for t in ([9], [1, 1, 1], [1], [0, 0, 0, 0], [1])]
    r = oracle.align(es, ts, 0, validity=[False, False, False, True, True])
    assert r.status.tolist() == [3, 4, 2, 3, 1]
    assert (r.labels == -1).all() and np.isneginf(r.scores).all()


@pytest.mark.parametrize("tokens", [1, 129, 257, 2047])
def test_exact_frame_feasibility(tokens):
    # tests/test_async_validation.py:132-149: T = 2U - 1 suffices for U equal
    # tokens; one frame fewer is status 4.
    target = np.ones(tokens, np.int64)
    enough = np.zeros((2 * tokens - 1, 3), np.float32)
    es, ts = [enough], [target]
    if tokens > 1:
        es.append(enough[:-1]); ts.append(target)
    r = oracle.align(es, ts, 0)
    assert r.status.tolist() == ([0, 4] if tokens > 1 else [0])
    np.testing.assert_array_equal(collapse(r.paths[0], 0), target)


def test_invalid_ids_and_unchecked_infeasible():
    # tests/test_async_validation.py:105-123, 211-219.
    e = np.zeros((7, 6), np.float32)
    token_lists = [[1, 1, 2], [-1], [6], [0], [2**32 + 1], [2**63 - 1], [-2**63], []]
    r = oracle.align([e] * len(token_lists), [np.array(t, np.int64) for t in token_lists], 0)
    assert r.status.tolist() == [0, 3, 3, 3, 3, 3, 3, 0]
    two = np.zeros((2, 4), np.float32)
    assert oracle.align([two], [np.array([1, 1])], 0).status.tolist() == [4]
    assert oracle.align([two], [np.array([1, 1])], 0, check_inputs=False).status.tolist() == [1]


def test_emission_validity_kat():
    # tests/test_emission_validity.py:10-31: NaN/+inf rejected, -inf allowed.
    good = np.zeros((7, 6), np.float32)
    nan, pinf, ninf = good.copy(), good.copy(), good.copy()
    nan[-1, 5] = np.nan; pinf[0, 5] = np.inf; ninf[:, 5] = -np.inf
    assert oracle.emission_validity([good, nan, pinf, ninf]).tolist() == [True, False, False, True]


def test_oracle_matches_reference_cpu_comparator_golden():
    # Golden paths produced by the reference's own CPU comparator
    # (tests/golden/make_golden.py), flat-tie cases included.
    cases = load_golden()
    r = oracle.align([c[0] for c in cases], [c[1] for c in cases], [c[2] for c in cases])
    assert (r.status == 0).all()
    for p, c in zip(r.paths, cases):
        np.testing.assert_array_equal(p, c[3])
    np.testing.assert_array_equal(r.scores, np.concatenate([c[4] for c in cases]))


def test_objective_is_sequential_fp32_path_sum():
    rng = np.random.default_rng(5)
    logits = rng.standard_normal((300, 32)).astype(np.float32)
    e = (logits - np.log(np.exp(logits).sum(1, keepdims=True))).astype(np.float32)
    r = oracle.align([e], [rng.integers(1, 32, 60)], 0)
    acc = np.float32(0)
    for k, v in enumerate(r.scores):
        acc = v if k == 0 else np.float32(acc + v)
    assert acc == r.objective[0]


# ---- the reference's greedy chunk counts (alignment.cu:29-153), restated in
#      oracle.greedy_chunk_stats: known answers on small hand-built records ----

def _one_hot(labels, V=4, hi=-0.1, lo=-5.0):
    e = np.full((len(labels), V), lo, np.float32)
    e[np.arange(len(labels)), labels] = hi
    return e


def test_greedy_chunk_accepts_a_unique_placement():
    # Frames follow blank 1 1 blank 2 exactly: one legal placement from state 0.
    e = _one_hot([0, 1, 1, 0, 2])
    assert oracle.greedy_chunk_stats(e, np.array([1, 2]), 0, chunk=5).tolist() == [1, 5, 0]


def test_greedy_chunk_counts_several_placements():
    # Transcript 1 2 1 2: the middle chunk "2 2" (frames 2-3) fits token
    # states 3 and 7, so it has two placements.
    e = _one_hot([1, 0, 2, 2, 0, 1, 0, 2])
    stats = oracle.greedy_chunk_stats(e, np.array([1, 2, 1, 2]), 0, chunk=2)
    assert stats[2] >= 1


def test_greedy_chunk_rejects_ties_and_illegal_sequences():
    e = _one_hot([0, 1, 1, 0, 2])
    e[2, 3] = e[2, 1]  # label 3 is not in the alphabet: no effect
    assert oracle.greedy_chunk_stats(e, np.array([1, 2]), 0, chunk=5).tolist() == [1, 5, 0]
    e[2, 2] = e[2, 1]  # a tie inside the alphabet rejects the chunk
    assert oracle.greedy_chunk_stats(e, np.array([1, 2]), 0, chunk=5).tolist() == [0, 0, 0]
    # Greedy labels 2 then 1 cannot follow transcript 1 2 in order.
    assert oracle.greedy_chunk_stats(_one_hot([2, 1]), np.array([1, 2]), 0, chunk=2).tolist() == [0, 0, 0]


# ---- the exact divergence classes the parity tests use (tests/helpers.py) ----

def test_divergence_classes():
    from tests.helpers import classify_divergence
    # Two frames, transcript [1]: paths 1,0 and 0,1 with equal emissions tie.
    e = np.array([[-1.0, -1.0], [-1.0, -1.0]], np.float32)
    t = np.array([1])
    assert classify_divergence(e, t, 0, np.array([1, 0]), np.array([1, 0])) == "identical"
    assert classify_divergence(e, t, 0, np.array([0, 1]), np.array([1, 1])) == "equal_fp32"
    e2 = np.array([[-1.0, -0.5], [-1.0, -2.0]], np.float32)
    # Path 1,0 scores -1.5 and path 0,1 scores -3: the second is worse.
    assert classify_divergence(e2, t, 0, np.array([0, 1]), np.array([1, 0])) == "worse"
    assert classify_divergence(e2, t, 0, np.array([1, 0]), np.array([0, 1])) == "better"
