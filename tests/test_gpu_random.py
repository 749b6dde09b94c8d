"""Randomised batches against the CPU oracle: every vocabulary kind (row-staged
V <= 64 with V % 4 == 0, gathered otherwise), tiny and piece-boundary lengths,
random blanks, adjacent repeats, -inf emissions, both modes in one batch."""
import numpy as np
import pytest
import torch

import fast_forced_aligner_b200 as ffa
from oracle import oracle
from tests.helpers import assert_matches_oracle, assert_same_optimum, cuda_records

pytestmark = pytest.mark.gpu


def random_batch(seed, count=200):
    rng = np.random.default_rng(seed)
    es, ts, blanks = [], [], []
    for _ in range(count):
        V = int(rng.choice([2, 3, 5, 8, 32, 33, 64, 129, 1025]))
        blank = int(rng.integers(0, V))
        T = int(rng.choice([1, 2, 31, 32, 33, 64, 65, 96, 97]) if rng.random() < 0.3 else rng.integers(1, 3000))
        U = int(rng.integers(0, max(1, min(T, 1500)) // 2 + 1))
        choices = np.array([c for c in range(V) if c != blank]) if V > 1 else np.array([0])
        tokens = rng.choice(choices, U).astype(np.int64) if U else np.zeros(0, np.int64)
        logits = rng.standard_normal((T, V)).astype(np.float32) * rng.uniform(0.5, 4.0)
        if U:  # boost a monotone labelling so that most records align confidently
            idx = np.sort(rng.choice(T, min(T, U), replace=False)) if U <= T else np.arange(T)
            logits[idx, tokens[:idx.size]] += rng.uniform(0.0, 6.0)
        e = (logits - np.log(np.exp(logits).sum(axis=1, keepdims=True))).astype(np.float32)
        if rng.random() < 0.1:
            e[rng.integers(0, T, 3), rng.integers(0, V, 3)] = -np.inf
        es.append(e); ts.append(tokens); blanks.append(blank)
    return es, ts, blanks


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_random_batches_match_oracle(cuda, seed):
    es, ts, blanks = random_batch(seed)
    ref = oracle.align(es, ts, blanks)
    d_es, d_ts = cuda_records(es, ts)
    conv = ffa.align(d_es, d_ts, blank_id=blanks, mode="conventional")
    assert_matches_oracle(conv, ref, f"seed {seed} conventional")
    opt = ffa.align(d_es, d_ts, blank_id=blanks, mode="optimized")
    same = assert_same_optimum(opt, ref, es, ts, blanks, f"seed {seed} optimized")
    assert same >= len(es) - 10
    statuses = ref.status
    assert (statuses == 0).sum() > len(es) // 3  # the batch exercises aligned records too
