"""Long records: transcripts of more than 2047 tokens (S > 4096 states, cfg2's
long-form recordings), which the reference rejects and this build aligns with
the conventional DP on a thread-block cluster (one CTA per 4096 states).
Every result is checked bit for bit against the CPU oracle."""
import os

import numpy as np
import pytest
import torch

import fast_forced_aligner_b200 as ffa
from fast_forced_aligner_b200 import workloads
from oracle import oracle
from tests.helpers import assert_matches_oracle, cuda_records

pytestmark = pytest.mark.gpu
MODES = ["optimized", "conventional"]
THREADS = max(1, os.cpu_count() or 1)


def long_record(rng, T, U, vocab=32, blank=0, repeat_rate=0.0):
    """A record of T frames and U tokens from the cfg2 generator (boost +4,
    lowered to +2.5 on 15% of frames, blank prior on 40% of frames)."""
    choices = np.array([v for v in range(vocab) if v != blank], dtype=np.int64)
    tokens = workloads._tokens(rng, U, choices, repeat_rate)
    labels, _, _ = workloads._frame_labels(rng, T, tokens, blank)
    e, _ = workloads._emissions(rng, labels, vocab, blank, 4.0, blank_prior=2.0, blank_frac=0.4,
                                low_boost=2.5, low_frac=0.15)
    return e, tokens


@pytest.mark.parametrize("mode", MODES)
def test_scaled_cfg2_matches_oracle(cuda, mode):
    wl = workloads.config(2, scale=0.1)  # 6 records of 9000 frames, S = 5401: 2-CTA clusters
    es, ts = wl.records()
    result = ffa.align(*cuda_records(es, ts), blank_id=wl.blank, mode=mode)
    assert_matches_oracle(result, oracle.align(es, ts, wl.blank, threads=THREADS), f"cfg2/10 {mode}")
    assert not result.stitched.any()


@pytest.mark.parametrize("mode", MODES)
def test_every_cluster_size_matches_oracle(cuda, mode):
    # S = 4097 (2 CTAs), 8193 (3), 28001 (7), 36865 (10), 54001 (14), 65535
    # (16, the largest), batched with short records that take the first pass.
    rng = np.random.default_rng(2026)
    shapes = [(2300, 2048), (4500, 4096), (16000, 14000), (20000, 18432), (29000, 27000),
              (34000, 32767), (700, 210), (64, 20), (1500, 450)]
    es, ts = zip(*(long_record(rng, T, U) for T, U in shapes))
    result = ffa.align(*cuda_records(es, ts), blank_id=0, mode=mode)
    ref = oracle.align(list(es), list(ts), 0, threads=THREADS)
    assert (ref.status == 0).all()
    assert_matches_oracle(result, ref, f"cluster sizes {mode}")


def test_sixteen_states_per_thread_when_clusters_do_not_all_fit(cuda):
    # 12 records of S = 37001 need 10-CTA clusters at 8 states per thread, of
    # which a B200 runs 11 at a time: the batch takes 16 states per thread
    # (5-CTA clusters) instead.
    rng = np.random.default_rng(5)
    es, ts = zip(*(long_record(rng, 19000, 18500) for _ in range(12)))
    result = ffa.align(*cuda_records(es, ts), blank_id=0, mode="conventional")
    assert_matches_oracle(result, oracle.align(list(es), list(ts), 0, threads=THREADS), "K=16 batch")


def test_gathered_long_record_matches_oracle(cuda):
    # V = 1025 rows are gathered per thread (no row staging); blank 1024.
    rng = np.random.default_rng(7)
    e, t = long_record(rng, 6000, 5000, vocab=1025, blank=1024, repeat_rate=0.05)
    result = ffa.align(*cuda_records([e], [t]), blank_id=1024, mode="conventional")
    assert_matches_oracle(result, oracle.align([e], [t], 1024), "gathered long record")


def test_full_size_cfg2_matches_oracle(cuda):
    # Benchmark configuration 2 at full size: 8 recordings of 90000 frames,
    # U = 27000 (S = 54001: 14-CTA clusters), 3.9e10 trellis cells.
    wl = workloads.config(2)
    es, ts = wl.records()
    result = ffa.align(*cuda_records(es, ts), blank_id=wl.blank, mode="optimized")
    assert_matches_oracle(result, oracle.align(es, ts, wl.blank, threads=THREADS), "cfg2")


def test_long_record_statuses(cuda):
    rng = np.random.default_rng(11)
    e, t = long_record(rng, 2600, 2300)
    bad = t.copy()
    bad[1700] = 0                                    # the blank as a target: status 3
    short = e[:2299]                                 # fewer frames than tokens: status 4
    nan_end = e.copy()
    nan_end[5, 0] = np.nan                           # blank column early: S-1 turns NaN, status 1
    records = [(e, t), (e, bad), (short, t), (nan_end, t), (e, t)]
    es, ts = zip(*records)
    mask = torch.tensor([True, True, True, True, False], device=cuda)  # last: status 2
    result = ffa.align(*cuda_records(es, ts), blank_id=0, emission_validity=mask)
    assert result.status.cpu().tolist() == [0, 3, 4, 1, 2]
    ref = oracle.align(list(es), list(ts), 0, validity=mask.cpu().numpy().astype(np.uint8))
    assert_matches_oracle(result, ref, "long statuses")
    with pytest.raises(ValueError, match="target IDs"):
        result.raise_for_status()


def test_transcripts_beyond_the_cluster_limit_are_rejected(cuda):
    # 32768 tokens: 65537 states, more than a 16-CTA cluster holds.
    e = torch.zeros(70000, 32, device=cuda)
    t = torch.ones(32768, dtype=torch.int64, device=cuda)
    with pytest.raises(ValueError):
        ffa.align([e], [t])
