"""Token spans and timestamps on the GPU against the conversion the
reference's README describes (README.md:509-517), restated here in numpy:
split a path into equal-label runs, drop blank runs, keep each run's start and
exclusive end frame."""
import numpy as np
import pytest
import torch

import fast_forced_aligner_b200 as ffa
from fast_forced_aligner_b200 import workloads
from tests.helpers import cuda_records

pytestmark = pytest.mark.gpu


def runs(path, blank):
    out, start = [], 0
    for t in range(1, len(path) + 1):
        if t == len(path) or path[t] != path[t - 1]:
            if path[start] != blank:
                out.append((start, t))
            start = t
    return out


@pytest.mark.parametrize("mode", ["optimized", "conventional"])
def test_spans_follow_the_readme_recipe_on_cfg1(cuda, mode):
    wl = workloads.config(1)
    es, ts = cuda_records(*wl.records())
    batch = ffa.align(es, ts, blank_id=wl.blank, mode=mode)
    spans = ffa.token_spans(batch, wl.target_lengths, blank_id=wl.blank).cpu().numpy()
    assert spans.shape == (int(wl.target_lengths.sum()), 2)
    labels = [p.cpu().numpy() for p in batch.paths]
    for (p, t), got in zip(zip(labels, wl.records()[1]), np.split(spans, np.cumsum(wl.target_lengths)[:-1])):
        want = np.array(runs(p, wl.blank)).reshape(-1, 2)
        np.testing.assert_array_equal(got, want)
        for k, (a, b) in enumerate(got):       # each span holds exactly token k
            assert (p[a:b] == t[k]).all()
    seconds = ffa.token_timestamps(batch, wl.target_lengths, 0.02, blank_id=wl.blank).cpu().numpy()
    np.testing.assert_allclose(seconds, spans * 0.02)


def test_spans_of_failed_empty_and_repeated_records(cuda):
    rng = np.random.default_rng(4)
    V = 6
    e = np.log(np.full((12, V), 1.0 / V, np.float32))
    good = rng.standard_normal((20, V)).astype(np.float32)
    records = [
        (e, np.array([2, 2, 3])),   # repeated token: two blank-separated runs
        (e, np.array([], np.int64)),  # empty transcript: all blank, no spans
        (e, np.array([0, 1])),      # blank as a target: status 3, -1 spans
        (e[:2], np.array([1, 2, 3])),  # too few frames: status 4, -1 spans
        (good, np.array([4, 1, 4, 5])),
    ]
    es, ts = cuda_records(*zip(*records))
    batch = ffa.align(es, ts, blank_id=0, mode="conventional")
    status = batch.status.cpu().tolist()
    assert status[2] == 3 and status[3] == 4 and status[0] == 0 and status[1] == 0
    lengths = [len(t) for _, t in records]
    spans = ffa.token_spans(batch, lengths, blank_id=0).cpu().numpy()
    parts = np.split(spans, np.cumsum(lengths)[:-1])
    for (p, (_, t), s, st) in zip(batch.paths, records, parts, status):
        if st != 0:
            assert (s == -1).all()
            continue
        np.testing.assert_array_equal(s, np.array(runs(p.cpu().numpy(), 0)).reshape(-1, 2))
        assert len(s) == len(t)
    a, b = parts[0][0], parts[0][1]
    assert a[1] < b[0]                      # the repeated token's occurrences stay apart
    ts_ = ffa.token_timestamps(batch, lengths, 0.04, blank_id=0).cpu().numpy()
    assert np.isnan(ts_[np.cumsum(lengths)[1]:np.cumsum(lengths)[3]]).all()
    with pytest.raises(ValueError):
        ffa.token_spans(batch, lengths[:-1])
