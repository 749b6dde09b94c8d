"""The reference's GPU test behaviours, re-expressed against this package.

Sources: tests/test_core.py, tests/test_async_validation.py and
tests/test_emission_validity.py of brthor/fast-forced-aligner (cited per
test).  Every result is also checked bit for bit against the CPU oracle.
"""
from dataclasses import fields

import numpy as np
import pytest
import torch

import fast_forced_aligner_b200 as ffa
from oracle import oracle
from tests.helpers import assert_matches_oracle, assert_same_optimum, collapse

pytestmark = pytest.mark.gpu
MODES = ["optimized", "conventional"]


def oracle_of(es, ts, blank=0, **kw):
    return oracle.align([e.cpu().numpy() for e in es], [t.cpu().numpy() for t in ts], blank, **kw)


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("blank", [0, 5])
def test_ragged_long_repeats_empty_transcript_and_exact_scores(cuda, mode, blank):
    # tests/test_core.py:29-48
    rng = np.random.default_rng(32)
    labels = np.array([i for i in range(6) if i != blank])
    values = [rng.integers(-9, 0, (n, 6)).astype(np.float32) for n in (7, 129, 257, 2305)]
    tokens = [rng.choice(labels, n) for n in (0, 11, 44, 120)]
    es = [torch.tensor(v, device=cuda) for v in values]
    ts = [torch.tensor(t, dtype=torch.int64, device=cuda) for t in tokens]
    actual = ffa.align(es, ts, blank_id=blank, mode=mode)
    actual.raise_for_status()
    offset = 0
    for v, t, path in zip(values, tokens, actual.paths, strict=True):
        p = path.cpu().numpy()
        np.testing.assert_array_equal(collapse(p, blank), t)
        selected = v[np.arange(len(p)), p]
        np.testing.assert_array_equal(actual.scores[offset:offset + len(p)].cpu(), selected)
        offset += len(p)
    # Integer-valued emissions tie everywhere: the optimized route must reach
    # the conventional optimum; the conventional route is the reference's.
    if mode == "optimized":
        assert_same_optimum(actual, oracle_of(es, ts, blank), values, tokens, blank, "ragged ties")
    else:
        assert_matches_oracle(actual, oracle_of(es, ts, blank))


@pytest.mark.parametrize("tokens", [[-1], [6], [0], [1, 1, 1, 1]])
def test_bad_tokens_are_rejected_before_native_read(cuda, tokens):
    # tests/test_core.py:51-55
    result = ffa.align([torch.zeros(4, 6, device=cuda)], [torch.tensor(tokens, device=cuda)])
    with pytest.raises(ValueError, match="target IDs|insufficient"):
        result.raise_for_status()


@pytest.mark.parametrize("mode", MODES)
def test_infeasible_status_and_input_mutation(cuda, mode):
    # tests/test_core.py:58-69
    e = torch.full((257, 4), -torch.inf, device=cuda)
    t = torch.tensor([1], device=cuda)
    failed = ffa.align([e], [t], mode=mode)
    with pytest.raises(ValueError, match="no finite"):
        failed.raise_for_status()
    e.zero_()
    good = ffa.align([e], [t], mode=mode)
    good.raise_for_status()
    assert good.status.item() == 0 and failed.status.item() == 1
    assert good.labels.data_ptr() != failed.labels.data_ptr()


def test_heterogeneous_blanks_and_nondefault_stream(cuda):
    # tests/test_core.py:72-82
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        es = [torch.zeros(256, 6, device=cuda), torch.zeros(2110, 8, device=cuda)]
        ts = [torch.tensor([1, 1, 2], device=cuda), torch.tensor([0, 1, 1], device=cuda)]
        ffa.validate_inputs(es, ts, blank_id=[0, 7])
        result = ffa.align(es, ts, blank_id=[0, 7], check_inputs=False)
        del es, ts
    torch.cuda.current_stream().wait_stream(stream)
    result.raise_for_status()
    assert result.lengths == (256, 2110)


def test_shape_and_option_contracts(cuda):
    # tests/test_core.py:85-93
    e = torch.zeros(12, 6, device=cuda)
    t = torch.tensor([1], device=cuda)
    for values, targets, kwargs in [([], [], {}), ([e], [], {}),
                                   ([e[:, ::2]], [t], {}), ([e.double()], [t], {}),
                                   ([e], [t.int()], {}), ([e], [t], {"blank_id": 6}),
                                   ([e], [t], {"mode": "unknown"})]:
        with pytest.raises(ValueError):
            ffa.align(values, targets, **kwargs)


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("frames", [7, 257, 2305])
def test_mixed_invalid_targets_preserve_good_outputs_and_cuda_context(cuda, mode, frames):
    # tests/test_async_validation.py:13-36
    generator = torch.Generator(device=cuda).manual_seed(12)
    emission = torch.randn(frames, 6, generator=generator, device=cuda).log_softmax(-1)
    token_lists = [[1, 1, 2], [-1], [6], [0], [2**32 + 1], [2**63 - 1], [-2**63], []]
    targets = [torch.tensor(t, dtype=torch.int64, device=cuda) for t in token_lists]
    result = ffa.align([emission] * len(targets), targets, mode=mode)
    assert result.status.tolist() == [0, 3, 3, 3, 3, 3, 3, 0]
    for i in range(1, 7):
        assert (result.paths[i] == -1).all()
        assert torch.isneginf(result.scores.split(result.lengths)[i]).all()
        assert torch.isneginf(result.objective[i])
        assert result.stitched[i] == 0
        assert result.repair_passes[i] == 0
        assert result.shortcut_stats[i].count_nonzero() == 0
    with pytest.raises(ValueError, match=r"invalid target IDs.*\[1, 2, 3, 4, 5, 6\]"):
        result.raise_for_status()
    expected = ffa.align([emission, emission], [targets[0], targets[-1]], mode=mode, check_inputs=False)
    expected.raise_for_status()
    for actual_i, expected_i in ((0, 0), (7, 1)):
        assert torch.equal(result.paths[actual_i], expected.paths[expected_i])
        assert torch.equal(result.scores.split(result.lengths)[actual_i],
                           expected.scores.split(expected.lengths)[expected_i])
    assert_matches_oracle(result, oracle_of([emission] * len(targets), targets))


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("tokens", [1, 129, 257, 2047])
def test_repeat_reduction_and_exact_frame_feasibility(cuda, mode, tokens):
    # tests/test_async_validation.py:39-56
    target = torch.ones(tokens, dtype=torch.int64, device=cuda)
    enough = torch.zeros(2 * tokens - 1, 3, device=cuda)
    targets, emissions = [target], [enough]
    if tokens > 1:
        targets.append(target)
        emissions.append(enough[:-1])
    result = ffa.align(emissions, targets, mode=mode)
    assert result.status.tolist() == ([0, 4] if tokens > 1 else [0])
    collapsed = torch.unique_consecutive(result.paths[0])
    assert torch.equal(collapsed[collapsed != 0], target)
    if tokens > 1:
        assert (result.paths[1] == -1).all()
        with pytest.raises(ValueError, match=r"insufficient CTC frames.*\[1\]"):
            result.raise_for_status()
    assert_matches_oracle(result, oracle_of(emissions, targets))


@pytest.mark.parametrize("mode", MODES)
def test_long_target_invalid_tail_and_per_record_blanks(cuda, mode):
    # tests/test_async_validation.py:59-68
    good = torch.arange(513, device=cuda, dtype=torch.int64) % 4
    bad = good.clone()
    bad[-1] = 2**32 + 1
    result = ffa.align([torch.zeros(600, 6, device=cuda), torch.zeros(600, 5, device=cuda)],
                       [good, bad], blank_id=[5, 4], mode=mode)
    assert result.status.tolist() == [0, 3]


@pytest.mark.parametrize("mode", MODES)
def test_error_precedence_and_all_failure_categories(cuda, mode):
    # tests/test_async_validation.py:71-85
    emissions = [torch.zeros(3, 4, device=cuda) for _ in range(5)]
    emissions[-1].fill_(-torch.inf)
    targets = [torch.tensor(t, device=cuda) for t in ([9], [1, 1, 1], [1], [0, 0, 0, 0], [1])]
    result = ffa.align(emissions, targets, mode=mode,
                       emission_validity=torch.tensor([False, False, False, True, True], device=cuda))
    assert result.status.tolist() == [3, 4, 2, 3, 1]
    with pytest.raises(ValueError) as error:
        result.raise_for_status()
    for message in ("invalid emissions at batch indices [2]", "no finite complete CTC path for batch indices [4]",
                    "invalid target IDs at batch indices [0, 3]", "insufficient CTC frames at batch indices [1]"):
        assert message in str(error.value)
    assert (result.labels == -1).all()
    assert torch.isneginf(result.scores).all()


@pytest.mark.parametrize("mode", MODES)
def test_default_validation_has_no_host_read(cuda, mode):
    # tests/test_async_validation.py:88-101
    e = torch.zeros(257, 4, device=cuda)
    good, bad = torch.tensor([1, 2], device=cuda), torch.tensor([-1], device=cuda)
    ffa.align([e, e], [good, bad], mode=mode)
    torch.cuda.synchronize()
    previous = torch.cuda.get_sync_debug_mode()
    torch.cuda.set_sync_debug_mode("error")
    try:
        result = ffa.align([e, e], [good, bad], mode=mode)
    finally:
        torch.cuda.set_sync_debug_mode(previous)
    assert result.status.tolist() == [0, 3]


@pytest.mark.parametrize("mode", MODES)
def test_checked_and_unchecked_outputs_and_diagnostics_match(cuda, mode):
    # tests/test_async_validation.py:104-115
    generator = torch.Generator(device=cuda).manual_seed(42)
    emissions = [torch.randn(n, 8, device=cuda, generator=generator).log_softmax(-1) for n in (7, 257, 2305)]
    targets = [torch.tensor([1, 1, 2], device=cuda) for _ in emissions]
    checked = ffa.align(emissions, targets, mode=mode)
    unchecked = ffa.align(emissions, targets, mode=mode, check_inputs=False)
    for field in fields(checked):
        a, b = getattr(checked, field.name), getattr(unchecked, field.name)
        assert torch.equal(a, b) if isinstance(a, torch.Tensor) else a == b
    checked.raise_for_status()
    unchecked.raise_for_status()


def test_disabled_validation_and_explicit_synchronous_validator(cuda):
    # tests/test_async_validation.py:118-126
    emission = torch.zeros(2, 4, device=cuda)
    target = torch.tensor([1, 1], device=cuda)
    assert ffa.align([emission], [target]).status.item() == 4
    assert ffa.align([emission], [target], check_inputs=False).status.item() == 1
    with pytest.raises(ValueError, match="insufficient CTC frames"):
        ffa.validate_inputs([emission], [target])


def test_validation_on_consumer_stream_preserves_input_lifetime(cuda):
    # tests/test_async_validation.py:129-139
    producer, consumer = torch.cuda.Stream(), torch.cuda.Stream()
    with torch.cuda.stream(producer):
        emissions = [torch.zeros(2305, 6, device=cuda) for _ in range(2)]
        targets = [torch.tensor(t, device=cuda) for t in ([1, 2], [2**32 + 1])]
    consumer.wait_stream(producer)
    with torch.cuda.stream(consumer):
        result = ffa.align(emissions, targets)
        del emissions, targets
    torch.cuda.current_stream().wait_stream(consumer)
    assert result.status.tolist() == [0, 3]


def test_unknown_status_still_raises(cuda):
    # tests/test_async_validation.py:142-147
    result = ffa.align([torch.zeros(7, 4, device=cuda)], [torch.tensor([1], device=cuda)])
    with torch.inference_mode():
        result.status.fill_(99)
    with pytest.raises(RuntimeError, match="unknown alignment status"):
        result.raise_for_status()


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("frames", [7, 257, 2305])
def test_invalid_records_are_excluded_and_valid_records_unchanged(cuda, mode, frames):
    # tests/test_emission_validity.py:10-43
    generator = torch.Generator(device=cuda).manual_seed(11)
    good = torch.randn(frames, 6, generator=generator, device=cuda).log_softmax(-1)
    negative_infinity = good.clone()
    negative_infinity[:, 5] = -torch.inf
    nan, positive_infinity = good.clone(), good.clone()
    nan[-1, 5] = torch.nan
    positive_infinity[0, 5] = torch.inf
    impossible = torch.full_like(good, -torch.inf)
    emissions = [good, nan, positive_infinity, negative_infinity, impossible]
    targets = [torch.tensor([1, 1, 2], device=cuda) for _ in emissions]
    mask = ffa.emission_validity(emissions)
    assert mask.dtype == torch.bool and mask.device == good.device
    assert mask.tolist() == [True, False, False, True, True]
    actual = ffa.align(emissions, targets, mode=mode, emission_validity=mask, check_inputs=False)
    assert actual.status.tolist() == [0, 2, 2, 0, 1]
    for i in (1, 2, 4):
        assert (actual.paths[i] == -1).all()
        assert torch.isneginf(actual.scores.split(actual.lengths)[i]).all()
    assert torch.isneginf(actual.objective[1:3]).all()
    assert actual.stitched[1:3].tolist() == [0, 0]
    assert actual.repair_passes[1:3].tolist() == [0, 0]
    assert actual.shortcut_stats[1:3].count_nonzero() == 0
    expected = ffa.align([good, negative_infinity], [targets[0], targets[3]], mode=mode, check_inputs=False)
    for actual_i, expected_i in ((0, 0), (3, 1)):
        assert torch.equal(actual.paths[actual_i], expected.paths[expected_i])
        assert torch.equal(actual.scores.split(actual.lengths)[actual_i],
                           expected.scores.split(expected.lengths)[expected_i])
    with pytest.raises(ValueError, match="invalid emissions.*1, 2.*no finite.*4"):
        actual.raise_for_status()
    assert mask.cpu().numpy().tolist() == oracle.emission_validity([e.cpu().numpy() for e in emissions]).tolist()


@pytest.mark.parametrize("mode", MODES)
def test_empty_target_and_subset_of_all_record_validity(cuda, mode):
    # tests/test_emission_validity.py:46-60
    emissions = [torch.zeros(260, 4, device=cuda) for _ in range(4)]
    emissions[0][-1, -1] = torch.nan
    emissions[1][-1, -1] = torch.inf
    emissions[3][-1, -1] = torch.nan
    all_records = ffa.emission_validity(emissions)
    selection = torch.tensor([1, 3], device=cuda)
    result = ffa.align([emissions[1], emissions[3]],
                       [torch.empty(0, dtype=torch.int64, device=cuda) for _ in range(2)],
                       mode=mode, check_inputs=False, emission_validity=all_records.index_select(0, selection))
    assert all_records.tolist() == [False, False, True, False]
    assert result.status.tolist() == [2, 2]
    assert (result.labels == -1).all()


def test_mask_does_not_bypass_target_validation(cuda):
    # tests/test_emission_validity.py:63-67
    emission = torch.full((7, 4), torch.nan, device=cuda)
    result = ffa.align([emission], [torch.tensor([20], device=cuda)],
                       emission_validity=ffa.emission_validity([emission]))
    with pytest.raises(ValueError, match="target IDs"):
        result.raise_for_status()


def test_numeric_scan_and_guarded_submission_do_not_read_device_values(cuda):
    # tests/test_emission_validity.py:70-84
    emission = torch.zeros(257, 4, device=cuda)
    target = torch.tensor([1, 2], device=cuda)
    ffa.align([emission], [target], check_inputs=False, emission_validity=ffa.emission_validity([emission]))
    torch.cuda.synchronize()
    previous = torch.cuda.get_sync_debug_mode()
    torch.cuda.set_sync_debug_mode("error")
    try:
        validity = ffa.emission_validity([emission])
        result = ffa.align([emission], [target], check_inputs=False, emission_validity=validity)
    finally:
        torch.cuda.set_sync_debug_mode(previous)
    assert result.status.item() == 0


def test_numeric_scan_and_mask_have_correct_nondefault_stream_lifetime(cuda):
    # tests/test_emission_validity.py:87-98
    producer, consumer = torch.cuda.Stream(), torch.cuda.Stream()
    with torch.cuda.stream(producer):
        emissions = [torch.zeros(2305, 6, device=cuda), torch.full((257, 4), torch.nan, device=cuda)]
        targets = [torch.tensor([1, 2], device=cuda) for _ in emissions]
        validity = ffa.emission_validity(emissions)
    consumer.wait_stream(producer)
    with torch.cuda.stream(consumer):
        result = ffa.align(emissions, targets, check_inputs=False, emission_validity=validity)
        del validity, emissions, targets
    torch.cuda.current_stream().wait_stream(consumer)
    assert result.status.tolist() == [0, 2]


@pytest.mark.parametrize("kind", ["cpu", "dtype", "count", "rank", "strided"])
def test_malformed_mask_is_rejected(cuda, kind):
    # tests/test_emission_validity.py:101-112
    mask = {
        "cpu": lambda: torch.tensor([True]),
        "dtype": lambda: torch.tensor([1], device=cuda),
        "count": lambda: torch.empty(2, dtype=torch.bool, device=cuda),
        "rank": lambda: torch.ones(1, 1, dtype=torch.bool, device=cuda),
        "strided": lambda: torch.ones(4, dtype=torch.bool, device=cuda)[::2],
    }[kind]()
    with pytest.raises(ValueError, match="emission_validity"):
        ffa.align([torch.zeros(7, 4, device=cuda)], [torch.tensor([1], device=cuda)], emission_validity=mask)


@pytest.mark.parametrize("kind", ["empty", "cpu", "dtype", "strided", "zero_frames"])
def test_malformed_scan_inputs_are_rejected(cuda, kind):
    # tests/test_emission_validity.py:115-124
    emissions = {
        "empty": lambda: [],
        "cpu": lambda: [torch.zeros(7, 4)],
        "dtype": lambda: [torch.zeros(7, 4, dtype=torch.float16, device=cuda)],
        "strided": lambda: [torch.zeros(7, 4, device=cuda).T],
        "zero_frames": lambda: [torch.zeros(0, 4, device=cuda)],
    }[kind]()
    with pytest.raises(ValueError):
        ffa.emission_validity(emissions)


def test_emission_validity_scans_unaligned_views_and_large_records(cuda):
    big = torch.zeros(70001, 33, device=cuda)
    views = [big[1:], big[2:5], big[:1]]
    assert ffa.emission_validity(views).tolist() == [True, True, True]
    big[-1, -1] = torch.inf
    big[3, 0] = torch.nan
    assert ffa.emission_validity([big[1:], big[4:], big[:3], big[:4]]).tolist() == [False, False, True, False]


def test_emission_validity_random_views_and_chunk_edges(cuda):
    # Views start at arbitrary element offsets (not 16-byte aligned) and end
    # anywhere; NaN, +inf and -inf land at random positions, some right at
    # 64 KiB chunk and view edges.  The mask must equal a host scan.
    rng = np.random.default_rng(99)
    n = 3_000_000
    host = rng.standard_normal(n).astype(np.float32)
    spots = np.r_[rng.integers(0, n, 40), np.arange(16383, n, 16384)[:20], [0, n - 1]]
    host[spots] = rng.choice(np.array([np.nan, np.inf, -np.inf], np.float32), spots.size)
    flat = torch.from_numpy(host).to(cuda)
    starts = rng.integers(0, n - 1, 300)
    sizes = np.minimum(rng.integers(1, 400_000, 300), n - starts)
    widths = rng.choice([1, 3, 4, 32, 33], 300)
    views, expect = [], []
    for s0, size, w in zip(starts, sizes, widths):
        rows = max(1, int(size) // int(w))
        if s0 + rows * w > n:
            rows = (n - s0) // w
        views.append(flat[s0:s0 + rows * w].view(rows, int(w)))
        chunk = host[s0:s0 + rows * w]
        expect.append(not (np.isnan(chunk).any() or np.isposinf(chunk).any()))
    assert ffa.emission_validity(views).tolist() == expect
