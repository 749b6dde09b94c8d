"""The window route of the optimized mode: the greedy pass, the 64-state and
128-state certified window DPs, and the full-DP fallback.

The route's contract is stronger than the chunked route's: its outputs are
the conventional DP's, bit for bit, on every input -- ties included -- since
a record the window cannot certify runs the wider window and then the full
DP.  Every test compares against the CPU oracle with no tolerance, on inputs
built to drive each tier; the greedy chunk statistics are compared with the
restatement of the reference's greedy_shortcuts (oracle.greedy_chunk_stats)
and, where its extension is built, with the reference's own counts.
"""
import numpy as np
import pytest
import torch

import fast_forced_aligner_b200 as ffa
from fast_forced_aligner_b200 import workloads
from oracle import oracle
from tests.helpers import assert_matches_oracle, cuda_records
from tests.test_gpu_optimized import synthetic

pytestmark = pytest.mark.gpu


def window(es, ts, blank, **kw):
    d_es, d_ts = cuda_records(es, ts)
    return ffa.align(d_es, d_ts, blank_id=blank, mode="optimized", route="window", **kw)


def greedy_counts(es, ts, blanks):
    blanks = blanks if np.ndim(blanks) else [blanks] * len(es)
    return np.stack([oracle.greedy_chunk_stats(e, t, b) for e, t, b in zip(es, ts, blanks)])


@pytest.mark.parametrize("index, scale", [(0, 1.0), (1, 1.0), (4, 0.25)])
def test_configs_are_exact(cuda, index, scale):
    wl = workloads.config(index, scale=scale)
    es, ts = wl.records()
    result = window(es, ts, wl.blank)
    assert_matches_oracle(result, oracle.align(es, ts, wl.blank), f"cfg{index} window")
    np.testing.assert_array_equal(result.shortcut_stats.cpu().numpy(), greedy_counts(es, ts, wl.blank))
    routing = result.routing_stats.cpu().numpy()
    print(f"cfg{index} x{scale}: full-DP fallbacks {int((routing[:, 0] == 2).sum())}/{wl.batch}, "
          f"greedy chunks accepted {int(result.shortcut_stats[:, 0].sum())}")
    for name in ("stitched", "repair_passes", "repaired_frames"):
        assert getattr(result, name).count_nonzero() == 0, name


def test_constructed_ties_are_exact(cuda):
    # cfg4's 64 tie records (two equal-score paths one boundary apart): the
    # window route returns the conventional DP's choice.
    wl = workloads.config(4)
    sub = wl.subset(sorted(wl.tie_frames))
    es, ts = sub.records()
    assert_matches_oracle(window(es, ts, 0), oracle.align(es, ts, 0), "cfg4 ties")


@pytest.mark.parametrize("boost", [0.5, 1.5, 3.0])
def test_weak_emissions_use_every_tier_and_stay_exact(cuda, boost):
    # Weak emissions leave many states viable: records that the 64-state
    # window cannot certify go to the 128-state window and on to the full DP,
    # and every record still comes out as the conventional DP's.
    rng = np.random.default_rng(int(boost * 10) + 100)
    es, ts = zip(*(synthetic(rng, int(T), boost=boost) for T in rng.integers(65, 2400, 24)))
    es, ts = list(es), list(ts)
    result = window(es, ts, 0)
    assert_matches_oracle(result, oracle.align(es, ts, 0), f"boost {boost}")
    fallbacks = int((result.routing_stats[:, 0] == 2).sum())
    print(f"boost {boost}: full-DP fallbacks {fallbacks}/24")
    if boost == 0.5:
        assert fallbacks > 0  # the last tier ran


@pytest.mark.parametrize("lengths", [[1, 2, 3, 7, 8, 9, 31, 32, 33, 63, 64, 65],
                                     [127, 128, 129, 255, 256, 257, 1023, 1024, 1025, 2047, 2048, 2049]])
def test_boundary_lengths(cuda, lengths):
    # Frame counts at the 8-frame group, 32-frame segment and 128-frame greedy
    # chunk boundaries; transcripts from empty (S = 1) up.
    rng = np.random.default_rng(len(lengths) + lengths[-1])
    es, ts = zip(*(synthetic(rng, T, ratio=0.25) for T in lengths))
    es, ts = list(es), list(ts)
    es.append(np.log(np.full((5, 4), 0.25, np.float32)))
    ts.append(np.zeros(0, np.int64))  # U = 0: the blank path
    result = window(es, ts, 0)
    assert_matches_oracle(result, oracle.align(es, ts, 0), "lengths")
    np.testing.assert_array_equal(result.shortcut_stats.cpu().numpy(), greedy_counts(es, ts, 0))


def test_states_that_fill_and_exceed_the_window(cuda):
    # S below, at and above the 64- and 128-state windows, and up to 4095.
    rng = np.random.default_rng(21)
    es, ts = [], []
    for U in (1, 20, 31, 32, 33, 63, 64, 65, 200, 1000, 2047):
        T = max(int(U * 3.3) + 5, 8)
        e, t = synthetic(rng, T, ratio=U / T)
        es.append(e); ts.append(t)
    result = window(es, ts, 0)
    assert_matches_oracle(result, oracle.align(es, ts, 0), "state counts")


def test_long_records_and_the_wide_tier_limit(cuda):
    # Records past the wide tier's 4096 frames that the 64-state window does
    # not certify go straight to the full DP; up to 8192 frames on the route.
    rng = np.random.default_rng(33)
    es, ts = [], []
    for T, boost in ((4000, 1.0), (5000, 0.8), (8192, 4.0), (6000, 0.6)):
        e, t = synthetic(rng, T, boost=boost)
        es.append(e); ts.append(t)
    result = window(es, ts, 0)
    assert_matches_oracle(result, oracle.align(es, ts, 0), "long")


@pytest.mark.parametrize("poison", [np.nan, np.inf])
def test_poisoned_alphabet_columns_take_the_full_dp(cuda, poison):
    rng = np.random.default_rng(5)
    es, ts = [], []
    for k in range(8):
        e, t = synthetic(rng, 900)
        e[int(rng.integers(1, 890)), t[int(rng.integers(0, len(t)))] if k % 2 else 0] = poison
        es.append(e); ts.append(t)
    result = window(es, ts, 0)
    assert_matches_oracle(result, oracle.align(es, ts, 0), f"poison {poison}")
    assert (result.routing_stats[:, 0] == 2).all()


def test_flat_ties_and_positive_emissions(cuda):
    # All paths tie (no window is certified by a strict margin) and emissions
    # above 0 (the rounding bound assumes log-probabilities): the full DP.
    rng = np.random.default_rng(9)
    es, ts = [], []
    for T in (150, 400, 1100):
        es.append(np.zeros((T, 6), np.float32))
        ts.append(rng.integers(1, 6, T // 5).astype(np.int64))
    e, t = synthetic(rng, 700)
    es.append(e + np.float32(0.5)); ts.append(t)
    result = window(es, ts, 0)
    assert_matches_oracle(result, oracle.align(es, ts, 0), "flat and positive")


def test_statuses_and_masks(cuda):
    wl = workloads.config(1, scale=0.5)
    es, ts = [list(x) for x in wl.records()]
    ts[1] = ts[1].copy(); ts[1][3] = wl.blank          # status 3
    es[2] = es[2][: max(1, len(ts[2]) - 3)]            # status 4
    mask = np.ones(wl.batch, bool); mask[4] = False    # status 2
    ref = oracle.align(es, ts, wl.blank, validity=mask.astype(np.uint8))
    result = window(es, ts, wl.blank, emission_validity=torch.from_numpy(mask).to(cuda))
    assert set(ref.status[:5].tolist()) >= {2, 3, 4}
    assert_matches_oracle(result, ref, "statuses")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_logits_are_aligned_as_their_log_softmax(cuda, dtype):
    wl = workloads.config(1, scale=0.5)
    es, ts = wl.records()
    rng = np.random.default_rng(3)
    logits = [torch.from_numpy(e + rng.uniform(-5, 5, (e.shape[0], 1)).astype(np.float32)).to(cuda, dtype)
              for e in es]
    d_ts = [torch.from_numpy(t).to(cuda) for t in ts]
    fused = ffa.align(logits, d_ts, blank_id=wl.blank, mode="optimized", route="window", from_logits=True)
    plain = ffa.align(ffa.log_softmax(logits), d_ts, blank_id=wl.blank, mode="conventional")
    for name in ("labels", "scores", "status", "objective"):
        a, b = getattr(fused, name), getattr(plain, name)
        assert torch.equal(a.view(torch.int32) if a.dtype == torch.float32 else a,
                           b.view(torch.int32) if b.dtype == torch.float32 else b), name


def test_auto_route_policy(cuda):
    # Many short records: the window route (exact); few or long ones: the
    # chunked route.  Both are checked against the oracle in the same call.
    wl = workloads.config(4, scale=0.12)   # ~990 records, a few longer than 2048 frames
    es, ts = wl.records()
    d_es, d_ts = cuda_records(es, ts)
    result = ffa.align(d_es, d_ts, blank_id=0, mode="optimized")
    ref = oracle.align(es, ts, 0)
    labels = result.labels.cpu().numpy()
    off = wl.frame_offsets
    short = [i for i in range(wl.batch) if wl.lengths[i] <= 2048]
    for i in short:
        np.testing.assert_array_equal(labels[off[i]:off[i + 1]], ref.labels[off[i]:off[i + 1]])
    stitched = result.stitched.cpu().numpy()
    assert stitched[short].sum() == 0  # window records are never joined from pieces


@pytest.mark.parametrize("route", ["window", "pieces", "auto"])
def test_matches_the_references_greedy_counts(cuda, route):
    # The reference's own extension counts greedy chunks (shortcut_stats,
    # alignment.cu:130-153) in optimized mode: every route reports the same
    # numbers (the chunked route runs the greedy pass for them alone).
    if not oracle.load_reference_cuda():
        pytest.skip("reference CUDA extension not built under oracle/_ref")
    for index in (0, 1, 3):  # cfg3: 1,025 columns (the statistics-only wide pass)
        wl = workloads.config(index)
        es, ts = cuda_records(*wl.records())
        tensors, _ = oracle.reference_cuda_align(es, ts, [wl.blank] * wl.batch, mode="optimized")
        mine = ffa.align(es, ts, blank_id=wl.blank, mode="optimized", route=route)
        np.testing.assert_array_equal(mine.shortcut_stats.cpu().numpy(), tensors[7].cpu().numpy())


@pytest.mark.parametrize("route", ["pieces", "auto"])
@pytest.mark.parametrize("index, scale", [(0, 1.0), (1, 1.0), (4, 0.12), (3, 0.25)])
def test_chunked_route_counts_greedy_chunks(cuda, route, index, scale):
    # Records off the window route (pieces, short records, mixed batches)
    # carry the greedy statistics of the oracle's greedy_shortcuts
    # restatement as well; the outputs stay the route's own.
    wl = workloads.config(index, scale=scale)
    es, ts = wl.records()
    d_es, d_ts = cuda_records(es, ts)
    result = ffa.align(d_es, d_ts, blank_id=wl.blank, mode="optimized", route=route)
    np.testing.assert_array_equal(result.shortcut_stats.cpu().numpy(), greedy_counts(es, ts, wl.blank))
    assert int(result.shortcut_stats[:, 0].sum()) > 0


@pytest.mark.parametrize("V", [32, 30, 1025])
def test_greedy_counts_skip_rejected_records(cuda, V):
    # A record of status >= 2 runs no greedy chunk (alignment.cu:35): masked,
    # invalid IDs, too few frames -- on both routes, beside valid records
    # whose counts are unchanged.  V = 30 rows are gathered (not 16-byte
    # multiples) and V = 1025 exceeds the 64-bit alphabet mask: the
    # statistics-only wide pass counts those.
    rng = np.random.default_rng(5)
    T = 700
    good = torch.randn(T, V, device=cuda).log_softmax(-1)
    path = torch.from_numpy(rng.integers(1, V, 120)).to(cuda)
    strong = good.clone()
    strong[torch.arange(T, device=cuda), path.repeat_interleave(T // 120 + 1)[:T]] += 8
    strong = strong.log_softmax(-1)
    short = strong[:100].contiguous()
    ems = [strong, strong, strong, short]
    tgts = [path, torch.tensor([1, V + 8, 2], device=cuda), path, path]  # an ID past the row
    mask = torch.tensor([True, True, False, True], device=cuda)
    for route in ("pieces", "window"):
        result = ffa.align(ems, tgts, mode="optimized", route=route, emission_validity=mask)
        assert result.status.tolist()[1:] == [3, 2, 4]
        assert result.shortcut_stats[1:].count_nonzero() == 0
        expected = oracle.greedy_chunk_stats(strong.cpu().numpy(), path.cpu().numpy(), 0)
        np.testing.assert_array_equal(result.shortcut_stats[0].cpu().numpy(), expected)
        assert expected[0] > 0


@pytest.mark.parametrize("V", [30, 33, 129])
def test_gathered_vocabularies_count_greedy_chunks(cuda, V):
    # Records whose rows are gathered (V * 4 not a multiple of 16, or more
    # than 64 columns), with repeated tokens, random blanks and lengths at
    # the chunk boundaries: the oracle's counts, every route.
    rng = np.random.default_rng(V)
    es, ts, blanks = [], [], []
    for T in [1, 2, 127, 128, 129, 255, 256, 257, 700, 1500]:
        blank = int(rng.integers(0, V))
        choices = np.array([c for c in range(V) if c != blank])
        U = int(rng.integers(0, T // 3 + 1))
        tokens = rng.choice(choices[:6], U) if rng.random() < 0.3 else rng.choice(choices, U)
        x = rng.standard_normal((T, V)).astype(np.float32)
        if U:
            idx = np.sort(rng.choice(T, min(T, U), replace=False))
            x[idx, tokens[:idx.size]] += 8.0
        x[:, blank] += 3.0
        es.append(torch.from_numpy(x).log_softmax(-1).numpy())
        ts.append(tokens.astype(np.int64))
        blanks.append(blank)
    d_es, d_ts = cuda_records(es, ts)
    expected = greedy_counts(es, ts, blanks)
    assert expected[:, 0].sum() > 0
    for route in ("pieces", "window", "auto"):
        result = ffa.align(d_es, d_ts, blank_id=blanks, mode="optimized", route=route)
        np.testing.assert_array_equal(result.shortcut_stats.cpu().numpy(), expected, err_msg=route)
    conventional = ffa.align(d_es, d_ts, blank_id=blanks, mode="conventional")
    assert conventional.shortcut_stats.count_nonzero() == 0  # the reference counts none there


@pytest.mark.parametrize("V", [32, 1025])
def test_greedy_ties_of_normalised_logits(cuda, V):
    # Logits are aligned as x - z.  Two columns that differ by one ulp as
    # logits, where z is large, round to the same emission: a tie, which
    # rejects the chunk as it does on the materialised log_softmax.  At one
    # label change per 128-frame chunk, the next label's column is set one ulp
    # above the current one's (raw, the greedy label would just change a frame
    # early).
    rng = np.random.default_rng(V + 1)
    T, U, blank = 1024, 160, 0
    far = V - 1  # a column no label uses; it makes z about 1000
    tokens = rng.integers(1, far, U)
    tokens[1:][tokens[1:] == tokens[:-1]] = far - 1
    path = np.repeat(np.arange(U), T // U + 1)[:T]
    x = rng.standard_normal((T, V)).astype(np.float32)
    x[np.arange(T), tokens[path]] += 8.0
    x[:, far] = 1000.0
    changes = [t for t in range(T - 1) if path[t] != path[t + 1]]
    planted = [next(t for t in changes if t >= c) for c in range(0, T - 128, 128)]
    for t in planted:
        cur, nxt = tokens[path[t]], tokens[path[t + 1]]
        x[t, nxt] = np.nextafter(x[t, cur], np.float32(np.inf))
    logits = torch.from_numpy(x).to(cuda)
    target = torch.from_numpy(tokens.astype(np.int64)).to(cuda)
    fused = ffa.align([logits], [target], blank_id=blank, mode="optimized", from_logits=True)
    emissions = ffa.log_softmax([logits])
    plain = ffa.align(emissions, [target], blank_id=blank, mode="optimized")
    e = emissions[0].cpu().numpy()
    ties = sum(int(e[t, tokens[path[t]]] == e[t, tokens[path[t + 1]]]) for t in planted)
    assert ties > 0  # the planted pairs collide after the subtraction
    expected = oracle.greedy_chunk_stats(e, tokens, blank)
    np.testing.assert_array_equal(plain.shortcut_stats[0].cpu().numpy(), expected)
    np.testing.assert_array_equal(fused.shortcut_stats[0].cpu().numpy(), expected)
