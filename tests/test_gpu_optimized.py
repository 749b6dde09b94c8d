"""The optimized route: records split into pieces, seams checked, repairs
resumed from saved frontiers, conventional fallback.

Its contract is the conventional DP's exact outputs on every input without
ties (the optimized route's contract), so every test here compares against the CPU
oracle bit for bit, on inputs built to drive each branch of the route:
confident and weak emissions (joins, repairs, chains of failing seams,
fallback), piece-boundary lengths, NaN and +inf emissions (fallback, and the
NaN that a reference DP leaves on a not yet reachable state), row-staged and
gathered vocabularies in one batch.
"""
import numpy as np
import pytest
import torch

import fast_forced_aligner_b200 as ffa
from fast_forced_aligner_b200 import workloads
from oracle import oracle
from tests.helpers import assert_matches_oracle, assert_same_optimum, cuda_records

pytestmark = pytest.mark.gpu

PIECE_MIN_FRAMES = 65  # records shorter than this run the conventional DP in both modes


def log_softmax(x):
    x = x - x.max(axis=1, keepdims=True)
    return (x - np.log(np.exp(x).sum(axis=1, keepdims=True))).astype(np.float32)


def synthetic(rng, T, V=32, blank=0, ratio=0.3, boost=4.0, repeats=0.1):
    """One record drawn like workloads.config(1): a random transcript, a
    random monotone frame labelling, N(0,1) logits with `boost` on the true
    label, log-softmax in fp32."""
    U = max(1, int(ratio * T))
    choices = np.array([c for c in range(V) if c != blank])
    tokens = [int(rng.choice(choices))]
    while len(tokens) < U:
        if rng.random() < repeats:
            tokens.append(tokens[-1])
        else:
            tokens.append(int(rng.choice(choices[choices != tokens[-1]])))
    tokens = np.array(tokens, np.int64)
    reps = int((tokens[1:] == tokens[:-1]).sum())
    assert U + reps <= T
    # Mandatory frames: one per token, one blank between repeats; the rest spread.
    slots = np.ones(2 * U + 1, np.int64)
    slots[0::2] = 0
    slots[2:-1:2][tokens[1:] == tokens[:-1]] = 1
    slots += rng.multinomial(T - slots.sum(), np.ones(2 * U + 1) / (2 * U + 1))
    states = np.repeat(np.arange(2 * U + 1), slots)
    labels = np.where(states % 2 == 1, tokens[(states - 1) // 2], blank)
    logits = rng.standard_normal((T, V)).astype(np.float32)
    logits[np.arange(T), labels] += boost
    return log_softmax(logits), tokens


def run_both(es, ts, blank, mode):
    ref = oracle.align(es, ts, blank)
    d_es, d_ts = cuda_records(es, ts)
    return ffa.align(d_es, d_ts, blank_id=blank, mode=mode), ref


def test_route_diagnostics_on_cfg1(cuda):
    wl = workloads.config(1)
    es, ts = cuda_records(*wl.records())
    opt = ffa.align(es, ts, blank_id=wl.blank, mode="optimized")
    conv = ffa.align(es, ts, blank_id=wl.blank, mode="conventional")
    stitched = opt.stitched.cpu().numpy()
    passes = opt.repair_passes.cpu().numpy()
    frames = opt.repaired_frames.cpu().numpy()
    long = wl.lengths >= PIECE_MIN_FRAMES
    print(f"cfg1 optimized: joined {int(stitched.sum())}/{wl.batch}, repaired {int((passes > 0).sum())}, "
          f"repair passes {np.bincount(passes).tolist()}, repaired frames {int(frames.sum())}")
    assert set(np.unique(stitched)) <= {0, 1}
    assert (stitched[~long] == 0).all()
    assert stitched[long].mean() >= 0.9   # confident emissions join (most after at most one repair)
    assert ((passes >= 0) & (passes <= 2)).all()
    assert ((frames > 0) == (passes > 0)).all()
    assert passes.sum() > 0                 # the repair path ran
    for name in ("stitched", "repair_passes", "repaired_frames", "shortcut_stats", "routing_stats"):
        assert getattr(conv, name).count_nonzero() == 0, name
    for name in ("labels", "scores", "status", "objective"):
        assert torch.equal(getattr(opt, name).view(torch.int32) if name in ("scores", "objective")
                           else getattr(opt, name),
                           getattr(conv, name).view(torch.int32) if name in ("scores", "objective")
                           else getattr(conv, name)), name


@pytest.mark.parametrize("boost", [0.5, 1.5, 3.0])
def test_weak_emissions_repairs_chains_and_fallback(cuda, boost):
    # Low-confidence emissions make many seams fail: consecutive failures
    # merge into multi-piece repairs, a second round and conventional
    # fallback all run.  Weak emissions also produce fp32 ties inside the
    # conventional DP: two paths whose scores differ by less than the
    # rounding step of the running sum (e.g. 8.8e-6 against a 1.2e-4 ulp at
    # -1800), which the conventional DP resolves by its stay-first rule and a
    # piece, summing from a smaller base, resolves by the actual scores.  So
    # every record must reach the conventional optimum (fp64 rescoring within
    # rounding), and almost every record must match bit for bit.
    rng = np.random.default_rng(int(boost * 10))
    es, ts = zip(*(synthetic(rng, int(T), boost=boost) for T in rng.integers(65, 2400, 24)))
    result, ref = run_both(list(es), list(ts), 0, "optimized")
    same = assert_same_optimum(result, ref, es, ts, 0, f"boost {boost}")
    passes = result.repair_passes.cpu().numpy()
    print(f"boost {boost}: joined {int(result.stitched.sum())}/24, conventional path on {same}/24, "
          f"repair passes {np.bincount(passes, minlength=3).tolist()}")
    assert same >= 21


@pytest.mark.parametrize("mode", ["optimized", "conventional"])
def test_piece_boundary_lengths(cuda, mode):
    rng = np.random.default_rng(7)
    lengths = [1, 2, 31, 32, 33, 47, 48, 49, 63, 64, 65, 66, 79, 80, 81, 95, 96, 97, 111, 112, 113, 127,
               128, 129, 130, 159, 160, 161, 191, 192, 193, 223, 224, 255, 256, 257, 319, 320, 321, 1000,
               1023, 1024, 1025]
    es, ts = zip(*(synthetic(rng, T, ratio=0.25) for T in lengths))
    result, ref = run_both(list(es), list(ts), 0, mode)
    assert_matches_oracle(result, ref, mode)
    # The same lengths with the last frame on the last token (terminal state
    # S-2, odd), so that every record's last frame carries a token label.
    ends = []
    for e, t in zip(es, ts):
        e = e.copy()
        e[-1, :] = -30.0
        e[-1, t[-1]] = 0.0
        ends.append(e)
    result, ref = run_both(ends, list(ts), 0, mode)
    last = np.cumsum([e.shape[0] for e in ends]) - 1
    assert (ref.labels[last] != 0).all()
    assert_matches_oracle(result, ref, mode + " token-ended")


def test_mixed_row_and_gather_vocabularies(cuda):
    # V=32 rows are TMA-staged, V=1025 columns are gathered: both launches of
    # every phase run in one call, short and long records mixed.
    rng = np.random.default_rng(11)
    es, ts = [], []
    for T, V in [(90, 32), (700, 32), (1500, 32), (120, 1025), (800, 1025), (1300, 1025), (400, 33)]:
        e, t = synthetic(rng, T, V=V, blank=V - 1 if V > 32 else 0)
        es.append(e); ts.append(t)
    blanks = [0, 0, 0, 1024, 1024, 1024, 32]
    ref = oracle.align(es, ts, blanks)
    d_es, d_ts = cuda_records(es, ts)
    for mode in ("optimized", "conventional"):
        result = ffa.align(d_es, d_ts, blank_id=blanks, mode=mode)
        assert_matches_oracle(result, ref, mode)


def test_nan_inside_the_band_falls_back(cuda):
    # A NaN emission on a reachable state stays NaN on that state; the route
    # cannot reason about it and hands the record to the conventional DP.
    rng = np.random.default_rng(3)
    es, ts = [], []
    for k in range(6):
        e, t = synthetic(rng, 600)
        f = int(rng.integers(100, 500))
        e[f, t[int(rng.integers(0, len(t)))] if k % 2 else 0] = np.nan
        es.append(e); ts.append(t)
    result, ref = run_both(es, ts, 0, "optimized")
    assert_matches_oracle(result, ref, "nan")
    assert (result.stitched.cpu().numpy() == 0).all()


@pytest.mark.parametrize("mode", ["optimized", "conventional"])
@pytest.mark.parametrize("poison", [np.nan, np.inf])
def test_poison_on_unreachable_states(cuda, mode, poison):
    # -inf + NaN and -inf + inf are NaN: the reference DP marks a state that is
    # not yet reachable as NaN when such an emission lands on it, and the NaN
    # stays.  Frames where whole warps sit above the reachable band must keep
    # that, so these records (poison early, on states far above the band)
    # must come out as the oracle says -- most of them infeasible.
    rng = np.random.default_rng(5)
    es, ts = [], []
    for k in range(8):
        e, t = synthetic(rng, 1600, ratio=0.3)
        f = int(rng.integers(1, 40))
        u = int(rng.integers(len(t) // 2, len(t)))
        e[f, t[u]] = poison           # every state of that label from frame f on
        if k % 4 == 3:
            e[f + 1, 0] = poison      # and every blank
        es.append(e); ts.append(t)
    # Controls: a token whose state is unreachable at the poisoned frame and
    # whose label occurs nowhere else keeps the record feasible only in the
    # band-skipping bug's world.
    result, ref = run_both(es, ts, 0, mode)
    assert_matches_oracle(result, ref, f"{mode} {poison}")
    print(f"{mode} {poison}: oracle status {ref.status.tolist()}")


def test_flat_ties_on_long_records(cuda):
    # Every legal path scores the same: the optimized route must return one of
    # them (the conventional one in conventional mode).
    rng = np.random.default_rng(9)
    es, ts = [], []
    for T in (150, 400, 1100):
        t = rng.integers(1, 6, T // 5).astype(np.int64)
        es.append(np.zeros((T, 6), np.float32)); ts.append(t)
    result, ref = run_both(es, ts, 0, "optimized")
    assert_same_optimum(result, ref, es, ts, 0, "flat")
    conv, _ = run_both(es, ts, 0, "conventional")
    assert_matches_oracle(conv, ref, "flat conventional")


def test_many_records_with_masks_and_rejections(cuda):
    # More records than SMs: round 0 is planned in the first pass, records it
    # joins skip the finisher, and the finisher's lists are built on the
    # device.  Masked records (status 2), invalid targets (3) and infeasible
    # lengths (4) must still get their routes and outputs.
    wl = workloads.config(1, scale=5)  # 320 records
    es, ts = [list(x) for x in wl.records()]
    rng = np.random.default_rng(12)
    for i in rng.choice(wl.batch, 12, replace=False):
        ts[i] = ts[i].copy()
        ts[i][len(ts[i]) // 2] = wl.blank          # status 3
    for i in rng.choice(wl.batch, 6, replace=False):
        es[i] = es[i][: max(1, len(ts[i]) - 3)]    # status 4
    mask = np.ones(wl.batch, bool)
    mask[rng.choice(wl.batch, 20, replace=False)] = False
    ref = oracle.align(es, ts, wl.blank, validity=mask.astype(np.uint8))
    d_es, d_ts = cuda_records(es, ts)
    validity = torch.from_numpy(mask).to(cuda)
    for mode in ("optimized", "conventional"):
        result = ffa.align(d_es, d_ts, blank_id=wl.blank, mode=mode, emission_validity=validity)
        assert set(np.unique(ref.status)) >= {0, 2, 3}
        if mode == "conventional":
            assert_matches_oracle(result, ref, mode)
        else:
            assert_same_optimum(result, ref, es, ts, wl.blank, mode)
            stitched = result.stitched.cpu().numpy()
            assert stitched[ref.status == 0].mean() > 0.9
            assert (stitched[ref.status != 0] == 0).all()
