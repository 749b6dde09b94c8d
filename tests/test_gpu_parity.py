"""Bit-exact parity of the CUDA path with the CPU oracle, the reference's
own CPU comparator (golden fixtures) and the reference's own CUDA extension.

Configs follow the benchmark configurations (fast_forced_aligner_b200.workloads); cfg4 runs
at full size.  Conventional mode returns the oracle's outputs bit for bit on
every record.  Optimized mode does too on the window route; on the chunked
route a record may get another path only where the conventional DP met an
fp32 tie, and every such record is classified exactly
(tests/helpers.classify_divergence) and counted against pinned numbers.
"""
import ctypes

import numpy as np
import pytest
import torch

import fast_forced_aligner_b200 as ffa
from fast_forced_aligner_b200 import workloads
from oracle import oracle
from tests.golden.make_golden import load as load_golden
from tests.helpers import (assert_matches_oracle, assert_same_bits, classify_divergence, collapse,
                           cuda_records, sequential_sum)

pytestmark = pytest.mark.gpu
MODES = ["optimized", "conventional"]

_CACHE = {}


def config(index, scale=1.0):
    key = (index, scale)
    if key not in _CACHE:
        wl = workloads.config(index, scale=scale)
        es, ts = wl.records()
        _CACHE[key] = (wl, oracle.align(es, ts, wl.blank))
    return _CACHE[key]


@pytest.mark.parametrize("mode", MODES)
def test_golden_reference_cpu_cases(cuda, mode):
    cases = load_golden()
    es, ts = cuda_records([c[0] for c in cases], [c[1] for c in cases])
    result = ffa.align(es, ts, blank_id=[c[2] for c in cases], mode=mode)
    assert result.status.tolist() == [0] * len(cases)
    assert_same_bits(result.labels.cpu().numpy(), np.concatenate([c[3] for c in cases]), "labels")
    assert_same_bits(result.scores.cpu().numpy(), np.concatenate([c[4] for c in cases]), "scores")


@pytest.mark.parametrize("index, scale", [(0, 1.0), (1, 1.0), (3, 1.0), (4, 1.0)])
def test_conventional_configs_match_oracle(cuda, index, scale):
    wl, ref = config(index, scale)
    es, ts = cuda_records(*wl.records())
    result = ffa.align(es, ts, blank_id=wl.blank, mode="conventional")
    assert (ref.status == 0).all()
    assert_matches_oracle(result, ref, f"cfg{index}")


# Records on which the optimized mode's path differs from the conventional
# DP's, by exact class (tests/helpers.classify_divergence), per route and
# config: the window route is exact everywhere (its certificate proves the
# conventional path); the chunked route may return another path only where
# the conventional DP met an fp32 tie.  Any "worse" record fails; the counts
# are pinned, so a new divergence of any class fails too.
EXPECTED_DIVERGENCES = {
    ("window", 0): {}, ("window", 1): {}, ("window", 4): {},
    ("pieces", 0): {}, ("pieces", 1): {}, ("pieces", 3): {}, ("pieces", 4): {"equal_fp32": 4},
    ("auto", 0): {}, ("auto", 1): {}, ("auto", 3): {}, ("auto", 4): {},
}


@pytest.mark.parametrize("route", ["auto", "window", "pieces"])
@pytest.mark.parametrize("index", [0, 1, 3, 4])
def test_optimized_divergences_are_proven_ties(cuda, route, index):
    if route == "window" and index == 3:
        pytest.skip("V = 1025 rows are not row-staged: the window route does not take them")
    wl, ref = config(index)
    es_h, ts_h = wl.records()
    es, ts = cuda_records(es_h, ts_h)
    result = ffa.align(es, ts, blank_id=wl.blank, mode="optimized", route=route)
    assert_same_bits(result.status.cpu().numpy(), ref.status, "status")
    labels = result.labels.cpu().numpy()
    scores = result.scores.cpu().numpy()
    objective = result.objective.cpu().numpy()
    off = wl.frame_offsets
    classes = {}
    for i in range(wl.batch):
        lo, hi = off[i], off[i + 1]
        p, q = labels[lo:hi], ref.labels[lo:hi]
        if np.array_equal(p, q):
            assert_same_bits(scores[lo:hi], ref.scores[lo:hi], f"record {i} scores")
            assert_same_bits(objective[i:i + 1], ref.objective[i:i + 1], f"record {i} objective")
            continue
        # A different path: legal, its own scores, and an exact class.
        np.testing.assert_array_equal(collapse(p, wl.blank), ts_h[i], f"record {i} transcript")
        selected = es_h[i][np.arange(hi - lo), p]
        assert_same_bits(scores[lo:hi], selected, f"record {i} scores")
        assert sequential_sum(selected) == objective[i], f"record {i} objective"
        cls = classify_divergence(es_h[i], ts_h[i], wl.blank, p, q)
        classes.setdefault(cls, []).append(i)
    counts = {k: len(v) for k, v in sorted(classes.items())}
    tie_records = set(wl.tie_frames)
    print(f"cfg{index} {route}: differing records by class {counts}; constructed ties among them: "
          f"{sorted(set(sum(classes.values(), [])) & tie_records)[:10]}; others {dict((k, v[:8]) for k, v in classes.items())}")
    assert "worse" not in classes, f"genuine divergences: {classes['worse'][:10]}"
    assert counts == EXPECTED_DIVERGENCES[(route, index)]


@pytest.mark.parametrize("mode", MODES)
def test_packed_form_equals_list_form(cuda, mode):
    wl, ref = config(1)
    e = torch.from_numpy(wl.emissions).cuda()
    t = torch.from_numpy(wl.targets).cuda()
    packed = ffa.align_packed(e, wl.lengths.tolist(), t, wl.target_lengths.tolist(),
                              blank_id=wl.blank, mode=mode)
    assert_matches_oracle(packed, ref, "packed cfg1")
    # Counts as NumPy arrays, as tensors, and per-record blanks as an array.
    arrays = ffa.align_packed(e, wl.lengths, t, torch.from_numpy(wl.target_lengths),
                              blank_id=np.full(wl.batch, wl.blank), mode=mode)
    assert_matches_oracle(arrays, ref, "packed cfg1 from arrays")
    assert arrays.lengths == packed.lengths


def test_tie_records_are_exact_in_conventional_mode(cuda):
    wl, ref = config(4)
    ties = sorted(wl.tie_frames)
    sub = wl.subset(ties)
    es, ts = cuda_records(*sub.records())
    result = ffa.align(es, ts, blank_id=0, mode="conventional")
    assert_matches_oracle(result, oracle.align(*sub.records(), 0), "cfg4 ties")


def test_full_size_properties_cfg4(cuda):
    # Size-independent properties at cfg4's full size: the path
    # collapses to the transcript, scores are the selected emissions and the
    # objective is the sequential fp32 sum along the path.
    wl, _ = config(4)
    es, ts = cuda_records(*wl.records())
    result = ffa.align(es, ts, blank_id=0, mode="optimized")
    assert (result.status == 0).all()
    labels = result.labels.cpu().numpy()
    scores = result.scores.cpu().numpy()
    objective = result.objective.cpu().numpy()
    rng = np.random.default_rng(0)
    offsets = wl.frame_offsets
    for i in rng.choice(wl.batch, 64, replace=False):
        e, t = wl.record(i)
        p = labels[offsets[i]:offsets[i + 1]]
        np.testing.assert_array_equal(collapse(p, 0), t)
        selected = e[np.arange(len(p)), p]
        assert_same_bits(scores[offsets[i]:offsets[i + 1]], selected, "scores")
        assert sequential_sum(selected) == objective[i]


# ---- the reference's own CUDA extension (compiled in place into oracle/_ref) ----

def reference_or_skip():
    if not oracle.load_reference_cuda():
        pytest.skip("reference CUDA extension not built under oracle/_ref")


@pytest.mark.parametrize("index, scale", [(0, 1.0), (1, 1.0), (3, 1.0), (4, 0.25)])
def test_matches_reference_cuda_conventional(cuda, index, scale):
    reference_or_skip()
    wl, _ = config(index, scale) if scale == 1.0 else (workloads.config(index, scale=scale), None)
    es, ts = cuda_records(*wl.records())
    blanks = [wl.blank] * wl.batch
    tensors, lengths = oracle.reference_cuda_align(es, ts, blanks, mode="conventional")
    keep = np.ones(wl.batch, bool)
    keep[list(wl.tie_frames)] = False  # optimized: ties are checked against the oracle above
    offsets = wl.frame_offsets
    frames = np.concatenate([np.arange(offsets[i], offsets[i + 1]) for i in np.flatnonzero(keep)])
    for mode in MODES:
        mine = ffa.align(es, ts, blank_id=wl.blank, mode=mode)
        assert tuple(mine.lengths) == tuple(lengths)
        for name, ref_tensor in zip(("labels", "scores", "status", "objective"), tensors[:4]):
            a, b = getattr(mine, name).cpu().numpy(), ref_tensor.cpu().numpy()
            if mode == "optimized":
                a, b = (a[frames], b[frames]) if name in ("labels", "scores") else (a[keep], b[keep])
            assert_same_bits(a, b, f"cfg{index} {mode} {name}")


def test_optimized_audit_against_reference_cuda(cuda):
    # The reference's own optimized mode and ours, each audited against the
    # conventional DP with the classes of the reference's accuracy audit
    # (benchmarks/accuracy.py:67-105): ours may not be worse anywhere, and
    # must be identical on at least as many records as the reference.
    reference_or_skip()
    for index in (1, 3):
        wl, ref = config(index)
        es_h, ts_h = wl.records()
        es, ts = cuda_records(es_h, ts_h)
        tensors, _ = oracle.reference_cuda_align(es, ts, [wl.blank] * wl.batch, mode="optimized")
        theirs = tensors[0].cpu().numpy()
        mine = ffa.align(es, ts, blank_id=wl.blank, mode="optimized").labels.cpu().numpy()
        off = wl.frame_offsets
        audit = {"ours": {}, "reference": {}}
        for name, labels in (("ours", mine), ("reference", theirs)):
            for i in range(wl.batch):
                lo, hi = off[i], off[i + 1]
                cls = classify_divergence(es_h[i], ts_h[i], wl.blank, labels[lo:hi], ref.labels[lo:hi]) \
                    if labels[lo] >= 0 else "failed"
                audit[name][cls] = audit[name].get(cls, 0) + 1
        print(f"cfg{index} optimized vs conventional: {audit}")
        assert "worse" not in audit["ours"] and "failed" not in audit["ours"]
        assert audit["ours"].get("identical", 0) >= audit["reference"].get("identical", 0)


def test_matches_reference_cuda_on_reference_test_inputs(cuda):
    reference_or_skip()
    rng = np.random.default_rng(32)
    for blank in (0, 5):
        labels = np.array([i for i in range(6) if i != blank])
        values = [rng.integers(-9, 0, (n, 6)).astype(np.float32) for n in (7, 129, 257, 2305)]
        tokens = [rng.choice(labels, n) for n in (0, 11, 44, 120)]
        es, ts = cuda_records(values, tokens)
        tensors, _ = oracle.reference_cuda_align(es, ts, [blank] * 4, mode="conventional")
        mine = ffa.align(es, ts, blank_id=blank, mode="conventional")
        for name, ref_tensor in zip(("labels", "scores", "status", "objective"), tensors[:4]):
            assert_same_bits(getattr(mine, name).cpu().numpy(), ref_tensor.cpu().numpy(), name)


# ---- direct call through the C ABI (include/ffa_b200.h) ----

class Record(ctypes.Structure):
    _fields_ = [("emissions", ctypes.c_void_p), ("targets", ctypes.c_void_p),
                ("frames", ctypes.c_int64), ("vocab", ctypes.c_int32), ("tokens", ctypes.c_int32),
                ("blank", ctypes.c_int32), ("reserved", ctypes.c_int32)]


class Sizes(ctypes.Structure):
    _fields_ = [("staging_bytes", ctypes.c_size_t), ("workspace_bytes", ctypes.c_size_t),
                ("total_frames", ctypes.c_int64)]


class Outputs(ctypes.Structure):
    _fields_ = [(name, ctypes.c_void_p) for name in (
        "labels", "scores", "status", "objective", "stitched", "repair_passes", "repaired_frames",
        "shortcut_stats", "routing_stats", "reuse_stats")]


def test_c_abi_direct_call_matches_oracle(cuda):
    from fast_forced_aligner_b200.build import LIB
    lib = ctypes.CDLL(str(LIB))
    lib.ffa_last_error.restype = ctypes.c_char_p
    wl, ref = config(0)
    es, ts = cuda_records(*wl.records())
    B = wl.batch
    recs = (Record * B)(*[Record(e.data_ptr(), t.data_ptr(), e.shape[0], e.shape[1], t.numel(), 0, 0)
                          for e, t in zip(es, ts)])
    sizes = Sizes()
    assert lib.ffa_align_query(recs, ctypes.c_int64(B), 0, 1, ctypes.byref(sizes)) == 0
    N = sizes.total_frames
    labels = torch.empty(N, dtype=torch.int64, device=cuda)
    scores = torch.empty(N, dtype=torch.float32, device=cuda)
    i32 = [torch.empty(B, dtype=torch.int32, device=cuda) for _ in range(3)]
    objective = torch.empty(B, dtype=torch.float32, device=cuda)
    repaired = torch.empty(B, dtype=torch.int64, device=cuda)
    shortcut = torch.empty(B, 3, dtype=torch.int64, device=cuda)
    routing = torch.empty(B, 3, dtype=torch.int32, device=cuda)
    out = Outputs(labels.data_ptr(), scores.data_ptr(), i32[0].data_ptr(), objective.data_ptr(),
                  i32[1].data_ptr(), i32[2].data_ptr(), repaired.data_ptr(), shortcut.data_ptr(),
                  routing.data_ptr(), None)
    staging = torch.empty(sizes.staging_bytes, dtype=torch.uint8, pin_memory=True)
    workspace = torch.empty(sizes.workspace_bytes, dtype=torch.uint8, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.ffa_align(recs, ctypes.c_int64(B), 0, 1, None, ctypes.byref(out),
                       ctypes.c_void_p(staging.data_ptr()), ctypes.c_size_t(sizes.staging_bytes),
                       ctypes.c_void_p(workspace.data_ptr()), ctypes.c_size_t(sizes.workspace_bytes),
                       ctypes.c_void_p(stream))
    assert rc == 0, lib.ffa_last_error()
    torch.cuda.synchronize()
    assert_same_bits(labels.cpu().numpy(), ref.labels, "labels")
    assert_same_bits(scores.cpu().numpy(), ref.scores, "scores")
    assert_same_bits(i32[0].cpu().numpy(), ref.status, "status")
    assert_same_bits(objective.cpu().numpy(), ref.objective, "objective")
