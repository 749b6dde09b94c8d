"""Logits inputs (fp32 and bf16) aligned as their log_softmax without writing
it out.  The row log-sum-exp is checked against an fp64 restatement and the
materialised log_softmax against torch.log_softmax, within tolerances
derived below.  Every alignment output of the fused path must equal,
bit for bit, the same call on the materialised log-probabilities
(``ffa.log_softmax``), which the CPU oracle pins in the conventional mode.
Row-staged and gathered kernels, odd bf16 addresses, long records on
clusters and both modes are covered."""
import numpy as np
import pytest
import torch

import fast_forced_aligner_b200 as ffa
from oracle import oracle
from tests.helpers import assert_matches_oracle, assert_same_bits

pytestmark = pytest.mark.gpu

DTYPES = {"f32": torch.float32, "bf16": torch.bfloat16}


def lse64(x: np.ndarray) -> np.ndarray:
    """Row log-sum-exp in fp64 (the checker's restatement)."""
    m = x.max(axis=1, keepdims=True)
    return (m + np.log(np.exp(x - m).sum(axis=1, keepdims=True)))[:, 0]


def lse_tolerance(V: int, z: np.ndarray) -> np.ndarray:
    """Bound on |z - lse64| for the kernel's fp32 arithmetic.  In log space:
    each of the ceil(V/32) + 5 additions of terms in (0, 1] contributes at
    most 2^-24 (6e-8); the rounded arguments x - m and __expf's error a few
    times that (the terms' weighted mean of 2^-24 |x - m|, and the
    intrinsic's few 1e-7 relative on each term); logf two ulps of
    log(s) < log(V) + 1; the final m + log(s) half an ulp of |z|.  Any
    algorithmic slip (a lost column, a wrong maximum) is orders of magnitude
    above this."""
    adds = -(-V // 32) + 5
    log_ulp = float(np.spacing(np.float32(np.log(V) + 1.0)))
    return 1e-7 * (adds + 16) + 2 * log_ulp + 2 * np.spacing(np.abs(z).astype(np.float32)).astype(np.float64)


def to_device(x: np.ndarray, dtype) -> torch.Tensor:
    return torch.from_numpy(x).to("cuda").to(dtype).contiguous()


def exact_values(t: torch.Tensor) -> np.ndarray:
    """The stored logits as fp64 (bf16 widens exactly)."""
    return t.float().cpu().numpy().astype(np.float64)


def logits_batch(seed, count, vocabs, lengths=(1, 2, 31, 32, 33, 64, 65, 96, 97), max_frames=1500):
    rng = np.random.default_rng(seed)
    logits, targets, blanks = [], [], []
    for _ in range(count):
        V = int(rng.choice(vocabs))
        blank = int(rng.integers(0, V))
        T = int(rng.choice(lengths)) if rng.random() < 0.3 else int(rng.integers(1, max_frames))
        U = int(rng.integers(0, max(1, min(T, 1500)) // 2 + 1)) if V > 1 else 0
        choices = np.array([c for c in range(V) if c != blank])
        tokens = rng.choice(choices, U).astype(np.int64) if U else np.zeros(0, np.int64)
        x = (rng.standard_normal((T, V)) * rng.uniform(0.5, 4.0) + rng.uniform(-20, 20)).astype(np.float32)
        if U:  # a monotone labelling the model is confident about, as real logits have
            idx = np.sort(rng.choice(T, min(T, U), replace=False)) if U <= T else np.arange(T)
            x[idx, tokens[:idx.size]] += rng.uniform(2.0, 8.0)
        logits.append(x)
        targets.append(tokens)
        blanks.append(blank)
    return logits, targets, blanks


def batch_fields(b):
    return {
        "labels": b.labels, "scores": b.scores, "status": b.status, "objective": b.objective,
        "stitched": b.stitched, "repair_passes": b.repair_passes, "repaired_frames": b.repaired_frames,
        "routing_stats": b.routing_stats, "reuse_stats": b.reuse_stats, "shortcut_stats": b.shortcut_stats,
    }


def assert_same_batch(a, b, what):
    assert tuple(a.lengths) == tuple(b.lengths)
    fa, fb = batch_fields(a), batch_fields(b)
    for name in fa:
        assert_same_bits(fa[name].cpu().numpy(), fb[name].cpu().numpy(), f"{what} {name}")


@pytest.mark.parametrize("dtype", list(DTYPES))
@pytest.mark.parametrize("V", [1, 2, 5, 32, 33, 64, 1025, 4097])
def test_row_logsumexp_accuracy(cuda, dtype, V):
    rng = np.random.default_rng(V)
    x = to_device((rng.standard_normal((300, V)) * 6 + rng.uniform(-30, 30, (300, 1))).astype(np.float32),
                  DTYPES[dtype])
    z = ffa.row_logsumexp(x).cpu().numpy().astype(np.float64)
    ref = lse64(exact_values(x))
    err = np.abs(z - ref)
    assert (err <= lse_tolerance(V, ref)).all(), f"max error {err.max()} at V={V}"
    if V == 1:
        assert_same_bits(z.astype(np.float32), exact_values(x)[:, 0].astype(np.float32), "V = 1")


@pytest.mark.parametrize("dtype", list(DTYPES))
def test_row_logsumexp_same_in_every_variant(cuda, dtype):
    # The kernel variant follows the call's widest row (register-resident rows
    # for V <= 32 and V <= 64, streaming otherwise); a row's z must not depend
    # on it, nor on the row's position in the batch.
    rng = np.random.default_rng(3)
    xs = [to_device((rng.standard_normal((37, V)) * 5).astype(np.float32), DTYPES[dtype])
          for V in (5, 32, 60, 100, 1000, 3000)]
    alone = torch.cat([ffa.row_logsumexp(x) for x in xs]).cpu().numpy()
    for k in range(2, len(xs) + 1):
        together = ffa.row_logsumexp(xs[:k]).cpu().numpy()
        assert_same_bits(together, alone[:together.size], f"first {k} tensors")
    shuffled = ffa.row_logsumexp(xs[::-1]).cpu().numpy()
    sizes = [x.shape[0] for x in xs]
    parts = np.split(alone, np.cumsum(sizes)[:-1])
    assert_same_bits(shuffled, np.concatenate(parts[::-1]), "reversed order")


@pytest.mark.parametrize("dtype", list(DTYPES))
@pytest.mark.parametrize("V", [65, 100, 1025, 2049])
def test_row_logsumexp_independent_of_address(cuda, dtype, V):
    # The same rows copied to every element offset within a 16-byte block
    # must give the same z bit for bit (and each within the fp64 bound): the
    # summation order is a function of V, not of where a row lies.
    rng = np.random.default_rng(V)
    x = to_device((rng.standard_normal((40, V)) * 4).astype(np.float32), DTYPES[dtype])
    per_block = 16 // x.element_size()
    results = []
    for shift in range(per_block):
        buf = torch.empty(x.numel() + per_block, dtype=x.dtype, device="cuda")
        view = buf[shift:shift + x.numel()].view(x.shape)
        view.copy_(x)
        results.append(ffa.row_logsumexp(view).cpu().numpy())
    for shift, z in enumerate(results[1:], 1):
        assert_same_bits(z, results[0], f"element offset {shift}")
    ref = lse64(exact_values(x))
    assert (np.abs(results[0] - ref) <= lse_tolerance(V, ref)).all()


@pytest.mark.parametrize("dtype", list(DTYPES))
def test_row_logsumexp_special_rows(cuda, dtype):
    x = np.zeros((6, 40), np.float32)
    x[0, 3] = np.nan
    x[1, 7] = np.inf
    x[2, :] = -np.inf
    x[3, :5] = -np.inf           # some -inf entries: finite
    x[4, :] = 80.0               # large equal logits: z = 80 + log(40)
    x[5, 0] = -np.inf
    x[5, 1:] = np.arange(39, dtype=np.float32)
    z = ffa.row_logsumexp(to_device(x, DTYPES[dtype])).cpu().numpy()
    assert np.isnan(z[:3]).all()
    ref = lse64(x[3:].astype(np.float64))
    assert (np.abs(z[3:] - ref) <= lse_tolerance(40, ref)).all(), (z[3:], ref)


@pytest.mark.parametrize("dtype", list(DTYPES))
def test_log_softmax_matches_torch(cuda, dtype):
    logits, _, _ = logits_batch(7, 12, [32, 33, 1025])
    xs = [to_device(x, DTYPES[dtype]) for x in logits]
    mine = ffa.log_softmax(xs)
    for x, e in zip(xs, mine):
        assert e.dtype == torch.float32 and e.shape == x.shape
        ref = torch.log_softmax(x.double(), dim=-1)
        # x - z rounds once more than z: |error| <= tol(z) + half an ulp of |e|.
        z = lse64(exact_values(x))
        tol = lse_tolerance(x.shape[1], z)[:, None] + np.spacing(np.abs(e.cpu().numpy()))
        assert (np.abs(e.double().cpu().numpy() - ref.cpu().numpy()) <= tol).all()
        torch.testing.assert_close(e, torch.log_softmax(x.float(), dim=-1), rtol=0, atol=2e-5)
    single = ffa.log_softmax(xs[0])
    assert_same_bits(single.cpu().numpy(), mine[0].cpu().numpy(), "single tensor")


@pytest.mark.parametrize("dtype", list(DTYPES))
@pytest.mark.parametrize("mode", ["conventional", "optimized"])
def test_fused_align_matches_materialised_log_softmax(cuda, dtype, mode):
    # Row-staged (V % 4 == 0 fp32, V % 8 == 0 bf16, V <= 64) and gathered
    # vocabularies, random blanks, piece-boundary lengths.
    logits, targets, blanks = logits_batch(11, 160, [2, 3, 8, 12, 32, 36, 40, 64, 129, 1025])
    xs = [to_device(x, DTYPES[dtype]) for x in logits]
    ts = [torch.from_numpy(t).to("cuda") for t in targets]
    fused = ffa.align(xs, ts, blank_id=blanks, mode=mode, from_logits=True)
    emissions = ffa.log_softmax(xs)
    plain = ffa.align(emissions, ts, blank_id=blanks, mode=mode)
    assert_same_batch(fused, plain, f"{dtype} {mode}")
    assert (fused.status.cpu().numpy() == 0).sum() > len(xs) // 3
    if mode == "conventional":
        ref = oracle.align([e.cpu().numpy() for e in emissions], targets, blanks)
        assert_matches_oracle(fused, ref, f"{dtype} conventional vs oracle")


@pytest.mark.parametrize("dtype", list(DTYPES))
@pytest.mark.parametrize("V", [7, 32, 33, 40, 1025])
def test_packed_logits_at_odd_offsets(cuda, dtype, V):
    # One packed [N, V] matrix: with odd V, bf16 records start at odd element
    # offsets (2-byte aligned), which the gathered kernels read as halves of
    # 4-byte words.
    rng = np.random.default_rng(V)
    frames = [int(t) for t in rng.integers(1, 700, 24)] + [65, 33, 97]
    tokens = [int(rng.integers(0, max(1, t // 2) + 1)) for t in frames]
    N = sum(frames)
    x = (rng.standard_normal((N, V)) * 3).astype(np.float32)
    tgt = np.concatenate([rng.integers(1, V, u) for u in tokens]).astype(np.int64)
    xd = to_device(x, DTYPES[dtype])
    td = torch.from_numpy(tgt).to("cuda")
    for mode in ("conventional", "optimized"):
        fused = ffa.align_packed(xd, frames, td, tokens, blank_id=0, mode=mode, from_logits=True)
        plain = ffa.align_packed(ffa.log_softmax(xd), frames, td, tokens, blank_id=0, mode=mode)
        assert_same_batch(fused, plain, f"packed {dtype} V={V} {mode}")


@pytest.mark.parametrize("dtype", list(DTYPES))
@pytest.mark.parametrize("V", [32, 37])
def test_long_record_logits_on_clusters(cuda, dtype, V):
    # 2100 tokens (4201 states): a 2-CTA cluster; V = 32 row-staged, 37 gathered.
    rng = np.random.default_rng(V)
    U, T = 2100, 2600
    tokens = rng.integers(1, V, U).astype(np.int64)
    x = (rng.standard_normal((T, V)) * 2).astype(np.float32)
    x[np.sort(rng.choice(T, U, replace=False)), tokens] += 5.0
    xs = [to_device(x, DTYPES[dtype]), to_device(x[:700], DTYPES[dtype])]
    ts = [torch.from_numpy(tokens).to("cuda"), torch.from_numpy(tokens[:300]).to("cuda")]
    fused = ffa.align(xs, ts, blank_id=0, mode="conventional", from_logits=True)
    emissions = ffa.log_softmax(xs)
    ref = oracle.align([e.cpu().numpy() for e in emissions], [t.cpu().numpy() for t in ts], 0)
    assert_matches_oracle(fused, ref, f"long {dtype} V={V}")
    assert (fused.status.cpu().numpy() == 0).all()
    opt = ffa.align(xs, ts, blank_id=0, mode="optimized", from_logits=True)
    assert_same_batch(opt, ffa.align(emissions, ts, blank_id=0, mode="optimized"), f"long {dtype} optimized")


def test_logits_argument_contract(cuda):
    x = torch.randn(50, 8, device="cuda")
    t = torch.tensor([1, 2, 3], device="cuda")
    with pytest.raises(ValueError, match="bfloat16"):
        ffa.align([x.double()], [t], from_logits=True)
    with pytest.raises(ValueError, match="float32"):
        ffa.align([x.bfloat16()], [t])  # bf16 log-probabilities are not an input format
    with pytest.raises(ValueError):
        ffa.align([x.bfloat16(), x], [t, t], from_logits=True)  # one dtype per call
    ffa.validate_inputs([x.bfloat16()], [t])
    with pytest.raises(ValueError, match="insufficient"):
        ffa.validate_inputs([x[:2].bfloat16()], [t])
    # NaN logits: the row's emissions are NaN, and the record fails as it
    # does with NaN log-probabilities.
    bad = x.clone()
    bad[10, 3] = float("nan")
    fused = ffa.align([bad], [t], from_logits=True, mode="conventional")
    plain = ffa.align(ffa.log_softmax([bad]), [t], mode="conventional")
    assert_same_batch(fused, plain, "NaN logits")
