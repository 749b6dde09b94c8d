"""Seeded synthetic CTC alignment workloads with the benchmark configurations' shapes.

The reference measures on a speech-emission suite that is not shipped; these
generators stand in for it with the shapes, lengths and value distributions
the five configs state:

  cfg0  B=16,   T~U[200,1000],  V=32,   blank 0,    U=T//6,    boost +6
  cfg1  B=64,   T~U[250,1750],  V=32,   blank 0,    U=0.3T,    boost +4,
        +2 on blank for 40% of frames
  cfg2  B=8,    T=90000,        V=32,   blank 0,    U=27000,   boost +4,
        lowered to +2.5 on 15% of frames
  cfg3  B=256,  T~U[100,1000],  V=1025, blank 1024, U=T//4,    boost +5,
        Zipf(1.1) tokens over 0..1023, 5% repeats
  cfg4  8192 lognormal(ln 600, 0.6) lengths clipped to [50, 6000] from the
        cfg1 generator, plus 64 constructed exact-tie records

Every record draws a ground-truth token sequence (10% adjacent repeats unless
stated), gives each token >= 1 frame and each repeated pair >= 1 separating
blank, spreads the spare frames multinomially over the 2U+1 CTC slots, adds the
boost to N(0,1) fp32 logits on the true label and applies log_softmax in fp32.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

SEED_BASE = 20261201


@dataclass
class Workload:
    name: str
    vocab: int
    blank: int
    lengths: np.ndarray          # int64 [B] frames per record
    emissions: np.ndarray        # float32 [sum T, V] packed rows
    target_lengths: np.ndarray   # int64 [B]
    targets: np.ndarray          # int64 [sum U] packed tokens
    tie_frames: dict[int, int] = field(default_factory=dict)  # record -> frame

    @property
    def batch(self) -> int:
        return int(self.lengths.size)

    @property
    def frame_offsets(self) -> np.ndarray:
        return np.concatenate([[0], np.cumsum(self.lengths)]).astype(np.int64)

    @property
    def target_offsets(self) -> np.ndarray:
        return np.concatenate([[0], np.cumsum(self.target_lengths)]).astype(np.int64)

    def record(self, i: int) -> tuple[np.ndarray, np.ndarray]:
        f, t = self.frame_offsets, self.target_offsets
        return self.emissions[f[i]:f[i + 1]], self.targets[t[i]:t[i + 1]]

    def records(self) -> tuple[list[np.ndarray], list[np.ndarray]]:
        pairs = [self.record(i) for i in range(self.batch)]
        return [p[0] for p in pairs], [p[1] for p in pairs]

    def subset(self, indices) -> "Workload":
        es, ts = zip(*(self.record(int(i)) for i in indices))
        ties = {k: self.tie_frames[int(i)] for k, i in enumerate(indices) if int(i) in self.tie_frames}
        return Workload(self.name, self.vocab, self.blank,
                        np.array([e.shape[0] for e in es], np.int64), np.concatenate(es),
                        np.array([t.size for t in ts], np.int64),
                        np.concatenate(ts) if ts else np.zeros(0, np.int64), ties)

    def cells(self) -> int:
        return int((self.lengths * (2 * self.target_lengths + 1)).sum())


def _tokens(rng, count, choices, repeat_rate, zipf=None):
    """Token sequence with the given adjacent-repeat rate; a non-repeat
    position never equals its predecessor."""
    if count == 0:
        return np.zeros(0, np.int64)

    def draw(n):
        if zipf is None:
            return rng.choice(choices, n)
        return np.minimum(rng.zipf(zipf, n) - 1, choices.size - 1).astype(np.int64)

    repeat = rng.random(count) < repeat_rate
    repeat[0] = False
    base = draw(count)
    positions = np.arange(count)
    while True:
        source = np.maximum.accumulate(np.where(repeat, 0, positions))
        tokens = base[source]
        clash = np.flatnonzero(~repeat[1:] & (tokens[1:] == tokens[:-1])) + 1
        if clash.size == 0:
            return tokens.astype(np.int64)
        base[clash] = draw(clash.size)


def _frame_labels(rng, T, tokens, blank):
    """Per-frame true labels: >= 1 frame per token, >= 1 blank between equal
    neighbours, spare frames spread multinomially over the 2U+1 slots."""
    U = tokens.size
    slots = np.full(2 * U + 1, blank, np.int64)
    slots[1::2] = tokens
    minimum = np.zeros(2 * U + 1, np.int64)
    minimum[1::2] = 1
    if U > 1:
        minimum[2:-1:2] = (tokens[1:] == tokens[:-1]).astype(np.int64)
    spare = T - int(minimum.sum())
    if spare < 0:
        raise ValueError("record too short for its transcript")
    durations = minimum + rng.multinomial(spare, np.full(2 * U + 1, 1.0 / (2 * U + 1)))
    return np.repeat(slots, durations), slots, durations


def _log_softmax(x: np.ndarray) -> np.ndarray:
    x = x - x.max(axis=1, keepdims=True)
    return (x - np.log(np.exp(x).sum(axis=1, keepdims=True, dtype=np.float32))).astype(np.float32)


def _emissions(rng, frame_labels, vocab, blank, boost, blank_prior=0.0, blank_frac=0.0,
               low_boost=None, low_frac=0.0, tie=False):
    T = frame_labels.size
    logits = rng.standard_normal((T, vocab), dtype=np.float32)
    gain = np.full(T, boost, np.float32)
    if low_boost is not None:
        gain[rng.random(T) < low_frac] = low_boost
    logits[np.arange(T), frame_labels] += gain
    if blank_prior:
        logits[rng.random(T) < blank_frac, blank] += np.float32(blank_prior)
    tie_frame = None
    if tie:
        # Last frame of a token lasting >= 2 frames and followed by blank:
        # copy its logit into the blank column, so moving that boundary one
        # frame earlier gives an exactly equal fp32 path sum.
        nxt = np.r_[frame_labels[1:], -1]
        prv = np.r_[-1, frame_labels[:-1]]
        ok = np.flatnonzero((frame_labels != blank) & (nxt == blank) & (prv == frame_labels))
        if ok.size:
            tie_frame = int(ok[rng.integers(ok.size)])
            logits[tie_frame, blank] = logits[tie_frame, frame_labels[tie_frame]]
    return _log_softmax(logits), tie_frame


def _build(name, vocab, blank, specs, rng, choices, repeat_rate, zipf=None, **emit):
    lengths, tlens, es, ts, ties = [], [], [], [], {}
    for index, (T, U, tie) in enumerate(specs):
        tokens = _tokens(rng, U, choices, repeat_rate, zipf)
        labels, _, _ = _frame_labels(rng, T, tokens, blank)
        e, tf = _emissions(rng, labels, vocab, blank, tie=tie, **emit)
        if tf is not None:
            ties[index] = tf
        lengths.append(T); tlens.append(U); es.append(e); ts.append(tokens)
    return Workload(name, vocab, blank, np.array(lengths, np.int64), np.concatenate(es),
                    np.array(tlens, np.int64), np.concatenate(ts) if ts else np.zeros(0, np.int64),
                    ties)


def config(index: int, *, scale: float = 1.0, shard: int = 0) -> Workload:
    """Generate configs[index]; ``scale`` < 1 shrinks the record count (and
    cfg2's frame count) for parity tests that must finish on the CPU oracle.
    ``shard`` > 0 draws an independent batch of the same shape (one per rank
    in multi-GPU runs)."""
    rng = np.random.default_rng([SEED_BASE + index, shard] if shard else SEED_BASE + index)
    v32 = np.arange(1, 32, dtype=np.int64)
    if index == 0:
        B = max(1, round(16 * scale))
        Ts = rng.integers(200, 1001, B)
        return _build("cfg0", 32, 0, [(int(T), int(T) // 6, False) for T in Ts], rng, v32, 0.10,
                      boost=6.0)
    if index == 1:
        B = max(1, round(64 * scale))
        Ts = rng.integers(250, 1751, B)
        return _build("cfg1", 32, 0, [(int(T), int(0.3 * T), False) for T in Ts], rng, v32, 0.10,
                      boost=4.0, blank_prior=2.0, blank_frac=0.4)
    if index == 2:
        B = max(1, round(8 * min(1.0, scale * 8)))
        T = max(600, round(90000 * min(1.0, scale)))
        return _build("cfg2", 32, 0, [(T, int(0.3 * T), False)] * B, rng, v32, 0.10,
                      boost=4.0, blank_prior=2.0, blank_frac=0.4, low_boost=2.5, low_frac=0.15)
    if index == 3:
        B = max(1, round(256 * scale))
        Ts = rng.integers(100, 1001, B)
        return _build("cfg3", 1025, 1024, [(int(T), int(T) // 4, False) for T in Ts], rng,
                      np.arange(1024, dtype=np.int64), 0.05, zipf=1.1, boost=5.0)
    if index == 4:
        B = max(1, round(8192 * scale))
        ties = max(1, round(64 * scale))
        Ts = np.clip(np.round(rng.lognormal(np.log(600.0), 0.6, B + ties)), 50, 6000).astype(int)
        specs = [(int(T), int(0.3 * T), k >= B) for k, T in enumerate(Ts)]
        return _build("cfg4", 32, 0, specs, rng, v32, 0.10,
                      boost=4.0, blank_prior=2.0, blank_frac=0.4)
    raise ValueError(f"unknown config {index}")
