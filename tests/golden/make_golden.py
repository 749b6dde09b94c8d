"""Generate tests/golden/reference_cpu_cases.npz from the reference itself.

The expected paths come from the reference repository's own CPU comparator
(benchmarks/patches/cpu_corrected.cpp, compiled in place into oracle/_ref by
oracle/build.py), which uses the same tie rule as the reference's GPU
conventional mode (stay > step > skip, terminal S-2 on ties;
cpu_corrected.cpp:104-118 vs alignment.cu:418-424, 497-499).  Its supported
domain is U >= 1 and T >= U + repeats + 2 (cpu_corrected.cpp:145, 158), so
every generated case satisfies that.

Run here (needs the reference tree):  python tests/golden/make_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import build, oracle  # noqa: E402

OUT = Path(__file__).resolve().parent / "reference_cpu_cases.npz"


def cases(rng):
    """Ragged cases: log-softmax and integer-valued emissions, flat ties,
    repeats, several vocabularies and blank positions."""
    out = []
    for index in range(40):
        V = [5, 6, 32, 67][index % 4]
        blank = [0, V - 1, 2, 0][index % 4]
        U = int(rng.integers(1, 25))
        vocab = np.array([c for c in range(V) if c != blank])
        tokens = rng.choice(vocab, U)
        if index % 5 == 0 and U > 2:
            tokens[1] = tokens[0]  # an adjacent repeat
        repeats = int((tokens[1:] == tokens[:-1]).sum())
        T = int(rng.integers(U + repeats + 2, U + repeats + 2 + 3 * U + 40))
        kind = index % 3
        if kind == 0:
            logits = rng.standard_normal((T, V)).astype(np.float32) * 2
            e = (logits - np.log(np.exp(logits).sum(1, keepdims=True))).astype(np.float32)
        elif kind == 1:
            e = rng.integers(-9, 1, (T, V)).astype(np.float32)
        else:
            e = np.zeros((T, V), np.float32)  # every legal path ties
            e[:, rng.integers(V)] = -1.0
        out.append((e, tokens.astype(np.int64), blank))
    return out


def main() -> None:
    build.build_corrected()
    module = oracle.corrected_module()
    if module is None:
        raise SystemExit("reference comparator unavailable (needs the reference tree)")
    rng = np.random.default_rng(20261201)
    es, ts, blanks, paths, scores = [], [], [], [], []
    for e, t, blank in cases(rng):
        p, s = module.forced_align(e[None], t[None], blank)
        es.append(e); ts.append(t); blanks.append(blank)
        paths.append(np.asarray(p[0], np.int64)); scores.append(np.asarray(s, np.float32))
    np.savez_compressed(
        OUT,
        vocab=np.array([e.shape[1] for e in es], np.int64),
        frames=np.array([e.shape[0] for e in es], np.int64),
        emissions=np.concatenate([e.ravel() for e in es]),
        tokens=np.array([t.size for t in ts], np.int64),
        targets=np.concatenate(ts),
        blanks=np.array(blanks, np.int64),
        paths=np.concatenate(paths),
        scores=np.concatenate(scores),
    )
    print(f"wrote {OUT} ({len(es)} cases, {sum(e.shape[0] for e in es)} frames)")


def load(path: Path = OUT):
    """Unpack the fixture into per-case (emissions, targets, blank, path, scores)."""
    z = np.load(path)
    result, eo, to, fo = [], 0, 0, 0
    for V, T, U, blank in zip(z["vocab"], z["frames"], z["tokens"], z["blanks"]):
        e = z["emissions"][eo:eo + T * V].reshape(T, V)
        result.append((e, z["targets"][to:to + U], int(blank), z["paths"][fo:fo + T],
                       z["scores"][fo:fo + T]))
        eo += T * V; to += U; fo += T
    return result


if __name__ == "__main__":
    main()
