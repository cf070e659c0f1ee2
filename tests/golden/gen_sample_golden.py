#!/usr/bin/env python3
"""Golden picks of the reference's sampler: ``Sampler.sample`` of
``tools/engine.py`` (mland2333/qwen3-tile-ops, imported unmodified from a
checkout) on seeded float32 logits, three consecutive draws per request so that
the request's ``default_rng(seed)`` stream advances as in the engine::

    python tests/golden/gen_sample_golden.py --reference <path to the checkout>

Writes ``sample_golden.npz``: per-case parameters, generated ids (padded with
-1) and the picked ids; the logits are rebuilt by ``logits_row`` (seeded)."""

from __future__ import annotations

import argparse
import importlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
V = 4096
# (temperature, top_k, top_p, repetition_penalty, seed, logit scale)
CASES = [(0.0, 0, 1.0, 1.0, 0, 3.0), (1.0, 0, 1.0, 1.0, 1, 3.0), (0.7, 0, 1.0, 1.0, 2, 3.0),
         (0.8, 50, 1.0, 1.0, 3, 3.0), (1.0, 0, 0.9, 1.0, 4, 3.0), (0.6, 40, 0.8, 1.0, 5, 3.0),
         (1.3, 0, 0.5, 1.2, 6, 2.0), (0.9, 1, 1.0, 1.0, 7, 3.0), (1.0, 4095, 0.95, 1.1, 8, 1.0),
         (0.5, 0, 0.99, 1.5, 9, 0.5), (2.0, 200, 0.3, 1.05, 2**40 + 3, 4.0),
         (1.0, 0, 1.0, 1.0, 11, 30.0), (0.25, 10, 1.0, 2.0, 12, 1.0), (1.0, 0, 0.999, 1.0, 13, 0.05)]


def logits_row(case: int, draw: int, scale: float, penalised: int) -> np.ndarray:
    row = (np.random.default_rng(10_000 + 10 * case + draw).standard_normal(V) * scale)
    row = row.astype(np.float32)
    row[penalised] = abs(row[penalised]) + np.float32(1.0)   # a penalised positive
    return row


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    a = ap.parse_args()
    sys.path.insert(0, str(Path(a.reference) / "tools"))
    eng = importlib.import_module("engine")
    rng = np.random.default_rng(2024)
    n = len(CASES)
    gen = np.full((n, 8), -1, np.int32)
    picks = np.zeros((n, 3), np.int32)
    for c, (t, k, p, rp, seed, scale) in enumerate(CASES):
        req = eng.Request(c, [1, 2, 3], eng.SamplingParams(max_new=16, temperature=t, top_k=k,
                                                            top_p=p, repetition_penalty=rp,
                                                            seed=seed))
        req.generated = [int(v) for v in rng.integers(0, V, 5)]
        gen[c, :5] = req.generated
        s = eng.Sampler()
        for d in range(3):
            row = logits_row(c, d, scale, req.generated[0])
            picks[c, d] = s.sample(row, req)
            req.generated.append(int(picks[c, d]))
            gen[c, 5 + d] = picks[c, d]
    np.savez_compressed(HERE / "sample_golden.npz", params=np.array(
        [c[:4] + c[5:] for c in CASES], np.float64), seeds=np.array([c[4] for c in CASES], np.uint64),
        generated=gen, picks=picks)
    print(picks.tolist())
    return 0


if __name__ == "__main__":
    sys.exit(main())
