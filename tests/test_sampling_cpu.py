"""The sampler's checker and host pieces, on the CPU: the native random
stream equals numpy's ``default_rng(seed).random()`` (the reference's
Request.rng), and the oracle restatement of ``Sampler.sample`` reproduces the
picks the reference's own Sampler made (``tests/golden/sample_golden.npz``,
``gen_sample_golden.py``)."""

from __future__ import annotations

import ctypes as C
import sys

import numpy as np
import pytest

from conftest import GOLDEN

sys.path.insert(0, str(GOLDEN))
from gen_sample_golden import V, logits_row  # noqa: E402

G = np.load(GOLDEN / "sample_golden.npz")


@pytest.mark.parametrize("seed", [0, 1, 7, 2**32 - 1, 2**32 + 5, 2**40 + 3, 2**63 + 11, 2**64 - 1])
def test_rng_matches_numpy_default_rng(q3, seed):
    out = (C.c_double * 6)()
    assert q3._lib.lib().q3_rng_uniforms(C.c_uint64(seed), 6, out) == 0
    want = np.random.default_rng(seed).random(6)
    assert list(out) == list(want)


def golden_cases():
    """(logits, params, generated, u, pick) for every golden draw."""
    for c in range(len(G["picks"])):
        t, k, p, rp, scale = G["params"][c]
        draws = np.random.default_rng(int(G["seeds"][c])).random(3)
        for d in range(3):
            gen = [int(v) for v in G["generated"][c, :5 + d]]
            row = logits_row(c, d, float(scale), gen[0])
            u = float(draws[d]) if t > 0 else 0.0
            yield row, (float(t), int(k), float(p), float(rp)), gen, u, int(G["picks"][c, d])


def test_oracle_sampler_matches_reference_picks():
    from oracle import sampler
    n = 0
    for row, (t, k, p, rp), gen, u, pick in golden_cases():
        # greedy picks draw nothing; a sampled pick uses the next draw
        assert sampler.sample(row, t, k, p, rp, gen, u) == pick
        n += 1
    assert n == 3 * len(G["picks"]) and V == 4096
