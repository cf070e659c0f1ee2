"""Sampling after the lm_head on the device (``q3_sample_logits``) against the
reference's Sampler: the golden picks of the reference's own
``Sampler.sample`` (``tests/golden/sample_golden.npz``) and, at the full
151936 vocabulary, the oracle restatement on seeded rows, including rows full
of equal values (ties ordered by index) and extreme top-k / top-p settings."""

from __future__ import annotations

import numpy as np
import pytest

from test_sampling_cpu import golden_cases

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from oracle import sampler  # noqa: E402

VOCAB = 151936


def _run(q3, rows, params, gens):
    from q3b200.ops import sample_logits
    lg = torch.from_numpy(np.stack(rows).astype(np.float32)).cuda()
    out = sample_logits(lg, params, gens)
    torch.cuda.synchronize()
    assert q3._lib.lib().q3_device_status() == 0
    return out.cpu().tolist()


def test_device_sampler_matches_reference_picks(q3):
    rows, params, gens, want = [], [], [], []
    for row, (t, k, p, rp), gen, u, pick in golden_cases():
        rows.append(row)
        params.append(dict(temperature=t, top_k=k, top_p=p, repetition_penalty=rp, u=u))
        gens.append(gen)
        want.append(pick)
    assert _run(q3, rows, params, gens) == want


def _full_vocab_cases():
    rng = np.random.default_rng(31)
    cases = []
    settings = [dict(temperature=1.0), dict(temperature=0.7, top_k=50),
                dict(temperature=1.0, top_p=0.9), dict(temperature=0.8, top_k=1000, top_p=0.95),
                dict(temperature=1.2, top_p=0.5, repetition_penalty=1.3),
                dict(temperature=0.6, top_k=VOCAB - 1, top_p=0.999),
                dict(temperature=1.0, top_k=1), dict(temperature=2.0, top_p=1e-9),
                dict(temperature=0.0), dict(temperature=1.0, top_p=0.3, top_k=20,
                                            repetition_penalty=2.0)]
    for i, s in enumerate(settings * 2):
        scale = [0.5, 2.0, 8.0][i % 3]
        row = (rng.standard_normal(VOCAB) * scale).astype(np.float32)
        if i >= len(settings):            # many exact ties, some at the top
            row = (np.round(row * 2.0) / 2.0).astype(np.float32)
        gen = [int(v) for v in rng.integers(0, VOCAB, 12)]
        row[gen[:4]] = np.abs(row[gen[:4]]) + 3.0       # penalised high logits
        cases.append((row, dict(s, u=float(rng.random())), gen))
    return cases


def test_device_sampler_full_vocab_matches_oracle(q3):
    cases = _full_vocab_cases()
    got = _run(q3, [c[0] for c in cases], [c[1] for c in cases], [c[2] for c in cases])
    want = [sampler.sample(row, p["temperature"], p.get("top_k", 0), p.get("top_p", 1.0),
                           p.get("repetition_penalty", 1.0), gen, p["u"]) for row, p, gen in cases]
    assert got == want


def test_device_sampler_draw_sweep(q3):
    """One row, many draws: every u in a sweep picks the oracle's index (the
    cumulative-sum walk of Generator.choice)."""
    rng = np.random.default_rng(8)
    row = (rng.standard_normal(VOCAB) * 1.5).astype(np.float32)
    us = list(np.linspace(0.0, 1.0, 64, endpoint=False)) + list(rng.random(64))
    params = [dict(temperature=0.9, top_p=0.97, u=float(u)) for u in us]
    got = _run(q3, [row] * len(us), params, [[]] * len(us))
    want = [sampler.sample(row, 0.9, 0, 0.97, 1.0, (), float(u)) for u in us]
    assert got == want
