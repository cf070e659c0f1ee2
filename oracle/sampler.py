"""CPU restatement of the reference's sampler (TEST INFRASTRUCTURE ONLY).

``tools/engine.py:118-149`` (``Sampler.sample``) with the uniform draw made
explicit: ``Generator.choice(V, p=probs)`` is ``searchsorted(cumsum(p) /
cumsum(p)[-1], random(), side="right")`` (numpy 2.x), so ``sample(..., u)``
with ``u = default_rng(seed).random()`` is the reference's pick.  The one
change: equal values are ordered by index in the top-p sort
(``argsort(kind="stable")``), where the reference's default ``argsort`` leaves
their order to numpy's introsort.  Pinned by ``tests/golden/sample_golden.npz``
(picks of the reference's own ``Sampler``).
"""

from __future__ import annotations

import numpy as np


def sample(logits, temperature: float, top_k: int = 0, top_p: float = 1.0,
           repetition_penalty: float = 1.0, generated=(), u: float = 0.0) -> int:
    x = np.asarray(logits, dtype=np.float64).copy()
    if temperature <= 0.0:
        return int(np.argmax(x))
    x /= temperature
    if repetition_penalty != 1.0:
        for t in set(int(g) for g in generated):
            if x[t] > 0:
                x[t] /= repetition_penalty
            else:
                x[t] *= repetition_penalty
    if 0 < top_k < x.size:
        kth = np.partition(x, -top_k)[-top_k]
        x[x < kth] = -np.inf
    if top_p < 1.0:
        order = np.argsort(-x, kind="stable")
        sorted_x = x[order]
        probs = np.exp(sorted_x - sorted_x[0])
        probs /= probs.sum()
        cum = np.cumsum(probs)
        keep = cum <= top_p
        keep[0] = True
        x[order[~keep]] = -np.inf
    m = np.max(x)
    probs = np.exp(x - m)
    probs /= probs.sum()
    cdf = probs.cumsum()
    cdf /= cdf[-1]
    return int(cdf.searchsorted(u, side="right"))
