"""CPU oracle (TEST INFRASTRUCTURE ONLY).

A numpy restatement of the reference's numpy mirror ``tools/ref_qwen3.py``.
Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import it, and only as the checker — the product path never does.
"""

from . import exp2, q3_oracle, synth  # noqa: F401
