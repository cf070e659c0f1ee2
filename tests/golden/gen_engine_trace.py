#!/usr/bin/env python3
"""Record the batches the REFERENCE's host engine (``tools/engine.py`` of
mland2333/qwen3-tile-ops, imported unmodified from a checkout) builds, step by
step, for a few request mixes driven by a deterministic mock guest, into
``engine_trace.json``::

    python tests/golden/gen_engine_trace.py --reference <path to the checkout>

The mock guest is the one of the reference's ``tools/check_engine.py``: for
each item that needs logits, all logits -100 except +100 at
``(rid * 7 + len(generated) + rows) % vocab``.  Scenario 0 is
``check_engine.py``'s own; the others add page pressure (requests wait for
pages), stop tokens and a small row budget.  Scenario 3 samples: its guest
returns row ``(rid * 7 + len(generated) + rows) % 64`` of a seeded float32
table (``table_logits``) and its requests carry temperature / top-k / top-p /
repetition penalty / seed, so the trace records the reference's Sampler picks
from each request's ``default_rng(seed)`` stream.
"""

from __future__ import annotations

import argparse
import importlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

SCENARIOS = [
    {"num_pages": 8, "max_rows": 32, "vocab": 32,
     "requests": [{"prompt": [1, 2, 3, 4, 5], "max_new": 4, "stop": []},
                  {"prompt": list(range(70)), "max_new": 4, "stop": []},
                  {"prompt": list(range(33)), "max_new": 4, "stop": []}]},
    {"num_pages": 5, "max_rows": 16, "vocab": 64,
     "requests": [{"prompt": list(range(40)), "max_new": 5, "stop": []},
                  {"prompt": list(range(3, 23)), "max_new": 6, "stop": [10]},
                  {"prompt": [7] * 9, "max_new": 3, "stop": []},
                  {"prompt": list(range(50, 62)), "max_new": 4, "stop": [24]}]},
    {"num_pages": 32, "max_rows": 6, "vocab": 50,
     "requests": [{"prompt": list(range(1, n + 1)), "max_new": 5, "stop": []} for n in range(1, 6)]
     + [{"prompt": list(range(50)), "max_new": 3, "stop": []}]},
    {"num_pages": 16, "max_rows": 24, "vocab": 300, "guest": "table",
     "requests": [
         {"prompt": list(range(5)), "max_new": 8, "stop": [], "temperature": 0.8, "seed": 1},
         {"prompt": list(range(40)), "max_new": 6, "stop": [], "temperature": 1.2, "top_k": 20,
          "seed": 2},
         {"prompt": list(range(3, 20)), "max_new": 7, "stop": [], "temperature": 0.7,
          "top_p": 0.9, "repetition_penalty": 1.3, "seed": 3},
         {"prompt": [9] * 12, "max_new": 6, "stop": [], "temperature": 1.0, "top_k": 50,
          "top_p": 0.8, "repetition_penalty": 1.1, "seed": 2**40 + 7},
         {"prompt": list(range(30, 36)), "max_new": 5, "stop": [], "temperature": 0.0},
         {"prompt": list(range(1, 9)), "max_new": 9, "stop": [11, 12, 13], "temperature": 1.5,
          "top_p": 0.95, "seed": 5}]},
]


def table_logits(vocab: int) -> np.ndarray:
    return (np.random.default_rng(77).standard_normal((64, vocab)) * 2.0).astype(np.float32)


def run(engine_mod, sc: dict) -> dict:
    vocab = sc["vocab"]

    table = table_logits(vocab) if sc.get("guest") == "table" else None

    def guest(batch):
        out = {}
        for it in batch.items:
            if it.needs_logits:
                j = it.req.rid * 7 + len(it.req.generated) + it.rows
                if table is not None:
                    out[it.req.rid] = table[j % 64]
                    continue
                x = np.full(vocab, -100.0, dtype=np.float64)
                x[j % vocab] = 100.0
                out[it.req.rid] = x
        return out

    eng = engine_mod.Engine(guest, num_pages=sc["num_pages"], max_rows=sc["max_rows"], vocab=vocab)
    reqs = [eng.add_request(r["prompt"], engine_mod.SamplingParams(
        max_new=r["max_new"], temperature=r.get("temperature", 0.0), top_k=r.get("top_k", 0),
        top_p=r.get("top_p", 1.0), repetition_penalty=r.get("repetition_penalty", 1.0),
        seed=r.get("seed", 0), stop_tokens=set(r["stop"])))
        for r in sc["requests"]]
    steps = []
    build = eng.sched.build_batch

    def recording_build():            # the reference's own scheduler, observed
        batch = build()
        if batch.items:
            steps.append([[it.req.rid, it.row_start, it.rows, it.pos,
                           list(map(int, it.token_ids)), int(it.prefill), int(it.needs_logits)]
                          for it in batch.items])
        return batch
    eng.sched.build_batch = recording_build
    eng.run(max_steps=1000)
    return {**sc, "steps": steps, "outputs": [list(map(int, r.generated)) for r in reqs],
            "finished": [int(r.done) for r in reqs], "free_pages": eng.pool.free_pages,
            "n_steps": eng.steps}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    a = ap.parse_args()
    sys.path.insert(0, str(Path(a.reference) / "tools"))
    engine_mod = importlib.import_module("engine")
    trace = [run(engine_mod, sc) for sc in SCENARIOS]
    (HERE / "engine_trace.json").write_text(json.dumps(trace))
    for t in trace:
        print(f"{len(t['steps'])} steps, outputs {t['outputs']}, free pages {t['free_pages']}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
