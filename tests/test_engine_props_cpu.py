"""The native engine against a restatement of the reference's engine
(``oracle/engine_ref.py``, tools/engine.py:81-243) on the CPU: the
restatement first reproduces the batches recorded from the reference itself
(``tests/golden/engine_trace.json``); then, on random request mixes (page
pressure, small row budgets, stop tokens, greedy and sampled requests), the
native engine must build the same batch at every step and produce the same
ids, finished flags and free pages."""

from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import GOLDEN

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402

from oracle.engine_ref import EngineRef  # noqa: E402

TRACE = json.loads((GOLDEN / "engine_trace.json").read_text())


def _guest_fn(vocab, table):
    def logits_for(rid, n_generated, rows):
        j = rid * 7 + n_generated + rows
        if table is not None:
            return table[j % 64]
        x = np.full(vocab, -100.0, np.float32)
        x[j % vocab] = 100.0
        return x
    return logits_for


def _table(sc):
    if sc.get("guest") != "table":
        return None
    return (np.random.default_rng(77).standard_normal((64, sc["vocab"])) * 2.0).astype(np.float32)


def _params(r):
    return dict(max_new=r["max_new"], temperature=r.get("temperature", 0.0), top_k=r.get("top_k", 0),
                top_p=r.get("top_p", 1.0), repetition_penalty=r.get("repetition_penalty", 1.0),
                seed=r.get("seed", 0), stop=set(r["stop"]))


def run_oracle(sc):
    f = _guest_fn(sc["vocab"], _table(sc))
    eng = EngineRef(None, sc["num_pages"], sc["max_rows"])
    eng.guest = lambda items: {it[0].rid: f(it[0].rid, len(it[0].generated), it[2])
                               for it in items if it[6]}
    rids = [eng.add(r["prompt"], **_params(r)) for r in sc["requests"]]
    steps = eng.run()
    return {"steps": steps, "outputs": [eng.reqs[i].generated for i in rids],
            "finished": [int(eng.reqs[i].done) for i in rids], "free_pages": len(eng.free),
            "n_steps": eng.steps}


def run_native(q3, sc):
    from q3b200._lib import Layout
    from q3b200.engine import Engine, SamplingParams
    f = _guest_fn(sc["vocab"], _table(sc))
    generated = {}

    def guest(items):
        out = {}
        for it in items:
            if it.needs_logits:
                n = generated.get(it.rid, 0)
                out[it.rid] = f(it.rid, n, it.rows)
                generated[it.rid] = n + 1
        return out
    L = Layout()
    L.hidden, L.layers, L.heads, L.kv_heads, L.head_dim = 1024, 1, 16, 8, 128
    L.inter, L.vocab, L.seq, L.max_seq = 3072, sc["vocab"], 32, 256
    eng = Engine(None, num_pages=sc["num_pages"], max_rows=sc["max_rows"], guest=guest, layout=L)
    rids = [eng.add_request(r["prompt"], SamplingParams(
        max_new=r["max_new"], temperature=r.get("temperature", 0.0), top_k=r.get("top_k", 0),
        top_p=r.get("top_p", 1.0), repetition_penalty=r.get("repetition_penalty", 1.0),
        seed=r.get("seed", 0), stop_tokens=set(r["stop"]))) for r in sc["requests"]]
    steps = []
    while eng.step():
        steps.append([[it.rid, it.row_start, it.rows, it.pos, it.token_ids, int(it.prefill),
                       int(it.needs_logits)] for it in eng.last_batch()])
        assert len(steps) <= 2000
    out = {"steps": steps, "outputs": [eng.result(r)[0] for r in rids],
           "finished": [int(eng.result(r)[1]) for r in rids], "free_pages": eng.free_pages,
           "n_steps": eng.steps}
    eng.close()
    return out


@pytest.mark.parametrize("k", range(len(TRACE)))
def test_oracle_engine_matches_reference_trace(k):
    sc = TRACE[k]
    got = run_oracle(sc)
    for key in ("steps", "outputs", "finished", "free_pages", "n_steps"):
        assert got[key] == sc[key], key


_request = st.fixed_dictionaries({
    "prompt": st.lists(st.integers(0, 199), min_size=1, max_size=80),
    "max_new": st.integers(1, 8),
    "stop": st.lists(st.integers(0, 199), max_size=3),
    "temperature": st.sampled_from([0.0, 0.0, 0.6, 1.0, 1.7]),
    "top_k": st.sampled_from([0, 0, 1, 5, 50]),
    "top_p": st.sampled_from([1.0, 1.0, 0.9, 0.5]),
    "repetition_penalty": st.sampled_from([1.0, 1.0, 1.3]),
    "seed": st.integers(0, 2 ** 40),
})


@settings(max_examples=150, deadline=None)
@given(st.integers(1, 12), st.integers(1, 40), st.lists(_request, min_size=1, max_size=6),
       st.sampled_from([None, "table"]))
def test_native_engine_matches_oracle_on_random_mixes(q3, num_pages, max_rows, requests, guest):
    sc = {"num_pages": num_pages, "max_rows": max_rows, "vocab": 200, "requests": requests}
    if guest:
        sc["guest"] = guest
    assert run_native(q3, sc) == run_oracle(sc)
