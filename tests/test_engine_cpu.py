"""The native host engine against the reference's own engine (tools/engine.py),
on the CPU: the batch of every step, the generated ids, the finished flags and
the free pages must match the trace ``tests/golden/engine_trace.json`` that
``tests/golden/gen_engine_trace.py`` recorded from the reference with the mock
guest of its ``tools/check_engine.py`` (and, in the sampling scenario, a table
guest: the sampled ids follow the reference's Sampler and random streams)."""

from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import GOLDEN

TRACE = json.loads((GOLDEN / "engine_trace.json").read_text())


def _layout(vocab, max_seq=256):
    from q3b200._lib import Layout
    L = Layout()
    L.hidden, L.layers, L.heads, L.kv_heads, L.head_dim = 1024, 1, 16, 8, 128
    L.inter, L.vocab, L.seq, L.max_seq = 3072, vocab, 32, max_seq
    return L


def _mock_engine(q3, sc):
    from q3b200.engine import Engine
    vocab = sc["vocab"]
    generated = {}
    table = None
    if sc.get("guest") == "table":     # gen_engine_trace.table_logits
        table = (np.random.default_rng(77).standard_normal((64, vocab)) * 2.0).astype(np.float32)

    def guest(items):        # tools/check_engine.py mock_guest
        out = {}
        for it in items:
            if it.needs_logits:
                n = generated.get(it.rid, 0)
                j = it.rid * 7 + n + it.rows
                if table is not None:
                    out[it.rid] = table[j % 64]
                else:
                    x = np.full(vocab, -100.0, np.float32)
                    x[j % vocab] = 100.0
                    out[it.rid] = x
                generated[it.rid] = n + 1
        return out
    return Engine(None, num_pages=sc["num_pages"], max_rows=sc["max_rows"], guest=guest,
                  layout=_layout(vocab))


@pytest.mark.parametrize("k", range(len(TRACE)))
def test_engine_matches_reference_trace(q3, k):
    from q3b200.engine import SamplingParams
    sc = TRACE[k]
    eng = _mock_engine(q3, sc)
    rids = [eng.add_request(r["prompt"], SamplingParams(
        max_new=r["max_new"], temperature=r.get("temperature", 0.0), top_k=r.get("top_k", 0),
        top_p=r.get("top_p", 1.0), repetition_penalty=r.get("repetition_penalty", 1.0),
        seed=r.get("seed", 0), stop_tokens=set(r["stop"])))
            for r in sc["requests"]]
    steps = []
    while eng.step():
        steps.append([[it.rid, it.row_start, it.rows, it.pos, it.token_ids, int(it.prefill),
                       int(it.needs_logits)] for it in eng.last_batch()])
        assert len(steps) < 1000
    assert steps == sc["steps"]
    assert [eng.result(r)[0] for r in rids] == sc["outputs"]
    assert [int(eng.result(r)[1]) for r in rids] == sc["finished"]
    assert eng.free_pages == sc["free_pages"]
    assert eng.steps == sc["n_steps"]
    eng.close()


def test_engine_sampling_is_seeded_and_top1_is_greedy(q3):
    from q3b200.engine import Engine, SamplingParams
    rng = np.random.default_rng(5)
    table = rng.standard_normal((64, 40)).astype(np.float32)

    def guest(items):
        return {it.rid: table[(it.token_ids[-1] + it.pos) % 64] for it in items if it.needs_logits}

    def run(params):
        eng = Engine(None, num_pages=16, max_rows=16, guest=guest, layout=_layout(40))
        rid = eng.add_request([3, 1, 4, 1, 5], params)
        eng.run(200)
        out = eng.result(rid)[0]
        eng.close()
        return out
    a = run(SamplingParams(max_new=12, temperature=0.8, top_p=0.9, seed=7))
    assert a == run(SamplingParams(max_new=12, temperature=0.8, top_p=0.9, seed=7))
    assert len(a) == 12 and all(0 <= t < 40 for t in a)
    greedy = run(SamplingParams(max_new=12))
    assert run(SamplingParams(max_new=12, temperature=1.3, top_k=1, seed=3)) == greedy
    assert run(SamplingParams(max_new=12, temperature=0.5, repetition_penalty=1.2, seed=1)) != []


def test_engine_rejects_bad_requests(q3):
    import ctypes as C
    from q3b200 import engine as E
    h = E._bind()
    L = _layout(32, max_seq=64)
    ptr = C.c_void_p()
    assert h.q3_engine_create(None, C.byref(L), 4, 8, C.byref(ptr)) == 0
    p = E._Params(40, 0.0, 0, 1.0, 1.0, 0, None, 0)
    rid = C.c_int32()
    ids = (C.c_int32 * 30)(*range(30))
    assert h.q3_engine_add_request(ptr, ids, 30, C.byref(p), C.byref(rid)) == 7   # 30 + 40 > 64
    work = C.c_int32()
    assert h.q3_engine_step(ptr, C.byref(work), None) == 1                        # no model, no guest
    assert h.q3_engine_destroy(ptr) == 0
