"""The host batching engine on the GPU: requests of different lengths are fed
through mixed batches (prompt chunks of several requests and decode rows in one
step) over the engine's page pool; every request's greedy ids must equal the
oracle's greedy generate for that request alone."""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from oracle import q3_oracle as O  # noqa: E402
from oracle import synth  # noqa: E402

LAYERS, VOCAB, MAX_SEQ = 2, 4096, 128
REQUESTS = [(5, 4), (40, 3), (33, 5), (70, 2), (1, 6)]   # (prompt length, max_new)


@pytest.fixture(scope="module")
def setup(q3):
    shape = synth.Shape(layers=LAYERS, vocab=VOCAB, max_seq=MAX_SEQ)
    w = synth.build_model(shape)
    bm = q3.model.BlobModel(q3.model.Dims(layers=LAYERS, vocab=VOCAB, max_seq=MAX_SEQ)).load_weights(w)
    rng = np.random.default_rng(9)
    prompts = [[int(t) for t in rng.integers(0, VOCAB, n)] for n, _ in REQUESTS]
    want = [O.generate(w, p, len(p), m)[1] for p, (_, m) in zip(prompts, REQUESTS)]
    return bm, prompts, want


@pytest.mark.parametrize("max_rows,num_pages", [(32, 24), (6, 12)])
def test_engine_greedy_matches_oracle(q3, setup, max_rows, num_pages):
    from q3b200.engine import Engine, SamplingParams
    bm, prompts, want = setup
    eng = Engine(bm, num_pages=num_pages, max_rows=max_rows)
    rids = [eng.add_request(p, SamplingParams(max_new=m)) for p, (_, m) in zip(prompts, REQUESTS)]
    mixed = False
    while eng.step():
        items = eng.last_batch()
        mixed |= any(it.prefill for it in items) and any(not it.prefill for it in items)
    torch.cuda.synchronize()
    assert q3._lib.lib().q3_device_status() == 0
    for rid, w in zip(rids, want):
        ids, done = eng.result(rid)
        assert done and ids == w, (rid, ids, w)
    assert eng.free_pages == num_pages
    assert mixed                       # some step held prompt chunks and decode rows
    eng.close()


def test_engine_sampling_on_gpu(q3, setup):
    from q3b200.engine import Engine, SamplingParams
    bm, prompts, _ = setup

    def run():
        eng = Engine(bm, num_pages=24, max_rows=32)
        rid = eng.add_request(prompts[1], SamplingParams(max_new=6, temperature=0.7, top_k=50, seed=11))
        eng.run(100)
        out = eng.result(rid)
        eng.close()
        return out
    a, done = run()
    assert done and len(a) == 6 and all(0 <= t < VOCAB for t in a)
    assert run()[0] == a
