"""CPU restatement of the reference's host engine (TEST INFRASTRUCTURE ONLY).

``tools/engine.py:81-243`` of mland2333/qwen3-tile-ops: the page pool
(PagePool: free list popped from the end, pages given back in table order on
finish, a request that cannot get all its pages keeps the ones it got and
waits), the scheduler (Scheduler.build_batch: admission order, a prompt chunk
of min(32, prompt left, rows left) per request still in its prompt, one decode
row per generating request) and Engine.step (feed, sample, finish on a stop
token or max_new; with nothing to schedule, finish the requests that reached
max_new and report no work).  Sampling is ``oracle.sampler.sample`` with the
request's ``np.random.default_rng(seed)`` draw.  Pinned by
``tests/golden/engine_trace.json`` (batches recorded from the reference's own
engine); used to check the native engine on random request mixes.
"""

from __future__ import annotations

import numpy as np

from .sampler import sample

PAGE = 32


class _Req:
    def __init__(self, rid, prompt, p):
        self.rid, self.prompt, self.p = rid, list(prompt), p
        self.generated, self.pages = [], []
        self.n_fed, self.done = 0, False
        self.rng = np.random.default_rng(p.get("seed", 0))


class EngineRef:
    def __init__(self, guest, num_pages: int, max_rows: int):
        self.guest, self.max_rows = guest, max_rows
        self.free, self.used = list(range(num_pages)), set()
        self.reqs: list[_Req] = []
        self.steps = 0

    def add(self, prompt, **p) -> int:
        self.reqs.append(_Req(len(self.reqs), prompt, p))
        return len(self.reqs) - 1

    # -- pool (engine.py:81-115)
    def _ensure(self, r: _Req, n_tokens: int) -> bool:
        while len(r.pages) < (n_tokens + PAGE - 1) // PAGE:
            if not self.free:
                return False
            pg = self.free.pop()
            self.used.add(pg)
            r.pages.append(pg)
        return True

    def _finish(self, r: _Req) -> None:
        if r.done:
            return
        r.done = True
        for pg in r.pages:
            if pg in self.used:
                self.used.remove(pg)
                self.free.append(pg)
        r.pages = []

    # -- scheduler (engine.py:172-205): (rid, row_start, rows, pos, ids, prefill, needs_logits)
    def _batch(self):
        items, rows = [], 0
        for r in self.reqs:
            if r.done:
                continue
            if r.n_fed < len(r.prompt):
                if rows >= self.max_rows:
                    continue
                chunk = min(32, len(r.prompt) - r.n_fed, self.max_rows - rows)
                if chunk <= 0 or not self._ensure(r, r.n_fed + chunk):
                    continue
                items.append((r, rows, chunk, r.n_fed, r.prompt[r.n_fed:r.n_fed + chunk], 1,
                              int(r.n_fed + chunk == len(r.prompt))))
                rows += chunk
                continue
            if len(r.generated) >= r.p.get("max_new", 16):
                self._finish(r)
                continue
            if rows >= self.max_rows or not r.generated:
                continue
            if not self._ensure(r, r.n_fed + 1):
                continue
            items.append((r, rows, 1, r.n_fed, [r.generated[-1]], 0, 1))
            rows += 1
        return items

    # -- Engine.step (engine.py:218-239)
    def step(self):
        items = self._batch()
        if not items:
            for r in self.reqs:
                if (not r.done and r.n_fed >= len(r.prompt)
                        and len(r.generated) >= r.p.get("max_new", 16)):
                    self._finish(r)
            return None
        logits = self.guest(items)
        for r, _, rows, _, _, _, need in items:
            r.n_fed += rows
            if need:
                t = r.p.get("temperature", 0.0)
                u = r.rng.random() if t > 0.0 else 0.0
                tok = sample(logits[r.rid], t, r.p.get("top_k", 0), r.p.get("top_p", 1.0),
                             r.p.get("repetition_penalty", 1.0), r.generated, u)
                r.generated.append(tok)
                if tok in r.p.get("stop", ()) or len(r.generated) >= r.p.get("max_new", 16):
                    self._finish(r)
        self.steps += 1
        return [[r.rid, rs, rows, pos, list(ids), pf, need] for r, rs, rows, pos, ids, pf, need in items]

    def run(self, max_steps: int = 2000):
        trace = []
        while self.steps < max_steps:
            b = self.step()
            if b is None:
                break
            trace.append(b)
        return trace
