"""The host batching engine (``q3_engine_*`` of ``include/q3_ops.h``) with the
reference's Python surface (``tools/engine.py``): ``Engine.add_request``,
``step``, ``run``, ``outputs``, ``pool.free_pages``.

Scheduling, page pool and sampling run in the library (C++); each step runs
the batch on the GPU over the device blob (``BlobModel``), or, without a model,
through a ``guest(items) -> {rid: logits}`` callable as the reference's
``guest_step`` (the items carry rid, row_start, rows, pos, token_ids, prefill,
needs_logits).
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from types import SimpleNamespace

import numpy as np
import torch

from ._lib import Layout, check, lib


class _Params(C.Structure):
    _fields_ = [("max_new", C.c_uint32), ("temperature", C.c_double), ("top_k", C.c_uint32),
                ("top_p", C.c_double), ("repetition_penalty", C.c_double), ("seed", C.c_uint64),
                ("stop_tokens", C.POINTER(C.c_int32)), ("n_stop", C.c_uint32)]


class _Item(C.Structure):
    _fields_ = [("rid", C.c_int32), ("row_start", C.c_uint32), ("rows", C.c_uint32),
                ("pos", C.c_uint32), ("prefill", C.c_int32), ("needs_logits", C.c_int32),
                ("tokens", C.POINTER(C.c_int32))]


_GUEST = C.CFUNCTYPE(C.c_int, C.c_void_p, C.POINTER(_Item), C.c_uint32, C.POINTER(C.c_float))


def _bind():
    h = lib()
    if getattr(h, "_q3_engine_bound", False):
        return h
    sig = {
        "q3_engine_device_bytes": ([C.POINTER(Layout), C.c_uint32, C.c_uint32], C.c_size_t),
        "q3_engine_create": ([C.c_void_p, C.POINTER(Layout), C.c_uint32, C.c_uint32,
                              C.POINTER(C.c_void_p)], C.c_int),
        "q3_engine_set_guest": ([C.c_void_p, _GUEST, C.c_void_p], C.c_int),
        "q3_engine_add_request": ([C.c_void_p, C.POINTER(C.c_int32), C.c_uint32, C.POINTER(_Params),
                                   C.POINTER(C.c_int32)], C.c_int),
        "q3_engine_step": ([C.c_void_p, C.POINTER(C.c_int32), C.c_void_p], C.c_int),
        "q3_engine_run": ([C.c_void_p, C.c_uint32, C.c_void_p], C.c_int),
        "q3_engine_last_batch": ([C.c_void_p, C.POINTER(_Item), C.c_uint32, C.POINTER(C.c_uint32)],
                                 C.c_int),
        "q3_engine_result": ([C.c_void_p, C.c_int32, C.POINTER(C.c_int32), C.c_uint32,
                              C.POINTER(C.c_uint32), C.POINTER(C.c_int32)], C.c_int),
        "q3_engine_free_pages": ([C.c_void_p], C.c_uint32),
        "q3_engine_steps": ([C.c_void_p], C.c_uint64),
        "q3_engine_destroy": ([C.c_void_p], C.c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(h, name)
        fn.argtypes = args
        fn.restype = res
    h._q3_engine_bound = True
    return h


@dataclass
class SamplingParams:
    """tools/engine.py SamplingParams."""
    max_new: int = 16
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    repetition_penalty: float = 1.0
    seed: int = 0
    stop_tokens: set = field(default_factory=set)


def _items(ptr, n):
    out = []
    for i in range(n):
        it = ptr[i]
        out.append(SimpleNamespace(rid=it.rid, row_start=it.row_start, rows=it.rows, pos=it.pos,
                                   token_ids=[it.tokens[t] for t in range(it.rows)],
                                   prefill=bool(it.prefill), needs_logits=bool(it.needs_logits)))
    return out


class Engine:
    """Continuous batching over a page pool (tools/engine.py Engine).

    ``model``: a ``BlobModel`` (the GPU step; the engine allocates its page
    pool on the model's device) or ``None`` with ``guest`` and ``layout``."""

    def __init__(self, model=None, num_pages: int = 256, max_rows: int = 32, guest=None,
                 layout: Layout | None = None):
        h = _bind()
        self.model, self.guest = model, guest
        self.layout = model.L if model is not None else layout
        self.vocab = int(self.layout.vocab)
        self.ptr = C.c_void_p()
        blob = model.blob.data_ptr() if model is not None else None
        check("q3_engine_create", h.q3_engine_create(blob, C.byref(self.layout), num_pages,
                                                     max_rows, C.byref(self.ptr)))
        self._cb = None
        if guest is not None:
            def trampoline(_user, items, n, logits):
                try:
                    its = _items(items, n)
                    out = guest(its)
                    k = 0
                    for it in its:
                        if it.needs_logits:
                            row = np.asarray(out[it.rid], dtype=np.float32)
                            C.memmove(C.addressof(logits.contents) + 4 * k * self.vocab,
                                      row.ctypes.data, 4 * self.vocab)
                            k += 1
                    return 0
                except Exception:        # noqa: BLE001 -- reported as a status
                    return 1
            self._cb = _GUEST(trampoline)
            check("q3_engine_set_guest", h.q3_engine_set_guest(self.ptr, self._cb, None))
        self.rids: list[int] = []

    def add_request(self, prompt, params: SamplingParams | None = None) -> int:
        p = params or SamplingParams()
        stop = (C.c_int32 * max(1, len(p.stop_tokens)))(*sorted(p.stop_tokens))
        cp = _Params(p.max_new, p.temperature, p.top_k, p.top_p, p.repetition_penalty, p.seed,
                     stop, len(p.stop_tokens))
        ids = (C.c_int32 * len(prompt))(*[int(t) for t in prompt])
        rid = C.c_int32()
        check("q3_engine_add_request",
              _bind().q3_engine_add_request(self.ptr, ids, len(prompt), C.byref(cp), C.byref(rid)))
        self.rids.append(rid.value)
        return rid.value

    def _stream(self):
        return torch.cuda.current_stream().cuda_stream if self.model is not None else None

    def step(self) -> bool:
        work = C.c_int32()
        check("q3_engine_step", _bind().q3_engine_step(self.ptr, C.byref(work), self._stream()))
        return bool(work.value)

    def run(self, max_steps: int = 10000) -> None:
        check("q3_engine_run", _bind().q3_engine_run(self.ptr, max_steps, self._stream()))

    def last_batch(self) -> list:
        n = C.c_uint32()
        buf = (_Item * 1024)()
        check("q3_engine_last_batch", _bind().q3_engine_last_batch(self.ptr, buf, 1024, C.byref(n)))
        return _items(buf, n.value)

    def result(self, rid: int) -> tuple[list[int], bool]:
        n, fin = C.c_uint32(), C.c_int32()
        check("q3_engine_result", _bind().q3_engine_result(self.ptr, rid, None, 0, C.byref(n),
                                                           C.byref(fin)))
        ids = (C.c_int32 * max(1, n.value))()
        check("q3_engine_result", _bind().q3_engine_result(self.ptr, rid, ids, n.value, C.byref(n),
                                                           C.byref(fin)))
        return list(ids[:n.value]), bool(fin.value)

    def outputs(self) -> dict[int, list[int]]:
        return {r: self.result(r)[0] for r in self.rids}

    @property
    def steps(self) -> int:
        return int(_bind().q3_engine_steps(self.ptr))

    @property
    def free_pages(self) -> int:
        return int(_bind().q3_engine_free_pages(self.ptr))

    def close(self) -> None:
        if self.ptr:
            check("q3_engine_destroy", _bind().q3_engine_destroy(self.ptr))
            self.ptr = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:    # noqa: BLE001 -- interpreter teardown
            pass
