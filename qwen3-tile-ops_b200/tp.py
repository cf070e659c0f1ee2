"""Tensor-parallel batched decode over the GPUs of one node (one process per GPU).

The C ABI does the work (``q3_tp_*`` in ``include/q3_ops.h``): each rank owns
``kv_heads/world`` KV heads (and their Q heads), a contiguous run of the 256-wide
MLP groups and a slice of the vocabulary; the O and down GEMMs store their
per-group partials straight into every rank's receive buffer over NVLink and
each rank sums all groups in group order, so every rank's residual stream is
bit-identical to the single-GPU one.  ``torch.distributed`` is used only here,
to swap the communicators' CUDA IPC handles once at setup.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from ._lib import Layout, check, lib


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    q_head0: int
    q_heads: int
    kv_head0: int
    kv_heads: int
    mlp_group0: int
    mlp_groups: int
    vocab0: int
    vocab_rows: int


class _CShard(C.Structure):
    _fields_ = [("rank", C.c_int32), ("world", C.c_int32), ("q_head0", C.c_uint32),
                ("q_heads", C.c_uint32), ("kv_head0", C.c_uint32), ("kv_heads", C.c_uint32),
                ("mlp_group0", C.c_uint32), ("mlp_groups", C.c_uint32), ("vocab0", C.c_uint32),
                ("vocab_rows", C.c_uint32)]


def _bind():
    h = lib()
    if getattr(h, "_q3_tp_bound", False):
        return h
    h.q3_tp_shard_of.argtypes = [C.POINTER(Layout), C.c_int32, C.c_int32, C.POINTER(_CShard)]
    h.q3_tp_handle_bytes.argtypes = []
    h.q3_tp_handle_bytes.restype = C.c_size_t
    h.q3_tp_comm_create.argtypes = [C.POINTER(Layout), C.c_int32, C.c_int32, C.c_uint32,
                                    C.POINTER(C.c_void_p), C.c_void_p]
    h.q3_tp_comm_connect.argtypes = [C.c_void_p, C.c_void_p]
    h.q3_tp_comm_reset.argtypes = [C.c_void_p, C.c_void_p]
    h.q3_tp_comm_destroy.argtypes = [C.c_void_p]
    h.q3_tp_decode_step_batch.argtypes = [C.c_void_p, C.c_void_p, C.POINTER(Layout), C.c_void_p,
                                          C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p,
                                          C.c_uint32, C.c_void_p, C.c_void_p, C.c_size_t,
                                          C.c_void_p]
    h.q3_tp_comm_set_wait_ns.argtypes = [C.c_void_p, C.c_uint64]
    h.q3_tp_comm_inject_missing_signals.argtypes = [C.c_void_p, C.c_int32, C.c_int32, C.c_uint32,
                                                    C.c_void_p]
    h.q3_tp_nccl_unique_id.argtypes = [C.c_void_p]
    h.q3_tp_comm_set_reduction.argtypes = [C.c_void_p, C.c_int32, C.c_void_p]
    h.q3_tp_nccl_unique_id.restype = C.c_int
    h.q3_tp_comm_set_reduction.restype = C.c_int
    h.q3_tp_prefill_comm_create.argtypes = [C.POINTER(Layout), C.c_int32, C.c_int32, C.c_uint32,
                                            C.c_uint32, C.POINTER(C.c_void_p), C.c_void_p]
    h.q3_tp_prefill_comm_connect.argtypes = [C.c_void_p, C.c_void_p]
    h.q3_tp_prefill_comm_reset.argtypes = [C.c_void_p, C.c_void_p]
    h.q3_tp_prefill_comm_set_wait_ns.argtypes = [C.c_void_p, C.c_uint64]
    h.q3_tp_prefill_comm_destroy.argtypes = [C.c_void_p]
    h.q3_tp_prefill_batch.argtypes = [C.c_void_p, C.c_void_p, C.POINTER(Layout), C.c_void_p,
                                      C.c_void_p, C.c_uint32, C.c_void_p, C.c_uint32, C.c_uint32,
                                      C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]
    for name in ("q3_tp_shard_of", "q3_tp_comm_create", "q3_tp_comm_connect", "q3_tp_comm_reset",
                 "q3_tp_comm_destroy", "q3_tp_decode_step_batch", "q3_tp_comm_set_wait_ns",
                 "q3_tp_comm_inject_missing_signals", "q3_tp_prefill_comm_create",
                 "q3_tp_prefill_comm_connect", "q3_tp_prefill_comm_reset",
                 "q3_tp_prefill_comm_set_wait_ns", "q3_tp_prefill_comm_destroy",
                 "q3_tp_prefill_batch"):
        getattr(h, name).restype = C.c_int
    h._q3_tp_bound = True
    return h


def shard_of(layout: Layout, rank: int, world: int) -> Shard:
    """The part of the model rank ``rank`` of ``world`` owns (host only)."""
    s = _CShard()
    check("q3_tp_shard_of", _bind().q3_tp_shard_of(C.byref(layout), rank, world, C.byref(s)))
    return Shard(*(getattr(s, f) for f, _ in _CShard._fields_))


class TPComm:
    """One rank's communicator: its exchange region, mapped by every rank.

    Collective over ``group`` (default: the default process group): every rank
    constructs it with the same layout and ``max_seqs``.  ``world == 1`` needs
    no process group."""

    def __init__(self, layout: Layout, rank: int, world: int, max_seqs: int, group=None):
        h = _bind()
        self.layout, self.rank, self.world, self.group = layout, rank, world, group
        self.shard = shard_of(layout, rank, world)
        hb = h.q3_tp_handle_bytes()
        handle = (C.c_ubyte * hb)()
        self.ptr = C.c_void_p()
        check("q3_tp_comm_create",
              h.q3_tp_comm_create(C.byref(layout), rank, world, max_seqs, C.byref(self.ptr), handle))
        handles = (C.c_ubyte * (hb * world))()
        if world == 1:
            C.memmove(handles, handle, hb)
        else:
            import torch.distributed as dist
            dev = torch.device("cuda", torch.cuda.current_device()) \
                if dist.get_backend(group) == "nccl" else torch.device("cpu")
            mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=dev)
            every = torch.empty(hb * world, dtype=torch.uint8, device=dev)
            dist.all_gather_into_tensor(every, mine, group=group)
            C.memmove(handles, bytes(every.cpu().tolist()), hb * world)
        check("q3_tp_comm_connect", h.q3_tp_comm_connect(self.ptr, handles))
        self._barrier()

    def _barrier(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier(group=self.group)

    def decode_step(self, blob: torch.Tensor, layout: Layout, pool, tables: torch.Tensor,
                    max_pages: int, ids: torch.Tensor, pos: torch.Tensor, n_seqs: int,
                    next_ids: torch.Tensor, ws: torch.Tensor, stream) -> None:
        """Enqueue this rank's share of one decode step (``pool`` = KVPool of
        this rank's KV heads); every rank passes the same ids/pos/tables."""
        check("q3_tp_decode_step_batch", _bind().q3_tp_decode_step_batch(
            self.ptr, blob.data_ptr(), C.byref(layout), C.byref(pool), tables.data_ptr(),
            max_pages, ids.data_ptr(), pos.data_ptr(), n_seqs, next_ids.data_ptr(),
            ws.data_ptr(), ws.numel(), stream.cuda_stream))

    def reset(self) -> None:
        """Zero every rank's signal counters (no step may be in flight)."""
        self._barrier()
        check("q3_tp_comm_reset", _bind().q3_tp_comm_reset(self.ptr, None))
        torch.cuda.synchronize()
        self._barrier()

    def use_nccl(self, on: bool = True) -> None:
        """Switch the O / down reductions to the ncclAllReduce comparison
        variant (``on``) or back to the exact ordered exchange.  The first
        switch on is collective: rank 0 makes the NCCL id and the process group
        carries it to the others."""
        h = _bind()
        uid = None
        if on:
            raw = (C.c_ubyte * 128)()
            if self.rank == 0:
                check("q3_tp_nccl_unique_id", h.q3_tp_nccl_unique_id(raw))
            if self.world > 1:
                import torch.distributed as dist
                box = [bytes(raw)]
                dist.broadcast_object_list(box, src=0, group=self.group)
                C.memmove(raw, box[0], 128)
            uid = raw
        check("q3_tp_comm_set_reduction",
              h.q3_tp_comm_set_reduction(self.ptr, 1 if on else 0, uid))

    def set_wait_ns(self, ns: int) -> None:
        """How long this rank's kernels wait for a peer's signal before they
        give up and set device status bit 20 (default 2 s)."""
        check("q3_tp_comm_set_wait_ns", _bind().q3_tp_comm_set_wait_ns(self.ptr, int(ns)))

    def inject_missing_signals(self, buf: int, producer: int, count: int = 1, stream=None) -> None:
        """Failure injection on the host side: raise this rank's expected
        signal count of exchange buffer ``buf`` (0 O, 1 down, 2 argmax keys)
        from ``producer`` by ``count``, as if that producer had fallen behind."""
        st = None if stream is None else stream.cuda_stream
        check("q3_tp_comm_inject_missing_signals",
              _bind().q3_tp_comm_inject_missing_signals(self.ptr, buf, producer, count, st))

    def close(self) -> None:
        if self.ptr:
            self._barrier()
            torch.cuda.synchronize()
            check("q3_tp_comm_destroy", _bind().q3_tp_comm_destroy(self.ptr))
            self.ptr = C.c_void_p()


def _gather_handles(handle, hb: int, world: int, group) -> "C.Array":
    handles = (C.c_ubyte * (hb * world))()
    if world == 1:
        C.memmove(handles, handle, hb)
        return handles
    import torch.distributed as dist
    dev = torch.device("cuda", torch.cuda.current_device()) \
        if dist.get_backend(group) == "nccl" else torch.device("cpu")
    mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=dev)
    every = torch.empty(hb * world, dtype=torch.uint8, device=dev)
    dist.all_gather_into_tensor(every, mine, group=group)
    C.memmove(handles, bytes(every.cpu().tolist()), hb * world)
    return handles


class TPPrefillComm:
    """One rank's communicator of the tensor-parallel prefill
    (``q3_tp_prefill_batch``): the exchanged o8/os, x and s8/ss buffers of up
    to ``max_rows`` prompt rows, mapped by every rank.  Collective over
    ``group`` (default: the default process group)."""

    def __init__(self, layout: Layout, rank: int, world: int, max_rows: int, max_seqs: int,
                 group=None):
        h = _bind()
        self.layout, self.rank, self.world, self.group = layout, rank, world, group
        self.shard = shard_of(layout, rank, world)
        hb = h.q3_tp_handle_bytes()
        handle = (C.c_ubyte * hb)()
        self.ptr = C.c_void_p()
        check("q3_tp_prefill_comm_create",
              h.q3_tp_prefill_comm_create(C.byref(layout), rank, world, max_rows, max_seqs,
                                          C.byref(self.ptr), handle))
        handles = _gather_handles(handle, hb, world, group)
        check("q3_tp_prefill_comm_connect", h.q3_tp_prefill_comm_connect(self.ptr, handles))
        self._barrier()

    def _barrier(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier(group=self.group)

    def prefill(self, blob: torch.Tensor, layout: Layout, pool, tables: torch.Tensor,
                max_pages: int, ids: torch.Tensor, n_seqs: int, T: int, next_ids: torch.Tensor,
                ws: torch.Tensor, stream) -> None:
        """Enqueue this rank's share of one batched prefill (``pool`` = KVPool
        of this rank's KV heads); every rank passes the same ids and tables."""
        check("q3_tp_prefill_batch", _bind().q3_tp_prefill_batch(
            self.ptr, blob.data_ptr(), C.byref(layout), C.byref(pool), tables.data_ptr(),
            max_pages, ids.data_ptr(), n_seqs, T, next_ids.data_ptr(), ws.data_ptr(),
            ws.numel(), stream.cuda_stream))

    def set_wait_ns(self, ns: int) -> None:
        check("q3_tp_prefill_comm_set_wait_ns",
              _bind().q3_tp_prefill_comm_set_wait_ns(self.ptr, int(ns)))

    def reset(self) -> None:
        """Zero every rank's counters (no prefill may be in flight)."""
        self._barrier()
        check("q3_tp_prefill_comm_reset", _bind().q3_tp_prefill_comm_reset(self.ptr, None))
        torch.cuda.synchronize()
        self._barrier()

    def close(self) -> None:
        if self.ptr:
            self._barrier()
            torch.cuda.synchronize()
            check("q3_tp_prefill_comm_destroy", _bind().q3_tp_prefill_comm_destroy(self.ptr))
            self.ptr = C.c_void_p()
