"""Tensor-parallel batched decode on 2+ GPUs against the single-GPU step.

Each rank is its own process on its own GPU (spawned; ``gloo`` carries only
the communicators' IPC handles).  Every rank builds the same random model and
its share of the same seeded KV pool (its KV heads), runs several greedy
decode steps through ``q3_tp_decode_step_batch``, and records the ids and the
residual stream; rank 0 then replays the steps with ``q3_decode_step_batch``
on the whole pool (itself checked against the oracle in test_model_gpu.py).
Ids, residual stream and the new K/V rows must be bit-identical.

Skipped on boxes with fewer GPUs than ranks: ranks whose kernels wait on each
other are never run as several processes on one GPU.
"""

from __future__ import annotations

import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

B, CTX, STEPS = 48, 300, 4


def _run_rank(rank, world, port, out_dir, layers):
    import ctypes as C
    import datetime
    import os
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo))
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    comm = None
    try:
        import __graft_entry__ as ge
        q3 = ge.load_package()
        from q3b200 import synthetic, tp
        from q3b200.model import Dims
        lib = q3._lib.lib()
        dev = torch.device("cuda", rank)
        max_seq = ((CTX + STEPS + 31) // 32) * 32
        dims = Dims(layers=layers, vocab=151936, max_seq=max_seq)
        bm = synthetic.random_blob_model(dims, seed=21, device=dev)
        sh = tp.shard_of(bm.L, rank, world)
        max_pages = max_seq // 32
        pool = synthetic.KVPoolTensors(layers, B * max_pages, sh.kv_heads, device=dev)
        pool.fill_random(seed=22, head0=sh.kv_head0, total_heads=8)
        g = torch.Generator().manual_seed(23)
        tables = torch.randperm(B * max_pages, generator=g).reshape(B, max_pages).to(torch.int16)
        tab = tables.to(dev)
        ids0 = torch.randint(0, 151936, (B,), generator=g, dtype=torch.int32)
        lens = torch.randint(CTX - 200, CTX, (B,), generator=g, dtype=torch.int32)
        wsb = lib.q3_decode_workspace_bytes(C.byref(bm.L), B)
        stream = torch.cuda.Stream(device=dev)

        def run(step_fn, cpool):
            ws = torch.zeros(wsb, dtype=torch.uint8, device=dev)
            ids, pos = ids0.to(dev), lens.to(dev)
            nxt = torch.zeros(B, dtype=torch.int32, device=dev)
            out = []
            for _ in range(STEPS):
                with torch.cuda.stream(stream):
                    step_fn(cpool, ids, pos, nxt, ws)
                torch.cuda.synchronize(dev)
                out.append(nxt.cpu().numpy().copy())
                ids.copy_(nxt)
                pos.add_(1)
            x = ws[:B * 1024 * 4].cpu().numpy().view(np.float32).reshape(B, 1024).copy()
            return np.stack(out), x

        comm = tp.TPComm(bm.L, rank, world, B)

        def tp_step(cpool, ids, pos, nxt, ws):
            comm.decode_step(bm.blob, bm.L, cpool, tab, max_pages, ids, pos, B, nxt, ws, stream)

        dist.barrier()
        got_ids, got_x = run(tp_step, pool.c())
        status = lib.q3_device_status()
        # the new K/V rows of this rank's heads, every layer
        kv_rows = []
        for s in range(B):
            for t in range(int(lens[s]), int(lens[s]) + STEPS):
                p = int(tables[s, t // 32]) & 0xFFFF
                kv_rows.append(pool.k[:, p, t % 32].cpu().numpy())
                kv_rows.append(pool.v[:, p, t % 32].cpu().numpy())
        res = {"ids": got_ids, "x": got_x, "status": np.asarray(status),
               "kv": np.stack(kv_rows)}
        dist.barrier()
        comm.close()
        comm = None
        if rank == 0:
            del pool
            full = synthetic.KVPoolTensors(layers, B * max_pages, 8, device=dev)
            full.fill_random(seed=22)

            def one_gpu(cpool, ids, pos, nxt, ws):
                q3._lib.check("q3_decode_step_batch", lib.q3_decode_step_batch(
                    bm.blob.data_ptr(), C.byref(bm.L), C.byref(cpool), tab.data_ptr(), max_pages,
                    ids.data_ptr(), pos.data_ptr(), B, nxt.data_ptr(), ws.data_ptr(), wsb,
                    stream.cuda_stream))

            ref_ids, ref_x = run(one_gpu, full.c())
            ref_kv = []
            for s in range(B):
                for t in range(int(lens[s]), int(lens[s]) + STEPS):
                    p = int(tables[s, t // 32]) & 0xFFFF
                    ref_kv.append(full.k[:, p, t % 32].cpu().numpy())
                    ref_kv.append(full.v[:, p, t % 32].cpu().numpy())
            res.update(ref_ids=ref_ids, ref_x=ref_x, ref_kv=np.stack(ref_kv))
        np.savez(Path(out_dir) / f"rank{rank}.npz", **res)
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_decode_matches_single_gpu(q3, tmp_path, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    layers = 3
    mp.start_processes(_run_rank, args=(world, port, str(tmp_path), layers), nprocs=world,
                       join=True, start_method="spawn")
    r0 = np.load(tmp_path / "rank0.npz")
    ref_ids, ref_x, ref_kv = r0["ref_ids"], r0["ref_x"], r0["ref_kv"]
    kvh = 8 // world
    for r in range(world):
        d = np.load(tmp_path / f"rank{r}.npz")
        assert int(d["status"]) == 0, f"rank {r}: device status {int(d['status'])}"
        np.testing.assert_array_equal(d["ids"], ref_ids)
        np.testing.assert_array_equal(d["x"].view(np.uint32), ref_x.view(np.uint32))
        np.testing.assert_array_equal(d["kv"], ref_kv[..., r * kvh * 128:(r + 1) * kvh * 128])


@pytest.mark.parametrize("buf", [0, 1, 2], ids=["o", "down", "keys"])
def test_tp_wait_timeout_then_reset(q3, buf):
    """Failure detection on one GPU, with no fault: a one-rank communicator is
    told that its own producer fell one signal behind on one exchange buffer
    (O partials, down partials or the argmax keys).  The consumer's bounded
    wait (set to 20 ms) runs out, the step returns, device status bit 20 is
    set and the context stays usable; after q3_tp_comm_reset the same step
    gives the single-GPU ids again with a clean status."""
    import ctypes as C
    import time

    from q3b200 import synthetic, tp
    from q3b200.model import Dims
    lib = q3._lib.lib()
    dev = torch.device("cuda", 0)
    Bq, ctx, layers = 4, 70, 1
    max_seq = 128
    dims = Dims(layers=layers, vocab=4096, max_seq=max_seq)
    bm = synthetic.random_blob_model(dims, seed=31, device=dev)
    max_pages = max_seq // 32
    pool = synthetic.KVPoolTensors(layers, Bq * max_pages, 8, device=dev)
    pool.fill_random(seed=32)
    g = torch.Generator().manual_seed(33)
    tab = torch.randperm(Bq * max_pages, generator=g).reshape(Bq, max_pages).to(torch.int16).to(dev)
    ids = torch.randint(0, 4096, (Bq,), generator=g, dtype=torch.int32).to(dev)
    pos = torch.full((Bq,), ctx, dtype=torch.int32, device=dev)
    wsb = lib.q3_decode_workspace_bytes(C.byref(bm.L), Bq)
    ws = torch.zeros(wsb, dtype=torch.uint8, device=dev)
    cpool = pool.c()
    stream = torch.cuda.current_stream()
    assert lib.q3_device_status() == 0

    ref = torch.zeros(Bq, dtype=torch.int32, device=dev)
    q3._lib.check("q3_decode_step_batch", lib.q3_decode_step_batch(
        bm.blob.data_ptr(), C.byref(bm.L), C.byref(cpool), tab.data_ptr(), max_pages,
        ids.data_ptr(), pos.data_ptr(), Bq, ref.data_ptr(), ws.data_ptr(), wsb,
        stream.cuda_stream))
    torch.cuda.synchronize()
    want = ref.cpu().tolist()

    comm = tp.TPComm(bm.L, 0, 1, Bq)
    try:
        comm.set_wait_ns(20_000_000)
        nxt = torch.zeros(Bq, dtype=torch.int32, device=dev)
        comm.inject_missing_signals(buf, 0, 1, stream)
        t0 = time.perf_counter()
        comm.decode_step(bm.blob, bm.L, cpool, tab, max_pages, ids, pos, Bq, nxt, ws, stream)
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
        st = lib.q3_device_status()
        assert st & (1 << 20), f"status {st:#x}: the wait did not time out"
        assert waited < 1.5, f"the step took {waited:.2f} s with a 20 ms wait limit"
        comm.reset()
        nxt.zero_()
        comm.decode_step(bm.blob, bm.L, cpool, tab, max_pages, ids, pos, Bq, nxt, ws, stream)
        torch.cuda.synchronize()
        assert lib.q3_device_status() == 0
        assert nxt.cpu().tolist() == want
    finally:
        comm.close()


PB, PT, PLAYERS = 3, 150, 2


def _run_prefill_rank(rank, world, port, out_dir):
    import ctypes as C
    import datetime
    import os
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo))
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    comm = None
    try:
        import __graft_entry__ as ge
        q3 = ge.load_package()
        from q3b200 import synthetic, tp
        from q3b200.model import Dims
        lib = q3._lib.lib()
        dev = torch.device("cuda", rank)
        max_seq = ((PT + 31) // 32) * 32
        dims = Dims(layers=PLAYERS, vocab=151936, max_seq=max_seq)
        bm = synthetic.random_blob_model(dims, seed=41, device=dev)
        sh = tp.shard_of(bm.L, rank, world)
        max_pages = max_seq // 32
        g = torch.Generator().manual_seed(43)
        tables = torch.randperm(PB * max_pages, generator=g).reshape(PB, max_pages).to(torch.int16)
        tab = tables.to(dev)
        ids = torch.randint(0, 151936, (PB * PT,), generator=g, dtype=torch.int32).to(dev)
        wsb = lib.q3_prefill_workspace_bytes(C.byref(bm.L), PB, PT)
        stream = torch.cuda.Stream(device=dev)

        def rows_of(pool):
            out = []
            for s in range(PB):
                for t in range(PT):
                    p = int(tables[s, t // 32]) & 0xFFFF
                    out.append(torch.cat([pool.k[:, p, t % 32].flatten(), pool.v[:, p, t % 32].flatten(),
                                          pool.ks[:, p, t % 32].flatten().contiguous().view(torch.int8),
                                          pool.vs[:, p, t % 32].flatten().contiguous().view(torch.int8)]).cpu().numpy())
            return np.stack(out)

        pool = synthetic.KVPoolTensors(PLAYERS, PB * max_pages, sh.kv_heads, device=dev)
        comm = tp.TPPrefillComm(bm.L, rank, world, PB * PT, PB)
        ws = torch.zeros(wsb, dtype=torch.uint8, device=dev)
        nxt = torch.full((PB,), -1, dtype=torch.int32, device=dev)
        dist.barrier()
        with torch.cuda.stream(stream):
            for _ in range(2):                 # twice: the counters carry over between calls
                comm.prefill(bm.blob, bm.L, pool.c(), tab, max_pages, ids, PB, PT, nxt, ws, stream)
        torch.cuda.synchronize(dev)
        res = {"ids": nxt.cpu().numpy(), "status": np.asarray(lib.q3_device_status()),
               "kv": rows_of(pool), "kv_head0": np.asarray(sh.kv_head0),
               "kv_heads": np.asarray(sh.kv_heads)}
        dist.barrier()
        comm.close()
        comm = None
        if rank == 0:
            del pool
            full = synthetic.KVPoolTensors(PLAYERS, PB * max_pages, 8, device=dev)
            ws = torch.zeros(wsb, dtype=torch.uint8, device=dev)
            ref = torch.full((PB,), -1, dtype=torch.int32, device=dev)
            q3._lib.check("q3_prefill_batch", lib.q3_prefill_batch(
                bm.blob.data_ptr(), C.byref(bm.L), C.byref(full.c()), tab.data_ptr(), max_pages,
                ids.data_ptr(), PB, PT, ref.data_ptr(), ws.data_ptr(), wsb, stream.cuda_stream))
            torch.cuda.synchronize(dev)
            res.update(ref_ids=ref.cpu().numpy(), ref_pk=full.k.cpu().numpy(),
                       ref_pv=full.v.cpu().numpy(), ref_pks=full.ks.cpu().numpy(),
                       ref_pvs=full.vs.cpu().numpy(), tables=tables.numpy())
        np.savez(Path(out_dir) / f"prefill_rank{rank}.npz", **res)
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_prefill_matches_single_gpu(q3, tmp_path, world):
    """Tensor-parallel batched prefill (3 prompts of 150 tokens, 2 layers, vocab
    151936) on 2/4/8 GPUs against q3_prefill_batch on one GPU: the greedy next
    ids and every prompt row's K/V (+ scales) of every layer in each rank's
    heads, bit for bit.  Layer 1's K/V depend on the residual stream after layer
    0, so they also pin the exchanged o8, x and s8 columns."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_run_prefill_rank, args=(world, port, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    r0 = np.load(tmp_path / "prefill_rank0.npz")
    tables = r0["tables"]
    for r in range(world):
        d = np.load(tmp_path / f"prefill_rank{r}.npz")
        assert int(d["status"]) == 0, f"rank {r}: device status {int(d['status'])}"
        np.testing.assert_array_equal(d["ids"], r0["ref_ids"])
        h0, nh = int(d["kv_head0"]), int(d["kv_heads"])
        want = []
        for s in range(PB):
            for t in range(PT):
                p = int(tables[s, t // 32]) & 0xFFFF
                want.append(np.concatenate([
                    r0["ref_pk"][:, p, t % 32, h0 * 128:(h0 + nh) * 128].ravel(),
                    r0["ref_pv"][:, p, t % 32, h0 * 128:(h0 + nh) * 128].ravel(),
                    r0["ref_pks"][:, p, t % 32, h0:h0 + nh].ravel().view(np.int8),
                    r0["ref_pvs"][:, p, t % 32, h0:h0 + nh].ravel().view(np.int8)]))
        np.testing.assert_array_equal(d["kv"], np.stack(want))


def _run_nccl_rank(rank, world, port, out_dir):
    import ctypes as C
    import datetime
    import os
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo))
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    comm = None
    try:
        import __graft_entry__ as ge
        q3 = ge.load_package()
        from q3b200 import synthetic, tp
        from q3b200.model import Dims
        lib = q3._lib.lib()
        dev = torch.device("cuda", rank)
        max_seq = ((CTX + 1 + 31) // 32) * 32
        dims = Dims(layers=1, vocab=151936, max_seq=max_seq)
        bm = synthetic.random_blob_model(dims, seed=51, device=dev)
        sh = tp.shard_of(bm.L, rank, world)
        max_pages = max_seq // 32
        g = torch.Generator().manual_seed(53)
        tab = torch.randperm(B * max_pages, generator=g).reshape(B, max_pages).to(torch.int16).to(dev)
        ids = torch.randint(0, 151936, (B,), generator=g, dtype=torch.int32).to(dev)
        pos = torch.randint(CTX - 200, CTX, (B,), generator=g, dtype=torch.int32).to(dev)
        wsb = lib.q3_decode_workspace_bytes(C.byref(bm.L), B)
        stream = torch.cuda.Stream(device=dev)
        comm = tp.TPComm(bm.L, rank, world, B)
        out = {}
        for name in ("exact", "nccl"):
            pool = synthetic.KVPoolTensors(1, B * max_pages, sh.kv_heads, device=dev)
            pool.fill_random(seed=52, head0=sh.kv_head0, total_heads=8)
            if name == "nccl":
                comm.use_nccl()
            ws = torch.zeros(wsb, dtype=torch.uint8, device=dev)
            nxt = torch.zeros(B, dtype=torch.int32, device=dev)
            dist.barrier()
            with torch.cuda.stream(stream):
                comm.decode_step(bm.blob, bm.L, pool.c(), tab, max_pages, ids, pos, B, nxt, ws,
                                 stream)
            torch.cuda.synchronize(dev)
            out[name + "_ids"] = nxt.cpu().numpy()
            out[name + "_x"] = ws[:B * 1024 * 4].cpu().numpy().view(np.float32).copy()
        out["status"] = np.asarray(lib.q3_device_status())
        dist.barrier()
        np.savez(Path(out_dir) / f"nccl_rank{rank}.npz", **out)
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


def test_tp_nccl_variant_close_to_exact(q3, tmp_path):
    """The ncclAllReduce form of the O / down reductions on 2 GPUs (48
    sequences, one layer, one step) against the exact ordered exchange.  The
    variant adds the ranks' partial sums in NCCL's order, so x differs in the
    last bits, and where that moves a value across an int8 rounding tie the
    requantised input of the next GEMM differs by one step.  Held to the
    tolerance of float32 stages with that allowance: at least 99.9 % of the
    residual elements within 1e-3 relative (floor 1e-3 absolute), the norm of
    the difference within 1e-3 of the norm of x, and at least 90 % of the
    greedy ids equal; every rank holds the same ids and x."""
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_run_nccl_rank, args=(world, port, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    r0 = np.load(tmp_path / "nccl_rank0.npz")
    for r in range(world):
        d = np.load(tmp_path / f"nccl_rank{r}.npz")
        assert int(d["status"]) == 0
        np.testing.assert_array_equal(d["exact_ids"], r0["exact_ids"])
        np.testing.assert_array_equal(d["nccl_ids"], r0["nccl_ids"])
        xe, xn = d["exact_x"].astype(np.float64), d["nccl_x"].astype(np.float64)
        close = np.abs(xn - xe) <= 1e-3 * np.maximum(np.abs(xe), 1e-3)
        rel = np.linalg.norm(xn - xe) / np.linalg.norm(xe)
        agree = float(np.mean(d["nccl_ids"] == d["exact_ids"]))
        msg = f"rank {r}: close {close.mean():.5f}, rel norm {rel:.2e}, ids agree {agree:.3f}"
        assert close.mean() >= 0.999 and rel <= 1e-3 and agree >= 0.9, msg
