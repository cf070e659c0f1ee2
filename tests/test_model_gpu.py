"""Model-level parity on the GPU: the greedy loop (q3_generate) and one chunk
(q3_forward_chunk) against the golden vectors of the reference's own mirror,
stage by stage like the reference's tools/compare.py; the batched paged decode
(q3_decode_step_batch) against the oracle run one sequence at a time."""

from __future__ import annotations

import ctypes as C
import hashlib

import numpy as np
import pytest

from conftest import load_golden

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
F = np.float32

from oracle import q3_oracle as O  # noqa: E402
from oracle import synth  # noqa: E402


def same_bits(a, b, what=""):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape, (what, a.shape, b.shape)
    if a.dtype == np.float32:
        bad = np.count_nonzero(a.view(np.uint32) != np.asarray(b, F).view(np.uint32))
    else:
        bad = np.count_nonzero(a != b)
    assert bad == 0, f"{what}: {bad}/{a.size} elements differ"


@pytest.fixture(scope="module")
def cfg1(q3):
    assert torch.cuda.is_available()
    w = synth.build_model(synth.Shape(layers=1, vocab=1024))
    dims = q3.model.Dims(layers=1, vocab=1024)
    bm = q3.model.BlobModel(dims).load_weights(w)
    return w, bm


@pytest.mark.parametrize("mode", [0, 1])
def test_config1_generate(cfg1, mode):
    """Config 1: 40-token prompt (32 + 8 rows), 2 greedy tokens; mode 0 is the
    fused lm_head+argmax production path, mode 1 writes logits."""
    w, bm = cfg1
    g = load_golden("model_cfg1_cr.npz")
    ids = synth.config1_ids()
    got = bm.generate(ids, 40, 2, mode=mode)
    assert got == [int(v) for v in g["generated"]]
    # KV cache of the (only) layer, un-paged through the reversed table
    k8, ks, v8, vs = bm.kv_layer(0)
    last = g["c3_kc"].shape[0]
    same_bits(k8[:last], g["c3_kc"], "kc")
    same_bits(ks[:last], g["c3_ks"], "ks")
    same_bits(v8[:last], g["c3_vc"], "vc")
    same_bits(vs[:last], g["c3_vs"], "vs")
    # last step (pos 41, 1 row): stage buffers left in the blob
    for st, key, shape, dt in (("x", "kX", (1, 1024), F), ("s8", "kS8", (1, 3072), np.int8),
                               ("ss", "kSS", (1, 12), F), ("o8", "kO8", (1, 2048), np.int8),
                               ("os", "kOS", (1, 16), F)):
        same_bits(bm.read(key, shape, dt), g[f"c3_{st}"], st)
    logits = g["c3_logits"].reshape(-1)
    if mode == 1:
        same_bits(bm.read("kLOGITS", (1, 1024), F), g["c3_logits"], "logits")
    else:
        argf = bm.read("kARGF", (1,), F)
        argi = bm.read("kARGI", (1,), np.int32)
        same_bits(argf, logits.max(keepdims=True), "argf")
        assert int(argi[0]) == int(np.argmax(logits))


def test_config1_forward_chunk_stages(cfg1, q3):
    """The 8-row prompt chunk (pos 32) after the 32-row one, non-fused: every
    materialised stage of the last layer equals the golden record."""
    w, bm = cfg1
    g = load_golden("model_cfg1_cr.npz")
    ids = [int(v) for v in g["ids"]]
    bm.set_ids(ids)
    bm.forward_chunk(0, 32, q3.model.LM_NONE, False)
    bm.forward_chunk(32, 8, q3.model.LM_LOGITS, False)
    torch.cuda.synchronize()
    r = 8
    for st, key, shape, dt in (("x", "kX", (r, 1024), F), ("h", "kH", (r, 1024), F),
                               ("h8", "kH8", (r, 1024), np.int8), ("hs", "kHS", (r, 4), F),
                               ("o8", "kO8", (r, 2048), np.int8), ("os", "kOS", (r, 16), F),
                               ("s8", "kS8", (r, 3072), np.int8), ("ss", "kSS", (r, 12), F)):
        same_bits(bm.read(key, shape, dt), g[f"c1_{st}"], st)
    # q8/qs rows 1.. (row 0 is the final-norm scratch, compare.py:197-205)
    same_bits(bm.read("kQ8", (r, 2048), np.int8)[1:], g["c1_q8"][1:], "q8")
    same_bits(bm.read("kQS", (r, 16), F)[1:], g["c1_qs"][1:], "qs")
    same_bits(bm.read("kLOGITS", (1, 1024), F), g["c1_logits"], "logits")
    # first chunk's int8 stages went into the KV cache
    k8, ks, v8, vs = bm.kv_layer(0)
    same_bits(k8[:32], g["c0_kc"][:32], "kc0")
    same_bits(v8[:32], g["c0_vc"][:32], "vc0")


def test_config3_full_shape_generate(q3):
    """Config 3: 28 layers, vocab 151936, 32-token seeded prompt, 6 greedy
    tokens (fused path) and the final logits of the non-fused path."""
    g = load_golden("model_cfg3_cr.npz")
    w = synth.build_model(synth.Shape())
    assert synth.weights_digest(w) == str(g["digest"])
    bm = q3.model.BlobModel(q3.model.Dims()).load_weights(w)
    ids = [int(v) for v in np.random.default_rng(1).integers(0, 151936, 32)]
    assert bm.generate(ids, 32, 6, mode=0) == [int(v) for v in g["generated"]]
    assert bm.generate(ids, 32, 6, mode=1) == [int(v) for v in g["generated"]]
    lg = bm.read("kLOGITS", (1, 151936), F)
    assert hashlib.sha256(np.ascontiguousarray(lg).tobytes()).hexdigest() == str(g["logits_sha"])


# ---------------------------------------------------------------- batched decode
def _decode_case(q3, layers, vocab, lens, seed=0, tp_world1=False, nccl=False):
    """Prefill each sequence on the oracle, load its KV into a shared page
    pool under a shuffled page table, run ONE batched decode step on the GPU
    and the oracle per sequence; return both.  ``tp_world1``: the step runs
    through the tensor-parallel entry point with a one-rank communicator (the
    partial-GEMM, ordered-reduce and key-exchange kernels, no peers)."""
    shape = synth.Shape(layers=layers, vocab=vocab, max_seq=(max(lens) + 64 + 31) // 32 * 32)
    w = synth.build_model(shape)
    rng = np.random.default_rng(seed)
    B = len(lens)
    max_pages = (shape.max_seq + 31) // 32
    total_pages = B * max_pages
    perm = rng.permutation(total_pages)
    tables = perm.reshape(B, max_pages).astype(np.uint16)
    kw = 8 * 128
    pk = np.zeros((layers, total_pages, 32, kw), np.int8)
    pv = np.zeros_like(pk)
    pks = np.zeros((layers, total_pages, 32, 8), F)
    pvs = np.zeros_like(pks)
    ids_now, want_ids, want_kv = [], [], []
    for s, n in enumerate(lens):
        prompt = [int(v) for v in rng.integers(0, vocab, n)]
        kv = O.KV.empty(w, shape.max_seq)
        pos = 0
        while pos < n:                       # oracle prefill in 32-row chunks
            rows = min(32, n - pos)
            O.forward_chunk(w, prompt[pos:pos + rows], kv, pos, rows, False)
            pos += rows
        for L in range(layers):
            for t in range(n):
                p, sl = tables[s, t // 32], t % 32
                pk[L, p, sl], pv[L, p, sl] = kv.k8[L][t], kv.v8[L][t]
                pks[L, p, sl], pvs[L, p, sl] = kv.ks[L][t], kv.vs[L][t]
        tok = int(rng.integers(0, vocab))
        ids_now.append(tok)
        lg = O.forward_chunk(w, [tok], kv, n, 1, True)
        want_ids.append(O.argmax_logits(lg))
        want_kv.append(kv)
    dims = q3.model.Dims(layers=layers, vocab=vocab, max_seq=shape.max_seq)
    bm = q3.model.BlobModel(dims).load_weights(w)
    d = {k: torch.from_numpy(v).cuda() for k, v in
         (("pk", pk), ("pv", pv), ("pks", pks), ("pvs", pvs))}
    pool = q3._lib.KVPool(d["pk"].data_ptr(), d["pv"].data_ptr(), d["pks"].data_ptr(),
                          d["pvs"].data_ptr(), total_pages * 32 * kw, total_pages * 32 * 8 * 4,
                          total_pages)
    tab = torch.from_numpy(tables.view(np.int16)).cuda()
    ids_d = torch.tensor(ids_now, dtype=torch.int32, device="cuda")
    pos_d = torch.tensor(lens, dtype=torch.int32, device="cuda")
    nxt = torch.zeros(B, dtype=torch.int32, device="cuda")
    lib = q3._lib.lib()
    wsb = lib.q3_decode_workspace_bytes(C.byref(bm.L), B)
    ws = torch.zeros(wsb, dtype=torch.uint8, device="cuda")
    if tp_world1:
        from q3b200 import tp
        comm = tp.TPComm(bm.L, 0, 1, B)
        if nccl:
            comm.use_nccl()
        comm.decode_step(bm.blob, bm.L, pool, tab, max_pages, ids_d, pos_d, B, nxt, ws,
                         torch.cuda.current_stream())
        torch.cuda.synchronize()
        comm.close()
    else:
        q3._lib.check("q3_decode_step_batch", lib.q3_decode_step_batch(
            bm.blob.data_ptr(), C.byref(bm.L), C.byref(pool), tab.data_ptr(), max_pages,
            ids_d.data_ptr(), pos_d.data_ptr(), B, nxt.data_ptr(), ws.data_ptr(), wsb,
            torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
    assert lib.q3_device_status() == 0
    return (nxt.cpu().numpy(), want_ids, {k: v.cpu().numpy() for k, v in d.items()}, tables,
            want_kv)


@pytest.mark.parametrize("variant", ["single", "tp1", "tp1-nccl"])
@pytest.mark.parametrize("layers,vocab,lens", [(1, 1024, [5, 40, 64, 33]),
                                               (2, 4096, [100, 1, 31, 32, 250])])
def test_decode_step_batch(q3, layers, vocab, lens, variant):
    """"tp1-nccl": the ncclAllReduce reduction variant with one rank, where the
    in-order sum of the rank's groups is the whole sum, so it must be exact."""
    got, want, pool, tables, kvs = _decode_case(q3, layers, vocab, lens,
                                                tp_world1=variant != "single",
                                                nccl=variant == "tp1-nccl")
    assert list(got) == want
    for s, n in enumerate(lens):          # the new K/V row of every layer
        p, sl = tables[s, n // 32], n % 32
        for L in range(layers):
            assert np.array_equal(pool["pk"][L, p, sl], kvs[s].k8[L][n])
            assert np.array_equal(pool["pv"][L, p, sl], kvs[s].v8[L][n])
            same_bits(pool["pks"][L, p, sl], kvs[s].ks[L][n])
            same_bits(pool["pvs"][L, p, sl], kvs[s].vs[L][n])


# ---------------------------------------------------------------- batched prefill
def _prefill_case(q3, layers, vocab, B, T, seed=0, tp_world1=False):
    """Prefill B prompts of T tokens on the oracle (32-row chunks) and in ONE
    batched GPU prefill into a shared page pool under shuffled page tables.
    ``tp_world1``: through the tensor-parallel entry point with a one-rank
    communicator (its exchange kernels run, with no peers)."""
    shape = synth.Shape(layers=layers, vocab=vocab, max_seq=(T + 31) // 32 * 32)
    w = synth.build_model(shape)
    rng = np.random.default_rng(seed)
    max_pages = shape.max_seq // 32
    total_pages = B * max_pages
    tables = rng.permutation(total_pages).reshape(B, max_pages).astype(np.uint16)
    prompts = rng.integers(0, vocab, (B, T))
    want_ids, want_kv = [], []
    for s in range(B):
        kv = O.KV.empty(w, shape.max_seq)
        pos, lg = 0, None
        while pos < T:
            rows = min(32, T - pos)
            lg = O.forward_chunk(w, [int(v) for v in prompts[s, pos:pos + rows]], kv, pos, rows,
                                 pos + rows == T)
            pos += rows
        want_ids.append(O.argmax_logits(lg))
        want_kv.append(kv)
    dims = q3.model.Dims(layers=layers, vocab=vocab, max_seq=shape.max_seq)
    bm = q3.model.BlobModel(dims).load_weights(w)
    kw = 8 * 128
    d = {"pk": torch.zeros((layers, total_pages, 32, kw), dtype=torch.int8, device="cuda"),
         "pv": torch.zeros((layers, total_pages, 32, kw), dtype=torch.int8, device="cuda"),
         "pks": torch.zeros((layers, total_pages, 32, 8), dtype=torch.float32, device="cuda"),
         "pvs": torch.zeros((layers, total_pages, 32, 8), dtype=torch.float32, device="cuda")}
    pool = q3._lib.KVPool(d["pk"].data_ptr(), d["pv"].data_ptr(), d["pks"].data_ptr(),
                          d["pvs"].data_ptr(), total_pages * 32 * kw, total_pages * 32 * 8 * 4,
                          total_pages)
    tab = torch.from_numpy(tables.view(np.int16)).cuda()
    ids_d = torch.from_numpy(prompts.astype(np.int32).reshape(-1)).cuda()
    nxt = torch.full((B,), -1, dtype=torch.int32, device="cuda")
    lib = q3._lib.lib()
    wsb = lib.q3_prefill_workspace_bytes(C.byref(bm.L), B, T)
    ws = torch.zeros(wsb, dtype=torch.uint8, device="cuda")
    if tp_world1:
        from q3b200 import tp
        comm = tp.TPPrefillComm(bm.L, 0, 1, B * T, B)
        comm.prefill(bm.blob, bm.L, pool, tab, max_pages, ids_d, B, T, nxt, ws,
                     torch.cuda.current_stream())
        torch.cuda.synchronize()
        comm.close()
    else:
        q3._lib.check("q3_prefill_batch", lib.q3_prefill_batch(
            bm.blob.data_ptr(), C.byref(bm.L), C.byref(pool), tab.data_ptr(), max_pages,
            ids_d.data_ptr(), B, T, nxt.data_ptr(), ws.data_ptr(), wsb,
            torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert q3._lib.lib().q3_device_status() == 0
    return (nxt.cpu().numpy(), want_ids, {k: v.cpu().numpy() for k, v in d.items()}, tables,
            want_kv)


@pytest.mark.parametrize("tp_world1", [False, True], ids=["single", "tp1"])
@pytest.mark.parametrize("layers,vocab,B,T", [(1, 1024, 3, 70), (2, 4096, 2, 128), (1, 1024, 2, 300)])
def test_prefill_batch(q3, layers, vocab, B, T, tp_world1):
    got, want, pool, tables, kvs = _prefill_case(q3, layers, vocab, B, T, tp_world1=tp_world1)
    assert list(got) == want
    for s in range(B):                    # every prompt row of every layer, un-paged
        for L in range(layers):
            for t in range(T):
                p, sl = tables[s, t // 32], t % 32
                assert np.array_equal(pool["pk"][L, p, sl], kvs[s].k8[L][t])
                assert np.array_equal(pool["pv"][L, p, sl], kvs[s].v8[L][t])
                same_bits(pool["pks"][L, p, sl], kvs[s].ks[L][t])
                same_bits(pool["pvs"][L, p, sl], kvs[s].vs[L][t])


# ------------------------------------------- batched decode at the benchmark shape
def test_decode_step_batch_benchmark_shape(q3):
    """The benchmarked decode regime: 64 sequences at contexts 2048-2111 (512
    attention CTAs, full 64-token cluster GEMM tiles), 2 layers, vocab 4096,
    shuffled page tables.  The seeded int8 K/V prefixes and their scales are
    written into the page pool and, through each sequence's page table, into
    the oracle's per-sequence cache (no CPU prefill).  One batched step on the
    GPU against the oracle's forward_chunk per sequence: the greedy ids, the
    residual stream x and the new K/V rows of every layer, bit for bit."""
    layers, vocab, B = 2, 4096, 64
    rng = np.random.default_rng(44)
    lens = [int(v) for v in rng.integers(2048, 2112, B)]
    max_seq = 2176
    shape = synth.Shape(layers=layers, vocab=vocab, max_seq=max_seq)
    w = synth.build_model(shape)
    max_pages = max_seq // 32
    total_pages = B * max_pages
    tables = rng.permutation(total_pages).reshape(B, max_pages).astype(np.uint16)
    kw = 8 * 128
    pk = rng.integers(-127, 128, (layers, total_pages, 32, kw), dtype=np.int8)
    pv = rng.integers(-127, 128, (layers, total_pages, 32, kw), dtype=np.int8)
    pks = rng.uniform(1e-3, 1e-2, (layers, total_pages, 32, 8)).astype(F)
    pvs = rng.uniform(1e-3, 1e-2, (layers, total_pages, 32, 8)).astype(F)
    ids_now = [int(v) for v in rng.integers(0, vocab, B)]
    dims = q3.model.Dims(layers=layers, vocab=vocab, max_seq=max_seq)
    bm = q3.model.BlobModel(dims).load_weights(w)
    d = {k: torch.from_numpy(v).cuda() for k, v in
         (("pk", pk), ("pv", pv), ("pks", pks), ("pvs", pvs))}
    pool = q3._lib.KVPool(d["pk"].data_ptr(), d["pv"].data_ptr(), d["pks"].data_ptr(),
                          d["pvs"].data_ptr(), total_pages * 32 * kw, total_pages * 32 * 8 * 4,
                          total_pages)
    tab = torch.from_numpy(tables.view(np.int16)).cuda()
    ids_d = torch.tensor(ids_now, dtype=torch.int32, device="cuda")
    pos_d = torch.tensor(lens, dtype=torch.int32, device="cuda")
    nxt = torch.zeros(B, dtype=torch.int32, device="cuda")
    lib = q3._lib.lib()
    wsb = lib.q3_decode_workspace_bytes(C.byref(bm.L), B)
    ws = torch.zeros(wsb, dtype=torch.uint8, device="cuda")
    q3._lib.check("q3_decode_step_batch", lib.q3_decode_step_batch(
        bm.blob.data_ptr(), C.byref(bm.L), C.byref(pool), tab.data_ptr(), max_pages,
        ids_d.data_ptr(), pos_d.data_ptr(), B, nxt.data_ptr(), ws.data_ptr(), wsb,
        torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert lib.q3_device_status() == 0
    got_ids = nxt.cpu().numpy()
    got_x = ws[:B * 1024 * 4].cpu().numpy().view(F).reshape(B, 1024)
    got = {k: v.cpu().numpy() for k, v in d.items()}
    slots = np.arange(max_seq) % 32
    for s, n in enumerate(lens):
        kv = O.KV.empty(w, max_seq)
        pages = tables[s, np.arange(n) // 32]
        for L in range(layers):
            kv.k8[L][:n] = pk[L, pages, slots[:n]]
            kv.v8[L][:n] = pv[L, pages, slots[:n]]
            kv.ks[L][:n] = pks[L, pages, slots[:n]]
            kv.vs[L][:n] = pvs[L, pages, slots[:n]]
        rec = {}
        lg = O.forward_chunk(w, [ids_now[s]], kv, n, 1, True, rec)
        assert int(got_ids[s]) == O.argmax_logits(lg), f"sequence {s}"
        same_bits(got_x[s:s + 1], rec["x"], f"x of sequence {s}")
        p, sl = tables[s, n // 32], n % 32
        for L in range(layers):
            assert np.array_equal(got["pk"][L, p, sl], kv.k8[L][n]), (s, L)
            assert np.array_equal(got["pv"][L, p, sl], kv.v8[L][n]), (s, L)
            same_bits(got["pks"][L, p, sl], kv.ks[L][n], f"ks {s} {L}")
            same_bits(got["pvs"][L, p, sl], kv.vs[L][n], f"vs {s} {L}")


# ------------------------------------------- batched prefill at the benchmark length
def test_prefill_batch_4096_causal(q3):
    """The long-prompt regime: 2 prompts of 4096 tokens, one layer, vocab 1024,
    in ONE batched prefill (8192 stacked GEMM rows; causal attention over 128
    pages per prompt).  Every prompt row's K/V in the pool, the residual stream
    x of a sample of rows (page edges, the first and last rows, 64 random rows;
    x carries the attention output through the O GEMM) and the greedy next id
    of each prompt, bit for bit against the oracle."""
    layers, vocab, B, T = 1, 1024, 2, 4096
    shape = synth.Shape(layers=layers, vocab=vocab, max_seq=T)
    w = synth.build_model(shape)
    rng = np.random.default_rng(45)
    max_pages = T // 32
    total_pages = B * max_pages
    tables = rng.permutation(total_pages).reshape(B, max_pages).astype(np.uint16)
    prompts = rng.integers(0, vocab, (B, T))
    dims = q3.model.Dims(layers=layers, vocab=vocab, max_seq=T)
    bm = q3.model.BlobModel(dims).load_weights(w)
    kw = 8 * 128
    d = {"pk": torch.zeros((layers, total_pages, 32, kw), dtype=torch.int8, device="cuda"),
         "pv": torch.zeros((layers, total_pages, 32, kw), dtype=torch.int8, device="cuda"),
         "pks": torch.zeros((layers, total_pages, 32, 8), dtype=torch.float32, device="cuda"),
         "pvs": torch.zeros((layers, total_pages, 32, 8), dtype=torch.float32, device="cuda")}
    pool = q3._lib.KVPool(d["pk"].data_ptr(), d["pv"].data_ptr(), d["pks"].data_ptr(),
                          d["pvs"].data_ptr(), total_pages * 32 * kw, total_pages * 32 * 8 * 4,
                          total_pages)
    tab = torch.from_numpy(tables.view(np.int16)).cuda()
    ids_d = torch.from_numpy(prompts.astype(np.int32).reshape(-1)).cuda()
    nxt = torch.full((B,), -1, dtype=torch.int32, device="cuda")
    lib = q3._lib.lib()
    wsb = lib.q3_prefill_workspace_bytes(C.byref(bm.L), B, T)
    ws = torch.zeros(wsb, dtype=torch.uint8, device="cuda")
    q3._lib.check("q3_prefill_batch", lib.q3_prefill_batch(
        bm.blob.data_ptr(), C.byref(bm.L), C.byref(pool), tab.data_ptr(), max_pages,
        ids_d.data_ptr(), B, T, nxt.data_ptr(), ws.data_ptr(), wsb,
        torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert lib.q3_device_status() == 0
    got_x = ws[:B * T * 1024 * 4].cpu().numpy().view(F).reshape(B, T, 1024)
    got = {k: v.cpu().numpy() for k, v in d.items()}
    got_ids = nxt.cpu().numpy()
    edges = [0, 1, 31, 32, 33, 127, 128, 1023, 1024, 2047, 2048, 2049, 3071, 4063, 4064, 4094]
    for s in range(B):
        rows = sorted(set(edges) | set(int(v) for v in rng.integers(0, T - 1, 64))) + [T - 1]
        (k8, ks, v8, vs), xr, logits = O.forward_prompt_rows(w, prompts[s], rows)
        t = np.arange(T)
        pages = tables[s, t // 32]
        assert np.array_equal(got["pk"][0, pages, t % 32], k8), f"K of prompt {s}"
        assert np.array_equal(got["pv"][0, pages, t % 32], v8), f"V of prompt {s}"
        same_bits(got["pks"][0, pages, t % 32], ks, f"K scales of prompt {s}")
        same_bits(got["pvs"][0, pages, t % 32], vs, f"V scales of prompt {s}")
        same_bits(got_x[s, rows], xr, f"x rows of prompt {s}")
        assert int(got_ids[s]) == O.argmax_logits(logits), f"next id of prompt {s}"
