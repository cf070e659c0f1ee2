"""Tensor-parallel decomposition, checked on the CPU against the oracle.

The shard plan comes from the library's host-only ``q3_tp_shard_of`` (the plan
the GPU path runs); the sharded arithmetic is the oracle's, split the way the
device splits it:

* Q/K/V GEMMs, head norm/rope/quant, the KV cache and attention: by KV head;
* O and down: each rank computes the dequantised partials of its own K groups,
  every rank receives all of them and adds them in group order (the order of
  ``ref_qwen3.py:151-157``), then the residual;
* gate/up + SwiGLU + quant: by 256-wide group; lm_head: by vocabulary rows,
  with a (value, first index) exchange.

Greedy ids and the residual stream must be bit-identical to the single-process
oracle.  Ranks are emulated as threads for world 1..8 (uneven MLP split at 8),
and run as two ``gloo`` processes for the process-group path.
"""

from __future__ import annotations

import socket
import threading

import numpy as np
import pytest

from oracle import q3_oracle as O
from oracle import synth

F = np.float32
SHAPE = synth.Shape(layers=2, vocab=1024, max_seq=64)


def _layout():
    import q3b200.model as M
    L, _ = M.layout(M.Dims(layers=SHAPE.layers, vocab=SHAPE.vocab, max_seq=SHAPE.max_seq))
    return L


def _shards(world):
    from q3b200 import tp
    L = _layout()
    return [tp.shard_of(L, r, world) for r in range(world)]


# ---------------------------------------------------------------------------
# the sharded forward (one rank)
# ---------------------------------------------------------------------------
def _partials(a8, a_s, w8, w_s, group):
    """Dequantised per-group partials [G][rows][n] (the terms of gemm_group)."""
    parts = O.group_partials(np.asarray(a8), np.asarray(w8), group)
    out = np.empty(parts.shape, F)
    for g in range(parts.shape[0]):
        pf = (parts[g].astype(F) * np.asarray(w_s, F)[None, :]).astype(F)
        out[g] = (pf * np.asarray(a_s, F)[:, g][:, None]).astype(F)
    return out


def _add_in_order(x, groups):
    acc = np.zeros_like(x)
    for p in groups:
        acc = (acc + p).astype(F)
    return (x + acc).astype(F)


def _key(v):
    bits = int(np.asarray([v], F).view(np.uint32)[0])
    return (~bits) & 0xFFFFFFFF if bits & 0x80000000 else bits | 0x80000000


def tp_forward_chunk(model, sh, kv, ids, pos, rows, want_logits, gather):
    """forward_chunk of one rank; ``gather(obj)`` returns every rank's obj."""
    H, HD = model.hidden, model.head_dim
    inv_h = F(F(1.0) / F(H))
    qk_scale = F(1.0 / np.sqrt(float(HD)))
    cos, sin = model.cos[pos:pos + rows], model.sin[pos:pos + rows]
    ids = np.asarray(ids, np.int64)
    qsl = slice(sh.q_head0 * HD, (sh.q_head0 + sh.q_heads) * HD)
    ksl = slice(sh.kv_head0 * HD, (sh.kv_head0 + sh.kv_heads) * HD)
    gsl = slice(sh.mlp_group0 * 256, (sh.mlp_group0 + sh.mlp_groups) * 256)
    x = (model.emb8[ids].astype(F) * model.emb_s[ids][:, None]).astype(F)
    h = O.rmsnorm(x, model.layers[0].n1, inv_h)
    qpos = pos + np.arange(rows)
    for li, L in enumerate(model.layers):
        if li:
            h = O.rmsnorm(x, L.n1, inv_h)
        h8, hs = O.quant_groups(h, 256)
        q = O.gemm_group(h8, hs, L.wq[qsl], L.wq_s[qsl], 256)
        k = O.gemm_group(h8, hs, L.wk[ksl], L.wk_s[ksl], 256)
        v = O.gemm_group(h8, hs, L.wv[ksl], L.wv_s[ksl], 256)
        _, k8, ks = O.qk_norm_rope_quant(k, L.nk, cos, sin, sh.kv_heads, HD)
        v8, vs = O.quant_groups(v, HD)
        kv.k8[li][pos:pos + rows], kv.ks[li][pos:pos + rows] = k8, ks
        kv.v8[li][pos:pos + rows], kv.vs[li][pos:pos + rows] = v8, vs
        _, q8, qs = O.qk_norm_rope_quant(q, L.nq, cos, sin, sh.q_heads, HD)
        T = pos + rows
        attn = O.attention(q8, qs, kv.k8[li][:T], kv.ks[li][:T], kv.v8[li][:T], kv.vs[li][:T],
                           qpos, sh.q_heads, sh.kv_heads, HD, qk_scale)
        o8, os_ = O.quant_groups(attn, HD)
        # O: one 128-wide K group per head; rank order is head order
        x = _add_in_order(x, np.concatenate(gather(_partials(o8, os_, L.wo[:, qsl], L.wo_s, HD))))
        h = O.rmsnorm(x, L.n2, inv_h)
        h8, hs = O.quant_groups(h, 256)
        g = O.gemm_group(h8, hs, L.wg[gsl], L.wg_s[gsl], 256)
        u = O.gemm_group(h8, hs, L.wu[gsl], L.wu_s[gsl], 256)
        s8, ss = O.quant_groups(O.swiglu(g, u), 256)
        x = _add_in_order(x, np.concatenate(gather(_partials(s8, ss, L.wd[:, gsl], L.wd_s, 256))))
    if not want_logits:
        return x, None
    hl = O.rmsnorm(x[rows - 1:rows], model.nf, inv_h)
    h8l, hsl = O.quant_groups(hl, 256)
    vsl = slice(sh.vocab0, sh.vocab0 + sh.vocab_rows)
    lg = O.gemm_group(h8l, hsl, model.lm8[vsl], model.lm_s[vsl], 256)
    i = O.argmax_logits(lg)
    mine = (_key(lg[0, i]), -(sh.vocab0 + i))
    best = max(gather(mine))
    return x, -best[1]


def tp_generate(model, sh, ids, n_prompt, n_gen, gather):
    """The greedy loop of oracle.generate on one rank's shard."""
    kw = sh.kv_heads * model.head_dim
    n = len(model.layers)
    t = model.max_seq
    kv = O.KV([np.zeros((t, kw), np.int8) for _ in range(n)],
              [np.zeros((t, sh.kv_heads), F) for _ in range(n)],
              [np.zeros((t, kw), np.int8) for _ in range(n)],
              [np.zeros((t, sh.kv_heads), F) for _ in range(n)])
    total = n_prompt + n_gen
    ids = list(ids) + [0] * (total - len(ids))
    pos, gen, x = 0, [], None
    while pos < total:
        rows = min(model.seq, n_prompt - pos) if pos < n_prompt else 1
        want = pos + rows >= n_prompt
        x, nxt = tp_forward_chunk(model, sh, kv, ids[pos:pos + rows], pos, rows, want, gather)
        pos += rows
        if n_prompt <= pos < total:
            ids[pos] = nxt
            gen.append(nxt)
    return gen, x, kv


class _ThreadGather:
    def __init__(self, world):
        self.bar = threading.Barrier(world)
        self.slots = [None] * world

    def for_rank(self, rank):
        def gather(obj):
            self.bar.wait()
            self.slots[rank] = obj
            self.bar.wait()
            out = list(self.slots)
            self.bar.wait()
            return out
        return gather


@pytest.fixture(scope="module")
def model():
    return synth.build_model(SHAPE)


@pytest.fixture(scope="module")
def single(model):
    """The single-process oracle: 40-id prompt (32 + 8 rows), 2 greedy ids."""
    rec = {}
    kv = O.KV.empty(model)
    ids = synth.config1_ids(SHAPE.vocab)
    last, gen, _ = O.generate(model, ids, len(ids), 3, record=rec, kv=kv)
    return ids, gen, rec["x"], kv


# ---------------------------------------------------------------------------
def test_shard_plan_covers_the_model(q3):
    import q3b200.model as M
    from q3b200 import tp
    for dims in (M.Dims(), M.Dims(layers=1, vocab=1024)):
        L, _ = M.layout(dims)
        for world in (1, 2, 4, 8):
            sh = [tp.shard_of(L, r, world) for r in range(world)]
            for name, total in (("q_head", dims.heads), ("kv_head", dims.kv_heads),
                                ("mlp_group", dims.inter // 256)):
                start = 0
                for s in sh:
                    assert getattr(s, name + "0") == start
                    start += getattr(s, name + "s")
                assert start == total
            start = 0
            for s in sh:
                assert s.vocab0 == start and s.vocab_rows % 128 == 0 and s.vocab_rows > 0
                start += s.vocab_rows
            assert start == dims.vocab
            assert all(s.q_head0 == 2 * s.kv_head0 and s.q_heads == 2 * s.kv_heads for s in sh)
        # 12 MLP groups over 8 ranks: 1 or 2 each
        assert [s.mlp_groups for s in (tp.shard_of(L, r, 8) for r in range(8))] == [1, 2] * 4


def test_shard_plan_rejects_bad_worlds(q3):
    import ctypes as C
    from q3b200 import tp
    L = _layout()
    lib = tp._bind()
    out = tp._CShard()
    for rank, world in ((0, 3), (0, 16), (2, 2), (-1, 2), (0, 0)):
        assert lib.q3_tp_shard_of(C.byref(L), rank, world, C.byref(out)) == 3


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_tp_decomposition_is_exact(q3, model, single, world):
    ids, gen_ref, x_ref, kv_ref = single
    shards = _shards(world)
    tg = _ThreadGather(world)
    results = [None] * world
    errors = []

    def run(r):
        try:
            results[r] = tp_generate(model, shards[r], ids, len(ids), 3, tg.for_rank(r))
        except BaseException as e:   # noqa: BLE001 -- reported below
            errors.append(e)
            tg.bar.abort()

    threads = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    HD = model.head_dim
    for r, (gen, x, kv) in enumerate(results):
        assert gen == gen_ref
        np.testing.assert_array_equal(x.view(np.uint32), x_ref.view(np.uint32))
        ksl = slice(shards[r].kv_head0 * HD, (shards[r].kv_head0 + shards[r].kv_heads) * HD)
        hsl = slice(shards[r].kv_head0, shards[r].kv_head0 + shards[r].kv_heads)
        for li in range(len(model.layers)):
            np.testing.assert_array_equal(kv.k8[li], kv_ref.k8[li][:, ksl])
            np.testing.assert_array_equal(kv.v8[li], kv_ref.v8[li][:, ksl])
            np.testing.assert_array_equal(kv.ks[li], kv_ref.ks[li][:, hsl])
            np.testing.assert_array_equal(kv.vs[li], kv_ref.vs[li][:, hsl])


# ---------------------------------------------------------------------------
# two gloo processes
# ---------------------------------------------------------------------------
def _gloo_rank(rank, world, port, out_dir):
    import os
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo))
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import __graft_entry__ as ge
        ge.load_package()
        from q3b200 import tp
        import q3b200.model as M
        L, _ = M.layout(M.Dims(layers=SHAPE.layers, vocab=SHAPE.vocab, max_seq=SHAPE.max_seq))
        sh = tp.shard_of(L, rank, world)
        mdl = synth.build_model(SHAPE)

        def gather(obj):
            out = [None] * world
            dist.all_gather_object(out, obj)
            return out
        ids = synth.config1_ids(SHAPE.vocab)
        gen, x, _ = tp_generate(mdl, sh, ids, len(ids), 3, gather)
        np.savez(Path(out_dir) / f"rank{rank}.npz", gen=np.asarray(gen), x=x)
    finally:
        dist.destroy_process_group()


def test_tp_gloo_world2(single, tmp_path):
    import torch.multiprocessing as mp
    ids, gen_ref, x_ref, _ = single
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_gloo_rank, args=(2, port, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
        d = np.load(tmp_path / f"rank{r}.npz")
        assert d["gen"].tolist() == gen_ref
        np.testing.assert_array_equal(d["x"].view(np.uint32), x_ref.view(np.uint32))
