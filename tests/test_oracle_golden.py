"""Pin the CPU oracle against vectors produced by the reference's own numpy
mirror (``tests/golden/gen_golden.py`` imports ``tools/ref_qwen3.py``).

Everything here is CPU-only and bit-exact (``cr`` exp flavour); the
``native`` flavour is bit-exact only on a host whose numpy SIMD dispatch equals
the one recorded in the fixture, and is otherwise held to the f32 tolerance (1e-3 relative).
"""

from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import load_golden
from oracle import q3_oracle as O
from oracle import synth

F = np.float32


def bits_equal(a, b) -> bool:
    a, b = np.asarray(a), np.asarray(b)
    if a.shape != b.shape:
        return False
    if a.dtype == np.float32:
        return np.array_equal(a.view(np.uint32), np.asarray(b, F).view(np.uint32))
    return np.array_equal(a, b)


@pytest.fixture(scope="module")
def ops():
    return load_golden("ops_cr.npz")


@pytest.mark.parametrize("tag,group", [("g256", 256), ("g128", 128), ("m1", 256)])
def test_gemm_group(ops, tag, group):
    out = O.gemm_group(ops[f"gemm_{tag}_a"], ops[f"gemm_{tag}_as"], ops[f"gemm_{tag}_w"],
                       ops[f"gemm_{tag}_ws"], group)
    assert bits_equal(out, ops[f"gemm_{tag}_out"])


@pytest.mark.parametrize("group", [256, 128])
def test_quant_groups(ops, group):
    q, s = O.quant_groups(ops["quant_x"], group)
    assert bits_equal(q, ops[f"quant_q{group}"])
    assert bits_equal(s, ops[f"quant_s{group}"])


def test_rmsnorm(ops):
    assert bits_equal(O.rmsnorm(ops["rms_x"], ops["rms_w"], F(1) / F(1024)), ops["rms_out"])
    assert bits_equal(O.rmsnorm(ops["rmsh_x"], ops["rmsh_w"], F(1) / F(128)), ops["rmsh_out"])


def test_rope(ops):
    assert bits_equal(O.rope(ops["rmsh_x"], ops["rope_cos"], ops["rope_sin"]), ops["rope_out"])


def test_swiglu(ops):
    assert bits_equal(O.swiglu(ops["swiglu_g"], ops["swiglu_u"]), ops["swiglu_out"])


def test_embedding_rmsnorm(ops):
    ids = ops["emb_ids"]
    x = (ops["emb_t"][ids].astype(F) * ops["emb_s"][ids][:, None]).astype(F)
    assert bits_equal(x, ops["emb_x"])
    assert bits_equal(O.rmsnorm(x, ops["emb_w"], F(1) / F(1024)), ops["emb_h"])


@pytest.mark.parametrize("tag,heads,kvh", [("prefill40", 16, 8), ("decode", 16, 8),
                                            ("guestlike", 4, 2), ("first32", 16, 8)])
def test_attention(ops, tag, heads, kvh):
    g = {k: ops[f"attn_{tag}_{k}"] for k in ("q8", "k8", "v8", "qs", "ks", "vs", "out")}
    rows, T = g["q8"].shape[0], g["k8"].shape[0]
    qpos = np.arange(T - rows, T)
    out = O.attention(g["q8"], g["qs"], g["k8"], g["ks"], g["v8"], g["vs"], qpos,
                      heads, kvh, 128, F(1.0 / np.sqrt(128.0)))
    assert bits_equal(out, g["out"])


def test_argmax(ops):
    assert O.argmax_logits(ops["argmax_logits"]) == int(ops["argmax_idx"]) == 300


def test_guest_fixtures(ops):
    out = O.gemm_group(ops["guest_gg_a"], np.ones((32, 2), F), ops["guest_gg_b"],
                       np.ones(128, F), 128)
    assert bits_equal(out, ops["guest_gg_out"])
    a, as_ = ops["guest_gu_a"], ops["guest_gu_as"]
    g = O.gemm_group(a, as_, ops["guest_gu_wg"], ops["guest_gu_wgs"], 256)
    u = O.gemm_group(a, as_, ops["guest_gu_wu"], ops["guest_gu_wus"], 256)
    s8, ss = O.quant_groups(O.swiglu(g, u), 256)
    assert bits_equal(s8, ops["guest_gu_s8"]) and bits_equal(ss, ops["guest_gu_ss"])
    p = {k: ops[f"guest_pa_{k}"] for k in ("q", "k", "v", "qs", "ks", "vs", "o8", "os")}
    att = O.attention(p["q"], p["qs"], p["k"], p["ks"], p["v"], p["vs"], np.arange(76, 80),
                      4, 2, 128, F(0.08838834764831845))
    o8, os_ = O.quant_groups(att, 128)
    assert bits_equal(o8, p["o8"]) and bits_equal(os_, p["os"])


# ---------------------------------------------------------------------------
# whole-model pins
# ---------------------------------------------------------------------------
STAGES = ("h", "h8", "hs", "q", "k", "v", "q8", "qs", "attn", "o8", "os", "o", "g", "u",
          "sw", "s8", "ss", "x")


def _run_cfg1(exp_mode: str):
    old = O.EXP_MODE
    O.EXP_MODE = exp_mode
    try:
        model = synth.build_model(synth.Shape(layers=1, vocab=1024))
        ids = synth.config1_ids()
        kv = O.KV.empty(model)
        recs, pos, total, n_prompt = [], 0, 42, 40
        ids = ids + [0, 0]
        while pos < total:
            rows = min(32, n_prompt - pos) if pos < n_prompt else 1
            want = pos + rows >= n_prompt
            rec: dict = {}
            lg = O.forward_chunk(model, ids[pos:pos + rows], kv, pos, rows, want, rec)
            recs.append((pos, rows, rec, lg))
            pos += rows
            if n_prompt <= pos < total:
                ids[pos] = O.argmax_logits(lg)
        return model, ids, recs, kv
    finally:
        O.EXP_MODE = old


def test_config1_model_digest():
    g = load_golden("model_cfg1_cr.npz")
    model = synth.build_model(synth.Shape(layers=1, vocab=1024))
    assert synth.weights_digest(model) == str(g["digest"])


def test_config1_cr_all_stages():
    g = load_golden("model_cfg1_cr.npz")
    model, ids, recs, kv = _run_cfg1("cr")
    assert list(ids) == [int(v) for v in g["ids"]]
    assert list(g["generated"]) == ids[40:42]
    for ci, (pos, rows, rec, lg) in enumerate(recs):
        assert int(g[f"c{ci}_pos"]) == pos and int(g[f"c{ci}_rows"]) == rows
        for st in STAGES:
            key = f"c{ci}_{st}"
            if key in g:
                assert bits_equal(rec[st], g[key]), key
        for st, ref_key in (("k8", "kc"), ("ks", "ks"), ("v8", "vc"), ("vs", "vs")):
            key = f"c{ci}_{ref_key}"
            assert bits_equal(rec[st], g[key][pos:pos + rows]), key
        if lg is not None:
            assert bits_equal(lg, g[f"c{ci}_logits"])
    assert bits_equal(recs[-1][3], g["logits"])


def test_config1_native_exp():
    g = load_golden("model_cfg1_native.npz")
    from numpy._core._multiarray_umath import __cpu_features__ as feats  # type: ignore
    here = sorted(k for k, v in feats.items() if v)
    model, ids, recs, kv = _run_cfg1("numpy")
    assert list(ids) == [int(v) for v in g["ids"]]
    lg = recs[-1][3]
    if here == json.loads(str(g["cpu"])):
        assert bits_equal(lg, g["logits"])
    else:  # different numpy exp2 dispatch: f32 tolerance
        np.testing.assert_allclose(lg, g["logits"], rtol=1e-3, atol=1e-3)


def test_config3_full_shape():
    """28 layers, vocab 151936, 32-token prompt + 6 greedy tokens (config 3)."""
    g = load_golden("model_cfg3_cr.npz")
    model = synth.build_model(synth.Shape())
    assert synth.weights_digest(model) == str(g["digest"])
    ids = [int(v) for v in np.random.default_rng(1).integers(0, 151936, 32)]
    rec: dict = {}
    last, gen, all_ids = O.generate(model, ids, 32, 6)
    assert gen == [int(v) for v in g["generated"]]
    import hashlib
    assert hashlib.sha256(np.ascontiguousarray(last).tobytes()).hexdigest() == str(g["logits_sha"])


def test_forward_prompt_rows_matches_forward_chunk():
    """The row-sampled one-layer prompt forward (used by the long-prompt GPU
    test) gives, for every selected row, the bits forward_chunk gives for that
    row when the whole prompt is one chunk: K/V of all rows, x, logits."""
    w = synth.build_model(synth.Shape(layers=1, vocab=1024, max_seq=128))
    ids = [int(v) for v in np.random.default_rng(3).integers(0, 1024, 100)]
    kv = O.KV.empty(w, 128)
    rec = {}
    lg = O.forward_chunk(w, ids, kv, 0, 100, True, rec)
    rows = [0, 5, 31, 32, 63, 64, 98, 99]
    (k8, ks, v8, vs), xr, logits = O.forward_prompt_rows(w, ids, rows)
    assert np.array_equal(k8, kv.k8[0][:100]) and np.array_equal(v8, kv.v8[0][:100])
    assert np.array_equal(ks.view(np.uint32), kv.ks[0][:100].view(np.uint32))
    assert np.array_equal(vs.view(np.uint32), kv.vs[0][:100].view(np.uint32))
    assert np.array_equal(xr.view(np.uint32), rec["x"][rows].view(np.uint32))
    assert np.array_equal(logits.view(np.uint32), lg.view(np.uint32))
