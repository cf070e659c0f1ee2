#!/usr/bin/env python3
"""Generate the golden fixtures in this directory by running the REFERENCE's own
numpy mirror (``tools/ref_qwen3.py``, ``tools/pqwf.py``, ``tools/convert_pqwf.py``
of mland2333/qwen3-tile-ops), imported unmodified from a checkout given on the
command line::

    python tests/golden/gen_golden.py --reference <path to the reference checkout>

Inputs are seeded and synthetic (the reference's HF weights are not available):
weights N(0, 0.02) from ``default_rng(0)`` quantised with ``pqwf.quantize_rows``;
RMSNorm weights ``1 + 0.05 N(0,1)`` from ``default_rng(2)``; RoPE tables from
``convert_pqwf.rope_tables`` with theta 1e6; ids from ``default_rng(1)``.

Two ``exp`` flavours are recorded:

* ``cr``: ``ref_qwen3.exp_f32`` is swapped (at run time, not in the source) for
  the correctly rounded float32 ``exp2`` of ``x * log2e`` — the host-independent
  target the device implements;
* ``native``: the reference exactly as shipped (numpy's float32 ``exp2``, whose
  rounding depends on the host CPU's SIMD dispatch; the CPU features are saved).

Outputs: ``ops_cr.npz``, ``model_cfg1_cr.npz``, ``model_cfg1_native.npz``,
``model_cfg3_cr.npz`` (28 layers, vocab 151936; digests + small arrays only),
``layout_default.h`` / ``layout_cfg1.h`` (``pqwf.Layout.header_text()``).
"""

from __future__ import annotations

import argparse
import hashlib
import importlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
F = np.float32


def load_reference(ref_root: Path):
    tools = ref_root / "tools"
    sys.path.insert(0, str(tools))
    ref = importlib.import_module("ref_qwen3")
    pqwf = importlib.import_module("pqwf")
    conv = importlib.import_module("convert_pqwf")
    return ref, pqwf, conv


def cr_exp_f32(x):
    sys.path.insert(0, str(REPO))
    from oracle.exp2 import exp2_cr
    log2e = np.array([0x3FB8AA3B], dtype=np.uint32).view(F)[0]
    return exp2_cr((np.asarray(x, F) * log2e).astype(F))


def build_ref_model(ref, pqwf, conv, layers, vocab, seq=32, max_seq=256):
    """Same draw order as oracle/synth.py, quantised by the reference."""
    hidden, heads, kvh, hd, inter = 1024, 16, 8, 128, 3072
    rng = np.random.default_rng(0)
    nrng = np.random.default_rng(2)

    def wq(rows, cols):
        w = (rng.standard_normal((rows, cols), dtype=F) * F(0.02)).astype(F)
        return pqwf.quantize_rows(w)

    def nw(n):
        return (F(1.0) + nrng.standard_normal(n, dtype=F) * F(0.05)).astype(F)

    emb8, emb_s = wq(vocab, hidden)
    lys = []
    for _ in range(layers):
        a = wq(heads * hd, hidden)
        b = wq(kvh * hd, hidden)
        c = wq(kvh * hd, hidden)
        d = wq(hidden, heads * hd)
        g = wq(inter, hidden)
        u = wq(inter, hidden)
        dn = wq(hidden, inter)
        lys.append(ref.LayerWeights(wq=a[0], wq_s=a[1], wk=b[0], wk_s=b[1], wv=c[0],
                                    wv_s=c[1], wo=d[0], wo_s=d[1], wg=g[0], wg_s=g[1],
                                    wu=u[0], wu_s=u[1], wd=dn[0], wd_s=dn[1],
                                    n1=nw(hidden), nq=nw(hd), nk=nw(hd), n2=nw(hidden)))
    lm8, lm_s = wq(vocab, hidden)
    nf = (F(1.0) + nrng.standard_normal(hidden, dtype=F) * F(0.05)).astype(F)
    cos_t, sin_t = conv.rope_tables(max_seq, hd, 1e6)
    model = ref.Model(hidden=hidden, layers=lys, heads=heads, kv_heads=kvh, head_dim=hd,
                      inter=inter, vocab=vocab, seq=seq, max_seq=max_seq, emb8=emb8,
                      emb_s=emb_s, lm8=lm8, lm_s=lm_s, nf=nf, cos_t=cos_t, sin_t=sin_t)
    return model


def digest(model) -> str:
    h = hashlib.sha256()
    arrs = [model.emb8, model.emb_s, model.lm8, model.lm_s, model.nf, model.cos_t, model.sin_t]
    for L in model.layers:
        arrs += [L.wq, L.wq_s, L.wk, L.wk_s, L.wv, L.wv_s, L.wo, L.wo_s, L.wg, L.wg_s,
                 L.wu, L.wu_s, L.wd, L.wd_s, L.n1, L.nq, L.nk, L.n2]
    for a in arrs:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# ---------------------------------------------------------------------------
def gen_ops(ref) -> dict:
    """Per-operator vectors (seeded + the guest tests' modular fixtures)."""
    out: dict = {}
    rng = np.random.default_rng(123)

    def i8(*shape):
        return rng.integers(-127, 128, size=shape, dtype=np.int64).astype(np.int8)

    def sc(*shape):
        return rng.uniform(1e-3, 1e-2, size=shape).astype(F)

    # gemm_nt_group (ref_qwen3.py:145-158): QKV-like g=256 and O-like g=128
    for tag, (m, k, n, g) in {"g256": (32, 1024, 256, 256), "g128": (5, 2048, 128, 128),
                              "m1": (1, 3072, 384, 256)}.items():
        a, w = i8(m, k), i8(n, k)
        a_s, w_s = sc(m, k // g), sc(n)
        out[f"gemm_{tag}_a"], out[f"gemm_{tag}_as"] = a, a_s
        out[f"gemm_{tag}_w"], out[f"gemm_{tag}_ws"] = w, w_s
        out[f"gemm_{tag}_out"] = ref.gemm_nt_group(a, a_s, w, w_s, group=g)

    # quant_rows_heads (ref_qwen3.py:86-97)
    x = rng.standard_normal((7, 1024)).astype(F) * F(3.0)
    x[2, 256:512] = 0.0                       # an all-zero group: 0/0 -> 0
    out["quant_x"] = x
    out["quant_q256"], out["quant_s256"] = ref.quant_rows_heads(x, 256)
    out["quant_q128"], out["quant_s128"] = ref.quant_rows_heads(x, 128)

    # rmsnorm_rows (ref_qwen3.py:161-177)
    x = rng.standard_normal((5, 1024)).astype(F)
    w = (1 + 0.1 * rng.standard_normal(1024)).astype(F)
    out["rms_x"], out["rms_w"] = x, w
    out["rms_out"] = ref.rmsnorm_rows(x, w, F(1.0) / F(1024))
    xh = rng.standard_normal((6, 128)).astype(F) * F(40.0)
    wh = (1 + 0.1 * rng.standard_normal(128)).astype(F)
    out["rmsh_x"], out["rmsh_w"] = xh, wh
    out["rmsh_out"] = ref.rmsnorm_rows(xh, wh, F(1.0) / F(128))

    # rope_head_hd (ref_qwen3.py:180-191)
    cos_t = rng.uniform(-1, 1, (6, 64)).astype(F)
    sin_t = rng.uniform(-1, 1, (6, 64)).astype(F)
    out["rope_cos"], out["rope_sin"] = cos_t, sin_t
    out["rope_out"] = ref.rope_head_hd(xh, cos_t, sin_t)

    # swiglu (ref_qwen3.py:194-200) — wide range to hit exp over/underflow
    g = (rng.standard_normal((4, 3072)) * 6).astype(F)
    g[0, :8] = [0.0, -0.0, 100.0, -100.0, 88.0, -88.0, 1e-30, -1e-30]
    u = rng.standard_normal((4, 3072)).astype(F)
    out["swiglu_g"], out["swiglu_u"] = g, u
    out["swiglu_out"] = ref.swiglu(g, u)

    # embedding_rmsnorm (ref_qwen3.py:292-296)
    emb8, emb_s = i8(50, 1024), sc(50)
    ids = rng.integers(0, 50, 9)
    wn = (1 + 0.1 * rng.standard_normal(1024)).astype(F)
    out["emb_t"], out["emb_s"], out["emb_ids"], out["emb_w"] = emb8, emb_s, ids.astype(np.int32), wn
    h, xx = ref.embedding_rmsnorm(emb8, emb_s, ids, wn, F(1.0) / F(1024))
    out["emb_h"], out["emb_x"] = h, xx

    # attention_heads_gqa_tokscale (ref_qwen3.py:269-289)
    cases = {"prefill40": (40, 72, 16, 8), "decode": (1, 100, 16, 8),
             "guestlike": (4, 80, 4, 2), "first32": (32, 32, 16, 8)}
    for tag, (rows, kv_len, heads, kvh) in cases.items():
        q8, k8, v8 = i8(rows, heads * 128), i8(kv_len, kvh * 128), i8(kv_len, kvh * 128)
        qs, ks, vs = sc(rows, heads), sc(kv_len, kvh), sc(kv_len, kvh)
        for nm, arr in (("q8", q8), ("k8", k8), ("v8", v8), ("qs", qs), ("ks", ks), ("vs", vs)):
            out[f"attn_{tag}_{nm}"] = arr
        out[f"attn_{tag}_out"] = ref.attention_heads_gqa_tokscale(
            q8, qs, k8, ks, v8, vs, heads, kvh, 128, True, F(1.0 / np.sqrt(128.0)))

    # argmax_logits (ref_qwen3.py:447-464), with a repeated maximum
    lg = rng.standard_normal((1, 1024)).astype(F)
    lg[0, 700] = lg[0, 300] = F(9.5)
    out["argmax_logits"] = lg
    out["argmax_idx"] = np.int64(ref.argmax_logits(lg, 1024))

    # the reference guest tests' modular fixtures (tests/guest/*.cpp)
    rows, K, N = 32, 256, 128       # group_gemm.cpp:17-55
    a = np.array([[(i * 7 + k * 3 + 1) % 7 - 3 for k in range(K)] for i in range(rows)], np.int8)
    b = np.array([[(j * 5 + k * 2 + 2) % 5 - 2 for k in range(K)] for j in range(N)], np.int8)
    out["guest_gg_a"], out["guest_gg_b"] = a, b
    out["guest_gg_out"] = ref.gemm_nt_group(a, np.ones((rows, 2), F), b, np.ones(N, F), group=128)
    sb = np.array([1.0, 0.5, 0.25, 2.0, 0.75], F)  # gate_up.cpp:48-65
    rows, K, N = 32, 512, 256
    a = np.array([[(i * 7 + k * 3 + 1) % 7 - 3 for k in range(K)] for i in range(rows)], np.int8)
    wg = np.array([[(j * 5 + k * 2 + 2) % 5 - 2 for k in range(K)] for j in range(N)], np.int8)
    wu = np.array([[(j * 3 + k * 7 + 4) % 7 - 3 for k in range(K)] for j in range(N)], np.int8)
    as_ = np.array([[sb[(i + g) % 5] for g in range(2)] for i in range(rows)], F)
    wgs = np.array([sb[j % 5] for j in range(N)], F)
    wus = np.array([sb[(j * 3) % 5] for j in range(N)], F)
    gg = ref.gemm_nt_group(a, as_, wg, wgs, group=256)
    uu = ref.gemm_nt_group(a, as_, wu, wus, group=256)
    s8, ss = ref.quant_rows_heads(ref.swiglu(gg, uu), 256)
    for nm, arr in (("a", a), ("wg", wg), ("wu", wu), ("as", as_), ("wgs", wgs), ("wus", wus),
                    ("s8", s8), ("ss", ss)):
        out[f"guest_gu_{nm}"] = arr
    sq = np.array([1.0, 0.5, 0.25, 0.75], F)     # paged_attn.cpp:8-19,44-66
    QR, KVL, HH, KH = 4, 80, 4, 2
    q = np.array([[(i * 7 + d * 3 + 1) % 7 - 3 for d in range(HH * 128)] for i in range(QR)], np.int8)
    k = np.array([[(t * 5 + d * 2 + 2) % 5 - 2 for d in range(KH * 128)] for t in range(KVL)], np.int8)
    v = np.array([[(t * 3 + d * 7 + 4) % 7 - 3 for d in range(KH * 128)] for t in range(KVL)], np.int8)
    qs = np.array([[sq[(i + h) % 4] for h in range(HH)] for i in range(QR)], F)
    ks = np.array([[sq[(t + h) % 4] for h in range(KH)] for t in range(KVL)], F)
    vs = np.array([[sq[(t * 3 + h) % 4] for h in range(KH)] for t in range(KVL)], F)
    att = ref.attention_heads_gqa_tokscale(q, qs, k, ks, v, vs, HH, KH, 128, True,
                                           F(0.08838834764831845))
    o8, os_ = ref.quant_rows_heads(att, 128)
    for nm, arr in (("q", q), ("k", k), ("v", v), ("qs", qs), ("ks", ks), ("vs", vs),
                    ("o8", o8), ("os", os_)):
        out[f"guest_pa_{nm}"] = arr
    return out


def run_model(ref, model, ids, n_prompt, n_gen, keep_chunks: bool):
    """ref.generate with per-chunk records of every chunk (last layer)."""
    caches = ref.new_caches(model)
    ids = list(ids) + [0] * (n_prompt + n_gen - len(ids))
    total = n_prompt + n_gen
    pos, gen, last, recs = 0, [], None, []
    while pos < total:
        rows = min(model.seq, n_prompt - pos) if pos < n_prompt else 1
        want = pos + rows >= n_prompt
        rec: dict = {}
        lg = ref.forward_chunk(model, np.asarray(ids[pos:pos + rows], np.int64), caches,
                               pos, rows, want, rec)
        recs.append((pos, rows, rec))
        if lg is not None:
            last = lg
        pos += rows
        if n_prompt <= pos < total:
            nxt = ref.argmax_logits(last, model.vocab)
            ids[pos] = nxt
            gen.append(nxt)
    return last, gen, ids, recs


def cpu_info() -> str:
    try:
        rt = np.show_runtime.__wrapped__ if hasattr(np.show_runtime, "__wrapped__") else None
    except Exception:
        rt = None
    from numpy._core._multiarray_umath import __cpu_features__ as feats  # type: ignore
    return json.dumps(sorted(k for k, v in feats.items() if v))


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--skip-cfg3", action="store_true")
    args = ap.parse_args()
    ref, pqwf, conv = load_reference(args.reference)
    native_exp = ref.exp_f32

    # layouts (pqwf.py:137-273)
    (HERE / "layout_default.h").write_text(pqwf.Layout().compute().header_text())
    (HERE / "layout_cfg1.h").write_text(pqwf.Layout(layers=1, vocab=1024).compute().header_text())

    ref.exp_f32 = cr_exp_f32
    np.savez_compressed(HERE / "ops_cr.npz", **gen_ops(ref))
    print("ops_cr.npz written")

    # config 1: 1 layer, vocab 1024, 40-token prompt from default_rng(1), 2 greedy tokens
    model = build_ref_model(ref, pqwf, conv, layers=1, vocab=1024)
    ids = [int(v) for v in np.random.default_rng(1).integers(0, 1024, 40)]
    for flavour in ("cr", "native"):
        ref.exp_f32 = cr_exp_f32 if flavour == "cr" else native_exp
        last, gen, all_ids, recs = run_model(ref, model, ids, 40, 2, True)
        pay = {"digest": np.array(digest(model)), "ids": np.asarray(all_ids, np.int32),
               "generated": np.asarray(gen, np.int32), "logits": last,
               "cpu": np.array(cpu_info())}
        for ci, (pos, rows, rec) in enumerate(recs):
            pay[f"c{ci}_pos"] = np.int32(pos)
            pay[f"c{ci}_rows"] = np.int32(rows)
            for key, val in rec.items():
                if key == "layer":
                    continue
                if ci == 0 and np.asarray(val).dtype == np.float32 and key not in (
                        "x", "hs", "qs", "ks", "vs", "os", "ss"):
                    continue    # keep the 32-row chunk small: int8 stages + scales + x
                pay[f"c{ci}_{key}"] = val
        np.savez_compressed(HERE / f"model_cfg1_{flavour}.npz", **pay)
        print(f"model_cfg1_{flavour}.npz: generated {gen}")

    if not args.skip_cfg3:
        ref.exp_f32 = cr_exp_f32
        model = build_ref_model(ref, pqwf, conv, layers=28, vocab=151936)
        ids = [int(v) for v in np.random.default_rng(1).integers(0, 151936, 32)]
        last, gen, all_ids, recs = run_model(ref, model, ids, 32, 6, False)
        pos, rows, rec = recs[0]
        pay = {"digest": np.array(digest(model)), "ids": np.asarray(all_ids, np.int32),
               "generated": np.asarray(gen, np.int32),
               "logits_sha": np.array(sha(last)), "logits_top": np.sort(last.reshape(-1))[-16:],
               "logits_argmax": np.int64(np.argmax(last))}
        for key in ("x", "k8", "v8", "ks", "vs", "s8", "o8"):
            src = {"k8": "kc", "v8": "vc"}.get(key, key)
            if src in rec:
                pay[f"c0_{key}_sha"] = np.array(sha(rec[src] if key not in ("k8", "v8", "ks", "vs")
                                                    else rec[src][pos:pos + rows]))
        pay["c0_x_row0"] = rec["x"][0]
        np.savez_compressed(HERE / "model_cfg3_cr.npz", **pay)
        print(f"model_cfg3_cr.npz: generated {gen}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
