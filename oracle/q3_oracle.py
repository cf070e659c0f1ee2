"""CPU oracle for the Qwen3 w8a8 forward path — TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the algorithm of the reference's numpy mirror
``tools/ref_qwen3.py`` (itself an instruction-by-instruction mirror of the
reference's ``kernels/*.h``).  It is the checker for the CUDA path: only the
tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import it, and never as the thing measured or shipped.

Every float32 operation is applied in the reference's order with one rounding
per step (numpy float32 arithmetic is IEEE single precision).  Integer dot
products are exact (float64 BLAS on int8 values, all sums far below 2^53, the
same device the reference uses in ``ref_qwen3.py:103-127``).

Parity pin: ``tests/golden/`` holds vectors produced by importing the
reference's own ``ref_qwen3.py``; ``tests/test_oracle_golden.py`` checks this
module against them bit for bit.

``exp`` mode: the reference rounds ``np.exp2`` on float32, whose result depends
on the host CPU's SIMD dispatch.  ``EXP_MODE = "cr"`` (default) uses the
correctly rounded float32 ``exp2`` (``oracle/exp2.py``), the host-independent
target the device implements; ``"numpy"`` reproduces the reference's own call.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .exp2 import exp2_cr, exp2_numpy_f32

F = np.float32
# ref_qwen3.py:18-21
LOG2E = np.array([0x3FB8AA3B], dtype=np.uint32).view(F)[0]
INV127 = F(F(1.0) / F(127.0))
EPS = F(1e-6)
NEG_FLT_MAX = F(-3.402823466e38)

EXP_MODE = "cr"


def _exp2(x: np.ndarray) -> np.ndarray:
    return exp2_cr(x) if EXP_MODE == "cr" else exp2_numpy_f32(x)


def exp_f32(x: np.ndarray) -> np.ndarray:
    """``exp`` as ``exp2(f32(x * log2e))`` — ref_qwen3.py:27-29."""
    return _exp2((np.asarray(x, F) * LOG2E).astype(F))


# ---------------------------------------------------------------------------
# reductions: the ISA's adjacent-pair tree (ref_qwen3.py:41-63).  Padding the
# reduced axis with the operation's identity up to a power of two gives the
# same tree as the reference's "carry the odd element" rule.
# ---------------------------------------------------------------------------
def _tree(v: np.ndarray, identity: float, op) -> np.ndarray:
    v = np.asarray(v, F)
    n = v.shape[-1]
    width = 1
    while width < n:
        width *= 2
    if width != n:
        pad = np.full(v.shape[:-1] + (width - n,), identity, dtype=F)
        v = np.concatenate([v, pad], axis=-1)
    while v.shape[-1] > 1:
        v = op(v[..., 0::2], v[..., 1::2]).astype(F)
    return v[..., 0]


def tree_sum(v: np.ndarray) -> np.ndarray:
    return _tree(v, 0.0, lambda a, b: a + b)


def tree_max(v: np.ndarray) -> np.ndarray:
    return _tree(v, -np.inf, lambda a, b: np.where(b > a, b, a))


# ---------------------------------------------------------------------------
# quantisation (ref_qwen3.py:69-97)
# ---------------------------------------------------------------------------
def quant_with_scale(x: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """rne(x / scale) saturated to +-127, NaN quotient -> 0 (ref_qwen3.py:69-76).

    ``scale`` broadcasts against ``x`` with one value per leading index.
    """
    with np.errstate(invalid="ignore", divide="ignore"):
        quot = (np.asarray(x, F) / np.asarray(scale, F)[..., None]).astype(F)
    q = np.rint(quot)
    q = np.where(np.isnan(quot), F(0.0), q)
    return np.clip(q, -127.0, 127.0).astype(np.int8)


def quant_groups(x: np.ndarray, group: int) -> tuple[np.ndarray, np.ndarray]:
    """Per-row, per-``group`` column int8 quantisation (ref_qwen3.py:86-97)."""
    x = np.asarray(x, F)
    rows, cols = x.shape
    xg = x.reshape(rows, cols // group, group)
    scale = (np.max(np.abs(xg), axis=2).astype(F) * INV127).astype(F)
    q = quant_with_scale(xg, scale)
    return q.reshape(rows, cols), scale


# ---------------------------------------------------------------------------
# GEMM: per-K-group int32 partial, (f32(part)*w_scale)*a_scale, f32 sum over
# groups in order (ref_qwen3.py:145-158)
# ---------------------------------------------------------------------------
def int_dot_nt(a8: np.ndarray, b8: np.ndarray) -> np.ndarray:
    """Exact int32 ``a8 @ b8.T`` for int8 operands (batched on leading dims).

    With an inner dimension of at most 1024, every partial sum is an integer
    of magnitude <= 1024 * 128^2 = 2^24, exact in float32 whatever order
    (or fused multiply-adds) the BLAS uses; longer dots go through float64
    (exact below 2^53)."""
    ft = np.float32 if a8.shape[-1] <= 1024 else np.float64
    out = np.matmul(a8.astype(ft), np.swapaxes(b8.astype(ft), -1, -2))
    return out.astype(np.int32)


def group_partials(a8: np.ndarray, w8: np.ndarray, group: int, chunk: int = 8192) -> np.ndarray:
    """int32 partials [G, rows, n] of every K-group."""
    rows, k = a8.shape
    n = w8.shape[0]
    g = k // group
    ag = a8.reshape(rows, g, group).transpose(1, 0, 2)
    out = np.empty((g, rows, n), dtype=np.int32)
    for n0 in range(0, n, chunk):
        n1 = min(n, n0 + chunk)
        wg = w8[n0:n1].reshape(n1 - n0, g, group).transpose(1, 0, 2)
        out[:, :, n0:n1] = int_dot_nt(ag, wg)
    return out


def gemm_group(a8, a_scale, w8, w_scale, group: int) -> np.ndarray:
    parts = group_partials(np.asarray(a8), np.asarray(w8), group)
    w_scale = np.asarray(w_scale, F)
    a_scale = np.asarray(a_scale, F)
    out = np.zeros(parts.shape[1:], dtype=F)
    for g in range(parts.shape[0]):
        pf = (parts[g].astype(F) * w_scale[None, :]).astype(F)
        pf = (pf * a_scale[:, g][:, None]).astype(F)
        out = (out + pf).astype(F)
    return out


# ---------------------------------------------------------------------------
# RMSNorm: sum of squares as a tree per 32-column block, blocks summed in
# order; (ss*inv)+eps; 1/sqrt; x*r then *w (ref_qwen3.py:161-177)
# ---------------------------------------------------------------------------
def rmsnorm(x: np.ndarray, w: np.ndarray, inv) -> np.ndarray:
    x = np.asarray(x, F)
    rows, cols = x.shape
    nblk = (cols + 31) // 32
    sq = (x * x).astype(F)
    if nblk * 32 != cols:
        sq = np.concatenate([sq, np.zeros((rows, nblk * 32 - cols), F)], axis=1)
    blk = tree_sum(sq.reshape(rows, nblk, 32))
    ss = np.zeros(rows, F)
    for b in range(nblk):
        ss = (ss + blk[:, b]).astype(F)
    ss = (ss * F(inv)).astype(F)
    ss = (ss + EPS).astype(F)
    r = (F(1.0) / np.sqrt(ss)).astype(F)
    out = (x * r[:, None]).astype(F)
    return (out * np.asarray(w, F)[None, :]).astype(F)


def rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Rotate-half RoPE with separately rounded products (ref_qwen3.py:180-191)."""
    half = x.shape[-1] // 2
    lft, rgt = x[..., :half], x[..., half:]
    out_l = ((lft * cos).astype(F) - (rgt * sin).astype(F)).astype(F)
    out_r = ((lft * sin).astype(F) + (rgt * cos).astype(F)).astype(F)
    return np.concatenate([out_l, out_r], axis=-1)


def swiglu(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """silu(g)*u as -g -> exp -> +1 -> 1/x -> g*e -> *u (ref_qwen3.py:194-200)."""
    e = exp_f32((gate * F(-1.0)).astype(F))
    e = (e + F(1.0)).astype(F)
    e = (F(1.0) / e).astype(F)
    return ((gate * e).astype(F) * up).astype(F)


# ---------------------------------------------------------------------------
# attention: GQA over 32-key blocks, online softmax, P requantised per block
# (ref_qwen3.py:210-289).  Rows are independent: a row at absolute position p
# sees keys 0..p; blocks beyond a row's horizon are exact no-ops for it, so all
# heads and rows are processed together here.
# ---------------------------------------------------------------------------
def attention(q8, q_scale, k8, k_scale, v8, v_scale, qpos, heads: int,
              kv_heads: int, hd: int, qk_scale) -> np.ndarray:
    """q8 [R, heads*hd] i8, q_scale [R, heads]; k8/v8 [T, kv_heads*hd] i8,
    k_scale/v_scale [T, kv_heads]; qpos [R] absolute position of each row.
    Returns f32 [R, heads*hd] (before the output quantisation)."""
    qk_scale = F(qk_scale)
    R = q8.shape[0]
    T = k8.shape[0]
    grp = heads // kv_heads
    kvh = np.arange(heads) // grp
    q = np.asarray(q8).reshape(R, heads, hd).transpose(1, 0, 2)       # [H,R,hd]
    qs = np.asarray(q_scale, F).T                                       # [H,R]
    k = np.asarray(k8).reshape(T, kv_heads, hd)
    v = np.asarray(v8).reshape(T, kv_heads, hd)
    ks = np.asarray(k_scale, F)
    vs = np.asarray(v_scale, F)
    qpos = np.asarray(qpos, np.int64)

    mx = np.full((heads, R), NEG_FLT_MAX, F)
    den = np.zeros((heads, R), F)
    res = np.zeros((heads, R, hd), F)
    kv_end = min(T, int(qpos.max()) + 1) if R else 0
    for j in range(0, kv_end, 32):
        nc = min(32, T - j)
        kb = k[j:j + nc][:, kvh, :].transpose(1, 0, 2)                  # [H,nc,hd]
        s = int_dot_nt(q, kb).astype(F)                                 # [H,R,nc]
        s = (s * ks[j:j + nc][:, kvh].T[:, None, :]).astype(F)
        s = (s * qs[:, :, None]).astype(F)
        s = (s * qk_scale).astype(F)
        keep = (j + np.arange(nc))[None, :] <= qpos[:, None]            # [R,nc]
        s = np.where(keep[None], s, F(-np.inf)).astype(F)
        nmm = np.maximum(tree_max(s), mx).astype(F)
        corr = exp_f32((mx - nmm).astype(F))
        den = (den * corr).astype(F)
        res = (res * corr[:, :, None]).astype(F)
        p = exp_f32((s - nmm[:, :, None]).astype(F))
        den = (den + tree_sum(p)).astype(F)
        mx = nmm
        p = (p * vs[j:j + nc][:, kvh].T[:, None, :]).astype(F)
        pmax = (tree_max(np.abs(p).astype(F)) * INV127).astype(F)
        pq = quant_with_scale(p, pmax)                                  # [H,R,nc]
        vb = v[j:j + nc][:, kvh, :].transpose(1, 2, 0)                  # [H,hd,nc]
        part = int_dot_nt(pq, vb).astype(F)                             # [H,R,hd]
        part = (part * pmax[:, :, None]).astype(F)
        res = (res + part).astype(F)
    with np.errstate(divide="ignore"):
        rden = (F(1.0) / den).astype(F)
    out = (res * rden[:, :, None]).astype(F)
    return out.transpose(1, 0, 2).reshape(R, heads * hd)


def argmax_logits(logits: np.ndarray) -> int:
    """Greedy pick over 32-column blocks with the monotone f32 key
    (ref_qwen3.py:447-464 / main_big.cpp:300-322)."""
    row = np.asarray(logits, F).reshape(-1)
    best, best_key = 0, None
    for n in range(0, row.size, 32):
        blk = row[n:n + 32]
        i = int(np.argmax(blk))
        bits = int(blk[i:i + 1].view(np.uint32)[0])
        key = (~bits) & 0xFFFFFFFF if bits & 0x80000000 else bits | 0x80000000
        if best_key is None or key > best_key:
            best_key, best = key, n + i
    return best


# ---------------------------------------------------------------------------
# model
# ---------------------------------------------------------------------------
@dataclass
class Layer:
    wq: np.ndarray
    wq_s: np.ndarray
    wk: np.ndarray
    wk_s: np.ndarray
    wv: np.ndarray
    wv_s: np.ndarray
    wo: np.ndarray
    wo_s: np.ndarray
    wg: np.ndarray
    wg_s: np.ndarray
    wu: np.ndarray
    wu_s: np.ndarray
    wd: np.ndarray
    wd_s: np.ndarray
    n1: np.ndarray
    nq: np.ndarray
    nk: np.ndarray
    n2: np.ndarray


@dataclass
class Model:
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    inter: int
    vocab: int
    seq: int
    max_seq: int
    emb8: np.ndarray
    emb_s: np.ndarray
    lm8: np.ndarray
    lm_s: np.ndarray
    nf: np.ndarray
    cos: np.ndarray
    sin: np.ndarray
    layers: list = field(default_factory=list)


@dataclass
class KV:
    """One sequence's contiguous int8 KV cache for every layer."""
    k8: list
    ks: list
    v8: list
    vs: list

    @classmethod
    def empty(cls, model: Model, max_seq: int | None = None) -> "KV":
        t = max_seq or model.max_seq
        kw = model.kv_heads * model.head_dim
        n = len(model.layers)
        return cls([np.zeros((t, kw), np.int8) for _ in range(n)],
                   [np.zeros((t, model.kv_heads), F) for _ in range(n)],
                   [np.zeros((t, kw), np.int8) for _ in range(n)],
                   [np.zeros((t, model.kv_heads), F) for _ in range(n)])


def qk_norm_rope_quant(x, w, cos, sin, heads, hd):
    """Per-head RMSNorm(hd) * w, rotate-half RoPE, per-head int8 quant
    (ref_qwen3.py:393-409; device: kernels/norm_rope_quant.h:17-86)."""
    rows = x.shape[0]
    inv_hd = F(F(1.0) / F(hd))
    xh = x.reshape(rows * heads, hd)
    y = rmsnorm(xh, w, inv_hd).reshape(rows, heads, hd)
    y = rope(y, cos[:, None, :], sin[:, None, :]).reshape(rows, heads * hd)
    q8, qs = quant_groups(y, hd)
    return y, q8, qs


def forward_chunk(model: Model, ids, kv: KV, pos: int, rows: int,
                  want_logits: bool, record: dict | None = None):
    """One prefill chunk or decode step (ref_qwen3.py:366-444)."""
    H, HD = model.hidden, model.head_dim
    inv_h = F(F(1.0) / F(H))
    qk_scale = F(1.0 / np.sqrt(float(HD)))
    cos = model.cos[pos:pos + rows]
    sin = model.sin[pos:pos + rows]
    ids = np.asarray(ids, np.int64)
    x = (model.emb8[ids].astype(F) * model.emb_s[ids][:, None]).astype(F)
    h = rmsnorm(x, model.layers[0].n1, inv_h)
    qpos = pos + np.arange(rows)
    for li, L in enumerate(model.layers):
        if li:
            h = rmsnorm(x, L.n1, inv_h)
        h8, hs = quant_groups(h, 256)
        q = gemm_group(h8, hs, L.wq, L.wq_s, 256)
        k = gemm_group(h8, hs, L.wk, L.wk_s, 256)
        v = gemm_group(h8, hs, L.wv, L.wv_s, 256)
        k, k8, ks = qk_norm_rope_quant(k, L.nk, cos, sin, model.kv_heads, HD)
        v8, vs = quant_groups(v, HD)
        kv.k8[li][pos:pos + rows] = k8
        kv.ks[li][pos:pos + rows] = ks
        kv.v8[li][pos:pos + rows] = v8
        kv.vs[li][pos:pos + rows] = vs
        q, q8, qs = qk_norm_rope_quant(q, L.nq, cos, sin, model.heads, HD)
        T = pos + rows
        attn = attention(q8, qs, kv.k8[li][:T], kv.ks[li][:T], kv.v8[li][:T],
                         kv.vs[li][:T], qpos, model.heads, model.kv_heads, HD, qk_scale)
        o8, os_ = quant_groups(attn, HD)
        o = gemm_group(o8, os_, L.wo, L.wo_s, HD)
        x = (x + o).astype(F)
        h = rmsnorm(x, L.n2, inv_h)
        h8, hs = quant_groups(h, 256)
        g = gemm_group(h8, hs, L.wg, L.wg_s, 256)
        u = gemm_group(h8, hs, L.wu, L.wu_s, 256)
        sw = swiglu(g, u)
        s8, ss = quant_groups(sw, 256)
        o = gemm_group(s8, ss, L.wd, L.wd_s, 256)
        x = (x + o).astype(F)
        if record is not None:
            record.clear()
            record.update(dict(h=h, h8=h8, hs=hs, q=q, k=k, v=v, q8=q8, qs=qs,
                               k8=k8, ks=ks, v8=v8, vs=vs, attn=attn, o8=o8,
                               os=os_, o=o, g=g, u=u, sw=sw, s8=s8, ss=ss, x=x,
                               layer=li))
    logits = None
    if want_logits:
        hl = rmsnorm(x[rows - 1:rows], model.nf, inv_h)
        h8l, hsl = quant_groups(hl, 256)
        logits = gemm_group(h8l, hsl, model.lm8, model.lm_s, 256)
        if record is not None:
            record["logits"] = logits
    return logits


def forward_prompt_rows(w: Model, ids, rows):
    """forward_chunk of a one-layer model over a whole T-token prompt as one
    chunk (ref_qwen3.py:366-444), evaluated past the K/V write only for the
    prompt rows ``rows``: rows interact only through attention, which reads
    the K/V of every row, so each selected row gets exactly its bits of the
    full computation.  Returns (k8, ks, v8, vs) of every row, x of the
    selected rows, and the logits of the last selected row."""
    assert len(w.layers) == 1, "later layers need the x of every row"
    L = w.layers[0]
    H, HD = w.hidden, w.head_dim
    T = len(ids)
    inv_h = F(F(1.0) / F(H))
    qk_scale = F(1.0 / np.sqrt(float(HD)))
    ids = np.asarray(ids, np.int64)
    x = (w.emb8[ids].astype(F) * w.emb_s[ids][:, None]).astype(F)
    h = rmsnorm(x, L.n1, inv_h)
    h8, hs = quant_groups(h, 256)
    k = gemm_group(h8, hs, L.wk, L.wk_s, 256)
    v = gemm_group(h8, hs, L.wv, L.wv_s, 256)
    _, k8, ks = qk_norm_rope_quant(k, L.nk, w.cos[:T], w.sin[:T], w.kv_heads, HD)
    v8, vs = quant_groups(v, HD)
    r = np.asarray(rows)
    q = gemm_group(h8[r], hs[r], L.wq, L.wq_s, 256)
    _, q8, qs = qk_norm_rope_quant(q, L.nq, w.cos[r], w.sin[r], w.heads, HD)
    attn = attention(q8, qs, k8, ks, v8, vs, r, w.heads, w.kv_heads, HD, qk_scale)
    o8, os_ = quant_groups(attn, HD)
    xr = (x[r] + gemm_group(o8, os_, L.wo, L.wo_s, HD)).astype(F)
    h = rmsnorm(xr, L.n2, inv_h)
    h8, hs = quant_groups(h, 256)
    sw = swiglu(gemm_group(h8, hs, L.wg, L.wg_s, 256), gemm_group(h8, hs, L.wu, L.wu_s, 256))
    s8, ss = quant_groups(sw, 256)
    xr = (xr + gemm_group(s8, ss, L.wd, L.wd_s, 256)).astype(F)
    hl = rmsnorm(xr[-1:], w.nf, inv_h)
    h8l, hsl = quant_groups(hl, 256)
    return (k8, ks, v8, vs), xr, gemm_group(h8l, hsl, w.lm8, w.lm_s, 256)


def generate(model: Model, ids, n_prompt: int, n_gen: int, record: dict | None = None,
             kv: KV | None = None):
    """Greedy loop with the reference's chunking (ref_qwen3.py:467-490,
    main_big.cpp:332-369): prompt in ``model.seq``-row chunks, then one row per
    step; the id picked after each chunk that reaches the prompt end is written
    to the next slot."""
    kv = kv or KV.empty(model)
    total = n_prompt + n_gen
    ids = list(ids) + [0] * (total - len(ids))
    pos, gen, last = 0, [], None
    while pos < total:
        rows = min(model.seq, n_prompt - pos) if pos < n_prompt else 1
        want = pos + rows >= n_prompt
        logits = forward_chunk(model, ids[pos:pos + rows], kv, pos, rows, want,
                               record if (record is not None and want) else None)
        if logits is not None:
            last = logits
        pos += rows
        if n_prompt <= pos < total:
            nxt = argmax_logits(last)
            ids[pos] = nxt
            gen.append(nxt)
    return last, gen, ids
