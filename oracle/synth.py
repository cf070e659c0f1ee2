"""Seeded synthetic Qwen3-shaped w8a8 models for the oracle and the tests.

TEST INFRASTRUCTURE.  The reference's weights come from HF safetensors that are
absent here; the configs use random-init weights instead:

* every weight matrix is N(0, 0.02) float32 from ``numpy.random.default_rng(0)``
  drawn in a fixed order (embedding, then per layer q k v o gate up down, then
  lm_head), quantised per output row as ``tools/pqwf.py:72-89`` does
  (``scale = absmax * (1/127)``, ``rne(x/scale)`` saturated to +-127);
* RMSNorm weights (unspecified by the configs) are ``1 + 0.05 * N(0,1)`` from
  ``default_rng(2)`` so that the ``* w`` step is exercised, not a no-op;
* RoPE tables follow ``tools/convert_pqwf.py:46-52`` with theta = 1e6:
  float64 angles ``pos * theta^(-i/half)``, cos/sin rounded to float32.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .q3_oracle import F, INV127, Layer, Model


@dataclass
class Shape:
    hidden: int = 1024
    layers: int = 28
    heads: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    inter: int = 3072
    vocab: int = 151936
    seq: int = 32
    max_seq: int = 256


def quantize_rows(m: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Per-output-row symmetric int8 quantisation (tools/pqwf.py:72-89)."""
    m = np.asarray(m, F)
    scale = (np.max(np.abs(m), axis=1).astype(F) * INV127).astype(F)
    with np.errstate(invalid="ignore", divide="ignore"):
        quot = (m / scale[:, None]).astype(F)
    q = np.rint(quot)
    q = np.where(np.isnan(quot), F(0.0), q)
    return np.clip(q, -127, 127).astype(np.int8), scale


def rope_tables(max_seq: int, head_dim: int, theta: float = 1e6):
    """float32 cos/sin tables [max_seq][head_dim/2] (convert_pqwf.py:46-52)."""
    half = head_dim // 2
    inv_freq = 1.0 / (float(theta) ** (np.arange(half, dtype=np.float64) / float(half)))
    ang = np.arange(max_seq, dtype=np.float64)[:, None] * inv_freq[None, :]
    return np.cos(ang).astype(F), np.sin(ang).astype(F)


def _normal_q(rng, rows, cols):
    w = (rng.standard_normal((rows, cols), dtype=F) * F(0.02)).astype(F)
    return quantize_rows(w)


def build_model(shape: Shape, seed: int = 0) -> Model:
    """The seeded random-init model of the parity and benchmark cases (shape-dependent)."""
    s = shape
    rng = np.random.default_rng(seed)
    nrng = np.random.default_rng(seed + 2)
    qw, kw = s.heads * s.head_dim, s.kv_heads * s.head_dim
    emb8, emb_s = _normal_q(rng, s.vocab, s.hidden)
    layers = []
    for _ in range(s.layers):
        wq, wq_s = _normal_q(rng, qw, s.hidden)
        wk, wk_s = _normal_q(rng, kw, s.hidden)
        wv, wv_s = _normal_q(rng, kw, s.hidden)
        wo, wo_s = _normal_q(rng, s.hidden, qw)
        wg, wg_s = _normal_q(rng, s.inter, s.hidden)
        wu, wu_s = _normal_q(rng, s.inter, s.hidden)
        wd, wd_s = _normal_q(rng, s.hidden, s.inter)

        def nw(n):
            return (F(1.0) + nrng.standard_normal(n, dtype=F) * F(0.05)).astype(F)

        layers.append(Layer(wq=wq, wq_s=wq_s, wk=wk, wk_s=wk_s, wv=wv, wv_s=wv_s,
                            wo=wo, wo_s=wo_s, wg=wg, wg_s=wg_s, wu=wu, wu_s=wu_s,
                            wd=wd, wd_s=wd_s, n1=nw(s.hidden), nq=nw(s.head_dim),
                            nk=nw(s.head_dim), n2=nw(s.hidden)))
    lm8, lm_s = _normal_q(rng, s.vocab, s.hidden)
    nf = (F(1.0) + nrng.standard_normal(s.hidden, dtype=F) * F(0.05)).astype(F)
    cos, sin = rope_tables(s.max_seq, s.head_dim)
    return Model(hidden=s.hidden, heads=s.heads, kv_heads=s.kv_heads,
                 head_dim=s.head_dim, inter=s.inter, vocab=s.vocab, seq=s.seq,
                 max_seq=s.max_seq, emb8=emb8, emb_s=emb_s, lm8=lm8, lm_s=lm_s,
                 nf=nf, cos=cos, sin=sin, layers=layers)


def config1_ids(vocab: int = 1024, n: int = 40) -> list[int]:
    """Config 1 prompt: 40 uniform ids from ``default_rng(1)``."""
    return [int(v) for v in np.random.default_rng(1).integers(0, vocab, n)]


def weights_digest(model: Model) -> str:
    """sha256 over every tensor of the model, in a fixed order."""
    import hashlib
    h = hashlib.sha256()
    arrs = [model.emb8, model.emb_s, model.lm8, model.lm_s, model.nf, model.cos, model.sin]
    for L in model.layers:
        arrs += [L.wq, L.wq_s, L.wk, L.wk_s, L.wv, L.wv_s, L.wo, L.wo_s, L.wg, L.wg_s,
                 L.wu, L.wu_s, L.wd, L.wd_s, L.n1, L.nq, L.nk, L.n2]
    for a in arrs:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()
