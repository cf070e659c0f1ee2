"""Seeded random-init Qwen3-shaped w8a8 weights and KV prefixes, generated on
the device (the reference's HF weights are not available).

Weights follow the random-init recipe of the benchmarks: N(0, 0.02) float32 per matrix,
quantised per output row with the path's own quantiser
(``q3_quant_rows_heads`` with one group per row == ``tools/pqwf.py:72-89``);
RMSNorm weights ``1 + 0.05 N(0,1)``; RoPE tables as
``tools/convert_pqwf.py:46-52`` (theta 1e6).  The values differ from the numpy
stream the tests use, the distribution does not.
"""

from __future__ import annotations

import numpy as np
import torch

from . import ops
from .model import BlobModel, Dims
from .ops import MatrixView


def _rope(max_seq: int, head_dim: int, theta: float = 1e6):
    half = head_dim // 2
    inv = 1.0 / (float(theta) ** (np.arange(half, dtype=np.float64) / float(half)))
    ang = np.arange(max_seq, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def _quant_into(bm: BlobModel, gen: torch.Generator, q_off: int, s_off: int, rows: int,
                cols: int, chunk: int = 16384) -> None:
    base = bm.blob.data_ptr()
    for r0 in range(0, rows, chunk):
        n = min(chunk, rows - r0)
        w = torch.randn((n, cols), generator=gen, device=bm.device, dtype=torch.float32) * 0.02
        q = MatrixView(base + q_off + r0 * cols, cols, 1, n, cols, 0, bm.blob)
        s = MatrixView(base + s_off + r0 * 4, 4, 4, n, 1, 4, bm.blob)
        ops.quant_rows_heads(w, q, s, cols)
    torch.cuda.synchronize(bm.device)


def random_blob_model(dims: Dims, seed: int = 0, device="cuda") -> BlobModel:
    bm = BlobModel(dims, device)
    gen = torch.Generator(device=bm.device)
    gen.manual_seed(seed)
    o, d = bm.off, dims
    V, H, HD, I = d.vocab, d.hidden, d.head_dim, d.inter
    QW, KW = d.heads * HD, d.kv_heads * HD
    _quant_into(bm, gen, o["kEMB"], o["kEMB"] + V * H, V, H)
    for li in range(d.layers):
        base = o["kLQ"] + li * o["kLAYERW_STRIDE"]
        for key, skey, rows, cols in (("kLQ", "kLQ_SCALE", QW, H), ("kLK", "kLK_SCALE", KW, H),
                                      ("kLV", "kLV_SCALE", KW, H), ("kLO", "kLO_SCALE", H, QW),
                                      ("kLG", "kLG_SCALE", I, H), ("kLU", "kLU_SCALE", I, H),
                                      ("kLD", "kLD_SCALE", H, I)):
            _quant_into(bm, gen, base + (o[key] - o["kLQ"]), base + (o[skey] - o["kLQ"]), rows, cols)
        nb = o["kN1"] + li * o["kLAYERN_STRIDE"]
        for key, n in (("kN1", H), ("kNQ", HD), ("kNK", HD), ("kN2", H)):
            nw = 1.0 + 0.05 * torch.randn(n, generator=gen, device=bm.device)
            off = nb + (o[key] - o["kN1"])
            bm.blob[off:off + 4 * n].copy_(nw.float().view(torch.uint8))
    _quant_into(bm, gen, o["kLM"], o["kLM"] + V * H, V, H)
    nf = 1.0 + 0.05 * torch.randn(H, generator=gen, device=bm.device)
    bm.blob[o["kNF"]:o["kNF"] + 4 * H].copy_(nf.float().view(torch.uint8))
    cos, sin = _rope(d.max_seq, HD)
    bm.put(o["kCOS"], cos)
    bm.put(o["kSIN"], sin)
    torch.cuda.synchronize(bm.device)
    return bm


class KVPoolTensors:
    """A page pool [layers][pages][32][kv_heads*128] (K, V) + f32 scales."""

    def __init__(self, layers: int, pages: int, kv_heads: int, device="cuda"):
        kw = kv_heads * 128
        self.layers, self.pages, self.kv_heads = layers, pages, kv_heads
        self.k = torch.zeros((layers, pages, 32, kw), dtype=torch.int8, device=device)
        self.v = torch.zeros_like(self.k)
        self.ks = torch.zeros((layers, pages, 32, kv_heads), dtype=torch.float32, device=device)
        self.vs = torch.zeros_like(self.ks)

    def fill_random(self, seed: int = 1, head0: int = 0, total_heads: int | None = None) -> None:
        """Seeded int8 K/V uniform in [-127, 127] and scales U[1e-3, 1e-2].

        With ``total_heads``, this pool holds KV heads ``head0 ..`` of a pool of
        ``total_heads`` heads filled with the same seed (a tensor-parallel
        rank's share): the values are drawn at full width and sliced."""
        total = total_heads or self.kv_heads
        c0, c1 = head0 * 128, (head0 + self.kv_heads) * 128
        g = torch.Generator(device=self.k.device)
        g.manual_seed(seed)
        for t in (self.k, self.v):
            for layer in t:              # per layer: bounded temporary memory
                full = torch.randint(-127, 128, (self.pages, 32, total * 128), generator=g,
                                     device=t.device, dtype=torch.int16)
                layer.copy_(full[..., c0:c1].to(torch.int8))
                del full
        for t in (self.ks, self.vs):
            full = torch.empty((self.layers, self.pages, 32, total), device=t.device)
            full.uniform_(1e-3, 1e-2, generator=g)
            t.copy_(full[..., head0:head0 + self.kv_heads])
            del full

    def c(self):
        from ._lib import KVPool
        return KVPool(self.k.data_ptr(), self.v.data_ptr(), self.ks.data_ptr(), self.vs.data_ptr(),
                      self.k[0].numel(), self.ks[0].numel() * 4, self.pages)

    def bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.k, self.v, self.ks, self.vs))
