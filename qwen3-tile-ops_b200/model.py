"""Model-level host API: the pqwf blob on the device and the reference's
entry points (``forward_chunk`` / greedy generate of ``src/main_big.cpp``).

The blob layout is ``tools/pqwf.py``'s (computed by ``q3_layout_compute`` in
the library); weights are written into a device copy of it.  A weights object
is anything with the attributes ``emb8 emb_s lm8 lm_s nf cos sin layers``
(each layer: ``wq wq_s wk wk_s wv wv_s wo wo_s wg wg_s wu wu_s wd wd_s n1 nq nk
n2``) holding numpy arrays in the pqwf conventions (``[out][in]`` int8 weights,
one float32 scale per output row).
"""

from __future__ import annotations

import ctypes as C
import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from ._lib import OFF_NAMES, Layout, check, lib
from .ops import MatrixView

LM_NONE, LM_LOGITS, LM_ARGMAX = 0, 1, 2
DT = {np.dtype(np.int8): 0, np.dtype(np.float32): 4, np.dtype(np.int32): 2}


@dataclass
class Dims:
    hidden: int = 1024
    layers: int = 28
    heads: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    inter: int = 3072
    vocab: int = 151936
    seq: int = 32
    max_seq: int = 256


def layout(d: Dims) -> tuple[Layout, dict[str, int]]:
    """tools/pqwf.py:137-218 — the blob offsets of config/model_big.h."""
    L = Layout(d.hidden, d.layers, d.heads, d.kv_heads, d.head_dim, d.inter, d.vocab, d.seq,
               d.max_seq)
    check("q3_layout_compute", lib().q3_layout_compute(C.byref(L)))
    return L, {name: int(L.off[i]) for i, name in enumerate(OFF_NAMES)}


def header_text(d: Dims) -> str:
    """The generated header (pqwf.py:251-273 format)."""
    _, off = layout(d)
    consts = {"kHidden": d.hidden, "kLayers": d.layers, "kHeads": d.heads,
              "kKvHeads": d.kv_heads, "kHeadDim": d.head_dim, "kInter": d.inter,
              "kVocab": d.vocab, "kSeq": d.seq, "kMaxSeq": d.max_seq, "kHalf": d.head_dim // 2}
    order = ["kIDS", "kCTRL", "kX", "kEMB", "kLM", "kNF", "kCOS", "kSIN", "kLAYERW_BASE",
             "kLAYERW_STRIDE", "kLQ", "kLQ_SCALE", "kLK", "kLK_SCALE", "kLV", "kLV_SCALE", "kLO",
             "kLO_SCALE", "kLG", "kLG_SCALE", "kLU", "kLU_SCALE", "kLD", "kLD_SCALE",
             "kLAYERN_BASE", "kLAYERN_STRIDE", "kN1", "kNQ", "kNK", "kN2", "kLOGITS",
             "kBLOCK_END", "kH", "kH8", "kHS", "kQ", "kK", "kV", "kQ8", "kK8", "kV8", "kQS",
             "kKS", "kVS", "kATTN", "kO", "kO8", "kOS", "kG", "kU", "kSW", "kS8", "kSS", "kARGF",
             "kARGI", "kKV_BASE", "kKV_STRIDE", "kKV_VOFF", "kKV_SOFF", "kSCRATCH_END"]
    lines = ["#pragma once", "namespace mb {"]
    lines += [f"inline constexpr int {k} = {v};" for k, v in consts.items()]
    lines += [f"inline constexpr long {k} = {off[k]};" for k in order]
    lines += ["}", ""]
    return "\n".join(lines)


def safetensors_tensor(path, name: str) -> tuple[str, tuple[int, ...]]:
    """(dtype, shape) of one tensor of a safetensors header, read by the
    library's own parser (tools/pqwf.py:279-304)."""
    dt, nd = C.c_int32(), C.c_int32()
    shape = (C.c_uint64 * 4)()
    check("q3_safetensors_tensor", lib().q3_safetensors_tensor(
        str(path).encode(), name.encode(), C.byref(dt), shape, C.byref(nd)))
    return {0: "F32", 1: "BF16", 2: "F16"}.get(dt.value, "other"), tuple(shape[:nd.value])


class BlobModel:
    """A device copy of the pqwf blob plus the workspace its entry points need."""

    def __init__(self, dims: Dims, device: str | torch.device = "cuda"):
        self.dims = dims
        self.L, self.off = layout(dims)
        self.device = torch.device(device)
        self.blob = torch.zeros(self.off["kSCRATCH_END"], dtype=torch.uint8, device=self.device)
        ws = lib().q3_forward_workspace_bytes(C.byref(self.L))
        self.ws = torch.zeros(max(ws, 256), dtype=torch.uint8, device=self.device)

    # -- writing ------------------------------------------------------------
    def put(self, off: int, arr: np.ndarray) -> None:
        raw = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
        self.blob[off:off + raw.size].copy_(torch.from_numpy(raw), non_blocking=False)

    def load_weights(self, w) -> "BlobModel":
        d, o = self.dims, self.off
        V, H = d.vocab, d.hidden
        self.put(o["kEMB"], w.emb8)
        self.put(o["kEMB"] + V * H, w.emb_s)
        self.put(o["kLM"], w.lm8)
        self.put(o["kLM"] + V * H, w.lm_s)
        self.put(o["kNF"], w.nf)
        self.put(o["kCOS"], w.cos[:d.max_seq])
        self.put(o["kSIN"], w.sin[:d.max_seq])
        for i, ly in enumerate(w.layers):
            base = o["kLQ"] + i * o["kLAYERW_STRIDE"]
            for key, arr in (("kLQ", ly.wq), ("kLQ_SCALE", ly.wq_s), ("kLK", ly.wk),
                             ("kLK_SCALE", ly.wk_s), ("kLV", ly.wv), ("kLV_SCALE", ly.wv_s),
                             ("kLO", ly.wo), ("kLO_SCALE", ly.wo_s), ("kLG", ly.wg),
                             ("kLG_SCALE", ly.wg_s), ("kLU", ly.wu), ("kLU_SCALE", ly.wu_s),
                             ("kLD", ly.wd), ("kLD_SCALE", ly.wd_s)):
                self.put(base + (o[key] - o["kLQ"]), arr)
            nb = o["kN1"] + i * o["kLAYERN_STRIDE"]
            self.put(nb, ly.n1)
            self.put(nb + (o["kNQ"] - o["kN1"]), ly.nq)
            self.put(nb + (o["kNK"] - o["kN1"]), ly.nk)
            self.put(nb + (o["kN2"] - o["kN1"]), ly.n2)
        return self

    @classmethod
    def from_checkpoint(cls, model_dir, layers: int = 0, vocab: int = 0, seq: int = 32,
                        max_seq: int = 256, device: str | torch.device = "cuda",
                        f16_as_uint16: bool = False) -> "BlobModel":
        """tools/convert_pqwf.py:125-219 on the device: the blob of an HF Qwen3
        checkpoint directory (``config.json`` + ``model.safetensors``), its
        weights quantised on the GPU by ``q3_blob_from_safetensors``.  ``layers``
        / ``vocab`` = 0 keep the config's counts (the converter's --layers /
        --vocab).  F16 tensors are decoded as IEEE half; ``f16_as_uint16``
        reads them as the reference's pqwf.SafeTensors does (the 16-bit
        patterns widened as unsigned integers, pqwf.py:302, 313)."""
        cfg = json.loads((Path(model_dir) / "config.json").read_text())
        d = Dims(hidden=int(cfg["hidden_size"]), layers=layers or int(cfg["num_hidden_layers"]),
                 heads=int(cfg["num_attention_heads"]), kv_heads=int(cfg["num_key_value_heads"]),
                 head_dim=int(cfg["head_dim"]), inter=int(cfg["intermediate_size"]),
                 vocab=vocab or int(cfg["vocab_size"]), seq=seq, max_seq=max_seq)
        bm = cls(d, device)
        path = str(Path(model_dir) / "model.safetensors").encode()
        stream = torch.cuda.current_stream(bm.device).cuda_stream
        check("q3_blob_from_safetensors",
              lib().q3_blob_from_safetensors(path, C.byref(bm.L), float(cfg.get("rope_theta", 1e6)),
                                             1 if f16_as_uint16 else 0,
                                             C.c_void_p(bm.blob.data_ptr()), C.c_void_p(stream)))
        return bm

    def set_ids(self, ids) -> None:
        self.put(self.off["kIDS"], np.asarray(ids, np.int32))

    def set_ctrl(self, n_prompt: int, n_gen: int, mode: int) -> None:
        self.put(self.off["kCTRL"], np.asarray([n_prompt, n_gen, self.dims.max_seq, mode], np.int32))

    # -- reading ------------------------------------------------------------
    def read(self, key_or_off, shape, dtype) -> np.ndarray:
        off = self.off[key_or_off] if isinstance(key_or_off, str) else int(key_or_off)
        n = int(np.prod(shape)) * np.dtype(dtype).itemsize
        return self.blob[off:off + n].cpu().numpy().view(dtype).reshape(shape)

    def view(self, key: str, rows: int, cols: int, dtype) -> MatrixView:
        es = np.dtype(dtype).itemsize
        return MatrixView(self.blob.data_ptr() + self.off[key], cols * es, es, rows, cols,
                          DT[np.dtype(dtype)], self.blob)

    def kv_layer(self, layer: int):
        """(k8, ks, v8, vs) of a layer in LOGICAL token order (un-paged)."""
        d, o = self.dims, self.off
        kw = d.kv_heads * d.head_dim
        base = o["kKV_BASE"] + layer * o["kKV_STRIDE"]
        pages = d.max_seq // 32
        order = [pages - 1 - p for p in range(pages)]   # ptab of main_big.cpp:168-171

        def unpage(off, width, dtype):
            raw = self.read(off, (pages, 32, width), dtype)
            return np.concatenate([raw[order[p]] for p in range(pages)], axis=0)
        k8 = unpage(base, kw, np.int8)
        ks = unpage(base + o["kKV_SOFF"], d.kv_heads, np.float32)
        v8 = unpage(base + o["kKV_VOFF"], kw, np.int8)
        vs = unpage(base + o["kKV_VOFF"] + o["kKV_SOFF"], d.kv_heads, np.float32)
        return k8, ks, v8, vs

    # -- entry points -------------------------------------------------------
    def forward_chunk(self, pos: int, rows: int, lm_out: int, optimize_tail: bool,
                      stream=None) -> None:
        s = torch.cuda.current_stream().cuda_stream if stream is None else stream.cuda_stream
        check("q3_forward_chunk",
              lib().q3_forward_chunk(self.blob.data_ptr(), C.byref(self.L), pos, rows, lm_out,
                                     1 if optimize_tail else 0, self.ws.data_ptr(),
                                     self.ws.numel(), s))

    def generate(self, ids, n_prompt: int, n_gen: int, mode: int = 0, stream=None) -> list[int]:
        """The greedy loop (main_big.cpp:332-369); returns the generated ids."""
        self.set_ids(list(ids) + [0] * (n_prompt + n_gen - len(ids)))
        self.set_ctrl(n_prompt, n_gen, mode)
        s = torch.cuda.current_stream().cuda_stream if stream is None else stream.cuda_stream
        check("q3_generate", lib().q3_generate(self.blob.data_ptr(), C.byref(self.L),
                                               self.ws.data_ptr(), self.ws.numel(), s))
        torch.cuda.synchronize(self.device)
        all_ids = self.read("kIDS", (self.dims.max_seq,), np.int32)
        return [int(v) for v in all_ids[n_prompt:n_prompt + n_gen]]
