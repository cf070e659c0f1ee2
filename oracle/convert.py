"""CPU restatement of the blob producer (TEST INFRASTRUCTURE ONLY).

``tools/convert_pqwf.py:125-219`` with ``tools/pqwf.py:279-360``: read an HF
Qwen3 ``model.safetensors`` (BF16 / F16 / F32), quantise every weight matrix
per output row (``synth.quantize_rows`` = ``pqwf.quantize_rows``), widen the
norm vectors to float32 and build the RoPE tables; the result is the byte image
of each weight region of the blob.  Parity pinned: ``tests/golden/
blob_golden.json`` holds the sha256 of every region as the reference's own
converter wrote it for the checkpoint of ``tests/golden/hf_synth.py``.

F16 tensors: the reference views them as uint16 and widens the bit patterns as
unsigned integers (pqwf.py:302, 313, 320); ``f16_as_uint16=True`` restates
that reading (the golden digests were made with it), the default decodes IEEE
half as the product converter does by default.
"""

from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

from .synth import quantize_rows, rope_tables

F = np.float32
PROJ = [("self_attn.q_proj", "kLQ", "kLQ_SCALE"), ("self_attn.k_proj", "kLK", "kLK_SCALE"),
        ("self_attn.v_proj", "kLV", "kLV_SCALE"), ("self_attn.o_proj", "kLO", "kLO_SCALE"),
        ("mlp.gate_proj", "kLG", "kLG_SCALE"), ("mlp.up_proj", "kLU", "kLU_SCALE"),
        ("mlp.down_proj", "kLD", "kLD_SCALE")]
NORMS = [("input_layernorm", "kN1"), ("self_attn.q_norm", "kNQ"), ("self_attn.k_norm", "kNK"),
         ("post_attention_layernorm", "kN2")]


def read_safetensors(path, f16_as_uint16: bool = False) -> dict[str, np.ndarray]:
    """Every tensor of the file widened to float32 (pqwf.py:279-322)."""
    data = Path(path).read_bytes()
    hlen = struct.unpack("<Q", data[:8])[0]
    header = json.loads(data[8:8 + hlen])
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        s, e = info["data_offsets"]
        raw = data[8 + hlen + s:8 + hlen + e]
        if info["dtype"] == "BF16":
            a = (np.frombuffer(raw, np.uint16).astype(np.uint32) << 16).view(F)
        elif info["dtype"] == "F16":
            a = np.frombuffer(raw, np.uint16 if f16_as_uint16 else np.float16).astype(F)
        else:
            a = np.frombuffer(raw, F).astype(F)
        out[name] = a.reshape(info["shape"])
    return out


def regions(off: dict, layers: int, vocab: int, hidden: int, max_seq: int, half: int) -> dict:
    """[start, end) of every region the producer writes."""
    return {
        "emb": (off["kEMB"], off["kEMB"] + vocab * hidden + 4 * vocab),
        "lm": (off["kLM"], off["kLM"] + vocab * hidden + 4 * vocab),
        "nf": (off["kNF"], off["kNF"] + 4 * hidden),
        "layer_weights": (off["kLAYERW_BASE"], off["kLAYERW_BASE"] + layers * off["kLAYERW_STRIDE"]),
        "layer_norms": (off["kLAYERN_BASE"], off["kLAYERN_BASE"] + layers * off["kLAYERN_STRIDE"]),
        "cos": (off["kCOS"], off["kCOS"] + 4 * max_seq * half),
        "sin": (off["kSIN"], off["kSIN"] + 4 * max_seq * half),
    }


def convert(model_dir, off: dict, layers: int, vocab: int, max_seq: int,
            f16_as_uint16: bool = False) -> bytearray:
    """The blob bytes [0, kSCRATCH_END) with the weight regions filled
    (convert_pqwf.py:174-215); every other byte stays zero."""
    model_dir = Path(model_dir)
    cfg = json.loads((model_dir / "config.json").read_text())
    t = read_safetensors(model_dir / "model.safetensors", f16_as_uint16)
    blob = bytearray(off["kSCRATCH_END"])

    def put(o, arr):
        raw = np.ascontiguousarray(arr).view(np.uint8).reshape(-1).tobytes()
        blob[o:o + len(raw)] = raw

    def quant(name, q_off, s_off, rows):
        q, s = quantize_rows(t[name][:rows])
        put(q_off, q)
        put(s_off, s)

    H = int(cfg["hidden_size"])
    put(off["kNF"], t["model.norm.weight"].astype(F))
    cos, sin = rope_tables(max_seq, int(cfg["head_dim"]), float(cfg.get("rope_theta", 1e6)))
    put(off["kCOS"], cos)
    put(off["kSIN"], sin)
    quant("model.embed_tokens.weight", off["kEMB"], off["kEMB"] + vocab * H, vocab)
    lm = "lm_head.weight" if "lm_head.weight" in t else "model.embed_tokens.weight"
    quant(lm, off["kLM"], off["kLM"] + vocab * H, vocab)
    for i in range(layers):
        pre = f"model.layers.{i}."
        base = off["kLQ"] + i * off["kLAYERW_STRIDE"]
        for proj, dk, sk in PROJ:
            w = t[pre + proj + ".weight"]
            quant(pre + proj + ".weight", base + off[dk] - off["kLQ"], base + off[sk] - off["kLQ"],
                  w.shape[0])
        nb = off["kN1"] + i * off["kLAYERN_STRIDE"]
        for norm, key in NORMS:
            put(nb + off[key] - off["kN1"], t[pre + norm + ".weight"].astype(F))
    return blob


def to_model(model_dir, layers: int, vocab: int, seq: int, max_seq: int,
             f16_as_uint16: bool = False):
    """The same conversion as an oracle ``Model`` (for greedy-generate checks
    of a converted blob)."""
    from .q3_oracle import Layer, Model
    model_dir = Path(model_dir)
    cfg = json.loads((model_dir / "config.json").read_text())
    t = read_safetensors(model_dir / "model.safetensors", f16_as_uint16)
    emb8, emb_s = quantize_rows(t["model.embed_tokens.weight"][:vocab])
    lm = "lm_head.weight" if "lm_head.weight" in t else "model.embed_tokens.weight"
    lm8, lm_s = quantize_rows(t[lm][:vocab])
    cos, sin = rope_tables(max_seq, int(cfg["head_dim"]), float(cfg.get("rope_theta", 1e6)))
    m = Model(int(cfg["hidden_size"]), int(cfg["num_attention_heads"]),
              int(cfg["num_key_value_heads"]), int(cfg["head_dim"]), int(cfg["intermediate_size"]),
              vocab, seq, max_seq, emb8, emb_s, lm8, lm_s, t["model.norm.weight"].astype(F), cos, sin)
    for i in range(layers):
        pre = f"model.layers.{i}."
        q = {}
        for proj, key in zip([p for p, _, _ in PROJ], "qkvogud"):
            q["w" + key], q["w" + key + "_s"] = quantize_rows(t[pre + proj + ".weight"])
        m.layers.append(Layer(**q, n1=t[pre + "input_layernorm.weight"].astype(F),
                              nq=t[pre + "self_attn.q_norm.weight"].astype(F),
                              nk=t[pre + "self_attn.k_norm.weight"].astype(F),
                              n2=t[pre + "post_attention_layernorm.weight"].astype(F)))
    return m
