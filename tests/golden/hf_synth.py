"""A seeded synthetic checkpoint in the layout the reference converter reads
(HF Qwen3: ``config.json`` + ``model.safetensors`` with the HF tensor names),
for the blob-producer tests.  Weights N(0, 0.02), norm weights 1 + 0.05 N(0,1),
rounded to BF16; a few tensors are stored as F16 / F32 so that every dtype the
converters accept is exercised.  Test infrastructure only."""

from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

DIMS = dict(hidden_size=1024, num_attention_heads=16, num_key_value_heads=8, head_dim=128,
            intermediate_size=3072, rope_theta=1000000.0)


def _bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bits, round to nearest even."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def write_hf_model(out_dir: str | Path, layers: int = 2, vocab: int = 1024, seed: int = 3,
                   tied: bool = False, poison: bool = False, fast: bool = False) -> Path:
    """``tied``: no lm_head.weight (the converters fall back to the embedding).
    ``poison``: a NaN, an infinity and an all-zero row in layer 0's q_proj.
    ``fast``: every weight matrix BF16 with random bit patterns of magnitude
    2^-7 .. 2^-5 and random sign (for timing full-size conversions; seconds
    instead of minutes to write)."""
    if fast:
        return _write_fast(Path(out_dir), layers, vocab, seed)
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    rng = np.random.default_rng(seed)
    H, I, HD = DIMS["hidden_size"], DIMS["intermediate_size"], DIMS["head_dim"]
    QW, KW = DIMS["num_attention_heads"] * HD, DIMS["num_key_value_heads"] * HD
    tensors: list[tuple[str, str, np.ndarray]] = []

    def mat(name, rows, cols, dtype="BF16"):
        w = (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        tensors.append((name, dtype, w))

    def vec(name, n, dtype="BF16"):
        v = (np.float32(1.0) + rng.standard_normal(n, dtype=np.float32) * np.float32(0.05)).astype(np.float32)
        tensors.append((name, dtype, v))

    mat("model.embed_tokens.weight", vocab, H)
    for i in range(layers):
        p = f"model.layers.{i}."
        mat(p + "self_attn.q_proj.weight", QW, H)
        mat(p + "self_attn.k_proj.weight", KW, H, "F16" if i == 0 else "BF16")
        mat(p + "self_attn.v_proj.weight", KW, H)
        mat(p + "self_attn.o_proj.weight", H, QW)
        mat(p + "mlp.gate_proj.weight", I, H)
        mat(p + "mlp.up_proj.weight", I, H, "F32" if i == 0 else "BF16")
        mat(p + "mlp.down_proj.weight", H, I)
        vec(p + "input_layernorm.weight", H)
        vec(p + "self_attn.q_norm.weight", HD, "F32")
        vec(p + "self_attn.k_norm.weight", HD)
        vec(p + "post_attention_layernorm.weight", H)
    vec("model.norm.weight", H)
    if not tied:
        mat("lm_head.weight", vocab, H)
    if poison:
        w = tensors[1][2]
        w[3, 17], w[5, 2], w[7, :] = np.nan, np.inf, 0.0

    header, blobs, off = {}, [], 0
    for name, dtype, arr in tensors:
        if dtype == "BF16":
            raw = _bf16(arr).tobytes()
        elif dtype == "F16":
            raw = arr.astype(np.float16).tobytes()
        else:
            raw = arr.astype(np.float32).tobytes()
        header[name] = {"dtype": dtype, "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    header["__metadata__"] = {"format": "pt"}
    hj = json.dumps(header).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(out / "model.safetensors", "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for raw in blobs:
            f.write(raw)
    cfg = dict(DIMS, vocab_size=vocab, num_hidden_layers=layers)
    (out / "config.json").write_text(json.dumps(cfg))
    return out


def _write_fast(out: Path, layers: int, vocab: int, seed: int) -> Path:
    out.mkdir(parents=True, exist_ok=True)
    rng = np.random.default_rng(seed)
    H, I, HD = DIMS["hidden_size"], DIMS["intermediate_size"], DIMS["head_dim"]
    QW, KW = DIMS["num_attention_heads"] * HD, DIMS["num_key_value_heads"] * HD
    shapes = [("model.embed_tokens.weight", (vocab, H))]
    for i in range(layers):
        p = f"model.layers.{i}."
        shapes += [(p + "self_attn.q_proj.weight", (QW, H)), (p + "self_attn.k_proj.weight", (KW, H)),
                   (p + "self_attn.v_proj.weight", (KW, H)), (p + "self_attn.o_proj.weight", (H, QW)),
                   (p + "mlp.gate_proj.weight", (I, H)), (p + "mlp.up_proj.weight", (I, H)),
                   (p + "mlp.down_proj.weight", (H, I)), (p + "input_layernorm.weight", (H,)),
                   (p + "self_attn.q_norm.weight", (HD,)), (p + "self_attn.k_norm.weight", (HD,)),
                   (p + "post_attention_layernorm.weight", (H,))]
    shapes += [("model.norm.weight", (H,)), ("lm_head.weight", (vocab, H))]
    header, off = {}, 0
    for name, shape in shapes:
        n = 2 * int(np.prod(shape))
        header[name] = {"dtype": "BF16", "shape": list(shape), "data_offsets": [off, off + n]}
        off += n
    hj = json.dumps(header).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(out / "model.safetensors", "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for name, shape in shapes:
            n = int(np.prod(shape))
            if len(shape) == 1:     # norm weights near 1
                bits = rng.integers(0x3F70, 0x3F90, n, dtype=np.uint16)
            else:                   # exponent 2^-7 .. 2^-5, random mantissa and sign
                bits = rng.integers(0x3C00, 0x3D00, n, dtype=np.uint16)
                bits |= (rng.integers(0, 2, n, dtype=np.uint16) << 15).astype(np.uint16)
            f.write(bits.tobytes())
    cfg = dict(DIMS, vocab_size=vocab, num_hidden_layers=layers)
    (out / "config.json").write_text(json.dumps(cfg))
    return out
