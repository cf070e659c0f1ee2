"""The blob producer's checker and host side, on the CPU: the oracle
restatement of ``tools/convert_pqwf.py`` reproduces the region digests the
reference's own converter wrote for the synthetic checkpoint of
``tests/golden/hf_synth.py`` (``blob_golden.json``, ``blob_rope.npz``), and the
library's safetensors header parser reports the file's tensors."""

from __future__ import annotations

import hashlib
import json
import sys

import numpy as np
import pytest

from conftest import GOLDEN

sys.path.insert(0, str(GOLDEN))
from hf_synth import write_hf_model  # noqa: E402

GOLD = json.loads((GOLDEN / "blob_golden.json").read_text())


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    return write_hf_model(tmp_path_factory.mktemp("hf") / "m", GOLD["layers"], GOLD["vocab"])


def _off(layers, vocab, max_seq):
    import q3b200.model as M
    return M.layout(M.Dims(layers=layers, vocab=vocab, max_seq=max_seq))[1]


def test_oracle_converter_matches_reference_digests(q3, ckpt):
    from oracle import convert
    off = _off(GOLD["layers"], GOLD["vocab"], GOLD["max_seq"])
    blob = convert.convert(ckpt, off, GOLD["layers"], GOLD["vocab"], GOLD["max_seq"],
                           f16_as_uint16=True)
    regs = convert.regions(off, GOLD["layers"], GOLD["vocab"], 1024, GOLD["max_seq"], 64)
    got = {k: hashlib.sha256(bytes(blob[s:e])).hexdigest() for k, (s, e) in regs.items()}
    assert got == GOLD["digests"]
    rope = np.load(GOLDEN / "blob_rope.npz")
    s, e = regs["cos"]
    assert np.array_equal(np.frombuffer(bytes(blob[s:e]), np.float32).reshape(-1, 64), rope["cos"])


def test_oracle_f16_decoding(q3, ckpt):
    """Default reading of the F16 tensor is IEEE half; the reference's reading
    (bit patterns as integers) is kept only behind the flag."""
    from oracle import convert
    name = "model.layers.0.self_attn.k_proj.weight"
    half = convert.read_safetensors(ckpt / "model.safetensors")[name]
    bits = convert.read_safetensors(ckpt / "model.safetensors", f16_as_uint16=True)[name]
    assert np.array_equal(half.astype(np.float16).view(np.uint16).astype(np.float32), bits)
    assert 0.005 < float(np.std(half)) < 0.05


def test_safetensors_header_parser(q3, ckpt):
    import q3b200.model as M
    st = ckpt / "model.safetensors"
    assert M.safetensors_tensor(st, "model.embed_tokens.weight") == ("BF16", (1024, 1024))
    assert M.safetensors_tensor(st, "model.layers.0.self_attn.k_proj.weight") == ("F16", (1024, 1024))
    assert M.safetensors_tensor(st, "model.layers.0.mlp.up_proj.weight") == ("F32", (3072, 1024))
    assert M.safetensors_tensor(st, "model.layers.1.mlp.down_proj.weight") == ("BF16", (1024, 3072))
    assert M.safetensors_tensor(st, "model.layers.0.self_attn.q_norm.weight") == ("F32", (128,))
    with pytest.raises(q3._lib.Q3Error):
        M.safetensors_tensor(st, "model.layers.9.mlp.up_proj.weight")


def test_safetensors_bad_files_are_rejected(q3, ckpt, tmp_path):
    import ctypes as C
    lib = q3._lib.lib()
    dt, nd = C.c_int32(), C.c_int32()
    shape = (C.c_uint64 * 4)()

    def probe(path):
        return lib.q3_safetensors_tensor(str(path).encode(), b"model.norm.weight", C.byref(dt),
                                         shape, C.byref(nd))
    assert probe(tmp_path / "absent.safetensors") == 1
    raw = (ckpt / "model.safetensors").read_bytes()
    (tmp_path / "cut.safetensors").write_bytes(raw[:len(raw) // 2])   # data ranges past the end
    assert probe(tmp_path / "cut.safetensors") == 3
    (tmp_path / "hdr.safetensors").write_bytes(raw[:8] + b"{" + raw[9:64])   # header cut short
    assert probe(tmp_path / "hdr.safetensors") == 3
