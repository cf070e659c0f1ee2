#!/usr/bin/env python3
"""Golden data for the blob producer: convert the synthetic checkpoint of
``hf_synth.py`` with the REFERENCE's own converter (``tools/convert_pqwf.py``
of mland2333/qwen3-tile-ops, imported unmodified from a checkout) and record
the sha256 of every region it writes, plus its RoPE tables::

    python tests/golden/gen_blob_golden.py --reference <path to the checkout>

The reference reads F16 tensors as unsigned 16-bit integers (pqwf.py:302,
313); the digests record that reading, which the product reproduces under
Q3_CONVERT_F16_AS_UINT16.  Outputs ``blob_golden.json`` (layout dims,
per-region digests) and
``blob_rope.npz`` (cos/sin, compared within one float32 ulp: the reference
computes them with numpy's float64 pow/cos/sin).
"""

from __future__ import annotations

import argparse
import hashlib
import importlib
import json
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from hf_synth import write_hf_model  # noqa: E402

LAYERS, VOCAB, SEQ, MAX_SEQ = 2, 1024, 32, 256


def regions(off: dict, layers: int, vocab: int, hidden: int, max_seq: int, half: int) -> dict:
    return {
        "emb": (off["kEMB"], off["kEMB"] + vocab * hidden + 4 * vocab),
        "lm": (off["kLM"], off["kLM"] + vocab * hidden + 4 * vocab),
        "nf": (off["kNF"], off["kNF"] + 4 * hidden),
        "layer_weights": (off["kLAYERW_BASE"], off["kLAYERW_BASE"] + layers * off["kLAYERW_STRIDE"]),
        "layer_norms": (off["kLAYERN_BASE"], off["kLAYERN_BASE"] + layers * off["kLAYERN_STRIDE"]),
        "cos": (off["kCOS"], off["kCOS"] + 4 * max_seq * half),
        "sin": (off["kSIN"], off["kSIN"] + 4 * max_seq * half),
    }


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    a = ap.parse_args()
    sys.path.insert(0, str(Path(a.reference) / "tools"))
    conv = importlib.import_module("convert_pqwf")
    pqwf = importlib.import_module("pqwf")
    with tempfile.TemporaryDirectory() as tmp:
        mdir = write_hf_model(Path(tmp) / "model", LAYERS, VOCAB)
        blob = Path(tmp) / "blob.bin"
        sys.argv = ["convert_pqwf.py", "--model-dir", str(mdir), "--layers", str(LAYERS),
                    "--vocab", str(VOCAB), "--seq", str(SEQ), "--max-seq", str(MAX_SEQ),
                    "--n-prompt", "8", "--blob", str(blob), "--header", str(Path(tmp) / "h.h"),
                    "--no-ref"]
        assert conv.main() == 0
        layout = pqwf.Layout(hidden=1024, layers=LAYERS, heads=16, kv_heads=8, head_dim=128,
                             inter=3072, vocab=VOCAB, seq=SEQ, max_seq=MAX_SEQ).compute()
        off = layout.offsets
        data = blob.read_bytes()
        regs = regions(off, LAYERS, VOCAB, 1024, MAX_SEQ, 64)
        digests = {k: hashlib.sha256(data[s:e]).hexdigest() for k, (s, e) in regs.items()}
        cos = np.frombuffer(data[regs["cos"][0]:regs["cos"][1]], np.float32).reshape(MAX_SEQ, 64)
        sin = np.frombuffer(data[regs["sin"][0]:regs["sin"][1]], np.float32).reshape(MAX_SEQ, 64)
    (HERE / "blob_golden.json").write_text(json.dumps(
        {"layers": LAYERS, "vocab": VOCAB, "seq": SEQ, "max_seq": MAX_SEQ, "digests": digests}, indent=1))
    np.savez(HERE / "blob_rope.npz", cos=cos, sin=sin)
    print(json.dumps(digests, indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
