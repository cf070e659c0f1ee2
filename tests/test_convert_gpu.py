"""The native blob producer on the GPU (``q3_blob_from_safetensors``): an HF
checkpoint converted on the device must give the blob the reference's
converter writes.

* reference reading of F16 (Q3_CONVERT_F16_AS_UINT16): every weight region's
  sha256 equals the reference converter's (``tests/golden/blob_golden.json``);
  RoPE tables within one float32 ulp of the reference's (numpy's float64
  cos/sin and the C library's may differ in the last double bit);
* default reading, a tied lm_head, NaN / inf / all-zero rows and a truncated
  layout: byte-equal to the oracle restatement of the converter;
* the converted blob runs greedy generate to the oracle's ids."""

from __future__ import annotations

import hashlib
import json
import sys

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

sys.path.insert(0, str(GOLDEN))
from hf_synth import write_hf_model  # noqa: E402
from oracle import convert  # noqa: E402
from oracle import q3_oracle as O  # noqa: E402

GOLD = json.loads((GOLDEN / "blob_golden.json").read_text())
EXACT = ("emb", "lm", "nf", "layer_weights", "layer_norms")


def _regions(bm):
    d = bm.dims
    return convert.regions(bm.off, d.layers, d.vocab, d.hidden, d.max_seq, d.head_dim // 2)


def _bytes(bm, s, e):
    return bm.blob[s:e].cpu().numpy().tobytes()


def _ulps(a, b):
    ai, bi = a.view(np.int32).astype(np.int64), b.view(np.int32).astype(np.int64)
    ai = np.where(ai < 0, -(ai & 0x7FFFFFFF), ai)
    bi = np.where(bi < 0, -(bi & 0x7FFFFFFF), bi)
    return np.abs(ai - bi)


@pytest.fixture(scope="module")
def ckpts(tmp_path_factory):
    root = tmp_path_factory.mktemp("hf")
    return {"plain": write_hf_model(root / "plain", GOLD["layers"], GOLD["vocab"]),
            "edge": write_hf_model(root / "edge", 3, 1024, seed=5, tied=True, poison=True)}


def test_producer_matches_reference_digests(q3, ckpts):
    from q3b200.model import BlobModel
    bm = BlobModel.from_checkpoint(ckpts["plain"], layers=GOLD["layers"], vocab=GOLD["vocab"],
                                   seq=GOLD["seq"], max_seq=GOLD["max_seq"], f16_as_uint16=True)
    regs = _regions(bm)
    for k in EXACT:
        s, e = regs[k]
        assert hashlib.sha256(_bytes(bm, s, e)).hexdigest() == GOLD["digests"][k], k
    rope = np.load(GOLDEN / "blob_rope.npz")
    for k in ("cos", "sin"):
        s, e = regs[k]
        got = np.frombuffer(_bytes(bm, s, e), np.float32).reshape(rope[k].shape)
        assert int(_ulps(got, rope[k]).max()) <= 1, k
    assert q3._lib.lib().q3_device_status() == 0


@pytest.mark.parametrize("case,layers,vocab,f16", [("plain", 2, 1024, False),
                                                    ("edge", 3, 1024, False),
                                                    ("edge", 1, 520, True)])
def test_producer_matches_oracle(q3, ckpts, case, layers, vocab, f16):
    from q3b200.model import BlobModel
    bm = BlobModel.from_checkpoint(ckpts[case], layers=layers, vocab=vocab, max_seq=256,
                                   f16_as_uint16=f16)
    want = convert.convert(ckpts[case], bm.off, layers, vocab, 256, f16_as_uint16=f16)
    for k, (s, e) in _regions(bm).items():
        got = _bytes(bm, s, e)
        if k in ("cos", "sin"):
            assert int(_ulps(np.frombuffer(got, np.float32),
                             np.frombuffer(bytes(want[s:e]), np.float32)).max()) <= 1, k
        else:
            assert got == bytes(want[s:e]), k
    if case == "edge":   # the poisoned rows of layer 0's q_proj: NaN scale, zero codes
        qs = bm.read(bm.off["kLQ_SCALE"], (8,), np.float32)
        q8 = bm.read(bm.off["kLQ"], (8, 1024), np.int8)
        assert np.isnan(qs[3]) and not q8[3].any()
        assert np.isinf(qs[5]) and qs[7] == 0 and not q8[7].any()


def test_converted_blob_generates_oracle_ids(q3, ckpts):
    from q3b200.model import BlobModel
    bm = BlobModel.from_checkpoint(ckpts["plain"], layers=2, vocab=1024, seq=32, max_seq=256)
    model = convert.to_model(ckpts["plain"], 2, 1024, 32, 256)
    ids = [int(t) for t in np.random.default_rng(4).integers(0, 1024, 40)]
    want = O.generate(model, ids, 40, 3)[1]
    assert bm.generate(ids, 40, 3) == want
