"""Property and fuzz checks of the host-side parsers (CPU): the tokenizer's
byte-level BPE round-trips any text; malformed tokenizer.json and safetensors
files are rejected with a status code, never a crash."""

from __future__ import annotations

import ctypes as C
import json
import struct

import pytest

from conftest import GOLDEN

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402


@pytest.fixture(scope="module")
def tok(q3):
    from q3b200.tokenizer import Tokenizer
    t = Tokenizer(GOLDEN / "tok_synth.json")
    yield t
    t.close()


@settings(max_examples=300, deadline=None)
@given(st.text(max_size=200))
def test_tokenizer_round_trip(tok, text):
    assert tok.decode(tok.encode(text)) == text


@settings(max_examples=200, deadline=None)
@given(st.lists(st.sampled_from(["<|im_start|>", "<|im_end|>", "<think>", "</think>",
                                 "user\n", " ", "\n\n", "你好", "'s", "x1"]), max_size=30))
def test_tokenizer_specials_round_trip(tok, parts):
    text = "".join(parts)
    ids = tok.encode(text)
    assert tok.decode(ids) == text
    assert ids.count(677) == text.count("<|im_start|>")


def _load_rc(q3, path):
    h = C.c_void_p()
    rc = q3._lib.lib().q3_tokenizer_load(str(path).encode(), C.byref(h))
    if rc == 0:
        q3._lib.lib().q3_tokenizer_destroy(h)
    return rc


@settings(max_examples=200, deadline=None)
@given(st.binary(max_size=400))
def test_tokenizer_json_fuzz(q3, tmp_path_factory, blob):
    p = tmp_path_factory.mktemp("tj") / "t.json"
    p.write_bytes(blob)
    assert _load_rc(q3, p) in (0, 3)


@settings(max_examples=100, deadline=None)
@given(st.integers(min_value=1, max_value=27000), st.binary(min_size=1, max_size=8))
def test_tokenizer_json_corruption(q3, tmp_path_factory, pos, junk):
    raw = (GOLDEN / "tok_synth.json").read_bytes()
    pos = pos % len(raw)
    p = tmp_path_factory.mktemp("tc") / "t.json"
    p.write_bytes(raw[:pos] + junk + raw[pos + len(junk):])
    assert _load_rc(q3, p) in (0, 3)


def _st_rc(q3, path):
    dt, nd = C.c_int32(), C.c_int32()
    shape = (C.c_uint64 * 4)()
    return q3._lib.lib().q3_safetensors_tensor(str(path).encode(), b"w", C.byref(dt), shape,
                                               C.byref(nd))


@settings(max_examples=200, deadline=None)
@given(st.binary(max_size=300), st.integers(min_value=0, max_value=2 ** 40))
def test_safetensors_header_fuzz(q3, tmp_path_factory, hdr, declared):
    p = tmp_path_factory.mktemp("st") / "m.safetensors"
    p.write_bytes(struct.pack("<Q", declared) + hdr)
    assert _st_rc(q3, p) in (3,)


@settings(max_examples=100, deadline=None)
@given(st.sampled_from(["F32", "BF16", "F16", "I8", "X"]),
       st.lists(st.integers(min_value=0, max_value=70000), max_size=3),
       st.integers(min_value=-5, max_value=300), st.integers(min_value=-5, max_value=300))
def test_safetensors_entry_fuzz(q3, tmp_path_factory, dtype, shape, a, b):
    hdr = json.dumps({"w": {"dtype": dtype, "shape": shape, "data_offsets": [a, b]}}).encode()
    p = tmp_path_factory.mktemp("se") / "m.safetensors"
    p.write_bytes(struct.pack("<Q", len(hdr)) + hdr + bytes(256))
    rc = _st_rc(q3, p)
    n = 1
    for d in shape:
        n *= d
    es = {"F32": 4, "BF16": 2, "F16": 2}.get(dtype)
    valid = es is not None and 0 <= a <= b <= 256 and b - a == n * es
    if dtype not in ("F32", "BF16", "F16"):
        valid = 0 <= a <= b <= 256            # unknown dtypes parse; their size is not checked
    assert rc == (0 if valid else 3)
