"""The native tokenizer (``q3_tokenizer_*``) against the reference's
``tools/tokenizer.py``: ids and decoded text of every case and of 160 seeded
fuzz strings in ``tests/golden/tokenizer_golden.json`` (recorded from the
reference's own Tokenizer by ``gen_tokenizer_golden.py``), for the vocabulary
file with "a b" merges and the one with [a, b] pairs and \\u escapes."""

from __future__ import annotations

import json

import pytest

from conftest import GOLDEN

G = json.loads((GOLDEN / "tokenizer_golden.json").read_text())
FILES = ["tok_synth.json", "tok_synth_pairs.json"]


@pytest.fixture(scope="module", params=FILES)
def tok(q3, request):
    from q3b200.tokenizer import Tokenizer
    t = Tokenizer(GOLDEN / request.param)
    yield t
    t.close()


def test_encode_decode_cases(tok):
    for c in G["cases"]:
        assert tok.encode(c["text"]) == c["ids"], c["text"]
        assert tok.decode(c["ids"]) == c["decoded"], c["text"]
    assert tok.eos_id == G["eos_id"]


def test_decode_cut_characters(tok):
    for c in G["decode_only"]:
        assert tok.decode(c["ids"]) == c["decoded"]


def test_fuzz_strings(tok):
    assert len(G["fuzz"]) == 160
    for c in G["fuzz"]:
        assert tok.encode(c["text"]) == c["ids"], c["text"]


def test_round_trip_and_errors(q3, tok):
    text = "Round trip: 你好 😀 café\r\n\t<|im_start|>x"
    assert tok.decode(tok.encode(text)) == text
    with pytest.raises(q3._lib.Q3Error):
        tok.decode([G["vocab_size"] + 1000])
    long = "word " * 3000          # grows the id buffer
    assert tok.decode(tok.encode(long)) == long


def test_load_errors(q3, tmp_path):
    import ctypes as C
    lib = q3._lib.lib()
    h = C.c_void_p()
    assert lib.q3_tokenizer_load(str(tmp_path / "missing.json").encode(), C.byref(h)) == 1
    (tmp_path / "bad.json").write_text('{"model": {"vocab": {"a": 0}, "merges": ["a b c"]}}')
    assert lib.q3_tokenizer_load(str(tmp_path / "bad.json").encode(), C.byref(h)) == 3
    (tmp_path / "cut.json").write_text('{"model": {"vocab": {"a": 0}')
    assert lib.q3_tokenizer_load(str(tmp_path / "cut.json").encode(), C.byref(h)) == 3
