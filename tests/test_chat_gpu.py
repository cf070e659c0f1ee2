"""Text in / text out on the GPU (``q3b200.chat``, tools/run_chat.py): a
seeded checkpoint converted on the device, the synthetic vocabulary's
tokenizer, ChatML prompt -> greedy generate -> decode.  The generated ids
must be the oracle's greedy ids for the same converted weights."""

from __future__ import annotations

import json
import sys

import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

sys.path.insert(0, str(GOLDEN))
from hf_synth import write_hf_model  # noqa: E402
from oracle import convert  # noqa: E402
from oracle import q3_oracle as O  # noqa: E402

VOCAB = 768   # the model's rows; the synthetic vocabulary has 681 ids


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    return write_hf_model(tmp_path_factory.mktemp("chat") / "m", 2, VOCAB, seed=9)


@pytest.fixture(scope="module")
def tok_path(tmp_path_factory):
    """tok_synth.json plus added tokens <xN> for ids 681..767, so that every id
    a random model can pick decodes."""
    tj = json.loads((GOLDEN / "tok_synth.json").read_text())
    n = len(tj["model"]["vocab"]) + len(tj["added_tokens"])
    tj["added_tokens"] += [{"id": k, "content": f"<x{k}>", "special": True} for k in range(n, VOCAB)]
    p = tmp_path_factory.mktemp("tok") / "tokenizer.json"
    p.write_text(json.dumps(tj, ensure_ascii=False))
    return p


def test_chat_matches_oracle(q3, ckpt, tok_path):
    from q3b200.chat import CHAT_TEMPLATE, chat
    from q3b200.model import BlobModel
    from q3b200.tokenizer import Tokenizer
    tok = Tokenizer(tok_path)
    bm = BlobModel.from_checkpoint(ckpt, layers=2, vocab=VOCAB, max_seq=256)
    out = chat(bm, tok, "hello, tile world", max_new=6)
    assert out["prompt_ids"] == tok.encode(CHAT_TEMPLATE.format(text="hello, tile world"))
    model = convert.to_model(ckpt, 2, VOCAB, 32, 256)
    want = O.generate(model, out["prompt_ids"], len(out["prompt_ids"]), 6)[1]
    assert out["generated"] == want
    stop = out["generated"].index(tok.eos_id) if tok.eos_id in out["generated"] else 6
    assert out["kept"] == want[:stop] and out["text"] == tok.decode(want[:stop])
    raw = chat(bm, tok, ids=[677, 117, 115], max_new=3)
    assert raw["prompt_ids"] == [677, 117, 115] and len(raw["generated"]) == 3
    with pytest.raises(ValueError):
        chat(bm, tok, ids=[1] * 250, max_new=8)


def test_chat_cli(q3, ckpt, tok_path, capsys):
    from q3b200.chat import main
    rc = main(["hi", "--tokenizer", str(tok_path), "--model-dir", str(ckpt),
               "--layers", "1", "--max-new", "4"])
    assert rc == 0
    lines = capsys.readouterr().out.splitlines()
    assert lines[0].startswith("prompt: ") and lines[1].startswith("new ids: ")
