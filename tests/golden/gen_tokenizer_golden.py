#!/usr/bin/env python3
"""Golden data for the native tokenizer.

1. ``tok_synth.json``: a small byte-level BPE vocabulary in the layout of an HF
   ``tokenizer.json`` (``model.vocab``, ``model.merges``, ``added_tokens``),
   trained here by plain pair counting on a short text of this file's own
   (no external vocabulary exists on this machine): the 256 byte symbols,
   ``N_MERGES`` merges, then the ChatML special tokens.  A second copy,
   ``tok_synth_pairs.json``, stores the merges as ``[a, b]`` pairs, the newer
   HF form the reference also reads.
2. ``tokenizer_golden.json``: for every case string, the ids the REFERENCE's
   ``Tokenizer.encode`` (``tools/tokenizer.py`` of mland2333/qwen3-tile-ops,
   imported unmodified from a checkout) returns and its ``decode`` of them;
   plus ``decode`` of id lists that cut multi-byte characters, and the ids of
   ``N_FUZZ`` seeded strings assembled from ``FUZZ_PIECES``::

    python tests/golden/gen_tokenizer_golden.py --reference <path to the checkout>
"""

from __future__ import annotations

import argparse
import importlib
import json
import random
import sys
from collections import Counter
from pathlib import Path

HERE = Path(__file__).resolve().parent
N_MERGES = 420
SPECIALS = ["<|endoftext|>", "<|im_start|>", "<|im_end|>", "<think>", "</think>"]

CORPUS = """
The quick brown fox jumps over the lazy dog while the compiler checks every
kernel twice.  Tokens, pages and shards: we'll stream them, they're cached,
it's fast.  DON'T PANIC -- the scheduler doesn't drop requests; it waits.
for (int i = 0; i < n; ++i) { acc += x[i] * w[i]; }  // 128-byte rows
def forward(x): return rmsnorm(x) @ weight.T + bias
数据并行的热点路径在八块显卡上运行，每个请求都有自己的页表。
你好，世界！今天的天气很好，我们一起去公园散步吧。
Numbers 0123456789 and 3.14159, 2048 tokens, 151936 entries, 1e-6 epsilon.
Emoji 😀🚀 and accents café naïve résumé Ångström; Greek αβγ δελτα; Cyrillic привет.
"""


def byte_map() -> list[str]:
    """The GPT-2 byte -> symbol table (the 256 base symbols)."""
    keep = list(range(ord("!"), ord("~") + 1)) + list(range(0xA1, 0xAD)) + list(range(0xAE, 0x100))
    out, extra = {}, 0
    for b in range(256):
        if b in keep:
            out[b] = chr(b)
        else:
            out[b] = chr(256 + extra)
            extra += 1
    return [out[b] for b in range(256)]


def train(corpus: str, n_merges: int):
    bm = byte_map()
    words = Counter()
    for w in corpus.replace("\n", " \n ").split(" "):
        if w:
            words[tuple(bm[b] for b in (" " + w).encode("utf-8"))] += 1
    vocab = {s: i for i, s in enumerate(bm)}
    merges = []
    for _ in range(n_merges):
        pairs = Counter()
        for w, c in words.items():
            for a, b in zip(w, w[1:]):
                pairs[(a, b)] += c
        if not pairs:
            break
        best = max(pairs.items(), key=lambda kv: (kv[1], kv[0]))[0]
        merges.append(best)
        vocab[best[0] + best[1]] = len(vocab)
        nw = Counter()
        for w, c in words.items():
            out, i = [], 0
            while i < len(w):
                if i + 1 < len(w) and (w[i], w[i + 1]) == best:
                    out.append(w[i] + w[i + 1])
                    i += 2
                else:
                    out.append(w[i])
                    i += 1
            nw[tuple(out)] += c
        words = nw
    return vocab, merges


CASES = [
    "", "a", "Hello world", "Hello  world", "Hello   world ", "  leading spaces",
    "trailing spaces   ", "tabs\tand\nnewlines\r\n\r\nend", "line one\n\n\nline two\n",
    "I'll go, she's here, they're fine, we've won, I'm done, you'd see, it'd've",
    "DON'T SHOUT, IT'S LOUD", "O'Neil's dog's bone", "'tis", "x = 12345 + 678;",
    "3.14159e-10", "price: $1,234.56!!!", "!!!???...\n\n", "(a+b)*c - d/e",
    "café naïve Ångström", "привет мир", "你好，世界！", "数据并行的热点路径",
    "emoji 😀🚀 mixed", "½ ² Ⅳ ٣ numbers", "non breaking em sep",
    "combining é marks", "<|im_start|>user\nhi<|im_end|>\n<|im_start|>assistant\n",
    "<|im_start|><|im_end|><|endoftext|>", "text<think>inner</think>after",
    "<|im_start", "partial <|im_end|x", "<|<|im_end|>|>", "\U0001F600\U0001F600 end",
    "for (int i = 0; i < n; ++i) { acc += x[i]; }", "  \n  \t x",
    "The quick brown fox jumps over the lazy dog while the compiler checks every kernel.",
]
DECODE_ONLY = [[0], [233, 101], [228], [228, 189], [240, 159, 152], [195, 40, 195, 169]]
# pieces the seeded fuzz strings are drawn from: every class the pretokenizer
# tells apart, contraction fragments and special-token fragments
FUZZ_PIECES = (list("abcXYZ019 ,.!?;:'\"-_()[]{}<>|/\\@#$%^&*+=~`") + [
    " ", "  ", "\t", "\n", "\r\n", "\r", "'s", "'T", "'re", "'LL", "'d", "'m", "'ve",
    "你", "好", "世界", "，", "！", "é", "ñ", "Å", "e\u0301", "\u0300", "😀", "🚀",
    "\u00a0", "\u2003", "\u2028", "\u3000", "½", "²", "Ⅳ", "٣", "Ω", "ß", "ǅ",
    "<|im_end|>", "<|im_start|>", "<think>", "<|", "|>", "<|im_", "the", " the", "ing",
    "12", "3.5", "\u200b", "\ufeff", "\x00", "\x7f"])
N_FUZZ = 160


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    a = ap.parse_args()
    vocab, merges = train(CORPUS, N_MERGES)
    added = [{"id": len(vocab) + k, "content": s, "special": True} for k, s in enumerate(SPECIALS)]
    tj = {"model": {"type": "BPE", "vocab": vocab, "merges": [f"{x} {y}" for x, y in merges]},
          "added_tokens": added}
    (HERE / "tok_synth.json").write_text(json.dumps(tj, ensure_ascii=False))
    tj["model"]["merges"] = [[x, y] for x, y in merges]
    (HERE / "tok_synth_pairs.json").write_text(json.dumps(tj))       # \\u escapes
    sys.path.insert(0, str(Path(a.reference) / "tools"))
    tok_mod = importlib.import_module("tokenizer")
    tok = tok_mod.Tokenizer(str(HERE / "tok_synth.json"))
    cases = []
    for text in CASES:
        ids = tok.encode(text)
        cases.append({"text": text, "ids": ids, "decoded": tok.decode(ids)})
    dec = [{"ids": ids, "decoded": tok.decode(ids)} for ids in DECODE_ONLY]
    frng = random.Random(11)
    fuzz = []
    for _ in range(N_FUZZ):
        text = "".join(frng.choice(FUZZ_PIECES) for _ in range(frng.randint(1, 24)))
        fuzz.append({"text": text, "ids": tok.encode(text)})
    (HERE / "tokenizer_golden.json").write_text(json.dumps(
        {"vocab_size": len(vocab), "merges": len(merges), "eos_id": tok.eos_id, "cases": cases,
         "decode_only": dec, "fuzz": fuzz}, ensure_ascii=False, indent=0))
    print(len(vocab), len(merges), sum(len(c["ids"]) for c in cases))
    return 0


if __name__ == "__main__":
    sys.exit(main())
