"""Text in / text out (tools/run_chat.py:48-112) on the GPU: the prompt is
wrapped in ChatML (unless ``--raw``), encoded by the native tokenizer, run
through the blob's greedy generate (prompt in 32-row chunks, then one token
per step, lm_head fused with argmax), and the new ids up to the first
end-of-sequence id are decoded.

    python qwen3-tile-ops_b200/chat.py "hello" --model-dir <HF checkpoint> --tokenizer <tokenizer.json>
    python qwen3-tile-ops_b200/chat.py --ids 151644,9707 --max-new 4 --model-dir ... --tokenizer ...

(run as a file, it imports its package through the repository's
``__graft_entry__.load_package``).  The reference patches a blob file and
runs its simulator; here the checkpoint is converted on the device
(``BlobModel.from_checkpoint``) and generate runs in place.
"""

from __future__ import annotations

import argparse
import sys

CHAT_TEMPLATE = "<|im_start|>user\n{text}<|im_end|>\n<|im_start|>assistant\n"
EOS_IDS = {151645, 151643}   # <|im_end|>, <|endoftext|> of the Qwen3 vocabulary


def chat(model, tokenizer, text: str | None = None, ids=None, max_new: int = 8,
         raw: bool = False) -> dict:
    """One greedy completion: returns the prompt ids, the generated ids, the
    ids kept before the first end-of-sequence id (the reference's EOS_IDS
    plus the tokenizer's own <|im_end|>) and their decoded text."""
    if ids:
        prompt_ids = [int(t) for t in ids]
    else:
        prompt_ids = tokenizer.encode(text if raw else CHAT_TEMPLATE.format(text=text))
    if len(prompt_ids) + max_new > model.dims.max_seq:
        raise ValueError(f"prompt {len(prompt_ids)} + max-new {max_new} > max_seq "
                         f"{model.dims.max_seq}")
    generated = model.generate(prompt_ids, len(prompt_ids), max_new)
    stop = EOS_IDS | {tokenizer.eos_id}
    kept = []
    for t in generated:
        if t in stop:
            break
        kept.append(t)
    return {"prompt_ids": prompt_ids, "generated": generated, "kept": kept,
            "text": tokenizer.decode(kept)}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("text", nargs="?", default="你好，请用一句话介绍你自己。")
    ap.add_argument("--tokenizer", required=True, help="HF tokenizer.json")
    ap.add_argument("--model-dir", required=True, help="HF checkpoint (config.json + model.safetensors)")
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--vocab", type=int, default=0)
    ap.add_argument("--max-seq", type=int, default=256)
    ap.add_argument("--max-new", type=int, default=8)
    ap.add_argument("--raw", action="store_true", help="do not wrap the text in ChatML")
    ap.add_argument("--ids", default="", help="use raw token ids instead of the text")
    a = ap.parse_args(argv)
    if __package__:
        from .model import BlobModel
        from .tokenizer import Tokenizer
    else:   # run as a file
        from pathlib import Path
        sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
        import __graft_entry__
        pkg = __graft_entry__.load_package()
        import importlib
        BlobModel = pkg.model.BlobModel
        Tokenizer = importlib.import_module(pkg.__name__ + ".tokenizer").Tokenizer
    tok = Tokenizer(a.tokenizer)
    bm = BlobModel.from_checkpoint(a.model_dir, layers=a.layers, vocab=a.vocab, max_seq=a.max_seq)
    ids = [int(t) for t in a.ids.split(",") if t.strip()] if a.ids else None
    try:
        out = chat(bm, tok, a.text, ids, a.max_new, a.raw)
    except ValueError as e:
        print(f"error: {e}", file=sys.stderr)
        return 2
    print(f"prompt: {len(out['prompt_ids'])} tokens")
    print(f"new ids: {out['generated']}")
    print("--- output ---")
    print(out["text"])
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
