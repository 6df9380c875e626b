"""Regenerate tokenizer_synth.json and tokenizer_synth_golden.json.

No real Qwen3 tokenizer.json ships with the reference or this image, so the
tokenizer fixtures are synthetic, in the real file's schema: a byte-level
BPE (all 256 byte tokens, ~3000 entries, merges in the ["a", "b"] pair form
that current tokenizer.json files use, added_tokens carrying Qwen3's
<|endoftext|> / <|im_start|> / <|im_end|>) trained with the HuggingFace
`tokenizers` library on a seeded synthetic corpus (words from random
syllables, numbers, punctuation, contractions, accented / CJK / emoji text,
tabs and newlines).  The trainer only produces the vocabulary and merges;
its own pre-tokenizer is not involved in any expected output.

tokenizer_synth_golden.json holds sample texts (a few with special tokens
inside) and their token ids from oracle/tokenizer_ref.py, the literal
restatement of nnmetal/src/tokenizer.zig.  Run:
    python tests/golden/make_tokenizer_golden.py
"""
import json
import random
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

SPECIALS = ["<|endoftext|>", "<|im_start|>", "<|im_end|>"]


def synth_corpus(seed: int, n_lines: int) -> list[str]:
    rng = random.Random(seed)
    syl = [a + b for a in "bcdfghjklmnprstvwz" for b in "aeiou"] + ["th", "sh", "ch", "qu", "ng"]
    extra = ["é", "ü", "ñ", "ø", "ß", "日本", "中文", "한국", "Ωμέγα", "😀", "🚀", "—", "…"]
    words = ["".join(rng.choice(syl) for _ in range(rng.randint(1, 4))) for _ in range(600)]
    lines = []
    for _ in range(n_lines):
        parts = []
        for _ in range(rng.randint(3, 14)):
            r = rng.random()
            if r < 0.70:
                w = rng.choice(words)
                parts.append(w.capitalize() if rng.random() < 0.15 else w)
            elif r < 0.80:
                parts.append(str(rng.randint(0, 100000)))
            elif r < 0.88:
                parts.append(rng.choice(extra))
            elif r < 0.94:
                parts.append(rng.choice(words) + rng.choice(["'s", "'t", "'re", "'ll", "'ve", "'m", "'d"]))
            else:
                parts.append(rng.choice(["(", ")", ",", ".", "!", "?", ":", ";", "--", "==", "{}", "[]"]))
        sep = rng.choice([" ", " ", " ", "  ", "\t"])
        lines.append(sep.join(parts) + rng.choice(["", ".", "!", "\n"]))
    return lines


def make_tokenizer_json() -> str:
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers, trainers
    tok = Tokenizer(models.BPE())
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=3000, min_frequency=2, special_tokens=SPECIALS,
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet(),
                                  show_progress=False)
    tok.train_from_iterator(synth_corpus(0, 4000), trainer=trainer)
    data = json.loads(tok.to_str())
    # special tokens at the end of the id range, as in Qwen3's file
    vocab = data["model"]["vocab"]
    n = len(vocab)
    remap = {}
    for s in SPECIALS:
        remap[vocab.pop(s)] = None
    ordered = sorted(vocab.items(), key=lambda kv: kv[1])
    data["model"]["vocab"] = {k: i for i, (k, _) in enumerate(ordered)}
    data["added_tokens"] = [
        {"id": n - len(SPECIALS) + i, "content": s, "single_word": False, "lstrip": False,
         "rstrip": False, "normalized": False, "special": True} for i, s in enumerate(SPECIALS)]
    return json.dumps(data, ensure_ascii=False, separators=(",", ":"))


def golden_texts() -> list[str]:
    lines = synth_corpus(1, 40)
    texts = [
        "Hello world",
        "It's a test: 1234567 apples, don't you think?",
        "  leading spaces\n\nand\r\nnewlines\t\ttabs",
        "<|im_start|>user\nbakodu<|im_end|>\n<|im_start|>assistant\n",
        "unicode: é ü 日本 中文 😀🚀 — …",
        "",
        "'S 'T 'RE 'LL 'Ve",
        "x" * 600,
        "<|endoftext|><|endoftext|>",
        "a<|im_end",
    ]
    return texts + ["".join(lines[i:i + 4]) for i in range(0, 40, 4)]


def main() -> None:
    from oracle.tokenizer_ref import TokError, Tokenizer
    js = make_tokenizer_json()
    (HERE / "tokenizer_synth.json").write_text(js, encoding="utf-8")
    ref = Tokenizer(js.encode())
    cases = []
    for t in golden_texts():
        try:
            cases.append({"text": t, "ids": ref.encode(t)})
        except TokError as e:
            cases.append({"text": t, "error": e.name})
    cases.append({"chat_prompt": "How are you?", "ids": ref.apply_chat_template("How are you?")})
    out = {"tokenizer": "tokenizer_synth.json", "vocab_size": ref.vocab_size,
           "eos_token_id": ref.eos_token_id, "im_start_token_id": ref.im_start_token_id,
           "im_end_token_id": ref.im_end_token_id, "cases": cases}
    (HERE / "tokenizer_synth_golden.json").write_text(json.dumps(out, ensure_ascii=False, indent=0),
                                                      encoding="utf-8")


if __name__ == "__main__":
    main()
