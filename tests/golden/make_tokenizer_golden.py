"""Generate ``tokenizer_golden.json``: token ids from the reference's own tokenizer library.

glypr builds its text tokenizer from GGUF metadata with the ``tokenizers`` crate 0.22.2
(crates/glypr-core/src/tokenizer.rs:77-138, Cargo.lock:3151-3153).  This script drives the
Python binding of that same crate version, configured exactly as ``from_gguf_metadata``
configures it (BPE from the vocabulary and merges, byte fallback, fused unknowns, unknown token
``<unk>``, normaliser Replace(' ' -> U+2581), pre-tokeniser Split(' ', MergedWithPrevious)),
over vocabularies made here (no Gemma vocabulary exists in this container):

* ``trained``: a BPE vocabulary trained by the same library on seeded synthetic multilingual
  text, laid out like a GGUF token table (specials, the 256 byte tokens, then the learned
  pieces), with a small alphabet so that rarer characters take the byte fallback;
* ``quirks``: hand-made vocabularies that reach the edge behaviour: byte tokens partly missing
  (unknowns fused around byte fallbacks), two merges producing the same token, a duplicated
  merge, duplicated tokens, single characters whose ids are BOS/EOS, merges that are not
  "a b" pairs;

and records, per text, the ids ``Tokenizer::encode(text, true)`` returns.  It also records the
build and encode errors the library raises.  Run it where ``tokenizers`` 0.22.2 is importable:
``python tests/golden/make_tokenizer_golden.py``.
"""
from __future__ import annotations

import json
import os
import random

import tokenizers
from tokenizers import Tokenizer, models, normalizers, pre_tokenizers, trainers

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "tokenizer_golden.json")

SPECIALS = ["<pad>", "<eos>", "<bos>", "<unk>"]
BYTES = ["<0x%02X>" % b for b in range(256)]

SYLLABLES = {
    "latin": ["ka", "lo", "mi", "ne", "ru", "sta", "tion", "er", "ing", "the", "and", "qu", "str", "ph", "ed"],
    "accented": ["é", "è", "ü", "ö", "ñ", "ç", "à", "ø", "ß", "ł"],
    "greek": ["κα", "λη", "μέ", "ρα", "σο", "φία", "ΣΟΦ", "Σ"],
    "cyrillic": ["при", "вет", "мир", "ска", "зка", "ЖИ"],
    "cjk": ["東京", "大学", "研究", "中文", "日本語", "한국어"],
    "symbols": ["3.14", "2026", "x=y+1", "(a,b)", "[0]", "{k:v}", "#", "@", "->", "::", "...", "!?"],
    "emoji": ["🙂", "🚀", "👍🏽", "🇯🇵"],
}
WHITES = [" ", " ", " ", " ", "  ", "\n", "\t", " \n "]


def synth_text(rng: random.Random, n_words: int) -> str:
    out = []
    for _ in range(n_words):
        kind = rng.choices(list(SYLLABLES), weights=[60, 8, 6, 6, 5, 10, 3])[0]
        word = "".join(rng.choice(SYLLABLES[kind]) for _ in range(rng.randint(1, 3)))
        if rng.random() < 0.1:
            word = word.capitalize()
        out.append(word)
        out.append(rng.choice(WHITES))
    return "".join(out).strip(" ") if rng.random() < 0.5 else "".join(out)


def reference_tokenizer(tokens, merges):
    """tokenizer.rs:77-138, through the library's Python binding."""
    vocab = {}
    for i, t in enumerate(tokens):
        vocab[t] = i
    pairs = []
    for m in merges:
        parts = m.split(" ")
        if len(parts) == 2:
            pairs.append((parts[0], parts[1]))
    bpe = models.BPE(vocab=vocab, merges=pairs, unk_token="<unk>", fuse_unk=True, byte_fallback=True)
    tok = Tokenizer(bpe)
    tok.normalizer = normalizers.Replace(" ", "▁")
    tok.pre_tokenizer = pre_tokenizers.Split(" ", behavior="merged_with_previous", invert=False)
    return tok


def encode_cases(tok, texts):
    cases = []
    for t in texts:
        try:
            cases.append({"text": t, "ids": tok.encode(t, add_special_tokens=True).ids})
        except Exception as e:  # noqa: BLE001 - the library's error text is the golden value
            cases.append({"text": t, "error": str(e)})
    return cases


def trained_vocab(rng):
    corpus = [synth_text(rng, rng.randint(5, 60)) for _ in range(3000)]
    trainer_tok = Tokenizer(models.BPE(unk_token="<unk>", byte_fallback=True, fuse_unk=True))
    trainer_tok.normalizer = normalizers.Replace(" ", "▁")
    trainer_tok.pre_tokenizer = pre_tokenizers.Split("▁", behavior="merged_with_next")
    trainer = trainers.BpeTrainer(vocab_size=1800, special_tokens=SPECIALS, limit_alphabet=90,
                                  show_progress=False)
    trainer_tok.train_from_iterator(corpus, trainer)
    model = json.loads(trainer_tok.to_str())["model"]
    learned = sorted(model["vocab"].items(), key=lambda kv: kv[1])
    tokens = list(SPECIALS) + BYTES + [t for t, _ in learned if t not in SPECIALS]
    merges = [" ".join(m) if isinstance(m, list) else m for m in model["merges"]]
    return tokens, merges


def trained_texts(rng):
    texts = [synth_text(rng, rng.randint(1, 40)) for _ in range(240)]
    texts += [synth_text(rng, 1500), synth_text(rng, 4000)]  # long documents (one BPE word)
    texts += [
        "", " ", "  ", "   ", "\t", "\n\n", "a", "A", "Σ", "ΣΣ", "é", "é", "ß", "🙂", "👍🏽",
        "<bos>", "<eos>", "<unk>", "<0x41>", "▁", "▁▁ ▁", " leading", "trailing ", " both ",
        "task: search result | query: What is a kernel?", "title: none | text: body",
        "\u0000", "\u007f", "\U0010FFFF", "�", " ", "zzzz qqqq", "ǅǈǋ", "İstanbul",
        "Привет, мир! 東京大学 🚀 x=y+1", "the" * 200, " the" * 200, "ing" * 333,
    ]
    return texts


def quirk_sets():
    sets = []
    # 1. partial byte table: 'c' and 'd' have byte tokens, 'x', 'y' and 'é' have none
    sets.append({
        "name": "partial_bytes",
        "tokens": SPECIALS + ["a", "b", "▁", "ab", "▁a", "<0x63>", "<0x64>", "<0xC3>"],
        "merges": ["a b", "▁ a"],
        "texts": ["ab ab", "abc", "xyz", "xcx", "xxcd", "é", "aéb", "cxdyc", "x", "xc", "cx", "ab x ab",
                  "ééé", "ac", "xaxbx", ""],
    })
    # 2. two merges yielding the same token, duplicated merge, later duplicate token wins
    sets.append({
        "name": "same_result_merges",
        "tokens": SPECIALS + BYTES + ["a", "b", "c", "ab", "bc", "abc", "▁", "▁abc", "b", "cc", "ccc"],
        "merges": ["b c", "a b", "a bc", "ab c", "a b", "▁ abc", "c c", "cc c", "c cc"],
        "texts": ["abc", "abcabc", " abc", "aabbcc", "abcbc", "ccc", "cccc", "ccccc", "cabc", "bcabc",
                  "ab c", "abcc", "ababab", "b"],
    })
    # 3. single characters carrying the BOS and EOS ids, and merge strings that are not pairs
    sets.append({
        "name": "bos_eos_ids",
        "tokens": ["<pad>", "z", "y", "<unk>", "a", "▁", "za", "a▁", "a▁y"] + BYTES,
        "merges": ["z a", "a ▁", "a▁ y", "a b c", "single", "a  b", ""],
        "texts": ["y", "z", "yz", "zy", "za", "ay", "a y", "a", "zz", "yy", ""],
    })
    return sets


def main():
    rng = random.Random(1234)
    tokens, merges = trained_vocab(rng)
    tok = reference_tokenizer(tokens, merges)
    sets = [{"name": "trained", "tokens": tokens, "merges": merges,
             "cases": encode_cases(tok, trained_texts(rng))}]
    for q in quirk_sets():
        tok = reference_tokenizer(q["tokens"], q["merges"])
        sets.append({"name": q["name"], "tokens": q["tokens"], "merges": q["merges"],
                     "cases": encode_cases(tok, q["texts"])})
    build_errors = []
    for name, toks, mrg in [
        ("merge_part_missing", SPECIALS + ["a", "b", "ab"], ["a q"]),
        ("merge_result_missing", SPECIALS + ["a", "b"], ["a b"]),
    ]:
        try:
            reference_tokenizer(toks, mrg)
            build_errors.append({"name": name, "tokens": toks, "merges": mrg, "error": None})
        except Exception as e:  # noqa: BLE001
            build_errors.append({"name": name, "tokens": toks, "merges": mrg, "error": str(e)})
    # no <unk> in the vocabulary: the first character without a token or bytes is an error
    toks = ["<pad>", "<eos>", "<bos>", "a", "b"]
    sets.append({"name": "no_unk", "tokens": toks, "merges": [],
                 "cases": encode_cases(reference_tokenizer(toks, []), ["ab", "abc", "", "c"])})
    doc = {
        "library": f"tokenizers {tokenizers.__version__} (Python binding)",
        "config": "BPE(vocab, merges, byte_fallback, fuse_unk, unk <unk>); Replace(' ', U+2581); "
                  "Split(' ', MergedWithPrevious); encode(text, add_special_tokens=true)",
        "sets": sets,
        "build_errors": build_errors,
    }
    with open(OUT, "w", encoding="utf-8") as f:
        json.dump(doc, f, ensure_ascii=False, separators=(",", ":"))
    n = sum(len(s["cases"]) for s in sets)
    print(f"wrote {OUT}: {len(sets)} vocabularies, {n} texts")


if __name__ == "__main__":
    main()
