"""Text front end on the host: the library's C++ tokenizer and prompt formatters.

Pins (no GPU needed, the tokenizer is host code):

* ``tests/golden/tokenizer_golden.json`` -- ids, build errors and encode errors from the
  ``tokenizers`` 0.22.2 library (the reference's pinned crate, through its Python binding)
  configured as tokenizer.rs:77-138 configures it; both the oracle restatement and the
  library are checked against it;
* the reference's own known answers for the task prompts (task.rs:76-125);
* a randomized differential run against the ``tokenizers`` library itself where it is
  importable (random vocabularies, merges with colliding results, partial byte tables);
* Python's ``str.lower`` (the same Unicode lowercase + Final_Sigma rule as Rust's
  ``str::to_lowercase``) over every code point, for the lowercase tables.
"""
from __future__ import annotations

import ctypes
import json
import os
import random
import threading

import numpy as np
import pytest

from glypr_b200 import api, synth
from oracle import tokenizer_ref as R

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = json.load(open(os.path.join(HERE, "golden", "tokenizer_golden.json"), encoding="utf-8"))
SETS = {s["name"]: s for s in GOLDEN["sets"]}
FORMS = (api.GLP_TOKENS_BARE, api.GLP_TOKENS_SINGLE, api.GLP_TOKENS_SEQUENCE)


def _tok(name):
    s = SETS[name]
    return api.Tokenizer.from_vocab(s["tokens"], s["merges"]), R.BpeTokenizer(s["tokens"], s["merges"])


def test_golden_comes_from_the_pinned_library():
    assert GOLDEN["library"].startswith("tokenizers 0.22.2")
    assert sum(len(s["cases"]) for s in GOLDEN["sets"]) >= 300


@pytest.mark.parametrize("name", sorted(SETS))
def test_oracle_matches_golden(name):
    s = SETS[name]
    ref = R.BpeTokenizer(s["tokens"], s["merges"])
    for c in s["cases"]:
        if "error" in c:
            with pytest.raises(R.EncodeError) as e:
                ref.bpe(c["text"])
            assert str(e.value) == c["error"]
        else:
            assert ref.bpe(c["text"]) == c["ids"], repr(c["text"])


@pytest.mark.parametrize("name", sorted(SETS))
def test_library_matches_golden(name):
    s = SETS[name]
    tok = api.Tokenizer.from_vocab(s["tokens"], s["merges"])
    for c in s["cases"]:
        if "error" in c:
            with pytest.raises(api.GlyprError) as e:
                tok.encode(c["text"], api.GLP_TOKENS_BARE)
            assert str(e.value.message) == "Encode error: " + c["error"]
        else:
            assert tok.encode(c["text"], api.GLP_TOKENS_BARE) == c["ids"], repr(c["text"])


def test_build_errors_match_golden():
    for b in GOLDEN["build_errors"]:
        lib_msg = b["error"].replace("Error while initializing BPE: ", "")
        with pytest.raises(api.GlyprError) as e:
            api.Tokenizer.from_vocab(b["tokens"], b["merges"])
        assert e.value.code == api.GLP_ERR_FORMAT
        assert e.value.message == "BPE build error: " + lib_msg  # tokenizer.rs:118-125
        with pytest.raises(R.BuildError) as e2:
            R.BpeTokenizer(b["tokens"], b["merges"])
        assert str(e2.value) == lib_msg


@pytest.mark.parametrize("name", ["trained", "bos_eos_ids", "partial_bytes"])
def test_sequence_forms(name):
    """GLP_TOKENS_SINGLE (tokenizer.rs:162-177) and _SEQUENCE (454-566) around the BPE ids."""
    tok, ref = _tok(name)
    for c in SETS[name]["cases"]:
        if "error" in c:
            continue
        for form in FORMS:
            assert tok.encode(c["text"], form) == ref.encode(c["text"], form), (repr(c["text"]), form)
    if name == "bos_eos_ids":  # 'y' is id 2 (BOS) and 'z' id 1 (EOS) in this vocabulary
        assert tok.encode("y", api.GLP_TOKENS_SINGLE) == [2, 1]
        assert tok.encode("yz", api.GLP_TOKENS_SINGLE) == [2, 1]
        assert tok.encode("zy", api.GLP_TOKENS_SINGLE) == [2, 1, 2, 1]
        assert tok.encode("yz", api.GLP_TOKENS_SEQUENCE) == [2, 2, 1, 1]
    assert tok.encode("", api.GLP_TOKENS_SINGLE) == [2, 1]
    assert tok.encode("", api.GLP_TOKENS_SEQUENCE) == [2, 1]
    assert tok.encode("", api.GLP_TOKENS_BARE) == []


def test_batch_matches_single_and_threads():
    tok, ref = _tok("trained")
    texts = [c["text"] for c in SETS["trained"]["cases"]]
    one = tok.encode_batch(texts, api.GLP_TOKENS_SINGLE, n_threads=1)
    many = tok.encode_batch(texts, api.GLP_TOKENS_SINGLE, n_threads=8)
    for t, a, b in zip(texts, one, many):
        assert a.tolist() == b.tolist() == ref.encode(t, R.FORM_SINGLE)
    ids, mask = tok.encode_batch_padded(texts[:20])
    rids, rlens = ref.encode_batch_padded(texts[:20], 10 ** 9)
    assert ids.tolist() == rids
    assert mask.sum(axis=1).tolist() == rlens


def test_batch_limit_and_empty_errors():
    tok, ref = _tok("trained")
    texts = ["short", "a much longer text " * 20, "x", "another long one " * 30]
    lens = [len(ref.encode(t)) for t in texts]
    limit = lens[1] - 1
    with pytest.raises(api.GlyprError) as e:
        tok.encode_batch(texts, api.GLP_TOKENS_SINGLE, limit=limit)
    assert e.value.code == api.GLP_ERR_CONTEXT_LIMIT
    # the first offending item in order, worded as encode_batch_padded_with_limit words it
    with pytest.raises(R.EncodeError) as e2:
        ref.encode_batch_padded(texts, limit)
    assert e.value.message == str(e2.value) == (
        f"Batch item 1 sequence length ({lens[1]} tokens) exceeds maximum context limit ({limit} tokens)")
    with pytest.raises(api.GlyprError) as e:
        tok.encode_batch([])
    assert e.value.message == "Cannot encode an empty batch"


def test_invalid_utf8_rejected():
    tok, _ = _tok("trained")
    L = api.load_library()
    ids = (ctypes.c_int32 * 16)()
    n = ctypes.c_int()
    for bad in (b"\xff", b"a\xc3", b"\xed\xa0\x80", b"\xc0\xaf", b"\xf4\x90\x80\x80"):
        rc = L.glp_tokenize(tok._h, bad, len(bad), api.GLP_TOKENS_BARE, ids, 16, ctypes.byref(n))
        assert rc == api.GLP_ERR_INVALID_ARG
        assert b"UTF-8" in L.glp_last_error()


def test_small_output_buffer_reports_size():
    tok, ref = _tok("trained")
    L = api.load_library()
    text = "the station and the quing".encode()
    want = ref.encode("the station and the quing")
    ids = (ctypes.c_int32 * 2)()
    n = ctypes.c_int()
    rc = L.glp_tokenize(tok._h, text, len(text), api.GLP_TOKENS_SINGLE, ids, 2, ctypes.byref(n))
    assert rc == api.GLP_ERR_INVALID_ARG and n.value == len(want)


def _random_vocab(rng: random.Random):
    alphabet = ["a", "b", "c", "d", "e", "é", "Σ", "東", "🙂", "▁", "x", "\n"]
    known = rng.sample(alphabet, rng.randint(4, len(alphabet)))
    tokens = ["<pad>", "<eos>", "<bos>"] + (["<unk>"] if rng.random() < 0.9 else [])
    byte_frac = rng.choice([0.0, 0.3, 1.0])
    tokens += ["<0x%02X>" % b for b in range(256) if rng.random() < byte_frac]
    tokens += known
    merges = []
    for _ in range(rng.randint(0, 60)):
        a, b = rng.choice(tokens[3:] or known), rng.choice(tokens[3:] or known)
        if a.startswith("<") or b.startswith("<") or " " in a + b:
            continue
        if a + b not in tokens:
            tokens.append(a + b)
        merges.append(f"{a} {b}")
    if rng.random() < 0.3 and tokens:
        tokens.append(rng.choice(tokens[3:]))  # a duplicate: the later index wins
    return tokens, merges, alphabet + ["z", "ß", " "]


def test_random_differential_against_the_library():
    tokenizers = pytest.importorskip("tokenizers")
    from tokenizers import Tokenizer, models, normalizers, pre_tokenizers
    rng = random.Random(7)
    checked = 0
    for _ in range(60):
        tokens, merges, chars = _random_vocab(rng)
        vocab = {}
        for i, t in enumerate(tokens):
            vocab[t] = i
        pairs = [tuple(m.split(" ")) for m in merges]
        lib = Tokenizer(models.BPE(vocab=vocab, merges=pairs, unk_token="<unk>", fuse_unk=True, byte_fallback=True))
        lib.normalizer = normalizers.Replace(" ", "▁")
        lib.pre_tokenizer = pre_tokenizers.Split(" ", behavior="merged_with_previous", invert=False)
        ours = api.Tokenizer.from_vocab(tokens, merges)
        for _ in range(40):
            text = "".join(rng.choice(chars) for _ in range(rng.randint(0, 40)))
            try:
                want = lib.encode(text, add_special_tokens=True).ids
            except Exception as e:  # noqa: BLE001
                with pytest.raises(api.GlyprError) as ge:
                    ours.encode(text, api.GLP_TOKENS_BARE)
                assert ge.value.message == "Encode error: " + str(e)
                continue
            assert ours.encode(text, api.GLP_TOKENS_BARE) == want, (tokens, merges, text)
            checked += 1
    assert checked > 1500
    assert tokenizers.__version__ == "0.22.2"


# ---- prompts ------------------------------------------------------------------------------

def test_task_known_answers():
    """task.rs:76-125, the reference's own tests."""
    assert api.task_format("SearchQuery", None, "quantum physics") == "task: search result | query: quantum physics"
    assert api.task_format("document", None, "content body") == "title: none | text: content body"
    assert api.task_format("document", "Physics 101", "content body") == "title: Physics 101 | text: content body"
    assert api.task_format("code_retrieval", None, "fn test()") == "task: code retrieval | query: fn test()"
    assert api.task_format("classification", None, "sentiment review") == \
        "task: classification | query: sentiment review"
    assert api.task_format(None, None, "unprompted text") == "unprompted text"
    assert api.task_format("qa", None, "q") == "task: question answering | query: q"
    assert api.task_format("Doc", "Doc A", "x") == "task: Doc | query: x"  # Custom keeps the name's case
    assert api.task_format("retrieval_document", "Doc A", "x") == "title: Doc A | text: x"


TASK_NAMES = ["search_query", "Retrieval", "retrieval-query", "query", "document", "Retrieval Document", "code",
              "CodeRetrieval", "classification", "multilabel_classification", "clustering", "Question-Answering",
              "qa", "fact checking", "STS", "pair_classification", "summarization", "sentence similarity", "raw",
              "NONE", "reranking", "bitext_mining", "BitextMining", "my task", "A:B", "x|y", "ΣΑΣ", "ΑΣ'Σ.",
              "İstanbul", "KELVINK", "ẞtraße", "ǅemal", "Σ", "ΑΣ́", "ΑΣ́Β", "·Σ", "", "-_ ",
              "ΌΣΟΣ ΟΣ", "aͅΣ"]


def test_formatters_match_oracle():
    for name in TASK_NAMES:
        for title in (None, "T", "Σ title"):
            assert api.task_format(name, title, "body") == R.task_format(name, title, "body"), (name, title)
        assert api.format_query("what?", name) == R.format_query("what?", name), name
    for title in (None, "", "Physics 101", "ΣΣ"):
        assert api.format_document("content", title) == R.format_document("content", title)


def test_lowercase_tables_cover_every_code_point():
    """glp_format_query's fallback lowercases the task: compare with str.lower over all of Unicode."""
    cps = [c for c in range(1, 0x110000) if not 0xD800 <= c <= 0xDFFF]
    rng = random.Random(3)
    for k in range(0, len(cps), 8192):
        chunk = cps[k:k + 8192]
        rng.shuffle(chunk)  # arbitrary neighbours, so Final_Sigma contexts get exercised too
        name = "".join(map(chr, chunk)) + "Σ"
        got = api.format_query("", name)
        assert got == R.format_query("", name), hex(chunk[0])


def test_engine_text_requests_tokenise_like_the_server():
    """glp_engine_embed_text: Task formatting + sequence tokens (handlers.rs:88-92,
    tokenizer.rs:454-566) reach the batch executor."""
    tok, ref = _tok("trained")
    seen = []
    lock = threading.Lock()

    def executor(ids, lengths, out_dim):
        with lock:
            for row, n in zip(ids, lengths):
                seen.append(row[:n].tolist())
        return np.ones((len(lengths), out_dim), dtype=np.float32)

    reqs = [("the quick station", "search_query", None), ("body text", "document", "Title"), ("raw", None, None),
            ("", "clustering", None), ("Σ ΣΟΦ", "my task", None)]
    with api.InferenceEngine.with_executor(executor, 16, max_batch_size=4) as eng:
        outs = [eng.embed_text(tok, t, task, title) for t, task, title in reqs]
        assert all(o.shape == (16,) for o in outs)
        with pytest.raises(api.GlyprError) as e:
            eng.embed_text(tok, "the " * 9000, None)
        assert e.value.code == api.GLP_ERR_CONTEXT_LIMIT
        assert e.value.message.startswith("Text sequence length (")
    want = [ref.encode(R.task_format(task, title, t), R.FORM_SEQUENCE) for t, task, title in reqs]
    assert sorted(seen) == sorted(want)


def test_tokenizer_from_gguf(tmp_path):
    s = SETS["trained"]
    cfg = synth.small_config()
    path = synth.write_gguf(str(tmp_path / "tok.gguf"), cfg, tokenizer=(s["tokens"], s["merges"]))
    tok = api.Tokenizer.from_gguf(path)
    assert tok.info() == {"tokens": cfg.vocab, "merges": len(s["merges"])}
    ref = R.BpeTokenizer(s["tokens"] + [f"<t{i}>" for i in range(len(s["tokens"]), cfg.vocab)], s["merges"])
    for c in s["cases"][:60]:
        assert tok.encode(c["text"]) == ref.encode(c["text"])
    # the filler-only synthetic files have no merges key: the reference's error
    bare = synth.write_gguf(str(tmp_path / "bare.gguf"), cfg)
    with pytest.raises(api.GlyprError) as e:
        api.Tokenizer.from_gguf(bare)
    assert e.value.message == "Missing tokenizer.ggml.merges in GGUF metadata"
    no_tokens = synth.write_gguf(str(tmp_path / "nt.gguf"), cfg, drop=["tokenizer.ggml.tokens"])
    with pytest.raises(api.GlyprError) as e:
        api.Tokenizer.from_gguf(no_tokens)
    assert e.value.message == "Missing tokenizer.ggml.tokens in GGUF metadata"
